// Decode-side ops around the MoE: one-kernel rotary and RMSNorm (with the residual add fused in).
#pragma once
#include "common.cuh"

namespace wisp {

// one warp per head (q heads first, then k heads); fp32 math with separately rounded products,
// out = x*c + rotate_half(x)*s, one rounding to bf16 (the form of wisp/kernels.py:347).
__global__ void rope_decode_kernel(const uint16_t* __restrict__ q, int64_t q_stride, int Hq,
                                   const uint16_t* __restrict__ k, int64_t k_stride, int Hk, int D,
                                   const uint16_t* __restrict__ cosv, const uint16_t* __restrict__ sinv,
                                   uint16_t* __restrict__ qo, uint16_t* __restrict__ ko) {
  const int head = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (head >= Hq + Hk) return;
  const bool is_q = head < Hq;
  const uint16_t* src = is_q ? q + int64_t(head) * q_stride : k + int64_t(head - Hq) * k_stride;
  uint16_t* dst = is_q ? qo + int64_t(head) * D : ko + int64_t(head - Hq) * D;
  const int half = D / 2;
  for (int i = lane; i < D; i += 32) {
    const float xv = bf16_to_f32(src[i]);
    const float xp = i < half ? -bf16_to_f32(src[i + half]) : bf16_to_f32(src[i - half]);
    const float r = __fadd_rn(__fmul_rn(xv, bf16_to_f32(cosv[i])), __fmul_rn(xp, bf16_to_f32(sinv[i])));
    dst[i] = f32_to_bf16(r);
  }
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.0f;
  return warp_sum(t);
}

// one block per row.  out = bf16(w * bf16(x * rsqrt(mean(x^2) + eps))); with delta, x := bf16(x + delta)
// first (stored to sum_out when given).  sum_out may alias x (in-place residual stream): every
// element is read and then written by the same thread.
__global__ void __launch_bounds__(256) rmsnorm_kernel(const uint16_t* x, const uint16_t* __restrict__ delta,
                                                      uint16_t* sum_out, const uint16_t* __restrict__ w,
                                                      int64_t H, float eps, uint16_t* __restrict__ out) {
  __shared__ float red[32];
  extern __shared__ float rowv[];  // H fp32
  const int64_t row = blockIdx.x;
  const uint16_t* xr = x + row * H;
  float ss = 0.0f;
  for (int64_t i = threadIdx.x; i < H; i += blockDim.x) {
    float v = bf16_to_f32(xr[i]);
    if (delta) {
      v = bf16_to_f32(f32_to_bf16(v + bf16_to_f32(delta[row * H + i])));
      if (sum_out) sum_out[row * H + i] = f32_to_bf16(v);
    }
    rowv[i] = v;
    ss = fmaf(v, v, ss);
  }
  const float tot = block_sum(ss, red);
  const float inv = rsqrtf(tot / float(H) + eps);
  for (int64_t i = threadIdx.x; i < H; i += blockDim.x) {
    const float nv = bf16_to_f32(f32_to_bf16(rowv[i] * inv));
    out[row * H + i] = f32_to_bf16(bf16_to_f32(w[i]) * nv);
  }
}

// H % 8 == 0 and H / 8 <= 1024: one thread per 8 elements, every load issued before any arithmetic
// (x, delta and w as 16-byte vectors), one block reduction.  Same rounding steps as rmsnorm_kernel.
__global__ void __launch_bounds__(1024) rmsnorm_vec_kernel(const uint16_t* x, const uint16_t* __restrict__ delta,
                                                           uint16_t* sum_out, const uint16_t* __restrict__ w, int64_t H,
                                                           float eps, uint16_t* __restrict__ out) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int t = threadIdx.x;
  const bool active = int64_t(t) * 8 < H;
  uint4 xv = make_uint4(0, 0, 0, 0), dv = make_uint4(0, 0, 0, 0), wv = make_uint4(0, 0, 0, 0);
  if (active) wv = reinterpret_cast<const uint4*>(w)[t];  // weights are not written by earlier kernels
  pdl_wait();
  pdl_launch_dependents();
  if (active) {
    xv = reinterpret_cast<const uint4*>(x + row * H)[t];
    if (delta) dv = reinterpret_cast<const uint4*>(delta + row * H)[t];
  }
  float v[8];
  const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w}, dw[4] = {dv.x, dv.y, dv.z, dv.w};
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(xw[i] << 16);
    v[2 * i + 1] = __uint_as_float(xw[i] & 0xFFFF0000u);
    if (delta) {
      v[2 * i] = bf16_to_f32(f32_to_bf16(v[2 * i] + __uint_as_float(dw[i] << 16)));
      v[2 * i + 1] = bf16_to_f32(f32_to_bf16(v[2 * i + 1] + __uint_as_float(dw[i] & 0xFFFF0000u)));
    }
    ss = fmaf(v[2 * i], v[2 * i], ss);
    ss = fmaf(v[2 * i + 1], v[2 * i + 1], ss);
  }
  if (active && delta && sum_out) {
    uint4 o;
    uint32_t* op = &o.x;
#pragma unroll
    for (int i = 0; i < 4; ++i) op[i] = uint32_t(f32_to_bf16(v[2 * i])) | (uint32_t(f32_to_bf16(v[2 * i + 1])) << 16);
    reinterpret_cast<uint4*>(sum_out + row * H)[t] = o;
  }
  const float tot = block_sum(active ? ss : 0.0f, red);
  const float inv = rsqrtf(tot / float(H) + eps);
  if (active) {
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
    uint4 o;
    uint32_t* op = &o.x;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a = __uint_as_float(ww[i] << 16) * bf16_to_f32(f32_to_bf16(v[2 * i] * inv));
      const float b = __uint_as_float(ww[i] & 0xFFFF0000u) * bf16_to_f32(f32_to_bf16(v[2 * i + 1] * inv));
      op[i] = uint32_t(f32_to_bf16(a)) | (uint32_t(f32_to_bf16(b)) << 16);
    }
    reinterpret_cast<uint4*>(out + row * H)[t] = o;
  }
}

}  // namespace wisp
