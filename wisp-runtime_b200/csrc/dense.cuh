// Dense bf16 GEMV of the decoder (attention projections, router, lm_head): y = W x for one token,
// W row-major [N, K] bf16, fp32 accumulation, one rounding to bf16 (what a bf16 nn.Linear gives).
//
// HBM-bound (2 bytes per multiply-add).  Each CTA owns a contiguous range of rows, which is one
// contiguous byte range of W: a producer warp streams it through a ring of shared-memory stages
// with TMA bulk copies (no multicast), and eight consumer warps take one row each per stage.  The
// first stages are issued before griddepcontrol.wait (weights never depend on earlier kernels), so
// a PDL-chained GEMV starts streaming while the previous kernel finishes.
//
// Fused around the product (all optional): x := bf16(x + x_add) (the residual add of the previous
// sub-layer, stored once to x_sum_out), x := RMSNorm(x) * norm_w (stored once to xn_out), and
// y := bf16(res + bf16(W x [+ bias])) (the layer's bias and this sub-layer's residual add).  Every CTA reads all of x while CTA 0
// writes x_sum_out / xn_out and all CTAs write y, so none of those may alias x or x_add; y may
// alias res (each row is read and written by the same thread).
#pragma once
#include "common.cuh"
#include "tma.cuh"

namespace wisp {
namespace dense {

constexpr int CONSUMERS = 8;
constexpr int THREADS = 32 * (CONSUMERS + 1);  // warp 0 produces, warps 1..8 consume
// ring of 3 stages (96 KB at K = 2048 / 4096: a GEMV CTA fits beside the previous kernel's CTA for the
// PDL prefetch), or 4 where 4 stages fit in 120 KB and a CTA's rows need them (K = 2880: 4 x 28.8 KB).
// The 4th stage (gpt-oss q/k/v and lm_head) measured 4.6% faster per token on the gpt-oss decoder; a 4th
// 32 KB stage measured 1.8% slower on Qwen3, and rings below 3 stages slower on both (they change how
// the neighbouring kernels' CTAs share the SMs).
constexpr int STAGES = 3;
constexpr int STAGES_MAX = 4;
constexpr int64_t RING_BYTES_MAX = 120 * 1024;
constexpr int STAGE_BYTES = 32 * 1024;

struct GemvArgs {
  const uint16_t* W;
  int64_t N, K;
  const uint16_t* x;
  const uint16_t* x_add;  // nullable
  uint16_t* x_sum_out;    // nullable (written by CTA 0)
  const uint16_t* norm_w; // nullable: no norm
  float eps;
  uint16_t* xn_out;       // nullable (written by CTA 0)
  const uint16_t* res;    // nullable
  uint16_t* y;
  const uint16_t* bias;   // nullable: y = bf16(W x + bias) before the residual add
};

struct GemvLayout {
  int rows_per_stage;
  int64_t stage_bytes, off_x, off_red, off_bars, bytes;
};

template <int NST = STAGES>
__host__ __device__ inline GemvLayout gemv_layout(int64_t K) {
  GemvLayout L;
  const int64_t row = K * 2;
  int64_t sr = STAGE_BYTES / row;
  L.rows_per_stage = int(sr < 1 ? 1 : (sr > 16 ? 16 : sr));
  L.stage_bytes = L.rows_per_stage * row;
  L.off_x = NST * L.stage_bytes;         // normalised x, bf16 [K]
  L.off_red = ru16(L.off_x + row);       // [CONSUMERS] f32 partial sums of squares
  L.off_bars = ru16(L.off_red + CONSUMERS * 4);  // full[NST], empty[NST]
  L.bytes = L.off_bars + 16 * NST;
  return L;
}

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

template <int STAGES>
__global__ void __launch_bounds__(THREADS, 1) gemv_kernel(GemvArgs A) {
  extern __shared__ __align__(128) uint8_t sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const GemvLayout L = gemv_layout<STAGES>(A.K);
  uint16_t* xs = reinterpret_cast<uint16_t*>(sm + L.off_x);
  float* red = reinterpret_cast<float*>(sm + L.off_red);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L.off_bars);
  uint64_t* empty = full + STAGES;
  const int64_t n0 = A.N * blockIdx.x / gridDim.x, n1 = A.N * (blockIdx.x + 1) / gridDim.x;
  const int SR = L.rows_per_stage;
  const int nstages = int((n1 - n0 + SR - 1) / SR);
  const int64_t row_bytes = A.K * 2;

  if (warp == 0) {
    // ---- producer: stream rows [n0, n1) through the ring (lane 0 only)
    if (lane == 0) {
      for (int s = 0; s < STAGES; ++s) {
        mbar_init(&full[s], 1);
        mbar_init(&empty[s], CONSUMERS);
      }
      mbar_fence_init();
    }
    named_sync(1, THREADS);  // barriers initialised before anyone waits on them
    pdl_launch_dependents();
    if (lane == 0) {
      const uint8_t* src = reinterpret_cast<const uint8_t*>(A.W) + n0 * row_bytes;
      for (int s = 0; s < nstages; ++s) {
        const int slot = s % STAGES;
        if (s >= STAGES && !mbar_wait(&empty[slot], uint32_t((s / STAGES - 1) & 1))) break;
        const int64_t r0 = int64_t(s) * SR;
        const int64_t nr = (n1 - n0 - r0) < SR ? (n1 - n0 - r0) : SR;
        const uint32_t bytes = uint32_t(nr * row_bytes);
        mbar_expect_tx(&full[slot], bytes);
        bulk_g2s(sm + int64_t(slot) * L.stage_bytes, src + r0 * row_bytes, bytes, &full[slot]);
      }
    }
    return;
  }
  named_sync(1, THREADS);
  pdl_launch_dependents();
  pdl_wait();  // x, x_add and res come from earlier kernels

  // ---- x: optional residual add and RMSNorm, into shared memory as bf16 --------------------------
  const int ct = threadIdx.x - 32;  // consumer thread 0..255
  const int64_t nch = A.K / 8;      // 16-byte chunks of x
  float ss = 0.0f;
  for (int64_t c = ct; c < nch; c += 32 * CONSUMERS) {
    uint4 v = reinterpret_cast<const uint4*>(A.x)[c];
    if (A.x_add) {
      const uint4 d = reinterpret_cast<const uint4*>(A.x_add)[c];
      const uint32_t xv[4] = {v.x, v.y, v.z, v.w}, dv[4] = {d.x, d.y, d.z, d.w};
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        o[i] = uint32_t(f32_to_bf16(bf_lo(xv[i]) + bf_lo(dv[i]))) | (uint32_t(f32_to_bf16(bf_hi(xv[i]) + bf_hi(dv[i]))) << 16);
      v = make_uint4(o[0], o[1], o[2], o[3]);
      if (A.x_sum_out && blockIdx.x == 0) reinterpret_cast<uint4*>(A.x_sum_out)[c] = v;
    }
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) ss += bf_lo(w4[i]) * bf_lo(w4[i]) + bf_hi(w4[i]) * bf_hi(w4[i]);
    reinterpret_cast<uint4*>(xs)[c] = v;
  }
  if (A.norm_w) {
    ss = warp_sum(ss);
    if (lane == 0) red[warp - 1] = ss;
    named_sync(2, 32 * CONSUMERS);
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < CONSUMERS; ++w) tot += red[w];
    const float inv = rsqrtf(tot / float(A.K) + A.eps);
    for (int64_t c = ct; c < nch; c += 32 * CONSUMERS) {
      const uint4 v = reinterpret_cast<const uint4*>(xs)[c];
      const uint4 wv = reinterpret_cast<const uint4*>(A.norm_w)[c];
      const uint32_t xv[4] = {v.x, v.y, v.z, v.w}, ww[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float a = bf_lo(ww[i]) * bf16_to_f32(f32_to_bf16(bf_lo(xv[i]) * inv));
        const float b = bf_hi(ww[i]) * bf16_to_f32(f32_to_bf16(bf_hi(xv[i]) * inv));
        o[i] = uint32_t(f32_to_bf16(a)) | (uint32_t(f32_to_bf16(b)) << 16);
      }
      const uint4 on = make_uint4(o[0], o[1], o[2], o[3]);
      reinterpret_cast<uint4*>(xs)[c] = on;
      if (A.xn_out && blockIdx.x == 0) reinterpret_cast<uint4*>(A.xn_out)[c] = on;
    }
  } else if (A.xn_out && blockIdx.x == 0) {
    for (int64_t c = ct; c < nch; c += 32 * CONSUMERS) reinterpret_cast<uint4*>(A.xn_out)[c] = reinterpret_cast<const uint4*>(xs)[c];
  }
  named_sync(2, 32 * CONSUMERS);

  // ---- rows: consumer warp w takes rows w, w + 8, ... of every stage; x read from shared memory ---
  const int cw = warp - 1;
  const uint4* xs4 = reinterpret_cast<const uint4*>(xs);
  for (int s = 0; s < nstages; ++s) {
    const int slot = s % STAGES;
    if (!mbar_wait(&full[slot], uint32_t((s / STAGES) & 1))) break;
    const int64_t r0 = int64_t(s) * SR;
    const int nr = int((n1 - n0 - r0) < SR ? (n1 - n0 - r0) : SR);
    const uint8_t* stage = sm + int64_t(slot) * L.stage_bytes;
    for (int r = cw; r < nr; r += CONSUMERS) {
      const uint4* wrow = reinterpret_cast<const uint4*>(stage + int64_t(r) * row_bytes);
      float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll 4
      for (int64_t c = lane; c < nch; c += 32) {
        const uint4 w = wrow[c], xv4 = xs4[c];
        const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
        const uint32_t xv[4] = {xv4.x, xv4.y, xv4.z, xv4.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc0 = fmaf(bf_lo(wv[q]), bf_lo(xv[q]), acc0);
          acc1 = fmaf(bf_hi(wv[q]), bf_hi(xv[q]), acc1);
        }
      }
      const float acc = warp_sum(acc0 + acc1);
      if (lane == 0) {
        const int64_t n = n0 + r0 + r;
        float out = bf16_to_f32(f32_to_bf16(A.bias ? acc + bf16_to_f32(A.bias[n]) : acc));
        if (A.res) out = bf16_to_f32(A.res[n]) + out;
        A.y[n] = f32_to_bf16(out);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
}

}  // namespace dense
}  // namespace wisp
