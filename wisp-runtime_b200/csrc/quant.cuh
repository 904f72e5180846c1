// Packed-format kernels: quantize (store build), dequantize and code unpack (bit-exact parity probes,
// bf16 weight feed for the batched / prefill path).
#pragma once
#include "common.cuh"

namespace wisp {

template <typename T>
__device__ __forceinline__ float load_weight(const T* p, int64_t i);
template <>
__device__ __forceinline__ float load_weight<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float load_weight<uint16_t>(const uint16_t* p, int64_t i) { return bf16_to_f32(p[i]); }

// One warp per quantization group.  Follows the RTN min/max rule of wisp/quant.py:65-73 step by step
// in IEEE fp32: scale = max((mx - mn) / levels, 1e-5); scale and min stored as fp16 (RNE);
// q = rint((v - fp32(min16)) / fp32(scale16)) clamped to [0, levels].
template <int BITS, typename T>
__global__ void __launch_bounds__(256) quantize_kernel(const T* __restrict__ w_all, int64_t batch, int64_t ngroups,
                                                        int group, uint8_t* __restrict__ out_all, int64_t ncode,
                                                        int64_t nbytes) {
  const int lane = threadIdx.x & 31;
  const int64_t gg = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (gg >= batch * ngroups) return;
  const int64_t b = gg / ngroups, g = gg - b * ngroups;
  const T* w = w_all + b * (ngroups * group);
  uint8_t* out = out_all + b * nbytes;
  const int64_t e0 = g * group;
  float mn = INFINITY, mx = -INFINITY;
  for (int i = lane; i < group; i += 32) {
    float v = load_weight(w, e0 + i);
    mn = fminf(mn, v);
    mx = fmaxf(mx, v);
  }
  mn = warp_min(mn);
  mx = warp_max(mx);
  constexpr float levels = float((1 << BITS) - 1);
  float scale = __fdiv_rn(__fsub_rn(mx, mn), levels);
  scale = scale < 1e-5f ? 1e-5f : scale;
  const uint16_t s16 = f32_to_f16_bits(scale), m16 = f32_to_f16_bits(mn);
  const float sf = f16_bits_to_f32(s16), mf = f16_bits_to_f32(m16);
  // 8 codes -> BITS bytes per chunk
  for (int c = lane; c < group / 8; c += 32) {
    uint32_t lo = 0, hi = 0;  // up to 64 bits of packed codes
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float v = load_weight(w, e0 + 8 * c + i);
      float q = rintf(__fdiv_rn(__fsub_rn(v, mf), sf));
      q = fminf(fmaxf(q, 0.0f), levels);
      uint32_t code = uint32_t(q);
      const int bit = BITS * i;
      if (bit < 32) {
        lo |= code << bit;
        if (bit + BITS > 32) hi |= code >> (32 - bit);
      } else {
        hi |= code << (bit - 32);
      }
    }
    uint8_t* dst = out + (e0 + 8 * c) * BITS / 8;
    if constexpr (BITS == 8) {
      *reinterpret_cast<uint2*>(dst) = make_uint2(lo, hi);
    } else if constexpr (BITS == 4) {
      *reinterpret_cast<uint32_t*>(dst) = lo;
    } else if constexpr (BITS == 2) {
      *reinterpret_cast<uint16_t*>(dst) = uint16_t(lo);
    } else {
      dst[0] = uint8_t(lo);
      dst[1] = uint8_t(lo >> 8);
      dst[2] = uint8_t(lo >> 16);
    }
  }
  if (lane == 0) {
    uint16_t* sc = reinterpret_cast<uint16_t*>(out + ncode);
    sc[g] = s16;
    sc[ngroups + g] = m16;
  }
}

template <typename T>
__global__ void to_bf16_kernel(const T* __restrict__ w, int64_t count, uint16_t* __restrict__ out) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += int64_t(gridDim.x) * blockDim.x)
    out[i] = f32_to_bf16(load_weight(w, i));
}

// One thread per 32-element unit of one selected row.  MODE 0: bf16 dequant, MODE 1: codes.
// Dequant follows wisp/quant.py:86-87: fp32(q) * fp32(scale) rounded, + fp32(min) rounded, -> bf16 RNE.
template <int BITS, int MODE>
__global__ void __launch_bounds__(256) unpack_kernel(const uint8_t* __restrict__ pool, int64_t pool_rows,
                                                     int64_t nbytes, const int64_t* __restrict__ rows,
                                                     int64_t nrows, int64_t n, int group, void* __restrict__ out) {
  const int64_t units_per_row = 3 * n / 32;
  const int64_t total = nrows * units_per_row;
  const int64_t ncode = 3 * n * BITS / 8;
  const int64_t ng = 3 * n / group;
  for (int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < total; t += int64_t(gridDim.x) * blockDim.x) {
    const int64_t b = t / units_per_row, u = t - b * units_per_row;
    const int64_t row = rows ? rows[b] : b;
    if (row < 0 || row >= pool_rows) {
      flag(WISP_STATUS_BAD_SLOT);
      continue;
    }
    const uint8_t* base = pool + row * nbytes;
    const Unit<BITS> cu = load_unit<BITS>(base + u * (4 * BITS));
    if constexpr (MODE == 1) {
      uint8_t* dst = reinterpret_cast<uint8_t*>(out) + b * (3 * n) + u * 32;
      uint32_t packed[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        packed[i] = unit_code<BITS>(cu, 4 * i) | (unit_code<BITS>(cu, 4 * i + 1) << 8) |
                    (unit_code<BITS>(cu, 4 * i + 2) << 16) | (unit_code<BITS>(cu, 4 * i + 3) << 24);
      uint4* d4 = reinterpret_cast<uint4*>(dst);
      d4[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
      d4[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
    } else {
      const uint16_t* sc = reinterpret_cast<const uint16_t*>(base + ncode);
      const uint16_t* mn = sc + ng;
      const int64_t e0 = u * 32;
      uint32_t packed[16];
      if (group % 32 == 0) {
        const int64_t gi = e0 / group;
        const float s = f16_bits_to_f32(sc[gi]), m = f16_bits_to_f32(mn[gi]);
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float a = __fadd_rn(__fmul_rn(small_u2f(unit_code<BITS>(cu, i)), s), m);
          float c = __fadd_rn(__fmul_rn(small_u2f(unit_code<BITS>(cu, i + 1)), s), m);
          packed[i / 2] = uint32_t(f32_to_bf16(a)) | (uint32_t(f32_to_bf16(c)) << 16);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const int64_t g0 = (e0 + i) / group, g1 = (e0 + i + 1) / group;
          float a = __fadd_rn(__fmul_rn(small_u2f(unit_code<BITS>(cu, i)), f16_bits_to_f32(sc[g0])),
                              f16_bits_to_f32(mn[g0]));
          float c = __fadd_rn(__fmul_rn(small_u2f(unit_code<BITS>(cu, i + 1)), f16_bits_to_f32(sc[g1])),
                              f16_bits_to_f32(mn[g1]));
          packed[i / 2] = uint32_t(f32_to_bf16(a)) | (uint32_t(f32_to_bf16(c)) << 16);
        }
      }
      uint4* d4 = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(out) + b * (3 * n) + e0);
#pragma unroll
      for (int i = 0; i < 4; ++i) d4[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
    }
  }
}

// 16-bit experts are raw bf16: "dequant" is a gather of rows.
__global__ void gather_rows_kernel(const uint8_t* __restrict__ pool, int64_t pool_rows, int64_t nbytes,
                                   const int64_t* __restrict__ rows, int64_t nrows, uint8_t* __restrict__ out) {
  const int64_t vec_per_row = nbytes / 16;
  const int64_t total = nrows * vec_per_row;
  for (int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < total; t += int64_t(gridDim.x) * blockDim.x) {
    const int64_t b = t / vec_per_row, v = t - b * vec_per_row;
    const int64_t row = rows ? rows[b] : b;
    if (row < 0 || row >= pool_rows) {
      flag(WISP_STATUS_BAD_SLOT);
      continue;
    }
    reinterpret_cast<uint4*>(out + b * nbytes)[v] = ld_stream_v4(pool + row * nbytes + 16 * v);
  }
}

}  // namespace wisp
