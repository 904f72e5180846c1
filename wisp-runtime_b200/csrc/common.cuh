// Shared helpers for the wisp-b200 kernels (sm_100a): error reporting, bf16/fp16 bit helpers,
// cache-hinted global loads and the device-side status word.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/wisp_b200.h"

namespace wisp {

// ------------------------------------------------------------------------------------------------
// host-side error reporting: each entry point returns a WISP_* code and leaves a message behind
// ------------------------------------------------------------------------------------------------
std::string& last_error_slot();

inline int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  last_error_slot() = buf;
  return code;
}

inline int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return WISP_OK;
}

#define WISP_REQUIRE(cond, ...)                          \
  do {                                                   \
    if (!(cond)) return ::wisp::fail(WISP_ERR_INVALID, __VA_ARGS__); \
  } while (0)

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ------------------------------------------------------------------------------------------------
// device-side status word: kernels never trap; a bad slot id, an out-of-range position or a wait
// that ran out of iterations sets a bit here and the kernel skips the access.  One word per device
// (static device memory, no allocation); read and cleared by wisp_device_status().
// ------------------------------------------------------------------------------------------------
// defined here: the library is built as one translation unit (wisp_b200.cu includes every .cuh)
__device__ unsigned int g_status = 0;

// programmatic dependent launch: wait for the preceding grid's completion and memory flush / allow
// the next grid in the stream to launch.  Both are no-ops when the launch did not opt in.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void flag(unsigned int bit) { atomicOr(&g_status, bit); }

// ------------------------------------------------------------------------------------------------
// numeric helpers
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ float bf16_to_f32(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

// round to nearest even; NaN -> canonical quiet NaN (the behaviour of torch's fp32 -> bf16 cast)
__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
  __nv_bfloat16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}

__device__ __forceinline__ float f16_bits_to_f32(uint16_t b) {
  __half h = *reinterpret_cast<__half*>(&b);
  return __half2float(h);
}

__device__ __forceinline__ uint16_t f32_to_f16_bits(float f) {
  __half h = __float2half_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}

// exact float of a small unsigned integer (< 2^23) without the I2F pipe: 2^23 + c, minus 2^23
__device__ __forceinline__ float small_u2f(uint32_t c) { return __uint_as_float(0x4B000000u | c) - 8388608.0f; }

// ------------------------------------------------------------------------------------------------
// streaming loads: read-only path, do not allocate in L1 (weights are touched exactly once)
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint2 ld_stream_v2(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t ld_stream_u32(const void* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ uint16_t ld_nc_u16(const void* p) {
  unsigned short v;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ------------------------------------------------------------------------------------------------
// packed-code units: 32 consecutive codes of a BITS-bit little-endian stream occupy BITS 32-bit words
// (element e of an expert sits at bit BITS*e of its code region; the region starts 16-byte aligned)
// ------------------------------------------------------------------------------------------------
template <int BITS>
struct Unit {
  uint32_t w[BITS];
};

template <int BITS>
__device__ __forceinline__ Unit<BITS> load_unit(const uint8_t* p) {
  Unit<BITS> u;
  if constexpr (BITS == 8) {
    uint4 a = ld_stream_v4(p), b = ld_stream_v4(p + 16);
    u.w[0] = a.x; u.w[1] = a.y; u.w[2] = a.z; u.w[3] = a.w;
    u.w[4] = b.x; u.w[5] = b.y; u.w[6] = b.z; u.w[7] = b.w;
  } else if constexpr (BITS == 4) {
    uint4 a = ld_stream_v4(p);
    u.w[0] = a.x; u.w[1] = a.y; u.w[2] = a.z; u.w[3] = a.w;
  } else if constexpr (BITS == 2) {
    uint2 a = ld_stream_v2(p);
    u.w[0] = a.x; u.w[1] = a.y;
  } else {  // 3-bit: 12-byte unit, 4-byte aligned
    u.w[0] = ld_stream_u32(p);
    u.w[1] = ld_stream_u32(p + 4);
    u.w[2] = ld_stream_u32(p + 8);
  }
  return u;
}

template <int BITS>
__device__ __forceinline__ uint32_t unit_code(const Unit<BITS>& u, int i) {
  const int bit = BITS * i;
  const int wi = bit >> 5, sh = bit & 31;
  uint32_t v = u.w[wi] >> sh;
  if (sh + BITS > 32) v |= u.w[wi + 1] << (32 - sh);
  return v & ((1u << BITS) - 1u);
}

}  // namespace wisp
