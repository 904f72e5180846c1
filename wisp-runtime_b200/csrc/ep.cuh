// Expert-parallel pack / unpack around the all-to-all exchanges of batched decode.
// The experts of a layer are split contiguously over `world` ranks (E_local each); a (token, choice)
// pair goes to rank sel / E_local.  Buffers have a fixed capacity C per destination, so every shape is
// static and the exchange can live in a CUDA graph.
//
//   ep_dispatch_kernel  pair p = t*k + j -> destination d, slot c = rank of p among the pairs bound for
//                       d (pair order); send_x[d][c] = x[t], send_meta[d][c] = [slot_base + local id, 1],
//                       unused capacity = [-1, 0] (the batched MoE skips it); src_pos[p] = d*C + c
//   ep_combine_kernel   out[t] = bf16(sum_j w[t][j] * y_back[src_pos[t*k + j]]), j in order
//
// Every CTA recomputes the bucketing of all pairs in shared memory (one warp, ballots per
// destination: pair order is preserved, no atomics), then copies its share of the rows.
#pragma once
#include "common.cuh"

namespace wisp {
namespace ep {

constexpr int MAX_PAIRS = 2048;
constexpr int MAX_WORLD = 64;

__global__ void __launch_bounds__(256) ep_dispatch_kernel(const uint16_t* __restrict__ x, int N, int64_t H,
                                                          const int64_t* __restrict__ sel, int k, int E_local, int world,
                                                          int64_t C, int64_t slot_base, uint16_t* __restrict__ send_x,
                                                          float* __restrict__ send_meta, int32_t* __restrict__ src_pos) {
  __shared__ int16_t dest_of[MAX_PAIRS];
  __shared__ int32_t cpos[MAX_PAIRS];
  __shared__ int count[MAX_WORLD];
  const int P = N * k, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  pdl_wait();
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    const int64_t e = sel[p];
    int d = int(e / E_local);
    if (e < 0 || d >= world) {  // not a valid expert id: dropped (flagged), contributes nothing
      d = -1;
      if (blockIdx.x == 0) flag(WISP_STATUS_BAD_ROUTE);
    }
    dest_of[p] = int16_t(d);
  }
  __syncthreads();
  if (warp == 0) {  // ranks within each destination, in pair order
    for (int d = lane; d < world; d += 32) count[d] = 0;
    __syncwarp();
    for (int base = 0; base < P; base += 32) {
      const int p = base + lane;
      const int d = p < P ? dest_of[p] : -1;
      int mine = 0;
      for (int dd = 0; dd < world; ++dd) {
        const unsigned m = __ballot_sync(0xffffffffu, d == dd);
        if (d == dd) mine = count[dd] + __popc(m & ((1u << lane) - 1u));
        __syncwarp();
        if (lane == 0) count[dd] += __popc(m);
        __syncwarp();
      }
      if (p < P) cpos[p] = d >= 0 ? mine : -1;
    }
  }
  __syncthreads();
  // routing of the capacity slots: CTA-strided over [world * C)
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < int64_t(world) * C; i += int64_t(gridDim.x) * blockDim.x) {
    const int d = int(i / C);
    const int64_t c = i - int64_t(d) * C;
    if (c >= count[d]) {
      send_meta[2 * i] = -1.0f;
      send_meta[2 * i + 1] = 0.0f;
    }
  }
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < P; p += gridDim.x * blockDim.x) {
    const int d = dest_of[p];
    if (d < 0) {
      src_pos[p] = -1;
      continue;
    }
    const int64_t slot = int64_t(d) * C + cpos[p];
    src_pos[p] = int32_t(slot);
    send_meta[2 * slot] = float(slot_base + (sel[p] - int64_t(d) * E_local));
    send_meta[2 * slot + 1] = 1.0f;
  }
  pdl_launch_dependents();
  // rows: pair p of this CTA (p = blockIdx.x, blockIdx.x + gridDim.x, ...), 16-byte chunks
  const int64_t H8 = H / 8;
  for (int p = blockIdx.x; p < P; p += gridDim.x) {
    const int d = dest_of[p];
    if (d < 0) continue;
    const uint4* src = reinterpret_cast<const uint4*>(x + int64_t(p / k) * H);
    uint4* dst = reinterpret_cast<uint4*>(send_x + (int64_t(d) * C + cpos[p]) * H);
    for (int64_t i = threadIdx.x; i < H8; i += blockDim.x) dst[i] = src[i];
  }
}

__global__ void ep_combine_kernel(const uint16_t* __restrict__ y_back, int N, int k, int64_t H, const int32_t* __restrict__ src_pos,
                                  const float* __restrict__ w, uint16_t* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t H4 = H / 4;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < int64_t(N) * H4; i += int64_t(gridDim.x) * blockDim.x) {
    const int t = int(i / H4);
    const int64_t h4 = i - int64_t(t) * H4;
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    for (int j = 0; j < k; ++j) {
      const int sp = src_pos[t * k + j];
      if (sp < 0) continue;
      const float wj = w[int64_t(t) * k + j];
      const uint2 v = reinterpret_cast<const uint2*>(y_back + int64_t(sp) * H)[h4];
      s0 = fmaf(wj, __uint_as_float(v.x << 16), s0);
      s1 = fmaf(wj, __uint_as_float(v.x & 0xFFFF0000u), s1);
      s2 = fmaf(wj, __uint_as_float(v.y << 16), s2);
      s3 = fmaf(wj, __uint_as_float(v.y & 0xFFFF0000u), s3);
    }
    const uint32_t lo = uint32_t(f32_to_bf16(s0)) | (uint32_t(f32_to_bf16(s1)) << 16);
    const uint32_t hi = uint32_t(f32_to_bf16(s2)) | (uint32_t(f32_to_bf16(s3)) << 16);
    reinterpret_cast<uint2*>(out + int64_t(t) * H)[h4] = make_uint2(lo, hi);
  }
}

}  // namespace ep
}  // namespace wisp
