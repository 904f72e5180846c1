// Expert-parallel pack / unpack around the all-to-all exchanges of batched decode (64 tokens per step over all ranks).
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


// ---- peer-memory exchange (one process per GPU, buffers mapped with CUDA IPC) ----------------------
// Each rank owns one allocation (P2PLayout) that every peer maps.  For call n (the n-th MoE layer of
// the run, the same sequence on every rank) buffer set = n % 2 and epoch = the value of the rank's
// call counter after the dispatch:
//   dispatch   rank r stores its rows / routing rows for destination d straight into d's
//              recv_x[set][r] / recv_meta[set][r] over NVLink; the last CTA to finish publishes
//              flags[0][r] = epoch on every d (release, system scope) and bumps the local counter
//   wait       rank d waits until flags[0][s] >= epoch for every source s (bounded; a wait that runs
//              out sets WISP_STATUS_WAIT_TIMEOUT and returns)
//   (the batched MoE runs on recv_x[set] / recv_meta[set])
//   return     rank d stores its result row for (s, c) into s's y_back[set][d][c] and publishes
//              flags[1][d] = epoch on every s
//   combine    rank s waits for flags[1][*] >= epoch, then sums w * y_back[set][src_pos] per token
// Alternating sets keep a write for call n away from a peer still reading call n - 1; a peer cannot
// still be reading call n - 2, because it had to answer call n - 1 first.
constexpr int MAX_P2P = 8;
constexpr unsigned long long P2P_WAIT_NS = 2000000000ull;  // 2 s: a peer that never signals ends the wait

struct P2PLayout {
  int64_t recv_x, recv_meta, y_back, flags, ctr, bytes;
};

__host__ __device__ inline int64_t ru256(int64_t v) { return (v + 255) & ~int64_t(255); }

__host__ __device__ inline P2PLayout p2p_layout(int world, int64_t C, int64_t H) {
  P2PLayout L;
  L.recv_x = 0;
  L.recv_meta = ru256(L.recv_x + 2 * int64_t(world) * C * H * 2);
  L.y_back = ru256(L.recv_meta + 2 * int64_t(world) * C * 2 * 4);
  L.flags = ru256(L.y_back + 2 * int64_t(world) * C * H * 2);
  L.ctr = ru256(L.flags + 2 * int64_t(world) * 4);  // [0] epoch, [1] dispatch done, [2] return done
  L.bytes = ru256(L.ctr + 16);
  return L;
}

struct Peers {
  uint8_t* base[MAX_P2P];  // base[r] = rank r's allocation as mapped here (base[own rank] = the local one)
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// wait until flags[s] >= epoch for s < world (threads 0..world-1 of the calling CTA), bounded
__device__ __forceinline__ void p2p_wait_flags(const uint32_t* flags, int world, uint32_t epoch) {
  if (int(threadIdx.x) < world) {
    const unsigned long long t0 = globaltimer_ns();
    while (ld_acquire_sys(flags + threadIdx.x) < epoch) {  // epochs never wrap within a run (2^32 calls)
      if (globaltimer_ns() - t0 > P2P_WAIT_NS) {
        flag(WISP_STATUS_WAIT_TIMEOUT);
        break;
      }
      __nanosleep(200);
    }
  }
  __syncthreads();
}

// the last CTA of the grid to get here publishes flags[phase][rank] = epoch on every peer; `done` is a
// local counter (reset by that CTA), `ctr_epoch` the local call counter (bumped when bump != 0)
__device__ __forceinline__ void p2p_publish(const Peers& P, const P2PLayout& L, int world, int rank, int phase, uint32_t epoch,
                                            uint32_t* done, uint32_t* ctr_epoch, bool bump) {
  __syncthreads();  // the CTA's peer stores happen before thread 0's fence (cumulative), one fence per CTA
  if (threadIdx.x == 0) {
    __threadfence_system();
    const uint32_t prev = atomicAdd(done, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();  // every CTA's stores (their fences precede their arrivals)
      for (int d = 0; d < world; ++d)
        st_release_sys(reinterpret_cast<uint32_t*>(P.base[d] + L.flags) + phase * world + rank, epoch);
      *done = 0u;
      if (bump) *ctr_epoch = epoch;
    }
  }
}

__global__ void __launch_bounds__(256) ep_dispatch_p2p_kernel(const uint16_t* __restrict__ x, int N, int64_t H,
                                                              const int64_t* __restrict__ sel, int k, int E_local, int world,
                                                              int rank, int64_t C, int64_t slot_base, int set, Peers P,
                                                              int32_t* __restrict__ src_pos) {
  __shared__ int16_t dest_of[MAX_PAIRS];
  __shared__ int32_t cpos[MAX_PAIRS];
  __shared__ int count[MAX_P2P];
  const P2PLayout Lo = p2p_layout(world, C, H);
  uint32_t* ctr = reinterpret_cast<uint32_t*>(P.base[rank] + Lo.ctr);
  const int P_ = N * k, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  pdl_wait();
  const uint32_t epoch = ctr[0] + 1u;  // every CTA reads it before the last one bumps it
  for (int p = threadIdx.x; p < P_; p += blockDim.x) {
    const int64_t e = sel[p];
    int d = int(e / E_local);
    if (e < 0 || d >= world) {
      d = -1;
      if (blockIdx.x == 0) flag(WISP_STATUS_BAD_ROUTE);
    }
    dest_of[p] = int16_t(d);
  }
  __syncthreads();
  if (warp == 0) {
    for (int d = lane; d < world; d += 32) count[d] = 0;
    __syncwarp();
    for (int base = 0; base < P_; base += 32) {
      const int p = base + lane;
      const int d = p < P_ ? dest_of[p] : -1;
      int mine = 0;
      for (int dd = 0; dd < world; ++dd) {
        const unsigned m = __ballot_sync(0xffffffffu, d == dd);
        if (d == dd) mine = count[dd] + __popc(m & ((1u << lane) - 1u));
        __syncwarp();
        if (lane == 0) count[dd] += __popc(m);
        __syncwarp();
      }
      if (p < P_) cpos[p] = d >= 0 ? mine : -1;
    }
  }
  __syncthreads();
  // routing rows: my chunk [rank] of every destination's recv_meta[set]
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < int64_t(world) * C; i += int64_t(gridDim.x) * blockDim.x) {
    const int d = int(i / C);
    const int64_t c = i - int64_t(d) * C;
    if (c >= count[d]) {
      float* m = reinterpret_cast<float*>(P.base[d] + Lo.recv_meta) + ((int64_t(set) * world + rank) * C + c) * 2;
      m[0] = -1.0f;
      m[1] = 0.0f;
    }
  }
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < P_; p += gridDim.x * blockDim.x) {
    const int d = dest_of[p];
    if (d < 0) {
      src_pos[p] = -1;
      continue;
    }
    const int64_t c = cpos[p];
    src_pos[p] = int32_t(int64_t(d) * C + c);
    float* m = reinterpret_cast<float*>(P.base[d] + Lo.recv_meta) + ((int64_t(set) * world + rank) * C + c) * 2;
    m[0] = float(slot_base + (sel[p] - int64_t(d) * E_local));
    m[1] = 1.0f;
  }
  // rows: pair p of this CTA, 16-byte chunks, stored into the destination's memory
  const int64_t H8 = H / 8;
  for (int p = blockIdx.x; p < P_; p += gridDim.x) {
    const int d = dest_of[p];
    if (d < 0) continue;
    const uint4* src = reinterpret_cast<const uint4*>(x + int64_t(p / k) * H);
    uint4* dst = reinterpret_cast<uint4*>(P.base[d] + Lo.recv_x) + ((int64_t(set) * world + rank) * C + cpos[p]) * H8;
    for (int64_t i = threadIdx.x; i < H8; i += blockDim.x) dst[i] = src[i];
  }
  pdl_launch_dependents();
  p2p_publish(P, Lo, world, rank, 0, epoch, ctr + 1, ctr, true);
}

// rank-local: wait for every source's dispatch of the current call (one CTA of >= world threads)
__global__ void ep_wait_kernel(uint8_t* local, int world, int64_t C, int64_t H, int phase) {
  const P2PLayout Lo = p2p_layout(world, C, H);
  pdl_wait();
  const uint32_t epoch = reinterpret_cast<const uint32_t*>(local + Lo.ctr)[0];
  p2p_wait_flags(reinterpret_cast<const uint32_t*>(local + Lo.flags) + phase * world, world, epoch);
  pdl_launch_dependents();
}

// expert results back to their sources: row (s, c) of y (bf16 [world * C, H], the batched MoE output
// over recv_x[set]) goes to rank s's y_back[set][rank][c]; unused capacity is skipped
__global__ void __launch_bounds__(256) ep_return_p2p_kernel(const uint16_t* __restrict__ y, int world, int rank, int64_t C,
                                                            int64_t H, int set, Peers P) {
  const P2PLayout Lo = p2p_layout(world, C, H);
  uint32_t* ctr = reinterpret_cast<uint32_t*>(P.base[rank] + Lo.ctr);
  pdl_wait();
  const uint32_t epoch = ctr[0];
  const float* meta = reinterpret_cast<const float*>(P.base[rank] + Lo.recv_meta) + int64_t(set) * world * C * 2;
  const int64_t H8 = H / 8;
  for (int64_t row = blockIdx.x; row < int64_t(world) * C; row += gridDim.x) {
    if (meta[2 * row] < 0.0f) continue;  // unused capacity: nothing to return
    const int s = int(row / C);
    const int64_t c = row - int64_t(s) * C;
    const uint4* src = reinterpret_cast<const uint4*>(y + row * H);
    uint4* dst = reinterpret_cast<uint4*>(P.base[s] + Lo.y_back) + ((int64_t(set) * world + rank) * C + c) * H8;
    for (int64_t i = threadIdx.x; i < H8; i += blockDim.x) dst[i] = src[i];
  }
  pdl_launch_dependents();
  p2p_publish(P, Lo, world, rank, 1, epoch, ctr + 2, ctr, false);
}

// wait for every rank's returns of the current call, then out[t] = bf16(sum_j w[t][j] *
// y_back[set][src_pos[t*k + j]]) in a fixed order
__global__ void ep_combine_p2p_kernel(uint8_t* local, int world, int64_t C, int set, int N, int k, int64_t H,
                                      const int32_t* __restrict__ src_pos, const float* __restrict__ w, uint16_t* __restrict__ out) {
  const P2PLayout Lo = p2p_layout(world, C, H);
  pdl_wait();
  const uint32_t epoch = reinterpret_cast<const uint32_t*>(local + Lo.ctr)[0];
  p2p_wait_flags(reinterpret_cast<const uint32_t*>(local + Lo.flags) + world, world, epoch);
  pdl_launch_dependents();
  const uint16_t* yb = reinterpret_cast<const uint16_t*>(local + Lo.y_back) + int64_t(set) * world * C * H;
  const int64_t H4 = H / 4;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < int64_t(N) * H4; i += int64_t(gridDim.x) * blockDim.x) {
    const int t = int(i / H4);
    const int64_t h4 = i - int64_t(t) * H4;
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    for (int j = 0; j < k; ++j) {
      const int sp = src_pos[t * k + j];
      if (sp < 0) continue;
      const float wj = w[int64_t(t) * k + j];
      const uint2 v = reinterpret_cast<const uint2*>(yb + int64_t(sp) * H)[h4];
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
