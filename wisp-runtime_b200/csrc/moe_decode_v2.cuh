// Fused MoE decode for one token, B200 form: two persistent kernels (one CTA per SM), chained with
// programmatic dependent launch (PDL).
//
//   gate/up : the k*I (gate row, up row) pairs are split evenly over the CTAs.  Each CTA copies its
//             rows (codes + fp16 scale/min windows) from the slot pool into shared memory with
//             cp.async.bulk, in chunks of CH rows, each chunk completing on its own mbarrier, and
//             computes a[j, r] = silu(g) * u as chunks land.  Right after issuing its copies it lets
//             the dependent grid launch (griddepcontrol.launch_dependents).
//   down    : the H output rows are split evenly over the CTAs; each CTA copies the down rows of all
//             k experts for its rows into shared memory BEFORE waiting on the gate/up grid
//             (griddepcontrol.wait), so the down-weight stream overlaps the gate/up phase.  Then it
//             reads a (fp32 [k, I], L2-resident) and produces out[h] = sum_j w_j (Wd_j[h] . a_j),
//             reduced in a fixed order (deterministic).
//
// Every byte of expert weight is moved by the bulk-copy engine straight into shared memory; the SMs
// only unpack and multiply.  Copies are 16-byte aligned windows: a scale/min run whose byte range
// does not start on a 16-byte boundary is fetched as the enclosing aligned window (always inside the
// slot, whose size is a multiple of 16) and indexed from its offset.
#pragma once
#include "common.cuh"
#include "moe_decode.cuh"

namespace wisp {
namespace v2 {

// Warps per CTA.  Sized so one gate/up CTA and one down CTA fit on an SM together (registers:
// 12 x 32 x <=120 + 8 x 32 x <=64 <= 64K; shared memory well under 227 KB at the Qwen3 shape), which is
// what lets the down grid start its weight copies while gate/up still computes.
constexpr int GU_WARPS = 12;
constexpr int DN_WARPS = 8;
constexpr int GU_THREADS = GU_WARPS * 32;
constexpr int DN_THREADS = DN_WARPS * 32;
constexpr int CH = 8;  // rows per gate/up chunk
constexpr unsigned WAIT_LIMIT = 1u << 24;  // bounded polling; a stuck copy sets WAIT_TIMEOUT

// ------------------------------------------------------------------------------------------------
// PTX wrappers: mbarrier, bulk copy, PDL
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// bounded wait on phase 0 of a single-use barrier; returns false (and flags) if it gave up
__device__ __forceinline__ bool mbar_wait(uint64_t* bar) {
  for (unsigned it = 0; it < WAIT_LIMIT; ++it)
    if (mbar_try_wait(bar, 0)) return true;
  flag(WISP_STATUS_WAIT_TIMEOUT);
  return false;
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }

// one 32-code unit from shared memory (vector loads; lane-contiguous units are bank-conflict free)
template <int BITS>
__device__ __forceinline__ Unit<BITS> load_unit_smem(const uint8_t* p) {
  Unit<BITS> u;
  if constexpr (BITS == 4) {
    const uint4 a = *reinterpret_cast<const uint4*>(p);
    u.w[0] = a.x; u.w[1] = a.y; u.w[2] = a.z; u.w[3] = a.w;
  } else if constexpr (BITS == 2) {
    const uint2 a = *reinterpret_cast<const uint2*>(p);
    u.w[0] = a.x; u.w[1] = a.y;
  } else {
#pragma unroll
    for (int w = 0; w < BITS; ++w) u.w[w] = reinterpret_cast<const uint32_t*>(p)[w];
  }
  return u;
}

__host__ __device__ __forceinline__ int64_t rd16(int64_t v) { return v & ~int64_t(15); }
__host__ __device__ __forceinline__ int64_t ru16(int64_t v) { return (v + 15) & ~int64_t(15); }

// window (aligned start, aligned size) covering [off, off+len) bytes; returns the start offset inside it
struct Win {
  int64_t start;
  uint32_t bytes;
  uint32_t skip;
};
__device__ __forceinline__ Win window(int64_t off, int64_t len) {
  Win w;
  w.start = rd16(off);
  w.bytes = uint32_t(ru16(off + len) - w.start);
  w.skip = uint32_t(off - w.start);
  return w;
}

// ------------------------------------------------------------------------------------------------
// shared-memory layouts (host and device agree through these formulas)
// ------------------------------------------------------------------------------------------------
struct GuLayout {
  int64_t row_bytes;   // code bytes per gate/up row
  int64_t sc_win;      // bytes reserved per scale (or min) window of one chunk
  int64_t chunk;       // bytes per chunk
  int max_rows;        // rows per CTA (upper bound)
  int max_chunks;      // chunks per CTA (upper bound)
  int64_t bytes;       // dynamic smem total (chunks + mbarriers)
};

__host__ __device__ inline GuLayout gu_layout(int H, int I, int k, int group, int bits, int nctas) {
  GuLayout L;
  L.row_bytes = int64_t(H) * bits / 8;
  const int64_t gpr = H / group;
  L.sc_win = ru16(int64_t(CH) * gpr * 2) + 16;
  L.chunk = 2 * CH * L.row_bytes + 4 * L.sc_win;
  const int64_t R = int64_t(k) * I;
  L.max_rows = int((R + nctas - 1) / nctas);
  L.max_chunks = (L.max_rows + CH - 1) / CH + 1;  // +1: a CTA range may straddle two experts
  L.bytes = L.max_chunks * L.chunk + 8 * L.max_chunks;
  return L;
}

struct DnLayout {
  int64_t row_bytes;   // code bytes per down row
  int64_t sc_win;      // bytes per scale (or min) window of one expert
  int64_t per_expert;  // bytes per expert block
  int max_rows;        // output rows per CTA (upper bound)
  int64_t bytes;       // dynamic smem total
};

__host__ __device__ inline DnLayout dn_layout(int H, int I, int k, int group, int bits, int nctas) {
  DnLayout L;
  L.row_bytes = int64_t(I) * bits / 8;
  L.max_rows = (H + nctas - 1) / nctas;
  const int64_t gpr = I / group;
  L.sc_win = ru16(int64_t(L.max_rows) * gpr * 2) + 16;
  L.per_expert = int64_t(L.max_rows) * L.row_bytes + 2 * L.sc_win;
  // + mbarrier per expert + partial sums [DN_WARPS][max_rows]
  L.bytes = int64_t(k) * L.per_expert + 8 * k + 4 * DN_WARPS * L.max_rows;
  return L;
}

// ------------------------------------------------------------------------------------------------
// gate/up
// ------------------------------------------------------------------------------------------------
template <int BITS, int UPL>
__global__ void __maxnreg__(120) gate_up_kernel(const uint8_t* __restrict__ pool,
                                                              const float* __restrict__ meta,
                                                              const uint16_t* __restrict__ x, MoeShape S,
                                                              float* __restrict__ a_out) {
  extern __shared__ __align__(128) uint8_t sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const GuLayout Lg = gu_layout(S.H, S.I, S.k, S.group, BITS, gridDim.x);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Lg.max_chunks * Lg.chunk);
  const int64_t R = int64_t(S.k) * S.I;
  const int64_t r_begin = R * blockIdx.x / gridDim.x, r_end = R * (blockIdx.x + 1) / gridDim.x;
  const int nrows = int(r_end - r_begin);
  const int gpr = S.H / S.group;
  const int64_t ngm = S.ng / 3;

  // routing and x come from the previous kernels in the stream
  pdl_wait();

  // chunk c covers rows [c_lo, c_hi) of the CTA range (cut at CH rows and at expert boundaries)
  // chunk starts: walk the range once (at most max_chunks chunks)
  if (threadIdx.x == 0) {
    for (int c = 0; c < Lg.max_chunks; ++c) mbar_init(&bars[c], 1);
    mbar_fence_init();
    int c = 0;
    for (int64_t r = r_begin; r < r_end; ++c) {
      const int j = int(r / S.I);
      const int64_t row = r - int64_t(j) * S.I;
      const int64_t cnt = min64(min64(CH, S.I - row), r_end - r);
      uint8_t* dst = sm + int64_t(c) * Lg.chunk;
      int64_t slot;
      const bool ok = route_slot(meta, j, S, slot);
      if (!ok) {
        flag(WISP_STATUS_BAD_SLOT);
        // nothing to copy: arrive with zero bytes so waiters pass; compute is skipped for bad slots
        mbar_expect_tx(&bars[c], 0);
      } else {
        const uint8_t* base = pool + slot * S.nbytes;
        const Win sg = window(S.ncode + 2 * (row * gpr), 2 * cnt * gpr);
        const Win mg = window(S.ncode + 2 * (S.ng + row * gpr), 2 * cnt * gpr);
        const Win su = window(S.ncode + 2 * (ngm + row * gpr), 2 * cnt * gpr);
        const Win mu = window(S.ncode + 2 * (S.ng + ngm + row * gpr), 2 * cnt * gpr);
        const uint32_t cb = uint32_t(cnt * Lg.row_bytes);
        mbar_expect_tx(&bars[c], 2 * cb + sg.bytes + mg.bytes + su.bytes + mu.bytes);
        bulk_g2s(dst, base + row * Lg.row_bytes, cb, &bars[c]);
        bulk_g2s(dst + CH * Lg.row_bytes, base + S.mat_bytes + row * Lg.row_bytes, cb, &bars[c]);
        uint8_t* sw = dst + 2 * CH * Lg.row_bytes;
        bulk_g2s(sw, base + sg.start, sg.bytes, &bars[c]);
        bulk_g2s(sw + Lg.sc_win, base + mg.start, mg.bytes, &bars[c]);
        bulk_g2s(sw + 2 * Lg.sc_win, base + su.start, su.bytes, &bars[c]);
        bulk_g2s(sw + 3 * Lg.sc_win, base + mu.start, mu.bytes, &bars[c]);
      }
      r += cnt;
    }
  }
  __syncthreads();
  // the down grid may launch now: its CTAs prefetch the down weights while this grid computes
  pdl_launch_dependents();

  // x in registers: lane owns units lane, lane+32, ... of a row (32 elements each)
  const int U = S.H / 32;
  float xv[UPL][32], xs[UPL];
#pragma unroll
  for (int t = 0; t < UPL; ++t) {
    const int u = min(lane + 32 * t, U - 1);
    const uint4* xp = reinterpret_cast<const uint4*>(x + u * 32);
    uint4 q[4];
#pragma unroll
    for (int v = 0; v < 4; ++v) q[v] = xp[v];
    float s = 0.0f;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const uint32_t wds[4] = {q[v].x, q[v].y, q[v].z, q[v].w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        xv[t][8 * v + 2 * h] = __uint_as_float(wds[h] << 16);
        xv[t][8 * v + 2 * h + 1] = __uint_as_float(wds[h] & 0xFFFF0000u);
        s += xv[t][8 * v + 2 * h] + xv[t][8 * v + 2 * h + 1];
      }
    }
    xs[t] = s;
  }

  // rows are dealt to warps round-robin; the chunk of row i is found by re-walking the cut rule
  for (int i = warp; i < nrows; i += GU_WARPS) {
    // locate row i: chunks are cut every CH rows and at expert boundaries
    int c = 0;
    int64_t r = r_begin, idx_in_chunk = 0;
    {
      int64_t remaining = i;
      while (true) {
        const int j = int(r / S.I);
        const int64_t row = r - int64_t(j) * S.I;
        const int64_t cnt = min64(min64(CH, S.I - row), r_end - r);
        if (remaining < cnt) {
          idx_in_chunk = remaining;
          break;
        }
        remaining -= cnt;
        r += cnt;
        ++c;
      }
    }
    const int64_t rr = r + idx_in_chunk;
    const int j = int(rr / S.I);
    const int64_t row_c0 = r - int64_t(j) * S.I;  // first row of the chunk
    int64_t slot;
    if (!route_slot(meta, j, S, slot)) {
      if (lane == 0) a_out[rr] = 0.0f;
      continue;
    }
    mbar_wait(&bars[c]);
    const uint8_t* cg = sm + int64_t(c) * Lg.chunk + idx_in_chunk * Lg.row_bytes;
    const uint8_t* cu = cg + CH * Lg.row_bytes;
    const uint8_t* sw = sm + int64_t(c) * Lg.chunk + 2 * CH * Lg.row_bytes;
    // offsets of this row's scales inside the four windows
    const uint32_t sk_sg = uint32_t((S.ncode + 2 * (row_c0 * gpr)) & 15);
    const uint32_t sk_mg = uint32_t((S.ncode + 2 * (S.ng + row_c0 * gpr)) & 15);
    const uint32_t sk_su = uint32_t((S.ncode + 2 * (ngm + row_c0 * gpr)) & 15);
    const uint32_t sk_mu = uint32_t((S.ncode + 2 * (S.ng + ngm + row_c0 * gpr)) & 15);
    const uint16_t* ssg = reinterpret_cast<const uint16_t*>(sw + sk_sg) + idx_in_chunk * gpr;
    const uint16_t* smg = reinterpret_cast<const uint16_t*>(sw + Lg.sc_win + sk_mg) + idx_in_chunk * gpr;
    const uint16_t* ssu = reinterpret_cast<const uint16_t*>(sw + 2 * Lg.sc_win + sk_su) + idx_in_chunk * gpr;
    const uint16_t* smu = reinterpret_cast<const uint16_t*>(sw + 3 * Lg.sc_win + sk_mu) + idx_in_chunk * gpr;
    float accg = 0.0f, accu = 0.0f;
#pragma unroll
    for (int t = 0; t < UPL; ++t) {
      const int u = lane + 32 * t;
      if (u < U) {
        const Unit<BITS> qg = load_unit_smem<BITS>(cg + u * 4 * BITS);
        const Unit<BITS> qu = load_unit_smem<BITS>(cu + u * 4 * BITS);
        float dg = 0.0f, du = 0.0f;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          dg = fmaf(small_u2f(unit_code<BITS>(qg, e)), xv[t][e], dg);
          du = fmaf(small_u2f(unit_code<BITS>(qu, e)), xv[t][e], du);
        }
        const int gi = (u * 32) / S.group;
        accg += f16_bits_to_f32(ssg[gi]) * dg + f16_bits_to_f32(smg[gi]) * xs[t];
        accu += f16_bits_to_f32(ssu[gi]) * du + f16_bits_to_f32(smu[gi]) * xs[t];
      }
    }
    accg = warp_sum(accg);
    accu = warp_sum(accu);
    if (lane == 0) a_out[rr] = silu_mul(accg, accu);
  }
  // make sure no copy is still landing in shared memory when the CTA retires
  if (threadIdx.x == 0) {
    int c = 0;
    for (int64_t r = r_begin; r < r_end; ++c) {
      const int j = int(r / S.I);
      const int64_t row = r - int64_t(j) * S.I;
      const int64_t cnt = min64(min64(CH, S.I - row), r_end - r);
      mbar_wait(&bars[c]);
      r += cnt;
    }
  }
}

// ------------------------------------------------------------------------------------------------
// down + weighted combine
// ------------------------------------------------------------------------------------------------
template <int BITS, int UPL>
__global__ void __maxnreg__(64) down_kernel(const uint8_t* __restrict__ pool,
                                                           const float* __restrict__ meta,
                                                           const float* __restrict__ a, MoeShape S,
                                                           uint16_t* __restrict__ out) {
  extern __shared__ __align__(128) uint8_t sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const DnLayout Ld = dn_layout(S.H, S.I, S.k, S.group, BITS, gridDim.x);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + int64_t(S.k) * Ld.per_expert);
  float* part = reinterpret_cast<float*>(bars + S.k);  // [DN_WARPS][max_rows]
  const int h0 = int(int64_t(S.H) * blockIdx.x / gridDim.x), h1 = int(int64_t(S.H) * (blockIdx.x + 1) / gridDim.x);
  const int nrows = h1 - h0;
  const int gpr = S.I / S.group;
  const int64_t ngm = S.ng / 3;

  // meta is final before the gate/up grid released us; the weights do not depend on it
  if (threadIdx.x == 0) {
    for (int j = 0; j < S.k; ++j) mbar_init(&bars[j], 1);
    mbar_fence_init();
    for (int j = 0; j < S.k; ++j) {
      int64_t slot;
      if (nrows <= 0 || !route_slot(meta, j, S, slot)) {
        mbar_expect_tx(&bars[j], 0);
        continue;
      }
      const uint8_t* base = pool + slot * S.nbytes;
      uint8_t* dst = sm + int64_t(j) * Ld.per_expert;
      const uint32_t cb = uint32_t(int64_t(nrows) * Ld.row_bytes);
      const Win ws = window(S.ncode + 2 * (2 * ngm + int64_t(h0) * gpr), 2 * int64_t(nrows) * gpr);
      const Win wm = window(S.ncode + 2 * (S.ng + 2 * ngm + int64_t(h0) * gpr), 2 * int64_t(nrows) * gpr);
      mbar_expect_tx(&bars[j], cb + ws.bytes + wm.bytes);
      bulk_g2s(dst, base + 2 * S.mat_bytes + int64_t(h0) * Ld.row_bytes, cb, &bars[j]);
      bulk_g2s(dst + int64_t(Ld.max_rows) * Ld.row_bytes, base + ws.start, ws.bytes, &bars[j]);
      bulk_g2s(dst + int64_t(Ld.max_rows) * Ld.row_bytes + Ld.sc_win, base + wm.start, wm.bytes, &bars[j]);
    }
  }
  for (int i = threadIdx.x; i < DN_WARPS * Ld.max_rows; i += DN_THREADS) part[i] = 0.0f;
  __syncthreads();
  // a is written by the gate/up grid
  pdl_wait();

  const int U = S.I / 32;
  // work split: piece p = (expert j, row subset sub) with p = j * per + sub; warp w takes pieces
  // w, w + DN_WARPS, ...; a warp accumulates into its own row of `part`, so the combine is ordered
  const int per = S.k <= DN_WARPS ? DN_WARPS / S.k : 1;
  const uint32_t sk_s = uint32_t((S.ncode + 2 * (2 * ngm + int64_t(h0) * gpr)) & 15);
  const uint32_t sk_m = uint32_t((S.ncode + 2 * (S.ng + 2 * ngm + int64_t(h0) * gpr)) & 15);
  for (int p = warp; p < S.k * per; p += DN_WARPS) {
    const int j = p / per, sub = p - j * per;
    int64_t slot;
    if (!route_slot(meta, j, S, slot)) continue;
    const float wj = meta[S.k + j];
    // this lane's slice of a_j in registers (L2-resident, written by the gate/up grid)
    float av[UPL][32], as[UPL];
#pragma unroll
    for (int t = 0; t < UPL; ++t) {
      const int u = min(lane + 32 * t, U - 1);
      const float4* ap = reinterpret_cast<const float4*>(a + int64_t(j) * S.I + u * 32);
      float4 q[8];
#pragma unroll
      for (int v = 0; v < 8; ++v) q[v] = ap[v];
      float s = 0.0f;
#pragma unroll
      for (int v = 0; v < 8; ++v) {
        av[t][4 * v] = q[v].x;
        av[t][4 * v + 1] = q[v].y;
        av[t][4 * v + 2] = q[v].z;
        av[t][4 * v + 3] = q[v].w;
        s += (q[v].x + q[v].y) + (q[v].z + q[v].w);
      }
      as[t] = s;
    }
    mbar_wait(&bars[j]);
    const uint8_t* blk = sm + int64_t(j) * Ld.per_expert;
    const uint16_t* ss = reinterpret_cast<const uint16_t*>(blk + int64_t(Ld.max_rows) * Ld.row_bytes + sk_s);
    const uint16_t* sm_ = reinterpret_cast<const uint16_t*>(blk + int64_t(Ld.max_rows) * Ld.row_bytes + Ld.sc_win + sk_m);
    for (int r = sub; r < nrows; r += per) {
      const uint8_t* row = blk + int64_t(r) * Ld.row_bytes;
      float acc = 0.0f;
#pragma unroll
      for (int t = 0; t < UPL; ++t) {
        const int u = lane + 32 * t;
        if (u < U) {
          const Unit<BITS> q = load_unit_smem<BITS>(row + u * 4 * BITS);
          float d = 0.0f;
#pragma unroll
          for (int e = 0; e < 32; ++e) d = fmaf(small_u2f(unit_code<BITS>(q, e)), av[t][e], d);
          const int gi = r * gpr + (u * 32) / S.group;
          acc += f16_bits_to_f32(ss[gi]) * d + f16_bits_to_f32(sm_[gi]) * as[t];
        }
      }
      acc = warp_sum(acc);
      if (lane == 0) part[warp * Ld.max_rows + r] += wj * acc;
    }
  }
  __syncthreads();
  // fixed-order reduction over warps: deterministic
  for (int r = threadIdx.x; r < nrows; r += DN_THREADS) {
    float s = 0.0f;
    for (int w = 0; w < DN_WARPS; ++w) s += part[w * Ld.max_rows + r];
    out[h0 + r] = f32_to_bf16(s);
  }
  // no copy may still be landing when the CTA retires (also covers experts no warp consumed)
  if (threadIdx.x == 0)
    for (int j = 0; j < S.k; ++j) mbar_wait(&bars[j]);
}

}  // namespace v2
}  // namespace wisp
