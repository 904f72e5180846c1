// Fused MoE decode for one token: TMA bulk copies (cp.async.bulk, no multicast) feeding warp-level MMA.
//
// Data movement.  gate/up: every warp owns one piece of work (8 gate + the same 8 up rows over one K
// half) and brings exactly its bytes from the slot pool into its own shared-memory region with one
// bulk copy per row, issued by lanes 0-15, plus four scale/min windows issued by lanes 16-19; all
// complete on the warp's mbarrier.  Rows land at stride (bytes + 16*BITS), which makes the per-lane
// fragment loads bank-conflict free.  No CTA-wide barrier sits between issuing and consuming.
// down: the CTA's output rows are contiguous in each expert's down matrix, so one bulk copy per
// routed expert (plus two windows) brings them in; it is issued before the grid waits on the gate/up
// grid (programmatic dependent launch), so the down weights stream while gate/up still computes.
//
// Math.  Codes become u8 operands of the integer MMA (mma.sync m16n8k32, u8 x s8 -> s32) with one AND
// per 4 codes (unpack_imma.cuh); activations enter as three int8 limbs of a per-group 23-bit fixed
// point, so every partial sum is an exact int32.  Groups are processed in pairs (independent chains);
// lanes that hold no B column read a shared zero block (no divergence).
//   gate/up piece: 8 gate rows (A rows 0-7) + the same 8 up rows (A rows 8-15) over half of H;
//                  B column 0 = scaled, permuted x.
//   down piece:    16 output rows of one expert over all of I; B columns 0/1 = bf16 hi/lo of a_j.
#pragma once
#include "common.cuh"
#include "moe_decode.cuh"
#include "tma.cuh"
#include "unpack_imma.cuh"

namespace wisp {
namespace v4 {

constexpr int GU_WARPS = 12;
constexpr int DN_WARPS = 8;
constexpr int GU_THREADS = GU_WARPS * 32;
constexpr int DN_THREADS = DN_WARPS * 32;
constexpr int CH = 8;           // rows per gate/up block (A rows 0-7 gate, 8-15 the same up rows)
constexpr int NSPLIT = 2;       // K halves: two warps per gate/up block
constexpr int DN_SPLIT = 1;     // a down piece is one expert over all of I (one accumulator chain)
constexpr int MAX_REGIONS = GU_WARPS / 2;  // gate/up blocks in flight per CTA (two warps each)
constexpr int SMEM_LIMIT = 220 * 1024;
// register caps that let one down CTA sit beside one gate/up CTA on an SM (65536 registers)
constexpr int SM_SMEM_BYTES = 228 * 1024;  // shared memory of one B200 SM
constexpr int GU_REGS = 96;
constexpr int DN_REGS = 104;
static_assert(GU_THREADS * GU_REGS + DN_THREADS * DN_REGS <= 65536, "gate/up and down CTAs must fit one SM together");

template <int BITS>
__device__ __forceinline__ void lds_unit(const uint8_t* p, uint32_t (&w)[BITS]) {
  if constexpr (BITS == 4) {
    const uint4 a = *reinterpret_cast<const uint4*>(p);
    w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
  } else if constexpr (BITS == 2) {
    const uint2 a = *reinterpret_cast<const uint2*>(p);
    w[0] = a.x; w[1] = a.y;
  } else {
#pragma unroll
    for (int i = 0; i < BITS; ++i) w[i] = reinterpret_cast<const uint32_t*>(p)[i];
  }
}

// ------------------------------------------------------------------------------------------------
// shared-memory layouts (host and device share these formulas)
// ------------------------------------------------------------------------------------------------
// routing scratch (MoeRoute): meta [64] + reduction [32] + logits/ids/probabilities [512 + 64] floats
constexpr int ROUTE_BYTES = (64 + 32 + 512 + 64) * 4;

struct GuL {
  int groups, gph, gpr;  // 128-code groups per row / per K half; quant groups per row
  int nblk_max, R;       // max 8-row blocks per CTA; block regions in flight
  int64_t row_bytes, sc_win, region;
  int64_t off_bx, off_gsum, off_zero, off_halves, off_bars, off_route, bytes;
};

// gate/up shared memory: R regions of [8 gate rows | 8 up rows | 4 scale/min windows], each row
// a contiguous copy of the matrix (row stride = row bytes), then the B operand and bookkeeping; every
// part starts on a 16-byte boundary
__host__ __device__ inline GuL gu_layout_for(int H, int I, int k, int group, int bits, int nctas, int R) {
  GuL L;
  L.groups = H / 128;
  L.gph = (L.groups + 1) / 2;
  L.gpr = H / group;
  L.nblk_max = (k * I / CH + nctas - 1) / nctas;
  L.R = R;
  L.row_bytes = int64_t(H) * bits / 8;
  L.sc_win = ru16(int64_t(CH) * L.gpr * 2) + 16;
  L.region = ru16(2 * CH * L.row_bytes + 4 * L.sc_win);
  L.off_bx = int64_t(R) * L.region;                             // [H/32 units][3 limbs][8] u32
  L.off_gsum = ru16(L.off_bx + int64_t(H / 32) * 24 * 4);       // [H/128][2] f32: (sum of x, 2^-e)
  L.off_zero = ru16(L.off_gsum + int64_t(L.groups) * 2 * 4);    // 64 zero bytes
  L.off_halves = ru16(L.off_zero + 64);                         // [nblk_max][2 halves][CH][2] f32
  L.off_bars = ru16(L.off_halves + int64_t(L.nblk_max) * NSPLIT * CH * 2 * 4);  // [R] mbarriers
  L.off_route = ru16(L.off_bars + 8 * int64_t(R));                 // routing scratch
  L.bytes = L.off_route + ROUTE_BYTES;
  return L;
}

// the largest region count (<= MAX_REGIONS, <= blocks per CTA) whose layout fits; R = 0 if none
__host__ __device__ inline GuL gu_layout(int H, int I, int k, int group, int bits, int nctas) {
  const int nblk_max = (k * I / CH + nctas - 1) / nctas;
  int R = nblk_max < MAX_REGIONS ? nblk_max : MAX_REGIONS;
  GuL L = gu_layout_for(H, I, k, group, bits, nctas, R);
  while (R > 1 && L.bytes > SMEM_LIMIT) L = gu_layout_for(H, I, k, group, bits, nctas, --R);
  if (L.bytes > SMEM_LIMIT) L.R = 0;
  return L;
}

struct DnL {
  int groups, groups_per_piece, gpr, units, rows_max;
  int64_t row_bytes, sc_win, per_expert;
  int64_t off_bd, off_dsum, off_zero, off_part, off_bar, off_route, bytes;
};

__host__ __device__ inline DnL dn_layout(int H, int I, int k, int group, int bits, int nctas) {
  DnL L;
  L.groups = I / 128;
  L.groups_per_piece = (L.groups + DN_SPLIT - 1) / DN_SPLIT;
  L.gpr = I / group;
  L.units = I / 32;
  L.rows_max = (H + nctas - 1) / nctas;  // <= 16 (checked on the host)
  L.row_bytes = int64_t(I) * bits / 8;
  L.sc_win = ru16(int64_t(16) * L.gpr * 2) + 16;
  // an expert's rows land contiguous (one bulk copy); 16 rows reserved so the MMA block never reads
  // past its slab (rows past nrows hold stale bytes and are never stored)
  L.per_expert = ru16(16 * L.row_bytes + 2 * L.sc_win);
  L.off_bd = int64_t(k) * L.per_expert;                              // [k][units][3 limbs][8] u32
  L.off_dsum = ru16(L.off_bd + int64_t(k) * L.units * 24 * 4);       // [k][groups][2] f32: (sum of a, 2^-e)
  L.off_zero = ru16(L.off_dsum + int64_t(k) * L.groups * 2 * 4);     // 64 zero bytes
  L.off_part = ru16(L.off_zero + 64);                                // [DN_WARPS][16] f32
  L.off_bar = ru16(L.off_part + DN_WARPS * 16 * 4);                  // [k] mbarriers
  L.off_route = ru16(L.off_bar + 8 * int64_t(k));                    // routing scratch
  L.bytes = L.off_route + ROUTE_BYTES;
  return L;
}

__device__ __forceinline__ void lds_b8(const uint32_t* p, uint32_t (&b)[8]) {
  const uint4* p4 = reinterpret_cast<const uint4*>(p);
  const uint4 t0 = p4[0], t1 = p4[1];
  b[0] = t0.x; b[1] = t0.y; b[2] = t0.z; b[3] = t0.w;
  b[4] = t1.x; b[5] = t1.y; b[6] = t1.z; b[7] = t1.w;
}

__device__ __forceinline__ float quad_max(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
  return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
}

// one unit's activations -> its B limbs in shared memory; returns its exponent e (shared by the
// 4 lanes of the group, which must be the 4 consecutive lanes calling together)
template <int BITS>
__device__ __forceinline__ int store_b_limbs(const float (&v)[32], uint32_t* dst, bool store) {
  float am = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) am = fmaxf(am, fabsf(v[i]));
  const int e = group_exponent(quad_max(am));
  uint32_t L[3][8];
  build_b_limbs<BITS>(v, e, L);
  if (store) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int l = 0; l < 3; ++l) {
      d4[2 * l] = make_uint4(L[l][0], L[l][1], L[l][2], L[l][3]);
      d4[2 * l + 1] = make_uint4(L[l][4], L[l][5], L[l][6], L[l][7]);
    }
  }
  return e;
}

// sum over the 4 lanes that hold the 4 units of one 128-code group (lanes 4i..4i+3)
__device__ __forceinline__ float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  return v;
}

// ------------------------------------------------------------------------------------------------
// Source of routed expert j.  PAGED = false compiles the host-store branch away (slots only), so the
// resident-pool path is the same code whether or not paging exists.
template <bool PAGED>
__device__ __forceinline__ const uint8_t* src_of(float f, const MoeShape& S, const uint8_t* pool, const MoeRoute& RT, bool& host) {
  if constexpr (PAGED) {
    return expert_src(f, S, pool, RT, host);
  } else {
    host = false;
    return (f >= 0.0f && f < float(S.nslots)) ? pool + int64_t(f) * S.nbytes : nullptr;
  }
}

template <int BITS, bool PAGED>
__global__ void __maxnreg__(GU_REGS) gate_up_kernel(const uint8_t* __restrict__ pool,
                                                                const float* __restrict__ meta,
                                                                const uint16_t* __restrict__ x, MoeShape S,
                                                                float* __restrict__ a_out, MoeRoute RT) {
  extern __shared__ __align__(128) uint8_t sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const GuL Lg = gu_layout(S.H, S.I, S.k, S.group, BITS, gridDim.x);
  const int R = Lg.R;
  uint32_t* bx = reinterpret_cast<uint32_t*>(sm + Lg.off_bx);
  float* gsum = reinterpret_cast<float*>(sm + Lg.off_gsum);
  const uint32_t* zero = reinterpret_cast<const uint32_t*>(sm + Lg.off_zero);
  float* halves = reinterpret_cast<float*>(sm + Lg.off_halves);
  uint64_t* gbar = reinterpret_cast<uint64_t*>(sm + Lg.off_bars);
  const int64_t ngm = S.ng / 3;
  // this CTA owns 8-row blocks [b0, b1) of the k*I (expert, row) list (I % 8 == 0: a block never
  // straddles two experts); region r takes blocks b0 + r, b0 + r + R, ...; warps 2r and 2r+1 take
  // its two K halves
  const int nblk_all = S.k * S.I / CH;
  const int b0 = int(int64_t(nblk_all) * blockIdx.x / gridDim.x), b1 = int(int64_t(nblk_all) * (blockIdx.x + 1) / gridDim.x);
  const int nb = b1 - b0;

  pdl_wait();  // routing and x come from earlier kernels in the stream
  // the down grid may launch now: routing is final (its CTAs read the intermediate only after their
  // own griddepcontrol.wait)
  pdl_launch_dependents();
  const float* mt = meta;  // [slots | weights]: the caller's buffer, or computed here from the logits
  if (RT.logits) {
    float* rs = reinterpret_cast<float*>(sm + Lg.off_route);
    route_from_logits<true>(RT, S.k, rs, rs + 64, rs + 96);
    mt = rs;
    if (PAGED && RT.miss_count && blockIdx.x == 0 && int(threadIdx.x) < S.k && rs[threadIdx.x] <= -1.0f) atomicAdd(RT.miss_count, 1);
  }

  // one warp (lanes 0-5) issues block bi into region bi % R: the 8 gate rows and the same 8 up rows
  // (each one contiguous range of its matrix) and the four scale/min windows, on the region's mbarrier
  auto issue_block = [&](int bi) {
    const int r = bi % R;
    const int blk = b0 + bi;
    const int j = blk * CH / S.I, row0 = blk * CH - j * S.I;
    bool host;
    const uint8_t* base = src_of<PAGED>(mt[j], S, pool, RT, host);
    const bool ok = base != nullptr;
    uint8_t* reg = sm + int64_t(r) * Lg.region;
    const uint32_t cb = uint32_t(CH * Lg.row_bytes);
    if (PAGED && host) {  // not resident: the warp copies the same ranges from the host store, then arrives
      warp_copy_g2s(reg, base + int64_t(row0) * Lg.row_bytes, cb, lane);
      warp_copy_g2s(reg + cb, base + S.mat_bytes + int64_t(row0) * Lg.row_bytes, cb, lane);
      for (int arr = 0; arr < 4; ++arr) {
        const Win w = window(S.ncode + 2 * ((arr & 1) * S.ng + (arr >> 1) * ngm + int64_t(row0) * Lg.gpr), 2 * CH * Lg.gpr);
        warp_copy_g2s(reg + 2 * cb + arr * Lg.sc_win, base + w.start, w.bytes, lane);
      }
      __syncwarp();
      if (lane == 0) mbar_expect_tx(&gbar[r], 0);
      return;
    }
    if (lane == 0) {
      if (!ok) flag(WISP_STATUS_BAD_SLOT);  // skipped: contributes nothing
      uint32_t tx = 0;
      if (ok) {
        tx = 2 * cb;
        for (int arr = 0; arr < 4; ++arr)
          tx += window(S.ncode + 2 * ((arr & 1) * S.ng + (arr >> 1) * ngm + int64_t(row0) * Lg.gpr), 2 * CH * Lg.gpr).bytes;
      }
      mbar_expect_tx(&gbar[r], tx);
    }
    __syncwarp();
    if (ok && lane < 6) {
      if (lane < 2) {  // 0: gate rows, 1: up rows
        bulk_g2s(reg + lane * cb, base + lane * S.mat_bytes + int64_t(row0) * Lg.row_bytes, cb, &gbar[r]);
      } else {
        const int arr = lane - 2;  // 0 gate s, 1 gate m, 2 up s, 3 up m
        const Win w = window(S.ncode + 2 * ((arr & 1) * S.ng + (arr >> 1) * ngm + int64_t(row0) * Lg.gpr), 2 * CH * Lg.gpr);
        bulk_g2s(reg + 2 * cb + arr * Lg.sc_win, base + w.start, w.bytes, &gbar[r]);
      }
    }
  };
  if (warp < 2 * R && (warp & 1) == 0) {
    if (lane == 0) {
      mbar_init(&gbar[warp >> 1], 1);
      mbar_fence_init();
    }
    __syncwarp();
    if ((warp >> 1) < nb) issue_block(warp >> 1);
  }
  // the down rows the down kernel's CTA of the same index will read, pulled into L2 now (unless that
  // CTA runs beside this one and brings them itself)
  if (warp == GU_WARPS - 1 && !S.dn_beside) {
    const int h0 = int(int64_t(S.H) * blockIdx.x / gridDim.x), h1 = int(int64_t(S.H) * (blockIdx.x + 1) / gridDim.x);
    const int64_t gpr_d = S.I / S.group, row_d = int64_t(S.I) * BITS / 8;
    for (int j = lane; j < S.k && h1 > h0; j += 32) {
      bool host;
      const uint8_t* base = src_of<PAGED>(mt[j], S, pool, RT, host);
      if (!base || host) continue;
      prefetch_l2(base + 2 * S.mat_bytes + int64_t(h0) * row_d, uint32_t(int64_t(h1 - h0) * row_d));
      const int64_t len = 2 * int64_t(h1 - h0) * gpr_d;
      const Win ws = window(S.ncode + 2 * (2 * ngm + int64_t(h0) * gpr_d), len);
      const Win wm = window(S.ncode + 2 * (S.ng + 2 * ngm + int64_t(h0) * gpr_d), len);
      prefetch_l2(base + ws.start, ws.bytes);
      prefetch_l2(base + wm.start, wm.bytes);
    }
  }

  // ---- B operand from x, one thread per 32-element unit: on the warps without a block when there
  //      are enough of them, else on all threads after their copies are issued
  const int units = S.H / 32;
  const int spare = (GU_WARPS - 2 * R) * 32;
  const int first = spare >= units ? 2 * R * 32 : 0;  // multiple of 32: whole warps build
  const int nthr = int(blockDim.x) - first;
  // warp-uniform loop (the quad shuffles need every lane); lanes past the last unit read a valid
  // unit and store nothing
  for (int ub = (int(threadIdx.x) - first) & ~31; int(threadIdx.x) >= first && ub < units; ub += nthr) {
    const int u = ub + lane;
    const int uu = min(u, units - 1);
    float v[32];
    const uint4* xp = reinterpret_cast<const uint4*>(x + uu * 32);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 t = xp[q];
      const uint32_t wd[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
      for (int hh = 0; hh < 4; ++hh) {
        v[8 * q + 2 * hh] = __uint_as_float(wd[hh] << 16);
        v[8 * q + 2 * hh + 1] = __uint_as_float(wd[hh] & 0xFFFF0000u);
      }
    }
    const int e = store_b_limbs<BITS>(v, bx + u * 24, u < units);
    float sx = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) sx += v[i];
    sx = quad_sum(u < units ? sx : 0.0f);
    if (u < units && (u & 3) == 0) {
      gsum[2 * (u >> 2)] = sx;
      gsum[2 * (u >> 2) + 1] = pow2(-e);
    }
  }
  if (threadIdx.x < 16) reinterpret_cast<uint32_t*>(sm + Lg.off_zero)[threadIdx.x] = 0u;
  __syncthreads();

  // ---- warp (2r + h) computes K half h of the blocks of region r
  if (warp < 2 * R) {
    const int r = warp >> 1, hf = warp & 1;
    const uint8_t* reg = sm + int64_t(r) * Lg.region;
    const int64_t cb = CH * Lg.row_bytes;
    const int G0 = hf * Lg.gph;
    const int ng = min(Lg.gph, Lg.groups - G0);
    const int sarr = c == 1 ? 2 : 0;  // lane c = 0 finishes the gate row g, c = 1 the up row g
    int round = 0;
    for (int bi = r; bi < nb; bi += R, ++round) {
      if (round > 0) {  // the region is free once both halves of its previous block are done
        named_sync(1 + r, 64);
        if (hf == 0) issue_block(bi);
      }
      const int blk = b0 + bi;
      const int j = blk * CH / S.I, row0 = blk * CH - j * S.I;
      bool host;
      const bool ok = src_of<PAGED>(mt[j], S, pool, RT, host) != nullptr;
      const uint32_t sskip = window(S.ncode + 2 * ((sarr >> 1) * ngm + int64_t(row0) * Lg.gpr), 1).skip;
      const uint32_t mskip = window(S.ncode + 2 * (S.ng + (sarr >> 1) * ngm + int64_t(row0) * Lg.gpr), 1).skip;
      const uint8_t* sw = reg + 2 * cb;
      const uint16_t* srow = reinterpret_cast<const uint16_t*>(sw + sarr * Lg.sc_win + sskip) + g * Lg.gpr;
      const uint16_t* mrow = reinterpret_cast<const uint16_t*>(sw + (sarr + 1) * Lg.sc_win + mskip) + g * Lg.gpr;
      const uint8_t* rowg = reg + g * Lg.row_bytes;
      const uint8_t* rowu = reg + cb + g * Lg.row_bytes;
      mbar_wait(&gbar[r], uint32_t(round & 1));  // completes at once (no bytes) for a skipped expert
      float acc = 0.0f;
      for (int G = 0; G < ng; G += 2) {
        if (!ok) break;
        const int Ga = G0 + G, Gb = G0 + min(G + 1, ng - 1);  // an odd tail repeats the last group
        uint32_t wa0[BITS], wb0[BITS], wa1[BITS], wb1[BITS], bb0[8], bb1[8];
        lds_unit<BITS>(rowg + (Ga * 4 + c) * 4 * BITS, wa0);
        lds_unit<BITS>(rowu + (Ga * 4 + c) * 4 * BITS, wb0);
        lds_unit<BITS>(rowg + (Gb * 4 + c) * 4 * BITS, wa1);
        lds_unit<BITS>(rowu + (Gb * 4 + c) * 4 * BITS, wb1);
        lds_b8(g < 3 ? bx + ((4 * Ga + c) * 3 + g) * 8 : zero, bb0);
        lds_b8(g < 3 ? bx + ((4 * Gb + c) * 3 + g) * 8 : zero, bb1);
        int d0[4], d1[4];
        imma_group<BITS>(wa0, wb0, bb0, d0);
        imma_group<BITS>(wa1, wb1, bb1, d1);
        const float D0 = quad_row_dot(d0, c), D1 = quad_row_dot(d1, c);
        {
          const int qg = Ga >> S.gshift;
          acc += f16_bits_to_f32(srow[qg]) * (D0 * gsum[2 * Ga + 1]) + f16_bits_to_f32(mrow[qg]) * gsum[2 * Ga];
        }
        if (Gb != Ga) {
          const int qg = Gb >> S.gshift;
          acc += f16_bits_to_f32(srow[qg]) * (D1 * gsum[2 * Gb + 1]) + f16_bits_to_f32(mrow[qg]) * gsum[2 * Gb];
        }
      }
      if (c < 2) halves[((bi * NSPLIT + hf) * CH + g) * 2 + c] = acc;
    }
  }
  __syncthreads();
  // ---- SwiGLU of complete rows: K halves summed in a fixed order, a written once
  for (int t = threadIdx.x; t < nb * CH; t += blockDim.x) {
    const int bi = t / CH, rw = t - bi * CH;
    const float gs = halves[((bi * NSPLIT) * CH + rw) * 2] + halves[((bi * NSPLIT + 1) * CH + rw) * 2];
    const float us = halves[((bi * NSPLIT) * CH + rw) * 2 + 1] + halves[((bi * NSPLIT + 1) * CH + rw) * 2 + 1];
    const int rr = (b0 + bi) * CH + rw;
    bool host;
    a_out[rr] = src_of<PAGED>(mt[rr / S.I], S, pool, RT, host) ? silu_mul(gs, us) : 0.0f;
  }
}

// ------------------------------------------------------------------------------------------------
template <int BITS, bool PAGED>
__global__ void __maxnreg__(DN_REGS) down_kernel(const uint8_t* __restrict__ pool,
                                                             const float* __restrict__ meta,
                                                             const float* __restrict__ a, MoeShape S,
                                                             uint16_t* __restrict__ out, MoeRoute RT) {
  extern __shared__ __align__(128) uint8_t sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const DnL Ld = dn_layout(S.H, S.I, S.k, S.group, BITS, gridDim.x);
  uint32_t* bd = reinterpret_cast<uint32_t*>(sm + Ld.off_bd);
  float* dsum = reinterpret_cast<float*>(sm + Ld.off_dsum);
  const uint32_t* zero = reinterpret_cast<const uint32_t*>(sm + Ld.off_zero);
  float* part = reinterpret_cast<float*>(sm + Ld.off_part);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Ld.off_bar);
  const int h0 = int(int64_t(S.H) * blockIdx.x / gridDim.x), h1 = int(int64_t(S.H) * (blockIdx.x + 1) / gridDim.x);
  const int nrows = h1 - h0;
  const int64_t ngm = S.ng / 3;
  const int units = Ld.units;
  const int npieces = S.k * DN_SPLIT;  // (expert, K piece)

  // routing: this runs before griddepcontrol.wait, after the producer of the routing inputs has
  // completed (the gate/up grid triggers this launch only after its own wait), so reads go to L2
  const float* mt = meta;
  if (RT.logits) {
    float* rs = reinterpret_cast<float*>(sm + Ld.off_route);
    route_from_logits<true>(RT, S.k, rs, rs + 64, rs + 96);
    mt = rs;
  }
  // ---- the down rows of every routed expert: one bulk copy of the CTA's contiguous rows plus the
  //      scale and min windows, issued before waiting on the gate/up grid (the routing is final)
  if (warp == 0) {
    for (int j = lane; j < S.k; j += 32) {
      mbar_init(&bars[j], 1);
      mbar_fence_init();
      const float f = RT.logits ? mt[j] : __ldcg(meta + j);
      bool host;
      const uint8_t* base = src_of<PAGED>(f, S, pool, RT, host);
      if (!base) flag(WISP_STATUS_BAD_SLOT);
      if (!base || nrows <= 0) {
        mbar_expect_tx(&bars[j], 0);
        continue;
      }
      if (host) continue;  // copied below by the whole CTA, which then arrives on the barrier
      const Win ws = window(S.ncode + 2 * (2 * ngm + int64_t(h0) * Ld.gpr), 2 * int64_t(nrows) * Ld.gpr);
      const Win wm = window(S.ncode + 2 * (S.ng + 2 * ngm + int64_t(h0) * Ld.gpr), 2 * int64_t(nrows) * Ld.gpr);
      const uint32_t cb = uint32_t(int64_t(nrows) * Ld.row_bytes);
      uint8_t* dst = sm + int64_t(j) * Ld.per_expert;
      mbar_expect_tx(&bars[j], cb + ws.bytes + wm.bytes);
      bulk_g2s(dst, base + 2 * S.mat_bytes + int64_t(h0) * Ld.row_bytes, cb, &bars[j]);
      bulk_g2s(dst + 16 * Ld.row_bytes, base + ws.start, ws.bytes, &bars[j]);
      bulk_g2s(dst + 16 * Ld.row_bytes + Ld.sc_win, base + wm.start, wm.bytes, &bars[j]);
    }
  }
  // experts read from the host store (paged calls only): the same mask in every thread, from the routing
  uint32_t hm = 0;
  if (PAGED && RT.host_store && nrows > 0)
    for (int j = 0; j < S.k; ++j) {
      bool host;
      src_of<PAGED>(RT.logits ? mt[j] : __ldcg(meta + j), S, pool, RT, host);
      hm |= host ? (1u << j) : 0u;
    }
  if (hm) {
    // non-resident experts: the same three ranges from the host store, one warp per (expert, range)
    const Win ws = window(S.ncode + 2 * (2 * ngm + int64_t(h0) * Ld.gpr), 2 * int64_t(nrows) * Ld.gpr);
    const Win wm = window(S.ncode + 2 * (S.ng + 2 * ngm + int64_t(h0) * Ld.gpr), 2 * int64_t(nrows) * Ld.gpr);
    for (int task = warp; task < S.k * 3; task += DN_WARPS) {
      const int j = task / 3, part = task - 3 * j;
      if (!((hm >> j) & 1u)) continue;
      bool host;
      const uint8_t* base = src_of<PAGED>(RT.logits ? mt[j] : __ldcg(meta + j), S, pool, RT, host);
      uint8_t* dst = sm + int64_t(j) * Ld.per_expert;
      if (part == 0) warp_copy_g2s(dst, base + 2 * S.mat_bytes + int64_t(h0) * Ld.row_bytes, int64_t(nrows) * Ld.row_bytes, lane);
      else if (part == 1) warp_copy_g2s(dst + 16 * Ld.row_bytes, base + ws.start, ws.bytes, lane);
      else warp_copy_g2s(dst + 16 * Ld.row_bytes + Ld.sc_win, base + wm.start, wm.bytes, lane);
    }
    __syncthreads();
    if (warp == 0 && ((hm >> lane) & 1u)) mbar_expect_tx(&bars[lane], 0);
  }
  for (int i = threadIdx.x; i < DN_WARPS * 16; i += blockDim.x) part[i] = 0.0f;
  if (threadIdx.x < 16) reinterpret_cast<uint32_t*>(sm + Ld.off_zero)[threadIdx.x] = 0u;

  pdl_wait();  // a is written by the gate/up grid

  // ---- B limbs of every routed expert, CTA-wide: one thread per (expert, unit).
  //      Warp-uniform loop (quad shuffles need every lane); tail lanes redo the last unit, store nothing.
  const int ntask = S.k * units;
  for (int tb = int(threadIdx.x) & ~31; tb < ntask; tb += blockDim.x) {
    const int t = tb + lane, tt = min(t, ntask - 1);
    const int j = tt / units, u = tt - j * units;
    float v[32];
    const float4* ap = reinterpret_cast<const float4*>(a + int64_t(j) * S.I + u * 32);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 f = ap[q];
      v[4 * q] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
    }
    const int e = store_b_limbs<BITS>(v, bd + int64_t(t) * 24, t < ntask);
    float sx = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) sx += v[i];
    // the 4 units of a group sit in 4 consecutive lanes (units % 4 == 0 and tb % 32 == 0)
    sx = quad_sum(sx);
    if (t < ntask && (u & 3) == 0) {
      dsum[2 * (j * Ld.groups + (u >> 2))] = sx;
      dsum[2 * (j * Ld.groups + (u >> 2)) + 1] = pow2(-e);
    }
  }
  __syncthreads();
  pdl_launch_dependents();

  for (int piece = warp; piece < npieces; piece += DN_WARPS) {
    const int j = piece / DN_SPLIT, sp = piece % DN_SPLIT;
    bool host;
    const bool ok = src_of<PAGED>(mt[j], S, pool, RT, host) != nullptr;
    const float wj = mt[S.k + j];
    if (!ok || nrows <= 0) continue;
    mbar_wait(&bars[j], 0);
    const uint8_t* eb = sm + int64_t(j) * Ld.per_expert;
    const uint32_t sskip = window(S.ncode + 2 * (2 * ngm + int64_t(h0) * Ld.gpr), 1).skip;
    const uint32_t mskip = window(S.ncode + 2 * (S.ng + 2 * ngm + int64_t(h0) * Ld.gpr), 1).skip;
    const uint16_t* ss = reinterpret_cast<const uint16_t*>(eb + 16 * Ld.row_bytes + sskip);
    const uint16_t* smn = reinterpret_cast<const uint16_t*>(eb + 16 * Ld.row_bytes + Ld.sc_win + mskip);
    // lane c = 0 finishes output row g, lane c = 1 row g + 8
    const int myrow = (c == 1) ? g + 8 : g;
    const uint16_t* srow = ss + myrow * Ld.gpr;
    const uint16_t* mrow = smn + myrow * Ld.gpr;
    const int G0 = sp * Ld.groups_per_piece;
    const int ng = min(Ld.groups_per_piece, Ld.groups - G0);
    float acc = 0.0f;
    const uint32_t* bj = bd + int64_t(j) * units * 24;
    const float* ds = dsum + 2 * int64_t(j) * Ld.groups;
    // groups in pairs (two independent MMA chains); an odd last group runs alone
    for (int G = 0; G < ng; G += 2) {
      const bool two = G + 1 < ng;  // warp-uniform
      uint32_t wa0[BITS], wb0[BITS], wa1[BITS], wb1[BITS], bb0[8], bb1[8];
      int d0[4], d1[4];
      lds_unit<BITS>(eb + g * Ld.row_bytes + (4 * (G0 + G) + c) * 4 * BITS, wa0);
      lds_unit<BITS>(eb + (g + 8) * Ld.row_bytes + (4 * (G0 + G) + c) * 4 * BITS, wb0);
      lds_b8(g < 3 ? bj + ((4 * (G0 + G) + c) * 3 + g) * 8 : zero, bb0);
      if (two) {
        lds_unit<BITS>(eb + g * Ld.row_bytes + (4 * (G0 + G + 1) + c) * 4 * BITS, wa1);
        lds_unit<BITS>(eb + (g + 8) * Ld.row_bytes + (4 * (G0 + G + 1) + c) * 4 * BITS, wb1);
        lds_b8(g < 3 ? bj + ((4 * (G0 + G + 1) + c) * 3 + g) * 8 : zero, bb1);
      }
      imma_group<BITS>(wa0, wb0, bb0, d0);
      if (two) imma_group<BITS>(wa1, wb1, bb1, d1);
      const float D0 = quad_row_dot(d0, c);
      {
        const int qg = (G0 + G) >> S.gshift;
        acc += f16_bits_to_f32(srow[qg]) * (D0 * ds[2 * (G0 + G) + 1]) + f16_bits_to_f32(mrow[qg]) * ds[2 * (G0 + G)];
      }
      if (two) {
        const float D1 = quad_row_dot(d1, c);
        const int qg = (G0 + G + 1) >> S.gshift;
        acc += f16_bits_to_f32(srow[qg]) * (D1 * ds[2 * (G0 + G + 1) + 1]) + f16_bits_to_f32(mrow[qg]) * ds[2 * (G0 + G + 1)];
      }
    }
    if (c < 2 && myrow < nrows) part[warp * 16 + myrow] += wj * acc;
  }
  __syncthreads();
  for (int r = threadIdx.x; r < nrows; r += blockDim.x) {
    float s = 0.0f;
    for (int w = 0; w < DN_WARPS; ++w) s += part[w * 16 + r];
    out[h0 + r] = f32_to_bf16(s);
  }
  // no copy may still be landing in shared memory when the CTA retires
  if (warp == 0)
    for (int j = lane; j < S.k; j += 32) mbar_wait(&bars[j], 0);
}

}  // namespace v4
}  // namespace wisp
