// Fused MoE decode for one token, tensor-core unpack form (variant 3).
//
// Same data movement as variant 2 (persistent CTAs, cp.async.bulk of each CTA's rows into shared
// memory, PDL-chained gate/up -> down), but the multiply-accumulate runs on warp-level MMA
// (mma.sync m16n8k16, bf16 x bf16 -> fp32) fed by the one-LOP3-per-pair unpack of unpack_mma.cuh.
// The SMs spend < 1 integer op per weight code; the HBM stream sets the pace.
//
//   gate/up: a warp's MMA row block is 8 gate rows (A rows 0-7) + the same 8 up rows (A rows 8-15),
//            so lane (g, 0) ends each quantization group holding gate row g in d[0] and up row g in d[2];
//            B column 0 is the permuted, scaled x (columns 1-7 zero).
//   down:    a warp's row block is 16 output rows of one expert; B column 0 / 1 hold the bf16 hi / lo
//            split of a_j (so fp32 a_j is carried to ~16 mantissa bits), read as d[0] + d[1].
// Per quantization group:  sum_e (q_e s + m) v_e = s (D - 128 SB) + m SX, with D the MMA result,
// SB the sum of the B values and SX the sum of v over the group.
//
// Rows land in shared memory at stride row_bytes + 16*BITS (one bulk copy per row, issued by the 32
// lanes of warp 0), which makes the per-lane unit loads bank-conflict free.
#pragma once
#include "common.cuh"
#include "moe_decode.cuh"
#include "moe_decode_v2.cuh"
#include "unpack_mma.cuh"

namespace wisp {
namespace v3 {

using v2::bulk_g2s;
using v2::mbar_expect_tx;
using v2::mbar_fence_init;
using v2::mbar_init;
using v2::mbar_wait;
using v2::min64;
using v2::pdl_launch_dependents;
using v2::pdl_wait;
using v2::rd16;
using v2::ru16;
using v2::window;
using v2::Win;

constexpr int GU_WARPS = 16;
constexpr int DN_WARPS = 8;
constexpr int GU_THREADS = GU_WARPS * 32;
constexpr int DN_THREADS = DN_WARPS * 32;
constexpr int CH = 8;      // rows per gate/up chunk = MMA half block
constexpr int NSPLIT = 2;  // gate/up K split per chunk (pieces = chunks x NSPLIT)

__host__ __device__ constexpr int row_pad(int bits) { return 16 * bits; }

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
struct GuL {
  int64_t row_bytes, stride, sc_win, chunk;
  int gpr, max_rows, max_chunks;
  int64_t off_bx, off_sb, off_sx, off_part, off_bar, bytes;
};

__host__ __device__ inline GuL gu_layout(int H, int I, int k, int group, int bits, int nctas) {
  GuL L;
  L.row_bytes = int64_t(H) * bits / 8;
  L.stride = L.row_bytes + row_pad(bits);
  L.gpr = H / group;
  L.sc_win = ru16(int64_t(CH) * L.gpr * 2) + 16;
  L.chunk = 2 * CH * L.stride + 4 * L.sc_win;
  const int64_t R = int64_t(k) * I;
  L.max_rows = int((R + nctas - 1) / nctas);
  L.max_chunks = (L.max_rows + CH - 1) / CH + 1;
  const int ngroups = H / 128 > 0 ? H / 128 : 1;  // B pairs are kept per 128-wide MMA group (4 units)
  L.off_bx = int64_t(L.max_chunks) * L.chunk;                 // [H/128][4 units][16] u32
  L.off_sb = L.off_bx + int64_t(ngroups) * 4 * 16 * 4;         // [H/32] f32 (per unit)
  L.off_sx = L.off_sb + int64_t(H / 32) * 4;                   // [H/32] f32
  L.off_part = L.off_sx + int64_t(H / 32) * 4;                 // [max_chunks][NSPLIT][CH][2] f32
  L.off_bar = ru16(L.off_part + int64_t(L.max_chunks) * NSPLIT * CH * 2 * 4);
  L.bytes = L.off_bar + 8 * L.max_chunks;
  return L;
}

struct DnL {
  int64_t row_bytes, stride, sc_win, per_expert;
  int gpr, max_rows, rows_alloc;
  int64_t off_bd, off_sb, off_sx, off_part, off_bar, bytes;
};

__host__ __device__ inline DnL dn_layout(int H, int I, int k, int group, int bits, int nctas) {
  DnL L;
  L.row_bytes = int64_t(I) * bits / 8;
  L.stride = L.row_bytes + row_pad(bits);
  L.gpr = I / group;
  L.max_rows = (H + nctas - 1) / nctas;
  L.rows_alloc = (L.max_rows + 15) / 16 * 16;
  L.sc_win = ru16(int64_t(L.max_rows) * L.gpr * 2) + 16;
  L.per_expert = int64_t(L.rows_alloc) * L.stride + 2 * L.sc_win;
  const int units = I / 32;
  L.off_bd = int64_t(k) * L.per_expert;                    // [k][I/32 units][2 parts][16] u32
  L.off_sb = L.off_bd + int64_t(k) * units * 2 * 16 * 4;    // [k][I/32] f32
  L.off_sx = L.off_sb + int64_t(k) * units * 4;             // [k][I/32] f32
  L.off_part = L.off_sx + int64_t(k) * units * 4;           // [DN_WARPS][rows_alloc] f32
  L.off_bar = ru16(L.off_part + int64_t(DN_WARPS) * L.rows_alloc * 4);
  L.bytes = L.off_bar + 8 * k;
  return L;
}

// Chunks of a gate/up CTA range [r_begin, r_end) of the k*I (expert, row) list: since I is a multiple
// of CH, cutting at multiples of CH also cuts at every expert boundary, so chunk ci is closed-form.
struct Chunk {
  int lo, cnt, j, row0;  // first list index, rows, expert, first row in the expert
};
__device__ __forceinline__ int chunk_count(int r_begin, int r_end) {
  return r_end > r_begin ? (r_end - 1) / CH - r_begin / CH + 1 : 0;
}
__device__ __forceinline__ Chunk chunk_at(int r_begin, int r_end, int I, int ci) {
  Chunk c;
  const int base = (r_begin / CH + ci) * CH;
  c.lo = max(r_begin, base);
  c.cnt = min(r_end, base + CH) - c.lo;
  c.j = c.lo / I;
  c.row0 = c.lo - c.j * I;
  return c;
}

// ------------------------------------------------------------------------------------------------
template <int BITS>
__global__ void __maxnreg__(72) gate_up_kernel(const uint8_t* __restrict__ pool, const float* __restrict__ meta,
                                               const uint16_t* __restrict__ x, MoeShape S, float* __restrict__ a_out) {
  extern __shared__ __align__(128) uint8_t sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const GuL Lg = gu_layout(S.H, S.I, S.k, S.group, BITS, gridDim.x);
  uint32_t* bx = reinterpret_cast<uint32_t*>(sm + Lg.off_bx);
  float* sbu = reinterpret_cast<float*>(sm + Lg.off_sb);
  float* sxu = reinterpret_cast<float*>(sm + Lg.off_sx);
  float* part = reinterpret_cast<float*>(sm + Lg.off_part);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Lg.off_bar);
  const int R = S.k * S.I;
  const int r_begin = int(int64_t(R) * blockIdx.x / gridDim.x), r_end = int(int64_t(R) * (blockIdx.x + 1) / gridDim.x);
  const int64_t ngm = S.ng / 3;
  const int gpr = Lg.gpr;
  const int nchunks = chunk_count(r_begin, r_end);

  pdl_wait();  // routing and x come from earlier kernels in the stream

  // ---- copies: lane 0 arms the barriers, then warp 0's lanes issue one bulk copy per row / window
  if (warp == 0) {
    if (lane == 0) {
      for (int ci = 0; ci < Lg.max_chunks; ++ci) mbar_init(&bars[ci], 1);
      mbar_fence_init();
    }
    __syncwarp();
    // lane ci arms chunk ci (the copies of a chunk are issued only after its expect_tx below)
    for (int ci = lane; ci < nchunks; ci += 32) {
      const Chunk ch = chunk_at(r_begin, r_end, S.I, ci);
      int64_t slot;
      if (!route_slot(meta, ch.j, S, slot)) {
        flag(WISP_STATUS_BAD_SLOT);
        mbar_expect_tx(&bars[ci], 0);
        continue;
      }
      const int64_t row = ch.row0, cnt = ch.cnt;
      uint32_t tx = uint32_t(2 * cnt * Lg.row_bytes);
      tx += window(S.ncode + 2 * (row * gpr), 2 * cnt * gpr).bytes;
      tx += window(S.ncode + 2 * (S.ng + row * gpr), 2 * cnt * gpr).bytes;
      tx += window(S.ncode + 2 * (ngm + row * gpr), 2 * cnt * gpr).bytes;
      tx += window(S.ncode + 2 * (S.ng + ngm + row * gpr), 2 * cnt * gpr).bytes;
      mbar_expect_tx(&bars[ci], tx);
    }
    __syncwarp();
    // op list: per chunk 2*CH row slots (gate rows then up rows) + 4 windows; lane l takes ops l, l+32, ...
    const int per_chunk = 2 * CH + 4;
    for (int op = lane; op < nchunks * per_chunk; op += 32) {
      const int ci = op / per_chunk, o = op - ci * per_chunk;
      const Chunk ch = chunk_at(r_begin, r_end, S.I, ci);
      int64_t slot;
      if (!route_slot(meta, ch.j, S, slot)) continue;
      const uint8_t* base = pool + slot * S.nbytes;
      uint8_t* dst = sm + int64_t(ci) * Lg.chunk;
      if (o < 2 * CH) {
        const int m = o / CH, rr = o - m * CH;  // matrix (0 gate, 1 up), row in chunk
        if (rr < ch.cnt)
          bulk_g2s(dst + (m * CH + rr) * Lg.stride, base + m * S.mat_bytes + int64_t(ch.row0 + rr) * Lg.row_bytes,
                   uint32_t(Lg.row_bytes), &bars[ci]);
      } else {
        const int wsel = o - 2 * CH;  // 0 gate scale, 1 gate min, 2 up scale, 3 up min
        const int64_t off = S.ncode + 2 * ((wsel & 1) * S.ng + (wsel >> 1) * ngm + int64_t(ch.row0) * gpr);
        const Win w = window(off, 2 * int64_t(ch.cnt) * gpr);
        bulk_g2s(dst + 2 * CH * Lg.stride + wsel * Lg.sc_win, base + w.start, w.bytes, &bars[ci]);
      }
    }
  }

  // ---- B operand from x: one thread per 32-element unit (natural order -> pair order, scaled)
  const int units = S.H / 32;
  for (int u = threadIdx.x; u < units; u += blockDim.x) {
    float v[32];
    const uint4* xp = reinterpret_cast<const uint4*>(x + u * 32);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 t = xp[q];
      const uint32_t wd[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        v[8 * q + 2 * h] = __uint_as_float(wd[h] << 16);
        v[8 * q + 2 * h + 1] = __uint_as_float(wd[h] & 0xFFFF0000u);
      }
    }
    uint32_t b[16];
    float bs;
    build_b_pairs<BITS>(v, 0, b, bs);
    uint4* dstb = reinterpret_cast<uint4*>(bx + u * 16);
#pragma unroll
    for (int q = 0; q < 4; ++q) dstb[q] = make_uint4(b[4 * q], b[4 * q + 1], b[4 * q + 2], b[4 * q + 3]);
    float sx = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) sx += v[i];
    sbu[u] = bs;
    sxu[u] = sx;
  }
  __syncthreads();
  pdl_launch_dependents();  // the down grid may start its weight copies now

  // ---- pieces: (chunk, K half); 8 gate + 8 up rows per MMA block
  const int groups = S.H / 128;  // MMA groups of 128 k (4 units)
  const int per_split = (groups + NSPLIT - 1) / NSPLIT;
  for (int piece = warp; piece < nchunks * NSPLIT; piece += GU_WARPS) {
    const int ci = piece / NSPLIT, sp = piece - ci * NSPLIT;
    const Chunk ch = chunk_at(r_begin, r_end, S.I, ci);
    const int j = ch.j;
    const int64_t row0 = ch.row0;
    int64_t slot;
    const bool ok = route_slot(meta, j, S, slot);
    float accg = 0.0f, accu = 0.0f;
    if (ok) {
      mbar_wait(&bars[ci]);
      const uint8_t* cb = sm + int64_t(ci) * Lg.chunk;
      const uint8_t* rowg = cb + g * Lg.stride;
      const uint8_t* rowu = cb + (CH + g) * Lg.stride;
      const uint8_t* sw = cb + 2 * CH * Lg.stride;
      const uint16_t* ssg = reinterpret_cast<const uint16_t*>(sw + ((S.ncode + 2 * (row0 * gpr)) & 15)) + g * gpr;
      const uint16_t* smg =
          reinterpret_cast<const uint16_t*>(sw + Lg.sc_win + ((S.ncode + 2 * (S.ng + row0 * gpr)) & 15)) + g * gpr;
      const uint16_t* ssu =
          reinterpret_cast<const uint16_t*>(sw + 2 * Lg.sc_win + ((S.ncode + 2 * (ngm + row0 * gpr)) & 15)) + g * gpr;
      const uint16_t* smu =
          reinterpret_cast<const uint16_t*>(sw + 3 * Lg.sc_win + ((S.ncode + 2 * (S.ng + ngm + row0 * gpr)) & 15)) +
          g * gpr;
      const int G0 = sp * per_split, G1 = min(groups, G0 + per_split);
      for (int G = G0; G < G1; ++G) {
        const int u = 4 * G + c;  // this lane's unit in the row
        uint32_t wg[BITS], wu[BITS];
        lds_unit<BITS>(rowg + u * 4 * BITS, wg);
        lds_unit<BITS>(rowu + u * 4 * BITS, wu);
        uint32_t b[16];
        if (g == 0) {
          const uint4* bp = reinterpret_cast<const uint4*>(bx + u * 16);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 t = bp[q];
            b[4 * q] = t.x; b[4 * q + 1] = t.y; b[4 * q + 2] = t.z; b[4 * q + 3] = t.w;
          }
        } else {
#pragma unroll
          for (int q = 0; q < 16; ++q) b[q] = 0u;
        }
        uint32_t ag[16], au[16];
        unpack_pairs<BITS>(wg, ag);
        unpack_pairs<BITS>(wu, au);
        float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int m = 0; m < 8; ++m) mma_bf16(d, ag[2 * m], au[2 * m], ag[2 * m + 1], au[2 * m + 1], b[2 * m], b[2 * m + 1]);
        if (c == 0) {
          // the group's sums over its 4 units (fixed order)
          const float sb = (sbu[4 * G] + sbu[4 * G + 1]) + (sbu[4 * G + 2] + sbu[4 * G + 3]);
          const float sx = (sxu[4 * G] + sxu[4 * G + 1]) + (sxu[4 * G + 2] + sxu[4 * G + 3]);
          // quantization group index of this 128-wide MMA group: groups are >= 128 wide or equal
          const int qg = (G * 128) / S.group;
          const float s_g = f16_bits_to_f32(ssg[qg]), m_g = f16_bits_to_f32(smg[qg]);
          const float s_u = f16_bits_to_f32(ssu[qg]), m_u = f16_bits_to_f32(smu[qg]);
          accg += s_g * (d[0] - 128.0f * sb) + m_g * sx;
          accu += s_u * (d[2] - 128.0f * sb) + m_u * sx;
        }
      }
    }
    if (c == 0) {
      part[((ci * NSPLIT + sp) * CH + g) * 2] = accg;
      part[((ci * NSPLIT + sp) * CH + g) * 2 + 1] = accu;
    }
  }
  __syncthreads();
  // ---- SwiGLU of the complete rows, written once
  for (int rr = threadIdx.x; rr < r_end - r_begin; rr += blockDim.x) {
    const int r = r_begin + rr;
    const int ci = r / CH - r_begin / CH;
    const int in_chunk = r - max(r_begin, (r / CH) * CH);
    float gs = 0.0f, us = 0.0f;
    for (int sp = 0; sp < NSPLIT; ++sp) {
      gs += part[((ci * NSPLIT + sp) * CH + in_chunk) * 2];
      us += part[((ci * NSPLIT + sp) * CH + in_chunk) * 2 + 1];
    }
    int64_t slot;
    a_out[r] = route_slot(meta, r / S.I, S, slot) ? silu_mul(gs, us) : 0.0f;
  }
  if (threadIdx.x == 0)
    for (int ci = 0; ci < nchunks; ++ci) mbar_wait(&bars[ci]);
}

// ------------------------------------------------------------------------------------------------
template <int BITS>
__global__ void __maxnreg__(80) down_kernel(const uint8_t* __restrict__ pool, const float* __restrict__ meta,
                                            const float* __restrict__ a, MoeShape S, uint16_t* __restrict__ out) {
  extern __shared__ __align__(128) uint8_t sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const DnL Ld = dn_layout(S.H, S.I, S.k, S.group, BITS, gridDim.x);
  uint32_t* bd = reinterpret_cast<uint32_t*>(sm + Ld.off_bd);
  float* sbu = reinterpret_cast<float*>(sm + Ld.off_sb);
  float* sxu = reinterpret_cast<float*>(sm + Ld.off_sx);
  float* part = reinterpret_cast<float*>(sm + Ld.off_part);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Ld.off_bar);
  const int h0 = int(int64_t(S.H) * blockIdx.x / gridDim.x), h1 = int(int64_t(S.H) * (blockIdx.x + 1) / gridDim.x);
  const int nrows = h1 - h0;
  const int gpr = Ld.gpr;
  const int64_t ngm = S.ng / 3;
  const int units = S.I / 32;

  // ---- copies of the down rows of every routed expert: issued before waiting on the gate/up grid
  if (warp == 0) {
    if (lane == 0) {
      for (int j = 0; j < S.k; ++j) mbar_init(&bars[j], 1);
      mbar_fence_init();
      for (int j = 0; j < S.k; ++j) {
        int64_t slot;
        if (nrows <= 0 || !route_slot(meta, j, S, slot)) {
          mbar_expect_tx(&bars[j], 0);
          continue;
        }
        uint32_t tx = uint32_t(int64_t(nrows) * Ld.row_bytes);
        tx += window(S.ncode + 2 * (2 * ngm + int64_t(h0) * gpr), 2 * int64_t(nrows) * gpr).bytes;
        tx += window(S.ncode + 2 * (S.ng + 2 * ngm + int64_t(h0) * gpr), 2 * int64_t(nrows) * gpr).bytes;
        mbar_expect_tx(&bars[j], tx);
      }
    }
    __syncwarp();
    int op = 0;
    for (int j = 0; j < S.k; ++j) {
      int64_t slot;
      if (nrows <= 0 || !route_slot(meta, j, S, slot)) continue;
      const uint8_t* base = pool + slot * S.nbytes;
      uint8_t* dst = sm + int64_t(j) * Ld.per_expert;
      for (int o = 0; o < nrows + 2; ++o, ++op) {
        if ((op & 31) != lane) continue;
        if (o < nrows) {
          bulk_g2s(dst + o * Ld.stride, base + 2 * S.mat_bytes + int64_t(h0 + o) * Ld.row_bytes, uint32_t(Ld.row_bytes),
                   &bars[j]);
        } else {
          const int wsel = o - nrows;  // 0 scales, 1 mins
          const Win w = window(S.ncode + 2 * (wsel * S.ng + 2 * ngm + int64_t(h0) * gpr), 2 * int64_t(nrows) * gpr);
          bulk_g2s(dst + int64_t(Ld.rows_alloc) * Ld.stride + wsel * Ld.sc_win, base + w.start, w.bytes, &bars[j]);
        }
      }
    }
  }
  for (int i = threadIdx.x; i < DN_WARPS * Ld.rows_alloc; i += blockDim.x) part[i] = 0.0f;

  pdl_wait();  // a is written by the gate/up grid

  // ---- B operand from a: per (expert, unit), bf16 hi part and lo part
  for (int t = threadIdx.x; t < S.k * units; t += blockDim.x) {
    const int j = t / units, u = t - j * units;
    float v[32];
    const float4* ap = reinterpret_cast<const float4*>(a + int64_t(j) * S.I + u * 32);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 f = ap[q];
      v[4 * q] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
    }
    uint32_t b[16];
    float bs0, bs1;
    uint4* dstb = reinterpret_cast<uint4*>(bd + (int64_t(t) * 2) * 16);
    build_b_pairs<BITS>(v, 0, b, bs0);
#pragma unroll
    for (int q = 0; q < 4; ++q) dstb[q] = make_uint4(b[4 * q], b[4 * q + 1], b[4 * q + 2], b[4 * q + 3]);
    build_b_pairs<BITS>(v, 1, b, bs1);
#pragma unroll
    for (int q = 0; q < 4; ++q) dstb[4 + q] = make_uint4(b[4 * q], b[4 * q + 1], b[4 * q + 2], b[4 * q + 3]);
    float sx = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) sx += v[i];
    sbu[t] = bs0 + bs1;
    sxu[t] = sx;
  }
  __syncthreads();

  // ---- pieces: (expert, 16-row block)
  const int nrb = (nrows + 15) / 16;
  const int groups = S.I / 128;
  for (int piece = warp; piece < S.k * nrb; piece += DN_WARPS) {
    const int j = piece / nrb, rb = piece - j * nrb;
    int64_t slot;
    if (!route_slot(meta, j, S, slot)) continue;
    const float wj = meta[S.k + j];
    mbar_wait(&bars[j]);
    const uint8_t* blk = sm + int64_t(j) * Ld.per_expert;
    const int r_a = rb * 16 + g, r_b = r_a + 8;
    const uint8_t* ra = blk + int64_t(r_a) * Ld.stride;
    const uint8_t* rbp = blk + int64_t(r_b) * Ld.stride;
    const uint8_t* sw = blk + int64_t(Ld.rows_alloc) * Ld.stride;
    const uint16_t* ss = reinterpret_cast<const uint16_t*>(sw + ((S.ncode + 2 * (2 * ngm + int64_t(h0) * gpr)) & 15));
    const uint16_t* smn =
        reinterpret_cast<const uint16_t*>(sw + Ld.sc_win + ((S.ncode + 2 * (S.ng + 2 * ngm + int64_t(h0) * gpr)) & 15));
    float acc_a = 0.0f, acc_b = 0.0f;
    for (int G = 0; G < groups; ++G) {
      const int u = 4 * G + c;
      uint32_t wa[BITS], wb[BITS];
      lds_unit<BITS>(ra + u * 4 * BITS, wa);
      lds_unit<BITS>(rbp + u * 4 * BITS, wb);
      uint32_t b[16];
      if (g < 2) {
        const uint4* bp = reinterpret_cast<const uint4*>(bd + ((int64_t(j) * units + u) * 2 + g) * 16);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 t = bp[q];
          b[4 * q] = t.x; b[4 * q + 1] = t.y; b[4 * q + 2] = t.z; b[4 * q + 3] = t.w;
        }
      } else {
#pragma unroll
        for (int q = 0; q < 16; ++q) b[q] = 0u;
      }
      uint32_t a_lo[16], a_hi[16];
      unpack_pairs<BITS>(wa, a_lo);
      unpack_pairs<BITS>(wb, a_hi);
      float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int m = 0; m < 8; ++m) mma_bf16(d, a_lo[2 * m], a_hi[2 * m], a_lo[2 * m + 1], a_hi[2 * m + 1], b[2 * m], b[2 * m + 1]);
      if (c == 0) {
        const int64_t ub = int64_t(j) * units + 4 * G;
        const float sb = (sbu[ub] + sbu[ub + 1]) + (sbu[ub + 2] + sbu[ub + 3]);
        const float sx = (sxu[ub] + sxu[ub + 1]) + (sxu[ub + 2] + sxu[ub + 3]);
        const int qg = (G * 128) / S.group;
        if (r_a < nrows) {
          const float s = f16_bits_to_f32(ss[r_a * gpr + qg]), m = f16_bits_to_f32(smn[r_a * gpr + qg]);
          acc_a += s * ((d[0] + d[1]) - 128.0f * sb) + m * sx;
        }
        if (r_b < nrows) {
          const float s = f16_bits_to_f32(ss[r_b * gpr + qg]), m = f16_bits_to_f32(smn[r_b * gpr + qg]);
          acc_b += s * ((d[2] + d[3]) - 128.0f * sb) + m * sx;
        }
      }
    }
    if (c == 0) {
      if (r_a < nrows) part[warp * Ld.rows_alloc + r_a] += wj * acc_a;
      if (r_b < nrows) part[warp * Ld.rows_alloc + r_b] += wj * acc_b;
    }
  }
  __syncthreads();
  for (int r = threadIdx.x; r < nrows; r += blockDim.x) {
    float s = 0.0f;
    for (int w = 0; w < DN_WARPS; ++w) s += part[w * Ld.rows_alloc + r];
    out[h0 + r] = f32_to_bf16(s);
  }
  if (threadIdx.x == 0)
    for (int j = 0; j < S.k; ++j) mbar_wait(&bars[j]);
}

}  // namespace v3
}  // namespace wisp
