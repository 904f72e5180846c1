// gpt-oss experts (gpt-oss-20b: H = I = 2880, 32 experts, top-4; the reference's PagedGptOssBlock,
// wisp/gptoss.py:107-143).
//
// An expert is gate_up [H, 2I] (gate and up interleaved along the output axis) and down [I, H], both
// stored input-major, plus biases, packed as the flat [gate_up | down] code stream of the wisp.quant
// layout (wisp/gptoss.py:35-40), so quantization groups run along the OUTPUT axis.  Each output
// column is then a strided column of the stored matrix, and the kernels are column-parallel: lane l
// owns 8 consecutive output columns (one 8-code word, coalesced across the warp), streams the rows
// of its K range, and dequantizes each word bit-exactly (bf16(q*s + m)).  K is split over warps; the
// split partials are summed in a fixed order.  Pairs (token, choice) are grouped by slot as in the
// batched kernels, so an expert's weights are read once for all of its tokens.
//
//   gemv_kernel<MAT 0>  per (group, 256-column tile of 2I, K split): partial x . W_gu
//   act_kernel    gu = bf16(sum + bias); a = bf16((clamp(up) + 1) * g * sigmoid(1.702 g)), g = clamp(gate)
//   gemv_kernel<MAT 1>  per (group, 256-column tile of H, K split): partial a . W_d
//   combine       out[t] = bf16(sum_j w[t,j] * (bf16(sum) + bias_d[e]))
#pragma once
#include <cuda.h>

#include "common.cuh"
#include "moe_batched.cuh"

namespace wisp {
namespace gptoss {

constexpr int WARPS = 8;
constexpr int THREADS = WARPS * 32;
constexpr int NTOK = 8;          // tokens of a group per pass
constexpr float ALPHA = 1.702f;
constexpr float LIMIT = 7.0f;

struct Ws {
  batched::Ws g;       // grouping (n_groups, groups, order, posof)
  float* part;         // [S][P][max(2I, H)] split partials
  uint16_t* act;       // [P][I] bf16
};

__host__ __device__ inline int64_t ws_bytes(int P, int S, int64_t H, int64_t I) {
  const int64_t w = (2 * I > H ? 2 * I : H);
  const int64_t head = batched::ws_bytes(P, 0, 0);  // the grouping ints
  return head + (int64_t(S) * P * w * 4 + 255) / 256 * 256 + int64_t(P) * I * 2;
}

__host__ __device__ inline Ws ws_carve(void* base, int P, int S, int64_t H, int64_t I) {
  Ws w;
  w.g = batched::ws_carve(base, P, 0);
  const int64_t wd = (2 * I > H ? 2 * I : H);
  uint8_t* b = static_cast<uint8_t*>(base) + batched::ws_bytes(P, 0, 0);
  w.part = reinterpret_cast<float*>(b);
  w.act = reinterpret_cast<uint16_t*>(b + (int64_t(S) * P * wd * 4 + 255) / 256 * 256);
  return w;
}

// the packed bytes of 8 codes starting at element e (e % 8 == 0) of the code stream
template <int BITS>
struct Word8 {
  uint32_t v[BITS == 8 ? 2 : 1];
};

template <int BITS>
__device__ __forceinline__ Word8<BITS> load_word8(const uint8_t* codes, int64_t e) {
  const uint8_t* p = codes + e * BITS / 8;
  Word8<BITS> w;
  if constexpr (BITS == 4) {
    w.v[0] = __ldg(reinterpret_cast<const uint32_t*>(p));
  } else if constexpr (BITS == 2) {
    w.v[0] = __ldg(reinterpret_cast<const uint16_t*>(p));
  } else if constexpr (BITS == 3) {
    w.v[0] = uint32_t(__ldg(p)) | (uint32_t(__ldg(p + 1)) << 8) | (uint32_t(__ldg(p + 2)) << 16);
  } else {
    const uint2 t = __ldg(reinterpret_cast<const uint2*>(p));
    w.v[0] = t.x;
    w.v[1] = t.y;
  }
  return w;
}

template <int BITS>
__device__ __forceinline__ uint32_t word8_code(const Word8<BITS>& w, int i) {
  if constexpr (BITS == 8) return (w.v[i >> 2] >> (8 * (i & 3))) & 255u;
  else return (w.v[0] >> (BITS * i)) & ((1u << BITS) - 1u);
}

// Partial products of one (group, column tile, K split) unit for tokens [t0, t0 + NT) of the group:
// part[sp][pos][j0 + c] = sum over rows r in [r0, r1) of bf16(q*s+m)(row r, column j0 + c) * in[t][r]
// (matrix base element e0, row pitch `pitch` elements).  The loads of RIF rows are issued together so
// that each lane keeps that many in flight.
template <int BITS, int MAT, int NT>
__device__ __forceinline__ void column_dot(const uint8_t* base, const MoeShape& S, int64_t e0, int64_t pitch, int64_t j0,
                                           int r0, int r1, const uint16_t* x, const Ws& W, int pos0, float* dst0,
                                           int64_t dst_pitch, int nt) {
  constexpr int RIF = NT >= 8 ? 4 : (NT >= 4 ? 8 : 16);
  const uint16_t* sc = reinterpret_cast<const uint16_t*>(base + S.ncode);
  const uint16_t* in[NT];  // input rows of the tokens (t >= nt repeats the first)
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const int pos = pos0 + (t < nt ? t : 0);
    in[t] = MAT == 0 ? x + int64_t(W.g.order[pos] / S.k) * S.H : W.act + int64_t(pos) * S.I;
  }
  float acc[8][NT] = {};
  for (int rb = r0; rb < r1; rb += RIF) {
    Word8<BITS> w[RIF];
    uint16_t sb[RIF], mb[RIF];
#pragma unroll
    for (int i = 0; i < RIF; ++i) {
      const int r = rb + i < r1 ? rb + i : r1 - 1;  // the tail repeats the last row and adds nothing
      const int64_t e = e0 + int64_t(r) * pitch + j0;
      w[i] = load_word8<BITS>(base, e);
      const int64_t gi = e / S.group;
      sb[i] = ld_nc_u16(sc + gi);
      mb[i] = ld_nc_u16(sc + S.ng + gi);
    }
#pragma unroll
    for (int i = 0; i < RIF; ++i) {
      if (rb + i >= r1) break;
      const float s = f16_bits_to_f32(sb[i]), m = f16_bits_to_f32(mb[i]);
      float xv[NT];
#pragma unroll
      for (int t = 0; t < NT; ++t) xv[t] = bf16_to_f32(in[t][rb + i]);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float wv = bf16_to_f32(f32_to_bf16(__fadd_rn(__fmul_rn(small_u2f(word8_code<BITS>(w[i], c)), s), m)));
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[c][t] = fmaf(wv, xv[t], acc[c][t]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    if (t < nt) {
      float* dst = dst0 + int64_t(t) * dst_pitch;
      reinterpret_cast<float4*>(dst)[0] = make_float4(acc[0][t], acc[1][t], acc[2][t], acc[3][t]);
      reinterpret_cast<float4*>(dst)[1] = make_float4(acc[4][t], acc[5][t], acc[6][t], acc[7][t]);
    }
  }
}

// one kernel for both products: MAT 0 = gate_up (K = H rows, 2I columns, input x rows of tokens),
// MAT 1 = down (K = I rows, H columns, input the activations a of the pairs)
template <int BITS, int MAT>
__global__ void __launch_bounds__(THREADS, 2) gemv_kernel(const uint8_t* __restrict__ pool, MoeShape S, int P, int nsplit,
                                                          const uint16_t* __restrict__ x, Ws W) {
  const int lane = threadIdx.x & 31;
  pdl_wait();
  pdl_launch_dependents();
  const int ngr = W.g.n_groups[0];
  const int64_t ncol = MAT == 0 ? 2 * int64_t(S.I) : S.H;
  const int K = MAT == 0 ? S.H : S.I;
  const int64_t e0 = MAT == 0 ? 0 : 2 * int64_t(S.H) * S.I;
  const int tiles = int((ncol + 255) / 256);
  const int64_t wd = (2 * int64_t(S.I) > S.H ? 2 * int64_t(S.I) : S.H);
  const int64_t nunits = int64_t(ngr) * tiles * nsplit;
  const int gw = blockIdx.x * WARPS + (threadIdx.x >> 5), nw = gridDim.x * WARPS;
  for (int64_t u = gw; u < nunits; u += nw) {
    const int sp = int(u % nsplit);
    const int64_t rest = u / nsplit;
    const int tile = int(rest % tiles), grp = int(rest / tiles);
    const uint8_t* base = pool + int64_t(W.g.grp_slot[grp]) * S.nbytes;
    const int start = W.g.grp_start[grp], cnt = W.g.grp_count[grp];
    const int r0 = int(int64_t(K) * sp / nsplit), r1 = int(int64_t(K) * (sp + 1) / nsplit);
    const int64_t j0 = int64_t(tile) * 256 + 8 * lane;
    if (j0 >= ncol || r1 <= r0) continue;  // lanes past the last column (lane-divergent; no shuffles below)
    for (int t0 = 0; t0 < cnt; t0 += NTOK) {
      const int nt = cnt - t0 < NTOK ? cnt - t0 : NTOK;
      float* dst0 = W.part + (int64_t(sp) * P + start + t0) * wd + j0;
      // the token count picks the unrolled width
      if (nt == 1) column_dot<BITS, MAT, 1>(base, S, e0, ncol, j0, r0, r1, x, W, start + t0, dst0, wd, nt);
      else if (nt == 2) column_dot<BITS, MAT, 2>(base, S, e0, ncol, j0, r0, r1, x, W, start + t0, dst0, wd, nt);
      else if (nt <= 4) column_dot<BITS, MAT, 4>(base, S, e0, ncol, j0, r0, r1, x, W, start + t0, dst0, wd, nt);
      else column_dot<BITS, MAT, NTOK>(base, S, e0, ncol, j0, r0, r1, x, W, start + t0, dst0, wd, nt);
    }
  }
}

// The split partials are summed by SG thread groups (group g takes splits g, g + SG, ..., all loads
// independent) and the groups' sums meet in a fixed tree through shared memory, so the result does not
// depend on scheduling.  A block covers RED_THREADS / SG float4 columns of one pair (act) or one token
// (combine).  Many splits over few pairs (one token) use 16 or 32 groups; few splits or many pairs use
// one group (each thread sums its column's splits in order), so no thread idles and the grid stays
// small (16 groups for 128 pairs of 3 splits measured 57 us for the activation grid).
constexpr int RED_THREADS = 256;
constexpr int RED_KB = 4;  // routed experts summed per pass of the combine

__device__ __forceinline__ float4 f4add(float4 a, float4 b) { return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }

// gu = bf16(bf16(sum of splits) + bias); a = bf16((clamp(up, -L, L) + 1) * (g * sigmoid(ALPHA g))), g = min(gate, L)
__device__ __forceinline__ uint16_t swiglu_clamped(float gs, float us, uint16_t gb, uint16_t ub) {
  const float g = bf16_to_f32(f32_to_bf16(bf16_to_f32(f32_to_bf16(gs)) + bf16_to_f32(gb)));
  const float u = bf16_to_f32(f32_to_bf16(bf16_to_f32(f32_to_bf16(us)) + bf16_to_f32(ub)));
  const float gc = fminf(g, LIMIT), uc = fminf(fmaxf(u, -LIMIT), LIMIT);
  const float glu = gc / (1.0f + expf(-gc * ALPHA));
  return f32_to_bf16((uc + 1.0f) * glu);
}

template <int RED_SG>
__global__ void __launch_bounds__(RED_THREADS) act_kernel(MoeShape S, int P, int nsplit, const int32_t* __restrict__ experts,
                                                          const uint16_t* __restrict__ gub, Ws W) {
  constexpr int RED_C4 = RED_THREADS / RED_SG;
  __shared__ float4 red[RED_SG][RED_C4];
  pdl_wait();
  pdl_launch_dependents();
  const int64_t wd = (2 * int64_t(S.I) > S.H ? 2 * int64_t(S.I) : S.H);
  const int64_t n4 = int64_t(S.I) / 2;  // float4 columns of a gate/up row (2I partial sums)
  const int c4 = threadIdx.x % RED_C4, sg = threadIdx.x / RED_C4;
  const int64_t chunks = (n4 + RED_C4 - 1) / RED_C4;
  const float4* part = reinterpret_cast<const float4*>(W.part);
  for (int64_t blk = blockIdx.x; blk < int64_t(P) * chunks; blk += gridDim.x) {
    const int pos = int(blk / chunks);
    const int64_t col4 = (blk - int64_t(pos) * chunks) * RED_C4 + c4;
    const int pair = W.g.order[pos];
    const int valid = W.g.posof[pair], e = experts[pair];
    if (valid < 0) continue;  // block-uniform
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    uint2 bias = make_uint2(0u, 0u);  // (gate, up) bf16 of activations 2 col4 and 2 col4 + 1
    if (col4 < n4) {
      if (sg == 0) bias = *reinterpret_cast<const uint2*>(gub + int64_t(e) * 2 * S.I + 4 * col4);
#pragma unroll 4
      for (int sp = sg; sp < nsplit; sp += RED_SG) acc = f4add(acc, part[((int64_t(sp) * P + pos) * wd) / 4 + col4]);
    }
    red[sg][c4] = acc;
    __syncthreads();
#pragma unroll
    for (int st = RED_SG / 2; st > 0; st >>= 1) {  // fixed tree over the groups
      if (sg < st) red[sg][c4] = f4add(red[sg][c4], red[sg + st][c4]);
      __syncthreads();
    }
    if (sg == 0 && col4 < n4) {
      const float4 v = red[0][c4];
      const uint32_t lo = swiglu_clamped(v.x, v.y, uint16_t(bias.x), uint16_t(bias.x >> 16)),
                     hi = swiglu_clamped(v.z, v.w, uint16_t(bias.y), uint16_t(bias.y >> 16));
      *reinterpret_cast<uint32_t*>(W.act + int64_t(pos) * S.I + 2 * col4) = lo | (hi << 16);
    }
    __syncthreads();
  }
}

// out[t] = bf16(sum_j w[t,j] * (bf16(sum of splits) + bias_d[e])); CMB_SG split groups of RED_THREADS / CMB_SG
// float4 columns (32 groups when there are many splits: one token has few columns to spread over)
template <int CMB_SG>
__global__ void __launch_bounds__(RED_THREADS) combine_kernel(const float* __restrict__ meta, int N, int k, MoeShape S,
                                                              int nsplit, const int32_t* __restrict__ experts,
                                                              const uint16_t* __restrict__ db, Ws W,
                                                              uint16_t* __restrict__ out) {
  constexpr int CMB_C4 = RED_THREADS / CMB_SG;
  __shared__ float4 red[RED_KB][CMB_SG][CMB_C4];
  pdl_wait();
  pdl_launch_dependents();
  const int64_t P = int64_t(N) * k;
  const int64_t wd = (2 * int64_t(S.I) > S.H ? 2 * int64_t(S.I) : S.H);
  const int64_t n4 = S.H / 4;
  const int c4 = threadIdx.x % CMB_C4, sg = threadIdx.x / CMB_C4;
  const int64_t chunks = (n4 + CMB_C4 - 1) / CMB_C4;
  const float4* part = reinterpret_cast<const float4*>(W.part);
  for (int64_t blk = blockIdx.x; blk < int64_t(N) * chunks; blk += gridDim.x) {
    const int t = int(blk / chunks);
    const int64_t col4 = (blk - int64_t(t) * chunks) * CMB_C4 + c4;
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    for (int j0 = 0; j0 < k; j0 += RED_KB) {
      const int nj = k - j0 < RED_KB ? k - j0 : RED_KB;
      float4 acc[RED_KB];
      int pos[RED_KB];
      uint2 bias[RED_KB];
      float w[RED_KB];
      // everything but the partials first: positions, routing weights and biases of the experts
#pragma unroll
      for (int jj = 0; jj < RED_KB; ++jj) {
        acc[jj] = make_float4(0.f, 0.f, 0.f, 0.f);
        pos[jj] = jj < nj && col4 < n4 ? W.g.posof[t * k + j0 + jj] : -1;
        bias[jj] = make_uint2(0u, 0u);
        w[jj] = 0.0f;
        if (sg == 0 && pos[jj] >= 0) {
          bias[jj] = *reinterpret_cast<const uint2*>(db + int64_t(experts[t * k + j0 + jj]) * S.H + 4 * col4);
          w[jj] = meta[int64_t(t) * 2 * k + k + j0 + jj];
        }
      }
#pragma unroll 2
      for (int sp = sg; sp < nsplit; sp += CMB_SG) {  // the experts' loads of one split are independent
#pragma unroll
        for (int jj = 0; jj < RED_KB; ++jj)
          if (pos[jj] >= 0) acc[jj] = f4add(acc[jj], part[((int64_t(sp) * P + pos[jj]) * wd) / 4 + col4]);
      }
#pragma unroll
      for (int jj = 0; jj < RED_KB; ++jj) red[jj][sg][c4] = acc[jj];
      __syncthreads();
      // the groups' sums meet in a fixed tree (every thread of the lower half adds, log2(CMB_SG) steps)
#pragma unroll
      for (int st = CMB_SG / 2; st > 0; st >>= 1) {
        if (sg < st)
#pragma unroll
          for (int jj = 0; jj < RED_KB; ++jj) red[jj][sg][c4] = f4add(red[jj][sg][c4], red[jj][sg + st][c4]);
        __syncthreads();
      }
      if (sg == 0 && col4 < n4) {
#pragma unroll
        for (int jj = 0; jj < RED_KB; ++jj) {
          if (pos[jj] < 0) continue;
          const float4 v = red[jj][0][c4];
          const float y[4] = {v.x, v.y, v.z, v.w};
          const uint16_t b[4] = {uint16_t(bias[jj].x), uint16_t(bias[jj].x >> 16), uint16_t(bias[jj].y), uint16_t(bias[jj].y >> 16)};
#pragma unroll
          for (int c = 0; c < 4; ++c)
            o[c] = fmaf(w[jj], bf16_to_f32(f32_to_bf16(bf16_to_f32(f32_to_bf16(y[c])) + bf16_to_f32(b[c]))), o[c]);
        }
      }
      __syncthreads();
    }
    if (sg == 0 && col4 < n4) {
      const uint32_t lo = uint32_t(f32_to_bf16(o[0])) | (uint32_t(f32_to_bf16(o[1])) << 16);
      const uint32_t hi = uint32_t(f32_to_bf16(o[2])) | (uint32_t(f32_to_bf16(o[3])) << 16);
      *reinterpret_cast<uint2*>(out + int64_t(t) * S.H + 4 * col4) = make_uint2(lo, hi);
    }
  }
}

// ------------------------------------------------------------------------------------------------
// Row-streaming GEMV for 4-bit codes with groups of 2^glog >= 64 along the output axis (the
// gpt-oss configuration).  A stored row of the matrix is contiguous, so a slab of 576 output
// columns over 16 rows is a 288-byte x 16-row box of a 3-D tensor map (uint32 elements; dimensions
// row words, rows, expert slots): a producer warp moves four such boxes per stage into shared memory
// with TMA tensor loads (no multicast), and the scale / min windows of those rows and the tokens'
// activation rows with 16-byte cp.async, all completing on one mbarrier per stage of a 4-deep ring.
// Nine consumer warps each own a 64-column block of the slab (a block never straddles a
// quantization group: 64 divides the group, the row length and the matrix offset), so within one
// k-step of 16 rows every output column of the block shares the scale s[r] and min m[r] of row r,
//   y[c] = sum_r (q[r,c] s[r] + m[r]) x[r] = sum_r q[r,c] (s[r] x[r]) + sum_r m[r] x[r].
// The first sum runs on the tensor cores (mma.sync m16n8k16, fp16 operands, fp32 accumulation):
// A holds 128 + q/8 (nibbles at bits 0-3 of a byte) or 128 + 2 q (bits 4-7) as exact fp16 built
// with one PRMT and one LOP3 per pair of rows, B holds fp16(s * x) per row and token (s is fp16 in
// the store, x bf16, so the product is the only rounding).  Two more MMAs with A = 1 give sum_r B
// and sum_r fp16(m * x), which remove the 128 offset and add the mins.
// The MMA's output rows (m) are mapped to columns so that every A register of one MMA has the same
// nibble position: m = g <-> column 8g + {0, 2, 4, 6} (low nibbles) or {1, 3, 5, 7} (high); its
// reduction index k is mapped to rows so that one load instruction reads rows t, t + 4, t + 8 or
// t + 12 (t = lane % 4), which with the 288-byte row pitch fall in disjoint banks.  Two CTAs per SM
// (18 consumer warps, 8 stages in flight) measured 50 us per gpt-oss-20b layer at one token against
// 62 us for one CTA of 15 consumer warps on 960-column slabs, and 52 us for four CTAs of 5.
// With `fuse_group` (at most 32 pairs) the gate_up grid groups the pairs itself: every CTA's producer
// warp ranks them into shared memory and CTA 0 also writes the grouping to the workspace for the
// activation, down and combine grids, so no grouping grid runs before it.
// Units (8-token pass, K split, slab) are dealt round-robin, so neighbouring CTAs read the slabs of
// the same rows at about the same time; the producer decodes a pass (slot, positions, token rows)
// only when it changes.  Each unit writes its own split partial, summed in a fixed order by the
// activation / combine kernels.
// ------------------------------------------------------------------------------------------------
namespace rows {
constexpr int CONS = 9;                    // consumer warps, one 64-column block each (9 | 45 and 90 blocks)
constexpr int THREADS = (CONS + 1) * 32;   // + the producer warp
constexpr int SLAB = CONS * 64;            // output columns per slab
constexpr int SR = 64;                     // rows per stage
constexpr int STAGES = 4;
constexpr int PITCH = SLAB / 2;            // bytes per staged row (the tensor box is dense): 72 words, rows t..t+3 in disjoint banks
constexpr int BOX_ROWS = 16;               // rows per tensor box (one k-step)
constexpr int XP = SR + 8;                 // bf16 per staged activation row (36 words: conflict-free across tokens)
constexpr int CODE_BYTES = SR * PITCH;
// halfs per window: a 16-byte aligned start (<= 7 groups before the slab's first) and the slab's groups (groups >= 64)
constexpr int WIN = 7 + (SLAB - 1) / 64 + 1 <= 16 ? 16 : 32;
constexpr int SWS = 4 * WIN + 16;          // bytes per row of windows: scales, mins, pad (rows 4 or 20 banks apart)
constexpr int SCALE_BYTES = SR * SWS;
constexpr int X_BYTES = 8 * XP * 2;
constexpr int STAGE_BYTES = CODE_BYTES + SCALE_BYTES + X_BYTES;
constexpr int META = 12;                   // ints of stage metadata
constexpr int GRP_INTS = 256;              // in-kernel grouping (<= 32 pairs): 7 arrays of 32, n_groups, n_gp
constexpr int SMEM = STAGES * STAGE_BYTES + STAGES * 2 * 8 + STAGES * META * 4 + GRP_INTS * 4;
static_assert(batched::TOK == 8, "a unit is one 8-token pass of the grouping");
static_assert(STAGE_BYTES % 128 == 0 && (BOX_ROWS * PITCH) % 128 == 0, "128-byte aligned tensor boxes");
static_assert(SLAB / 8 <= 256, "a tensor box is at most 256 elements wide");

enum { M_END, M_SLOT, M_POS0, M_NT, M_SLAB, M_SP, M_ROW0, M_NROWS, M_FIRST, M_LAST };

__device__ __forceinline__ void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// the barrier's pending count drops by one when every cp.async this thread issued so far has landed
__device__ __forceinline__ void cp_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// one box of the 3-D tensor map at (x words, y rows, z slot) into shared memory, completing on `bar` (no multicast)
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
// fp16 pair product, one rounding
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
// bf16 pair -> fp16 pair (exact for |x| in [2^-14, 65504])
__device__ __forceinline__ uint32_t bf2_to_h2(uint32_t v) {
  __half2 r = __floats2half2_rn(__uint_as_float(v << 16), __uint_as_float(v & 0xFFFF0000u));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
constexpr uint32_t MAGIC = 0x58005800u;  // fp16 pair (128, 128): mantissa unit 1/8
constexpr uint32_t ONES = 0x3C003C00u;   // fp16 pair (1, 1)
__device__ __forceinline__ uint32_t lo_pair(uint32_t w) { return (w & 0x000F000Fu) | MAGIC; }  // 128 + q/8
__device__ __forceinline__ uint32_t hi_pair(uint32_t w) { return (w & 0x00F000F0u) | MAGIC; }  // 128 + 2 q

struct Geo {
  int64_t ncol, e0;  // output columns, first element of the matrix in the code stream
  int K, kst, nslab;
};
template <int MAT>
__device__ __forceinline__ Geo geo(const MoeShape& S) {
  Geo g;
  g.ncol = MAT == 0 ? 2 * int64_t(S.I) : S.H;
  g.K = MAT == 0 ? S.H : S.I;
  g.e0 = MAT == 0 ? 0 : 2 * int64_t(S.H) * S.I;
  g.kst = g.K / 16;
  g.nslab = int((g.ncol + SLAB - 1) / SLAB);
  return g;
}

template <int MAT>
__global__ void __launch_bounds__(THREADS, 2) rows_kernel(const __grid_constant__ CUtensorMap tmap, const uint8_t* __restrict__ pool,
                                                          MoeShape S, int P, int nsplit, const uint16_t* __restrict__ x, Ws W,
                                                          const float* __restrict__ meta_in, int N, int fuse_group) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  int* meta = reinterpret_cast<int*>(empty + STAGES);
  int* grp = meta + STAGES * META;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int b = 0; b < STAGES; ++b) {
      mbar_init(&full[b], 33);  // the producer's expect_tx arrival + one cp.async arrival per producer lane
      mbar_init(&empty[b], CONS);
    }
    mbar_fence_init();
  }
  __syncthreads();
  pdl_wait();
  pdl_launch_dependents();
  const Geo G = geo<MAT>(S);
  const int64_t wd = (2 * int64_t(S.I) > S.H ? 2 * int64_t(S.I) : S.H);

  if (warp == CONS) {  // ---------------- producer ----------------
    batched::Ws g = W.g;  // where this warp reads the grouping
    if (fuse_group) {
      batched::Ws sg = W.g;
      sg.order = grp + 32;
      sg.posof = grp + 64;
      sg.grp_slot = grp + 96;
      sg.grp_start = grp + 128;
      sg.grp_count = grp + 160;
      sg.gp_list = grp + 192;
      sg.n_groups = grp + 224;
      sg.n_gp = grp + 225;
      sg.next_unit = nullptr;
      batched::warp_group(meta_in, N, S.k, S.nslots, sg, grp);
      if (blockIdx.x == 0) {  // publish for the later grids (they wait for this grid's completion)
        const int ng = sg.n_groups[0], ngp = sg.n_gp[0];
        if (lane < P) {
          W.g.order[lane] = sg.order[lane];
          W.g.posof[lane] = sg.posof[lane];
        }
        if (lane < ng) {
          W.g.grp_slot[lane] = sg.grp_slot[lane];
          W.g.grp_start[lane] = sg.grp_start[lane];
          W.g.grp_count[lane] = sg.grp_count[lane];
        }
        if (lane < ngp) W.g.gp_list[lane] = sg.gp_list[lane];
        if (lane == 0) {
          W.g.n_groups[0] = ng;
          W.g.n_gp[0] = ngp;
          W.g.next_unit[0] = 0;
          W.g.next_unit[1] = 0;
        }
      }
      g = sg;
    }
    const int64_t total = int64_t(g.n_gp[0]) * G.nslab * nsplit;
    int stage = 0, cur = -1, slot = 0, pos0 = 0, nt = 0;
    const uint16_t* xr = x;  // lane t < nt: the activation row of token t of the pass
    for (int64_t u = blockIdx.x;; u += gridDim.x) {
      const bool end = u >= total;
      int slab = 0, sp = 0, ks0 = 0, ks1 = 1;
      if (!end) {
        slab = int(u % G.nslab);
        const int64_t rest = u / G.nslab;
        sp = int(rest % nsplit);
        const int gpi = int(rest / nsplit);
        if (gpi != cur) {
          const int gp = g.gp_list[gpi];
          const int gr = gp >> 8, t0 = (gp & 255) * 8, cnt = g.grp_count[gr];
          slot = g.grp_slot[gr];
          pos0 = g.grp_start[gr] + t0;
          nt = cnt - t0 < 8 ? cnt - t0 : 8;
          if (lane < nt)
            xr = MAT == 0 ? x + int64_t(g.order[pos0 + lane] / S.k) * S.H : W.act + int64_t(pos0 + lane) * S.I;
          cur = gpi;
        }
        ks0 = int(int64_t(G.kst) * sp / nsplit);
        ks1 = int(int64_t(G.kst) * (sp + 1) / nsplit);
      }
      const int64_t c0 = int64_t(slab) * SLAB;
      const int ncols = int(G.ncol - c0 < SLAB ? G.ncol - c0 : SLAB);
      const uint16_t* sc = reinterpret_cast<const uint16_t*>(pool + int64_t(slot) * S.nbytes + S.ncode);
      const int nst = end ? 1 : (16 * (ks1 - ks0) + SR - 1) / SR;
      for (int st = 0; st < nst; ++st, ++stage) {
        const int b = stage % STAGES, n = stage / STAGES;
        if (n > 0 && !mbar_wait(&empty[b], (n - 1) & 1)) return;
        const int row0 = 16 * ks0 + st * SR;
        const int nrows = end ? 0 : (16 * ks1 - row0 < SR ? 16 * ks1 - row0 : SR);
        uint8_t* stg = smem + b * STAGE_BYTES;
        if (lane == 0) {
          int* m = meta + b * META;
          m[M_END] = end;
          m[M_SLOT] = slot;
          m[M_POS0] = pos0;
          m[M_NT] = nt;
          m[M_SLAB] = slab;
          m[M_SP] = sp;
          m[M_ROW0] = row0;
          m[M_NROWS] = nrows;
          m[M_FIRST] = st == 0;
          m[M_LAST] = st == nst - 1;
          mbar_expect_tx(&full[b], uint32_t(nrows) * PITCH);  // whole boxes: a narrower last slab reads zero fill
        }
        __syncwarp();
        if (!end) {
          if (lane < nrows / BOX_ROWS)
            tma_load_3d(stg + lane * BOX_ROWS * PITCH, &tmap, int(c0 / 8), row0 + lane * BOX_ROWS, slot, &full[b]);
          // scale and min windows: 16-byte chunk c of array a (0 scales, 1 mins) of row r, the chunks the row's groups reach
          uint8_t* sw = stg + CODE_BYTES;
          constexpr int NCH = WIN / 8;  // 16-byte chunks per window
          for (int t = lane; t < 2 * NCH * nrows; t += 32) {
            const int r = t / (2 * NCH), a = (t / NCH) & 1, c = t % NCH;
            const int64_t e = G.e0 + int64_t(row0 + r) * G.ncol + c0;
            const int64_t g0 = e >> S.glog, gw = g0 & ~int64_t(7), g1 = (e + ncols - 1) >> S.glog;
            if (g1 >= gw + 8 * c) cp16(sw + r * SWS + 2 * WIN * a + 16 * c, sc + int64_t(a) * S.ng + gw + 8 * c);
          }
          // activation rows: lane t copies token t's row (8 rows of bf16 per chunk)
          uint16_t* xs = reinterpret_cast<uint16_t*>(stg + CODE_BYTES + SCALE_BYTES);
          if (lane < nt)
            for (int c = 0; c < nrows / 8; ++c) cp16(xs + lane * XP + 8 * c, xr + row0 + 8 * c);
        }
        cp_arrive_noinc(&full[b]);
      }
      if (end) break;
    }
    return;
  }

  // ---------------- consumers: warp `warp` owns columns [64 warp, 64 warp + 64) of each slab ----------------
  const int gid = lane >> 2, tig = lane & 3;
  float acc[4][4], accS[4], accM[4];
  for (int stage = 0;; ++stage) {
    const int b = stage % STAGES, n = stage / STAGES;
    if (!mbar_wait(&full[b], n & 1)) return;
    const int* m = meta + b * META;
    if (m[M_END]) break;
    // every field is read before this warp releases the stage (the producer then rewrites it)
    const int pos0 = m[M_POS0], nt = m[M_NT], row0 = m[M_ROW0], nrows = m[M_NROWS], sp = m[M_SP];
    const bool first = m[M_FIRST] != 0, last = m[M_LAST] != 0;
    const int64_t c0 = int64_t(m[M_SLAB]) * SLAB;
    const bool active = c0 + 64 * warp < G.ncol;  // warp-uniform: the last slab may be narrower
    if (first) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[j][i] = 0.0f;
        accS[j] = 0.0f;
        accM[j] = 0.0f;
      }
    }
    const uint8_t* stg = smem + b * STAGE_BYTES;
    if (active) {
      // this lane's rows lane and lane + 32 of the stage, each as (scale | min << 16) in fp16
      const uint8_t* sw = stg + CODE_BYTES;
      uint32_t smv[2] = {0u, 0u};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = lane + 32 * h;
        if (r < nrows) {
          const int64_t e = G.e0 + int64_t(row0 + r) * G.ncol + c0;
          const int off = int(((e + 64 * warp) >> S.glog) - ((e >> S.glog) & ~int64_t(7)));
          smv[h] = uint32_t(*reinterpret_cast<const uint16_t*>(sw + r * SWS + 2 * off)) |
                   (uint32_t(*reinterpret_cast<const uint16_t*>(sw + r * SWS + 2 * WIN + 2 * off)) << 16);
        }
      }
      // k-step j: reduction index (2 tig, 2 tig + 1, 2 tig + 8, 2 tig + 9) <-> rows 16 j + tig + (0, 4, 8, 12)
      const uint8_t* cb = stg + tig * PITCH + 32 * warp + 4 * gid;
      const uint16_t* xs = reinterpret_cast<const uint16_t*>(stg + CODE_BYTES + SCALE_BYTES) + gid * XP + tig;
      const bool tok = gid < nt;
#pragma unroll
      for (int j = 0; j < SR / 16; ++j) {
        if (16 * j < nrows) {  // warp-uniform
          const uint8_t* c = cb + 16 * j * PITCH;
          const uint32_t w0 = *reinterpret_cast<const uint32_t*>(c);
          const uint32_t w1 = *reinterpret_cast<const uint32_t*>(c + 4 * PITCH);
          const uint32_t w8 = *reinterpret_cast<const uint32_t*>(c + 8 * PITCH);
          const uint32_t w9 = *reinterpret_cast<const uint32_t*>(c + 12 * PITCH);
          uint32_t x01 = 0u, x89 = 0u;
          if (tok) {
            const uint16_t* xj = xs + 16 * j;
            x01 = bf2_to_h2(uint32_t(xj[0]) | (uint32_t(xj[4]) << 16));
            x89 = bf2_to_h2(uint32_t(xj[8]) | (uint32_t(xj[12]) << 16));
          }
          // rows 16 j + tig + {0, 4, 8, 12}: held by lanes (16 j + tig + {0, 4, 8, 12}) mod 32, slot j / 2
          const int lr = (16 * j + tig) & 31;
          const uint32_t v0 = __shfl_sync(0xffffffffu, smv[j / 2], lr), v1 = __shfl_sync(0xffffffffu, smv[j / 2], lr + 4);
          const uint32_t v8 = __shfl_sync(0xffffffffu, smv[j / 2], lr + 8), v9 = __shfl_sync(0xffffffffu, smv[j / 2], lr + 12);
          const uint32_t s01 = prmt(v0, v1, 0x5410), m01 = prmt(v0, v1, 0x7632);
          const uint32_t s89 = prmt(v8, v9, 0x5410), m89 = prmt(v8, v9, 0x7632);
          const uint32_t b0 = hmul2(s01, x01), b1 = hmul2(s89, x89);
          const uint32_t n0 = hmul2(m01, x01), n1 = hmul2(m89, x89);
          const uint32_t u01 = prmt(w0, w1, 0x5410), v01 = prmt(w0, w1, 0x7632);
          const uint32_t u89 = prmt(w8, w9, 0x5410), v89 = prmt(w8, w9, 0x7632);
          const uint32_t uu01 = u01 >> 8, vv01 = v01 >> 8, uu89 = u89 >> 8, vv89 = v89 >> 8;
          mma_f16(acc[0], lo_pair(u01), lo_pair(uu01), lo_pair(u89), lo_pair(uu89), b0, b1);  // columns 0, 2
          mma_f16(acc[1], hi_pair(u01), hi_pair(uu01), hi_pair(u89), hi_pair(uu89), b0, b1);  // columns 1, 3
          mma_f16(acc[2], lo_pair(v01), lo_pair(vv01), lo_pair(v89), lo_pair(vv89), b0, b1);  // columns 4, 6
          mma_f16(acc[3], hi_pair(v01), hi_pair(vv01), hi_pair(v89), hi_pair(vv89), b0, b1);  // columns 5, 7
          mma_f16(accS, ONES, ONES, ONES, ONES, b0, b1);
          mma_f16(accM, ONES, ONES, ONES, ONES, n0, n1);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[b]);
    if (last && active) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int t = 2 * tig + h;
        if (t < nt) {
          const float s128 = 128.0f * accS[h], mm = accM[h];
          float* dst = W.part + (int64_t(sp) * P + pos0 + t) * wd + c0 + 64 * warp + 8 * gid;
          // low nibbles carry q/8, high nibbles 2 q
          const float y0 = (acc[0][h] - s128) * 8.0f + mm, y2 = (acc[0][2 + h] - s128) * 8.0f + mm;
          const float y1 = (acc[1][h] - s128) * 0.5f + mm, y3 = (acc[1][2 + h] - s128) * 0.5f + mm;
          const float y4 = (acc[2][h] - s128) * 8.0f + mm, y6 = (acc[2][2 + h] - s128) * 8.0f + mm;
          const float y5 = (acc[3][h] - s128) * 0.5f + mm, y7 = (acc[3][2 + h] - s128) * 0.5f + mm;
          reinterpret_cast<float4*>(dst)[0] = make_float4(y0, y1, y2, y3);
          reinterpret_cast<float4*>(dst)[1] = make_float4(y4, y5, y6, y7);
        }
      }
    }
  }
}
}  // namespace rows

}  // namespace gptoss
}  // namespace wisp
