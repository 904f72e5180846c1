// gpt-oss experts (the reference's PagedGptOssBlock, wisp/gptoss.py:107-143).
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

// gu = bf16(bf16(sum of splits) + bias); a = bf16((clamp(up, -L, L) + 1) * (g * sigmoid(ALPHA g))), g = min(gate, L)
__global__ void act_kernel(MoeShape S, int P, int nsplit, const int32_t* __restrict__ experts, const uint16_t* __restrict__ gub,
                           Ws W) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t wd = (2 * int64_t(S.I) > S.H ? 2 * int64_t(S.I) : S.H);
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < int64_t(P) * S.I; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t pos = i / S.I, c = i - pos * S.I;
    const int pair = W.g.order[pos];
    if (W.g.posof[pair] < 0) continue;
    const int e = experts[pair];
    float gs = 0.0f, us = 0.0f;
    for (int s = 0; s < nsplit; ++s) {
      const float* row = W.part + (int64_t(s) * P + pos) * wd;
      gs += row[2 * c];
      us += row[2 * c + 1];
    }
    const float g = bf16_to_f32(f32_to_bf16(bf16_to_f32(f32_to_bf16(gs)) + bf16_to_f32(gub[int64_t(e) * 2 * S.I + 2 * c])));
    const float u = bf16_to_f32(f32_to_bf16(bf16_to_f32(f32_to_bf16(us)) + bf16_to_f32(gub[int64_t(e) * 2 * S.I + 2 * c + 1])));
    const float gc = fminf(g, LIMIT), uc = fminf(fmaxf(u, -LIMIT), LIMIT);
    const float glu = gc / (1.0f + expf(-gc * ALPHA));
    W.act[pos * S.I + c] = f32_to_bf16((uc + 1.0f) * glu);
  }
}

__global__ void combine_kernel(const float* __restrict__ meta, int N, int k, MoeShape S, int nsplit,
                               const int32_t* __restrict__ experts, const uint16_t* __restrict__ db, Ws W,
                               uint16_t* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t P = int64_t(N) * k, H = S.H;
  const int64_t wd = (2 * int64_t(S.I) > S.H ? 2 * int64_t(S.I) : S.H);
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < int64_t(N) * H; i += int64_t(gridDim.x) * blockDim.x) {
    const int t = int(i / H);
    const int64_t h = i - int64_t(t) * H;
    float o = 0.0f;
    for (int j = 0; j < k; ++j) {
      const int pair = t * k + j;
      const int pos = W.g.posof[pair];
      if (pos < 0) continue;
      float y = 0.0f;
      for (int s = 0; s < nsplit; ++s) y += W.part[(int64_t(s) * P + pos) * wd + h];
      y = bf16_to_f32(f32_to_bf16(bf16_to_f32(f32_to_bf16(y)) + bf16_to_f32(db[int64_t(experts[pair]) * H + h])));
      o = fmaf(meta[int64_t(t) * 2 * k + k + j], y, o);
    }
    out[i] = f32_to_bf16(o);
  }
}

}  // namespace gptoss
}  // namespace wisp
