// Batched MoE decode: N tokens, each with its own top-k experts (BASELINE configs 2 and 4; the
// reference's bs > 1 branch, wisp/moe.py:62-137: unique experts, dequant, per-expert MLP, weighted
// index_add).  The (token, choice) pairs are grouped by slot on the device, so every routed expert's
// weights are read once per call however many tokens chose it, and the per-expert products run on the
// tensor cores (mma.sync m16n8k16 bf16, fp32 accumulation) with the weights dequantized in registers
// bit-exactly as the reference does (bf16(q*s + m), wisp/quant.py:76-87).
//
// K layout: a lane streams one 32-code unit of a weight row per 128-code block (16 bytes at 4 bit);
// MMA step s of the block takes code pairs 2s and 2s+1 of that unit as its A elements (k = 2c, 2c+1
// and 8+2c, 9+2c).  The B operand (activations) is gathered with the same permutation of k, so the
// products are the plain dot products.
//
//   group_kernel    sort the N*k pairs by slot (bitonic, one CTA): groups (slot, start, count)
//   gate_up_kernel  per (group, 16 rows of I): a = silu(Wg x) * (Wu x) for the group's tokens, bf16
//   down_kernel     per (group, 16 rows of H): y = Wd a, fp32
//   combine_kernel  out[t] = bf16(sum_j w[t,j] * y[t,j]) in a fixed order
#pragma once
#include "common.cuh"
#include "moe_decode.cuh"

namespace wisp {
namespace batched {

constexpr int MAX_PAIRS = 2048;  // N * k
constexpr int WARPS = 8;
constexpr int THREADS = WARPS * 32;
constexpr int NT_MAX = 4;        // token n-tiles (of 8) per pass over the weights

struct Ws {
  int* n_groups;     // [1]
  int* grp_slot;     // [P]
  int* grp_start;    // [P]
  int* grp_count;    // [P]
  int* order;        // [P] pair index at each sorted position
  int* posof;        // [P] sorted position of each pair (-1: skipped)
  uint16_t* a;       // [P][I] bf16
  float* y;          // [P][H] fp32
};

__host__ __device__ inline int64_t ws_bytes(int P, int64_t H, int64_t I) {
  const int64_t ints = ((1 + 5 * int64_t(P)) * 4 + 255) / 256 * 256;
  const int64_t a = (int64_t(P) * I * 2 + 255) / 256 * 256;
  return ints + a + int64_t(P) * H * 4;
}

__host__ __device__ inline Ws ws_carve(void* base, int P, int64_t I) {
  Ws w;
  int* ip = static_cast<int*>(base);
  w.n_groups = ip;
  w.grp_slot = ip + 1;
  w.grp_start = w.grp_slot + P;
  w.grp_count = w.grp_start + P;
  w.order = w.grp_count + P;
  w.posof = w.order + P;
  uint8_t* b = static_cast<uint8_t*>(base) + ((1 + 5 * int64_t(P)) * 4 + 255) / 256 * 256;
  w.a = reinterpret_cast<uint16_t*>(b);
  w.y = reinterpret_cast<float*>(b + (int64_t(P) * I * 2 + 255) / 256 * 256);
  return w;
}

// ---- grouping ---------------------------------------------------------------------------------------
// One CTA of 1024 threads.  Key = slot << 32 | pair; invalid slots sort last and are skipped (flagged,
// except -1, which marks an empty pair such as the padding of an expert-parallel dispatch buffer).
__global__ void __launch_bounds__(1024) group_kernel(const float* __restrict__ meta, int N, int k, int64_t nslots, Ws W) {
  __shared__ unsigned long long key[MAX_PAIRS];
  __shared__ int scan[MAX_PAIRS];
  const int P = N * k;
  int n2 = 1;
  while (n2 < P) n2 <<= 1;
  pdl_wait();
  for (int i = threadIdx.x; i < n2; i += blockDim.x) {
    unsigned long long kk = ~0ull;
    if (i < P) {
      const int t = i / k, j = i - t * k;
      const float f = meta[int64_t(t) * 2 * k + j];
      if (f >= 0.0f && f < float(nslots)) kk = (static_cast<unsigned long long>(int64_t(f)) << 32) | unsigned(i);
      else {
        if (f != -1.0f) flag(WISP_STATUS_BAD_SLOT);  // -1: an empty pair (padding), skipped silently
        kk = (0xFFFFFFFFull << 32) | unsigned(i);
      }
    }
    key[i] = kk;
  }
  __syncthreads();
  for (int size = 2; size <= n2; size <<= 1)
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < n2; i += blockDim.x) {
        const int o = i ^ stride;
        if (o > i) {
          const bool up = (i & size) == 0;
          const unsigned long long a = key[i], b = key[o];
          if ((a > b) == up) {
            key[i] = b;
            key[o] = a;
          }
        }
      }
      __syncthreads();
    }
  // group starts -> ids by an inclusive scan
  for (int i = threadIdx.x; i < n2; i += blockDim.x) {
    const unsigned s = unsigned(key[i] >> 32);
    const bool valid = i < P && s != 0xFFFFFFFFu;
    scan[i] = valid && (i == 0 || unsigned(key[i - 1] >> 32) != s) ? 1 : 0;
  }
  __syncthreads();
  for (int off = 1; off < n2; off <<= 1) {
    int v[2] = {0, 0};
    for (int i = threadIdx.x, q = 0; i < n2 && q < 2; i += blockDim.x, ++q) v[q] = i >= off ? scan[i - off] : 0;
    __syncthreads();
    for (int i = threadIdx.x, q = 0; i < n2 && q < 2; i += blockDim.x, ++q) scan[i] += v[q];
    __syncthreads();
  }
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    const unsigned s = unsigned(key[i] >> 32);
    const int pair = int(key[i] & 0xFFFFFFFFu);
    W.order[i] = pair;
    const bool valid = s != 0xFFFFFFFFu;
    W.posof[pair] = valid ? i : -1;
    if (valid && (i == 0 || unsigned(key[i - 1] >> 32) != s)) {
      const int gid = scan[i] - 1;
      W.grp_slot[gid] = int(s);
      W.grp_start[gid] = i;
      int e = i + 1;
      while (e < P && unsigned(key[e] >> 32) == s) ++e;
      W.grp_count[gid] = e - i;
    }
  }
  if (threadIdx.x == 0) W.n_groups[0] = n2 > 0 ? scan[P - 1 < 0 ? 0 : P - 1] : 0;
  pdl_launch_dependents();
}

// ---- dequantized A fragments ------------------------------------------------------------------------
// 32 codes (one unit) of a row -> 16 bf16 pairs: pair p = codes 2p, 2p+1 -> bf16(q*s + m)
template <int BITS>
__device__ __forceinline__ void dequant_unit(const Unit<BITS>& u, float s, float m, uint32_t (&pr)[16]) {
#pragma unroll
  for (int p = 0; p < 16; ++p) {
    const float w0 = __fadd_rn(__fmul_rn(small_u2f(unit_code<BITS>(u, 2 * p)), s), m);
    const float w1 = __fadd_rn(__fmul_rn(small_u2f(unit_code<BITS>(u, 2 * p + 1)), s), m);
    pr[p] = uint32_t(f32_to_bf16(w0)) | (uint32_t(f32_to_bf16(w1)) << 16);
  }
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// one row's unit (codes [kc, kc + 32)) of matrix `mat` of the expert at `base`, with its scale and min
template <int BITS>
__device__ __forceinline__ void row_unit(const uint8_t* base, const MoeShape& S, int mat, int64_t row, int64_t K, int64_t kc,
                                         uint32_t (&pr)[16]) {
  const int64_t e = int64_t(mat) * S.H * S.I + row * K + kc;  // element index in the expert's code stream
  const Unit<BITS> u = load_unit<BITS>(base + e * BITS / 8);
  const int64_t gi = e / S.group;
  const float s = f16_bits_to_f32(ld_nc_u16(reinterpret_cast<const uint16_t*>(base + S.ncode) + gi));
  const float m = f16_bits_to_f32(ld_nc_u16(reinterpret_cast<const uint16_t*>(base + S.ncode) + S.ng + gi));
  dequant_unit<BITS>(u, s, m, pr);
}

// ---- gate/up: a[pos][r] = bf16(silu(Wg[r] . x_t) * (Wu[r] . x_t)) ---------------------------------------
template <int BITS>
__global__ void __launch_bounds__(THREADS) gate_up_kernel(const uint8_t* __restrict__ pool, MoeShape S,
                                                          const uint16_t* __restrict__ x, Ws W) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  pdl_wait();
  pdl_launch_dependents();
  const int ngr = W.n_groups[0];
  const int tiles = S.I / 16;
  const int64_t nunits = int64_t(ngr) * tiles;
  const int gw = blockIdx.x * WARPS + (threadIdx.x >> 5), nw = gridDim.x * WARPS;
  for (int64_t u = gw; u < nunits; u += nw) {
    const int grp = int(u / tiles), tile = int(u - int64_t(grp) * tiles);
    const uint8_t* base = pool + int64_t(W.grp_slot[grp]) * S.nbytes;
    const int start = W.grp_start[grp], cnt = W.grp_count[grp];
    const int r0 = tile * 16;
    for (int t0 = 0; t0 < cnt; t0 += 8 * NT_MAX) {
      // the B column (token) each lane feeds for each n-tile: lane g' -> token of position t0 + 8 nt + g'
      const uint16_t* xrow[NT_MAX];
#pragma unroll
      for (int nt = 0; nt < NT_MAX; ++nt) {
        const int p = t0 + 8 * nt + g;
        xrow[nt] = p < cnt ? x + int64_t(W.order[start + p] / S.k) * S.H : nullptr;
      }
      float dg[NT_MAX][4] = {}, du[NT_MAX][4] = {};
      for (int64_t kb = 0; kb < S.H; kb += 128) {
        const int64_t kc = kb + 32 * c;
        uint32_t ga[16], gb[16], ua[16], ub[16];
        row_unit<BITS>(base, S, 0, r0 + g, S.H, kc, ga);
        row_unit<BITS>(base, S, 0, r0 + g + 8, S.H, kc, gb);
        row_unit<BITS>(base, S, 1, r0 + g, S.H, kc, ua);
        row_unit<BITS>(base, S, 1, r0 + g + 8, S.H, kc, ub);
#pragma unroll
        for (int s = 0; s < 8; ++s) {
#pragma unroll
          for (int nt = 0; nt < NT_MAX; ++nt) {
            if (8 * nt < cnt - t0) {  // warp-uniform
              uint2 b = make_uint2(0, 0);
              if (xrow[nt]) b = *reinterpret_cast<const uint2*>(xrow[nt] + kc + 4 * s);
              mma16816(dg[nt], ga[2 * s], gb[2 * s], ga[2 * s + 1], gb[2 * s + 1], b.x, b.y);
              mma16816(du[nt], ua[2 * s], ub[2 * s], ua[2 * s + 1], ub[2 * s + 1], b.x, b.y);
            }
          }
        }
      }
      // D: rows r0 + g (d0, d1) and r0 + g + 8 (d2, d3), token columns 2c, 2c + 1 of each n-tile
#pragma unroll
      for (int nt = 0; nt < NT_MAX; ++nt) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int p = t0 + 8 * nt + 2 * c + (q & 1);
          const int r = r0 + g + (q >> 1) * 8;
          if (p < cnt) W.a[int64_t(start + p) * S.I + r] = f32_to_bf16(silu_mul(dg[nt][q], du[nt][q]));
        }
      }
    }
  }
}

// ---- down: y[pos][h] = Wd[h] . a[pos] --------------------------------------------------------------------
template <int BITS>
__global__ void __launch_bounds__(THREADS) down_kernel(const uint8_t* __restrict__ pool, MoeShape S, Ws W) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  pdl_wait();
  pdl_launch_dependents();
  const int ngr = W.n_groups[0];
  const int tiles = S.H / 16;
  const int64_t nunits = int64_t(ngr) * tiles;
  const int gw = blockIdx.x * WARPS + (threadIdx.x >> 5), nw = gridDim.x * WARPS;
  for (int64_t u = gw; u < nunits; u += nw) {
    const int grp = int(u / tiles), tile = int(u - int64_t(grp) * tiles);
    const uint8_t* base = pool + int64_t(W.grp_slot[grp]) * S.nbytes;
    const int start = W.grp_start[grp], cnt = W.grp_count[grp];
    const int r0 = tile * 16;
    for (int t0 = 0; t0 < cnt; t0 += 8 * NT_MAX) {
      const uint16_t* arow[NT_MAX];
#pragma unroll
      for (int nt = 0; nt < NT_MAX; ++nt) {
        const int p = t0 + 8 * nt + g;
        arow[nt] = p < cnt ? W.a + int64_t(start + p) * S.I : nullptr;
      }
      float d[NT_MAX][4] = {};
      for (int64_t kb = 0; kb < S.I; kb += 128) {
        const int64_t kc = kb + 32 * c;
        uint32_t wa[16], wb[16];
        row_unit<BITS>(base, S, 2, r0 + g, S.I, kc, wa);
        row_unit<BITS>(base, S, 2, r0 + g + 8, S.I, kc, wb);
#pragma unroll
        for (int s = 0; s < 8; ++s) {
#pragma unroll
          for (int nt = 0; nt < NT_MAX; ++nt) {
            if (8 * nt < cnt - t0) {
              uint2 b = make_uint2(0, 0);
              if (arow[nt]) b = *reinterpret_cast<const uint2*>(arow[nt] + kc + 4 * s);
              mma16816(d[nt], wa[2 * s], wb[2 * s], wa[2 * s + 1], wb[2 * s + 1], b.x, b.y);
            }
          }
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT_MAX; ++nt) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int p = t0 + 8 * nt + 2 * c + (q & 1);
          const int r = r0 + g + (q >> 1) * 8;
          if (p < cnt) W.y[int64_t(start + p) * S.H + r] = d[nt][q];
        }
      }
    }
  }
}

// ---- combine: out[t][h] = bf16(sum_j w[t][j] * y[posof(t, j)][h]), j in order ------------------------------
__global__ void combine_kernel(const float* __restrict__ meta, int N, int k, int64_t H, Ws W, uint16_t* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < int64_t(N) * H; i += int64_t(gridDim.x) * blockDim.x) {
    const int t = int(i / H);
    const int64_t h = i - int64_t(t) * H;
    float s = 0.0f;
    for (int j = 0; j < k; ++j) {
      const int pos = W.posof[t * k + j];
      if (pos >= 0) s = fmaf(meta[int64_t(t) * 2 * k + k + j], W.y[int64_t(pos) * H + h], s);
    }
    out[i] = f32_to_bf16(s);
  }
}

}  // namespace batched
}  // namespace wisp
