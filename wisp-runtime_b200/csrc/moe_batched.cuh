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
//   grouped_kernel<0>  per (group, 128 rows of I): a = silu(Wg x) * (Wu x) for the group's tokens, bf16
//   grouped_kernel<2>  per (group, 128 rows of H): y = Wd a, fp32
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

// ---- the grouped products -----------------------------------------------------------------------------
// A CTA takes one group (expert) and 8 tiles of 16 rows (one per warp) of the output matrix; the
// activation rows of the group's tokens (up to TOK per pass) are staged once in shared memory (rows
// padded by 4 elements: the fragment loads stay within two-way bank conflicts) and every warp streams
// its rows' weight units from HBM, the next K block's units loaded while the current one computes.
constexpr int TOK = 8 * NT_MAX;  // tokens per pass
constexpr int ROWS_PER_CTA = 16 * WARPS;

__host__ __device__ inline int64_t stage_bytes(int64_t K) { return int64_t(TOK) * (K + 4) * 2; }

// MAT 0: gate and up (rows of I, K = H, input x of the tokens) -> a = bf16(silu(g) * u)
// MAT 2: down (rows of H, K = I, input a of the pairs) -> y (fp32)
template <int BITS, int MAT>
__global__ void __launch_bounds__(THREADS, 1) grouped_kernel(const uint8_t* __restrict__ pool, MoeShape S,
                                                             const uint16_t* __restrict__ x, Ws W) {
  extern __shared__ __align__(16) uint16_t xs[];  // [TOK][K + 4]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  pdl_wait();
  pdl_launch_dependents();
  const int ngr = W.n_groups[0];
  const int64_t rows = MAT == 0 ? S.I : S.H;
  const int64_t K = MAT == 0 ? S.H : S.I;
  const int64_t KP = K + 4;
  const int chunks = int((rows + ROWS_PER_CTA - 1) / ROWS_PER_CTA);
  for (int64_t u = blockIdx.x; u < int64_t(ngr) * chunks; u += gridDim.x) {
    const int grp = int(u / chunks), ch = int(u - int64_t(grp) * chunks);
    const uint8_t* base = pool + int64_t(W.grp_slot[grp]) * S.nbytes;
    const int start = W.grp_start[grp], cnt = W.grp_count[grp];
    const int64_t r0 = int64_t(ch) * ROWS_PER_CTA + 16 * warp;
    const bool active = r0 < rows;  // warp-uniform
    for (int t0 = 0; t0 < cnt; t0 += TOK) {
      const int nt_used = (cnt - t0 + 7) / 8 < NT_MAX ? (cnt - t0 + 7) / 8 : NT_MAX;
      // ---- stage the activation rows of tokens [t0, t0 + TOK) (zeros past the group)
      __syncthreads();  // the previous pass's readers are done
      for (int64_t i = threadIdx.x; i < int64_t(TOK) * (K / 8); i += blockDim.x) {
        const int t = int(i / (K / 8));
        const int64_t cp = i - int64_t(t) * (K / 8);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (t0 + t < cnt) {
          const uint16_t* src = MAT == 0 ? x + int64_t(W.order[start + t0 + t] / S.k) * S.H : W.a + int64_t(start + t0 + t) * S.I;
          v = reinterpret_cast<const uint4*>(src)[cp];
        }
        uint2* d = reinterpret_cast<uint2*>(xs + int64_t(t) * KP + cp * 8);  // KP % 4 == 0: 8-byte aligned
        d[0] = make_uint2(v.x, v.y);
        d[1] = make_uint2(v.z, v.w);
      }
      __syncthreads();
      if (!active) continue;
      float d0[NT_MAX][4] = {}, d1[NT_MAX][4] = {};
      // weight units of the current K block (cur) and the next one (nxt)
      Unit<BITS> cu[4], nu[4];
      float csc[4], cmn[4], nsc[4], nmn[4];
      auto fetch = [&](int64_t kb, Unit<BITS> (&uu)[4], float (&sc)[4], float (&mn)[4]) {
#pragma unroll
        for (int q = 0; q < (MAT == 0 ? 4 : 2); ++q) {
          const int mat = MAT == 0 ? (q >> 1) : 2;
          const int64_t row = r0 + g + (q & 1) * 8;
          const int64_t e = int64_t(mat) * S.H * S.I + row * K + kb + 32 * c;
          uu[q] = load_unit<BITS>(base + e * BITS / 8);
          const int64_t gi = e / S.group;
          sc[q] = f16_bits_to_f32(ld_nc_u16(reinterpret_cast<const uint16_t*>(base + S.ncode) + gi));
          mn[q] = f16_bits_to_f32(ld_nc_u16(reinterpret_cast<const uint16_t*>(base + S.ncode) + S.ng + gi));
        }
      };
      fetch(0, cu, csc, cmn);
      for (int64_t kb = 0; kb < K; kb += 128) {
        if (kb + 128 < K) fetch(kb + 128, nu, nsc, nmn);
        uint32_t pa[4][16];
#pragma unroll
        for (int q = 0; q < (MAT == 0 ? 4 : 2); ++q) dequant_unit<BITS>(cu[q], csc[q], cmn[q], pa[q]);
        const int64_t kc = kb + 32 * c;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
#pragma unroll
          for (int nt = 0; nt < NT_MAX; ++nt) {
            if (nt < nt_used) {  // warp-uniform
              const uint2 bb = *reinterpret_cast<const uint2*>(xs + int64_t(8 * nt + g) * KP + kc + 4 * s);
              mma16816(d0[nt], pa[0][2 * s], pa[1][2 * s], pa[0][2 * s + 1], pa[1][2 * s + 1], bb.x, bb.y);
              if (MAT == 0) mma16816(d1[nt], pa[2][2 * s], pa[3][2 * s], pa[2][2 * s + 1], pa[3][2 * s + 1], bb.x, bb.y);
            }
          }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          cu[q] = nu[q];
          csc[q] = nsc[q];
          cmn[q] = nmn[q];
        }
      }
      // D: rows r0 + g (d0, d1) and r0 + g + 8 (d2, d3), token columns 2c, 2c + 1 of each n-tile
#pragma unroll
      for (int nt = 0; nt < NT_MAX; ++nt) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int p = t0 + 8 * nt + 2 * c + (q & 1);
          const int64_t r = r0 + g + (q >> 1) * 8;
          if (p < cnt) {
            if (MAT == 0) W.a[int64_t(start + p) * S.I + r] = f32_to_bf16(silu_mul(d0[nt][q], d1[nt][q]));
            else W.y[int64_t(start + p) * S.H + r] = d0[nt][q];
          }
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
