// Batched MoE decode: N tokens, each with its own top-k experts (N = 1 to 64 per step; the
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
#include "tma.cuh"

namespace wisp {
namespace batched {

constexpr int MAX_PAIRS = 2048;  // N * k
constexpr int WARPS = 8;
constexpr int THREADS = WARPS * 32;
constexpr int NT_MAX = 1;        // token n-tiles (of 8) per pass over the weights

constexpr int TOK = 8 * NT_MAX;  // tokens per pass over an expert's weights

struct Ws {
  int* n_groups;     // [1]
  int* grp_slot;     // [P]
  int* grp_start;    // [P]
  int* grp_count;    // [P]
  int* order;        // [P] pair index at each sorted position
  int* posof;        // [P] sorted position of each pair (-1: skipped)
  int* n_gp;         // [1] number of (group, pass) entries
  int* next_unit;    // [2] work counters of the gate/up and down grids
  int* gp_list;      // [P] (group << 8 | pass), passes with more token tiles first
  uint16_t* a;       // [P][I] bf16
  float* y;          // [P][H] fp32
  uint16_t* xp;      // [P][H] bf16: the tokens' rows pair-permuted (4-bit / 2-bit kernels)
};

__host__ __device__ inline int64_t ws_ints_bytes(int P) { return ((4 + 6 * int64_t(P)) * 4 + 255) / 256 * 256; }

__host__ __device__ inline int64_t ws_bytes(int P, int64_t H, int64_t I) {
  const int64_t ints = ws_ints_bytes(P);
  const int64_t a = (int64_t(P) * I * 2 + 255) / 256 * 256;
  const int64_t y = (int64_t(P) * H * 4 + 255) / 256 * 256;
  return ints + a + y + int64_t(P) * H * 2;
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
  w.n_gp = w.posof + P;
  w.next_unit = w.n_gp + 1;
  w.gp_list = w.next_unit + 2;
  uint8_t* b = static_cast<uint8_t*>(base) + ws_ints_bytes(P);
  w.a = reinterpret_cast<uint16_t*>(b);
  w.y = reinterpret_cast<float*>(b + (int64_t(P) * I * 2 + 255) / 256 * 256);
  w.xp = nullptr;
  return w;
}

// the pair-permuted token rows live after the grouping ints, a and y
__host__ __device__ inline uint16_t* ws_xp(void* base, int P, int64_t H, int64_t I) {
  const int64_t ints = ws_ints_bytes(P);
  const int64_t a = (int64_t(P) * I * 2 + 255) / 256 * 256;
  const int64_t y = (int64_t(P) * H * 4 + 255) / 256 * 256;
  return reinterpret_cast<uint16_t*>(static_cast<uint8_t*>(base) + ints + a + y);
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
  pdl_launch_dependents();  // the next grid may launch now; its own wait covers this whole grid
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
    }
  }
  __syncthreads();  // group starts are written (global memory, this CTA)
  for (int i = threadIdx.x; i < P; i += blockDim.x) {  // the last pair of each group closes it
    const unsigned s = unsigned(key[i] >> 32);
    if (s != 0xFFFFFFFFu && (i + 1 == P || unsigned(key[i + 1] >> 32) != s)) {
      const int gid = scan[i] - 1;
      W.grp_count[gid] = i + 1 - W.grp_start[gid];
    }
  }
  if (threadIdx.x == 0) W.n_groups[0] = n2 > 0 ? scan[P - 1 < 0 ? 0 : P - 1] : 0;
  // the (group, pass) work list of the grouped kernels, bucketed by the pass's token tiles (4 first), so
  // the dynamically scheduled grids start with their most expensive units
  __shared__ int bcnt[NT_MAX + 1], bofs[NT_MAX + 1];
  if (threadIdx.x <= NT_MAX) bcnt[threadIdx.x] = 0;
  __syncthreads();  // group arrays (written above by this CTA) and the bucket counters
  const int ngr = P > 0 ? scan[P - 1] : 0;
  for (int gid = threadIdx.x; gid < ngr; gid += blockDim.x) {
    const int cnt = W.grp_count[gid];
    for (int t0 = 0; t0 < cnt; t0 += TOK) atomicAdd(&bcnt[min(NT_MAX, (cnt - t0 + 7) / 8)], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int o = 0;
    for (int nt = NT_MAX; nt >= 1; --nt) {
      bofs[nt] = o;
      o += bcnt[nt];
    }
    W.n_gp[0] = o;
    W.next_unit[0] = 0;
    W.next_unit[1] = 0;
  }
  __syncthreads();
  for (int gid = threadIdx.x; gid < ngr; gid += blockDim.x) {
    const int cnt = W.grp_count[gid];
    for (int t0 = 0, p = 0; t0 < cnt; t0 += TOK, ++p) W.gp_list[atomicAdd(&bofs[min(NT_MAX, (cnt - t0 + 7) / 8)], 1)] = gid << 8 | p;
  }
}

// ---- grouping by counting sort (pools up to CS_MAX_SLOTS slots) -------------------------------------------
// The same outputs as group_kernel (groups in slot order, pairs of a group contiguous, invalid pairs
// after the valid ones, the work list) from a shared-memory histogram of the slots: one atomic per
// pair, two block scans over the slots, one scatter.  Pairs inside a group come in atomic order, which
// changes nothing downstream: every pair's result is computed on its own.
constexpr int CS_MAX_SLOTS = 24576;  // counts + starts: 192 KB of shared memory
__host__ __device__ inline size_t count_group_smem(int64_t nslots) { return size_t(nslots) * 8; }

// exclusive block scan of two values (blockDim.x a multiple of 32, <= 1024); totals to every thread
__device__ __forceinline__ void block_scan2(int a, int g, int& ea, int& eg, int& ta, int& tg, int* wa, int* wg) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int ia = a, ig = g;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int ya = __shfl_up_sync(0xffffffffu, ia, o), yg = __shfl_up_sync(0xffffffffu, ig, o);
    if (lane >= o) {
      ia += ya;
      ig += yg;
    }
  }
  if (lane == 31) {
    wa[warp] = ia;
    wg[warp] = ig;
  }
  __syncthreads();
  if (warp == 0) {
    int va = lane < nw ? wa[lane] : 0, vg = lane < nw ? wg[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int ya = __shfl_up_sync(0xffffffffu, va, o), yg = __shfl_up_sync(0xffffffffu, vg, o);
      if (lane >= o) {
        va += ya;
        vg += yg;
      }
    }
    if (lane < nw) {
      wa[lane] = va;
      wg[lane] = vg;
    }
  }
  __syncthreads();
  const int pa = warp > 0 ? wa[warp - 1] : 0, pg = warp > 0 ? wg[warp - 1] : 0;
  ea = pa + ia - a;
  eg = pg + ig - g;
  ta = wa[nw - 1];
  tg = wg[nw - 1];
  __syncthreads();  // wa / wg may be reused
}

// The same outputs for at most 32 pairs, in one warp: each lane ranks its pair by (slot, index) with
// shuffles (invalid pairs after the valid ones), the ranked keys go through shared memory, and group
// starts, indices and sizes come from ballots.  No histogram over the slots and no global read-back,
// which is what the one-CTA kernels spend their time on for a handful of pairs.
constexpr int SMALL_PAIRS = 32;
static_assert(NT_MAX == 1, "the warp grouping lists passes in group order (no token-tile buckets)");
// one warp (lane = threadIdx.x % 32) writes the grouping of P = N * k <= 32 pairs into W; key_at is 32 ints of
// the warp's shared memory; W's arrays may be shared or global memory (next_unit is skipped when null)
__device__ __forceinline__ void warp_group(const float* __restrict__ meta, int N, int k, int64_t nslots, const Ws& W,
                                           int* key_at) {
  const int P = N * k, p = threadIdx.x & 31;
  int sl = -1;
  if (p < P) {
    const int tk = p / k, j = p - tk * k;
    const float f = meta[int64_t(tk) * 2 * k + j];
    if (f >= 0.0f && f < float(nslots)) sl = int(f);
    else if (f != -1.0f) flag(WISP_STATUS_BAD_SLOT);  // -1: an empty pair (padding), skipped silently
  }
  // sort key: valid pairs by slot, then invalid ones; ties by pair index; lanes >= P last of all
  const int key = p >= P ? 0x7FFFFFFF : (sl >= 0 ? sl : 0x7FFFFFFE);
  int rank = 0;
  for (int q = 0; q < SMALL_PAIRS; ++q) {
    const int kq = __shfl_sync(0xffffffffu, key, q);
    rank += (kq < key || (kq == key && q < p)) ? 1 : 0;
  }
  key_at[rank] = key;
  __syncwarp();
  if (p < P) {
    W.order[rank] = p;
    W.posof[p] = sl >= 0 ? rank : -1;
  }
  // lane i now stands for sorted position i
  const int ki = key_at[p], kprev = p > 0 ? key_at[p - 1] : -1;
  const bool valid = p < P && ki < 0x7FFFFFFE;
  const unsigned starts = __ballot_sync(0xffffffffu, valid && ki != kprev);
  const unsigned validm = __ballot_sync(0xffffffffu, valid);
  const int ngroups = __popc(starts);
  if (valid && ki != kprev) {
    const int gid = __popc(starts & ((1u << p) - 1u));
    const unsigned later = starts & ~((2u << p) - 1u);  // starts after this one (p <= 31: 2u << 31 wraps to 0)
    const int end = later ? __ffs(later) - 1 : __popc(validm);  // valid positions are a prefix
    const int cnt = end - p;
    W.grp_slot[gid] = ki;
    W.grp_start[gid] = p;
    W.grp_count[gid] = cnt;
  }
  // (group, pass) list in group order: group g's passes start after all earlier groups' passes
  const bool st = valid && ki != kprev;
  int npass = 0;
  if (st) {
    const unsigned later = starts & ~((2u << p) - 1u);
    const int end = later ? __ffs(later) - 1 : __popc(validm);
    npass = (end - p + TOK - 1) / TOK;
  }
  int before = npass;  // inclusive prefix over lanes
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, before, o);
    if (p >= o) before += v;
  }
  const int total = __shfl_sync(0xffffffffu, before, 31);
  if (st) {
    const int gid = __popc(starts & ((1u << p) - 1u));
    for (int pp = 0; pp < npass; ++pp) W.gp_list[before - npass + pp] = gid << 8 | pp;
  }
  if (p == 0) {
    W.n_groups[0] = ngroups;
    W.n_gp[0] = total;
    if (W.next_unit) {
      W.next_unit[0] = 0;
      W.next_unit[1] = 0;
    }
  }
  __syncwarp();
}

__global__ void __launch_bounds__(32) small_group_kernel(const float* __restrict__ meta, int N, int k, int64_t nslots, Ws W) {
  __shared__ int key_at[SMALL_PAIRS];
  pdl_wait();
  pdl_launch_dependents();  // the next grid may launch now; its own wait covers this whole grid
  warp_group(meta, N, k, nslots, W, key_at);
}

__global__ void __launch_bounds__(1024) count_group_kernel(const float* __restrict__ meta, int N, int k, int64_t nslots, Ws W) {
  extern __shared__ int cs[];  // [nslots] counts, then [nslots] group starts
  __shared__ int rank_in[MAX_PAIRS];
  __shared__ int slot_of[MAX_PAIRS];
  __shared__ int wa[32], wg[32];
  __shared__ int tail;
  __shared__ int bcnt[NT_MAX + 1], bofs[NT_MAX + 1];
  int* cnt = cs;
  int* st = cs + nslots;
  const int P = N * k, t = threadIdx.x, nt = blockDim.x;
  pdl_wait();
  pdl_launch_dependents();  // the next grid may launch now; its own wait covers this whole grid
  for (int64_t i = t; i < nslots; i += nt) cnt[i] = 0;
  if (t == 0) tail = 0;
  if (t <= NT_MAX) bcnt[t] = 0;
  __syncthreads();
  for (int p = t; p < P; p += nt) {
    const int tk = p / k, j = p - tk * k;
    const float f = meta[int64_t(tk) * 2 * k + j];
    int sl = -1;
    if (f >= 0.0f && f < float(nslots)) sl = int(f);
    else if (f != -1.0f) flag(WISP_STATUS_BAD_SLOT);  // -1: an empty pair (padding), skipped silently
    slot_of[p] = sl;
    rank_in[p] = sl >= 0 ? atomicAdd(&cnt[sl], 1) : -1;
  }
  __syncthreads();
  // slot range of this thread: counts -> starts, non-empty slots -> groups
  const int64_t per = (nslots + nt - 1) / nt;
  const int64_t lo = int64_t(t) * per, hi = lo + per < nslots ? lo + per : nslots;
  int a = 0, g = 0;
  for (int64_t i = lo; i < hi; ++i) {
    a += cnt[i];
    g += cnt[i] > 0 ? 1 : 0;
  }
  int ea, eg, ta, tg;
  block_scan2(a, g, ea, eg, ta, tg, wa, wg);
  for (int64_t i = lo; i < hi; ++i) {
    const int c = cnt[i];
    st[i] = ea;
    if (c > 0) {
      W.grp_slot[eg] = int(i);
      W.grp_start[eg] = ea;
      W.grp_count[eg] = c;
      ++eg;
    }
    ea += c;
  }
  if (t == 0) W.n_groups[0] = tg;
  __syncthreads();
  for (int p = t; p < P; p += nt) {
    const int sl = slot_of[p];
    const int pos = sl >= 0 ? st[sl] + rank_in[p] : ta + atomicAdd(&tail, 1);  // invalid pairs after the valid ones
    W.order[pos] = p;
    W.posof[p] = sl >= 0 ? pos : -1;
  }
  __syncthreads();  // group arrays (global memory, this CTA)
  // the (group, pass) work list, bucketed by the pass's token tiles (as group_kernel)
  for (int gid = t; gid < tg; gid += nt) {
    const int c = W.grp_count[gid];
    for (int t0 = 0; t0 < c; t0 += TOK) atomicAdd(&bcnt[min(NT_MAX, (c - t0 + 7) / 8)], 1);
  }
  __syncthreads();
  if (t == 0) {
    int o = 0;
    for (int ntl = NT_MAX; ntl >= 1; --ntl) {
      bofs[ntl] = o;
      o += bcnt[ntl];
    }
    W.n_gp[0] = o;
    W.next_unit[0] = 0;
    W.next_unit[1] = 0;
  }
  __syncthreads();
  for (int gid = t; gid < tg; gid += nt) {
    const int c = W.grp_count[gid];
    for (int t0 = 0, pp = 0; t0 < c; t0 += TOK, ++pp) W.gp_list[atomicAdd(&bofs[min(NT_MAX, (c - t0 + 7) / 8)], 1)] = gid << 8 | pp;
  }
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
  const int64_t gi = group_of(e, S);
  const float s = f16_bits_to_f32(ld_nc_u16(reinterpret_cast<const uint16_t*>(base + S.ncode) + gi));
  const float m = f16_bits_to_f32(ld_nc_u16(reinterpret_cast<const uint16_t*>(base + S.ncode) + S.ng + gi));
  dequant_unit<BITS>(u, s, m, pr);
}

// ---- the grouped products -----------------------------------------------------------------------------
// A CTA takes one group (expert) and 8 tiles of 16 rows (one per warp) of the output matrix; the
// activation rows of the group's tokens (up to TOK per pass) are staged once in shared memory (rows
// padded by 4 elements: the fragment loads stay within two-way bank conflicts) and every warp streams
// its rows' weight units from HBM, the next K block's units loaded while the current one computes.
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
          const int64_t gi = group_of(e, S);
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

// ---- 4-bit and 2-bit codes straight into the MMA ----------------------------------------------------------
// bf16(128 + q) is exact for q < 128, so two codes become one A register with two integer ops: the pair
// (n_i, n_{i + W/2}) of a 32-bit code word (W = 32 / BITS codes) is ((w >> BITS*i) & mask) | 0x43004300.
// Over one 128-code block (one scale s and min m per row: group % 128 == 0) the MMA then yields
// D = sum_k (128 + q_k) x_k, and the block's dot product with the dequantized weights q*s + m is
// s*D + (m - 128 s) * sum_k x_k, folded once per block.  (The reference rounds each weight to bf16
// before the product; this form skips that rounding, well inside the parity tolerance.)
//
// Activations are kept "pair-permuted": inside every W-element word, position 2i holds element i and
// 2i + 1 holds element i + W/2, so the four B elements of MMA step s of a lane's 32-code unit sit at
// unit offset 4s, contiguous.  In shared memory each 128-element block is further stored step-major
// ([step][lane c][4]) with a row pitch of K + 16 elements: the fragment loads are bank-conflict free.
template <int BITS>
__host__ __device__ constexpr int pair_word() { return 32 / BITS; }

template <int BITS>
__device__ __forceinline__ int perm_pos(int e) {  // position of natural element e in the pair-permuted row
  constexpr int Wc = 32 / BITS, h = Wc / 2;
  const int i = e & (Wc - 1);
  return (e & ~(Wc - 1)) + (i < h ? 2 * i : 2 * (i - h) + 1);
}

template <int BITS>
__device__ __forceinline__ uint32_t code_pair(uint32_t w, int i) {
  constexpr uint32_t mask = BITS == 4 ? 0x000F000Fu : 0x00030003u;
  return ((w >> (BITS * i)) & mask) | 0x43004300u;
}

// rows [rows][K] bf16 (natural order) -> pair-permuted copy
template <int BITS>
__global__ void permute_rows_kernel(const uint16_t* __restrict__ x, int64_t nwords, uint16_t* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < nwords; i += int64_t(gridDim.x) * blockDim.x) {
    if constexpr (BITS == 4) {  // 8 elements: out word q = (x_q, x_{q+4})
      const uint4 a = reinterpret_cast<const uint4*>(x)[i];
      reinterpret_cast<uint4*>(out)[i] = make_uint4(__byte_perm(a.x, a.z, 0x5410), __byte_perm(a.x, a.z, 0x7632),
                                                    __byte_perm(a.y, a.w, 0x5410), __byte_perm(a.y, a.w, 0x7632));
    } else {  // 16 elements: out word q = (x_q, x_{q+8})
      const uint4 a = reinterpret_cast<const uint4*>(x)[2 * i], b = reinterpret_cast<const uint4*>(x)[2 * i + 1];
      reinterpret_cast<uint4*>(out)[2 * i] = make_uint4(__byte_perm(a.x, b.x, 0x5410), __byte_perm(a.x, b.x, 0x7632),
                                                        __byte_perm(a.y, b.y, 0x5410), __byte_perm(a.y, b.y, 0x7632));
      reinterpret_cast<uint4*>(out)[2 * i + 1] = make_uint4(__byte_perm(a.z, b.z, 0x5410), __byte_perm(a.z, b.z, 0x7632),
                                                            __byte_perm(a.w, b.w, 0x5410), __byte_perm(a.w, b.w, 0x7632));
    }
  }
}

constexpr int NIB_PAD = 16;  // row pitch K + 16 elements: (K + 16) / 2 words = 8 mod 32 banks
__host__ __device__ inline int64_t nib_stage_bytes(int64_t K) {
  return int64_t(TOK) * (K + NIB_PAD) * 2 + int64_t(TOK) * (K / 128) * 4;
}

// MAT 0: gate and up (rows of I, K = H, input the pair-permuted x of the tokens) -> a (pair-permuted, bf16)
// MAT 2: down (rows of H, K = I, input the pair-permuted a of the pairs) -> y (fp32)
// A unit is (group, pass of up to TOK tokens, 128-row chunk); CTAs take units from a counter in the
// order of the work list (passes with more token tiles first), which balances Zipf-skewed groups.  At
// the start of a unit every warp asks L2 for its 16 rows (one contiguous range per matrix) and the
// per-lane register loads then find them there.
template <int BITS, int MAT>
__global__ void __launch_bounds__(THREADS, 3) grouped_nib_kernel(const uint8_t* __restrict__ pool, MoeShape S,
                                                                 const uint16_t* __restrict__ xp, Ws W) {
  extern __shared__ __align__(16) uint16_t xs[];  // [TOK][K + NIB_PAD] bf16, then xsum [TOK][K / 128] fp32
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  pdl_wait();
  pdl_launch_dependents();
  const int ngr = W.n_groups[0];
  const int64_t rows = MAT == 0 ? S.I : S.H;
  const int64_t K = MAT == 0 ? S.H : S.I;
  const int64_t KP = K + NIB_PAD;
  const int nblk = int(K / 128);
  float* xsum = reinterpret_cast<float*>(xs + int64_t(TOK) * KP);
  const int chunks = int((rows + ROWS_PER_CTA - 1) / ROWS_PER_CTA);
  const int64_t nunits = int64_t(W.n_gp[0]) * chunks;
  (void)ngr;
  constexpr int NQ = MAT == 0 ? 4 : 2;  // rows of a lane: gate g, gate g+8, up g, up g+8 (MAT 0); g, g+8
  const int64_t row_bytes = K * BITS / 8;
  int staged_grp = -1, staged_t0 = -1;
  __shared__ int64_t s_unit;
  for (;;) {
    __syncthreads();  // every thread has read s_unit
    if (threadIdx.x == 0) s_unit = atomicAdd(&W.next_unit[MAT == 0 ? 0 : 1], 1);
    __syncthreads();
    const int64_t u = s_unit;
    if (u >= nunits) break;
    const int gp = W.gp_list[u / chunks];
    const int grp = gp >> 8, ch = int(u % chunks);
    const uint8_t* base = pool + int64_t(W.grp_slot[grp]) * S.nbytes;
    const int start = W.grp_start[grp], cnt = W.grp_count[grp];
    const int64_t r0 = int64_t(ch) * ROWS_PER_CTA + 16 * warp;
    const bool active = r0 < rows;  // warp-uniform
    if (active && lane < (MAT == 0 ? 2 : 1)) {
      // lane 0: gate (or down) rows r0..r0+15, lane 1 (MAT 0): up rows -- one contiguous range each
      const int mat = MAT == 0 ? lane : 2;
      prefetch_l2(base + int64_t(mat) * S.mat_bytes + r0 * row_bytes, uint32_t(16 * row_bytes));
    }
    {
      const int t0 = (gp & 255) * TOK;
      const int nt_used = (cnt - t0 + 7) / 8 < NT_MAX ? (cnt - t0 + 7) / 8 : NT_MAX;
      if (grp != staged_grp || t0 != staged_t0) {
        // ---- stage the activation rows of tokens [t0, t0 + TOK) (zeros past the group), block b's
        //      4-element chunk q = 8 c + s at chunk 4 s + c; block sums into xsum
        __syncthreads();  // the previous readers are done
        const int nchunk = int(K / 4);
        const int rows_used = 8 * nt_used;  // rows past the pass's token tiles are never read
        for (int i = threadIdx.x; i < rows_used * (nchunk / 2); i += blockDim.x) {
          const int t = i / (nchunk / 2);
          const int q2 = i - t * (nchunk / 2);  // a pair of chunks: 2 q2, 2 q2 + 1 (same block)
          uint4 v = make_uint4(0, 0, 0, 0);
          if (t0 + t < cnt) {
            const uint16_t* src = MAT == 0 ? xp + int64_t(W.order[start + t0 + t] / S.k) * S.H : W.a + int64_t(start + t0 + t) * S.I;
            v = reinterpret_cast<const uint4*>(src)[q2];
          }
          const int q = 2 * q2, blk = q >> 5, qq = q & 31;  // 32 chunks per 128-element block
          const int d0 = blk * 32 + (qq & 7) * 4 + (qq >> 3), d1 = blk * 32 + ((qq + 1) & 7) * 4 + ((qq + 1) >> 3);
          uint16_t* row = xs + int64_t(t) * KP;
          *reinterpret_cast<uint2*>(row + 4 * d0) = make_uint2(v.x, v.y);
          *reinterpret_cast<uint2*>(row + 4 * d1) = make_uint2(v.z, v.w);
        }
        __syncthreads();
        // block sums: one warp per (token, block), fixed order
        for (int i = warp; i < rows_used * nblk; i += WARPS) {
          const int t = i / nblk, blk = i - t * nblk;
          const uint2 v = *reinterpret_cast<const uint2*>(xs + int64_t(t) * KP + blk * 128 + 4 * lane);
          float sx = __uint_as_float(v.x << 16) + __uint_as_float(v.x & 0xFFFF0000u) + __uint_as_float(v.y << 16) +
                     __uint_as_float(v.y & 0xFFFF0000u);
          sx = warp_sum(sx);
          if (lane == 0) xsum[t * nblk + blk] = sx;
        }
        __syncthreads();
        staged_grp = grp, staged_t0 = t0;
      }
      if (!active) continue;
      float acc0[NT_MAX][4] = {}, acc1[NT_MAX][4] = {};
      uint32_t cw[NQ][BITS], nw[NQ][BITS];
      float csc[NQ], cmn[NQ], nsc[NQ], nmn[NQ];
      auto fetch = [&](int blk, uint32_t (&ww)[NQ][BITS], float (&sc)[NQ], float (&mn)[NQ]) {
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
          const int mat = MAT == 0 ? (q >> 1) : 2;
          const int64_t row = r0 + g + (q & 1) * 8;
          const int64_t e = int64_t(mat) * S.H * S.I + row * K + int64_t(blk) * 128 + 32 * c;
          const Unit<BITS> uu = load_unit<BITS>(base + e * BITS / 8);
#pragma unroll
          for (int i = 0; i < BITS; ++i) ww[q][i] = uu.w[i];
          const int64_t gi = group_of(e, S);
          sc[q] = f16_bits_to_f32(ld_nc_u16(reinterpret_cast<const uint16_t*>(base + S.ncode) + gi));
          mn[q] = f16_bits_to_f32(ld_nc_u16(reinterpret_cast<const uint16_t*>(base + S.ncode) + S.ng + gi));
        }
      };
      fetch(0, cw, csc, cmn);
      for (int blk = 0; blk < nblk; ++blk) {
        if (blk + 1 < nblk) fetch(blk + 1, nw, nsc, nmn);
        float D0[NT_MAX][4] = {}, D1[NT_MAX][4] = {};
        const uint16_t* xb = xs + int64_t(blk) * 128 + 4 * c;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          constexpr int SPW = 32 / BITS / 4;  // MMA steps per code word: 2 (4-bit), 4 (2-bit)
          const int j = s / SPW, i0 = 2 * (s % SPW);
          uint32_t a[NQ][2];
#pragma unroll
          for (int q = 0; q < NQ; ++q) {
            a[q][0] = code_pair<BITS>(cw[q][j], i0);
            a[q][1] = code_pair<BITS>(cw[q][j], i0 + 1);
          }
#pragma unroll
          for (int nt = 0; nt < NT_MAX; ++nt) {
            if (nt < nt_used) {  // warp-uniform
              const uint2 bb = *reinterpret_cast<const uint2*>(xb + int64_t(8 * nt + g) * KP + 16 * s);
              mma16816(D0[nt], a[0][0], a[1][0], a[0][1], a[1][1], bb.x, bb.y);
              if (MAT == 0) mma16816(D1[nt], a[2][0], a[3][0], a[2][1], a[3][1], bb.x, bb.y);
            }
          }
        }
        // fold: rows g (q 0, 1) and g + 8 (q 2, 3) of the tile, token columns 2c, 2c + 1
#pragma unroll
        for (int nt = 0; nt < NT_MAX; ++nt) {
          if (nt < nt_used) {
            const float xs0 = xsum[(8 * nt + 2 * c) * nblk + blk], xs1 = xsum[(8 * nt + 2 * c + 1) * nblk + blk];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int rq = q >> 1;  // 0: row g, 1: row g + 8
              const float xsv = (q & 1) ? xs1 : xs0;
              acc0[nt][q] = fmaf(csc[rq], D0[nt][q], fmaf(cmn[rq] - 128.0f * csc[rq], xsv, acc0[nt][q]));
              if (MAT == 0)
                acc1[nt][q] = fmaf(csc[2 + rq], D1[nt][q], fmaf(cmn[2 + rq] - 128.0f * csc[2 + rq], xsv, acc1[nt][q]));
            }
          }
        }
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
#pragma unroll
          for (int i = 0; i < BITS; ++i) cw[q][i] = nw[q][i];
          csc[q] = nsc[q];
          cmn[q] = nmn[q];
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT_MAX; ++nt) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int p = t0 + 8 * nt + 2 * c + (q & 1);
          const int64_t r = r0 + g + (q >> 1) * 8;
          if (p < cnt) {
            if (MAT == 0) W.a[int64_t(start + p) * S.I + perm_pos<BITS>(int(r))] = f32_to_bf16(silu_mul(acc0[nt][q], acc1[nt][q]));
            else W.y[int64_t(start + p) * S.H + r] = acc0[nt][q];
          }
        }
      }
    }
  }
}

// ---- combine: out[t][h] = bf16(sum_j w[t][j] * y[posof(t, j)][h]), j in order ------------------------------
// four outputs per thread (H % 4 == 0): float4 loads of y, one 8-byte store
__global__ void combine_kernel(const float* __restrict__ meta, int N, int k, int64_t H, Ws W, uint16_t* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t H4 = H / 4;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < int64_t(N) * H4; i += int64_t(gridDim.x) * blockDim.x) {
    const int t = int(i / H4);
    const int64_t h4 = i - int64_t(t) * H4;
    float4 s = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int j = 0; j < k; ++j) {
      const int pos = W.posof[t * k + j];
      if (pos < 0) continue;
      const float w = meta[int64_t(t) * 2 * k + k + j];
      const float4 y = reinterpret_cast<const float4*>(W.y + int64_t(pos) * H)[h4];
      s.x = fmaf(w, y.x, s.x);
      s.y = fmaf(w, y.y, s.y);
      s.z = fmaf(w, y.z, s.z);
      s.w = fmaf(w, y.w, s.w);
    }
    const uint32_t lo = uint32_t(f32_to_bf16(s.x)) | (uint32_t(f32_to_bf16(s.y)) << 16);
    const uint32_t hi = uint32_t(f32_to_bf16(s.z)) | (uint32_t(f32_to_bf16(s.w)) << 16);
    reinterpret_cast<uint2*>(out + int64_t(t) * H)[h4] = make_uint2(lo, hi);
  }
}

}  // namespace batched
}  // namespace wisp
