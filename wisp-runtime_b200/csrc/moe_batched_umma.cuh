// Batched MoE expert products on the 5th-generation tensor cores (tcgen05, accumulators in TMEM), for
// 4-bit and 2-bit codes with quantization groups of a multiple of 128 (the reference's bs > 1 branch,
// wisp/moe.py:62-137: unique experts, dequant, per-expert MLP, weighted index_add).
//
// Work item = (group of pairs routed to one slot, N tile of up to NMAX of its tokens, tile of BM = 128
// weight rows).  Per item the whole K range streams through shared memory in BK = 64 slices:
//
//   warp 0      code producer: TMA tensor loads of the slice's packed codes (one 128-row box per
//               matrix), per item one bulk copy of the tile's scales and mins and an L2 prefetch of the
//               item's (and the next item's) code rows
//   warp 22     activation producer: the tokens' activation rows (fp16, 128-byte swizzled boxes of 32
//               rows); a ring of its own, so the code ring runs ahead of the tensor core by its full depth
//   warps 2-17  dequantize the codes into the MMA's A operand, which lives in TMEM: per 8 codes one
//               LOP3 builds fp16 pairs 1024 + q, one HSUB2 makes q exact, one HFMA2 applies scale and
//               min (a single rounding of q*s + m to fp16: closer to the exact weight than the
//               reference's bf16(q*s + m)); thread t of a warp owns weight row 32 (warp % 4) + t (the
//               TMEM lane it may write) and stores its K pairs with tcgen05.st, four warps per lane
//               quarter splitting the stage's code words
//   warp 1      one thread issues tcgen05.mma (kind::f16, A from TMEM, B from shared memory, M = 128,
//               N = the item's tokens rounded up to 32, K = 16 per instruction) for gate and up (or
//               down) into TMEM accumulators, and commits each stage back to the producers
//   warps 18-21 epilogue: tcgen05.ld of the accumulators; gate/up -> a = silu(g)*u as fp16 rows of the
//               intermediate (pair-permuted, the down pass's activation operand); down -> fp32 rows of
//               y that the combine kernel sums per token in a fixed order.  Two accumulator buffers in
//               TMEM let this run while the other warps stream the next item.
//
// Each code word is read from HBM once per item, however many tokens the expert received (up to
// NMAX per N tile), and it is unpacked once.  With A in TMEM the dequantized tile never passes through
// shared memory: the tensor core reads only the codes' staging and the activation tiles there (the
// shared-memory A tile, 32 KB written and read per stage, bounded the stage time at small N).  Inside a code word the MMA's K order is the pair order
// (codes i and i + W/2 of a W-code word sit side by side); the activations are staged in the same
// order, so the products are the plain dot products.
//
// No TMA multicast, no clusters: the kernels run on one GPU's own memory.  Every wait on an
// mbarrier is bounded; a wait that gives up flags WISP_STATUS_WAIT_TIMEOUT and makes every role
// leave its loop, the producer waits for its copies in flight, the MMA thread for its MMAs, and the
// TMEM is released before the CTA exits.
#pragma once
#include "common.cuh"
#include "moe_batched.cuh"
#include "moe_decode.cuh"
#include "tma.cuh"

namespace wisp {
namespace umma {

constexpr int BM = 128;       // weight rows per tile (MMA M)
constexpr int BK = 64;        // K per stage: 64 fp16 = one 128-byte swizzle row
constexpr int NMAX = 64;      // tokens per N tile (MMA N <= 64; an expert with more tokens takes several tiles)
constexpr int BOXR = 32;      // token rows per activation box; MMA N is a multiple of it
constexpr int CST = 4;        // code stages
constexpr int AST = 3;        // dequantized A stages (in TMEM)
constexpr int BST = 6;        // activation stages
constexpr int DQ_WARPS = 16;  // dequantizing warps (warps 2..17)
constexpr int EPI_WARPS = 4;  // epilogue warps (warps 18..21: one per TMEM lane quarter)
constexpr int EPI0 = 2 + DQ_WARPS;
constexpr int BPROD = EPI0 + EPI_WARPS;  // warp 22: activation producer
constexpr int THREADS = (BPROD + 1) * 32;
// TMEM columns: two accumulator buffers (the epilogue of one item overlaps the main loop of the next),
// gate/up [gate | up] of NMAX columns each, down [down]; then AST stages of the A operand, BK/2
// columns (fp16 pairs) per matrix.  The allocation is the next power of two.
template <int MAT>
constexpr uint32_t acc_cols() { return MAT == 0 ? 2 * NMAX : NMAX; }
template <int MAT>
constexpr uint32_t a_cols() { return (MAT == 0 ? 2 : 1) * (BK / 2); }
template <int MAT>
constexpr uint32_t a_base() { return 2 * acc_cols<MAT>(); }
template <int MAT>
constexpr uint32_t tmem_cols() {
  constexpr uint32_t need = 2 * acc_cols<MAT>() + AST * a_cols<MAT>();
  return need <= 32 ? 32 : need <= 64 ? 64 : need <= 128 ? 128 : need <= 256 ? 256 : 512;
}
static_assert(2 * acc_cols<0>() + AST * a_cols<0>() <= 512, "TMEM holds the accumulators and the A stages");

template <int BITS, int MAT>
struct Cfg {
  static constexpr int NMAT = MAT == 0 ? 2 : 1;
  static constexpr int CODE_ROW = BK * BITS / 8;            // code bytes of one row per stage
  static constexpr int CODE_MAT = BM * CODE_ROW;
  static constexpr int CODE_STAGE = NMAT * CODE_MAT;
  static constexpr int B_STAGE = NMAX * BK * 2;             // 8 KB
  static constexpr int OFF_B = 0;                           // 1024-aligned pieces first
  static constexpr int OFF_C = OFF_B + BST * B_STAGE;
  static constexpr int OFF_S = OFF_C + CST * CODE_STAGE;    // scales/mins: 2 item buffers
  static __host__ __device__ constexpr int scale_bytes(int gpr) { return NMAT * 2 * BM * gpr * 2; }
};

template <int BITS, int MAT>
__host__ __device__ inline int64_t smem_bytes(int gpr) {
  using C = Cfg<BITS, MAT>;
  const int64_t sc = (C::scale_bytes(gpr) + 127) / 128 * 128;
  // + barriers (2 CST + 2 AST + 2 BST + 4 + 5) * 8, the TMEM address, the abort flag, 1 KB alignment slack
  return C::OFF_S + 2 * sc + 256 + 1024;
}

// ---- tcgen05 / TMA wrappers --------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void mbar_arrive1(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// 16 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
        "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// D[tmem] (+)= A[tmem] . B[smem]^T, fp16 inputs, fp32 accumulation (A: 128 lanes = rows, K/2 columns)
__device__ __forceinline__ void tc_mma_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// this thread's TMEM lane, N consecutive 32-bit columns from taddr
__device__ __forceinline__ void tc_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]),
      "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tc_st8(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr), "r"(r[0]), "r"(r[1]),
               "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// shared-memory matrix descriptor: K-major operand in the 128-byte swizzled canonical layout (rows of
// 128 bytes, 8-row atoms of 1 KB stacked at a stride of 1 KB), Blackwell descriptor version 1
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
  return uint64_t((saddr >> 4) & 0x3FFF) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) | (uint64_t(1) << 46) |
         (uint64_t(2) << 61);
}
// instruction descriptor of kind::f16: fp32 accumulator, fp16 A and B, both K-major, M = 128, N = n
__device__ __forceinline__ uint32_t idesc_f16(int n) {
  return (1u << 4) | (uint32_t(n >> 3) << 17) | (uint32_t(BM >> 4) << 24);
}

// bounded wait by a whole warp (every lane polls, the answer is the same on every lane); it also gives
// up as soon as another role raised the CTA's abort flag
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  for (unsigned it = 0; it < WAIT_LIMIT; ++it) {
    if (__all_sync(0xFFFFFFFFu, mbar_try_wait(bar, parity))) return true;
    if ((it & 127) == 127 && __any_sync(0xFFFFFFFFu, *abort != 0)) return false;
  }
  if ((threadIdx.x & 31) == 0) {
    flag(WISP_STATUS_WAIT_TIMEOUT);
    *abort = 1;
  }
  __syncwarp();
  return false;
}

// fp16 pair of codes (i, i + W/2) of word w: 1024 + q each, then q exact
template <int BITS>
__device__ __forceinline__ uint32_t q_pair(uint32_t w, int i) {
  constexpr uint32_t mask = BITS == 4 ? 0x000F000Fu : 0x00030003u;
  uint32_t h;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(h) : "r"(w >> (BITS * i)), "r"(mask), "r"(0x64006400u));  // (a & b) | c
  const __half2 q = __hsub2(*reinterpret_cast<__half2*>(&h), __half2(__float2half_rn(1024.0f), __float2half_rn(1024.0f)));
  return *reinterpret_cast<const uint32_t*>(&q);
}
__device__ __forceinline__ uint32_t deq2(uint32_t q, __half2 s, __half2 m) {
  const __half2 v = __hfma2(*reinterpret_cast<__half2*>(&q), s, m);
  return *reinterpret_cast<const uint32_t*>(&v);
}

struct Item {
  int grp, nt, rt;
};

__device__ __forceinline__ Item item_of(int i, int rtiles, int maxnt) {
  Item it;
  it.rt = i % rtiles;
  const int j = i / rtiles;
  it.nt = j % maxnt;
  it.grp = j / maxnt;
  return it;
}


// ---- activation staging: the tokens' rows in group order, fp16, pair-permuted ---------------------------
// xh[p] = x[order[p] / k] for every sorted position p; inside each code word's span of W = 32/BITS
// elements, element i goes to 2i (i < W/2) or 2(i - W/2) + 1.  bf16 -> fp16 is exact inside fp16's range.
template <int BITS>
__global__ void stage_rows_kernel(const uint16_t* __restrict__ x, int P, int k, int64_t H, batched::Ws W, uint16_t* __restrict__ xh) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t per = H / 16;  // 16 elements (two code words at 4 bit, one at 2 bit) per item
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < int64_t(P) * per; i += int64_t(gridDim.x) * blockDim.x) {
    const int p = int(i / per);
    const int64_t q = i - int64_t(p) * per;
    const int t = W.order[p] / k;
    const uint4* src = reinterpret_cast<const uint4*>(x + int64_t(t) * H + 16 * q);
    const uint4 a = src[0], b = src[1];
    const uint32_t in[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    float v[16];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      v[2 * j] = __uint_as_float(in[j] << 16);
      v[2 * j + 1] = __uint_as_float(in[j] & 0xFFFF0000u);
    }
    uint32_t o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      // output positions 2j, 2j+1 hold elements (e0, e1) of the word span
      int e0, e1;
      if (BITS == 4) {
        const int w = j >> 2, i2 = j & 3;  // word w covers elements 8w..8w+7
        e0 = 8 * w + i2;
        e1 = 8 * w + i2 + 4;
      } else {
        e0 = j;
        e1 = j + 8;
      }
      const __half2 h = __floats2half2_rn(v[e0], v[e1]);
      o[j] = *reinterpret_cast<const uint32_t*>(&h);
    }
    uint4* dst = reinterpret_cast<uint4*>(xh + int64_t(p) * H + 16 * q);
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

// ---- the tensor-core grouped GEMM ------------------------------------------------------------------------
// MAT 0: gate/up rows [I] of every item's expert against the staged token rows (mapB over xh [P][H]),
//        a = silu(gate) * up -> ah [P][I] fp16, pair-permuted
// MAT 2: down rows [H] against ah (mapB over ah [P][I]) -> y [P][H] fp32
// mapC: 3-D map (code bytes of a row, rows, slots) of the codes of gate+up (2I rows) or down (H rows)
template <int BITS, int MAT>
__global__ void __launch_bounds__(THREADS, 1) grouped_umma_kernel(const __grid_constant__ CUtensorMap mapC,
                                                                  const __grid_constant__ CUtensorMap mapB,
                                                                  const uint8_t* __restrict__ pool, MoeShape S, batched::Ws W,
                                                                  uint16_t* __restrict__ ah) {
  using C = Cfg<BITS, MAT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int K = MAT == 0 ? S.H : S.I;
  const int rows = MAT == 0 ? S.I : S.H;
  const int KT = K / BK;
  const int gpr = K / S.group;                      // quantization groups per row
  const int sc_bytes = (C::scale_bytes(gpr) + 127) / 128 * 128;
  uint8_t* sB = smem + C::OFF_B;
  uint8_t* sC = smem + C::OFF_C;
  uint8_t* sS = smem + C::OFF_S;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sS + 2 * sc_bytes);
  uint64_t* code_full = bars;
  uint64_t* code_empty = code_full + CST;
  uint64_t* a_full = code_empty + CST;
  uint64_t* a_empty = a_full + AST;
  uint64_t* b_full = a_empty + AST;
  uint64_t* b_empty = b_full + BST;
  uint64_t* sc_full = b_empty + BST;    // [2]
  uint64_t* sc_empty = sc_full + 2;     // [2]
  uint64_t* acc_full = sc_empty + 2;    // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint64_t* mma_done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  __shared__ int s_maxcnt;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < CST; ++i) {
      mbar_init(code_full + i, 1);
      mbar_init(code_empty + i, DQ_WARPS);
    }
    for (int i = 0; i < AST; ++i) {
      mbar_init(a_full + i, DQ_WARPS);
      mbar_init(a_empty + i, 1);
    }
    for (int i = 0; i < BST; ++i) {
      mbar_init(b_full + i, 1);
      mbar_init(b_empty + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(sc_full + i, 1);
      mbar_init(sc_empty + i, DQ_WARPS);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(acc_full + i, 1);
      mbar_init(acc_empty + i, EPI_WARPS);
    }
    mbar_init(mma_done, 1);
    *abort = 0;
    s_maxcnt = 0;
    mbar_fence_init();
  }
  if (warp == 1) {  // TMEM for the accumulators (the whole warp allocates)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"(tmem_cols<MAT>())
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  pdl_wait();  // the grouping (and, for MAT 2, the gate/up pass) has finished
  pdl_launch_dependents();
  const int ngr = W.n_groups[0];
  __syncthreads();
  for (int g = threadIdx.x; g < ngr; g += blockDim.x) atomicMax(&s_maxcnt, W.grp_count[g]);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int maxnt = (s_maxcnt + NMAX - 1) / NMAX;
  const int rtiles = rows / BM;
  const int nitems = ngr * maxnt * rtiles;

  if (warp == 0) {
    // ================= producer (the whole warp loops, lane 0 issues) =================
    uint32_t cs = 0, cph = 0, ss = 0, sph = 0;
    bool ok = true;
    for (int i = blockIdx.x; i < nitems && ok; i += gridDim.x) {
      const Item it = item_of(i, rtiles, maxnt);
      const int cnt = W.grp_count[it.grp];
      if (it.nt * NMAX >= cnt) continue;
      const int slot = W.grp_slot[it.grp];
      const int r0 = it.rt * BM;
      // the item's code rows (one contiguous range per matrix) and the next item's, pulled into L2 now so
      // the per-stage tensor loads below hit L2 instead of paying HBM latency one small stage at a time
      if (lane < 2 * C::NMAT) {
        const int which = lane / C::NMAT, m = lane % C::NMAT;
        int ii = i;
        if (which) {  // the next item this CTA takes that has tokens
          ii = -1;
          for (int jn = i + int(gridDim.x); jn < nitems; jn += gridDim.x) {
            const Item nx = item_of(jn, rtiles, maxnt);
            if (nx.nt * NMAX < W.grp_count[nx.grp]) {
              ii = jn;
              break;
            }
          }
        }
        if (ii >= 0) {
          const Item px = item_of(ii, rtiles, maxnt);
          const int mat = MAT == 0 ? m : 2;
          const int64_t rb = int64_t(K) * BITS / 8;
          prefetch_l2(pool + int64_t(W.grp_slot[px.grp]) * S.nbytes + mat * S.mat_bytes + int64_t(px.rt) * BM * rb,
                      uint32_t(BM * rb));
        }
      }
      __syncwarp();
      // scales and mins of the tile's rows: one contiguous run per (matrix, kind)
      ok = warp_wait(sc_empty + ss, sph ^ 1, abort);
      if (!ok) break;
      if (lane == 0) {
        const uint32_t run = uint32_t(BM * gpr * 2);
        mbar_expect_tx(sc_full + ss, run * 2 * C::NMAT);
        const uint8_t* base = pool + int64_t(slot) * S.nbytes;
#pragma unroll
        for (int m = 0; m < C::NMAT; ++m) {
          const int mat = MAT == 0 ? m : 2;
          const int64_t gi0 = (int64_t(mat) * S.H * S.I + int64_t(r0) * K) / S.group;
          bulk_g2s(sS + ss * sc_bytes + (2 * m) * run, base + S.ncode + 2 * gi0, run, sc_full + ss);
          bulk_g2s(sS + ss * sc_bytes + (2 * m + 1) * run, base + S.ncode + 2 * (S.ng + gi0), run, sc_full + ss);
        }
      }
      __syncwarp();
      ss ^= 1;
      if (ss == 0) sph ^= 1;
      for (int kt = 0; kt < KT && ok; ++kt) {
        ok = warp_wait(code_empty + cs, cph ^ 1, abort);
        if (!ok) break;
        if (lane == 0) {
          mbar_expect_tx(code_full + cs, C::CODE_STAGE);
          tma_load_3d(sC + cs * C::CODE_STAGE, &mapC, kt * C::CODE_ROW, r0, slot, code_full + cs);
          if (MAT == 0) tma_load_3d(sC + cs * C::CODE_STAGE + C::CODE_MAT, &mapC, kt * C::CODE_ROW, S.I + r0, slot, code_full + cs);
        }
        __syncwarp();
        if (++cs == CST) cs = 0, cph ^= 1;
      }
    }
    // copies still in flight land before the CTA can exit: wait for the last arming of every stage
    // (bounded, ignoring the abort flag; a phase that already completed passes at once)
    if (lane == 0) {
      for (int j = 0; j < CST; ++j) {
        cs = cs == 0 ? CST - 1 : cs - 1;
        if (cs == CST - 1) cph ^= 1;
        mbar_wait(code_full + cs, cph);
      }
      for (int j = 0; j < 2; ++j) {
        ss ^= 1;
        if (ss == 1) sph ^= 1;
        mbar_wait(sc_full + ss, sph);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ================= MMA issuer (the whole warp loops, lane 0 issues) =================
    uint32_t as = 0, aph = 0, bs = 0, bph = 0, eph0 = 0, eph1 = 0, buf = 0;
    bool ok = true;
    for (int i = blockIdx.x; i < nitems && ok; i += gridDim.x) {
      const Item it = item_of(i, rtiles, maxnt);
      const int cnt = W.grp_count[it.grp];
      if (it.nt * NMAX >= cnt) continue;
      const int ntok = cnt - it.nt * NMAX < NMAX ? cnt - it.nt * NMAX : NMAX;
      const int NT = (ntok + BOXR - 1) / BOXR * BOXR;
      const uint32_t idesc = idesc_f16(NT);
      // the epilogue has read what this buffer held two items ago
      uint32_t& eph = buf ? eph1 : eph0;
      ok = warp_wait(acc_empty + buf, eph ^ 1, abort);
      if (!ok) break;
      eph ^= 1;
      const uint32_t d0 = tmem + buf * acc_cols<MAT>();
      for (int kt = 0; kt < KT; ++kt) {
        ok = warp_wait(a_full + as, aph, abort) && warp_wait(b_full + bs, bph, abort);
        if (!ok) break;
        if (lane == 0) {
          tc_fence_after();
          const uint32_t a0 = tmem + a_base<MAT>() + as * a_cols<MAT>(), b0 = smem_u32(sB + bs * C::B_STAGE);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t bd = sdesc_sw128(b0 + kk * 32);
            const uint32_t acc = kt != 0 || kk != 0;
            tc_mma_ta(d0, a0 + kk * 8, bd, idesc, acc);  // A: 8 columns = 16 fp16 of K per lane (row)
            if (MAT == 0) tc_mma_ta(d0 + NMAX, a0 + BK / 2 + kk * 8, bd, idesc, acc);
          }
          tc_commit(a_empty + as);  // arrives once these MMAs have read the stage
          tc_commit(b_empty + bs);
        }
        __syncwarp();
        if (++as == AST) as = 0, aph ^= 1;
        if (++bs == BST) bs = 0, bph ^= 1;
      }
      if (ok && lane == 0) tc_commit(acc_full + buf);
      __syncwarp();
      buf ^= 1;
    }
    if (lane == 0) {
      tc_commit(mma_done);  // every MMA issued so far has completed
      mbar_wait(mma_done, 0);
    }
    __syncwarp();
  } else if (warp < EPI0) {
    // ================= dequantize into TMEM =================
    // thread t of warp w writes weight row 32 (w % 4) + t (its TMEM lane); the four warps of a lane
    // quarter split the stage's code words: flat word f = sub * WPS + j over [matrix][word of the row]
    const int q4 = warp & 3, sub = (warp - 2) >> 2;  // warps 2..17: four per quarter
    const int r = 32 * q4 + lane;                      // weight row of the tile
    constexpr int WPR = BK * BITS / 32;               // code words per row per stage and matrix: 8 (4-bit), 4 (2-bit)
    constexpr int WPS = C::NMAT * WPR / 4;            // words of a row this thread takes per stage: 4/2 (gate/up), 2/1 (down)
    constexpr int UPW = 16 / BITS;                    // fp16 pairs (TMEM columns) per code word: 4 / 8
    constexpr int NCOL = WPS * UPW;                   // 16 (gate/up) or 8 (down)
    static_assert(NCOL == 16 || NCOL == 8, "one tcgen05.st per stage");
    const int m = (sub * WPS) / WPR, wc0 = (sub * WPS) % WPR;  // the thread's matrix and first word
    const uint32_t lane_addr = tmem + (uint32_t(32 * q4) << 16) + a_base<MAT>() + uint32_t(m * (BK / 2) + wc0 * UPW);
    uint32_t cs = 0, cph = 0, as = 0, aph = 0, ss = 0, sph = 0;
    bool ok = true;
    for (int i = blockIdx.x; i < nitems && ok; i += gridDim.x) {
      const Item it = item_of(i, rtiles, maxnt);
      const int cnt = W.grp_count[it.grp];
      if (it.nt * NMAX >= cnt) continue;
      ok = warp_wait(sc_full + ss, sph, abort);
      if (!ok) break;
      const __half* scl = reinterpret_cast<const __half*>(sS + ss * sc_bytes);
      __half2 s2 = __half2(__float2half_rn(0.0f), __float2half_rn(0.0f)), m2 = s2;
      int gcur = -1;
      for (int kt = 0; kt < KT; ++kt) {
        ok = warp_wait(code_full + cs, cph, abort) && warp_wait(a_empty + as, aph ^ 1, abort);
        if (!ok) break;
        tc_fence_after();  // the MMAs that read this A stage have completed
        const int gcol = kt * BK / S.group;  // the stage's quantization group within the row
        if (gcol != gcur) {  // scale and min stay in registers for the stages of one group
          gcur = gcol;
          const __half sv = scl[((2 * m) * BM + r) * gpr + gcol], mv = scl[((2 * m + 1) * BM + r) * gpr + gcol];
          s2 = __half2(sv, sv);
          m2 = __half2(mv, mv);
        }
        const uint8_t* cst = sC + cs * C::CODE_STAGE + m * C::CODE_MAT + r * C::CODE_ROW + 4 * wc0;
        uint32_t w[WPS];
#pragma unroll
        for (int j = 0; j < WPS; ++j) w[j] = reinterpret_cast<const uint32_t*>(cst)[j];
        uint32_t o[16];
#pragma unroll
        for (int j = 0; j < WPS; ++j)
#pragma unroll
          for (int u = 0; u < UPW; ++u) o[j * UPW + u] = deq2(q_pair<BITS>(w[j], u), s2, m2);
        if (NCOL == 16) tc_st16(lane_addr + as * a_cols<MAT>(), o);
        else tc_st8(lane_addr + as * a_cols<MAT>(), o);
        tc_wait_st();
        tc_fence_before();  // the stores are ordered before the arrival the MMA thread waits on
        __syncwarp();
        if (lane == 0) {
          mbar_arrive1(a_full + as);
          mbar_arrive1(code_empty + cs);
        }
        if (++cs == CST) cs = 0, cph ^= 1;
        if (++as == AST) as = 0, aph ^= 1;
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive1(sc_empty + ss);
      ss ^= 1;
      if (ss == 0) sph ^= 1;
    }
  } else if (warp == BPROD) {
    // ================= activation producer (the whole warp loops, lane 0 issues) =================
    uint32_t bs = 0, bph = 0;
    bool ok = true;
    for (int i = blockIdx.x; i < nitems && ok; i += gridDim.x) {
      const Item it = item_of(i, rtiles, maxnt);
      const int cnt = W.grp_count[it.grp];
      if (it.nt * NMAX >= cnt) continue;
      const int row0 = W.grp_start[it.grp] + it.nt * NMAX;
      const int ntok = cnt - it.nt * NMAX < NMAX ? cnt - it.nt * NMAX : NMAX;
      const int NT = (ntok + BOXR - 1) / BOXR * BOXR;
      for (int kt = 0; kt < KT && ok; ++kt) {
        ok = warp_wait(b_empty + bs, bph ^ 1, abort);
        if (!ok) break;
        if (lane == 0) {
          mbar_expect_tx(b_full + bs, uint32_t(NT * BK * 2));
          for (int j = 0; j < NT / BOXR; ++j)
            tma_load_2d(sB + bs * C::B_STAGE + j * BOXR * BK * 2, &mapB, kt * BK, row0 + j * BOXR, b_full + bs);
        }
        __syncwarp();
        if (++bs == BST) bs = 0, bph ^= 1;
      }
    }
    if (lane == 0) {  // copies in flight land before the CTA can exit
      for (int j = 0; j < BST; ++j) {
        bs = bs == 0 ? BST - 1 : bs - 1;
        if (bs == BST - 1) bph ^= 1;
        mbar_wait(b_full + bs, bph);
      }
    }
    __syncwarp();
  } else {
    // ================= epilogue =================
    const int q4 = warp & 3;  // the TMEM lane quarter this warp may read
    uint32_t eph0 = 0, eph1 = 0, buf = 0;
    bool ok = true;
    for (int i = blockIdx.x; i < nitems && ok; i += gridDim.x) {
      const Item it = item_of(i, rtiles, maxnt);
      const int cnt = W.grp_count[it.grp];
      if (it.nt * NMAX >= cnt) continue;
      const int row0 = W.grp_start[it.grp] + it.nt * NMAX;
      const int ntok = cnt - it.nt * NMAX < NMAX ? cnt - it.nt * NMAX : NMAX;
      const int r0 = it.rt * BM;
      uint32_t& eph = buf ? eph1 : eph0;
      ok = warp_wait(acc_full + buf, eph, abort);
      if (!ok) break;
      eph ^= 1;
      tc_fence_after();
      const int r = r0 + 32 * q4 + lane;  // this thread's weight row (its TMEM lane)
      const uint32_t lane_base = tmem + (uint32_t(32 * q4) << 16) + buf * acc_cols<MAT>();
      const int pr = batched::perm_pos<BITS>(r);
      for (int c0 = 0; c0 < ntok; c0 += 16) {
        uint32_t g[16];
        tc_ld16(lane_base + c0, g);
        if (MAT == 0) {
          uint32_t u[16];
          tc_ld16(lane_base + NMAX + c0, u);
          tc_wait_ld();
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            if (c0 + c < ntok) {
              float a = silu_mul(__uint_as_float(g[c]), __uint_as_float(u[c]));
              if (!(fabsf(a) <= 65504.0f)) {  // outside fp16 (or NaN): saturate and say so
                flag(WISP_STATUS_RANGE);
                a = a != a ? 0.0f : copysignf(65504.0f, a);
              }
              const __half h = __float2half_rn(a);
              ah[int64_t(row0 + c0 + c) * S.I + pr] = *reinterpret_cast<const uint16_t*>(&h);
            }
          }
        } else {
          tc_wait_ld();
#pragma unroll
          for (int c = 0; c < 16; ++c)
            if (c0 + c < ntok) W.y[int64_t(row0 + c0 + c) * S.H + r] = __uint_as_float(g[c]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive1(acc_empty + buf);
      buf ^= 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_cols<MAT>()) : "memory");
  }
}

}  // namespace umma
}  // namespace wisp
