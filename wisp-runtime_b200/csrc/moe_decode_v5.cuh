// Fused MoE decode for one token in one grid, without a grid-wide dependency between gate/up and down.
//
// CTA (j, r) of the k x cs grid owns 8-row blocks [b0, b1) of expert j's intermediate rows, i.e. the
// values a_j[i0..i1) = silu(g) * u of those rows, and right away the contribution of exactly those
// values to every output row: y_{j,r}[h] = w_j * sum_{i in [i0, i1)} Wd_j[h, i] a_j[i].  So nothing
// waits for another CTA's a, and a small combine grid sums the k * cs partial vectors in a fixed
// order (out = bf16(sum)).  Everything a CTA reads is requested at its start:
//   gate/up  one region per block: 8 gate rows + the same 8 up rows (two contiguous bulk copies, no
//            multicast) and four scale/min windows, on the block's mbarrier (the v4 region layout);
//   down     the strided column slice: for every output row h the 16-byte-aligned window holding
//            codes i0..i1 of row h (plain 16-byte loads), plus the scale/min of the one or two
//            quantization groups the slice touches.
// gate/up math is the v4 integer MMA (u8 codes x int8 activation limbs, exact int32 sums, two warps
// per block for the K halves).  The down slice is short (I / cs codes per row), so it runs on the CUDA
// cores: per row sum_i q_i a_i per group, then s * dot + m * sum(a) (the dequant fold).
//
// The plan (cs, blocks per CTA, window width, shared-memory layout) is computed on the host and on
// the device by the same function; a shape whose plan does not fit uses the two-kernel path.
#pragma once
#include "common.cuh"
#include "moe_decode.cuh"
#include "moe_decode_v4.cuh"
#include "tma.cuh"
#include "unpack_imma.cuh"

namespace wisp {
namespace v5 {

constexpr int WARPS = 16;
constexpr int THREADS = WARPS * 32;
constexpr int CH = 8;
constexpr int MAX_BLOCKS = 8;  // two warps per block
constexpr int SMEM_LIMIT = 220 * 1024;

struct Plan {
  int cs, nb_max, dsw, groups, gph, gpr;
  int64_t row_bytes, sc_win, region;
  int64_t off_bx, off_gsum, off_zero, off_halves, off_bars, off_route, off_a, off_dn, off_dsc, bytes;
  bool ok;
};

// blocks [b0, b1) of CTA r (of cs) over an expert's I / CH blocks
__host__ __device__ inline void cta_blocks(int I, int cs, int r, int& b0, int& b1) {
  const int nblk = I / CH;
  b0 = int(int64_t(nblk) * r / cs);
  b1 = int(int64_t(nblk) * (r + 1) / cs);
}

__host__ __device__ inline Plan plan(int H, int I, int k, int group, int bits, int nsms) {
  Plan P;
  P.ok = false;
  int cs = nsms / (k > 0 ? k : 1);
  if (cs > I / CH) cs = I / CH;
  P.cs = cs;
  if (cs < 1) return P;
  P.nb_max = (I / CH + cs - 1) / cs;
  // the down slice window: 16-byte-aligned bytes covering codes [i0, i1) of one row, widest CTA
  int dsw = 0;
  for (int r = 0; r < cs; ++r) {
    int b0, b1;
    cta_blocks(I, cs, r, b0, b1);
    const int bs = b0 * CH * bits / 8, be = b1 * CH * bits / 8;
    const int w = int(ru16(be) - (bs & ~15));
    dsw = w > dsw ? w : dsw;
  }
  P.dsw = dsw;
  P.groups = H / 128;
  P.gph = (P.groups + 1) / 2;
  P.gpr = H / group;
  P.row_bytes = int64_t(H) * bits / 8;
  P.sc_win = ru16(int64_t(CH) * P.gpr * 2) + 16;
  P.region = ru16(2 * CH * P.row_bytes + 4 * P.sc_win);
  P.off_bx = int64_t(P.nb_max) * P.region;                      // [H/32 units][3 limbs][8] u32
  P.off_gsum = ru16(P.off_bx + int64_t(H / 32) * 24 * 4);       // [H/128][2] f32
  P.off_zero = ru16(P.off_gsum + int64_t(P.groups) * 2 * 4);    // 64 zero bytes
  P.off_halves = ru16(P.off_zero + 64);                         // [nb_max][2][CH][2] f32
  P.off_bars = ru16(P.off_halves + int64_t(P.nb_max) * 2 * CH * 2 * 4);
  P.off_route = ru16(P.off_bars + 8 * int64_t(P.nb_max));
  P.off_a = ru16(P.off_route + v4::ROUTE_BYTES);                // [nb_max * CH] f32 a, then 2 group sums
  P.off_dn = ru16(P.off_a + (int64_t(P.nb_max) * CH + 2) * 4);  // [H][dsw] down code windows
  P.off_dsc = ru16(P.off_dn + int64_t(H) * dsw);                // [H][4] f16: sA, mA, sB, mB
  P.bytes = P.off_dsc + int64_t(H) * 8;
  // a slice of at most one group boundary (cols <= group), two warps per block, and the memory budget
  P.ok = P.nb_max <= MAX_BLOCKS && P.nb_max * CH <= group && P.bytes <= SMEM_LIMIT;
  return P;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <int BITS>
__device__ __forceinline__ uint32_t slice_word(const uint8_t* p, int m) {  // bytes of codes [8m, 8m + 8)
  if constexpr (BITS == 4) return *reinterpret_cast<const uint32_t*>(p + 4 * m);
  else if constexpr (BITS == 2) return *reinterpret_cast<const uint16_t*>(p + 2 * m);
  else return uint32_t(p[3 * m]) | (uint32_t(p[3 * m + 1]) << 8) | (uint32_t(p[3 * m + 2]) << 16);
}

template <int BITS, bool PAGED>
__global__ void __launch_bounds__(THREADS, 1) fused_kernel(const uint8_t* __restrict__ pool, const float* __restrict__ meta,
                                                           const uint16_t* __restrict__ x, MoeShape S, Plan P,
                                                           float* __restrict__ partial, MoeRoute RT) {
  extern __shared__ __align__(128) uint8_t sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int j = blockIdx.x / P.cs, r = blockIdx.x - j * P.cs;
  int b0, b1;
  cta_blocks(S.I, P.cs, r, b0, b1);
  const int nb = b1 - b0, i0 = b0 * CH, i1 = b1 * CH;
  uint32_t* bx = reinterpret_cast<uint32_t*>(sm + P.off_bx);
  float* gsum = reinterpret_cast<float*>(sm + P.off_gsum);
  const uint32_t* zero = reinterpret_cast<const uint32_t*>(sm + P.off_zero);
  float* halves = reinterpret_cast<float*>(sm + P.off_halves);
  uint64_t* gbar = reinterpret_cast<uint64_t*>(sm + P.off_bars);
  float* av = reinterpret_cast<float*>(sm + P.off_a);
  uint8_t* dn = sm + P.off_dn;
  uint16_t* dsc = reinterpret_cast<uint16_t*>(sm + P.off_dsc);
  const int64_t ngm = S.ng / 3;
  const int glog = 7 + S.gshift;  // group = 128 * 2^gshift

  pdl_wait();  // routing and x come from earlier kernels in the stream
  pdl_launch_dependents();
  const float* mt = meta;
  if (RT.logits) {
    float* rs = reinterpret_cast<float*>(sm + P.off_route);
    route_from_logits<true>(RT, S.k, rs, rs + 64, rs + 96);
    mt = rs;
  }
  const float f = RT.logits ? mt[j] : __ldg(meta + j);
  const float wj = RT.logits ? mt[S.k + j] : __ldg(meta + S.k + j);
  bool host;  // PAGED: a non-resident expert is read from the mapped host store (plain loads, no TMA)
  const uint8_t* base = v4::src_of<PAGED>(f, S, pool, RT, host);
  const bool ok = base != nullptr;
  if (!ok && r == 0 && threadIdx.x == 0) flag(WISP_STATUS_BAD_SLOT);  // skipped: contributes nothing
  if (PAGED && host && r == 0 && threadIdx.x == 0 && RT.miss_count) atomicAdd(RT.miss_count, 1);

  // ---- gate/up blocks: warp 2b issues block b into region b (lanes 0-5), as the two-kernel path
  const uint32_t cb = uint32_t(CH * P.row_bytes);
  if (warp < 2 * nb && (warp & 1) == 0) {
    const int bi = warp >> 1, row0 = (b0 + bi) * CH;
    uint8_t* reg = sm + int64_t(bi) * P.region;
    if (lane == 0) {
      mbar_init(&gbar[bi], 1);
      mbar_fence_init();
    }
    __syncwarp();
    if (PAGED && host) {  // the same ranges with warp copies, then one arrival
      warp_copy_g2s(reg, base + int64_t(row0) * P.row_bytes, cb, lane);
      warp_copy_g2s(reg + cb, base + S.mat_bytes + int64_t(row0) * P.row_bytes, cb, lane);
      for (int arr = 0; arr < 4; ++arr) {
        const Win w = window(S.ncode + 2 * ((arr & 1) * S.ng + (arr >> 1) * ngm + int64_t(row0) * P.gpr), 2 * CH * P.gpr);
        warp_copy_g2s(reg + 2 * cb + arr * P.sc_win, base + w.start, w.bytes, lane);
      }
      __syncwarp();
      if (lane == 0) mbar_expect_tx(&gbar[bi], 0);
    } else if (lane == 0) {
      uint32_t tx = 0;
      if (ok) {
        tx = 2 * cb;
        for (int arr = 0; arr < 4; ++arr)
          tx += window(S.ncode + 2 * ((arr & 1) * S.ng + (arr >> 1) * ngm + int64_t(row0) * P.gpr), 2 * CH * P.gpr).bytes;
      }
      mbar_expect_tx(&gbar[bi], tx);
    }
    __syncwarp();
    if (ok && !(PAGED && host) && lane < 6) {
      if (lane < 2) {
        bulk_g2s(reg + lane * cb, base + lane * S.mat_bytes + int64_t(row0) * P.row_bytes, cb, &gbar[bi]);
      } else {
        const int arr = lane - 2;
        const Win w = window(S.ncode + 2 * ((arr & 1) * S.ng + (arr >> 1) * ngm + int64_t(row0) * P.gpr), 2 * CH * P.gpr);
        bulk_g2s(reg + 2 * cb + arr * P.sc_win, base + w.start, w.bytes, &gbar[bi]);
      }
    }
  }

  // ---- B operand from x, all threads (one per 32-element unit)
  const int units = S.H / 32;
  for (int ub = int(threadIdx.x) & ~31; ub < units; ub += blockDim.x) {
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
    const int e = v4::store_b_limbs<BITS>(v, bx + u * 24, u < units);
    float sx = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) sx += v[i];
    sx = v4::quad_sum(u < units ? sx : 0.0f);
    if (u < units && (u & 3) == 0) {
      gsum[2 * (u >> 2)] = sx;
      gsum[2 * (u >> 2) + 1] = pow2(-e);
    }
  }
  // ---- down slice: row h's window of codes [i0, i1) (asynchronous 16-byte copies into shared
  //      memory, waited for before the down step) and the scales/mins of its one or two groups
  const int64_t drow = int64_t(S.I) * BITS / 8;
  const int bs = i0 * BITS / 8;
  const int ws = bs & ~15, wn = int(ru16(i1 * BITS / 8) - ws) / 16;  // 16-byte chunks per row window
  const int ncross = ((i0 >> glog) != ((i1 - 1) >> glog)) ? 1 : 0;   // the slice crosses a group boundary
  if (ok) {
    const uint16_t* scl = reinterpret_cast<const uint16_t*>(base + S.ncode);
    if (PAGED && host) {
      for (int h = threadIdx.x; h < S.H; h += blockDim.x) {
        const uint8_t* src = base + 2 * S.mat_bytes + int64_t(h) * drow + ws;
        uint4* dst = reinterpret_cast<uint4*>(dn + int64_t(h) * P.dsw);
        for (int q = 0; q < wn; ++q) dst[q] = *reinterpret_cast<const uint4*>(src + 16 * q);
        const int64_t gA = (2 * int64_t(S.H) * S.I + int64_t(h) * S.I + i0) >> glog;
        dsc[4 * h] = scl[gA];
        dsc[4 * h + 1] = scl[S.ng + gA];
        dsc[4 * h + 2] = ncross ? scl[gA + 1] : uint16_t(0);
        dsc[4 * h + 3] = ncross ? scl[S.ng + gA + 1] : uint16_t(0);
      }
    } else {
      for (int i = threadIdx.x; i < S.H * wn; i += blockDim.x) {
        const int h = i / wn, q = i - h * wn;
        cp_async16(dn + int64_t(h) * P.dsw + 16 * q, base + 2 * S.mat_bytes + int64_t(h) * drow + ws + 16 * q);
      }
      cp_async_commit();
      // scales and mins: every load of this thread's rows issued before any store
      constexpr int MAXR = 8;  // rows per thread (H <= 4096 with 512 threads)
      uint16_t sv[MAXR][4];
#pragma unroll
      for (int m = 0; m < MAXR; ++m) {
        const int h = int(threadIdx.x) + m * int(blockDim.x);
        if (h < S.H) {
          const int64_t gA = (2 * int64_t(S.H) * S.I + int64_t(h) * S.I + i0) >> glog;
          sv[m][0] = ld_nc_u16(scl + gA);
          sv[m][1] = ld_nc_u16(scl + S.ng + gA);
          sv[m][2] = ncross ? ld_nc_u16(scl + gA + 1) : uint16_t(0);
          sv[m][3] = ncross ? ld_nc_u16(scl + S.ng + gA + 1) : uint16_t(0);
        }
      }
#pragma unroll
      for (int m = 0; m < MAXR; ++m) {
        const int h = int(threadIdx.x) + m * int(blockDim.x);
        if (h < S.H) *reinterpret_cast<uint2*>(dsc + 4 * h) = make_uint2(uint32_t(sv[m][0]) | (uint32_t(sv[m][1]) << 16),
                                                                         uint32_t(sv[m][2]) | (uint32_t(sv[m][3]) << 16));
      }
    }
  }

  if (threadIdx.x < 16) reinterpret_cast<uint32_t*>(sm + P.off_zero)[threadIdx.x] = 0u;
  __syncthreads();

  // ---- gate/up: warp (2b + hf) computes K half hf of block b (the v4 math)
  if (warp < 2 * nb) {
    const int bi = warp >> 1, hf = warp & 1;
    const uint8_t* reg = sm + int64_t(bi) * P.region;
    const int G0 = hf * P.gph;
    const int ng = min(P.gph, P.groups - G0);
    const int sarr = c == 1 ? 2 : 0;
    const int row0 = (b0 + bi) * CH;
    const uint32_t sskip = window(S.ncode + 2 * ((sarr >> 1) * ngm + int64_t(row0) * P.gpr), 1).skip;
    const uint32_t mskip = window(S.ncode + 2 * (S.ng + (sarr >> 1) * ngm + int64_t(row0) * P.gpr), 1).skip;
    const uint8_t* sw = reg + 2 * int64_t(cb);
    const uint16_t* srow = reinterpret_cast<const uint16_t*>(sw + sarr * P.sc_win + sskip) + g * P.gpr;
    const uint16_t* mrow = reinterpret_cast<const uint16_t*>(sw + (sarr + 1) * P.sc_win + mskip) + g * P.gpr;
    const uint8_t* rowg = reg + g * P.row_bytes;
    const uint8_t* rowu = reg + cb + g * P.row_bytes;
    mbar_wait(&gbar[bi], 0);
    float acc = 0.0f;
    for (int G = 0; G < ng; G += 2) {
      if (!ok) break;
      const int Ga = G0 + G, Gb = G0 + min(G + 1, ng - 1);
      uint32_t wa0[BITS], wb0[BITS], wa1[BITS], wb1[BITS], bb0[8], bb1[8];
      v4::lds_unit<BITS>(rowg + (Ga * 4 + c) * 4 * BITS, wa0);
      v4::lds_unit<BITS>(rowu + (Ga * 4 + c) * 4 * BITS, wb0);
      v4::lds_unit<BITS>(rowg + (Gb * 4 + c) * 4 * BITS, wa1);
      v4::lds_unit<BITS>(rowu + (Gb * 4 + c) * 4 * BITS, wb1);
      v4::lds_b8(g < 3 ? bx + ((4 * Ga + c) * 3 + g) * 8 : zero, bb0);
      v4::lds_b8(g < 3 ? bx + ((4 * Gb + c) * 3 + g) * 8 : zero, bb1);
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
    if (c < 2) halves[((bi * 2 + hf) * CH + g) * 2 + c] = acc;
  }
  __syncthreads();
  // SwiGLU of this CTA's rows (K halves in a fixed order)
  for (int t = threadIdx.x; t < nb * CH; t += blockDim.x) {
    const int bi = t / CH, rw = t - bi * CH;
    const float gs = halves[((bi * 2) * CH + rw) * 2] + halves[((bi * 2 + 1) * CH + rw) * 2];
    const float us = halves[((bi * 2) * CH + rw) * 2 + 1] + halves[((bi * 2 + 1) * CH + rw) * 2 + 1];
    av[t] = ok ? silu_mul(gs, us) : 0.0f;
  }
  __syncthreads();
  // sums of a over the slice's first group (columns < nA) and the rest, fixed order
  const int nA = ncross ? ((((i0 >> glog) + 1) << glog) - i0) : (i1 - i0);
  float* asum = av + P.nb_max * CH;
  cp_async_wait_all();  // this thread's slice copies (none for a skipped or host-read expert)
  if (warp == 0) {
    float sa = 0.0f, sb = 0.0f;
    for (int t = lane; t < i1 - i0; t += 32) (t < nA ? sa : sb) += av[t];
    sa = warp_sum(sa);
    sb = warp_sum(sb);
    if (lane == 0) {
      asum[0] = sa;
      asum[1] = sb;
    }
  }
  __syncthreads();

  // ---- down slice: y[h] = w_j * (sA * sum_{i<nA} q_i a_i + mA * SA + sB * sum_{i>=nA} q_i a_i + mB * SB)
  const float SA = asum[0], SB = asum[1];
  const int boff = bs - ws;      // byte offset of column i0 in the row window
  const int nwords = (i1 - i0) / 8;
  float* out = partial + int64_t(blockIdx.x) * S.H;
  for (int h = threadIdx.x; h < S.H; h += blockDim.x) {
    float y = 0.0f;
    if (ok) {
      const uint8_t* p = dn + int64_t(h) * P.dsw + boff;
      float da = 0.0f, db = 0.0f;
      for (int m = 0; m < nwords; ++m) {
        const uint32_t wv = slice_word<BITS>(p, m);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int col = 8 * m + q;
          const float prod = small_u2f((wv >> (BITS * q)) & ((1u << BITS) - 1u)) * av[col];
          if (col < nA) da += prod;
          else db += prod;
        }
      }
      y = f16_bits_to_f32(dsc[4 * h]) * da + f16_bits_to_f32(dsc[4 * h + 1]) * SA;
      if (ncross) y += f16_bits_to_f32(dsc[4 * h + 2]) * db + f16_bits_to_f32(dsc[4 * h + 3]) * SB;
      y *= wj;
    }
    out[h] = y;
  }
  // no copy may still be landing in shared memory when the CTA retires (a skipped expert has none)
  if (warp < 2 * nb && (warp & 1) == 0 && lane == 0) mbar_wait(&gbar[warp >> 1], 0);
}

// out[h] = bf16(sum over the nparts partial vectors in order); one warp per 32 outputs per CTA slice
__global__ void combine_kernel(const float* __restrict__ partial, int nparts, int64_t H, uint16_t* __restrict__ out) {
  __shared__ float red[8][32];
  pdl_wait();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int64_t h0 = int64_t(blockIdx.x) * 32; h0 < H; h0 += int64_t(gridDim.x) * 32) {
    const int64_t h = h0 + lane;
    float s = 0.0f;
    if (h < H)
      for (int b = warp; b < nparts; b += 8) s += partial[int64_t(b) * H + h];  // partials b = warp (mod 8), in order
    red[warp][lane] = s;
    __syncthreads();
    if (warp == 0 && h < H) {
      float t = 0.0f;
#pragma unroll
      for (int w = 0; w < 8; ++w) t += red[w][lane];
      out[h] = f32_to_bf16(t);
    }
    __syncthreads();
  }
}

}  // namespace v5
}  // namespace wisp
