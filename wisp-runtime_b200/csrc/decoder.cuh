// Decode-step kernels around the projections and the MoE, for one token:
//   qk_norm_rope_kv  per-head RMSNorm of q and k, rotary at the token's position, K/V written into
//                    the static cache at that position (wisp/graphdec.py:160-168)
//   attn_split       GQA decode attention over positions [0, pos], split into chunks of CHUNK
//   attn_combine     merge of the chunk partials (log-sum-exp), bf16 out
//   router_topk      softmax (fp32) -> top-k -> renormalise -> bf16 weights; writes the routing row
//                    and the MoE meta buffer (wisp/graphdec.py:177-181, wisp/moe.py:67-72)
//   embed            token row of the embedding table
//   argmax_partial / argmax_final   greedy next token over the logits
// The position and the token are read from device memory, so one captured graph serves every step.
#pragma once
#include "common.cuh"
#include "dense.cuh"
#include "tma.cuh"

namespace wisp {
namespace dec {
using dense::bf_hi;
using dense::bf_lo;

constexpr int CHUNK = 64;       // positions per attention CTA
constexpr int ATTN_THREADS = 128;
constexpr int QK_MAX_D = 256;   // head_dim limit of the norm/rotary kernel
constexpr int MAX_D = 128;      // head_dim limit of the attention kernels
constexpr int MAX_G = 8;        // query heads per KV head (attention)

// ---- per-head RMSNorm + rotary + cache write -----------------------------------------------------
// qkv: per token [Hq*D | Hk*D | Hk*D] bf16 (q heads, k heads, v heads), token t at qkv + t*qkv_stride.
// One warp per head; grid y = token t, at position pos_ptr[t * pos_step] + t * pos_inc, writing the
// caches at kc/vc + t * kv_bstride; its q goes to q_out + t*Hq*D.  One token per decode step
// (pos_step 0); a chunk of one sequence's prompt (pos_step 0, pos_inc 1); one token of each of
// several sequences (pos_step 1, pos_inc 0, kv_bstride = one sequence's cache).  qn_w == nullptr:
// no per-head RMSNorm (models without q/k norms).
// One warp, one head of D values: optional RMSNorm (HF: weight * bf16(x * rsqrt(mean(x^2) + eps)),
// rounded to bf16) then rotate-half rotary in fp32 with one rounding per element (no FMA contraction),
// into dst (bf16 [D], shared or global memory).  x: fp32 scratch [D] of this warp.
__device__ __forceinline__ void norm_rope_warp(const uint16_t* __restrict__ src, const uint16_t* __restrict__ w, float eps,
                                               const uint16_t* __restrict__ cs, const uint16_t* __restrict__ sn, int D, int lane,
                                               float* x, uint16_t* dst) {
  float ss = 0.0f;
  for (int i = lane; i < D; i += 32) {
    const float v = bf16_to_f32(src[i]);
    x[i] = v;
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / float(D) + eps);
  __syncwarp();
  if (w)
    for (int i = lane; i < D; i += 32) x[i] = bf16_to_f32(f32_to_bf16(bf16_to_f32(w[i]) * bf16_to_f32(f32_to_bf16(x[i] * inv))));
  __syncwarp();
  const int half = D / 2;
  for (int i = lane; i < D; i += 32) {
    const float xp = i < half ? -x[i + half] : x[i - half];
    dst[i] = f32_to_bf16(__fadd_rn(__fmul_rn(x[i], bf16_to_f32(cs[i])), __fmul_rn(xp, bf16_to_f32(sn[i]))));
  }
  __syncwarp();
}

__global__ void qk_norm_rope_kv_kernel(const uint16_t* __restrict__ qkv, int Hq, int Hk, int D,
                                       const uint16_t* __restrict__ qn_w, const uint16_t* __restrict__ kn_w, float eps,
                                       const uint16_t* __restrict__ cos_t, const uint16_t* __restrict__ sin_t,
                                       const int64_t* __restrict__ pos_ptr, int64_t tmax, uint16_t* __restrict__ q_out,
                                       uint16_t* __restrict__ kc, uint16_t* __restrict__ vc, int64_t qkv_stride, int pos_step,
                                       int pos_inc, int64_t kv_bstride) {
  __shared__ float xs[8][QK_MAX_D];
  const int wib = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.x * (blockDim.x >> 5) + wib;
  pdl_wait();
  pdl_launch_dependents();
  if (head >= Hq + 2 * Hk) return;
  const int64_t pos = pos_ptr[int64_t(blockIdx.y) * pos_step] + int64_t(blockIdx.y) * pos_inc;
  if (pos < 0 || pos >= tmax) {
    if (lane == 0 && head == 0) flag(WISP_STATUS_BAD_POS);
    return;
  }
  qkv += int64_t(blockIdx.y) * qkv_stride;
  q_out += int64_t(blockIdx.y) * Hq * D;
  kc += int64_t(blockIdx.y) * kv_bstride;
  vc += int64_t(blockIdx.y) * kv_bstride;
  const uint16_t* src = qkv + int64_t(head) * D;
  if (head >= Hq + Hk) {  // v: straight into the cache
    const int hv = head - Hq - Hk;
    uint16_t* dst = vc + (int64_t(hv) * tmax + pos) * D;
    for (int i = lane; i < D; i += 32) dst[i] = src[i];
    return;
  }
  const bool is_q = head < Hq;
  uint16_t* dst = is_q ? q_out + int64_t(head) * D : kc + (int64_t(head - Hq) * tmax + pos) * D;
  norm_rope_warp(src, is_q ? qn_w : kn_w, eps, cos_t + pos * D, sin_t + pos * D, D, lane, xs[wib], dst);
}

// ---- attention: chunk partials --------------------------------------------------------------------
// grid (Hk, tmax / CHUNK): CTA (h, c) covers positions [c*CHUNK, min((c+1)*CHUNK, pos+1)) for the
// G = Hq/Hk query heads of KV head h.  Partial record per (h, c, g): D unnormalised outputs, then
// the running max and the sum of exponentials.
// grid (Hk, chunks, batch): sequence b = blockIdx.z has its query at q + b*Hq*D, its caches at
// kc/vc + b*kv_bstride and its position at pos_ptr[b]; window > 0 keeps only positions
// (pos - window, pos] (sliding-window attention).  Records: part[((b*Hk + h)*chunks + c)*G + g].
__device__ __forceinline__ int64_t window_lo(int64_t pos, int window) {
  return window > 0 && pos - window + 1 > 0 ? pos - window + 1 : 0;
}
// floats per chunk record: D outputs, the maximum, the sum, two pad floats (records start 16-byte aligned)
__host__ __device__ constexpr int rec_floats(int D) { return D + 4; }

__global__ void __launch_bounds__(ATTN_THREADS) attn_split_kernel(const uint16_t* __restrict__ q, int Hq, int Hk, int D,
                                                                  const uint16_t* __restrict__ kc,
                                                                  const uint16_t* __restrict__ vc, int64_t tmax,
                                                                  const int64_t* __restrict__ pos_ptr, float scale,
                                                                  float* __restrict__ part, int64_t kv_bstride, int window) {
  // the chunk's K and V rows are contiguous in the cache ([Hk, tmax, D] per sequence): both are copied
  // into shared memory first with 16-byte loads all in flight at once, so the score and P V loops
  // below wait on shared-memory latency instead of one dependent HBM load per position
  __shared__ __align__(16) uint16_t kvs[2][CHUNK * MAX_D];
  __shared__ __align__(16) float qs[MAX_G][MAX_D];
  __shared__ float ps[MAX_G][CHUNK];
  // per-warp P V sums, lane-major; they reuse the K rows, which are dead once the scores are taken
  static_assert(sizeof(float) * (ATTN_THREADS / 32) * MAX_G * MAX_D <= sizeof(uint16_t) * CHUNK * MAX_D, "red fits in K");
  float (*red)[MAX_G][MAX_D] = reinterpret_cast<float (*)[MAX_G][MAX_D]>(&kvs[0][0]);
  const int h = blockIdx.x, c = blockIdx.y, b = blockIdx.z;
  const int G = Hq / Hk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = ATTN_THREADS / 32;
  pdl_wait();
  pdl_launch_dependents();
  const int64_t pos = pos_ptr[b];
  if (pos < 0 || pos >= tmax) return;  // flagged by the cache-write kernel
  const int64_t lo = window_lo(pos, window);
  const int64_t t0 = int64_t(c) * CHUNK > lo ? int64_t(c) * CHUNK : lo;
  if (t0 > pos || t0 >= int64_t(c + 1) * CHUNK) return;  // outside [lo, pos]: the combine never reads this record
  const int n = int((pos + 1 - t0) < int64_t(c + 1) * CHUNK - t0 ? (pos + 1 - t0) : int64_t(c + 1) * CHUNK - t0);
  q += int64_t(b) * Hq * D;
  kc += int64_t(b) * kv_bstride;
  vc += int64_t(b) * kv_bstride;
  part += int64_t(b) * Hk * gridDim.y * G * rec_floats(D);
  {
    const uint4* kg = reinterpret_cast<const uint4*>(kc + (int64_t(h) * tmax + t0) * D);
    const uint4* vg = reinterpret_cast<const uint4*>(vc + (int64_t(h) * tmax + t0) * D);
    uint4* ks4 = reinterpret_cast<uint4*>(&kvs[0][0]);
    uint4* vs4 = reinterpret_cast<uint4*>(&kvs[1][0]);
    const int nv = n * D / 8;  // 16-byte pieces of n rows (D % 32 == 0)
    constexpr int PER = CHUNK * MAX_D / 8 / ATTN_THREADS;
    uint4 kr[PER], vr[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int i = threadIdx.x + j * ATTN_THREADS;
      if (i < nv) {
        kr[j] = kg[i];
        vr[j] = vg[i];
      }
    }
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int i = threadIdx.x + j * ATTN_THREADS;
      if (i < nv) {
        ks4[i] = kr[j];
        vs4[i] = vr[j];
      }
    }
  }
  // q of the G heads, pre-scaled, fp32
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) qs[i / D][i % D] = bf16_to_f32(q[(int64_t(h) * G) * D + i]) * scale;
  __syncthreads();
  const uint16_t* kb = &kvs[0][0];
  const uint16_t* vb = &kvs[1][0];
  const int dpl = D / 32;  // elements of a row per lane (D % 32 == 0, D <= MAX_D)
  // scores: each thread takes whole dot products, positions lane, lane + 32 and heads warp, warp + 4, ...
  // (no cross-lane reductions on the critical path); lane l starts its row at word l, so the lanes of a
  // warp read distinct banks of their different rows
  {
    const int hw = D / 2;  // 32-bit words (bf16 pairs) of a row
    for (int g = warp; g < G; g += nw) {
      const float2* qg = reinterpret_cast<const float2*>(&qs[g][0]);
#pragma unroll
      for (int i = 0; i < CHUNK / 32; ++i) {
        const int t = lane + 32 * i;
        if (t < n) {
          const uint32_t* kr = reinterpret_cast<const uint32_t*>(kb + t * D);
          float s0 = 0.0f, s1 = 0.0f;
          int j = lane % hw;
#pragma unroll 8
          for (int c = 0; c < hw; ++c) {
            const uint32_t kv = kr[j];
            const float2 qv = qg[j];
            s0 = fmaf(qv.x, bf_lo(kv), s0);
            s1 = fmaf(qv.y, bf_hi(kv), s1);
            j = j + 1 == hw ? 0 : j + 1;
          }
          ps[g][t] = s0 + s1;
        }
      }
    }
  }
  __syncthreads();
  // softmax within the chunk: warp w takes heads w, w + 4, ...
  for (int g = warp; g < G; g += nw) {
    float m = -INFINITY;
    for (int t = lane; t < n; t += 32) m = fmaxf(m, ps[g][t]);
    m = warp_max(m);
    float l = 0.0f;
    for (int t = lane; t < n; t += 32) {
      const float p = __expf(ps[g][t] - m);
      ps[g][t] = p;
      l += p;
    }
    l = warp_sum(l);
    if (lane == 0) {
      float* rec = part + ((int64_t(h) * gridDim.y + c) * G + g) * rec_floats(D);
      rec[D] = m;
      rec[D + 1] = l;
    }
  }
  __syncthreads();
  // P V: warp w accumulates positions w, w + 4, ... for all heads; lanes split the row
  float acc[MAX_G][MAX_D / 32];
#pragma unroll
  for (int g = 0; g < MAX_G; ++g)
#pragma unroll
    for (int e = 0; e < MAX_D / 32; ++e) acc[g][e] = 0.0f;
  for (int t = warp; t < n; t += nw) {
    float vv[MAX_D / 32];
#pragma unroll
    for (int e = 0; e < MAX_D / 32; ++e) vv[e] = e < dpl ? bf16_to_f32(vb[t * D + lane * dpl + e]) : 0.0f;
#pragma unroll
    for (int g = 0; g < MAX_G; ++g) {
      if (g < G) {
        const float p = ps[g][t];
#pragma unroll
        for (int e = 0; e < MAX_D / 32; ++e) acc[g][e] = fmaf(p, vv[e], acc[g][e]);
      }
    }
  }
#pragma unroll
  for (int g = 0; g < MAX_G; ++g)
#pragma unroll
    for (int e = 0; e < MAX_D / 32; ++e) red[warp][g][lane * (MAX_D / 32) + e] = acc[g][e];
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    const int ln = d / dpl, e = d % dpl;
    float s = 0.0f;
    for (int w = 0; w < nw; ++w) s += red[w][g][ln * (MAX_D / 32) + e];
    part[((int64_t(h) * gridDim.y + c) * G + g) * rec_floats(D) + d] = s;
  }
}

// one CTA per (query head, sequence): out = sum_c O_c e^(m_c - M) / (sum_c l_c e^(m_c - M) [+ e^(sink - M)]);
// sinks (fp32 [Hq], nullable) are per-head logits that take part in the softmax's normalisation but
// contribute no value (attention sinks).  One pass over the records: warp w merges chunks c0 + w,
// c0 + w + 4, ... with a running maximum (each lane holds D / 32 outputs, loaded as float4 / float2 from
// 16-byte aligned records), and the warps' states are merged in a fixed order, so the result does not
// depend on scheduling.
constexpr int CMB_THREADS = 128;
__global__ void __launch_bounds__(CMB_THREADS) attn_combine_kernel(const float* __restrict__ part, int Hq, int Hk, int D,
                                                                   int nchunk_max, const int64_t* __restrict__ pos_ptr, int64_t tmax,
                                                                   uint16_t* __restrict__ out, int window,
                                                                   const float* __restrict__ sinks, int chunk) {
  constexpr int NW = CMB_THREADS / 32;
  __shared__ float wm[NW], wl[NW];
  __shared__ float osum[NW][MAX_D];
  const int head = blockIdx.x, b = blockIdx.y;
  const int G = Hq / Hk, h = head / G, g = head % G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();
  pdl_launch_dependents();
  const int64_t pos = pos_ptr[b];
  if (pos < 0 || pos >= tmax) return;
  const int rs = rec_floats(D);
  part += int64_t(b) * Hk * nchunk_max * G * rs;
  out += int64_t(b) * Hq * D;
  const int c0 = int(window_lo(pos, window) / chunk), nc = int(pos / chunk) + 1;  // chunk: positions per record
  const float* rec0 = part + (int64_t(h) * nchunk_max * G + g) * rs;  // record of chunk c: rec0 + c * G * rs
  const int dpl = D / 32;  // outputs per lane: 1, 2, 3 or 4
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  float m = -INFINITY, l = 0.0f;
#pragma unroll 4
  for (int c = c0 + warp; c < nc; c += NW) {
    const float* rec = rec0 + int64_t(c) * G * rs;
    const float2 ml = *reinterpret_cast<const float2*>(rec + D);
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (dpl == 4) {
      const float4 t = reinterpret_cast<const float4*>(rec)[lane];
      v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
    } else if (dpl == 2) {
      const float2 t = reinterpret_cast<const float2*>(rec)[lane];
      v[0] = t.x, v[1] = t.y;
    } else {
      for (int e = 0; e < dpl; ++e) v[e] = rec[lane * dpl + e];
    }
    const float mn = fmaxf(m, ml.x);
    const float so = __expf(m - mn), sc = __expf(ml.x - mn);  // m = -inf at the first chunk: so = 0
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[e] = acc[e] * so + v[e] * sc;
    l = l * so + ml.y * sc;
    m = mn;
  }
  if (lane == 0) wm[warp] = m, wl[warp] = l;
#pragma unroll
  for (int e = 0; e < 4; ++e)
    if (e < dpl) osum[warp][lane * dpl + e] = acc[e];
  __syncthreads();
  float M = sinks ? sinks[head] : -INFINITY;
#pragma unroll
  for (int w = 0; w < NW; ++w) M = fmaxf(M, wm[w]);
  float L = sinks ? __expf(sinks[head] - M) : 0.0f;
  float f[NW];
#pragma unroll
  for (int w = 0; w < NW; ++w) {
    f[w] = wm[w] == -INFINITY ? 0.0f : __expf(wm[w] - M);  // a warp with no chunk contributes nothing
    L += wl[w] * f[w];
  }
  for (int d = threadIdx.x; d < D; d += CMB_THREADS) {
    float o = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; ++w) o += osum[w][d] * f[w];
    out[int64_t(head) * D + d] = f32_to_bf16(o / L);
  }
}

// ---- fused decode attention: one cluster of CTAs per KV head --------------------------------------
// Per-head RMSNorm + rotary of the G query heads and of the new key (the arithmetic of
// qk_norm_rope_kv_kernel), the new K/V row written into the cache at *pos, then attention over
// positions [0, *pos]: CTA r of the cluster takes the r-th slice of the positions and streams it
// through shared memory in chunks of FCHUNK.  Scores and P.V run on the tensor cores (mma.sync
// m16n8k16 bf16, fp32 accumulation; the G query heads are rows 0..G-1 of the 16-row A tile), softmax
// is online in fp32 on log2-scaled scores, and the per-CTA partial states are merged through
// distributed shared memory: CTA r finishes one (head, half of D) piece of the output.
constexpr int FCHUNK = 128;              // positions per shared-memory chunk
constexpr int FWARPS = 8;
constexpr int FTHREADS = FWARPS * 32;
constexpr int FD = 128;                  // head_dim of this kernel
constexpr int KP = FD + 8;               // padded row (bf16): fragment loads are conflict-free
constexpr int PP = FCHUNK + 8;           // padded P row (bf16)
constexpr int MAX_SPLIT = 16;

struct AttnSmem {
  uint16_t q[MAX_G][KP];       // normed, rotated query heads (bf16)
  uint16_t k[FCHUNK][KP];
  uint16_t v[FCHUNK][KP];
  uint16_t p[16][PP];          // probabilities (bf16), rows >= G stay zero
  float s[MAX_G][FCHUNK];      // log2-scaled scores of the chunk
  float o[MAX_G][FD];          // this CTA's unnormalised output
  uint16_t knew[FD], vnew[FD];
  float m[MAX_G], l[MAX_G], alpha[MAX_G];
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

// ---- attention chunk partials on the tensor cores (D = 64 or 128) ------------------------------------
// The same records as attn_split_kernel, one per CTA of grid (Hk, chunk groups, batch): CTA y takes the
// `span` consecutive chunks of CHUNK positions y*span .. y*span + span - 1, one after another, with an
// online softmax across them (span = 1: one record per chunk, the same bits as a single pass), with
// S = Q K^T and O = P V as mma.sync m16n8k16 (bf16 operands, fp32 accumulation): the G query heads are
// rows 0..G-1 of the 16-row A tile (the rest zero), K rows are the B operand as stored, V enters
// through ldmatrix.trans.  Warp w scores positions 16w..16w+15 and owns D/4 output columns.  Scores
// are kept in log2 units (exp2) and the record's maximum is stored back in natural units, which is
// what attn_combine_kernel reads; P is rounded to bf16 for its MMA.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <int TD>
struct SplitSmem {
  static constexpr int KP = TD + 8;  // padded rows: fragment loads are conflict-free
  uint16_t q[16][KP];
  uint16_t k[CHUNK][KP];
  uint16_t v[CHUNK][KP];
  uint16_t p[16][CHUNK + 8];
  float s[MAX_G][CHUNK];
  float x[ATTN_THREADS / 32][TD];  // per-warp scratch of the fused norm + rotary
  float mrun[MAX_G], lrun[MAX_G], alpha[MAX_G];  // running softmax state over the CTA's chunks (log2 units)
};

// Operands of the fused form: the projection's raw q/k/v rows instead of rotated queries.
struct RopeArgs {
  const uint16_t* qkv;  // [B, qkv_stride]: q heads, k heads, v heads
  int64_t qkv_stride;
  const uint16_t *qn_w, *kn_w;  // nullable (no q/k norm)
  float eps;
  const uint16_t *cos_t, *sin_t;  // [tmax, D]
};

// ROPE: the queries come raw from qkv (RopeArgs); every CTA norms and rotates its G query heads itself,
// and the CTA whose chunk holds pos also makes the new key / value row, writes it into the cache and
// uses it directly (the arithmetic of qk_norm_rope_kv_kernel, so both forms give the same bits).
template <int TD, bool ROPE>
__global__ void __launch_bounds__(ATTN_THREADS) attn_split_tc_kernel(const uint16_t* __restrict__ q, int Hq, int Hk,
                                                                     uint16_t* __restrict__ kc, uint16_t* __restrict__ vc,
                                                                     int64_t tmax, const int64_t* __restrict__ pos_ptr, float scale,
                                                                     float* __restrict__ part, int64_t kv_bstride, int window,
                                                                     RopeArgs ra, int span) {
  static_assert(ATTN_THREADS == 128 && CHUNK == 64, "four warps of 16 positions");
  using Sm = SplitSmem<TD>;
  constexpr int KP = Sm::KP;
  __shared__ __align__(16) Sm S;
  const int h = blockIdx.x, cs = blockIdx.y, b = blockIdx.z;
  const int G = Hq / Hk;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, cq = lane & 3;  // mma fragment row / column pair
  pdl_wait();
  pdl_launch_dependents();
  const int64_t pos = pos_ptr[b];
  if (pos < 0 || pos >= tmax) {  // the unfused form's cache-write kernel flags it
    if (ROPE && h == 0 && cs == 0 && tid == 0) flag(WISP_STATUS_BAD_POS);
    return;
  }
  const int64_t lo = window_lo(pos, window);
  // this CTA's chunks [cs*span, cs*span + span) that meet [lo, pos]; none: the combine never reads its record
  const int cfirst = max(cs * span, int(lo / CHUNK)), clast = min(cs * span + span - 1, int(pos / CHUNK));
  if (cfirst > clast) return;
  q += int64_t(b) * Hq * TD;
  kc += int64_t(b) * kv_bstride;
  vc += int64_t(b) * kv_bstride;
  part += int64_t(b) * Hk * gridDim.y * G * rec_floats(TD);
  const float qscale = scale * 1.4426950408889634f;  // log2 units
  constexpr int NT = TD / 32;  // P V n-tiles of 8 per warp
  float o[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  for (int c = cfirst; c <= clast; ++c) {
    const int64_t t0 = int64_t(c) * CHUNK > lo ? int64_t(c) * CHUNK : lo;
    const int n = int((pos + 1 - t0) < int64_t(c + 1) * CHUNK - t0 ? (pos + 1 - t0) : int64_t(c + 1) * CHUNK - t0);
    // positions t0 .. t0 + n - 1 sit in smem rows r0 .. r0 + n - 1 with r0 = t0 - c*CHUNK (a window can cut the chunk's start)
    const int r0 = int(t0 - int64_t(c) * CHUNK);
    // fused form: the chunk holding pos makes the new row (smem row rnew); -1 elsewhere
    const int rnew = ROPE && pos < int64_t(c + 1) * CHUNK ? int(pos - int64_t(c) * CHUNK) : -1;
    const uint16_t* kb = kc + (int64_t(h) * tmax + int64_t(c) * CHUNK) * TD;
    const uint16_t* vb = vc + (int64_t(h) * tmax + int64_t(c) * CHUNK) * TD;
    constexpr int PR = TD / 8;  // 16-byte pieces per row
    // every piece of the chunk's K and V rows in flight at once (cp.async), rows outside [r0, r0 + n) zero
    for (int i = tid; i < CHUNK * PR; i += ATTN_THREADS) {
      const int r = i / PR, cp = i % PR;
      if (r == rnew) continue;  // made below
      if (r >= r0 && r < r0 + n) {
        cp_async16(&S.k[r][8 * cp], kb + int64_t(r) * TD + 8 * cp);
        cp_async16(&S.v[r][8 * cp], vb + int64_t(r) * TD + 8 * cp);
      } else {
        reinterpret_cast<uint4*>(&S.k[r][0])[cp] = make_uint4(0, 0, 0, 0);
        reinterpret_cast<uint4*>(&S.v[r][0])[cp] = make_uint4(0, 0, 0, 0);
      }
    }
    if (c == cfirst) {  // the queries and the running state, while the first chunk's rows are in flight
      if (ROPE) {
        for (int i = tid; i < 16 * PR; i += ATTN_THREADS) {
          const int r = i / PR, cp = i % PR;
          if (r >= G) reinterpret_cast<uint4*>(&S.q[r][0])[cp] = make_uint4(0, 0, 0, 0);
        }
        const uint16_t* row = ra.qkv + int64_t(b) * ra.qkv_stride;
        for (int g = warp; g < G; g += ATTN_THREADS / 32)
          norm_rope_warp(row + int64_t(h * G + g) * TD, ra.qn_w, ra.eps, ra.cos_t + pos * TD, ra.sin_t + pos * TD, TD, lane,
                         S.x[warp], &S.q[g][0]);
      } else {
        for (int i = tid; i < 16 * PR; i += ATTN_THREADS) {
          const int r = i / PR, cp = i % PR;
          reinterpret_cast<uint4*>(&S.q[r][0])[cp] =
              r < G ? reinterpret_cast<const uint4*>(q + (int64_t(h) * G + r) * TD)[cp] : make_uint4(0, 0, 0, 0);
        }
      }
      for (int i = tid; i < 16 * (CHUNK + 8) / 2; i += ATTN_THREADS) reinterpret_cast<uint32_t*>(&S.p[0][0])[i] = 0u;
      if (tid < G) S.mrun[tid] = -INFINITY, S.lrun[tid] = 0.0f;
    }
    if (ROPE && rnew >= 0) {
      // warp 0: the new key (norm + rotary) into the cache and into smem row rnew; warp 1: the value
      const uint16_t* row = ra.qkv + int64_t(b) * ra.qkv_stride;
      uint16_t* kdst = kc + (int64_t(h) * tmax + pos) * TD;
      if (warp == 0) {
        norm_rope_warp(row + int64_t(Hq + h) * TD, ra.kn_w, ra.eps, ra.cos_t + pos * TD, ra.sin_t + pos * TD, TD, lane, S.x[0],
                       &S.k[rnew][0]);
        for (int i = lane; i < TD; i += 32) kdst[i] = S.k[rnew][i];
      } else if (warp == 1) {
        const uint16_t* vs = row + int64_t(Hq + Hk + h) * TD;
        uint16_t* vdst = vc + (int64_t(h) * tmax + pos) * TD;
        for (int i = lane; i < TD; i += 32) {
          const uint16_t v = vs[i];
          S.v[rnew][i] = v;
          vdst[i] = v;
        }
      }
    }
    cp_async_wait_all();  // the chunk's K / V rows (the query work above overlapped their flight)
    __syncthreads();
    // scores: warp w, positions 16w + 8nt + (0..7)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int t = 16 * warp + 8 * nt;
      float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < TD / 16; ++j) {
        const uint32_t a0 = *reinterpret_cast<const uint32_t*>(&S.q[gq][16 * j + 2 * cq]);
        const uint32_t a2 = *reinterpret_cast<const uint32_t*>(&S.q[gq][16 * j + 8 + 2 * cq]);
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&S.k[t + gq][16 * j + 2 * cq]);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&S.k[t + gq][16 * j + 8 + 2 * cq]);
        mma_bf16(d, a0, 0u, a2, 0u, b0, b1);
      }
      if (gq < G) {
        const int p0 = t + 2 * cq;
        S.s[gq][p0] = p0 >= r0 && p0 < r0 + n ? d[0] * qscale : -INFINITY;
        S.s[gq][p0 + 1] = p0 + 1 >= r0 && p0 + 1 < r0 + n ? d[1] * qscale : -INFINITY;
      }
    }
    __syncthreads();
    // online softmax: warp w takes heads w, w + 4; the running maximum rescales what came before
    for (int g = warp; g < G; g += ATTN_THREADS / 32) {
      const float v0 = S.s[g][lane], v1 = S.s[g][lane + 32];
      const float mp = S.mrun[g];
      const float m = fmaxf(mp, warp_max(fmaxf(v0, v1)));  // finite: the chunk holds at least one position
      const float al = exp2f(mp - m);                      // 0 at the CTA's first chunk
      const float e0 = exp2f(v0 - m), e1 = exp2f(v1 - m);
      const float l = warp_sum(e0 + e1);
      S.p[g][lane] = f32_to_bf16(e0);
      S.p[g][lane + 32] = f32_to_bf16(e1);
      __syncwarp();
      if (lane == 0) {
        S.lrun[g] = S.lrun[g] * al + l;
        S.mrun[g] = m;
        S.alpha[g] = al;
      }
    }
    __syncthreads();
    // P V: warp w owns output columns w * TD/4 .. (w + 1) * TD/4 - 1 (rows >= G of P are zero)
    if (gq < G) {
      const float al = S.alpha[gq];
#pragma unroll
      for (int i = 0; i < NT; ++i) o[i][0] *= al, o[i][1] *= al;
    }
    const int mi = lane >> 3, ri = lane & 7;  // ldmatrix: matrix mi, row ri
#pragma unroll
    for (int j = 0; j < CHUNK / 16; ++j) {
      const uint32_t a0 = *reinterpret_cast<const uint32_t*>(&S.p[gq][16 * j + 2 * cq]);
      const uint32_t a2 = *reinterpret_cast<const uint32_t*>(&S.p[gq][16 * j + 8 + 2 * cq]);
#pragma unroll
      for (int pr = 0; pr < NT / 2; ++pr) {
        uint32_t bv[4];
        ldsm_x4_trans(bv, &S.v[16 * j + (mi & 1) * 8 + ri][warp * (TD / 4) + 16 * pr + (mi >> 1) * 8]);
        mma_bf16(o[2 * pr], a0, 0u, a2, 0u, bv[0], bv[1]);
        mma_bf16(o[2 * pr + 1], a0, 0u, a2, 0u, bv[2], bv[3]);
      }
    }
    __syncthreads();  // the next chunk overwrites K, V, P and the scores
  }
  if (gq < G) {
    float* rec = part + ((int64_t(h) * gridDim.y + cs) * G + gq) * rec_floats(TD);
#pragma unroll
    for (int i = 0; i < NT; ++i)
      *reinterpret_cast<float2*>(rec + warp * (TD / 4) + 8 * i + 2 * cq) = make_float2(o[i][0], o[i][1]);
    if (warp == 0 && cq == 0) {
      rec[TD] = S.mrun[gq] * 0.6931471805599453f;  // back to natural units
      rec[TD + 1] = S.lrun[gq];
    }
  }
}

// one warp, one head of FD values (4 per lane): bf16(w * bf16(x * rsqrt(mean(x^2) + eps))), then
// rotate-half rotary (fp32, one rounding) -> 4 bf16 packed in two words; every load issued first
__device__ __forceinline__ uint2 norm_rope_head(const uint16_t* __restrict__ src, const uint16_t* __restrict__ w, float eps,
                                                const uint16_t* __restrict__ cs, const uint16_t* __restrict__ sn, int lane) {
  const uint2 xv = reinterpret_cast<const uint2*>(src)[lane];
  const uint2 wv = reinterpret_cast<const uint2*>(w)[lane];
  const uint2 cv = reinterpret_cast<const uint2*>(cs)[lane];
  const uint2 sv = reinterpret_cast<const uint2*>(sn)[lane];
  float x[4] = {__uint_as_float(xv.x << 16), __uint_as_float(xv.x & 0xFFFF0000u), __uint_as_float(xv.y << 16),
                __uint_as_float(xv.y & 0xFFFF0000u)};
  const float wf[4] = {__uint_as_float(wv.x << 16), __uint_as_float(wv.x & 0xFFFF0000u), __uint_as_float(wv.y << 16),
                       __uint_as_float(wv.y & 0xFFFF0000u)};
  const float c[4] = {__uint_as_float(cv.x << 16), __uint_as_float(cv.x & 0xFFFF0000u), __uint_as_float(cv.y << 16),
                      __uint_as_float(cv.y & 0xFFFF0000u)};
  const float sn4[4] = {__uint_as_float(sv.x << 16), __uint_as_float(sv.x & 0xFFFF0000u), __uint_as_float(sv.y << 16),
                        __uint_as_float(sv.y & 0xFFFF0000u)};
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) ss = fmaf(x[i], x[i], ss);
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / float(FD) + eps);
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = bf16_to_f32(f32_to_bf16(wf[i] * bf16_to_f32(f32_to_bf16(x[i] * inv))));
  // partner of element 4*lane + i is 4*(lane ^ 16) + i (D / 2 = 64 elements = 16 lanes away)
  uint32_t o[2];
#pragma unroll
  for (int i = 0; i < 4; i += 2) {
    const float p0 = __shfl_xor_sync(0xffffffffu, x[i], 16), p1 = __shfl_xor_sync(0xffffffffu, x[i + 1], 16);
    const float xp0 = lane < 16 ? -p0 : p0, xp1 = lane < 16 ? -p1 : p1;
    const float r0 = __fadd_rn(__fmul_rn(x[i], c[i]), __fmul_rn(xp0, sn4[i]));
    const float r1 = __fadd_rn(__fmul_rn(x[i + 1], c[i + 1]), __fmul_rn(xp1, sn4[i + 1]));
    o[i / 2] = uint32_t(f32_to_bf16(r0)) | (uint32_t(f32_to_bf16(r1)) << 16);
  }
  return make_uint2(o[0], o[1]);
}

__global__ void __launch_bounds__(FTHREADS)
    attn_fused_kernel(const uint16_t* __restrict__ qkv, int Hq, int Hk, const uint16_t* __restrict__ qn_w,
                      const uint16_t* __restrict__ kn_w, float eps, const uint16_t* __restrict__ cos_t,
                      const uint16_t* __restrict__ sin_t, const int64_t* __restrict__ pos_ptr, int64_t tmax,
                      uint16_t* __restrict__ kc, uint16_t* __restrict__ vc, float scale, uint16_t* __restrict__ out) {
  extern __shared__ __align__(16) uint8_t smraw[];
  AttnSmem& S = *reinterpret_cast<AttnSmem*>(smraw);
  const int h = blockIdx.y;
  const int G = Hq / Hk;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int rank = int(cluster_rank()), nsplit = int(cluster_size());
  // zero the padding rows of P and the per-head state while the previous kernel finishes
  for (int i = tid; i < 16 * PP / 2; i += FTHREADS) reinterpret_cast<uint32_t*>(&S.p[0][0])[i] = 0u;
  for (int i = tid; i < MAX_G * FD; i += FTHREADS) (&S.o[0][0])[i] = 0.0f;
  if (tid < MAX_G) {
    S.m[tid] = -INFINITY;
    S.l[tid] = 0.0f;
  }
  pdl_wait();  // qkv comes from the projection GEMV
  pdl_launch_dependents();
  const int64_t pos = *pos_ptr;
  const bool pos_ok = pos >= 0 && pos < tmax;
  if (!pos_ok && rank == 0 && h == 0 && tid == 0) flag(WISP_STATUS_BAD_POS);
  const int64_t n_all = pos_ok ? pos + 1 : 0;
  const int64_t per = (n_all + nsplit - 1) / nsplit;
  const int64_t t0 = rank * per, t1 = (t0 + per) < n_all ? (t0 + per) : n_all;
  const uint16_t* cs = cos_t + (pos_ok ? pos : 0) * FD;
  const uint16_t* sn = sin_t + (pos_ok ? pos : 0) * FD;
  const bool mine = pos_ok && pos >= t0 && pos < t1;  // this CTA holds the new position

  // ---- query heads (warp j: head j), the new key and value --------------------------------------
  if (warp < G) reinterpret_cast<uint2*>(S.q[warp])[lane] = norm_rope_head(qkv + int64_t(h * G + warp) * FD, qn_w, eps, cs, sn, lane);
  if (mine && warp == FWARPS - 1) {
    const uint2 kn = norm_rope_head(qkv + int64_t(Hq + h) * FD, kn_w, eps, cs, sn, lane);
    const uint2 vv = reinterpret_cast<const uint2*>(qkv + int64_t(Hq + Hk + h) * FD)[lane];
    reinterpret_cast<uint2*>(S.knew)[lane] = kn;
    reinterpret_cast<uint2*>(S.vnew)[lane] = vv;
    reinterpret_cast<uint2*>(kc + (int64_t(h) * tmax + pos) * FD)[lane] = kn;
    reinterpret_cast<uint2*>(vc + (int64_t(h) * tmax + pos) * FD)[lane] = vv;
  }
  __syncthreads();
  // A fragments of the query tile (rows g < G real, rows g + 8 zero), all 8 k-steps
  uint32_t qa[FD / 16][2];
#pragma unroll
  for (int j = 0; j < FD / 16; ++j) {
    qa[j][0] = g < G ? *reinterpret_cast<const uint32_t*>(&S.q[g][16 * j + 2 * c]) : 0u;
    qa[j][1] = g < G ? *reinterpret_cast<const uint32_t*>(&S.q[g][16 * j + 8 + 2 * c]) : 0u;
  }
  const float qscale = scale * 1.4426950408889634f;  // scores in log2 units
  float oacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};  // this warp's d n-tiles 2w, 2w+1

  const uint16_t* kb = kc + int64_t(h) * tmax * FD;
  const uint16_t* vb = vc + int64_t(h) * tmax * FD;
  for (int64_t c0 = t0; c0 < t1; c0 += FCHUNK) {
    const int n = int((t1 - c0) < FCHUNK ? (t1 - c0) : FCHUNK);
    // K and V rows [c0, c0 + n) into padded rows; rows past n are zero (P is zero there too)
    for (int i = tid; i < FCHUNK * (FD / 8); i += FTHREADS) {
      const int r = i / (FD / 8), cpart = i % (FD / 8);
      uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
      if (r < n) {
        kv = reinterpret_cast<const uint4*>(kb + (c0 + r) * FD)[cpart];
        vv = reinterpret_cast<const uint4*>(vb + (c0 + r) * FD)[cpart];
      }
      reinterpret_cast<uint4*>(&S.k[r][0])[cpart] = kv;
      reinterpret_cast<uint4*>(&S.v[r][0])[cpart] = vv;
    }
    __syncthreads();
    if (mine && pos >= c0 && pos < c0 + n) {  // the cache row of pos may not be visible yet: patch it
      const int r = int(pos - c0);
      if (tid < FD / 2) {
        reinterpret_cast<uint32_t*>(&S.k[r][0])[tid] = reinterpret_cast<const uint32_t*>(S.knew)[tid];
        reinterpret_cast<uint32_t*>(&S.v[r][0])[tid] = reinterpret_cast<const uint32_t*>(S.vnew)[tid];
      }
      __syncthreads();
    }
    // scores: warp w takes positions 16w .. 16w + 15 (two n-tiles of 8)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int t = 16 * warp + 8 * nt;
      float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < FD / 16; ++j) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&S.k[t + g][16 * j + 2 * c]);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&S.k[t + g][16 * j + 8 + 2 * c]);
        mma_bf16(d, qa[j][0], 0u, qa[j][1], 0u, b0, b1);
      }
      if (g < G) {
        const int p0 = t + 2 * c;
        S.s[g][p0] = p0 < n ? d[0] * qscale : -INFINITY;
        S.s[g][p0 + 1] = p0 + 1 < n ? d[1] * qscale : -INFINITY;
      }
    }
    __syncthreads();
    // online softmax: warp w -> head w
    if (warp < G) {
      float v4[FCHUNK / 32], mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < FCHUNK / 32; ++i) {
        v4[i] = S.s[warp][lane + 32 * i];
        mx = fmaxf(mx, v4[i]);
      }
      mx = warp_max(mx);
      const float m_old = S.m[warp], m_new = fmaxf(m_old, mx);
      float sum = 0.0f;
#pragma unroll
      for (int i = 0; i < FCHUNK / 32; ++i) {
        const float e = exp2f(v4[i] - m_new);
        sum += e;
        S.p[warp][lane + 32 * i] = f32_to_bf16(e);
      }
      sum = warp_sum(sum);
      if (lane == 0) {
        const float al = exp2f(m_old - m_new);
        S.alpha[warp] = al;
        S.l[warp] = S.l[warp] * al + sum;
        S.m[warp] = m_new;
      }
    }
    __syncthreads();
    // P V: warp w owns output columns 16w .. 16w + 15 (two n-tiles), all positions of the chunk
    {
      const float al = g < G ? S.alpha[g] : 0.0f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        oacc[nt][0] *= al;
        oacc[nt][1] *= al;
      }
      const int mi = lane >> 3, ri = lane & 7;  // ldmatrix: matrix mi, row ri
#pragma unroll 4
      for (int j = 0; j < FCHUNK / 16; ++j) {
        const uint32_t a0 = *reinterpret_cast<const uint32_t*>(&S.p[g][16 * j + 2 * c]);
        const uint32_t a2 = *reinterpret_cast<const uint32_t*>(&S.p[g][16 * j + 8 + 2 * c]);
        uint32_t bv[4];
        ldsm_x4_trans(bv, &S.v[16 * j + (mi & 1) * 8 + ri][16 * warp + (mi >> 1) * 8]);
        mma_bf16(oacc[0], a0, 0u, a2, 0u, bv[0], bv[1]);
        mma_bf16(oacc[1], a0, 0u, a2, 0u, bv[2], bv[3]);
      }
    }
    __syncthreads();
  }
  if (g < G) {
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      S.o[g][16 * warp + 8 * nt + 2 * c] = oacc[nt][0];
      S.o[g][16 * warp + 8 * nt + 2 * c + 1] = oacc[nt][1];
    }
  }

  // ---- merge the partials through distributed shared memory ---------------------------------------
  cluster_sync_all();
  const int pieces = G * 2;  // (head, half of D)
  for (int pc = rank; pos_ok && pc < pieces; pc += nsplit) {
    const int hg = pc >> 1, d0 = (pc & 1) * (FD / 2);
    float M = -INFINITY;
    for (int r = 0; r < nsplit; ++r) {
      const AttnSmem* R = static_cast<const AttnSmem*>(__cluster_map_shared_rank(static_cast<void*>(&S), r));
      M = fmaxf(M, R->m[hg]);
    }
    float Ls = 0.0f;
    for (int r = 0; r < nsplit; ++r) {
      const AttnSmem* R = static_cast<const AttnSmem*>(__cluster_map_shared_rank(static_cast<void*>(&S), r));
      Ls += R->l[hg] * exp2f(R->m[hg] - M);
    }
    for (int d = d0 + tid; d < d0 + FD / 2; d += FTHREADS) {
      float o = 0.0f;
      for (int r = 0; r < nsplit; ++r) {
        const AttnSmem* R = static_cast<const AttnSmem*>(__cluster_map_shared_rank(static_cast<void*>(&S), r));
        o += R->o[hg][d] * exp2f(R->m[hg] - M);
      }
      out[int64_t(h * G + hg) * FD + d] = f32_to_bf16(o / Ls);
    }
  }
  cluster_sync_all();  // no CTA leaves while another still reads its shared memory
}

// ---- router ------------------------------------------------------------------------------------
// One warp.  logits bf16 [E] -> p = softmax(fp32) -> top-k (ties: lower expert id first) -> p / sum
// -> bf16.  row (nullable) = [experts as float..., weights...]; meta = [slots..., weights...] with
// slot = slot_table[base + e] when a table is given (a negative entry is passed through and the MoE
// kernels skip and flag it), else base + e.
// Top-k of one token's router logits held (as fp32 values of bf16 logits) in p[0..E) of shared memory,
// by one warp; p is overwritten.  norm_topk 0: softmax over all E in fp32, the k largest; 1: the same,
// renormalised over the k; 2 (gpt-oss, wisp/gptoss.py:122-123): softmax over the k selected logits
// only.  Lane j < k gets the j-th expert (ties: lower expert id) and its weight rounded to bf16.
__device__ __forceinline__ void topk_weights(float* p, int E, int k, int norm_topk, int lane, int& sele, float& w) {
  float m = -INFINITY;
  for (int e = lane; e < E; e += 32) m = fmaxf(m, p[e]);
  m = warp_max(m);
  float s = 0.0f;
  for (int e = lane; e < E; e += 32) {
    p[e] = expf(p[e] - m);
    s += p[e];
  }
  s = warp_sum(s);
  __syncwarp();
  for (int e = lane; e < E; e += 32) p[e] = p[e] / s;
  __syncwarp();
  float selw = 0.0f, tot = 0.0f;
  sele = 0;
  for (int j = 0; j < k; ++j) {
    float bv = -1.0f;
    int be = E;
    for (int e = lane; e < E; e += 32)
      if (p[e] > bv) { bv = p[e]; be = e; }  // first (lowest) index wins within the lane
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) { bv = ov; be = oe; }
    }
    if (be >= E) {  // nothing left that compares (NaN logits): a valid id with weight 0, never an id past E
      be = j;
      bv = 0.0f;
    }
    if (lane == j) { selw = bv; sele = be; }
    tot += bv;
    __syncwarp();
    if (lane == 0) p[be] = -2.0f;
    __syncwarp();
  }
  // norm_topk 2: p = e^(l - m) / s is monotone in l, so the selected probabilities give back the
  // logits' ratios: e^(l_j - l_max) = p_j / p_max
  float sm_w = 0.0f;
  if (norm_topk == 2) {
    const float pmax = __shfl_sync(0xffffffffu, selw, 0);  // the first pick is the largest
    const float r = lane < k ? selw / pmax : 0.0f;
    const float rs = warp_sum(r);
    sm_w = r / rs;
  }
  w = bf16_to_f32(f32_to_bf16(norm_topk == 2 ? sm_w : (norm_topk ? selw / tot : selw)));
}

__global__ void router_topk_kernel(const uint16_t* __restrict__ logits, int E, int k, int norm_topk,
                                   const int32_t* __restrict__ slot_table, int64_t base, float* __restrict__ row,
                                   float* __restrict__ meta) {
  __shared__ float p[1024];
  const int lane = threadIdx.x;
  pdl_wait();
  pdl_launch_dependents();
  for (int e = lane; e < E; e += 32) p[e] = bf16_to_f32(logits[e]);
  __syncwarp();
  int sele;
  float w;
  topk_weights(p, E, k, norm_topk, lane, sele, w);
  if (lane < k) {
    if (row) {
      row[lane] = float(sele);
      row[k + lane] = w;
    }
    const int64_t slot = slot_table ? int64_t(slot_table[base + sele]) : base + sele;
    meta[lane] = float(slot);
    meta[k + lane] = w;
  }
}

// ---- the router of B tokens in one launch: RMSNorm, gate logits, top-k ------------------------------
// One CTA per token b: xn = RMSNorm(x[b]) * norm_w (the rounding of wisp_rmsnorm; stored to xn_out,
// the experts' input), logits[e] = bf16(xn . W[e] + bias[e]) in fp32 (one rounding, as a bf16 linear
// layer with bias gives), then topk_weights.  Writes meta[b] = [k slots | k weights] (slot =
// slot_table[base + e] or base + e), experts[b] = the k expert ids (int32, nullable) and row[b] =
// [k ids | k weights] in fp32 (nullable).  H % 8 == 0, H <= ROUTER_MAX_H, E <= 1024, k <= 32.
constexpr int ROUTER_THREADS = 1024;  // one warp per expert for E <= 32: a row's loads are all in flight at once
constexpr int ROUTER_MAX_H = 8192;
__global__ void __launch_bounds__(ROUTER_THREADS) router_rows_kernel(
    const uint16_t* __restrict__ x, int64_t H, const uint16_t* __restrict__ norm_w, float eps, uint16_t* __restrict__ xn_out,
    const uint16_t* __restrict__ W, const uint16_t* __restrict__ bias, int E, int k, int norm_topk,
    const int32_t* __restrict__ slot_table, int64_t base, float* __restrict__ meta, int32_t* __restrict__ experts,
    float* __restrict__ row) {
  __shared__ __align__(16) uint16_t xs[ROUTER_MAX_H];
  __shared__ float p[1024];
  __shared__ float red[ROUTER_THREADS / 32];
  const int b = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int NW = ROUTER_THREADS / 32;
  pdl_wait();
  pdl_launch_dependents();
  const int64_t nch = H / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + int64_t(b) * H);
  float ss = 0.0f;
  for (int64_t c = threadIdx.x; c < nch; c += ROUTER_THREADS) {
    const uint4 v = xr[c];
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) ss += bf_lo(w4[i]) * bf_lo(w4[i]) + bf_hi(w4[i]) * bf_hi(w4[i]);
    reinterpret_cast<uint4*>(xs)[c] = v;
  }
  if (norm_w) {
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; ++w) tot += red[w];
    const float inv = rsqrtf(tot / float(H) + eps);
    for (int64_t c = threadIdx.x; c < nch; c += ROUTER_THREADS) {
      const uint4 v = reinterpret_cast<const uint4*>(xs)[c];
      const uint4 wv = reinterpret_cast<const uint4*>(norm_w)[c];
      const uint32_t xv[4] = {v.x, v.y, v.z, v.w}, ww[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float lo = bf_lo(ww[i]) * bf16_to_f32(f32_to_bf16(bf_lo(xv[i]) * inv));
        const float hi = bf_hi(ww[i]) * bf16_to_f32(f32_to_bf16(bf_hi(xv[i]) * inv));
        o[i] = uint32_t(f32_to_bf16(lo)) | (uint32_t(f32_to_bf16(hi)) << 16);
      }
      const uint4 on = make_uint4(o[0], o[1], o[2], o[3]);
      reinterpret_cast<uint4*>(xs)[c] = on;
      if (xn_out) reinterpret_cast<uint4*>(xn_out + int64_t(b) * H)[c] = on;
    }
  } else if (xn_out) {
    for (int64_t c = threadIdx.x; c < nch; c += ROUTER_THREADS)
      reinterpret_cast<uint4*>(xn_out + int64_t(b) * H)[c] = reinterpret_cast<const uint4*>(xs)[c];
  }
  __syncthreads();
  // gate logits: warp w takes experts w, w + NW, ...; lanes split the row
  const uint4* xs4 = reinterpret_cast<const uint4*>(xs);
  for (int e = warp; e < E; e += NW) {
    const uint4* wr = reinterpret_cast<const uint4*>(W + int64_t(e) * H);
    float a0 = 0.0f, a1 = 0.0f;
#pragma unroll 8
    for (int64_t c = lane; c < nch; c += 32) {
      const uint4 w = __ldg(wr + c), xv4 = xs4[c];
      const uint32_t wv[4] = {w.x, w.y, w.z, w.w}, xv[4] = {xv4.x, xv4.y, xv4.z, xv4.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        a0 = fmaf(bf_lo(wv[q]), bf_lo(xv[q]), a0);
        a1 = fmaf(bf_hi(wv[q]), bf_hi(xv[q]), a1);
      }
    }
    const float acc = warp_sum(a0 + a1);
    if (lane == 0) p[e] = bf16_to_f32(f32_to_bf16(acc + (bias ? bf16_to_f32(bias[e]) : 0.0f)));
  }
  __syncthreads();
  if (warp == 0) {
    int sele;
    float w;
    topk_weights(p, E, k, norm_topk, lane, sele, w);
    if (lane < k) {
      const int64_t slot = slot_table ? int64_t(slot_table[base + sele]) : base + sele;
      meta[int64_t(b) * 2 * k + lane] = float(slot);
      meta[int64_t(b) * 2 * k + k + lane] = w;
      if (experts) experts[int64_t(b) * k + lane] = sele;
      if (row) {
        row[int64_t(b) * 2 * k + lane] = float(sele);
        row[int64_t(b) * 2 * k + k + lane] = w;
      }
    }
  }
}

// The same router with the gate split over CTAs: grid (B, ceil(E / ROUTER_SPLIT_E)); CTA (b, s) norms
// token b's row (every CTA of the token redundantly; CTA 0 stores it) and computes the logits of experts
// [s*ROUTER_SPLIT_E, ...) with one warp per expert, into ws_logits [B, E] (fp32 values of the bf16
// logits).  The last CTA of a token to finish (an arrival counter per token, after a fence) loads the
// token's E logits and runs the top-k; it then resets the counter, so the workspace stays ready for
// the next launch (it must be zero before the first one).  No CTA waits for another: the counter only
// elects which one finishes.
constexpr int ROUTER_SPLIT_E = 4;
constexpr int ROUTER_SPLIT_THREADS = 32 * ROUTER_SPLIT_E;
__global__ void __launch_bounds__(ROUTER_SPLIT_THREADS) router_split_kernel(
    const uint16_t* __restrict__ x, int64_t H, const uint16_t* __restrict__ norm_w, float eps, uint16_t* __restrict__ xn_out,
    const uint16_t* __restrict__ W, const uint16_t* __restrict__ bias, int E, int k, int norm_topk,
    const int32_t* __restrict__ slot_table, int64_t base, float* __restrict__ meta, int32_t* __restrict__ experts,
    float* __restrict__ row, float* __restrict__ ws_logits, unsigned int* __restrict__ ws_count) {
  __shared__ __align__(16) uint16_t xs[ROUTER_MAX_H];
  __shared__ float p[1024];
  __shared__ float red[ROUTER_SPLIT_E];
  __shared__ unsigned int s_last;
  const int b = blockIdx.x, sl = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int NW = ROUTER_SPLIT_E;
  pdl_wait();
  pdl_launch_dependents();
  const int64_t nch = H / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + int64_t(b) * H);
  float ss = 0.0f;
  for (int64_t c = threadIdx.x; c < nch; c += ROUTER_SPLIT_THREADS) {
    const uint4 v = xr[c];
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) ss += bf_lo(w4[i]) * bf_lo(w4[i]) + bf_hi(w4[i]) * bf_hi(w4[i]);
    reinterpret_cast<uint4*>(xs)[c] = v;
  }
  if (norm_w) {
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; ++w) tot += red[w];
    const float inv = rsqrtf(tot / float(H) + eps);
    for (int64_t c = threadIdx.x; c < nch; c += ROUTER_SPLIT_THREADS) {
      const uint4 v = reinterpret_cast<const uint4*>(xs)[c];
      const uint4 wv = reinterpret_cast<const uint4*>(norm_w)[c];
      const uint32_t xv[4] = {v.x, v.y, v.z, v.w}, ww[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float lo = bf_lo(ww[i]) * bf16_to_f32(f32_to_bf16(bf_lo(xv[i]) * inv));
        const float hi = bf_hi(ww[i]) * bf16_to_f32(f32_to_bf16(bf_hi(xv[i]) * inv));
        o[i] = uint32_t(f32_to_bf16(lo)) | (uint32_t(f32_to_bf16(hi)) << 16);
      }
      const uint4 on = make_uint4(o[0], o[1], o[2], o[3]);
      reinterpret_cast<uint4*>(xs)[c] = on;
      if (xn_out && sl == 0) reinterpret_cast<uint4*>(xn_out + int64_t(b) * H)[c] = on;
    }
  } else if (xn_out && sl == 0) {
    for (int64_t c = threadIdx.x; c < nch; c += ROUTER_SPLIT_THREADS)
      reinterpret_cast<uint4*>(xn_out + int64_t(b) * H)[c] = reinterpret_cast<const uint4*>(xs)[c];
  }
  __syncthreads();
  // this CTA's experts: warp w takes expert sl * NW + w
  const int e = sl * NW + warp;
  if (e < E) {
    const uint4* xs4 = reinterpret_cast<const uint4*>(xs);
    const uint4* wr = reinterpret_cast<const uint4*>(W + int64_t(e) * H);
    float a0 = 0.0f, a1 = 0.0f;
#pragma unroll 8
    for (int64_t c = lane; c < nch; c += 32) {
      const uint4 w = __ldg(wr + c), xv4 = xs4[c];
      const uint32_t wv[4] = {w.x, w.y, w.z, w.w}, xv[4] = {xv4.x, xv4.y, xv4.z, xv4.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        a0 = fmaf(bf_lo(wv[q]), bf_lo(xv[q]), a0);
        a1 = fmaf(bf_hi(wv[q]), bf_hi(xv[q]), a1);
      }
    }
    const float acc = warp_sum(a0 + a1);
    if (lane == 0) ws_logits[int64_t(b) * E + e] = bf16_to_f32(f32_to_bf16(acc + (bias ? bf16_to_f32(bias[e]) : 0.0f)));
  }
  __threadfence();  // this CTA's logits are visible device-wide before it counts itself in
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&ws_count[b], 1u) == gridDim.y - 1 ? 1u : 0u;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (warp == 0) {
    for (int i = lane; i < E; i += 32) p[i] = __ldcg(ws_logits + int64_t(b) * E + i);
    __syncwarp();
    int sele;
    float w;
    topk_weights(p, E, k, norm_topk, lane, sele, w);
    if (lane < k) {
      const int64_t slot = slot_table ? int64_t(slot_table[base + sele]) : base + sele;
      meta[int64_t(b) * 2 * k + lane] = float(slot);
      meta[int64_t(b) * 2 * k + k + lane] = w;
      if (experts) experts[int64_t(b) * k + lane] = sele;
      if (row) {
        row[int64_t(b) * 2 * k + lane] = float(sele);
        row[int64_t(b) * 2 * k + k + lane] = w;
      }
    }
    if (lane == 0) ws_count[b] = 0u;  // every CTA of this token has counted itself in: ready for the next launch
  }
}

// ---- embedding and greedy pick -------------------------------------------------------------------
__global__ void embed_kernel(const uint16_t* __restrict__ table, int64_t V, int64_t H, const int64_t* __restrict__ tok,
                             uint16_t* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t t = *tok;
  if (t < 0 || t >= V) {
    if (threadIdx.x == 0 && blockIdx.x == 0) flag(WISP_STATUS_BAD_ROUTE);
    return;
  }
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < H / 8; i += int64_t(gridDim.x) * blockDim.x)
    reinterpret_cast<uint4*>(out)[i] = reinterpret_cast<const uint4*>(table + t * H)[i];
}

// order-preserving key of (value, index): larger value first, then lower index
__device__ __forceinline__ unsigned long long argmax_key(float v, int64_t i) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(b) << 32) | static_cast<unsigned long long>(0xFFFFFFFFu - uint32_t(i));
}

__global__ void argmax_partial_kernel(const uint16_t* __restrict__ x, int64_t n, unsigned long long* __restrict__ part) {
  __shared__ unsigned long long red[32];
  pdl_wait();
  pdl_launch_dependents();
  unsigned long long best = 0;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const float v = bf16_to_f32(x[i]);
    if (v == v) {  // NaN never wins
      const unsigned long long key = argmax_key(v, i);
      best = key > best ? key : best;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long ob = __shfl_xor_sync(0xffffffffu, best, o);
    best = ob > best ? ob : best;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < int(blockDim.x >> 5); ++w) best = red[w] > best ? red[w] : best;
    part[blockIdx.x] = best;
  }
}

__global__ void argmax_final_kernel(const unsigned long long* __restrict__ part, int nparts, int64_t* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  unsigned long long best = 0;
  for (int i = threadIdx.x; i < nparts; i += 32) best = part[i] > best ? part[i] : best;
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long ob = __shfl_xor_sync(0xffffffffu, best, o);
    best = ob > best ? ob : best;
  }
  if (threadIdx.x == 0) *out = best ? int64_t(0xFFFFFFFFu - uint32_t(best & 0xFFFFFFFFu)) : 0;
}

}  // namespace dec
}  // namespace wisp
