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
#include "tma.cuh"

namespace wisp {
namespace dec {

constexpr int CHUNK = 64;       // positions per attention CTA
constexpr int ATTN_THREADS = 128;
constexpr int QK_MAX_D = 256;   // head_dim limit of the norm/rotary kernel
constexpr int MAX_D = 128;      // head_dim limit of the attention kernels
constexpr int MAX_G = 8;        // query heads per KV head (attention)

// ---- per-head RMSNorm + rotary + cache write -----------------------------------------------------
// qkv: [Hq*D | Hk*D | Hk*D] bf16 (q heads, k heads, v heads).  One warp per head.
__global__ void qk_norm_rope_kv_kernel(const uint16_t* __restrict__ qkv, int Hq, int Hk, int D,
                                       const uint16_t* __restrict__ qn_w, const uint16_t* __restrict__ kn_w, float eps,
                                       const uint16_t* __restrict__ cos_t, const uint16_t* __restrict__ sin_t,
                                       const int64_t* __restrict__ pos_ptr, int64_t tmax, uint16_t* __restrict__ q_out,
                                       uint16_t* __restrict__ kc, uint16_t* __restrict__ vc) {
  __shared__ float xs[8][QK_MAX_D];
  const int wib = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.x * (blockDim.x >> 5) + wib;
  pdl_wait();
  pdl_launch_dependents();
  if (head >= Hq + 2 * Hk) return;
  const int64_t pos = *pos_ptr;
  if (pos < 0 || pos >= tmax) {
    if (lane == 0 && head == 0) flag(WISP_STATUS_BAD_POS);
    return;
  }
  const uint16_t* src = qkv + int64_t(head) * D;
  if (head >= Hq + Hk) {  // v: straight into the cache
    const int hv = head - Hq - Hk;
    uint16_t* dst = vc + (int64_t(hv) * tmax + pos) * D;
    for (int i = lane; i < D; i += 32) dst[i] = src[i];
    return;
  }
  const bool is_q = head < Hq;
  const uint16_t* w = is_q ? qn_w : kn_w;
  float* x = xs[wib];
  float ss = 0.0f;
  for (int i = lane; i < D; i += 32) {
    const float v = bf16_to_f32(src[i]);
    x[i] = v;
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / float(D) + eps);
  __syncwarp();
  // HF RMSNorm: weight * bf16(x * rsqrt(mean(x^2) + eps)), rounded to bf16
  for (int i = lane; i < D; i += 32) x[i] = bf16_to_f32(f32_to_bf16(bf16_to_f32(w[i]) * bf16_to_f32(f32_to_bf16(x[i] * inv))));
  __syncwarp();
  const uint16_t* cs = cos_t + pos * D;
  const uint16_t* sn = sin_t + pos * D;
  uint16_t* dst = is_q ? q_out + int64_t(head) * D : kc + (int64_t(head - Hq) * tmax + pos) * D;
  const int half = D / 2;
  for (int i = lane; i < D; i += 32) {
    const float xp = i < half ? -x[i + half] : x[i - half];
    dst[i] = f32_to_bf16(__fadd_rn(__fmul_rn(x[i], bf16_to_f32(cs[i])), __fmul_rn(xp, bf16_to_f32(sn[i]))));
  }
}

// ---- attention: chunk partials --------------------------------------------------------------------
// grid (Hk, tmax / CHUNK): CTA (h, c) covers positions [c*CHUNK, min((c+1)*CHUNK, pos+1)) for the
// G = Hq/Hk query heads of KV head h.  Partial record per (h, c, g): D unnormalised outputs, then
// the running max and the sum of exponentials.
__global__ void __launch_bounds__(ATTN_THREADS) attn_split_kernel(const uint16_t* __restrict__ q, int Hq, int Hk, int D,
                                                                  const uint16_t* __restrict__ kc,
                                                                  const uint16_t* __restrict__ vc, int64_t tmax,
                                                                  const int64_t* __restrict__ pos_ptr, float scale,
                                                                  float* __restrict__ part) {
  __shared__ float qs[MAX_G][MAX_D];
  __shared__ float ps[MAX_G][CHUNK];
  __shared__ float red[ATTN_THREADS / 32][MAX_G][MAX_D];  // per-warp P V sums, lane-major
  const int h = blockIdx.x, c = blockIdx.y;
  const int G = Hq / Hk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = ATTN_THREADS / 32;
  pdl_wait();
  pdl_launch_dependents();
  const int64_t pos = *pos_ptr;
  if (pos < 0 || pos >= tmax) return;  // flagged by the cache-write kernel
  const int64_t t0 = int64_t(c) * CHUNK;
  if (t0 > pos) return;  // beyond the current length: the combine never reads this record
  const int n = int((pos + 1 - t0) < CHUNK ? (pos + 1 - t0) : CHUNK);
  // q of the G heads, pre-scaled, fp32
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) qs[i / D][i % D] = bf16_to_f32(q[(int64_t(h) * G) * D + i]) * scale;
  __syncthreads();
  const uint16_t* kb = kc + (int64_t(h) * tmax + t0) * D;
  const uint16_t* vb = vc + (int64_t(h) * tmax + t0) * D;
  const int dpl = D / 32;  // elements of a row per lane (D % 32 == 0, D <= MAX_D)
  // scores: warp w takes positions w, w + 4, ...; lanes split the row
  for (int t = warp; t < n; t += nw) {
    float kv[MAX_D / 32];
#pragma unroll
    for (int e = 0; e < MAX_D / 32; ++e) kv[e] = e < dpl ? bf16_to_f32(kb[int64_t(t) * D + lane * dpl + e]) : 0.0f;
    for (int g = 0; g < G; ++g) {
      float s = 0.0f;
#pragma unroll
      for (int e = 0; e < MAX_D / 32; ++e)
        if (e < dpl) s = fmaf(qs[g][lane * dpl + e], kv[e], s);
      s = warp_sum(s);
      if (lane == 0) ps[g][t] = s;
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
      float* rec = part + ((int64_t(h) * gridDim.y + c) * G + g) * (D + 2);
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
    for (int e = 0; e < MAX_D / 32; ++e) vv[e] = e < dpl ? bf16_to_f32(vb[int64_t(t) * D + lane * dpl + e]) : 0.0f;
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
    part[((int64_t(h) * gridDim.y + c) * G + g) * (D + 2) + d] = s;
  }
}

// one CTA per query head: out = sum_c O_c e^(m_c - M) / sum_c l_c e^(m_c - M)
__global__ void attn_combine_kernel(const float* __restrict__ part, int Hq, int Hk, int D, int nchunk_max,
                                    const int64_t* __restrict__ pos_ptr, int64_t tmax, uint16_t* __restrict__ out) {
  const int head = blockIdx.x;
  const int G = Hq / Hk, h = head / G, g = head % G;
  pdl_wait();
  pdl_launch_dependents();
  const int64_t pos = *pos_ptr;
  if (pos < 0 || pos >= tmax) return;
  const int nc = int(pos / CHUNK) + 1;
  float M = -INFINITY;
  for (int c = 0; c < nc; ++c) M = fmaxf(M, part[((int64_t(h) * nchunk_max + c) * G + g) * (D + 2) + D]);
  float Ls = 0.0f;
  for (int c = 0; c < nc; ++c) {
    const float* rec = part + ((int64_t(h) * nchunk_max + c) * G + g) * (D + 2);
    Ls += rec[D + 1] * __expf(rec[D] - M);
  }
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float o = 0.0f;
    for (int c = 0; c < nc; ++c) {
      const float* rec = part + ((int64_t(h) * nchunk_max + c) * G + g) * (D + 2);
      o += rec[d] * __expf(rec[D] - M);
    }
    out[int64_t(head) * D + d] = f32_to_bf16(o / Ls);
  }
}

// ---- router ------------------------------------------------------------------------------------
// One warp.  logits bf16 [E] -> p = softmax(fp32) -> top-k (ties: lower expert id first) -> p / sum
// -> bf16.  row (nullable) = [experts as float..., weights...]; meta = [slots..., weights...] with
// slot = slot_table[base + e] when a table is given (a negative entry is passed through and the MoE
// kernels skip and flag it), else base + e.
__global__ void router_topk_kernel(const uint16_t* __restrict__ logits, int E, int k, int norm_topk,
                                   const int32_t* __restrict__ slot_table, int64_t base, float* __restrict__ row,
                                   float* __restrict__ meta) {
  __shared__ float p[1024];
  const int lane = threadIdx.x;
  pdl_wait();
  pdl_launch_dependents();
  float m = -INFINITY;
  for (int e = lane; e < E; e += 32) {
    p[e] = bf16_to_f32(logits[e]);
    m = fmaxf(m, p[e]);
  }
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
  int sele = 0;
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
    if (lane == j) { selw = bv; sele = be; }
    tot += bv;
    __syncwarp();
    if (lane == 0) p[be] = -2.0f;
    __syncwarp();
  }
  if (lane < k) {
    const float w = bf16_to_f32(f32_to_bf16(norm_topk ? selw / tot : selw));
    if (row) {
      row[lane] = float(sele);
      row[k + lane] = w;
    }
    const int64_t slot = slot_table ? int64_t(slot_table[base + sele]) : base + sele;
    meta[lane] = float(slot);
    meta[k + lane] = w;
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
