// Fused group-wise dequant + GEMV over the top-k routed experts of one decode token, read straight
// from the packed slot pool.  Two phases:
//   gate/up : a[j, r]  = silu(s.(q_g . x) + m.sum(x)) * (s.(q_u . x) + m.sum(x))     (per group)
//   down    : out[h]   = sum_j w_j * sum_groups (s.(q_d . a_j) + m.sum(a_j))
// The dequant is folded into the dot products (sum_i (q_i s + m) x_i = s (q . x) + m sum x), so no
// bf16 weight is ever materialised; the codes are unpacked in registers from 128-bit streaming loads.
#pragma once
#include "common.cuh"

namespace wisp {

struct MoeShape {
  int64_t nslots, nbytes;
  int k, H, I, group;
  int gshift;         // log2(group / 128) when group is 128 * 2^s (tensor-core path), else 0
  int64_t ncode;      // bytes of the code region
  int64_t ng;         // groups per expert
  int64_t mat_bytes;  // code bytes per matrix
  int glog;           // log2(group) when group is a power of two, else -1
  int dn_beside;      // two-kernel pipeline: a down CTA fits beside a gate/up CTA (it fetches its own rows early)
};

// group index of element e of an expert's code stream (3n < 2^32 for every accepted shape): a shift
// when group is a power of two, else one 32-bit division
__device__ __forceinline__ int64_t group_of(int64_t e, const MoeShape& S) {
  return S.glog >= 0 ? (e >> S.glog) : int64_t(uint32_t(e) / uint32_t(S.group));
}

__host__ __device__ inline int log2_or_neg(int v) {
  if (v <= 0 || (v & (v - 1)) != 0) return -1;
  int l = 0;
  while ((1 << l) < v) ++l;
  return l;
}

// Routing computed inside the MoE kernels from the router logits (instead of a meta buffer written
// by a separate top-k launch): softmax in fp32, the k largest (ties: lower expert id), renormalised
// when norm_topk, rounded to bf16 (wisp/graphdec.py:177-182, wisp/moe.py:67-72).
struct MoeRoute {
  const uint16_t* logits;     // bf16 [E]; NULL: the kernels read the meta buffer instead
  int E, norm_topk;
  const int32_t* slot_table;  // NULL: slot = base + e
  int64_t base;
  float* row_out;             // nullable: [k experts | k weights], written by CTA 0 of the gate/up grid
  // Expert paging without a host decision: a negative slot_table entry means "not resident", and
  // when host_store (a device-accessible pointer to pinned host memory, rows of nbytes, key =
  // base + e) is given the kernels read that expert's bytes from it instead of from a slot.  The
  // routing entry then holds -(key + 1).  miss_count (nullable) counts such experts per call.
  const uint8_t* host_store;
  int64_t host_rows;
  int* miss_count;
};

// All threads of the CTA (blockDim.x >= E, k <= 32): meta[0..2k) in shared memory = [slots | weights];
// red: blockDim.x / 32 floats, xs: E + 64 floats of scratch.  LDCG: read the logits through L2 (the
// caller may run before its griddepcontrol.wait, after the producer of the logits has completed).
template <bool LDCG>
__device__ void route_from_logits(const MoeRoute& R, int k, float* meta, float* red, float* xs) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5, nw = blockDim.x >> 5;
  float x = -INFINITY;
  if (t < R.E) {
    const uint16_t b = LDCG ? __ldcg(reinterpret_cast<const unsigned short*>(R.logits) + t) : R.logits[t];
    x = bf16_to_f32(b);
    xs[t] = x;
  }
  float m = warp_max(x);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = red[0];
  for (int w = 1; w < nw; ++w) m = fmaxf(m, red[w]);
  const float e = t < R.E ? expf(x - m) : 0.0f;
  __syncthreads();
  float s = warp_sum(e);
  if (lane == 0) red[warp] = s;
  __syncthreads();
  s = 0.0f;
  for (int w = 0; w < nw; ++w) s += red[w];
  // rank of this expert: experts with a larger logit, or an equal one and a lower id, come first
  int rank = 0;
  if (t < R.E)
    for (int u = 0; u < R.E; ++u) {
      const float y = xs[u];
      rank += (y > x || (y == x && u < t)) ? 1 : 0;
    }
  __syncthreads();
  const float p = e / s;
  if (t < R.E && rank < k) {
    float m = float(R.base + t);
    if (R.slot_table) {  // through L2: the table may be republished by copies on another stream
      const int32_t s = __ldcg(R.slot_table + R.base + t);
      m = (s < 0 && R.host_store) ? -float(R.base + t) - 1.0f : float(s);
    }
    meta[rank] = m;
    xs[R.E + rank] = float(t);
    xs[R.E + 32 + rank] = p;
  }
  __syncthreads();
  if (t < k) {
    float tot = 0.0f;
    for (int j = 0; j < k; ++j) tot += xs[R.E + 32 + j];  // fixed order: the same sum in every CTA
    const float pt = xs[R.E + 32 + t];
    const float w = bf16_to_f32(f32_to_bf16(R.norm_topk ? pt / tot : pt));
    meta[k + t] = w;
    if (R.row_out && blockIdx.x == 0) {
      R.row_out[t] = xs[R.E + t];
      R.row_out[k + t] = w;
    }
  }
  __syncthreads();
}

__device__ __forceinline__ bool route_slot(const float* meta, int j, const MoeShape& S, int64_t& slot) {
  const float f = meta[j];
  if (!(f >= 0.0f) || f >= float(S.nslots)) return false;
  slot = int64_t(f);
  return true;
}

// Bytes of routed expert j given its routing entry f: slot f of the pool, or row -(f + 1) of the
// host store (when one is given); NULL when the entry is neither (the expert is skipped and flagged).
__device__ __forceinline__ const uint8_t* expert_src(float f, const MoeShape& S, const uint8_t* pool, const MoeRoute& RT,
                                                     bool& host) {
  host = false;
  if (f >= 0.0f && f < float(S.nslots)) return pool + int64_t(f) * S.nbytes;
  if (RT.host_store && f <= -1.0f) {
    const int64_t key = int64_t(-f) - 1;
    if (key < RT.host_rows) {
      host = true;
      return RT.host_store + key * S.nbytes;
    }
  }
  return nullptr;
}

// Warp-wide copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from global memory
// (device or mapped pinned host memory) into shared memory, four 16-byte loads in flight per lane.
__device__ __forceinline__ void warp_copy_g2s(void* dst, const void* src, int64_t bytes, int lane) {
  const uint4* s = static_cast<const uint4*>(src);
  uint4* d = static_cast<uint4*>(dst);
  const int64_t n = bytes >> 4;
  int64_t i = lane;
  for (; i + 96 < n; i += 128) {
    const uint4 a = s[i], b = s[i + 32], c = s[i + 64], e = s[i + 96];
    d[i] = a;
    d[i + 32] = b;
    d[i + 64] = c;
    d[i + 96] = e;
  }
  for (; i < n; i += 32) d[i] = s[i];
}

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

// grid (ceil(I / (8*RPW)), k); 8 warps; a warp owns RPW consecutive rows r of expert j (gate row r and
// up row r together, so SwiGLU is applied in registers).  Lane l owns units l, l+32, ... of a row.
template <int BITS, int UPL, int RPW>
__global__ void __launch_bounds__(256) moe_gate_up_kernel(const uint8_t* __restrict__ pool,
                                                          const float* __restrict__ meta,
                                                          const uint16_t* __restrict__ x, MoeShape S,
                                                          float* __restrict__ a_out) {
  const int j = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = (blockIdx.x * 8 + warp) * RPW;
  if (row0 >= S.I) return;
  int64_t slot;
  if (!route_slot(meta, j, S, slot)) {
    if (lane < RPW && row0 + lane < S.I) a_out[int64_t(j) * S.I + row0 + lane] = 0.0f;
    if (lane == 0 && row0 == 0) flag(WISP_STATUS_BAD_SLOT);
    return;
  }
  const int U = S.H / 32;
  const int GPR = S.H / S.group;
  const int64_t row_bytes = int64_t(S.H) * BITS / 8;
  const uint8_t* base = pool + slot * S.nbytes;
  const uint16_t* sc = reinterpret_cast<const uint16_t*>(base + S.ncode);
  const uint16_t* mn = sc + S.ng;
  const int64_t ngm = S.ng / 3;

  // issue every weight load of this warp first (codes + scales), then fetch x and compute
  Unit<BITS> cg[RPW][UPL], cu[RPW][UPL];
  uint16_t sg[RPW][UPL], mg[RPW][UPL], su[RPW][UPL], mu[RPW][UPL];
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int row = min(row0 + r, S.I - 1);
#pragma unroll
    for (int t = 0; t < UPL; ++t) {
      const int u = min(lane + 32 * t, U - 1);
      const uint8_t* p = base + row * row_bytes + u * (4 * BITS);
      cg[r][t] = load_unit<BITS>(p);
      cu[r][t] = load_unit<BITS>(p + S.mat_bytes);
      const int64_t gi = int64_t(row) * GPR + (u * 32) / S.group;
      sg[r][t] = ld_nc_u16(sc + gi);
      mg[r][t] = ld_nc_u16(mn + gi);
      su[r][t] = ld_nc_u16(sc + ngm + gi);
      mu[r][t] = ld_nc_u16(mn + ngm + gi);
    }
  }
  float xv[UPL][32], xs[UPL];
#pragma unroll
  for (int t = 0; t < UPL; ++t) {
    const int u = min(lane + 32 * t, U - 1);
    const uint4* xp = reinterpret_cast<const uint4*>(x + u * 32);
    float s = 0.0f;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      uint4 q = xp[v];
      uint32_t wds[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        xv[t][8 * v + 2 * h] = __uint_as_float(wds[h] << 16);
        xv[t][8 * v + 2 * h + 1] = __uint_as_float(wds[h] & 0xFFFF0000u);
      }
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) s += xv[t][i];
    xs[t] = s;
  }
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    float accg = 0.0f, accu = 0.0f;
#pragma unroll
    for (int t = 0; t < UPL; ++t) {
      if (lane + 32 * t < U) {
        float dg = 0.0f, du = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          dg = fmaf(small_u2f(unit_code<BITS>(cg[r][t], i)), xv[t][i], dg);
          du = fmaf(small_u2f(unit_code<BITS>(cu[r][t], i)), xv[t][i], du);
        }
        accg += f16_bits_to_f32(sg[r][t]) * dg + f16_bits_to_f32(mg[r][t]) * xs[t];
        accu += f16_bits_to_f32(su[r][t]) * du + f16_bits_to_f32(mu[r][t]) * xs[t];
      }
    }
    accg = warp_sum(accg);
    accu = warp_sum(accu);
    if (lane == 0 && row0 + r < S.I) a_out[int64_t(j) * S.I + row0 + r] = silu_mul(accg, accu);
  }
}

// grid ceil(H / 8); 8 warps; warp w owns output row h and walks all k experts, so the weighted
// combine happens in registers and out[h] is written once.  a (fp32 [k, I]) is staged in shared memory
// transposed per unit ([k][32][UP], UP odd) so lane l reading element i of unit l is conflict free.
template <int BITS, int UPL>
__global__ void __launch_bounds__(256) moe_down_kernel(const uint8_t* __restrict__ pool,
                                                       const float* __restrict__ meta,
                                                       const float* __restrict__ a, MoeShape S,
                                                       uint16_t* __restrict__ out) {
  extern __shared__ float sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int U = S.I / 32, UP = U | 1;
  float* at = sm;                          // [k][32][UP]
  float* as = sm + S.k * 32 * UP;          // [k][U] unit sums
  const int h = blockIdx.x * 8 + warp;
  const int GPR = S.I / S.group;
  const int64_t row_bytes = int64_t(S.I) * BITS / 8;
  const int64_t ngm = S.ng / 3;
  float acc = 0.0f;
  for (int j0 = 0; j0 < S.k; j0 += 8) {
    // issue this chunk's weight loads before waiting on anything
    Unit<BITS> cd[8][UPL];
    uint16_t sd[8][UPL], md[8][UPL];
    bool ok[8];
    float wj[8];
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      const int j = j0 + jj;
      int64_t slot = 0;
      ok[jj] = j < S.k && h < S.H && route_slot(meta, j, S, slot);
      wj[jj] = j < S.k ? meta[S.k + j] : 0.0f;
      const uint8_t* base = pool + slot * S.nbytes;
      const uint16_t* sc = reinterpret_cast<const uint16_t*>(base + S.ncode);
      const uint16_t* mn = sc + S.ng;
#pragma unroll
      for (int t = 0; t < UPL; ++t) {
        const int u = min(lane + 32 * t, U - 1);
        if (ok[jj]) {
          cd[jj][t] = load_unit<BITS>(base + 2 * S.mat_bytes + h * row_bytes + u * (4 * BITS));
          const int64_t gi = 2 * ngm + int64_t(h) * GPR + (u * 32) / S.group;
          sd[jj][t] = ld_nc_u16(sc + gi);
          md[jj][t] = ld_nc_u16(mn + gi);
        }
      }
    }
    if (j0 == 0) {
      // stage a (all experts) while the weight loads are in flight: four independent 16-byte loads
      // per thread per round, then the transposed scatter; unit sums are taken from shared memory
      const float4* a4 = reinterpret_cast<const float4*>(a);
      const int n4 = S.k * S.I / 4;
      for (int b0 = threadIdx.x; b0 < n4; b0 += 4 * blockDim.x) {
        float4 v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int idx = b0 + q * blockDim.x;
          if (idx < n4) v[q] = a4[idx];
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int idx = b0 + q * blockDim.x;
          if (idx < n4) {
            const float vv[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const int flat = 4 * idx + c;
              const int j = flat / S.I, e = flat - j * S.I;
              at[(j * 32 + (e & 31)) * UP + (e >> 5)] = vv[c];
            }
          }
        }
      }
      __syncthreads();
      for (int idx = threadIdx.x; idx < S.k * U; idx += blockDim.x) {
        const int j = idx / U, u = idx - j * U;
        float s = 0.0f;
        for (int i = 0; i < 32; ++i) s += at[(j * 32 + i) * UP + u];
        as[idx] = s;
      }
      __syncthreads();
    }
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      if (!ok[jj]) continue;
      const int j = j0 + jj;
#pragma unroll
      for (int t = 0; t < UPL; ++t) {
        const int u = lane + 32 * t;
        if (u < U) {
          const float* ap = at + j * 32 * UP + u;
          float d = 0.0f;
#pragma unroll
          for (int i = 0; i < 32; ++i) d = fmaf(small_u2f(unit_code<BITS>(cd[jj][t], i)), ap[i * UP], d);
          acc += wj[jj] * (f16_bits_to_f32(sd[jj][t]) * d + f16_bits_to_f32(md[jj][t]) * as[j * U + u]);
        }
      }
    }
  }
  if (lane == 0 && threadIdx.x == 0) {
    // one thread per block reports routing errors (cheap, idempotent)
    for (int j = 0; j < S.k; ++j) {
      int64_t slot;
      if (!route_slot(meta, j, S, slot)) flag(WISP_STATUS_BAD_SLOT);
    }
  }
  acc = warp_sum(acc);
  if (lane == 0 && h < S.H) out[h] = f32_to_bf16(acc);
}

}  // namespace wisp
