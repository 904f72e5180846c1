/*
 * wisp_b200.h -- C ABI of libwisp_b200.so, the B200 (sm_100a) kernels behind the WiSP decode hot path.
 *
 * Conventions
 *   - Every entry point returns WISP_OK (0) or a WISP_ERR_* code; wisp_last_error() gives the message
 *     (per host thread).  Argument checks happen on the host before anything is launched.
 *   - All array pointers are DEVICE pointers unless the name ends in _host.  Nothing here allocates,
 *     synchronises or reads device memory from the host, so every call can be captured in a CUDA
 *     graph.  Work is enqueued on `stream` (a cudaStream_t; NULL = the legacy default stream).
 *   - Kernels never trap.  A bad slot id or position found on the device sets a bit of the per-device
 *     status word (WISP_STATUS_*) and that access is skipped; wisp_device_status() reads it.
 *   - dtypes: bf16/f16 are passed as uint16_t bit patterns, fp32 as float.
 *   - Packed expert layout (byte-identical to the reference store):
 *       [codes: 3*n*bits/8 bytes | fp16 scales [3n/group] | fp16 mins [3n/group]],
 *     matrices gate [I,H], up [I,H], down [H,I] flat in that order; element e of the expert's
 *     3n-element stream sits at bit bits*e of the code region (little endian); group g covers
 *     `group` consecutive elements; value = fp32(q)*fp32(scale) + fp32(min).
 *
 * Reference citations are `path:line` in imronpuji/wisp-runtime 0.1.0.
 */
#ifndef WISP_B200_H
#define WISP_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WISP_OK 0
#define WISP_ERR_INVALID 1     /* bad argument (shape, dtype, size, alignment) */
#define WISP_ERR_CUDA 2        /* a CUDA runtime call or launch failed */
#define WISP_ERR_UNSUPPORTED 3 /* valid input this build does not handle */

#define WISP_STATUS_BAD_SLOT 0x1u    /* a slot id outside [0, nslots) was skipped */
#define WISP_STATUS_BAD_POS 0x2u     /* a position outside the KV capacity was skipped */
#define WISP_STATUS_WAIT_TIMEOUT 0x4u /* a bounded device-side wait gave up */
#define WISP_STATUS_BAD_ROUTE 0x8u   /* a routing entry (expert id / token index) was out of range */
#define WISP_STATUS_RANGE 0x10u      /* a value outside the fp16 range met an fp16 operand and was saturated */

#define WISP_DTYPE_F32 0
#define WISP_DTYPE_BF16 1
#define WISP_DTYPE_F16 2

/* ---- library ----------------------------------------------------------------------------------- */
int wisp_version(void);                 /* 10000*major + 100*minor + patch */
const char* wisp_last_error(void);      /* message of the last failed call on this host thread */
/* Reads (and with clear != 0, resets) the status word of `device`.  Synchronises that device. */
int wisp_device_status(int device, int clear, uint32_t* status_host);

/* Bytes of one packed expert of 3*n elements, or -1 if the shape is invalid.
 * Replaces wisp/quant.py:17-22 (expert_nbytes). */
int64_t wisp_expert_nbytes(int64_t n, int bits, int group);

/* ---- packed format ------------------------------------------------------------------------------ */
/* Quantize `batch` experts [batch, 3, n] (w_dtype F32 or BF16) into `out` [batch, nbytes] with
 * nbytes = wisp_expert_nbytes(n, bits, group), bit-exact with the reference RTN min/max quantizer
 * (fp32 math, fp16 round-to-nearest-even scale/min, half-to-even code rounding).
 * bits in {16, 8, 4, 3, 2}.  Replaces wisp/quant.py:60-73 (quantize) and the per-expert loop of
 * wisp/store.py:38-40 (put). */
int wisp_quantize(const void* w3, int w_dtype, int64_t batch, int64_t n, int bits, int group, uint8_t* out,
                  void* stream);

/* Dequantize rows of a packed pool [pool_rows, nbytes] into bf16 [nrows, 3, n], bit-exact with the
 * reference (fp32 q*s then +m, each rounded, then round-to-nearest-even to bf16).  `rows` (int64
 * [nrows]) selects pool rows; NULL means rows 0..nrows-1.  Replaces wisp/quant.py:76-111
 * (dequant / dequant_fast) and the gather of wisp/cache.py:121-127 (weights_batched). */
int wisp_dequant(const uint8_t* pool, int64_t pool_rows, int64_t nbytes, const int64_t* rows, int64_t nrows,
                 int64_t n, int bits, int group, uint16_t* out_bf16, void* stream);

/* Integer codes of rows of a packed pool -> uint8 [nrows, 3n].  Same row selection as wisp_dequant.
 * Replaces wisp/quant.py:44-57 (_unpack) for the code-level parity probe. */
int wisp_unpack_codes(const uint8_t* pool, int64_t pool_rows, int64_t nbytes, const int64_t* rows, int64_t nrows,
                      int64_t n, int bits, uint8_t* codes, void* stream);

/* ---- fused MoE decode, one token ---------------------------------------------------------------- */
/* Floats of scratch every path needs for this shape: k*I (the intermediate a = silu(g) * u).
 * Host-only; -1 for an invalid shape. */
int64_t wisp_moe_scratch_floats(int k, int64_t H, int64_t I, int bits, int group);

/* out[h] = sum_j w_j * Wd_j[h,:] . (silu(Wg_j x) * (Wu_j x)), dequant folded into the dot products,
 * weights read straight from the slot pool.  meta: fp32 [2k] = [slot_0..slot_{k-1}, w_0..w_{k-1}] on
 * the device.  x, out: bf16 [H].  scratch: fp32 [scratch_floats], at least k*I (the intermediate
 * a = silu(g) * u).
 * bits in {8, 4, 3, 2}; H, I multiples of 32 and of group; group a multiple of 32; pool 16-byte
 * aligned with nbytes a multiple of 16.
 * Replaces wisp/kernels.py:188-203 (moe_decode_q4_fast), :310-322 (moe_decode_q3_fast), and adds the
 * 2-bit and 8-bit variants the reference runs through dequant + bmm (wisp/moe.py:122-130). */
int wisp_moe_decode(const uint8_t* pool, int64_t nslots, int64_t nbytes, const float* meta, int k,
                    const uint16_t* x, int64_t H, int64_t I, int bits, int group, float* scratch, int64_t scratch_floats,
                    uint16_t* out, void* stream);

/* Same computation with an explicit kernel choice: 0 = automatic (what wisp_moe_decode does),
 * 1 = warp-per-row CUDA-core kernels (any supported shape), 2 = TMA bulk copies into shared memory
 * feeding the warp-level integer MMA (u8 codes x int8 activation limbs, exact int32 sums), gate/up
 * and down as two kernels chained by programmatic dependent launch, the gate/up grid pulling the
 * down rows into L2 while it computes (bits 4/3/2, group a multiple of 128, H and I multiples of
 * 128, k <= 32, at most 16 output rows per SM; WISP_ERR_UNSUPPORTED otherwise).
 * Automatic = 2 when it applies, else 1. */
int wisp_moe_decode_variant(const uint8_t* pool, int64_t nslots, int64_t nbytes, const float* meta, int k,
                            const uint16_t* x, int64_t H, int64_t I, int bits, int group, float* scratch,
                            int64_t scratch_floats, uint16_t* out, int variant, void* stream);

/* wisp_moe_decode with the router's top-k folded into the MoE kernels: every CTA computes the
 * routing from the router logits (bf16 [E], E <= 512) itself -- softmax in fp32, the k largest (ties:
 * lower expert id), renormalised when norm_topk, bf16 weights; slot of expert e = slot_table[base + e]
 * when slot_table is given (a negative entry is skipped and flagged), else base + e.  row (nullable)
 * receives [k experts | k weights] as fp32.  Tensor-core shapes only (WISP_ERR_UNSUPPORTED otherwise).
 * Replaces wisp/graphdec.py:177-182 + :194-203 (router softmax/top-k, then moe_decode_q*_fast). */
int wisp_moe_decode_routed(const uint8_t* pool, int64_t nslots, int64_t nbytes, const uint16_t* logits, int E, int k,
                           int norm_topk, const int32_t* slot_table, int64_t base, float* row, const uint16_t* x, int64_t H,
                           int64_t I, int bits, int group, float* scratch, int64_t scratch_floats, uint16_t* out, void* stream);

/* wisp_moe_decode_routed over a partially resident expert pool with no host decision: slot_table
 * (int32 [host_rows], required) maps key = base + e to a slot, or to a negative value when the expert
 * is not resident; such experts are read by the kernels from store_host, one pinned host allocation of
 * host_rows * nbytes bytes whose row `key` is that expert (the ExpertStore layout), so the call needs
 * no synchronisation and a whole decode step stays one CUDA graph.  miss_count (nullable int32 on the
 * device) is incremented once per expert read from store_host.  The table may be rewritten by
 * copies on other streams while the call runs: an entry is read once per CTA through L2, and both
 * sources of an expert hold the same bytes, so either answer is correct.  Replaces the per-layer host
 * decision of the reference's paged decoder (wisp/graphdec.py:216-235, :296-308: row to the host,
 * cache.ensure / split, slots into meta) and its hybrid miss path (wisp/moe.py:152-164: misses
 * computed outside the cache, cache.admit_async, wisp/cache.py:96-104). */
int wisp_moe_decode_paged(const uint8_t* pool, int64_t nslots, int64_t nbytes, const uint16_t* logits, int E, int k,
                          int norm_topk, const int32_t* slot_table, int64_t base, const uint8_t* store_host, int64_t host_rows,
                          int* miss_count, float* row, const uint16_t* x, int64_t H, int64_t I, int bits, int group,
                          float* scratch, int64_t scratch_floats, uint16_t* out, void* stream);

/* ---- batched MoE decode ------------------------------------------------------------------------ */
/* Bytes of the workspace wisp_moe_batched needs for N tokens of k choices (host-only; -1 if N*k is
 * outside [1, 2048]). */
int64_t wisp_moe_batched_workspace_bytes(int N, int k, int64_t H, int64_t I);

/* MoE of N tokens: meta fp32 [N, 2k] = per token [k slots | k weights]; x bf16 [N, H]; out bf16 [N, H],
 * out[t] = sum_j w[t,j] * Wd_j (silu(Wg_j x_t) * (Wu_j x_t)).  The (token, choice) pairs are grouped by
 * slot on the device, so each routed expert's weights are read once per call; the products run on the
 * tensor cores with the weights dequantized bit-exactly to bf16 (q*s + m).  bits 8/4/3/2, H and I
 * multiples of 128, group a multiple of 32; workspace 256-byte aligned, of the size above.  A slot of
 * -1 marks an empty pair (contributes nothing); other invalid slots are skipped and flagged.
 * Replaces the reference's bs > 1 MoE (wisp/moe.py:62-137: unique experts, dequant, per-expert MLP,
 * weighted index_add). */
int wisp_moe_batched(const uint8_t* pool, int64_t nslots, int64_t nbytes, const float* meta, int N, int k, const uint16_t* x,
                     int64_t H, int64_t I, int bits, int group, void* workspace, int64_t workspace_bytes, uint16_t* out,
                     void* stream);

/* wisp_moe_batched with an explicit path: 0 = automatic (what wisp_moe_batched does), 1 = the warp-level
 * tensor-core kernels (mma.sync; any supported format), 2 = the 5th-generation tensor cores: per
 * (expert, 128 weight rows, up to 64 tokens) one CTA streams the packed codes through TMA tensor
 * loads, dequantizes them once into fp16 (q*s + m with a single rounding) in the 128-byte-swizzled
 * K-major layout, and one thread issues tcgen05.mma (M = 128, N = the expert's tokens, fp32
 * accumulators in TMEM) for gate and up, then down; the activations and the intermediate enter as
 * fp16 (values outside fp16's range saturate and set WISP_STATUS_RANGE).  Path 2 needs 4-bit or
 * 2-bit codes and groups a multiple of 128 dividing H and I (WISP_ERR_UNSUPPORTED otherwise).
 * Automatic = 1 (measured faster on the 64-token Zipf layer).  Same replacement as wisp_moe_batched
 * (wisp/moe.py:62-137). */
int wisp_moe_batched_variant(const uint8_t* pool, int64_t nslots, int64_t nbytes, const float* meta, int N, int k, const uint16_t* x,
                             int64_t H, int64_t I, int bits, int group, void* workspace, int64_t workspace_bytes, uint16_t* out,
                             int variant, void* stream);

/* ---- expert parallelism (batched decode over ranks) ------------------------------------------------ */
/* Pack for the dispatch all-to-all: pair p = t*k + j of this rank's N tokens (sel: int64 [N, k] global
 * expert ids) goes to rank d = sel / E_local at capacity slot c = its rank among the pairs bound for d
 * (pair order).  send_x [world, capacity, H] bf16 gets x[t] at (d, c); send_meta [world, capacity, 2]
 * fp32 gets [slot_base + sel - d*E_local, 1] there and [-1, 0] in unused capacity (the batched MoE
 * skips those), so after the exchange the receiver's meta feeds wisp_moe_batched with k = 1;
 * src_pos [N*k] int32 = d*capacity + c for the combine.  capacity >= N*k.  Does the dispatch
 * bucketing of a pack-then-all-to-all exchange over NCCL (the reference itself has no expert parallelism). */
int wisp_ep_dispatch(const uint16_t* x, int N, int64_t H, const int64_t* sel, int k, int E_local, int world, int64_t capacity,
                     int64_t slot_base, uint16_t* send_x, float* send_meta, int32_t* src_pos, void* stream);

/* Unpack after the combine all-to-all: out[t] = bf16(sum_j w[t, j] * y_back[src_pos[t*k + j]]) with
 * the choices summed in order (w: fp32 [N, k]; y_back: bf16 [world * capacity, H]), the weighted sum of
 * wisp/moe.py:131-137 (index_add over the experts). */
int wisp_ep_combine(const uint16_t* y_back, int N, int k, int64_t H, const int32_t* src_pos, const float* w, uint16_t* out,
                    void* stream);

/* Peer-memory variant of the exchange (one process per GPU on one node, NVLink): every rank owns one
 * device allocation of wisp_ep_p2p_bytes(world, capacity, H) bytes (receive rows and routing rows,
 * returned results, flags, counters; two buffer sets) that every peer maps with CUDA IPC.
 * peers_host[r] = rank r's allocation as mapped in this process (the local one for r = rank).
 * Call n of a run (the same sequence on every rank) uses buffer set n % 2:
 *   wisp_ep_dispatch_p2p  stores this rank's rows and routing rows straight into each destination's
 *                         receive buffers and then raises its dispatch flag there (release, system scope)
 *   wisp_ep_wait          (phase 0) waits until every source's dispatch flag reached this call
 *   ...                   the batched MoE on receive rows [world * capacity, H] / routing [.., 2] of the set
 *   wisp_ep_return_p2p    stores result row (s, c) into rank s's returned-results buffer, raises its flag
 *   wisp_ep_combine_p2p   waits for every rank's return flag, then the fixed-order weighted sum
 * Waits are bounded (2 s): a peer that never signals sets WISP_STATUS_WAIT_TIMEOUT instead of hanging.
 * No TMA: peers are written with ordinary stores.  The kernel-fused form of the dispatch / combine
 * all-to-alls that wisp_ep_dispatch / wisp_ep_combine surround with NCCL. */
int wisp_ipc_alloc(int64_t bytes, void** ptr_host, uint8_t* handle_host); /* cudaMalloc (zeroed) + 64-byte IPC handle */
int wisp_ipc_open(const uint8_t* handle_host, void** ptr_host);          /* map a peer's allocation */
int wisp_ipc_close(void* ptr);
int wisp_ipc_free(void* ptr);
int64_t wisp_ep_p2p_bytes(int world, int64_t capacity, int64_t H);       /* -1 if world is outside [1, 8] */
int wisp_ep_dispatch_p2p(const uint16_t* x, int N, int64_t H, const int64_t* sel, int k, int E_local, int world, int rank,
                         int64_t capacity, int64_t slot_base, int set, void* const* peers_host, int32_t* src_pos, void* stream);
int wisp_ep_wait(void* local, int world, int64_t capacity, int64_t H, int phase, void* stream);
int wisp_ep_return_p2p(const uint16_t* y, int world, int rank, int64_t capacity, int64_t H, int set, void* const* peers_host,
                       void* stream);
int wisp_ep_combine_p2p(void* local, int world, int64_t capacity, int64_t H, int set, int N, int k, const int32_t* src_pos,
                        const float* w, uint16_t* out, void* stream);

/* ---- gpt-oss experts ------------------------------------------------------------------------------ */
/* Bytes of the workspace wisp_moe_gptoss needs (host-only; -1 if N*k is outside [1, 2048]). */
int64_t wisp_moe_gptoss_workspace_bytes(int N, int k, int64_t H, int64_t I);

/* gpt-oss MoE of N tokens: experts packed as [gate_up [H, 2I] (gate/up interleaved) | down [I, H]],
 * input-major, wisp.quant layout (H == I); meta fp32 [N, 2k] = per token [k slots | k weights],
 * experts int32 [N, k] = the expert ids (bias rows), gate_up_bias bf16 [E, 2I], down_bias bf16 [E, H].
 * out[t] = sum_j w[t,j] * (bf16(a . W_d) + b_d), a = (clamp(up, -7, 7) + 1) * g * sigmoid(1.702 g),
 * g = min(gate, 7), [gate | up] = bf16(x . W_gu) + b_gu (interleaved).
 * 4-bit codes with power-of-two groups >= 64 and 64 | H stream rows through tensor-map TMA boxes into
 * fp16 tensor-core MMAs: weights enter as q*s + m exactly and s*x, m*x are rounded to fp16 (one GEMV
 * emulated on the CPU lands within 0.25% of the bf16(q*s+m) matmul; the tests bound a whole layer
 * against the oracle at 1e-2 of its largest output); other formats dequantize bit-exactly
 * (bf16(q*s+m)) in a column kernel.  pool, x: 16-byte aligned; out and both biases: 8-byte aligned.
 * Results are bitwise repeatable (split sums in a fixed order).
 * Replaces the reference's PagedGptOssBlock expert math (wisp/gptoss.py:107-143: dequant + bmm). */
int wisp_moe_gptoss(const uint8_t* pool, int64_t nslots, int64_t nbytes, const float* meta, const int32_t* experts, int N, int k,
                    const uint16_t* x, int64_t H, int64_t I, int bits, int group, const uint16_t* gate_up_bias,
                    const uint16_t* down_bias, void* workspace, int64_t workspace_bytes, uint16_t* out, void* stream);

/* Allocation-free twin of wisp_moe_decode for callers that cannot allocate device memory (a host
 * stack that owns no allocator, e.g. a CUDA-graph node builder or an embedding runtime that hands over
 * only the pool, x and out): the fp32 intermediate a = silu(g)*u lives in a file-scope device array
 * of WISP_MOE_NOALLOC_MAX_SCRATCH floats inside the library, so no scratch argument is taken and no
 * device memory is allocated or freed.  Everything else (arguments, kernels, results) is
 * wisp_moe_decode's.  k*I must be <= WISP_MOE_NOALLOC_MAX_SCRATCH (WISP_ERR_INVALID otherwise).
 *   - Nothing in the array needs to start at zero: each call writes all k*I values before reading them.
 *   - The array is one per device and shared by every call on that device: two calls that can run at
 *     the same time (different streams, or threads without ordering) race on it.  Order them.
 *   - The array's device address belongs to a CUDA context.  The first call made in a context looks
 *     it up (cudaGetSymbolAddress, with that context current) and remembers it under the context's
 *     unique id (cuCtxGetId); later calls in the same context reuse it.  A context rebuilt by
 *     cudaDeviceReset, or a second context on the same device, has its own array and gets its own
 *     lookup on its first call.  Make the first call in each context outside stream capture.
 *   - The array's name in host code is only a host-side stand-in for the symbol, not a device
 *     address; the library passes the looked-up address to its kernels.
 * No counterpart in the reference (its kernels allocate their intermediate with torch.empty). */
#define WISP_MOE_NOALLOC_MAX_SCRATCH 65536
int wisp_moe_decode_noalloc(const uint8_t* pool, int64_t nslots, int64_t nbytes, const float* meta, int k,
                            const uint16_t* x, int64_t H, int64_t I, int bits, int group, uint16_t* out,
                            void* stream);

/* ---- decode-side ops ---------------------------------------------------------------------------- */
/* Rotate-half RoPE for one token: q [Hq, D] (head stride q_stride elements), k [Hk, D] (k_stride),
 * cos/sin bf16 [D]; writes contiguous qo [Hq, D], ko [Hk, D].  fp32 math, one rounding to bf16.
 * Replaces wisp/kernels.py:328-371 (rope_decode). */
int wisp_rope_decode(const uint16_t* q, int64_t q_stride, int Hq, const uint16_t* k, int64_t k_stride, int Hk, int D,
                     const uint16_t* cos, const uint16_t* sin, uint16_t* qo, uint16_t* ko, void* stream);

/* ---- decoder step (bs = 1) --------------------------------------------------------------------- */
/* y[n] = bf16(W[n,:] . x') for W row-major [N, K] bf16 (fp32 accumulation), where x' is x, or
 * bf16(x + x_add) when x_add is given (stored to x_sum_out when non-NULL), then RMSNorm-ed with
 * norm_w when given: x' = bf16(norm_w * bf16(x' * rsqrt(mean(x'^2) + eps))) (stored to xn_out when
 * non-NULL).  With res: y[n] = bf16(res[n] + bf16(W[n,:] . x')).  K % 8 == 0, K <= 4096; W, x,
 * x_add, norm_w, x_sum_out and xn_out 16-byte aligned; y, x_sum_out and xn_out must not alias x or
 * x_add (y may alias res).  The weight stream starts before the previous kernel in the stream ends
 * (programmatic dependent launch).
 * Replaces the bf16 nn.Linear calls of the decode step (q/k/v/o projections, the router gate, lm_head:
 * wisp/graphdec.py:160-162, :175, :177, :213) together with the RMSNorm before them and the residual
 * add after them (wisp/graphdec.py:159, :175-176, :209, :213; wisp/model.py:94-107). */
int wisp_gemv(const uint16_t* W, int64_t N, int64_t K, const uint16_t* x, const uint16_t* x_add, uint16_t* x_sum_out,
              const uint16_t* norm_w, float eps, uint16_t* xn_out, const uint16_t* res, uint16_t* y, void* stream);

/* wisp_gemv with a bias: y[n] = bf16(W[n,:] . x' + bias[n]) (fp32 sum and bias, one rounding, as a bf16
 * nn.Linear with bias gives), then y[n] = bf16(res[n] + y[n]) when res is given.  bias may be NULL.
 * Replaces the biased projections of gpt-oss attention (q/k/v/o with attention_bias, HF
 * GptOssAttention as loaded by wisp/gptoss.py:146-183). */
int wisp_gemv_bias(const uint16_t* W, int64_t N, int64_t K, const uint16_t* x, const uint16_t* x_add, uint16_t* x_sum_out,
                   const uint16_t* norm_w, float eps, uint16_t* xn_out, const uint16_t* bias, const uint16_t* res, uint16_t* y,
                   void* stream);

/* Per-head RMSNorm of the q and k heads of qkv = [Hq*D | Hk*D | Hk*D] (weights qn_w, kn_w [D]),
 * rotate-half rotary with cos/sin rows `*pos` of the [tmax, D] tables (fp32 math, one rounding), q to
 * q_out [Hq, D], k and v into row `*pos` of the caches [Hk, tmax, D].  *pos outside [0, tmax) writes
 * nothing and sets WISP_STATUS_BAD_POS.  D even, D <= 256.
 * Replaces wisp/graphdec.py:160-170 (q_norm/k_norm, rope_decode, the two index_copy_ into the cache). */
int wisp_qk_norm_rope_kv(const uint16_t* qkv, int Hq, int Hk, int D, const uint16_t* qn_w, const uint16_t* kn_w, float eps,
                         const uint16_t* cos_t, const uint16_t* sin_t, const int64_t* pos, int64_t tmax, uint16_t* q_out,
                         uint16_t* k_cache, uint16_t* v_cache, void* stream);

/* wisp_qk_norm_rope_kv for T consecutive tokens (a prefill chunk): token t's [q | k | v] heads at
 * qkv + t*qkv_stride go to position *pos0 + t -- q to q_out [T, Hq, D], k and v into the caches.
 * Positions outside [0, tmax) write nothing and set WISP_STATUS_BAD_POS.  1 <= T <= 65535.
 * Replaces the per-chunk q_norm / k_norm, apply_rotary_pos_emb and cache copies of the reference's
 * chunked prefill (wisp/graphdec.py:122-130). */
int wisp_qk_norm_rope_kv_rows(const uint16_t* qkv, int T, int64_t qkv_stride, int Hq, int Hk, int D, const uint16_t* qn_w,
                              const uint16_t* kn_w, float eps, const uint16_t* cos_t, const uint16_t* sin_t, const int64_t* pos0,
                              int64_t tmax, uint16_t* q_out, uint16_t* k_cache, uint16_t* v_cache, void* stream);

/* One decode token of each of B sequences: qkv row b (at qkv + b*qkv_stride) is sequence b's token at
 * position pos[b] (int64 [B] on the device); q goes to q_out [B, Hq, D], k and v into row pos[b] of
 * sequence b's caches (k_cache, v_cache [B, Hk, tmax, D]).  qn_w and kn_w NULL: no per-head RMSNorm
 * (models without q/k norms, e.g. gpt-oss), only the rotary embedding.
 * Replaces the per-sequence q/k norm, rotary and cache writes of a batched HF decode step
 * (wisp/graphdec.py:160-170 per sequence). */
int wisp_qk_norm_rope_kv_batched(const uint16_t* qkv, int B, int64_t qkv_stride, int Hq, int Hk, int D, const uint16_t* qn_w,
                                 const uint16_t* kn_w, float eps, const uint16_t* cos_t, const uint16_t* sin_t, const int64_t* pos,
                                 int64_t tmax, uint16_t* q_out, uint16_t* k_cache, uint16_t* v_cache, void* stream);

/* fp32 elements of the workspace wisp_gqa_decode_attn_batched needs (host-only; -1 for a bad shape). */
int64_t wisp_attn_batched_workspace_floats(int B, int Hq, int Hk, int D, int64_t tmax);

/* GQA decode attention of one token of each of B sequences: q [B, Hq, D] over positions [lo, pos[b]] of
 * sequence b's caches [B, Hk, tmax, D], lo = pos[b] - window + 1 (0 when window == 0: full attention);
 * softmax(scale * q.k) in fp32, with sinks (fp32 [Hq], nullable) as one extra logit per head that
 * enters the normalisation only; out [B, Hq, D] bf16.  Split over chunks of 64 positions, then one
 * combine launch.  Hq/Hk <= 8, D % 32 == 0, D <= 128.
 * Replaces the masked SDPA of a batched decode step, with the sliding windows and attention sinks of
 * gpt-oss attention (the HF GptOssAttention the reference's gpt-oss runs, wisp/gptoss.py:146-183). */
int wisp_gqa_decode_attn_batched(const uint16_t* q, int B, int Hq, int Hk, int D, const uint16_t* k_cache, const uint16_t* v_cache,
                                 int64_t tmax, const int64_t* pos, int window, const float* sinks, float scale, float* workspace,
                                 int64_t workspace_floats, uint16_t* out, void* stream);

/* wisp_qk_norm_rope_kv_batched and wisp_gqa_decode_attn_batched in one pass over the cache: qkv
 * [B, qkv_stride] holds each sequence's raw q, k, v heads; every attention CTA norms (qn_w, kn_w:
 * both or neither) and rotates its query heads itself, and the CTA whose chunk holds pos[b] makes the
 * new key / value row, writes it into the caches and uses it.  Same arithmetic, hence the same bits,
 * as the two calls; one launch fewer, but every chunk CTA re-does its query heads' norm and rotary, so
 * it pays only at short contexts (at 64 sequences x 4096 positions the two calls measured 14.5 ms per
 * 48-layer step against 18.3 ms with this form).  D = 64 or 128 (WISP_ERR_UNSUPPORTED otherwise). */
int wisp_attn_decode_batched(const uint16_t* qkv, int64_t qkv_stride, int B, int Hq, int Hk, int D, const uint16_t* qn_w,
                             const uint16_t* kn_w, float eps, const uint16_t* cos_t, const uint16_t* sin_t, uint16_t* k_cache,
                             uint16_t* v_cache, int64_t tmax, const int64_t* pos, int window, const float* sinks, float scale,
                             float* workspace, int64_t workspace_floats, uint16_t* out, void* stream);

/* fp32 elements of the workspace wisp_gqa_decode_attn needs (host-only; -1 for a bad shape). */
int64_t wisp_attn_workspace_floats(int Hq, int Hk, int D, int64_t tmax);

/* GQA decode attention of one token: q [Hq, D] (query head i uses KV head i / (Hq/Hk)) over cache
 * positions 0..*pos of k_cache, v_cache [Hk, tmax, D]; softmax(scale * q.k) fp32; out [Hq, D] bf16.
 * Split over chunks of 64 positions, then one combine launch.  Hq/Hk <= 8, D % 32 == 0, D <= 128.
 * Replaces wisp/graphdec.py:171-174 (SDPA over the static cache with mask ar <= pos) and the patched
 * decode attention of wisp/model.py:136-150. */
int wisp_gqa_decode_attn(const uint16_t* q, int Hq, int Hk, int D, const uint16_t* k_cache, const uint16_t* v_cache, int64_t tmax,
                         const int64_t* pos, float scale, float* workspace, uint16_t* out, void* stream);

/* Fused decode attention of one token: wisp_qk_norm_rope_kv and wisp_gqa_decode_attn in one launch.
 * One cluster of 16 (or 8) CTAs per KV head splits positions 0..*pos; each CTA norms and rotates its
 * query heads itself, the CTA holding *pos writes the new K/V row, scores and P.V run on the tensor
 * cores, and the partial softmax states are merged through distributed shared memory (no
 * workspace).  D == 128, Hq/Hk <= 8.
 * Replaces wisp/graphdec.py:160-174 (q/k norms, rope_decode, cache writes, masked SDPA). */
int wisp_attn_decode(const uint16_t* qkv, int Hq, int Hk, int D, const uint16_t* qn_w, const uint16_t* kn_w, float eps,
                     const uint16_t* cos_t, const uint16_t* sin_t, const int64_t* pos, int64_t tmax, uint16_t* k_cache,
                     uint16_t* v_cache, float scale, uint16_t* out, void* stream);

/* Router of one token: p = softmax(logits bf16 [E]) in fp32, the k largest (ties: lower expert id),
 * renormalised when norm_topk == 1; norm_topk == 2 (gpt-oss): softmax over the k selected logits
 * (wisp/gptoss.py:122-123); rounded to bf16.  row (nullable) = fp32 [k experts | k weights];
 * meta = fp32 [k slots | k weights], slot = slot_table[base + e] when slot_table is given, else
 * base + e.  E <= 1024, k <= 32.
 * Replaces wisp/graphdec.py:177-182 and wisp/moe.py:67-72 (softmax, topk, renormalise, bf16). */
int wisp_router_topk(const uint16_t* logits, int E, int k, int norm_topk, const int32_t* slot_table, int64_t base, float* row,
                     float* meta, void* stream);

/* Router of B tokens in one launch, one CTA per token: xn = RMSNorm(x[b]) * norm_w (wisp_rmsnorm's
 * rounding; norm_w NULL: xn = x) stored to xn_out [B, H] (nullable), logits[e] = bf16(xn . W[e] + bias[e])
 * (W [E, H] bf16, bias [E] nullable; fp32 sum, one rounding), then wisp_router_topk's selection and
 * weights (norm_topk 0, 1 or 2).  meta [B, 2k] = [k slots | k weights] (slot = slot_table[base + e]
 * or base + e); experts [B, k] int32 expert ids (nullable); row [B, 2k] fp32 [k ids | k weights]
 * (nullable).  H % 8 == 0, H <= 8192, E <= 1024, k <= 32; x, W, norm_w, xn_out 16-byte aligned.
 * Replaces the router of a batched decode step: gpt-oss (post-attention RMSNorm, F.linear with bias,
 * topk, softmax over the k: wisp/gptoss.py:116-123) and Qwen3-MoE (gate, softmax, topk, renormalise:
 * wisp/moe.py:67-72). */
int wisp_router_rows(const uint16_t* x, int B, int64_t H, const uint16_t* norm_w, float eps, uint16_t* xn_out, const uint16_t* W,
                     const uint16_t* bias, int E, int k, int norm_topk, const int32_t* slot_table, int64_t base, float* meta,
                     int32_t* experts, float* row, void* stream);

/* Bytes of the workspace of wisp_router_rows_ws (host-only; -1 for a bad shape). */
int64_t wisp_router_workspace_bytes(int B, int E);

/* wisp_router_rows with the gate split over CTAs (grid B x ceil(E / 4), one warp per expert): each
 * CTA norms its token's row and computes four logits into the workspace; the last CTA of a token (an
 * arrival counter in the workspace) runs the top-k and resets its counter.  The workspace (256-byte
 * aligned, wisp_router_workspace_bytes(B, E) bytes) must be zero-filled before its first use and is
 * left ready for the next launch; calls sharing one workspace must not overlap.  NULL workspace: the
 * one-CTA-per-token kernel of wisp_router_rows.  Same results either way. */
int wisp_router_rows_ws(const uint16_t* x, int B, int64_t H, const uint16_t* norm_w, float eps, uint16_t* xn_out, const uint16_t* W,
                        const uint16_t* bias, int E, int k, int norm_topk, const int32_t* slot_table, int64_t base, float* meta,
                        int32_t* experts, float* row, void* workspace, int64_t workspace_bytes, void* stream);

/* out [H] = table[*token] (bf16 rows, H % 8 == 0).  *token outside [0, V) sets WISP_STATUS_BAD_ROUTE. */
int wisp_embed(const uint16_t* table, int64_t V, int64_t H, const int64_t* token, uint16_t* out, void* stream);

/* *out = the index of the largest of x[0..n) (bf16; ties: the lower index; NaN never wins), over a
 * workspace of WISP_ARGMAX_WORKSPACE u64. */
#define WISP_ARGMAX_WORKSPACE 256
int wisp_argmax(const uint16_t* x, int64_t n, uint64_t* workspace, int64_t* out, void* stream);

/* RMSNorm of `rows` rows of H bf16 values: out = bf16(w * bf16(x * rsqrt(mean(x^2) + eps))).
 * If `delta` is non-NULL the row is first replaced by bf16(x + delta) and, when `sum_out` is
 * non-NULL, that sum is stored there (the residual add fused in).
 * Replaces wisp/model.py:94-107 (patched Qwen3MoeRMSNorm) and the residual adds of
 * wisp/graphdec.py:175-176, :209. */
int wisp_rmsnorm(const uint16_t* x, const uint16_t* delta, uint16_t* sum_out, const uint16_t* w, int64_t rows,
                 int64_t H, float eps, uint16_t* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* WISP_B200_H */
