// libwisp_b200.so: the C ABI declared in include/wisp_b200.h.  One translation unit (the kernels live
// in the included .cuh files) so the per-device status word is a single __device__ symbol.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "common.cuh"
#include "ctx_cache.h"
#include "decode_ops.cuh"
#include "decoder.cuh"
#include "dense.cuh"
#include "moe_decode.cuh"
#include "moe_decode_v4.cuh"
#include "moe_batched.cuh"
#include "moe_batched_umma.cuh"
#include "moe_gptoss.cuh"
#include "ep.cuh"
#include "quant.cuh"

namespace wisp {

std::string& last_error_slot() {
  static thread_local std::string s;
  return s;
}

static int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

static int64_t grid_for(int64_t work, int threads, int per_sm = 8) {
  int64_t g = (work + threads - 1) / threads;
  const int64_t cap = int64_t(sm_count()) * per_sm;
  if (g > cap) g = cap;
  return g < 1 ? 1 : g;
}

static bool valid_bits(int b) { return b == 16 || b == 8 || b == 4 || b == 3 || b == 2; }

}  // namespace wisp

using namespace wisp;

extern "C" {

int wisp_version(void) { return 100; }

const char* wisp_last_error(void) { return last_error_slot().c_str(); }

int wisp_device_status(int device, int clear, uint32_t* status_host) {
  WISP_REQUIRE(status_host != nullptr, "wisp_device_status: status_host is NULL");
  int prev = 0;
  cudaGetDevice(&prev);
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
  unsigned int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_status, sizeof(v));
  if (e == cudaSuccess && clear) {
    unsigned int z = 0;
    e = cudaMemcpyToSymbol(g_status, &z, sizeof(z));
  }
  cudaSetDevice(prev);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_device_status: %s", cudaGetErrorString(e));
  *status_host = v;
  return WISP_OK;
}

int64_t wisp_expert_nbytes(int64_t n, int bits, int group) {
  if (n <= 0 || !valid_bits(bits)) return -1;
  if (bits == 16) return 3 * n * 2;
  if (group <= 0 || (3 * n) % group != 0 || (3 * n * bits) % 8 != 0) return -1;
  return (3 * n * bits) / 8 + 4 * (3 * n / group);
}

int wisp_quantize(const void* w3, int w_dtype, int64_t batch, int64_t n, int bits, int group, uint8_t* out,
                  void* stream) {
  WISP_REQUIRE(w3 && out, "wisp_quantize: NULL pointer");
  WISP_REQUIRE(batch >= 0, "wisp_quantize: negative batch");
  if (batch == 0) return WISP_OK;
  WISP_REQUIRE(w_dtype == WISP_DTYPE_F32 || w_dtype == WISP_DTYPE_BF16, "wisp_quantize: w_dtype must be F32 or BF16");
  const int64_t nb = wisp_expert_nbytes(n, bits, group);
  WISP_REQUIRE(nb > 0, "wisp_quantize: invalid shape n=%lld bits=%d group=%d", (long long)n, bits, group);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (bits == 16) {
    const int64_t cnt = batch * 3 * n;
    if (w_dtype == WISP_DTYPE_F32)
      to_bf16_kernel<float><<<grid_for(cnt, 256), 256, 0, s>>>(static_cast<const float*>(w3), cnt, reinterpret_cast<uint16_t*>(out));
    else
      to_bf16_kernel<uint16_t><<<grid_for(cnt, 256), 256, 0, s>>>(static_cast<const uint16_t*>(w3), cnt, reinterpret_cast<uint16_t*>(out));
    return check_launch("quantize(16)");
  }
  WISP_REQUIRE(group % 8 == 0, "wisp_quantize: group must be a multiple of 8 (got %d)", group);
  if ((3 * n * bits / 8) % 2 != 0)
    return fail(WISP_ERR_UNSUPPORTED, "wisp_quantize: the code region (3*n*bits/8 bytes) must be even so the fp16 scales stay aligned");
  WISP_REQUIRE(aligned(out, 8) && (batch == 1 || nb % 8 == 0), "wisp_quantize: out rows must be 8-byte aligned");
  const int64_t ngroups = 3 * n / group;
  const int64_t ncode = 3 * n * bits / 8;
  const int64_t grid = (batch * ngroups * 32 + 255) / 256;
#define WISP_Q(B)                                                                                           \
  if (w_dtype == WISP_DTYPE_F32)                                                                            \
    quantize_kernel<B, float><<<grid, 256, 0, s>>>(static_cast<const float*>(w3), batch, ngroups, group, out, ncode, nb); \
  else                                                                                                      \
    quantize_kernel<B, uint16_t><<<grid, 256, 0, s>>>(static_cast<const uint16_t*>(w3), batch, ngroups, group, out, ncode, nb);
  switch (bits) {
    case 8: WISP_Q(8) break;
    case 4: WISP_Q(4) break;
    case 3: WISP_Q(3) break;
    case 2: WISP_Q(2) break;
  }
#undef WISP_Q
  return check_launch("quantize");
}

static int unpack_common(const uint8_t* pool, int64_t pool_rows, int64_t nbytes, const int64_t* rows, int64_t nrows,
                         int64_t n, int bits, int group, void* out, int mode, void* stream) {
  WISP_REQUIRE(pool && out, "NULL pointer");
  WISP_REQUIRE(nrows >= 0 && pool_rows >= 0, "negative row count");
  if (mode == 0) {
    const int64_t nb = wisp_expert_nbytes(n, bits, group);
    WISP_REQUIRE(nb > 0 && nb == nbytes, "nbytes=%lld does not match n=%lld bits=%d group=%d (expected %lld)",
                 (long long)nbytes, (long long)n, bits, group, (long long)nb);
  } else {
    WISP_REQUIRE(n > 0 && nbytes >= 3 * n * bits / 8, "nbytes=%lld smaller than the code region", (long long)nbytes);
    group = 32;  // unused for codes
  }
  WISP_REQUIRE(aligned(pool, 16) && nbytes % 16 == 0, "pool must be 16-byte aligned with nbytes a multiple of 16");
  WISP_REQUIRE(aligned(out, 16), "out must be 16-byte aligned");
  if (nrows == 0) return WISP_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (bits == 16) {
    WISP_REQUIRE(mode == 0, "16-bit experts have no codes");
    gather_rows_kernel<<<grid_for(nrows * nbytes / 16, 256), 256, 0, s>>>(pool, pool_rows, nbytes, rows, nrows,
                                                                          static_cast<uint8_t*>(out));
    return check_launch("dequant(16)");
  }
  if (n % 32 != 0) return fail(WISP_ERR_UNSUPPORTED, "n must be a multiple of 32 (got %lld)", (long long)n);
  const int64_t work = nrows * (3 * n / 32);
  const int64_t grid = grid_for(work, 256);
#define WISP_U(B)                                                                                                \
  if (mode == 0)                                                                                                 \
    unpack_kernel<B, 0><<<grid, 256, 0, s>>>(pool, pool_rows, nbytes, rows, nrows, n, group, out);               \
  else                                                                                                           \
    unpack_kernel<B, 1><<<grid, 256, 0, s>>>(pool, pool_rows, nbytes, rows, nrows, n, group, out);
  switch (bits) {
    case 8: WISP_U(8) break;
    case 4: WISP_U(4) break;
    case 3: WISP_U(3) break;
    case 2: WISP_U(2) break;
  }
#undef WISP_U
  return check_launch(mode == 0 ? "dequant" : "unpack_codes");
}

int wisp_dequant(const uint8_t* pool, int64_t pool_rows, int64_t nbytes, const int64_t* rows, int64_t nrows, int64_t n,
                 int bits, int group, uint16_t* out_bf16, void* stream) {
  return unpack_common(pool, pool_rows, nbytes, rows, nrows, n, bits, group, out_bf16, 0, stream);
}

int wisp_unpack_codes(const uint8_t* pool, int64_t pool_rows, int64_t nbytes, const int64_t* rows, int64_t nrows,
                      int64_t n, int bits, uint8_t* codes, void* stream) {
  WISP_REQUIRE(bits != 16, "wisp_unpack_codes: 16-bit experts have no codes");
  return unpack_common(pool, pool_rows, nbytes, rows, nrows, n, bits, 32, codes, 1, stream);
}

}  // extern "C"

static int moe_shape(const uint8_t* pool, int64_t nslots, int64_t nbytes, const float* meta, int k, const uint16_t* x,
                     int64_t H, int64_t I, int bits, int group, const float* scratch, const uint16_t* out, MoeShape& S) {
  WISP_REQUIRE(pool && meta && x && scratch && out, "wisp_moe_decode: NULL pointer");
  WISP_REQUIRE(bits == 8 || bits == 4 || bits == 3 || bits == 2, "wisp_moe_decode: bits must be 8, 4, 3 or 2 (got %d)", bits);
  WISP_REQUIRE(k >= 1 && k <= 64, "wisp_moe_decode: k must be in [1, 64] (got %d)", k);
  WISP_REQUIRE(group > 0 && group % 32 == 0, "wisp_moe_decode: group must be a positive multiple of 32 (got %d)", group);
  WISP_REQUIRE(H > 0 && I > 0 && H % group == 0 && I % group == 0,
               "wisp_moe_decode: H and I must be multiples of group (H=%lld I=%lld group=%d)", (long long)H, (long long)I, group);
  const int64_t n = H * I;
  const int64_t nb = wisp_expert_nbytes(n, bits, group);
  WISP_REQUIRE(nb == nbytes, "wisp_moe_decode: nbytes=%lld, expected %lld", (long long)nbytes, (long long)nb);
  WISP_REQUIRE(aligned(pool, 16) && nbytes % 16 == 0, "wisp_moe_decode: pool must be 16-byte aligned, nbytes % 16 == 0");
  WISP_REQUIRE(aligned(x, 16) && aligned(scratch, 16), "wisp_moe_decode: x and scratch must be 16-byte aligned");
  WISP_REQUIRE(H <= 4096 && I <= 4096, "wisp_moe_decode: H and I up to 4096 are supported");
  S.nslots = nslots;
  S.nbytes = nbytes;
  S.k = k;
  S.H = int(H);
  S.I = int(I);
  S.group = group;
  S.ncode = 3 * n * bits / 8;
  S.ng = 3 * n / group;
  S.mat_bytes = n * bits / 8;
  S.gshift = 0;
  for (int gq = group / 128; gq > 1 && (gq & 1) == 0; gq >>= 1) ++S.gshift;
  S.glog = log2_or_neg(group);
  S.dn_beside = 0;
  return WISP_OK;
}

// The opt-in for dynamic shared memory beyond 48 KB is an attribute of the kernel function, and a
// captured graph node keeps its launch's size while the attribute keeps whatever was set last.  So
// the attribute only ever grows: a later launch of the same kernel with less shared memory (a GEMV of
// smaller K) must not lower it under a node captured earlier with more (profilers and graph updates
// re-launch nodes against the function's current attribute).
static void raise_smem_limit(const void* fn, size_t smem) {
  if (smem == 0) return;
  static std::mutex mu;
  struct Entry {
    const void* fn;
    int dev;
    size_t smem;
  };
  static Entry seen[512];
  static int nseen = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < nseen; ++i)
    if (seen[i].fn == fn && seen[i].dev == dev) {
      if (smem > seen[i].smem && cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) == cudaSuccess)
        seen[i].smem = smem;
      return;
    }
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) == cudaSuccess && nseen < 512)
    seen[nseen++] = Entry{fn, dev, smem};
}

static int v1_launch(const uint8_t* pool, const float* meta, const uint16_t* x, const MoeShape& S, int bits,
                     float* scratch, uint16_t* out, cudaStream_t s) {
  const int64_t H = S.H, I = S.I;
  const int k = S.k;
  const int upl_gu = int((H / 32 + 31) / 32);
  const int upl_dn = int((I / 32 + 31) / 32);
  const int UP = int(I / 32) | 1;
  const size_t smem = size_t(k) * 32 * UP * 4 + size_t(k) * (I / 32) * 4;
  WISP_REQUIRE(smem <= 200 * 1024, "wisp_moe_decode: k*I too large for the shared-memory stage");
  constexpr int RPW = 2;
  dim3 g1((unsigned)((I + 8 * RPW - 1) / (8 * RPW)), (unsigned)k);
  dim3 g2((unsigned)((H + 7) / 8));
#define WISP_GU(B, U) moe_gate_up_kernel<B, U, RPW><<<g1, 256, 0, s>>>(pool, meta, x, S, scratch)
#define WISP_DN(B, U)                                                                                   \
  do {                                                                                                  \
    auto kern = moe_down_kernel<B, U>;                                                                  \
    if (smem > 48 * 1024) raise_smem_limit(reinterpret_cast<const void*>(kern), smem);                   \
    kern<<<g2, 256, smem, s>>>(pool, meta, scratch, S, out);                                            \
  } while (0)
#define WISP_BITS(B)                                   \
  {                                                    \
    if (upl_gu <= 1) WISP_GU(B, 1);                    \
    else if (upl_gu <= 2) WISP_GU(B, 2);               \
    else WISP_GU(B, 4);                                \
    int rc = check_launch("moe_decode gate/up");       \
    if (rc) return rc;                                 \
    if (upl_dn <= 1) WISP_DN(B, 1);                    \
    else if (upl_dn <= 2) WISP_DN(B, 2);               \
    else WISP_DN(B, 4);                                \
  }
  switch (bits) {
    case 8: WISP_BITS(8) break;
    case 4: WISP_BITS(4) break;
    case 3: WISP_BITS(3) break;
    case 2: WISP_BITS(2) break;
  }
#undef WISP_BITS
#undef WISP_GU
#undef WISP_DN
  return check_launch("moe_decode down");
}

static int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return sm_count();
  if (!cached[dev]) cached[dev] = sm_count();
  return cached[dev];
}

template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, int block, size_t smem, cudaStream_t s, Args... args) {
  // dynamic shared memory beyond the default 48 KB window (static + dynamic) needs the opt-in
  raise_smem_limit(reinterpret_cast<const void*>(kern), smem);
  if (smem > 48 * 1024) {
    // the whole unified L1 as shared memory, so CTAs of the next kernel in a PDL chain fit beside
    // this one's (the carveout is chosen per launch; a smaller one would keep them out)
    cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, int(cudaSharedmemCarveoutMaxShared));
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// the two-kernel tensor-core pipeline applies when: 4/3/2-bit codes, quantization groups made of whole
// 128-code MMA groups, 8-row blocks never straddling experts, at most 16 down rows per CTA, k <= 32
// (one copy lane per routed expert), and both kernels' shared memory fits
static bool v4_supported(const MoeShape& S, int bits, int nctas) {
  if (bits != 4 && bits != 3 && bits != 2) return false;
  if (S.group % 128 != 0 || (128 << S.gshift) != S.group || S.H % 128 != 0 || S.I % 128 != 0) return false;
  if (S.ncode % 16 || S.mat_bytes % 16 || (int64_t(S.H) * bits / 8) % 16 || (int64_t(S.I) * bits / 8) % 16) return false;
  if ((S.H + nctas - 1) / nctas > 16) return false;
  if (S.k > 32) return false;
  const v4::GuL Lg = v4::gu_layout(S.H, S.I, S.k, S.group, bits, nctas);
  const v4::DnL Ld = v4::dn_layout(S.H, S.I, S.k, S.group, bits, nctas);
  return Lg.R > 0 && Ld.bytes <= v4::SMEM_LIMIT;
}

static int v4_launch(const uint8_t* pool, const float* meta, const uint16_t* x, const MoeShape& S_in, int bits,
                     float* scratch, uint16_t* out, cudaStream_t s, int nctas, const MoeRoute& RT = MoeRoute{}) {
  const int64_t gsm = v4::gu_layout(S_in.H, S_in.I, S_in.k, S_in.group, bits, nctas).bytes;
  const v4::DnL Ld = v4::dn_layout(S_in.H, S_in.I, S_in.k, S_in.group, bits, nctas);
  // registers always allow a down CTA beside a gate/up CTA; shared memory (1 KB reserved per CTA) decides
  MoeShape S = S_in;
  S.dn_beside = gsm + Ld.bytes + 2 * 1024 <= int64_t(v4::SM_SMEM_BYTES);
  cudaError_t e = cudaSuccess;
  const bool paged = RT.host_store != nullptr;
#define WISP_V4(B)                                                                                                    \
  e = paged ? launch_pdl(v4::gate_up_kernel<B, true>, nctas, v4::GU_THREADS, size_t(gsm), s, pool, meta, x, S, scratch, RT)   \
            : launch_pdl(v4::gate_up_kernel<B, false>, nctas, v4::GU_THREADS, size_t(gsm), s, pool, meta, x, S, scratch, RT); \
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "moe_decode gate/up: %s", cudaGetErrorString(e));                  \
  e = paged ? launch_pdl(v4::down_kernel<B, true>, nctas, v4::DN_THREADS, size_t(Ld.bytes), s, pool, meta,              \
                         (const float*)scratch, S, out, RT)                                                           \
            : launch_pdl(v4::down_kernel<B, false>, nctas, v4::DN_THREADS, size_t(Ld.bytes), s, pool, meta,             \
                         (const float*)scratch, S, out, RT);
  switch (bits) {
    case 4: WISP_V4(4) break;
    case 3: WISP_V4(3) break;
    case 2: WISP_V4(2) break;
  }
#undef WISP_V4
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "moe_decode down: %s", cudaGetErrorString(e));
  return check_launch("moe_decode");
}

// ---- built-in scratch of wisp_moe_decode_noalloc -------------------------------------------------
// One instance per CUDA context that loads this module.  Its device address is looked up with
// cudaGetSymbolAddress and remembered per context, keyed on the context's unique id (cuCtxGetId), so
// a context rebuilt by cudaDeviceReset or a second context on the same device gets its own lookup.
static __device__ __align__(256) float g_noalloc_scratch[WISP_MOE_NOALLOC_MAX_SCRATCH];
static std::mutex g_noalloc_mu;
static wisp::ContextAddressTable<64> g_noalloc_addr;

struct CtxApi {
  PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
  PFN_cuCtxGetId_v12000 get_id = nullptr;
};

static const CtxApi& ctx_api() {
  static CtxApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
      api.get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
      api.get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
  });
  return api;
}

// unique id of the calling thread's current context; 0 when there is none yet
static int current_ctx_id(uint64_t* id) {
  const CtxApi& api = ctx_api();
  if (!api.get_current || !api.get_id) return fail(WISP_ERR_CUDA, "wisp_moe_decode_noalloc: cuCtxGetCurrent / cuCtxGetId unavailable");
  CUcontext ctx = nullptr;
  if (api.get_current(&ctx) != CUDA_SUCCESS) return fail(WISP_ERR_CUDA, "wisp_moe_decode_noalloc: cuCtxGetCurrent failed");
  *id = 0;
  if (!ctx) return WISP_OK;
  unsigned long long v = 0;
  if (api.get_id(ctx, &v) != CUDA_SUCCESS) return fail(WISP_ERR_CUDA, "wisp_moe_decode_noalloc: cuCtxGetId failed");
  *id = uint64_t(v);
  return WISP_OK;
}

// the current context's array, looked up on the first call made in that context
static int noalloc_scratch(float** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_moe_decode_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  uint64_t id = 0;
  int rc = current_ctx_id(&id);
  if (rc) return rc;
  void* p = id ? g_noalloc_addr.find(id) : nullptr;
  if (!p) {
    // also makes the runtime bind the device's primary context when no context is current yet
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(WISP_ERR_CUDA, "wisp_moe_decode_noalloc: cudaGetSymbolAddress on device %d: %s", dev, cudaGetErrorString(e));
    if (!id && (rc = current_ctx_id(&id))) return rc;
    if (id) g_noalloc_addr.put(id, p);
  }
  *out = static_cast<float*>(p);
  return WISP_OK;
}

extern "C" {

int64_t wisp_moe_scratch_floats(int k, int64_t H, int64_t I, int bits, int group) {
  (void)H, (void)bits, (void)group;
  if (k < 1 || H <= 0 || I <= 0) return -1;
  return int64_t(k) * I;
}

int wisp_moe_decode_variant(const uint8_t* pool, int64_t nslots, int64_t nbytes, const float* meta, int k,
                            const uint16_t* x, int64_t H, int64_t I, int bits, int group, float* scratch, int64_t scratch_floats,
                            uint16_t* out, int variant, void* stream) {
  MoeShape S;
  int rc = moe_shape(pool, nslots, nbytes, meta, k, x, H, I, bits, group, scratch, out, S);
  if (rc) return rc;
  WISP_REQUIRE(variant >= 0 && variant <= 2, "wisp_moe_decode_variant: variant must be 0 (auto), 1 or 2");
  WISP_REQUIRE(scratch_floats >= int64_t(k) * I, "wisp_moe_decode: scratch of %lld floats, need at least k*I = %lld",
               (long long)scratch_floats, (long long)(int64_t(k) * I));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int nctas = num_sms();
  const bool ok2 = v4_supported(S, bits, nctas);
  if (variant == 2 && !ok2) return fail(WISP_ERR_UNSUPPORTED, "wisp_moe_decode_variant: shape not supported by variant 2");
  if (variant == 2 || (variant == 0 && ok2)) return v4_launch(pool, meta, x, S, bits, scratch, out, s, nctas);
  return v1_launch(pool, meta, x, S, bits, scratch, out, s);
}

int wisp_moe_decode(const uint8_t* pool, int64_t nslots, int64_t nbytes, const float* meta, int k, const uint16_t* x,
                    int64_t H, int64_t I, int bits, int group, float* scratch, int64_t scratch_floats, uint16_t* out,
                    void* stream) {
  return wisp_moe_decode_variant(pool, nslots, nbytes, meta, k, x, H, I, bits, group, scratch, scratch_floats, out, 0, stream);
}

int wisp_moe_decode_routed(const uint8_t* pool, int64_t nslots, int64_t nbytes, const uint16_t* logits, int E, int k,
                           int norm_topk, const int32_t* slot_table, int64_t base, float* row, const uint16_t* x, int64_t H,
                           int64_t I, int bits, int group, float* scratch, int64_t scratch_floats, uint16_t* out, void* stream) {
  WISP_REQUIRE(logits, "wisp_moe_decode_routed: NULL logits");
  WISP_REQUIRE(E >= 1 && E <= v4::GU_THREADS && E <= v4::DN_THREADS && k >= 1 && k <= E,
               "wisp_moe_decode_routed: need 1 <= k <= E <= %d", v4::GU_THREADS);
  MoeShape S;
  // the routing lives in shared memory; moe_shape only needs a non-NULL meta to validate the rest
  int rc = moe_shape(pool, nslots, nbytes, reinterpret_cast<const float*>(logits), k, x, H, I, bits, group, scratch, out, S);
  if (rc) return rc;
  const int nctas = num_sms();
  if (!v4_supported(S, bits, nctas))
    return fail(WISP_ERR_UNSUPPORTED, "wisp_moe_decode_routed: shape not supported by the tensor-core kernels");
  WISP_REQUIRE(scratch_floats >= int64_t(k) * I, "wisp_moe_decode_routed: scratch of %lld floats, need at least k*I = %lld",
               (long long)scratch_floats, (long long)(int64_t(k) * I));
  MoeRoute RT{logits, E, norm_topk, slot_table, base, row};
  return v4_launch(pool, nullptr, x, S, bits, scratch, out, static_cast<cudaStream_t>(stream), nctas, RT);
}

// Device address of [p, p + bytes) in pinned host memory, or NULL when the range is not one mapped
// pinned allocation (the last answer is kept: the decoder asks once before capturing its graph).
static const uint8_t* mapped_host_range(const uint8_t* p, int64_t bytes) {
  static std::mutex mu;
  static const uint8_t *last_p = nullptr, *last_dev = nullptr;
  static int64_t last_bytes = 0;
  static int last_device = -1;
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (p == last_p && bytes == last_bytes && device == last_device) return last_dev;
  cudaPointerAttributes a0{}, a1{};
  if (cudaPointerGetAttributes(&a0, p) != cudaSuccess || cudaPointerGetAttributes(&a1, p + bytes - 1) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (a0.type != cudaMemoryTypeHost || a1.type != cudaMemoryTypeHost || !a0.devicePointer || !a1.devicePointer) return nullptr;
  const uint8_t* d0 = static_cast<const uint8_t*>(a0.devicePointer);
  if (static_cast<const uint8_t*>(a1.devicePointer) != d0 + bytes - 1) return nullptr;  // not one contiguous mapping
  last_p = p, last_bytes = bytes, last_device = device, last_dev = d0;
  return d0;
}

int wisp_moe_decode_paged(const uint8_t* pool, int64_t nslots, int64_t nbytes, const uint16_t* logits, int E, int k,
                          int norm_topk, const int32_t* slot_table, int64_t base, const uint8_t* store_host, int64_t host_rows,
                          int* miss_count, float* row, const uint16_t* x, int64_t H, int64_t I, int bits, int group,
                          float* scratch, int64_t scratch_floats, uint16_t* out, void* stream) {
  WISP_REQUIRE(logits && slot_table && store_host, "wisp_moe_decode_paged: NULL logits, slot_table or store_host");
  WISP_REQUIRE(E >= 1 && E <= v4::GU_THREADS && E <= v4::DN_THREADS && k >= 1 && k <= E,
               "wisp_moe_decode_paged: need 1 <= k <= E <= %d", v4::GU_THREADS);
  WISP_REQUIRE(base >= 0 && host_rows >= base + E, "wisp_moe_decode_paged: host store of %lld rows has no row %lld",
               (long long)host_rows, (long long)(base + E - 1));
  MoeShape S;
  int rc = moe_shape(pool, nslots, nbytes, reinterpret_cast<const float*>(logits), k, x, H, I, bits, group, scratch, out, S);
  if (rc) return rc;
  const int nctas = num_sms();
  if (!v4_supported(S, bits, nctas))
    return fail(WISP_ERR_UNSUPPORTED, "wisp_moe_decode_paged: shape not supported by the tensor-core kernels");
  const uint8_t* hs = mapped_host_range(store_host, host_rows * nbytes);
  WISP_REQUIRE(hs, "wisp_moe_decode_paged: store_host must be one pinned (page-locked, mapped) host allocation of host_rows * nbytes bytes");
  WISP_REQUIRE(aligned(hs, 16), "wisp_moe_decode_paged: store_host must be 16-byte aligned");
  WISP_REQUIRE(scratch_floats >= int64_t(k) * I, "wisp_moe_decode_paged: scratch of %lld floats, need at least k*I = %lld",
               (long long)scratch_floats, (long long)(int64_t(k) * I));
  MoeRoute RT{logits, E, norm_topk, slot_table, base, row, hs, host_rows, miss_count};
  return v4_launch(pool, nullptr, x, S, bits, scratch, out, static_cast<cudaStream_t>(stream), nctas, RT);
}

int64_t wisp_moe_batched_workspace_bytes(int N, int k, int64_t H, int64_t I) {
  if (N < 1 || k < 1 || int64_t(N) * k > batched::MAX_PAIRS || H <= 0 || I <= 0) return -1;
  return batched::ws_bytes(N * k, H, I);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (the library does not link libcuda)
static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// the tensor-core (tcgen05) grouped GEMM: 4-bit or 2-bit codes, groups a multiple of 128 dividing the rows
static bool umma_batched_ok(const MoeShape& S, int bits) {
  return (bits == 4 || bits == 2) && S.group % 128 == 0 && S.H % 128 == 0 && S.I % 128 == 0 && S.H % S.group == 0 &&
         S.I % S.group == 0 && S.nslots < (int64_t(1) << 31);
}

// 3-D map (code bytes of a row, rows, slots) over one matrix run of every slot, boxes of BK codes x 128 rows
static bool umma_code_map(CUtensorMap* m, const uint8_t* base, int64_t nslots, int64_t nbytes, int64_t rowbytes, int64_t rows, int bits) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tmap_encoder();
  if (!enc) return false;
  cuuint64_t dims[3] = {cuuint64_t(rowbytes), cuuint64_t(rows), cuuint64_t(nslots)};
  cuuint64_t strides[2] = {cuuint64_t(rowbytes), cuuint64_t(nbytes)};
  cuuint32_t box[3] = {cuuint32_t(umma::BK * bits / 8), cuuint32_t(umma::BM), 1};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D map over fp16 rows [P][K] (the staged tokens or the intermediate), 128-byte swizzled boxes of 64 x 32
static bool umma_row_map(CUtensorMap* m, const uint16_t* base, int64_t K, int64_t P) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tmap_encoder();
  if (!enc) return false;
  cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(P)};
  cuuint64_t strides[1] = {cuuint64_t(K * 2)};
  cuuint32_t box[2] = {cuuint32_t(umma::BK), cuuint32_t(umma::BOXR)};
  cuuint32_t es[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<uint16_t*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// staging, gate/up and down on the tensor cores (after the grouping); false if a tensor map cannot be encoded
static int umma_batched_launch(const uint8_t* pool, const MoeShape& S, int bits, const uint16_t* x, int N, int k, batched::Ws W,
                               cudaStream_t s, bool& launched) {
  launched = false;
  const int P = N * k;
  CUtensorMap mc0, mc2, mb0, mb2;
  if (!umma_code_map(&mc0, pool, S.nslots, S.nbytes, int64_t(S.H) * bits / 8, 2 * int64_t(S.I), bits) ||
      !umma_code_map(&mc2, pool + 2 * S.mat_bytes, S.nslots, S.nbytes, int64_t(S.I) * bits / 8, S.H, bits) ||
      !umma_row_map(&mb0, W.xp, S.H, P) || !umma_row_map(&mb2, W.a, S.I, P))
    return WISP_OK;
  const int grid = num_sms();
  const int64_t items = int64_t(P) * (S.H / 16);
  const int sgrid = int(items / 256 + 1 < int64_t(grid) * 8 ? items / 256 + 1 : int64_t(grid) * 8);
  const size_t sm0 = size_t(bits == 4 ? umma::smem_bytes<4, 0>(S.H / S.group) : umma::smem_bytes<2, 0>(S.H / S.group));
  const size_t sm2 = size_t(bits == 4 ? umma::smem_bytes<4, 2>(S.I / S.group) : umma::smem_bytes<2, 2>(S.I / S.group));
  if (sm0 > 227 * 1024 || sm2 > 227 * 1024) return WISP_OK;
  cudaError_t e = cudaSuccess;
#define WISP_UMMA(B)                                                                                                   \
  e = launch_pdl(umma::stage_rows_kernel<B>, sgrid, 256, 0, s, x, P, k, int64_t(S.H), W, W.xp);                          \
  if (e == cudaSuccess) e = launch_pdl(umma::grouped_umma_kernel<B, 0>, grid, umma::THREADS, sm0, s, mc0, mb0, pool, S, W, W.a); \
  if (e == cudaSuccess) e = launch_pdl(umma::grouped_umma_kernel<B, 2>, grid, umma::THREADS, sm2, s, mc2, mb2, pool, S, W, W.a);
  if (bits == 4) {
    WISP_UMMA(4)
  } else {
    WISP_UMMA(2)
  }
#undef WISP_UMMA
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_moe_batched (tensor-core path): %s", cudaGetErrorString(e));
  launched = true;
  return WISP_OK;
}

int wisp_moe_batched_variant(const uint8_t* pool, int64_t nslots, int64_t nbytes, const float* meta, int N, int k, const uint16_t* x,
                             int64_t H, int64_t I, int bits, int group, void* workspace, int64_t workspace_bytes, uint16_t* out,
                             int variant, void* stream) {
  WISP_REQUIRE(N >= 1 && k >= 1 && int64_t(N) * k <= batched::MAX_PAIRS, "wisp_moe_batched: need 1 <= N*k <= %d", batched::MAX_PAIRS);
  WISP_REQUIRE(variant >= 0 && variant <= 2, "wisp_moe_batched_variant: variant must be 0, 1 or 2");
  MoeShape S;
  int rc = moe_shape(pool, nslots, nbytes, meta, k, x, H, I, bits, group, reinterpret_cast<const float*>(workspace), out, S);
  if (rc) return rc;
  WISP_REQUIRE(H % 128 == 0 && I % 128 == 0, "wisp_moe_batched: H and I must be multiples of 128");
  WISP_REQUIRE(bits == 8 || bits == 4 || bits == 3 || bits == 2, "wisp_moe_batched: bits must be 8, 4, 3 or 2");
  WISP_REQUIRE(workspace_bytes >= batched::ws_bytes(N * k, H, I), "wisp_moe_batched: workspace of %lld bytes is too small (%lld needed)",
               (long long)workspace_bytes, (long long)batched::ws_bytes(N * k, H, I));
  WISP_REQUIRE(aligned(workspace, 256), "wisp_moe_batched: workspace must be 256-byte aligned");
  if (variant == 2 && !umma_batched_ok(S, bits))
    return fail(WISP_ERR_UNSUPPORTED, "wisp_moe_batched: the tensor-core path needs 4-bit or 2-bit codes and groups a multiple of 128");
  batched::Ws W = batched::ws_carve(workspace, N * k, I);
  W.xp = batched::ws_xp(workspace, N * k, H, I);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = num_sms();
  cudaError_t e = N * k <= batched::SMALL_PAIRS ? launch_pdl(batched::small_group_kernel, 1, 32, 0, s, meta, N, k, nslots, W)
                  : nslots <= batched::CS_MAX_SLOTS
                      ? launch_pdl(batched::count_group_kernel, 1, 1024, batched::count_group_smem(nslots), s, meta, N, k, nslots, W)
                      : launch_pdl(batched::group_kernel, 1, 1024, 0, s, meta, N, k, nslots, W);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_moe_batched: %s", cudaGetErrorString(e));
  // variant 0 (automatic) takes the warp-level kernels below: on the 64-token Zipf(1.1) layer of the
  // Qwen3-30B-A3B shape they measured 118.7 us against 132 us for the tcgen05 pipeline, whose stages are
  // bound by the per-stage latency of dequantizing into shared memory and of the small-N MMAs
  bool done = false;
  if (variant == 2 && umma_batched_ok(S, bits)) {
    rc = umma_batched_launch(pool, S, bits, x, N, k, W, s, done);
    if (rc) return rc;
    if (!done && variant == 2) return fail(WISP_ERR_UNSUPPORTED, "wisp_moe_batched: tensor maps of the tensor-core path unavailable");
  }
  // 4-bit and 2-bit codes with 128-multiple groups go straight into the MMA (two CTAs per SM, units
  // taken from a counter); 3-bit, 8-bit and finer groups dequantize to bf16 first
  const bool nib = (bits == 4 || bits == 2) && group % 128 == 0;
  if (done) {
  } else if (nib) {
    const size_t sm_gu = size_t(batched::nib_stage_bytes(H)), sm_dn = size_t(batched::nib_stage_bytes(I));
    const int64_t nwords = int64_t(N) * H / (32 / bits);
    const int pgrid = int(nwords / 256 + 1 < int64_t(grid) * 4 ? nwords / 256 + 1 : int64_t(grid) * 4);
#define WISP_NIB(B)                                                                                                     \
  if (e == cudaSuccess) e = launch_pdl(batched::permute_rows_kernel<B>, pgrid, 256, 0, s, x, nwords, W.xp);              \
  if (e == cudaSuccess) e = launch_pdl(batched::grouped_nib_kernel<B, 0>, 3 * grid, batched::THREADS, sm_gu, s, pool, S, W.xp, W); \
  if (e == cudaSuccess) e = launch_pdl(batched::grouped_nib_kernel<B, 2>, 3 * grid, batched::THREADS, sm_dn, s, pool, S, W.xp, W);
    if (bits == 4) {
      WISP_NIB(4)
    } else {
      WISP_NIB(2)
    }
#undef WISP_NIB
  } else {
    const size_t sm_gu = size_t(batched::stage_bytes(H)), sm_dn = size_t(batched::stage_bytes(I));
#define WISP_BATCHED(B)                                                                                                \
  if (e == cudaSuccess) e = launch_pdl(batched::grouped_kernel<B, 0>, grid, batched::THREADS, sm_gu, s, pool, S, x, W); \
  if (e == cudaSuccess) e = launch_pdl(batched::grouped_kernel<B, 2>, grid, batched::THREADS, sm_dn, s, pool, S, x, W);
    switch (bits) {
      case 8: WISP_BATCHED(8) break;
      case 4: WISP_BATCHED(4) break;
      case 3: WISP_BATCHED(3) break;
      default: WISP_BATCHED(2) break;
    }
#undef WISP_BATCHED
  }
  if (e == cudaSuccess) e = launch_pdl(batched::combine_kernel, grid * 4, 256, 0, s, meta, N, k, H, W, out);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_moe_batched: %s", cudaGetErrorString(e));
  return check_launch("moe_batched");
}

int wisp_moe_batched(const uint8_t* pool, int64_t nslots, int64_t nbytes, const float* meta, int N, int k, const uint16_t* x,
                     int64_t H, int64_t I, int bits, int group, void* workspace, int64_t workspace_bytes, uint16_t* out,
                     void* stream) {
  return wisp_moe_batched_variant(pool, nslots, nbytes, meta, N, k, x, H, I, bits, group, workspace, workspace_bytes, out, 0, stream);
}

// K splits of the gpt-oss GEMVs: enough (group, column tile, split) units for about four per warp of
// the grid (2 CTAs x 8 warps per SM on 148 SMs), estimating the groups as min(pairs, 32)
static int gptoss_splits(int P, int64_t I) {
  const int64_t groups = P < 1 ? 1 : (P < 32 ? P : 32);
  const int64_t tiles = (2 * I + 255) / 256;
  const int64_t s = 4 * 2 * 148 * 8 / (groups * tiles);
  return int(s < 1 ? 1 : (s > 32 ? 32 : s));
}

// K splits of the row-streaming GEMVs (gate_up, down): two (pass, split, slab) units per CTA of the grid
// (2 per SM) for fewer than 8 passes, three otherwise, estimating the 8-token passes as min(pairs, 32);
// every split keeps >= 1 k-step.  More units balance the CTAs better but leave more split partials to
// sum: per gpt-oss-20b layer 43.0 / 44.5 / 45.4 / 49.7 us at one token for 2 / 3 / 4 / 6 units per CTA,
// 261 / 251 / 258 / 266 us at 32 tokens.
static void gptoss_rows_splits(int P, int64_t H, int64_t I, int& ns0, int& ns1) {
  const int64_t passes = P < 1 ? 1 : (P < 32 ? P : 32), ctas = 2 * int64_t(num_sms());
  const int64_t per = passes < 8 ? 2 : 3;
  auto pick = [&](int64_t ncol, int64_t K) {
    const int64_t slabs = (ncol + gptoss::rows::SLAB - 1) / gptoss::rows::SLAB, kst = K / 16 > 0 ? K / 16 : 1;
    const int64_t sp = (per * ctas + passes * slabs - 1) / (passes * slabs);
    return int(sp < 1 ? 1 : (sp > kst ? kst : sp));
  };
  ns0 = pick(2 * I, H);
  ns1 = pick(H, I);
}

// the row-streaming path: 4-bit codes, power-of-two groups >= 64, 64 | H (so every 64-column block of
// both matrices lies in one group and rows are 16-byte multiples), scale and min arrays 16-byte aligned
static bool gptoss_rows_ok(int64_t H, int64_t I, int bits, int group) {
  const int64_t n = H * I;
  return bits == 4 && group >= 64 && (group & (group - 1)) == 0 && H == I && H % 64 == 0 && (3 * n * bits / 8) % 16 == 0 &&
         (2 * (3 * n / group)) % 16 == 0;
}

// splits the workspace is sized for: the larger of the column path's and the row path's
static int gptoss_ws_splits(int P, int64_t H, int64_t I) {
  int ns0, ns1;
  gptoss_rows_splits(P, H, I, ns0, ns1);
  const int c = gptoss_splits(P, I);
  const int r = ns0 > ns1 ? ns0 : ns1;
  return c > r ? c : r;
}

// the 3-D map (row words, rows, slots) of one gpt-oss matrix across the pool, boxes of one slab x 16 rows
static bool gptoss_tmap(CUtensorMap* m, const uint8_t* pool, int64_t nslots, int64_t nbytes, int64_t mat_off, int64_t ncol, int64_t K) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tmap_encoder();
  if (!enc) return false;
  const int64_t rowbytes = ncol / 2;
  cuuint64_t dims[3] = {cuuint64_t(rowbytes / 4), cuuint64_t(K), cuuint64_t(nslots)};
  cuuint64_t strides[2] = {cuuint64_t(rowbytes), cuuint64_t(nbytes)};
  cuuint32_t box[3] = {gptoss::rows::SLAB / 8, gptoss::rows::BOX_ROWS, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint8_t*>(pool + mat_off), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int64_t wisp_moe_gptoss_workspace_bytes(int N, int k, int64_t H, int64_t I) {
  if (N < 1 || k < 1 || int64_t(N) * k > batched::MAX_PAIRS || H <= 0 || I <= 0) return -1;
  return gptoss::ws_bytes(N * k, gptoss_ws_splits(N * k, H, I), H, I);
}

int wisp_moe_gptoss(const uint8_t* pool, int64_t nslots, int64_t nbytes, const float* meta, const int32_t* experts, int N, int k,
                    const uint16_t* x, int64_t H, int64_t I, int bits, int group, const uint16_t* gate_up_bias,
                    const uint16_t* down_bias, void* workspace, int64_t workspace_bytes, uint16_t* out, void* stream) {
  WISP_REQUIRE(experts && gate_up_bias && down_bias, "wisp_moe_gptoss: NULL pointer");
  WISP_REQUIRE(N >= 1 && k >= 1 && int64_t(N) * k <= batched::MAX_PAIRS, "wisp_moe_gptoss: need 1 <= N*k <= %d", batched::MAX_PAIRS);
  WISP_REQUIRE(H == I, "wisp_moe_gptoss: the gpt-oss layout needs intermediate == hidden (got H=%lld I=%lld)", (long long)H,
               (long long)I);
  // quantization groups run along the flat code stream and may straddle rows (2880 % 128 = 64): an
  // 8-code word never straddles a group as long as group and H are multiples of 8
  WISP_REQUIRE(pool && meta && x && workspace && out, "wisp_moe_gptoss: NULL pointer");
  WISP_REQUIRE(bits == 8 || bits == 4 || bits == 3 || bits == 2, "wisp_moe_gptoss: bits must be 8, 4, 3 or 2");
  WISP_REQUIRE(group > 0 && group % 8 == 0 && H > 0 && H % 8 == 0 && H <= 8192, "wisp_moe_gptoss: group and H must be multiples of 8");
  const int64_t n = H * I;
  WISP_REQUIRE(wisp_expert_nbytes(n, bits, group) == nbytes, "wisp_moe_gptoss: nbytes=%lld, expected %lld", (long long)nbytes,
               (long long)wisp_expert_nbytes(n, bits, group));
  WISP_REQUIRE(aligned(pool, 16) && nbytes % 16 == 0 && aligned(x, 16), "wisp_moe_gptoss: pool and x must be 16-byte aligned");
  WISP_REQUIRE(aligned(out, 8) && aligned(gate_up_bias, 8) && aligned(down_bias, 8),
               "wisp_moe_gptoss: out and the biases must be 8-byte aligned");
  MoeShape S;
  S.nslots = nslots;
  S.nbytes = nbytes;
  S.k = k;
  S.H = int(H);
  S.I = int(I);
  S.group = group;
  S.gshift = 0;
  S.glog = log2_or_neg(group);
  S.ncode = 3 * n * bits / 8;
  S.ng = 3 * n / group;
  S.mat_bytes = n * bits / 8;
  const int P = N * k, nsw = gptoss_ws_splits(P, H, I);
  WISP_REQUIRE(workspace_bytes >= gptoss::ws_bytes(P, nsw, H, I), "wisp_moe_gptoss: workspace too small (%lld needed)",
               (long long)gptoss::ws_bytes(P, nsw, H, I));
  WISP_REQUIRE(aligned(workspace, 256), "wisp_moe_gptoss: workspace must be 256-byte aligned");
  const gptoss::Ws W = gptoss::ws_carve(workspace, P, nsw, H, I);
  CUtensorMap map0, map1;
  const bool rows = gptoss_rows_ok(H, I, bits, group) && nslots < (int64_t(1) << 31) &&
                    gptoss_tmap(&map0, pool, nslots, nbytes, 0, 2 * I, H) &&
                    gptoss_tmap(&map1, pool, nslots, nbytes, H * I * bits / 4, H, I);
  int ns0 = gptoss_splits(P, I), ns1 = ns0;
  if (rows) gptoss_rows_splits(P, H, I, ns0, ns1);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = num_sms() * 2;
  // the row path groups up to 32 pairs inside its gate_up grid
  const int fuse_group = rows && N * k <= batched::SMALL_PAIRS ? 1 : 0;
  // reduction shapes of the activation and combine grids (see gptoss::RED_THREADS)
  const bool act_wide = P <= 8 && ns0 > 4;
  auto act = act_wide ? gptoss::act_kernel<16> : gptoss::act_kernel<1>;
  auto cmb = ns1 > 16 ? gptoss::combine_kernel<32> : (N <= 2 && ns1 > 4 ? gptoss::combine_kernel<16> : gptoss::combine_kernel<1>);
  cudaError_t e = fuse_group ? cudaSuccess
                  : N * k <= batched::SMALL_PAIRS ? launch_pdl(batched::small_group_kernel, 1, 32, 0, s, meta, N, k, nslots, W.g)
                  : nslots <= batched::CS_MAX_SLOTS
                      ? launch_pdl(batched::count_group_kernel, 1, 1024, batched::count_group_smem(nslots), s, meta, N, k, nslots, W.g)
                      : launch_pdl(batched::group_kernel, 1, 1024, 0, s, meta, N, k, nslots, W.g);
#define WISP_GPTOSS(B)                                                                                                      \
  if (e == cudaSuccess) e = launch_pdl(gptoss::gemv_kernel<B, 0>, grid, gptoss::THREADS, 0, s, pool, S, P, ns0, x, W);         \
  if (e == cudaSuccess) e = launch_pdl(act, grid, gptoss::RED_THREADS, 0, s, S, P, ns0, experts, gate_up_bias, W);             \
  if (e == cudaSuccess) e = launch_pdl(gptoss::gemv_kernel<B, 1>, grid, gptoss::THREADS, 0, s, pool, S, P, ns1, x, W);
  if (rows) {
    const int rgrid = 2 * num_sms();  // two CTAs per SM (shared memory and registers)
    if (e == cudaSuccess)
      e = launch_pdl(gptoss::rows::rows_kernel<0>, rgrid, gptoss::rows::THREADS, gptoss::rows::SMEM, s, map0, pool, S, P, ns0, x, W,
                     meta, N, fuse_group);
    if (e == cudaSuccess) e = launch_pdl(act, grid, gptoss::RED_THREADS, 0, s, S, P, ns0, experts, gate_up_bias, W);
    if (e == cudaSuccess)
      e = launch_pdl(gptoss::rows::rows_kernel<1>, rgrid, gptoss::rows::THREADS, gptoss::rows::SMEM, s, map1, pool, S, P, ns1, x, W,
                     meta, N, 0);
  } else {
    switch (bits) {
      case 8: WISP_GPTOSS(8) break;
      case 4: WISP_GPTOSS(4) break;
      case 3: WISP_GPTOSS(3) break;
      default: WISP_GPTOSS(2) break;
    }
  }
#undef WISP_GPTOSS
  if (e == cudaSuccess) e = launch_pdl(cmb, grid, gptoss::RED_THREADS, 0, s, meta, N, k, S, ns1, experts, down_bias, W, out);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_moe_gptoss: %s", cudaGetErrorString(e));
  return check_launch("moe_gptoss");
}

int wisp_moe_decode_noalloc(const uint8_t* pool, int64_t nslots, int64_t nbytes, const float* meta, int k,
                            const uint16_t* x, int64_t H, int64_t I, int bits, int group, uint16_t* out,
                            void* stream) {
  WISP_REQUIRE(k >= 1 && I > 0, "wisp_moe_decode_noalloc: k and I must be positive (k=%d I=%lld)", k, (long long)I);
  WISP_REQUIRE(int64_t(k) * I <= WISP_MOE_NOALLOC_MAX_SCRATCH,
               "wisp_moe_decode_noalloc: k*I = %lld exceeds the built-in scratch of %d floats "
               "(use wisp_moe_decode with caller-provided scratch)",
               (long long)(int64_t(k) * I), WISP_MOE_NOALLOC_MAX_SCRATCH);
  float* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return wisp_moe_decode_variant(pool, nslots, nbytes, meta, k, x, H, I, bits, group, scratch, WISP_MOE_NOALLOC_MAX_SCRATCH, out,
                                 0, stream);
}

int wisp_rope_decode(const uint16_t* q, int64_t q_stride, int Hq, const uint16_t* k, int64_t k_stride, int Hk, int D,
                     const uint16_t* cos, const uint16_t* sin, uint16_t* qo, uint16_t* ko, void* stream) {
  WISP_REQUIRE(q && k && cos && sin && qo && ko, "wisp_rope_decode: NULL pointer");
  WISP_REQUIRE(Hq > 0 && Hk >= 0 && D > 0 && D % 2 == 0, "wisp_rope_decode: bad shape");
  const int heads = Hq + Hk;
  const int warps = 4;
  rope_decode_kernel<<<(heads + warps - 1) / warps, 32 * warps, 0, static_cast<cudaStream_t>(stream)>>>(
      q, q_stride, Hq, k, k_stride, Hk, D, cos, sin, qo, ko);
  return check_launch("rope_decode");
}

int wisp_gemv(const uint16_t* W, int64_t N, int64_t K, const uint16_t* x, const uint16_t* x_add, uint16_t* x_sum_out,
              const uint16_t* norm_w, float eps, uint16_t* xn_out, const uint16_t* res, uint16_t* y, void* stream) {
  return wisp_gemv_bias(W, N, K, x, x_add, x_sum_out, norm_w, eps, xn_out, nullptr, res, y, stream);
}

int wisp_gemv_bias(const uint16_t* W, int64_t N, int64_t K, const uint16_t* x, const uint16_t* x_add, uint16_t* x_sum_out,
                   const uint16_t* norm_w, float eps, uint16_t* xn_out, const uint16_t* bias, const uint16_t* res, uint16_t* y,
                   void* stream) {
  WISP_REQUIRE(W && x && y, "wisp_gemv: NULL pointer");
  WISP_REQUIRE(N > 0 && K > 0 && K % 8 == 0 && K <= 4096, "wisp_gemv: need N > 0, K a multiple of 8 and <= 4096 (N=%lld K=%lld)",
               (long long)N, (long long)K);
  WISP_REQUIRE(aligned(W, 16) && aligned(x, 16) && (!x_add || aligned(x_add, 16)) && (!x_sum_out || aligned(x_sum_out, 16)) &&
                   (!norm_w || aligned(norm_w, 16)) && (!xn_out || aligned(xn_out, 16)),
               "wisp_gemv: W, x, x_add, x_sum_out, norm_w and xn_out must be 16-byte aligned");
  WISP_REQUIRE(x_sum_out == nullptr || x_add != nullptr, "wisp_gemv: x_sum_out needs x_add");
  WISP_REQUIRE(y != x && y != x_add && (!x_sum_out || (x_sum_out != x && x_sum_out != x_add)) &&
                   (!xn_out || (xn_out != x && xn_out != x_add)),
               "wisp_gemv: y, x_sum_out and xn_out must not alias x or x_add");
  dense::GemvArgs A{W, N, K, x, x_add, x_sum_out, norm_w, eps, xn_out, res, y, bias};
  const int grid = int(N < num_sms() ? N : num_sms());
  // a 4th ring stage where 4 fit in 120 KB and a CTA's rows need more than 3
  const dense::GemvLayout L3 = dense::gemv_layout<dense::STAGES>(K);
  const int64_t rows_cta = (N + grid - 1) / grid;
  const bool four = dense::STAGES_MAX * L3.stage_bytes <= dense::RING_BYTES_MAX && rows_cta > dense::STAGES * L3.rows_per_stage;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (four)
    e = launch_pdl(dense::gemv_kernel<dense::STAGES_MAX>, grid, dense::THREADS, size_t(dense::gemv_layout<dense::STAGES_MAX>(K).bytes), s, A);
  else
    e = launch_pdl(dense::gemv_kernel<dense::STAGES>, grid, dense::THREADS, size_t(L3.bytes), s, A);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_gemv: %s", cudaGetErrorString(e));
  return check_launch("gemv");
}

int wisp_qk_norm_rope_kv(const uint16_t* qkv, int Hq, int Hk, int D, const uint16_t* qn_w, const uint16_t* kn_w, float eps,
                         const uint16_t* cos_t, const uint16_t* sin_t, const int64_t* pos, int64_t tmax, uint16_t* q_out,
                         uint16_t* k_cache, uint16_t* v_cache, void* stream) {
  WISP_REQUIRE(qkv && qn_w && kn_w && cos_t && sin_t && pos && q_out && k_cache && v_cache, "wisp_qk_norm_rope_kv: NULL pointer");
  WISP_REQUIRE(Hq > 0 && Hk > 0 && D > 0 && D % 2 == 0 && D <= dec::QK_MAX_D && tmax > 0, "wisp_qk_norm_rope_kv: bad shape");
  const int heads = Hq + 2 * Hk;
  const cudaError_t e = launch_pdl(dec::qk_norm_rope_kv_kernel, (heads + 7) / 8, 256, 0, static_cast<cudaStream_t>(stream), qkv, Hq,
                                   Hk, D, qn_w, kn_w, eps, cos_t, sin_t, pos, tmax, q_out, k_cache, v_cache, int64_t(0), 0, 1,
                                   int64_t(0));
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_qk_norm_rope_kv: %s", cudaGetErrorString(e));
  return check_launch("qk_norm_rope_kv");
}

int wisp_qk_norm_rope_kv_rows(const uint16_t* qkv, int T, int64_t qkv_stride, int Hq, int Hk, int D, const uint16_t* qn_w,
                              const uint16_t* kn_w, float eps, const uint16_t* cos_t, const uint16_t* sin_t, const int64_t* pos0,
                              int64_t tmax, uint16_t* q_out, uint16_t* k_cache, uint16_t* v_cache, void* stream) {
  WISP_REQUIRE(qkv && qn_w && kn_w && cos_t && sin_t && pos0 && q_out && k_cache && v_cache,
               "wisp_qk_norm_rope_kv_rows: NULL pointer");
  WISP_REQUIRE(Hq > 0 && Hk > 0 && D > 0 && D % 2 == 0 && D <= dec::QK_MAX_D && tmax > 0, "wisp_qk_norm_rope_kv_rows: bad shape");
  WISP_REQUIRE(T >= 1 && T <= 65535 && qkv_stride >= int64_t(Hq + 2 * Hk) * D,
               "wisp_qk_norm_rope_kv_rows: need 1 <= T <= 65535 and qkv_stride >= (Hq + 2 Hk) D");
  const int heads = Hq + 2 * Hk;
  const cudaError_t e = launch_pdl(dec::qk_norm_rope_kv_kernel, dim3((heads + 7) / 8, T), 256, 0, static_cast<cudaStream_t>(stream),
                                   qkv, Hq, Hk, D, qn_w, kn_w, eps, cos_t, sin_t, pos0, tmax, q_out, k_cache, v_cache, qkv_stride, 0, 1,
                                   int64_t(0));
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_qk_norm_rope_kv_rows: %s", cudaGetErrorString(e));
  return check_launch("qk_norm_rope_kv_rows");
}

int wisp_qk_norm_rope_kv_batched(const uint16_t* qkv, int B, int64_t qkv_stride, int Hq, int Hk, int D, const uint16_t* qn_w,
                                 const uint16_t* kn_w, float eps, const uint16_t* cos_t, const uint16_t* sin_t, const int64_t* pos,
                                 int64_t tmax, uint16_t* q_out, uint16_t* k_cache, uint16_t* v_cache, void* stream) {
  WISP_REQUIRE(qkv && cos_t && sin_t && pos && q_out && k_cache && v_cache, "wisp_qk_norm_rope_kv_batched: NULL pointer");
  WISP_REQUIRE((qn_w == nullptr) == (kn_w == nullptr), "wisp_qk_norm_rope_kv_batched: give both norm weights or neither");
  WISP_REQUIRE(Hq > 0 && Hk > 0 && D > 0 && D % 2 == 0 && D <= dec::QK_MAX_D && tmax > 0, "wisp_qk_norm_rope_kv_batched: bad shape");
  WISP_REQUIRE(B >= 1 && B <= 65535 && qkv_stride >= int64_t(Hq + 2 * Hk) * D,
               "wisp_qk_norm_rope_kv_batched: need 1 <= B <= 65535 and qkv_stride >= (Hq + 2 Hk) D");
  const int heads = Hq + 2 * Hk;
  const cudaError_t e = launch_pdl(dec::qk_norm_rope_kv_kernel, dim3((heads + 7) / 8, B), 256, 0, static_cast<cudaStream_t>(stream),
                                   qkv, Hq, Hk, D, qn_w, kn_w, eps, cos_t, sin_t, pos, tmax, q_out, k_cache, v_cache, qkv_stride, 1, 0,
                                   int64_t(Hk) * tmax * D);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_qk_norm_rope_kv_batched: %s", cudaGetErrorString(e));
  return check_launch("qk_norm_rope_kv_batched");
}

int64_t wisp_attn_workspace_floats(int Hq, int Hk, int D, int64_t tmax) {
  if (Hq <= 0 || Hk <= 0 || D <= 0 || tmax <= 0 || Hq % Hk) return -1;
  return int64_t(Hk) * ((tmax + dec::CHUNK - 1) / dec::CHUNK) * (Hq / Hk) * dec::rec_floats(D);
}

// Chunks of CHUNK positions per attention CTA (tensor-core kernel): the largest of 1, 2, 4, 8 that still
// leaves at least 16 CTAs per SM, so long contexts write (and the merge reads) a fraction of the records
// while short ones keep one chunk per CTA.
static int attn_span(int D, int Hk, int nchunk, int B) {
  if (D != 64 && D != 128) return 1;  // the CUDA-core kernel takes one chunk per CTA
  int span = 1;
  while (span < 8 && int64_t(Hk) * ((nchunk + 2 * span - 1) / (2 * span)) * B >= 16 * int64_t(num_sms())) span *= 2;
  return span;
}

// chunk partials of decode attention: the tensor-core kernel for head_dim 64 and 128, the CUDA-core one
// otherwise; grid.y = chunk groups of `span` chunks
static cudaError_t launch_attn_split(dim3 grid, const uint16_t* q, int Hq, int Hk, int D, const uint16_t* k_cache,
                                     const uint16_t* v_cache, int64_t tmax, const int64_t* pos, float scale, float* workspace,
                                     int64_t kv_bstride, int window, int span, cudaStream_t s) {
  const dec::RopeArgs none{};
  uint16_t* kc = const_cast<uint16_t*>(k_cache);  // not written without the fused rotary
  uint16_t* vc = const_cast<uint16_t*>(v_cache);
  if (D == 128)
    return launch_pdl(dec::attn_split_tc_kernel<128, false>, grid, dec::ATTN_THREADS, 0, s, q, Hq, Hk, kc, vc, tmax, pos, scale,
                      workspace, kv_bstride, window, none, span);
  if (D == 64)
    return launch_pdl(dec::attn_split_tc_kernel<64, false>, grid, dec::ATTN_THREADS, 0, s, q, Hq, Hk, kc, vc, tmax, pos, scale,
                      workspace, kv_bstride, window, none, span);
  return launch_pdl(dec::attn_split_kernel, grid, dec::ATTN_THREADS, 0, s, q, Hq, Hk, D, k_cache, v_cache, tmax, pos, scale, workspace,
                    kv_bstride, window);
}

int wisp_gqa_decode_attn(const uint16_t* q, int Hq, int Hk, int D, const uint16_t* k_cache, const uint16_t* v_cache, int64_t tmax,
                         const int64_t* pos, float scale, float* workspace, uint16_t* out, void* stream) {
  WISP_REQUIRE(q && k_cache && v_cache && pos && workspace && out, "wisp_gqa_decode_attn: NULL pointer");
  WISP_REQUIRE(Hq > 0 && Hk > 0 && Hq % Hk == 0 && Hq / Hk <= dec::MAX_G, "wisp_gqa_decode_attn: need Hq a multiple of Hk, Hq/Hk <= %d",
               dec::MAX_G);
  WISP_REQUIRE(D > 0 && D % 32 == 0 && D <= dec::MAX_D && tmax > 0, "wisp_gqa_decode_attn: need D a multiple of 32, <= %d", dec::MAX_D);
  WISP_REQUIRE(aligned(k_cache, 16) && aligned(v_cache, 16), "wisp_gqa_decode_attn: caches must be 16-byte aligned");
  const int nchunk = int((tmax + dec::CHUNK - 1) / dec::CHUNK);
  const int span = attn_span(D, Hk, nchunk, 1), ngrp = (nchunk + span - 1) / span;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_attn_split(dim3(Hk, ngrp), q, Hq, Hk, D, k_cache, v_cache, tmax, pos, scale, workspace, 0, 0, span, s);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_gqa_decode_attn: %s", cudaGetErrorString(e));
  e = launch_pdl(dec::attn_combine_kernel, Hq, dec::CMB_THREADS, 0, s, (const float*)workspace, Hq, Hk, D, ngrp, pos, tmax, out, 0,
                 (const float*)nullptr, dec::CHUNK * span);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_gqa_decode_attn: %s", cudaGetErrorString(e));
  return check_launch("gqa_decode_attn");
}

int64_t wisp_attn_batched_workspace_floats(int B, int Hq, int Hk, int D, int64_t tmax) {
  if (B < 1 || Hq <= 0 || Hk <= 0 || D <= 0 || tmax <= 0 || Hq % Hk) return -1;
  return int64_t(B) * Hk * ((tmax + dec::CHUNK - 1) / dec::CHUNK) * (Hq / Hk) * dec::rec_floats(D);
}

int wisp_gqa_decode_attn_batched(const uint16_t* q, int B, int Hq, int Hk, int D, const uint16_t* k_cache, const uint16_t* v_cache,
                                 int64_t tmax, const int64_t* pos, int window, const float* sinks, float scale, float* workspace,
                                 int64_t workspace_floats, uint16_t* out, void* stream) {
  WISP_REQUIRE(q && k_cache && v_cache && pos && workspace && out, "wisp_gqa_decode_attn_batched: NULL pointer");
  WISP_REQUIRE(B >= 1 && B <= 65535, "wisp_gqa_decode_attn_batched: need 1 <= B <= 65535");
  WISP_REQUIRE(Hq > 0 && Hk > 0 && Hq % Hk == 0 && Hq / Hk <= dec::MAX_G,
               "wisp_gqa_decode_attn_batched: need Hq a multiple of Hk, Hq/Hk <= %d", dec::MAX_G);
  WISP_REQUIRE(D > 0 && D % 32 == 0 && D <= dec::MAX_D && tmax > 0, "wisp_gqa_decode_attn_batched: need D a multiple of 32, <= %d",
               dec::MAX_D);
  WISP_REQUIRE(window >= 0, "wisp_gqa_decode_attn_batched: window must be >= 0");
  WISP_REQUIRE(aligned(k_cache, 16) && aligned(v_cache, 16), "wisp_gqa_decode_attn_batched: caches must be 16-byte aligned");
  WISP_REQUIRE(workspace_floats >= wisp_attn_batched_workspace_floats(B, Hq, Hk, D, tmax),
               "wisp_gqa_decode_attn_batched: workspace of %lld floats is too small", (long long)workspace_floats);
  const int nchunk = int((tmax + dec::CHUNK - 1) / dec::CHUNK);
  const int span = attn_span(D, Hk, nchunk, B), ngrp = (nchunk + span - 1) / span;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_attn_split(dim3(Hk, ngrp, B), q, Hq, Hk, D, k_cache, v_cache, tmax, pos, scale, workspace,
                                    int64_t(Hk) * tmax * D, window, span, s);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_gqa_decode_attn_batched: %s", cudaGetErrorString(e));
  e = launch_pdl(dec::attn_combine_kernel, dim3(Hq, B), dec::CMB_THREADS, 0, s, (const float*)workspace, Hq, Hk, D, ngrp, pos, tmax, out, window,
                 sinks, dec::CHUNK * span);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_gqa_decode_attn_batched: %s", cudaGetErrorString(e));
  return check_launch("gqa_decode_attn_batched");
}

int wisp_attn_decode_batched(const uint16_t* qkv, int64_t qkv_stride, int B, int Hq, int Hk, int D, const uint16_t* qn_w,
                             const uint16_t* kn_w, float eps, const uint16_t* cos_t, const uint16_t* sin_t, uint16_t* k_cache,
                             uint16_t* v_cache, int64_t tmax, const int64_t* pos, int window, const float* sinks, float scale,
                             float* workspace, int64_t workspace_floats, uint16_t* out, void* stream) {
  WISP_REQUIRE(qkv && cos_t && sin_t && k_cache && v_cache && pos && workspace && out, "wisp_attn_decode_batched: NULL pointer");
  WISP_REQUIRE((qn_w == nullptr) == (kn_w == nullptr), "wisp_attn_decode_batched: give both norm weights or neither");
  WISP_REQUIRE(B >= 1 && B <= 65535, "wisp_attn_decode_batched: need 1 <= B <= 65535");
  WISP_REQUIRE(Hq > 0 && Hk > 0 && Hq % Hk == 0 && Hq / Hk <= dec::MAX_G, "wisp_attn_decode_batched: need Hq a multiple of Hk, Hq/Hk <= %d",
               dec::MAX_G);
  if (D != 64 && D != 128) return fail(WISP_ERR_UNSUPPORTED, "wisp_attn_decode_batched: head_dim must be 64 or 128 (got %d)", D);
  WISP_REQUIRE(tmax > 0 && window >= 0 && qkv_stride >= int64_t(Hq + 2 * Hk) * D, "wisp_attn_decode_batched: bad shape");
  WISP_REQUIRE(aligned(k_cache, 16) && aligned(v_cache, 16), "wisp_attn_decode_batched: caches must be 16-byte aligned");
  WISP_REQUIRE(workspace_floats >= wisp_attn_batched_workspace_floats(B, Hq, Hk, D, tmax),
               "wisp_attn_decode_batched: workspace of %lld floats is too small", (long long)workspace_floats);
  const int nchunk = int((tmax + dec::CHUNK - 1) / dec::CHUNK);
  const int span = attn_span(D, Hk, nchunk, B), ngrp = (nchunk + span - 1) / span;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dec::RopeArgs ra{qkv, qkv_stride, qn_w, kn_w, eps, cos_t, sin_t};
  const int64_t kvb = int64_t(Hk) * tmax * D;
  cudaError_t e = D == 128 ? launch_pdl(dec::attn_split_tc_kernel<128, true>, dim3(Hk, ngrp, B), dec::ATTN_THREADS, 0, s,
                                        (const uint16_t*)nullptr, Hq, Hk, k_cache, v_cache, tmax, pos, scale, workspace, kvb, window, ra,
                                        span)
                           : launch_pdl(dec::attn_split_tc_kernel<64, true>, dim3(Hk, ngrp, B), dec::ATTN_THREADS, 0, s,
                                        (const uint16_t*)nullptr, Hq, Hk, k_cache, v_cache, tmax, pos, scale, workspace, kvb, window, ra,
                                        span);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_attn_decode_batched: %s", cudaGetErrorString(e));
  e = launch_pdl(dec::attn_combine_kernel, dim3(Hq, B), dec::CMB_THREADS, 0, s, (const float*)workspace, Hq, Hk, D, ngrp, pos, tmax, out,
                 window, sinks, dec::CHUNK * span);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_attn_decode_batched: %s", cudaGetErrorString(e));
  return check_launch("attn_decode_batched");
}

int wisp_attn_decode(const uint16_t* qkv, int Hq, int Hk, int D, const uint16_t* qn_w, const uint16_t* kn_w, float eps,
                     const uint16_t* cos_t, const uint16_t* sin_t, const int64_t* pos, int64_t tmax, uint16_t* k_cache,
                     uint16_t* v_cache, float scale, uint16_t* out, void* stream) {
  WISP_REQUIRE(qkv && qn_w && kn_w && cos_t && sin_t && pos && k_cache && v_cache && out, "wisp_attn_decode: NULL pointer");
  WISP_REQUIRE(D == dec::FD, "wisp_attn_decode: head_dim must be %d (got %d)", dec::FD, D);
  WISP_REQUIRE(Hq > 0 && Hk > 0 && Hq % Hk == 0 && Hq / Hk <= dec::MAX_G && tmax > 0,
               "wisp_attn_decode: need Hq a multiple of Hk with Hq/Hk <= %d", dec::MAX_G);
  WISP_REQUIRE(aligned(k_cache, 16) && aligned(v_cache, 16), "wisp_attn_decode: caches must be 16-byte aligned");
  const size_t smem = sizeof(dec::AttnSmem);
  cudaFuncSetAttribute(dec::attn_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  cudaFuncSetAttribute(dec::attn_fused_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  auto config = [&](int split, cudaLaunchAttribute (&attr)[2]) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(split, Hk);
    cfg.blockDim = dim3(dec::FTHREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = split;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cfg;
  };
  // 16 CTAs per KV head where the GPU can co-schedule such clusters, else the portable 8 (decided once)
  static int split = 0;
  if (split == 0) {
    split = 8;
    cudaLaunchAttribute attr[2];
    const cudaLaunchConfig_t cfg = config(dec::MAX_SPLIT, attr);
    int nclusters = 0;
    if (cudaOccupancyMaxActiveClusters(&nclusters, dec::attn_fused_kernel, &cfg) == cudaSuccess && nclusters >= 1)
      split = dec::MAX_SPLIT;
    cudaGetLastError();
  }
  cudaLaunchAttribute attr[2];
  const cudaLaunchConfig_t cfg = config(split, attr);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, dec::attn_fused_kernel, qkv, Hq, Hk, qn_w, kn_w, eps, cos_t, sin_t, pos, tmax,
                                           k_cache, v_cache, scale, out);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_attn_decode: %s", cudaGetErrorString(e));
  return check_launch("attn_decode");
}

int wisp_router_topk(const uint16_t* logits, int E, int k, int norm_topk, const int32_t* slot_table, int64_t base, float* row,
                     float* meta, void* stream) {
  WISP_REQUIRE(logits && meta, "wisp_router_topk: NULL pointer");
  WISP_REQUIRE(E > 0 && E <= 1024 && k >= 1 && k <= 32 && k <= E, "wisp_router_topk: need 1 <= k <= min(E, 32), E <= 1024");
  const cudaError_t e = launch_pdl(dec::router_topk_kernel, 1, 32, 0, static_cast<cudaStream_t>(stream), logits, E, k, norm_topk,
                                   slot_table, base, row, meta);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_router_topk: %s", cudaGetErrorString(e));
  return check_launch("router_topk");
}

int64_t wisp_router_workspace_bytes(int B, int E) {
  if (B < 1 || E < 1 || E > 1024) return -1;
  return (int64_t(B) * E * 4 + 255) / 256 * 256 + int64_t(B) * 4;
}

int wisp_router_rows(const uint16_t* x, int B, int64_t H, const uint16_t* norm_w, float eps, uint16_t* xn_out, const uint16_t* W,
                     const uint16_t* bias, int E, int k, int norm_topk, const int32_t* slot_table, int64_t base, float* meta,
                     int32_t* experts, float* row, void* stream) {
  return wisp_router_rows_ws(x, B, H, norm_w, eps, xn_out, W, bias, E, k, norm_topk, slot_table, base, meta, experts, row, nullptr, 0,
                             stream);
}

int wisp_router_rows_ws(const uint16_t* x, int B, int64_t H, const uint16_t* norm_w, float eps, uint16_t* xn_out, const uint16_t* W,
                        const uint16_t* bias, int E, int k, int norm_topk, const int32_t* slot_table, int64_t base, float* meta,
                        int32_t* experts, float* row, void* workspace, int64_t workspace_bytes, void* stream) {
  WISP_REQUIRE(x && W && meta, "wisp_router_rows: NULL pointer");
  WISP_REQUIRE(B >= 1 && B <= 65535, "wisp_router_rows: need 1 <= B <= 65535");
  WISP_REQUIRE(H > 0 && H % 8 == 0 && H <= dec::ROUTER_MAX_H, "wisp_router_rows: need H a multiple of 8, <= %d", dec::ROUTER_MAX_H);
  WISP_REQUIRE(E > 0 && E <= 1024 && k >= 1 && k <= 32 && k <= E, "wisp_router_rows: need 1 <= k <= min(E, 32), E <= 1024");
  WISP_REQUIRE(norm_topk >= 0 && norm_topk <= 2, "wisp_router_rows: norm_topk must be 0, 1 or 2");
  WISP_REQUIRE(aligned(x, 16) && aligned(W, 16) && (!norm_w || aligned(norm_w, 16)) && (!xn_out || aligned(xn_out, 16)),
               "wisp_router_rows: x, W, norm_w and xn_out must be 16-byte aligned");
  WISP_REQUIRE(xn_out != x, "wisp_router_rows: xn_out must not alias x");
  cudaError_t e;
  if (workspace) {
    WISP_REQUIRE(workspace_bytes >= wisp_router_workspace_bytes(B, E) && aligned(workspace, 256),
                 "wisp_router_rows: workspace must be 256-byte aligned and hold wisp_router_workspace_bytes(B, E) bytes");
    float* logits = static_cast<float*>(workspace);
    unsigned int* count = reinterpret_cast<unsigned int*>(static_cast<uint8_t*>(workspace) + (int64_t(B) * E * 4 + 255) / 256 * 256);
    const dim3 grid(B, (E + dec::ROUTER_SPLIT_E - 1) / dec::ROUTER_SPLIT_E);
    e = launch_pdl(dec::router_split_kernel, grid, dec::ROUTER_SPLIT_THREADS, 0, static_cast<cudaStream_t>(stream), x, H, norm_w, eps,
                   xn_out, W, bias, E, k, norm_topk, slot_table, base, meta, experts, row, logits, count);
  } else {
    e = launch_pdl(dec::router_rows_kernel, B, dec::ROUTER_THREADS, 0, static_cast<cudaStream_t>(stream), x, H, norm_w, eps, xn_out, W,
                   bias, E, k, norm_topk, slot_table, base, meta, experts, row);
  }
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_router_rows: %s", cudaGetErrorString(e));
  return check_launch("router_rows");
}

int wisp_embed(const uint16_t* table, int64_t V, int64_t H, const int64_t* token, uint16_t* out, void* stream) {
  WISP_REQUIRE(table && token && out, "wisp_embed: NULL pointer");
  WISP_REQUIRE(V > 0 && H > 0 && H % 8 == 0 && aligned(table, 16) && aligned(out, 16), "wisp_embed: need H % 8 == 0, 16-byte aligned rows");
  const int threads = 256;
  const int grid = int((H / 8 + threads - 1) / threads);
  const cudaError_t e = launch_pdl(dec::embed_kernel, grid, threads, 0, static_cast<cudaStream_t>(stream), table, V, H, token, out);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_embed: %s", cudaGetErrorString(e));
  return check_launch("embed");
}

int wisp_argmax(const uint16_t* x, int64_t n, uint64_t* workspace, int64_t* out, void* stream) {
  WISP_REQUIRE(x && workspace && out, "wisp_argmax: NULL pointer");
  WISP_REQUIRE(n > 0 && n < (int64_t(1) << 32), "wisp_argmax: need 0 < n < 2^32");
  const int parts = WISP_ARGMAX_WORKSPACE;
  const int grid = int((n + 255) / 256 < parts ? (n + 255) / 256 : parts);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_pdl(dec::argmax_partial_kernel, grid, 256, 0, s, x, n, (unsigned long long*)workspace);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_argmax: %s", cudaGetErrorString(e));
  e = launch_pdl(dec::argmax_final_kernel, 1, 32, 0, s, (const unsigned long long*)workspace, grid, out);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_argmax: %s", cudaGetErrorString(e));
  return check_launch("argmax");
}

int wisp_rmsnorm(const uint16_t* x, const uint16_t* delta, uint16_t* sum_out, const uint16_t* w, int64_t rows, int64_t H,
                 float eps, uint16_t* out, void* stream) {
  WISP_REQUIRE(x && w && out, "wisp_rmsnorm: NULL pointer");
  WISP_REQUIRE(rows >= 0 && H > 0 && H <= 16384, "wisp_rmsnorm: bad shape");
  if (rows == 0) return WISP_OK;
  const bool vec_ok = H % 8 == 0 && H / 8 <= 1024 && aligned(x, 16) && aligned(w, 16) && aligned(out, 16) &&
                      (!delta || aligned(delta, 16)) && (!sum_out || aligned(sum_out, 16));
  if (vec_ok) {
    const int threads = int((H / 8 + 31) / 32 * 32);
    const cudaError_t e = launch_pdl(rmsnorm_vec_kernel, int(rows), threads, 0, static_cast<cudaStream_t>(stream), x, delta,
                                     sum_out, w, H, eps, out);
    if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "rmsnorm: %s", cudaGetErrorString(e));
    return check_launch("rmsnorm");
  }
  const size_t smem = size_t(H) * 4;
  // the kernel also has a small static array: opt in to large dynamic shared memory well before 48 KB
  if (smem > 32 * 1024) raise_smem_limit(reinterpret_cast<const void*>(rmsnorm_kernel), smem);
  rmsnorm_kernel<<<(unsigned)rows, 256, smem, static_cast<cudaStream_t>(stream)>>>(x, delta, sum_out, w, H, eps, out);
  return check_launch("rmsnorm");
}


int wisp_ep_dispatch(const uint16_t* x, int N, int64_t H, const int64_t* sel, int k, int E_local, int world, int64_t capacity,
                     int64_t slot_base, uint16_t* send_x, float* send_meta, int32_t* src_pos, void* stream) {
  WISP_REQUIRE(x && sel && send_x && send_meta && src_pos, "wisp_ep_dispatch: NULL pointer");
  WISP_REQUIRE(N >= 1 && k >= 1 && int64_t(N) * k <= ep::MAX_PAIRS, "wisp_ep_dispatch: need 1 <= N*k <= %d", ep::MAX_PAIRS);
  WISP_REQUIRE(world >= 1 && world <= ep::MAX_WORLD && E_local >= 1, "wisp_ep_dispatch: need 1 <= world <= %d, E_local >= 1",
               ep::MAX_WORLD);
  WISP_REQUIRE(capacity >= int64_t(N) * k, "wisp_ep_dispatch: capacity %lld < N*k = %d (a rank may send every pair to one peer)",
               (long long)capacity, N * k);
  WISP_REQUIRE(H > 0 && H % 8 == 0 && aligned(x, 16) && aligned(send_x, 16), "wisp_ep_dispatch: H %% 8 == 0 and 16-byte aligned rows");
  const int P = N * k;
  const int grid = P < 2 * num_sms() ? P : 2 * num_sms();
  cudaError_t e = launch_pdl(ep::ep_dispatch_kernel, grid, 256, 0, static_cast<cudaStream_t>(stream), x, N, H, sel, k, E_local,
                             world, capacity, slot_base, send_x, send_meta, src_pos);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_ep_dispatch: %s", cudaGetErrorString(e));
  return check_launch("ep_dispatch");
}

int wisp_ep_combine(const uint16_t* y_back, int N, int k, int64_t H, const int32_t* src_pos, const float* w, uint16_t* out,
                    void* stream) {
  WISP_REQUIRE(y_back && src_pos && w && out, "wisp_ep_combine: NULL pointer");
  WISP_REQUIRE(N >= 1 && k >= 1 && H > 0 && H % 4 == 0, "wisp_ep_combine: need N, k >= 1 and H %% 4 == 0");
  WISP_REQUIRE(aligned(y_back, 8) && aligned(out, 8), "wisp_ep_combine: y_back and out must be 8-byte aligned");
  const int64_t work = int64_t(N) * H / 4;
  const int64_t g = (work + 255) / 256;
  const int grid = int(g < 4 * num_sms() ? g : 4 * num_sms());
  cudaError_t e = launch_pdl(ep::ep_combine_kernel, grid, 256, 0, static_cast<cudaStream_t>(stream), y_back, N, k, H, src_pos, w, out);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_ep_combine: %s", cudaGetErrorString(e));
  return check_launch("ep_combine");
}


// ---- peer-memory expert-parallel exchange ---------------------------------------------------------------
int wisp_ipc_alloc(int64_t bytes, void** ptr_host, uint8_t* handle_host) {
  WISP_REQUIRE(bytes > 0 && ptr_host && handle_host, "wisp_ipc_alloc: bad arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, size_t(bytes));
  if (e == cudaSuccess) e = cudaMemset(p, 0, size_t(bytes));
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return fail(WISP_ERR_CUDA, "wisp_ipc_alloc: %s", cudaGetErrorString(e));
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handles are 64 bytes");
  std::memcpy(handle_host, &h, 64);
  *ptr_host = p;
  return WISP_OK;
}

int wisp_ipc_open(const uint8_t* handle_host, void** ptr_host) {
  WISP_REQUIRE(handle_host && ptr_host, "wisp_ipc_open: NULL argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle_host, 64);
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_ipc_open: %s", cudaGetErrorString(e));
  *ptr_host = p;
  return WISP_OK;
}

int wisp_ipc_close(void* ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_ipc_close: %s", cudaGetErrorString(e));
  return WISP_OK;
}

int wisp_ipc_free(void* ptr) {
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_ipc_free: %s", cudaGetErrorString(e));
  return WISP_OK;
}

int64_t wisp_ep_p2p_bytes(int world, int64_t capacity, int64_t H) {
  if (world < 1 || world > ep::MAX_P2P || capacity < 1 || H < 1) return -1;
  return ep::p2p_layout(world, capacity, H).bytes;
}

static int p2p_peers(void* const* peers_host, int world, int rank, ep::Peers& P) {
  WISP_REQUIRE(peers_host && world >= 1 && world <= ep::MAX_P2P && rank >= 0 && rank < world,
               "ep p2p: need 1 <= world <= %d, 0 <= rank < world and the peers' base pointers", ep::MAX_P2P);
  for (int r = 0; r < ep::MAX_P2P; ++r) {
    P.base[r] = r < world ? static_cast<uint8_t*>(peers_host[r]) : nullptr;
    if (r < world) WISP_REQUIRE(P.base[r] && aligned(P.base[r], 256), "ep p2p: peer %d base must be a 256-byte aligned mapping", r);
  }
  return WISP_OK;
}

int wisp_ep_dispatch_p2p(const uint16_t* x, int N, int64_t H, const int64_t* sel, int k, int E_local, int world, int rank,
                         int64_t capacity, int64_t slot_base, int set, void* const* peers_host, int32_t* src_pos, void* stream) {
  WISP_REQUIRE(x && sel && src_pos, "wisp_ep_dispatch_p2p: NULL pointer");
  WISP_REQUIRE(N >= 1 && k >= 1 && int64_t(N) * k <= ep::MAX_PAIRS, "wisp_ep_dispatch_p2p: need 1 <= N*k <= %d", ep::MAX_PAIRS);
  WISP_REQUIRE(E_local >= 1 && capacity >= int64_t(N) * k && (set == 0 || set == 1), "wisp_ep_dispatch_p2p: bad capacity or set");
  WISP_REQUIRE(H > 0 && H % 8 == 0 && aligned(x, 16), "wisp_ep_dispatch_p2p: H %% 8 == 0 and 16-byte aligned x");
  ep::Peers P;
  int rc = p2p_peers(peers_host, world, rank, P);
  if (rc) return rc;
  const int Pn = N * k;
  const int grid = Pn < 2 * num_sms() ? Pn : 2 * num_sms();
  cudaError_t e = launch_pdl(ep::ep_dispatch_p2p_kernel, grid, 256, 0, static_cast<cudaStream_t>(stream), x, N, H, sel, k,
                             E_local, world, rank, capacity, slot_base, set, P, src_pos);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_ep_dispatch_p2p: %s", cudaGetErrorString(e));
  return check_launch("ep_dispatch_p2p");
}

int wisp_ep_wait(void* local, int world, int64_t capacity, int64_t H, int phase, void* stream) {
  WISP_REQUIRE(local && world >= 1 && world <= ep::MAX_P2P && (phase == 0 || phase == 1), "wisp_ep_wait: bad arguments");
  cudaError_t e = launch_pdl(ep::ep_wait_kernel, 1, 32, 0, static_cast<cudaStream_t>(stream), static_cast<uint8_t*>(local), world,
                             capacity, H, phase);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_ep_wait: %s", cudaGetErrorString(e));
  return check_launch("ep_wait");
}

int wisp_ep_return_p2p(const uint16_t* y, int world, int rank, int64_t capacity, int64_t H, int set, void* const* peers_host,
                       void* stream) {
  WISP_REQUIRE(y && (set == 0 || set == 1) && H % 8 == 0 && aligned(y, 16), "wisp_ep_return_p2p: bad arguments");
  ep::Peers P;
  int rc = p2p_peers(peers_host, world, rank, P);
  if (rc) return rc;
  const int64_t rows = int64_t(world) * capacity;
  const int grid = int(rows < 2 * num_sms() ? rows : 2 * num_sms());
  cudaError_t e = launch_pdl(ep::ep_return_p2p_kernel, grid, 256, 0, static_cast<cudaStream_t>(stream), y, world, rank, capacity, H,
                             set, P);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_ep_return_p2p: %s", cudaGetErrorString(e));
  return check_launch("ep_return_p2p");
}

int wisp_ep_combine_p2p(void* local, int world, int64_t capacity, int64_t H, int set, int N, int k, const int32_t* src_pos,
                        const float* w, uint16_t* out, void* stream) {
  WISP_REQUIRE(local && src_pos && w && out && (set == 0 || set == 1), "wisp_ep_combine_p2p: bad arguments");
  WISP_REQUIRE(world >= 1 && world <= ep::MAX_P2P && N >= 1 && k >= 1 && H % 4 == 0 && aligned(out, 8),
               "wisp_ep_combine_p2p: bad shape");
  const int64_t work = int64_t(N) * H / 4;
  const int64_t g = (work + 255) / 256;
  const int grid = int(g < 4 * num_sms() ? g : 4 * num_sms());
  cudaError_t e = launch_pdl(ep::ep_combine_p2p_kernel, grid, 256, 0, static_cast<cudaStream_t>(stream), static_cast<uint8_t*>(local),
                             world, capacity, set, N, k, H, src_pos, w, out);
  if (e != cudaSuccess) return fail(WISP_ERR_CUDA, "wisp_ep_combine_p2p: %s", cudaGetErrorString(e));
  return check_launch("ep_combine_p2p");
}

}  // extern "C"
