// C ABI of the evict() prefill path (declared in include/flash_evict.h).
//
// Host side only: argument checks, TMA tensor-map encoding for arbitrarily
// strided Q/K/V, kernel selection by head dimension and dtype, launches on the
// caller's stream.  No device allocation and no host synchronization on the
// compute entry points; the first compute call of the process allocates one
// small array of mapped pinned host memory for the per-device status words
// (see attach_status).  The library links the CUDA runtime statically; because the
// caller (PyTorch) has its own runtime instance, every entry point first makes
// the device that owns the input pointer current for this runtime.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "fe_forward.cuh"
#include "fe_gather.cuh"
#include "fe_replay.cuh"
#include "fe_select.cuh"
#include "fe_snap.cuh"

namespace {

thread_local char g_err[512] = "";
int64_t g_watchdog_ns = 2000000000LL;

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(FE_STATUS_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Identity of the CUDA context current on this thread (cuCtxGetId + 1; 0 if
// unknown).  Per-device caches below are keyed on it, so a context that was
// destroyed and re-created (cudaDeviceReset) is set up again instead of
// reusing addresses that belonged to the old one.
unsigned long long current_ctx_id() {
  static PFN_cuCtxGetCurrent_v4000 get_cur = nullptr;
  static PFN_cuCtxGetId_v12000 get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_cur = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
  });
  if (!get_cur || !get_id) return 0;
  CUcontext c = nullptr;
  if (get_cur(&c) != CUDA_SUCCESS) return 0;
  if (c == nullptr) {
    // No context bound to this thread yet: cudaSetDevice creates (or binds)
    // the device's primary context.
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess || cudaSetDevice(d) != cudaSuccess) return 0;
    if (get_cur(&c) != CUDA_SUCCESS || c == nullptr) return 0;
  }
  unsigned long long id = 0;
  if (get_id(c, &id) != CUDA_SUCCESS) return 0;
  return id + 1;
}

// ------------------------------------------------ host-visible status word --
// Kernels that give up on a wait (watchdog) raise the device status word and,
// once the library has attached it, also write the code into this device's
// word of a mapped pinned host array.  Every compute entry point reads that
// word on entry (plain host memory, no synchronization): a code left there by
// an earlier call's kernel is returned as that call's error and cleared, so an
// asynchronous failure surfaces at the caller's next call on the device.
constexpr int kMaxDevices = 64;
std::mutex g_status_mu;
int* g_status_words = nullptr;                        // [kMaxDevices], mapped pinned host memory
unsigned long long g_status_ctx[kMaxDevices] = {0};  // context the word was attached in
thread_local bool g_no_attach = false;                 // set inside the allocation-free entry point

__global__ void fe_attach_status_kernel(int* word) { fe::g_status_host = word; }

// Attach `dev`'s host word for the current context: allocate the pinned array
// once per process (the only allocation this library makes on its own) and
// publish the word's address to the device with a one-thread kernel on the
// caller's stream (stream-ordered before the caller's kernels).  Skipped
// while the stream is being captured; a later uncaptured call attaches.
int attach_status(int dev, void* stream) {
  if (dev < 0 || dev >= kMaxDevices || g_no_attach) return FE_STATUS_OK;
  const unsigned long long ctx = current_ctx_id();
  if (ctx == 0) return FE_STATUS_OK;
  std::lock_guard<std::mutex> lock(g_status_mu);
  if (g_status_ctx[dev] == ctx) return FE_STATUS_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) return FE_STATUS_OK;
  if (g_status_words == nullptr) {
    // Relaxed capture mode for this one allocation, in case another thread
    // of the process is capturing a graph in global mode.
    cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
    cudaThreadExchangeStreamCaptureMode(&mode);
    void* h = nullptr;
    cudaError_t e = cudaHostAlloc(&h, kMaxDevices * sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable);
    cudaThreadExchangeStreamCaptureMode(&mode);
    if (e != cudaSuccess) return cuda_fail(e, "cudaHostAlloc (status words)");
    memset(h, 0, kMaxDevices * sizeof(int));
    g_status_words = static_cast<int*>(h);
  }
  int* dptr = nullptr;
  cudaError_t e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&dptr), g_status_words + dev, 0);
  if (e != cudaSuccess) return cuda_fail(e, "cudaHostGetDevicePointer (status word)");
  fe_attach_status_kernel<<<1, 1, 0, s>>>(dptr);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "status attach launch");
  g_status_ctx[dev] = ctx;
  return FE_STATUS_OK;
}

const char* status_name(int code) {
  switch (code) {
    case FE_STATUS_TIMEOUT: return "device watchdog timeout";
    case FE_STATUS_BAD_INDEX: return "gather index out of range";
    default: return "device error";
  }
}

// Take (read and clear) a status code that an earlier call's kernel left in
// `dev`'s host word; non-zero codes become this call's error.
int take_pending(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return FE_STATUS_OK;
  int* words = __atomic_load_n(&g_status_words, __ATOMIC_ACQUIRE);
  if (words == nullptr) return FE_STATUS_OK;
  const int code = __atomic_exchange_n(words + dev, 0, __ATOMIC_ACQ_REL);
  if (code == FE_STATUS_OK) return FE_STATUS_OK;
  return fail(code, "a kernel launched by an earlier call on device %d stopped: %s (its outputs are NaN where "
              "the kernel could mark them, otherwise undefined); this call launched nothing", dev, status_name(code));
}

// Make the device owning `ptr` current for this runtime instance.
int bind_device(const void* ptr, int* dev_out) {
  cudaPointerAttributes a;
  cudaError_t e = cudaPointerGetAttributes(&a, ptr);
  if (e != cudaSuccess) return cuda_fail(e, "cudaPointerGetAttributes");
  if (a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged)
    return fail(FE_STATUS_INVALID, "pointer %p is not device memory", ptr);
  int cur = -1;
  cudaGetDevice(&cur);
  if (cur != a.device) {
    e = cudaSetDevice(a.device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  }
  if (dev_out) *dev_out = a.device;
  return FE_STATUS_OK;
}

// Entry of a compute call: bind the device owning `ptr`, report a status an
// earlier call's kernel raised, and attach the host status word if needed.
int enter(const void* ptr, void* stream, int* dev_out = nullptr) {
  int dev = 0;
  int rc = bind_device(ptr, &dev);
  if (rc) return rc;
  if ((rc = take_pending(dev))) return rc;
  if ((rc = attach_status(dev, stream))) return rc;
  if (dev_out) *dev_out = dev;
  return FE_STATUS_OK;
}

int padded_dim(int64_t d) { return d <= 64 ? 64 : (d <= 128 ? 128 : (d <= 256 ? 256 : 0)); }

// TMA map over a [B, H, N, D] view with element strides s[4] (s[3] == 1),
// box = 64 channels x box_rows tokens, 128-byte swizzle, zero fill out of bounds.
int make_map(CUtensorMap* m, const void* ptr, const int64_t* s, int64_t B, int64_t H, int64_t N, int64_t D,
             int dtype, const char* name, int box_rows = 128) {
  if (s[3] != 1) return fail(FE_STATUS_UNSUPPORTED, "%s: channel stride must be 1 (got %lld)", name, (long long)s[3]);
  if (reinterpret_cast<uintptr_t>(ptr) % 16)
    return fail(FE_STATUS_UNSUPPORTED, "%s: base pointer must be 16-byte aligned", name);
  const int64_t ext[3] = {N, H, B};
  const int64_t st[3] = {s[2], s[1], s[0]};
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)N, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t gstr[3];
  int64_t fallback = D * 2;
  for (int i = 0; i < 3; ++i) {
    int64_t bytes = st[i] * 2;
    if (ext[i] == 1) {
      // Never stepped over: any legal stride works.
      bytes = (fallback + 15) / 16 * 16;
    }
    if (bytes <= 0 || bytes % 16 != 0 || bytes >= (int64_t(1) << 40))
      return fail(FE_STATUS_UNSUPPORTED, "%s: stride %lld elements is not a positive multiple of 8", name,
                  (long long)st[i]);
    gstr[i] = (cuuint64_t)bytes;
    fallback = bytes * ext[i];
  }
  if (box_rows < 1 || box_rows > 256) return fail(FE_STATUS_INVALID, "%s: bad TMA box", name);
  cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  auto enc = encode_fn();
  if (!enc) return fail(FE_STATUS_CUDA, "cuTensorMapEncodeTiled unavailable");
  CUresult r = enc(m, dtype == FE_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                   const_cast<void*>(ptr), dims, gstr, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FE_STATUS_UNSUPPORTED, "%s: cuTensorMapEncodeTiled failed (%d)", name, (int)r);
  return FE_STATUS_OK;
}

int check_shapes(int64_t B, int64_t Hq, int64_t Hkv, int64_t N, int64_t D, int dtype) {
  if (B < 1 || Hq < 1 || Hkv < 1 || N < 1 || D < 1)
    return fail(FE_STATUS_INVALID, "empty shape B=%lld Hq=%lld Hkv=%lld N=%lld D=%lld", (long long)B, (long long)Hq,
                (long long)Hkv, (long long)N, (long long)D);
  if (Hq % Hkv) return fail(FE_STATUS_INVALID, "q_heads must be divisible by kv_heads");
  if (dtype != FE_DTYPE_F16 && dtype != FE_DTYPE_BF16) return fail(FE_STATUS_INVALID, "dtype must be f16 or bf16");
  if (D > 256) return fail(FE_STATUS_INVALID, "channels must be <= 256");
  if (padded_dim(D) == 0) return fail(FE_STATUS_UNSUPPORTED, "channels > 256 are not supported by the sm_100a kernels");
  if (N > (int64_t(1) << 30) || B * Hq > (int64_t(1) << 30)) return fail(FE_STATUS_UNSUPPORTED, "problem too large");
  return FE_STATUS_OK;
}

// Opt a kernel into `bytes` of dynamic shared memory, once per (kernel,
// device).  Keyed by the kernel's address: every template instantiation is a
// distinct kernel even when the function types coincide.
template <typename K>
int set_smem(K kernel, int bytes) {
  struct Entry {
    const void* fn;
    int dev;
    int bytes;
  };
  static Entry cache[256];
  static int used = 0;
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  const void* fn = reinterpret_cast<const void*>(kernel);
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (cache[i].fn == fn && cache[i].dev == dev && cache[i].bytes >= bytes) return FE_STATUS_OK;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
  if (used < 256) cache[used++] = Entry{fn, dev, bytes};
  return FE_STATUS_OK;
}

template <bool BF16, int DQK, int DV>
int launch_fwd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const fe::FwdParams& p,
               int64_t items, cudaStream_t stream) {
  using C = fe::FwdCfg<DQK, DV>;
  auto kern = fe::fe_fwd_kernel<BF16, DQK, DV>;
  int rc = set_smem(kern, C::SMEM);
  if (rc) return rc;
  // The kernel moves registers between its warpgroups (setmaxnreg); that is
  // only safe if the launch allocation covers the split.  Refuse otherwise.
  // (one cached value per instantiation; host threads may race to fill it
  // with the same number)
  static std::atomic<int> checked_regs{0};
  int regs = checked_regs.load(std::memory_order_relaxed);
  if (regs == 0) {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncGetAttributes");
    regs = fa.numRegs;
    checked_regs.store(regs, std::memory_order_relaxed);
  }
  if (regs < fe::FWD_REGS_NEEDED)
    return fail(FE_STATUS_UNSUPPORTED, "attention kernel compiled with %d registers/thread, needs %d", regs,
                fe::FWD_REGS_NEEDED);
  kern<<<dim3((unsigned)items), dim3(C::THREADS), C::SMEM, stream>>>(tq, tk, tv, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "attention launch");
  return FE_STATUS_OK;
}

template <bool BF16, int DP>
int launch_replay(const CUtensorMap& tq, const CUtensorMap& tk, const fe::ReplayParams& p, int64_t items,
                  cudaStream_t stream) {
  using C = fe::ReplayCfg<DP>;
  auto kern = fe::fe_replay_kernel<BF16, DP>;
  int rc = set_smem(kern, C::SMEM);
  if (rc) return rc;
  kern<<<dim3((unsigned)items), dim3(C::THREADS), C::SMEM, stream>>>(tq, tk, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "replay launch");
  return FE_STATUS_OK;
}

// Describe a K/V gather: byte strides, destination rows and the widest chunk
// (16/8/4/2/1 bytes) that divides the row size, every stride that is stepped
// over and every base address.
int make_gather_spec(fe::GatherSpec* g, const void* k, const int64_t* k_strides, const void* v,
                     const int64_t* v_strides, void* k_out, void* v_out, int64_t batch, int64_t heads, int64_t tokens,
                     int64_t budget, int64_t channels, int64_t elem_bytes) {
  if (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4 && elem_bytes != 8)
    return fail(FE_STATUS_INVALID, "elem_bytes must be 1, 2, 4 or 8");
  if (channels < 1 || channels > (int64_t(1) << 20)) return fail(FE_STATUS_INVALID, "bad channels");
  if (!k || !k_strides || !k_out) return fail(FE_STATUS_INVALID, "null pointer");
  if ((v == nullptr) != (v_out == nullptr) || (v && !v_strides))
    return fail(FE_STATUS_INVALID, "v and v_out must both be given or both be null");
  const int64_t* strides[2] = {k_strides, v_strides};
  const char* names[2] = {"k", "v"};
  for (int t = 0; t < (v ? 2 : 1); ++t) {
    if (strides[t][3] != 1) return fail(FE_STATUS_UNSUPPORTED, "%s: channel stride must be 1", names[t]);
    for (int i = 0; i < 3; ++i)
      if (strides[t][i] < 0) return fail(FE_STATUS_UNSUPPORTED, "%s: negative strides are not supported", names[t]);
  }
  memset(g, 0, sizeof(*g));
  g->k_src = static_cast<const uint8_t*>(k);
  g->v_src = static_cast<const uint8_t*>(v);
  g->k_sb = k_strides[0] * elem_bytes;
  g->k_sh = k_strides[1] * elem_bytes;
  g->k_sn = k_strides[2] * elem_bytes;
  if (v) {
    g->v_sb = v_strides[0] * elem_bytes;
    g->v_sh = v_strides[1] * elem_bytes;
    g->v_sn = v_strides[2] * elem_bytes;
  }
  g->k_dst = static_cast<uint8_t*>(k_out);
  g->v_dst = static_cast<uint8_t*>(v_out);
  g->heads = heads;
  g->tokens = tokens;
  g->budget = budget;
  g->row_bytes = (int)(channels * elem_bytes);
  int64_t vals[12];
  int nv = 0;
  vals[nv++] = g->row_bytes;
  vals[nv++] = (int64_t)reinterpret_cast<uintptr_t>(k);
  vals[nv++] = (int64_t)reinterpret_cast<uintptr_t>(k_out);
  if (batch > 1) vals[nv++] = g->k_sb;
  if (heads > 1) vals[nv++] = g->k_sh;
  if (tokens > 1) vals[nv++] = g->k_sn;
  if (v) {
    vals[nv++] = (int64_t)reinterpret_cast<uintptr_t>(v);
    vals[nv++] = (int64_t)reinterpret_cast<uintptr_t>(v_out);
    if (batch > 1) vals[nv++] = g->v_sb;
    if (heads > 1) vals[nv++] = g->v_sh;
    if (tokens > 1) vals[nv++] = g->v_sn;
  }
  int vec = 16;
  for (int i = 0; i < nv; ++i)
    while (vec > 1 && vals[i] % vec) vec >>= 1;
  g->vec = vec;
  return FE_STATUS_OK;
}

// SnapKV geometry: row groups of the packed window rows and the key chunks of
// the statistics pass (a pure function of the shape, so the workspace size
// query and the launch agree).
struct SnapGeometry {
  int w, w8, hpg, ppg, groups, nchunk, chunk_tiles, box;
  int64_t workspace_floats;
};

int snap_geometry(int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t tokens, int64_t window, SnapGeometry* g) {
  if (batch < 1 || q_heads < 1 || kv_heads < 1 || tokens < 1 || q_heads % kv_heads)
    return fail(FE_STATUS_INVALID, "bad shape");
  if (window < 1) return fail(FE_STATUS_INVALID, "window must be a positive integer");
  if (tokens > (int64_t(1) << 30)) return fail(FE_STATUS_UNSUPPORTED, "problem too large");
  const int64_t G = q_heads / kv_heads;
  g->w = (int)(window < tokens ? window : tokens);
  g->w8 = (g->w + 7) / 8 * 8;
  if (g->w8 <= 256) {
    g->hpg = 256 / g->w8;
    g->ppg = 0;
    g->groups = (int)((G + g->hpg - 1) / g->hpg);
    g->box = g->w8;
  } else {
    g->hpg = 0;
    g->ppg = (g->w + 255) / 256;
    g->groups = (int)(G * g->ppg);
    g->box = 256;
  }
  const int64_t units = batch * kv_heads * g->groups;
  const int64_t ntiles = (tokens + 127) / 128;
  // About one statistics CTA per SM, at most 32 partials per row.
  int64_t n = (148 + units - 1) / units;
  if (n > 32) n = 32;
  if (n > ntiles) n = ntiles;
  if (n < 1) n = 1;
  g->chunk_tiles = (int)((ntiles + n - 1) / n);
  g->nchunk = (int)((ntiles + g->chunk_tiles - 1) / g->chunk_tiles);
  g->workspace_floats = units * g->nchunk * 256 * 2;
  if (units * g->nchunk > 0x7fffffff || batch * kv_heads * ntiles > 0x7fffffff)
    return fail(FE_STATUS_UNSUPPORTED, "grid too large");
  return FE_STATUS_OK;
}

template <bool BF16, int DP>
int launch_snap(const CUtensorMap& tq, const CUtensorMap& tk, const fe::SnapParams& p, int64_t stats_items,
                int64_t score_items, cudaStream_t stream) {
  using C = fe::SnapCfg<DP>;
  auto ka = fe::fe_snap_stats_kernel<BF16, DP>;
  auto kb = fe::fe_snap_score_kernel<BF16, DP>;
  int rc = set_smem(ka, C::A_SMEM);
  if (rc) return rc;
  rc = set_smem(kb, C::B_SMEM);
  if (rc) return rc;
  ka<<<dim3((unsigned)stats_items), dim3(C::THREADS), C::A_SMEM, stream>>>(tq, tk, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "snap statistics launch");
  kb<<<dim3((unsigned)score_items), dim3(C::THREADS), C::B_SMEM, stream>>>(tq, tk, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "snap score launch");
  return FE_STATUS_OK;
}

__global__ void fe_watchdog_kernel(uint64_t timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    fe::mbar_init(&bar, 1);
    fe::fence_mbar_init();
  }
  __syncthreads();
  // Nothing ever arrives on `bar`: the bounded wait must give up and report.
  fe::mbar_wait(&bar, 0, timeout_ns, &abort_flag);
  __syncthreads();
}

__global__ void fe_exp2_selftest_kernel(const float* in, float* poly, float* mufu, int64_t n) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i < n) {
    float lo, hi;
    fe::f2_unpack(fe::exp2_poly_x2(fe::f2_pack(in[i], in[i])), lo, hi);
    poly[i] = lo;
    mufu[i] = fe::ex2_approx(in[i]);
  }
}

}  // namespace

extern "C" {

int fe_abi_version(void) { return 3; }

int fe_selftest_exp2(const float* in, float* out_poly, float* out_mufu, int64_t n, void* stream) {
  g_err[0] = 0;
  if (n < 0 || (n > 0 && (!in || !out_poly || !out_mufu))) return fail(FE_STATUS_INVALID, "bad arguments");
  if (n == 0) return FE_STATUS_OK;
  int rc = enter(in, stream);
  if (rc) return rc;
  const int64_t blocks = (n + 255) / 256;
  if (blocks > 0x7fffffff) return fail(FE_STATUS_UNSUPPORTED, "n too large");
  fe_exp2_selftest_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(in, out_poly, out_mufu,
                                                                                              n);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "exp2 self-test launch");
  return FE_STATUS_OK;
}

const char* fe_last_error(void) { return g_err; }

void fe_set_watchdog_ns(int64_t ns) { g_watchdog_ns = ns > 0 ? ns : 2000000000LL; }

int fe_attention_fwd(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                     const void* v, const int64_t* v_strides, void* out, float* row_stats, int64_t batch,
                     int64_t q_heads, int64_t kv_heads, int64_t tokens, int64_t channels, int dtype, int causal,
                     float scale, const int32_t* query_blocks, int64_t num_query_blocks, void* stream) {
  g_err[0] = 0;
  int rc = check_shapes(batch, q_heads, kv_heads, tokens, channels, dtype);
  if (rc) return rc;
  if (!q || !k || !v || !out || !row_stats) return fail(FE_STATUS_INVALID, "null pointer");
  if (!std::isfinite(scale)) return fail(FE_STATUS_INVALID, "scale must be finite");
  if (reinterpret_cast<uintptr_t>(out) % 16) return fail(FE_STATUS_UNSUPPORTED, "out must be 16-byte aligned");
  rc = enter(q, stream);
  if (rc) return rc;
  CUtensorMap tq, tk, tv;
  if ((rc = make_map(&tq, q, q_strides, batch, q_heads, tokens, channels, dtype, "q"))) return rc;
  if ((rc = make_map(&tk, k, k_strides, batch, kv_heads, tokens, channels, dtype, "k"))) return rc;
  if ((rc = make_map(&tv, v, v_strides, batch, kv_heads, tokens, channels, dtype, "v"))) return rc;
  const int64_t nblk_all = (tokens + FE_QUERY_BLOCK - 1) / FE_QUERY_BLOCK;
  if (query_blocks && (num_query_blocks < 0 || num_query_blocks > nblk_all))
    return fail(FE_STATUS_INVALID, "num_query_blocks out of range");
  fe::FwdParams p;
  p.out = out;
  p.row_stats = row_stats;
  p.blocks = query_blocks;
  p.num_blocks = (int)(query_blocks ? num_query_blocks : nblk_all);
  p.B = (int)batch;
  p.Hq = (int)q_heads;
  p.Hkv = (int)kv_heads;
  p.N = (int)tokens;
  p.D = (int)channels;
  p.G = (int)(q_heads / kv_heads);
  p.sc = (float)((double)scale * 1.4426950408889634);
  p.causal = causal ? 1 : 0;
  p.timeout_ns = (uint64_t)g_watchdog_ns;
  const int64_t items = (int64_t)p.num_blocks * batch * q_heads;
  if (items == 0) return FE_STATUS_OK;
  if (items > 0x7fffffff) return fail(FE_STATUS_UNSUPPORTED, "grid too large");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int dp = padded_dim(channels);
  p.vcol0 = 0;
  if (dp == 256) {
    // Two launches, one per 128-channel half of V and O; both compute the
    // same S and row statistics (written by the first).
    rc = dtype == FE_DTYPE_BF16 ? launch_fwd<true, 256, 128>(tq, tk, tv, p, items, s)
                                : launch_fwd<false, 256, 128>(tq, tk, tv, p, items, s);
    if (rc) return rc;
    p.vcol0 = 128;
    return dtype == FE_DTYPE_BF16 ? launch_fwd<true, 256, 128>(tq, tk, tv, p, items, s)
                                  : launch_fwd<false, 256, 128>(tq, tk, tv, p, items, s);
  }
  if (dtype == FE_DTYPE_BF16)
    return dp == 64 ? launch_fwd<true, 64, 64>(tq, tk, tv, p, items, s)
                    : launch_fwd<true, 128, 128>(tq, tk, tv, p, items, s);
  return dp == 64 ? launch_fwd<false, 64, 64>(tq, tk, tv, p, items, s)
                  : launch_fwd<false, 128, 128>(tq, tk, tv, p, items, s);
}

int64_t fe_replay_first_scored_row(int64_t tokens, float recency_decay, int64_t observation_window) {
  const int64_t W = (observation_window <= 0 || observation_window > tokens) ? tokens : observation_window;
  int64_t s_lo = tokens - W;
  if (recency_decay > 0) {
    // Rows farther than this from the end have FP32 weights below 2^-127.
    const double reach = 127.0 / ((double)recency_decay * 1.4426950408889634);
    if (reach < (double)tokens) {
      const int64_t cut = tokens - 1 - (int64_t)std::floor(reach);
      if (cut > s_lo) s_lo = cut;
    }
  }
  return s_lo;
}

int fe_replay_scores(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides, const void* v,
                     const int64_t* v_strides, const float* row_stats, float* importance, int64_t batch,
                     int64_t q_heads, int64_t kv_heads, int64_t tokens, int64_t channels, int dtype, int causal,
                     float scale, float recency_decay, int64_t observation_window, int value_weighted,
                     const int32_t* query_blocks, int64_t num_query_blocks, void* stream) {
  return fe_replay_scores_range(q, q_strides, k, k_strides, v, v_strides, row_stats, importance, batch, q_heads,
                                kv_heads, tokens, channels, dtype, causal, scale, recency_decay, observation_window,
                                value_weighted, query_blocks, num_query_blocks, 0, (tokens + 127) / 128, stream);
}

int fe_replay_scores_range(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                           const void* v, const int64_t* v_strides, const float* row_stats, float* importance,
                           int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t tokens, int64_t channels,
                           int dtype, int causal, float scale, float recency_decay, int64_t observation_window,
                           int value_weighted, const int32_t* query_blocks, int64_t num_query_blocks,
                           int64_t key_tile_begin, int64_t key_tile_end, void* stream) {
  g_err[0] = 0;
  const int64_t ntiles_all = (tokens + 127) / 128;
  if (key_tile_begin < 0 || key_tile_end > ntiles_all || key_tile_begin > key_tile_end)
    return fail(FE_STATUS_INVALID, "key tile range [%lld, %lld) outside [0, %lld)", (long long)key_tile_begin,
                (long long)key_tile_end, (long long)ntiles_all);
  if (key_tile_begin == key_tile_end) return FE_STATUS_OK;
  int rc = check_shapes(batch, q_heads, kv_heads, tokens, channels, dtype);
  if (rc) return rc;
  if (!q || !k || !v || !row_stats || !importance) return fail(FE_STATUS_INVALID, "null pointer");
  if (!std::isfinite(scale)) return fail(FE_STATUS_INVALID, "scale must be finite");
  if (!std::isfinite(recency_decay) || recency_decay < 0)
    return fail(FE_STATUS_INVALID, "recency_decay must be finite and nonnegative");
  if (observation_window < 0) return fail(FE_STATUS_INVALID, "observation_window must be >= 0");
  if (v_strides[3] != 1) return fail(FE_STATUS_UNSUPPORTED, "v: channel stride must be 1");
  rc = enter(q, stream);
  if (rc) return rc;
  CUtensorMap tq, tk;
  if ((rc = make_map(&tq, q, q_strides, batch, q_heads, tokens, channels, dtype, "q"))) return rc;
  if ((rc = make_map(&tk, k, k_strides, batch, kv_heads, tokens, channels, dtype, "k"))) return rc;
  const int64_t nblk_all = (tokens + FE_QUERY_BLOCK - 1) / FE_QUERY_BLOCK;
  if (query_blocks) {
    if (num_query_blocks < 0 || num_query_blocks > nblk_all)
      return fail(FE_STATUS_INVALID, "num_query_blocks out of range");
    if (nblk_all > fe::ReplayCfg<64>::MAP_WORDS * 32)
      return fail(FE_STATUS_UNSUPPORTED, "query-block lists are limited to %d blocks", fe::ReplayCfg<64>::MAP_WORDS * 32);
  }
  fe::ReplayParams p;
  p.row_stats = row_stats;
  p.importance = importance;
  p.v = reinterpret_cast<const uint8_t*>(v);
  p.v_sb = v_strides[0];
  p.v_sh = v_strides[1];
  p.v_sn = v_strides[2];
  p.blocks = query_blocks;
  p.num_blocks = (int)(query_blocks ? num_query_blocks : nblk_all);
  p.B = (int)batch;
  p.Hq = (int)q_heads;
  p.Hkv = (int)kv_heads;
  p.N = (int)tokens;
  p.D = (int)channels;
  p.G = (int)(q_heads / kv_heads);
  p.sc = (float)((double)scale * 1.4426950408889634);
  p.decay_log2 = (float)((double)recency_decay * 1.4426950408889634);
  p.s_lo = (int)fe_replay_first_scored_row(tokens, recency_decay, observation_window);
  p.causal = causal ? 1 : 0;
  p.weighted = value_weighted ? 1 : 0;
  p.timeout_ns = (uint64_t)g_watchdog_ns;
  p.kt0 = (int)key_tile_begin;
  p.nkt = (int)(key_tile_end - key_tile_begin);
  const int64_t items = (int64_t)p.nkt * batch * kv_heads;
  if (items > 0x7fffffff) return fail(FE_STATUS_UNSUPPORTED, "grid too large");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int dp = padded_dim(channels);
  if (dtype == FE_DTYPE_BF16)
    return dp == 64    ? launch_replay<true, 64>(tq, tk, p, items, s)
           : dp == 128 ? launch_replay<true, 128>(tq, tk, p, items, s)
                       : launch_replay<true, 256>(tq, tk, p, items, s);
  return dp == 64    ? launch_replay<false, 64>(tq, tk, p, items, s)
         : dp == 128 ? launch_replay<false, 128>(tq, tk, p, items, s)
                     : launch_replay<false, 256>(tq, tk, p, items, s);
}

}  // extern "C"

namespace {

// Selection launch for npol policies over the same rows x tokens shape; with
// g[i] != nullptr policy i's launch also compacts K/V.
int select_multi_impl(int64_t rows, int64_t tokens, int npol, const float* const* importance,
                      const int64_t* budgets, const int64_t* recents, const int64_t* pools, int64_t* const* indices,
                      uint8_t* const* masks, int mask_evict, const fe::GatherSpec* const* g, void* stream) {
  if (rows < 0 || tokens < 1) return fail(FE_STATUS_INVALID, "bad rows/tokens");
  if (npol < 1 || npol > fe::SEL_MAX_POLICIES)
    return fail(FE_STATUS_INVALID, "npolicies must be in [1, %d]", fe::SEL_MAX_POLICIES);
  for (int i = 0; i < npol; ++i) {
    if (budgets[i] < 1 || budgets[i] > tokens)
      return fail(FE_STATUS_INVALID, "budget must be an integer in [1, sequence length]");
    if (recents[i] < 0 || recents[i] > budgets[i]) return fail(FE_STATUS_INVALID, "recent must be an integer in [0, budget]");
    if (pools[i] < 1 || pools[i] % 2 != 1) return fail(FE_STATUS_INVALID, "pool_kernel must be a positive odd integer");
  }
  if (rows == 0) return FE_STATUS_OK;
  for (int i = 0; i < npol; ++i)
    if (!importance[i] || !indices[i] || !masks[i]) return fail(FE_STATUS_INVALID, "null pointer");
  int rc = enter(importance[0], stream);
  if (rc) return rc;
  const int64_t max_slice = fe::SEL_SMEM_KEYS;
  // Cluster size (shared by the policies): enough CTAs for the longest past
  // region to fit in shared memory, and up to 8 for long rows (>= 4096 keys
  // per CTA) so few rows still use many SMs.  Rows longer than 16 slices
  // run the global-key variant (keys recomputed from the scores each pass).
  int64_t pmax = 0;
  for (int i = 0; i < npol; ++i) pmax = std::max<int64_t>(pmax, tokens - recents[i]);
  int cl = 1;
  while (cl < 16 && (pmax + cl - 1) / cl > max_slice) cl *= 2;
  while (cl < 8 && pmax / (2 * cl) >= 4096) cl *= 2;
  const bool smem_keys = (pmax + cl - 1) / cl <= max_slice;
  if (pmax / cl > 0x7fffffff - fe::SEL_THREADS)
    return fail(FE_STATUS_UNSUPPORTED, "sequence length %lld exceeds the selection limit", (long long)tokens);
  if (rows * cl * npol > 0x7fffffff) return fail(FE_STATUS_UNSUPPORTED, "too many rows");
  fe::SelectLaunch L;
  memset(&L, 0, sizeof(L));
  L.rows = rows;
  L.npol = npol;
  int64_t max_chunk = 1;
  for (int i = 0; i < npol; ++i) {
    fe::SelectParams& p = L.pol[i];
    const int64_t P = tokens - recents[i];
    int64_t chunk = (P + cl - 1) / cl;
    if (chunk < 1) chunk = 1;
    max_chunk = std::max(max_chunk, chunk);
    p.importance = importance[i];
    p.N = tokens;
    p.budget = budgets[i];
    p.recent = recents[i];
    p.pool = (int)pools[i];
    p.indices = indices[i];
    p.mask = masks[i];
    p.mask_evict = mask_evict ? 1 : 0;
    p.chunk = chunk;
    p.gather = (g && g[i]) ? 1 : 0;
    if (p.gather) p.g = *g[i];
  }
  const int smem = smem_keys ? (int)(max_chunk * 4) : 0;
  auto kern = smem_keys ? fe::fe_select_kernel<true> : fe::fe_select_kernel<false>;
  rc = set_smem(kern, smem < 49152 ? 49152 : smem);
  if (rc) return rc;
  if (cl > 8) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return cuda_fail(e, "cluster attribute");
  }
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3((unsigned)(rows * cl * npol));
  cfg.blockDim = dim3(fe::SEL_THREADS);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, L);
  if (e != cudaSuccess) return cuda_fail(e, "selection launch");
  return FE_STATUS_OK;
}

// Single-policy selection (with an optional gather).
int select_impl(const float* importance, int64_t rows, int64_t tokens, int64_t budget, int64_t recent,
                int64_t pool_kernel, int64_t* indices, uint8_t* mask, int mask_evict, const fe::GatherSpec* g,
                void* stream) {
  const fe::GatherSpec* gs[1] = {g};
  return select_multi_impl(rows, tokens, 1, &importance, &budget, &recent, &pool_kernel, &indices, &mask, mask_evict,
                           gs, stream);
}

}  // namespace

extern "C" {

int fe_select_tokens(const float* importance, int64_t rows, int64_t tokens, int64_t budget, int64_t recent,
                     int64_t pool_kernel, int64_t* indices, uint8_t* mask, int mask_evict, void* stream) {
  g_err[0] = 0;
  return select_impl(importance, rows, tokens, budget, recent, pool_kernel, indices, mask, mask_evict, nullptr,
                     stream);
}

int fe_gather_tokens(const void* k, const int64_t* k_strides, const void* v, const int64_t* v_strides,
                     const int64_t* indices, void* k_out, void* v_out, int64_t batch, int64_t heads, int64_t tokens,
                     int64_t budget, int64_t channels, int64_t elem_bytes, void* stream) {
  g_err[0] = 0;
  if (batch < 0 || heads < 0 || tokens < 1 || budget < 0) return fail(FE_STATUS_INVALID, "bad shape");
  if (batch == 0 || heads == 0 || budget == 0) return FE_STATUS_OK;
  if (!indices) return fail(FE_STATUS_INVALID, "null pointer");
  fe::GatherSpec g;
  int rc = make_gather_spec(&g, k, k_strides, v, v_strides, k_out, v_out, batch, heads, tokens, budget, channels,
                            elem_bytes);
  if (rc) return rc;
  rc = enter(k, stream);
  if (rc) return rc;
  const int64_t per_row = (budget + fe::GATHER_POSITIONS - 1) / fe::GATHER_POSITIONS;
  const int64_t blocks = per_row * batch * heads;
  if (blocks > 0x7fffffff) return fail(FE_STATUS_UNSUPPORTED, "grid too large");
  fe::fe_gather_kernel<<<(unsigned)blocks, fe::GATHER_THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      g, indices, per_row);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gather launch");
  return FE_STATUS_OK;
}

int fe_select_gather(const float* importance, int64_t batch, int64_t heads, int64_t tokens, int64_t budget,
                     int64_t recent, int64_t pool_kernel, int64_t* indices, uint8_t* mask, int mask_evict,
                     const void* k, const int64_t* k_strides, const void* v, const int64_t* v_strides, void* k_out,
                     void* v_out, int64_t channels, int64_t elem_bytes, void* stream) {
  g_err[0] = 0;
  if (batch < 0 || heads < 0 || tokens < 1) return fail(FE_STATUS_INVALID, "bad shape");
  if (budget < 1 || budget > tokens) return fail(FE_STATUS_INVALID, "budget must be an integer in [1, sequence length]");
  fe::GatherSpec g;
  int rc = make_gather_spec(&g, k, k_strides, v, v_strides, k_out, v_out, batch, heads, tokens, budget, channels,
                            elem_bytes);
  if (rc) return rc;
  return select_impl(importance, batch * heads, tokens, budget, recent, pool_kernel, indices, mask, mask_evict, &g,
                     stream);
}

int fe_select_multi(const float* const* importance, int64_t batch, int64_t heads, int64_t tokens, int npolicies,
                    const int64_t* budgets, const int64_t* recents, const int64_t* pool_kernels,
                    int64_t* const* indices, uint8_t* const* masks, int mask_evict, const void* k,
                    const int64_t* k_strides, const void* v, const int64_t* v_strides, void* const* k_outs,
                    void* const* v_outs, int64_t channels, int64_t elem_bytes, void* stream) {
  g_err[0] = 0;
  if (batch < 0 || heads < 0 || tokens < 1) return fail(FE_STATUS_INVALID, "bad shape");
  if (npolicies < 1 || npolicies > fe::SEL_MAX_POLICIES)
    return fail(FE_STATUS_INVALID, "npolicies must be in [1, %d]", fe::SEL_MAX_POLICIES);
  if (!importance || !budgets || !recents || !pool_kernels || !indices || !masks)
    return fail(FE_STATUS_INVALID, "null pointer");
  fe::GatherSpec specs[fe::SEL_MAX_POLICIES];
  const fe::GatherSpec* gp[fe::SEL_MAX_POLICIES] = {nullptr};
  if (k != nullptr) {
    if (!k_outs) return fail(FE_STATUS_INVALID, "null pointer");
    for (int i = 0; i < npolicies; ++i) {
      if (budgets[i] < 1 || budgets[i] > tokens)
        return fail(FE_STATUS_INVALID, "budget must be an integer in [1, sequence length]");
      int rc = make_gather_spec(&specs[i], k, k_strides, v, v_strides, k_outs[i], v ? (v_outs ? v_outs[i] : nullptr) : nullptr,
                                batch, heads, tokens, budgets[i], channels, elem_bytes);
      if (rc) return rc;
      gp[i] = &specs[i];
    }
  }
  return select_multi_impl(batch * heads, tokens, npolicies, importance, budgets, recents, pool_kernels, indices, masks,
                           mask_evict, gp, stream);
}

int fe_evict(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides, const void* v,
             const int64_t* v_strides, void* out, float* importance, int64_t* indices, uint8_t* mask,
             float* row_stats, int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t tokens, int64_t channels,
             int dtype, int causal, float scale, float recency_decay, int64_t observation_window, int value_weighted,
             int64_t budget, int64_t recent, int64_t pool_kernel, void* stream) {
  if (budget < 1 || budget > tokens) return fail(FE_STATUS_INVALID, "budget must be an integer in [1, sequence length]");
  if (recent < 0 || recent > budget) return fail(FE_STATUS_INVALID, "recent must be an integer in [0, budget]");
  if (pool_kernel < 1 || pool_kernel % 2 != 1) return fail(FE_STATUS_INVALID, "pool_kernel must be a positive odd integer");
  int rc = fe_attention_fwd(q, q_strides, k, k_strides, v, v_strides, out, row_stats, batch, q_heads, kv_heads, tokens,
                            channels, dtype, causal, scale, nullptr, 0, stream);
  if (rc) return rc;
  rc = fe_replay_scores(q, q_strides, k, k_strides, v, v_strides, row_stats, importance, batch, q_heads, kv_heads,
                        tokens, channels, dtype, causal, scale, recency_decay, observation_window, value_weighted,
                        nullptr, 0, stream);
  if (rc) return rc;
  return fe_select_tokens(importance, batch * kv_heads, tokens, budget, recent, pool_kernel, indices, mask, 1, stream);
}

int fe_evict_compact(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides, const void* v,
                     const int64_t* v_strides, void* out, float* importance, int64_t* indices, uint8_t* mask,
                     void* k_out, void* v_out, float* row_stats, int64_t batch, int64_t q_heads, int64_t kv_heads,
                     int64_t tokens, int64_t channels, int dtype, int causal, float scale, float recency_decay,
                     int64_t observation_window, int value_weighted, int64_t budget, int64_t recent,
                     int64_t pool_kernel, void* stream) {
  if (budget < 1 || budget > tokens) return fail(FE_STATUS_INVALID, "budget must be an integer in [1, sequence length]");
  if (recent < 0 || recent > budget) return fail(FE_STATUS_INVALID, "recent must be an integer in [0, budget]");
  if (pool_kernel < 1 || pool_kernel % 2 != 1) return fail(FE_STATUS_INVALID, "pool_kernel must be a positive odd integer");
  if (!k_out || !v_out) return fail(FE_STATUS_INVALID, "null pointer");
  int rc = fe_attention_fwd(q, q_strides, k, k_strides, v, v_strides, out, row_stats, batch, q_heads, kv_heads, tokens,
                            channels, dtype, causal, scale, nullptr, 0, stream);
  if (rc) return rc;
  rc = fe_replay_scores(q, q_strides, k, k_strides, v, v_strides, row_stats, importance, batch, q_heads, kv_heads,
                        tokens, channels, dtype, causal, scale, recency_decay, observation_window, value_weighted,
                        nullptr, 0, stream);
  if (rc) return rc;
  return fe_select_gather(importance, batch, kv_heads, tokens, budget, recent, pool_kernel, indices, mask, 1, k,
                          k_strides, v, v_strides, k_out, v_out, channels, 2, stream);
}

int64_t fe_snap_workspace_floats(int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t tokens, int64_t window) {
  g_err[0] = 0;
  SnapGeometry g;
  if (snap_geometry(batch, q_heads, kv_heads, tokens, window, &g)) return -1;
  return g.workspace_floats;
}

int fe_snap_scores(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides, float* scores,
                   float* workspace, int64_t workspace_floats, int64_t batch, int64_t q_heads, int64_t kv_heads,
                   int64_t tokens, int64_t channels, int dtype, float scale, int64_t window, void* stream) {
  g_err[0] = 0;
  int rc = check_shapes(batch, q_heads, kv_heads, tokens, channels, dtype);
  if (rc) return rc;
  if (!q || !k || !scores || !workspace) return fail(FE_STATUS_INVALID, "null pointer");
  if (!std::isfinite(scale)) return fail(FE_STATUS_INVALID, "scale must be finite");
  SnapGeometry g;
  if ((rc = snap_geometry(batch, q_heads, kv_heads, tokens, window, &g))) return rc;
  if (workspace_floats < g.workspace_floats)
    return fail(FE_STATUS_INVALID, "workspace too small: %lld floats needed", (long long)g.workspace_floats);
  if (reinterpret_cast<uintptr_t>(workspace) % 8) return fail(FE_STATUS_INVALID, "workspace must be 8-byte aligned");
  rc = enter(q, stream);
  if (rc) return rc;
  CUtensorMap tq, tk;
  if ((rc = make_map(&tq, q, q_strides, batch, q_heads, tokens, channels, dtype, "q", g.box))) return rc;
  if ((rc = make_map(&tk, k, k_strides, batch, kv_heads, tokens, channels, dtype, "k"))) return rc;
  fe::SnapParams p;
  p.partial = reinterpret_cast<float2*>(workspace);
  p.scores = scores;
  p.B = (int)batch;
  p.Hq = (int)q_heads;
  p.Hkv = (int)kv_heads;
  p.N = (int)tokens;
  p.D = (int)channels;
  p.G = (int)(q_heads / kv_heads);
  p.w = g.w;
  p.w8 = g.w8;
  p.hpg = g.hpg;
  p.ppg = g.ppg;
  p.groups = g.groups;
  p.nchunk = g.nchunk;
  p.chunk_tiles = g.chunk_tiles;
  p.sc = (float)((double)scale * 1.4426950408889634);
  p.timeout_ns = (uint64_t)g_watchdog_ns;
  const int64_t stats_items = batch * kv_heads * g.groups * g.nchunk;
  const int64_t score_items = batch * kv_heads * ((tokens + 127) / 128);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int dp = padded_dim(channels);
  if (dtype == FE_DTYPE_BF16)
    return dp == 64    ? launch_snap<true, 64>(tq, tk, p, stats_items, score_items, s)
           : dp == 128 ? launch_snap<true, 128>(tq, tk, p, stats_items, score_items, s)
                       : launch_snap<true, 256>(tq, tk, p, stats_items, score_items, s);
  return dp == 64    ? launch_snap<false, 64>(tq, tk, p, stats_items, score_items, s)
         : dp == 128 ? launch_snap<false, 128>(tq, tk, p, stats_items, score_items, s)
                     : launch_snap<false, 256>(tq, tk, p, stats_items, score_items, s);
}

int fe_device_status(int device, int clear, int* status_out) {
  g_err[0] = 0;
  int cur = -1;
  cudaGetDevice(&cur);
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  int st = 0;
  e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&st, fe::g_status, sizeof(int));
  if (e == cudaSuccess && clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(fe::g_status, &zero, sizeof(int));
    // The device is idle, so the host word holds its final value: clear it
    // too, so the next call does not report what was just read here.
    int* words = __atomic_load_n(&g_status_words, __ATOMIC_ACQUIRE);
    if (words != nullptr && device >= 0 && device < kMaxDevices) __atomic_store_n(words + device, 0, __ATOMIC_RELEASE);
  }
  if (cur >= 0 && cur != device) cudaSetDevice(cur);
  if (e != cudaSuccess) return cuda_fail(e, "status read");
  if (status_out) *status_out = st;
  return FE_STATUS_OK;
}

int fe_watchdog_selftest(int64_t timeout_ns, void* stream) {
  g_err[0] = 0;
  if (timeout_ns <= 0 || timeout_ns > 10000000000LL) return fail(FE_STATUS_INVALID, "timeout out of range");
  int dev = 0;
  cudaError_t e0 = cudaGetDevice(&dev);
  if (e0 != cudaSuccess) return cuda_fail(e0, "cudaGetDevice");
  int rc = attach_status(dev, stream);
  if (rc) return rc;
  fe_watchdog_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>((uint64_t)timeout_ns);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "watchdog launch");
  return FE_STATUS_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free evict().
//
// Some callers cannot allocate device memory at the point where they run
// eviction: code inside a custom memory pool that owns all of the GPU's
// memory, engines that reserve every byte up front and forbid cudaMalloc on
// the serving path, or plain C/FFI hosts that have no allocator of their own.
// fe_evict needs one piece of scratch besides the caller's inputs and outputs:
// the per-row softmax statistics {m, l} written by the attention kernel and
// read back by the replay kernel.  This variant keeps that scratch in a
// fixed-size array that lives in the library itself.
//
// The array is reserved on every GPU that loads this library and stays there
// until the process exits (32 MiB).
// ---------------------------------------------------------------------------
namespace {

constexpr int64_t kNoAllocMaxRows = int64_t(1) << 22;  // batch*q_heads*tokens rows of {m, l}

static __device__ __align__(256) float2 fe_noalloc_row_stats[kNoAllocMaxRows];

// Device address of fe_noalloc_row_stats on each device, looked up once per
// device and context (a context created anew after cudaDeviceReset has its
// own copy of the array, so the address is looked up again).
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {nullptr};
unsigned long long g_noalloc_ctx[kMaxDevices] = {0};

int noalloc_scratch(int dev, float** out) {
  if (dev < 0 || dev >= kMaxDevices)
    return fail(FE_STATUS_UNSUPPORTED, "fe_evict_noalloc: device index %d out of range", dev);
  const unsigned long long ctx = current_ctx_id();
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr || ctx == 0 || g_noalloc_ctx[dev] != ctx) {
    // The caller's device is current here (bind_device); the symbol's host
    // name is only a stand-in, so ask the runtime for its device address.
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, fe_noalloc_row_stats);
    if (e != cudaSuccess) return cuda_fail(e, "fe_evict_noalloc: cudaGetSymbolAddress");
    g_noalloc_ptr[dev] = p;
    g_noalloc_ctx[dev] = ctx;
  }
  *out = static_cast<float*>(g_noalloc_ptr[dev]);
  return FE_STATUS_OK;
}

// Keeps the entry points called by fe_evict_noalloc from attaching the host
// status word (which allocates pinned host memory) on this thread.
struct NoAttachScope {
  bool prev;
  NoAttachScope() : prev(g_no_attach) { g_no_attach = true; }
  ~NoAttachScope() { g_no_attach = prev; }
};

}  // namespace

extern "C" int fe_evict_noalloc(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                                const void* v, const int64_t* v_strides, void* out, float* importance,
                                int64_t* indices, uint8_t* mask, int64_t batch, int64_t q_heads, int64_t kv_heads,
                                int64_t tokens, int64_t channels, int dtype, int causal, float scale,
                                float recency_decay, int64_t observation_window, int value_weighted, int64_t budget,
                                int64_t recent, int64_t pool_kernel, void* stream) {
  g_err[0] = 0;
  if (batch < 1 || q_heads < 1 || tokens < 1)
    return fail(FE_STATUS_INVALID, "fe_evict_noalloc: empty shape");
  if (batch > kNoAllocMaxRows || q_heads > kNoAllocMaxRows || tokens > kNoAllocMaxRows ||
      batch * q_heads > kNoAllocMaxRows || batch * q_heads * tokens > kNoAllocMaxRows)
    return fail(FE_STATUS_UNSUPPORTED,
                "fe_evict_noalloc: batch*q_heads*tokens = %lld exceeds the built-in scratch capacity of %lld rows; "
                "use fe_evict with a caller-provided workspace",
                (long long)(batch * q_heads * tokens), (long long)kNoAllocMaxRows);
  if (!q) return fail(FE_STATUS_INVALID, "null pointer");
  int dev = 0;
  int rc = bind_device(q, &dev);
  if (rc) return rc;
  float* scratch = nullptr;
  rc = noalloc_scratch(dev, &scratch);
  if (rc) return rc;
  // Every row the replay reads is written by the attention kernel earlier on
  // the same stream (valid statistics, or NaN when that kernel gave up on a
  // wait), so the scratch needs no clearing between calls.  The host status
  // word is used when an earlier call of another entry point attached it;
  // this entry point never attaches it itself (that allocates).
  NoAttachScope no_attach;
  return fe_evict(q, q_strides, k, k_strides, v, v_strides, out, importance, indices, mask, scratch, batch, q_heads,
                  kv_heads, tokens, channels, dtype, causal, scale, recency_decay, observation_window, value_weighted,
                  budget, recent, pool_kernel, stream);
}
