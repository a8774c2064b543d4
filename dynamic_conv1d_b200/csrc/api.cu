// api.cu -- the extern "C" boundary of libdynconv (declared in include/dynconv.h).
//
// Validates shapes, pointers and dtypes, carves the caller's workspace, and
// dispatches to the kernels.  It never allocates device memory and never
// synchronises (except dynconv_check_device, whose job is to synchronise, and the
// one-time set-up of the host-visible error word on a device's first call).
#include <atomic>
#include <mutex>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include "common.cuh"
#include "lowrank_tc.cuh"

namespace dynconv {

namespace {
thread_local char g_last_error[512] = "";
std::atomic<uint64_t> g_launches{0};
}  // namespace

thread_local int t_no_alloc_scope = 0;

NoAllocScope::NoAllocScope() { ++t_no_alloc_scope; }
NoAllocScope::~NoAllocScope() { --t_no_alloc_scope; }

void note_launch(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return DYNCONV_OK;
  return set_error(DYNCONV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int ensure_context() {
  thread_local int bound_device = -1;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  if (dev == bound_device) return DYNCONV_OK;
  e = cudaSetDevice(dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaSetDevice");
  bound_device = dev;
  return DYNCONV_OK;
}

int encode_tensor_map_bf16(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims,
                           const cuuint64_t* strides_bytes, const cuuint32_t* box) {
  int s = ensure_context();
  if (s) return s;
  using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  if (!fn) return set_error(DYNCONV_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)rank, const_cast<void*>(base), dims, strides_bytes,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(DYNCONV_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return DYNCONV_OK;
}

int sm_count() {
  static std::atomic<int> cached[64];  // zero-initialised; 0 = not queried yet
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cached[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

unsigned int lr_tc_error_word();
unsigned int lr_bwd_tm_error_word();
unsigned int hw_tma_error_word();
unsigned int selftest_error_word();
int lr_tc_error_word_wire(unsigned int* host_word);
int lr_bwd_tm_error_word_wire(unsigned int* host_word);
int hw_tma_error_word_wire(unsigned int* host_word);
int selftest_error_word_wire(unsigned int* host_word);
bool hw_tma_supported(int64_t D, int64_t H, int W, int log2hs, int dtype, const void* const* ptrs, int nptrs);
int hw_tma_partial_rows(int64_t B, int64_t T, int64_t D, int log2hs);
int hw_tma_fwd_launch(const void* x, const void* w, const void* sw, void* y, int64_t B, int64_t T, int64_t D, int64_t H,
                      int W, int log2hs, int residual, cudaStream_t st);
int hw_tma_bwd_launch(const void* x, const void* w, const void* sw, const void* dy, void* dx, void* dw, float* part,
                      int64_t B, int64_t T, int64_t D, int64_t H, int W, int log2hs, int residual, cudaStream_t st);
int wait_selftest_launch(uint64_t limit_ns, int* out, cudaStream_t st);

// kernels (other translation units)
int hw_partial_rows(int64_t B, int64_t T, int64_t D, int dtype);
int hw_fwd_launch(const void* x, const void* w, const void* sw, void* y, int64_t B, int64_t T, int64_t D, int64_t H,
                  int W, int log2hs, int dtype, int residual, cudaStream_t st);
int hw_bwd_launch(const void* x, const void* w, const void* sw, const void* dy, void* dx, void* dw, float* part,
                  int64_t B, int64_t T, int64_t D, int64_t H, int W, int log2hs, int dtype, int residual,
                  cudaStream_t st);
int reduce_partials_launch(const float* part, int P, int64_t n, float* out_f32, void* out, int dtype, cudaStream_t st);
int cast_f32_launch(const float* src, void* dst, int64_t n, int dtype, cudaStream_t st);
int64_t lr_simple_partial_rows(int64_t B, int64_t T);
int lr_fwd_simple_launch(const void* x, const void* z, const void* U, const void* sw, void* y, int64_t B, int64_t T,
                         int64_t D, int R, int Rk, int W, int dtype, int residual, cudaStream_t st);
int lr_bwd_simple_launch(const void* x, const void* z, const void* U, const void* sw, const void* dy, void* dx,
                         void* dz, float* part, int64_t B, int64_t T, int64_t D, int R, int Rk, int W, int dtype,
                         int residual, cudaStream_t st);
int umma_selftest_launch(const void* A, const void* B, float* D, int M, int N, int K, int Nb, int a_major, int a_sbo,
                         int a_lbo, int b_major, int b_sbo, int b_lbo, int b_off, int a_off, cudaStream_t st);
bool lr_tc_supported(int64_t D, int Rk, int W, int dtype, const void* const* ptrs, int nptrs, int G);
bool lr_tc_bwd_supported(int64_t D, int Rk, int W, int dtype, const void* const* ptrs, int nptrs, int G);
size_t lr_tc_bwd_workspace(int64_t B, int64_t T, int64_t D, int Rk, int W, int G);
size_t lr_tc_fwd_workspace(int64_t B, int64_t T, int Rk, int G);
int lr_tc_fwd_launch(const void* x, const void* z, const void* U, const void* sw, void* y, void* ws, size_t ws_bytes,
                     int64_t B, int64_t T, int64_t D, int G, int R, int Rk, int W, int residual, cudaStream_t st);
int lr_tc_bwd_launch(const void* x, const void* z, const void* U, const void* sw, const void* dy, void* dx, void* dz,
                     float* dU_f32, void* dU, void* dsw, void* ws, size_t ws_bytes, int64_t B, int64_t T, int64_t D,
                     int G, int R, int Rk, int W, int residual, const void* zp, cudaStream_t st);
int lr_tm_bwd_launch(const void* x, const void* z, const void* U, const void* sw, const void* dy, void* dx, void* dz,
                     float* dU_f32, void* dU, void* dsw, void* ws, size_t ws_bytes, int64_t B, int64_t T, int64_t D,
                     int G, int R, int Rk, int W, int residual, const lrtc::DpPeers* peers, const void* zp,
                     cudaStream_t st);
bool comm_peers(const void* comm, lrtc::DpPeers* out);
int comm_device(const void* comm);

namespace {

constexpr size_t kAlign = 256;
constexpr int kMaxGroups = 16;
size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

int check_dtype(int dtype) {
  if (dtype != DYNCONV_DTYPE_BF16 && dtype != DYNCONV_DTYPE_F32)
    return set_error(DYNCONV_ERR_UNSUPPORTED, "dtype %d (expected bf16=0 or f32=1)", dtype);
  return DYNCONV_OK;
}

int check_common(int64_t B, int64_t T, int64_t D, int64_t W) {
  if (B < 0 || T < 0 || D <= 0) return set_error(DYNCONV_ERR_SHAPE, "bad sizes B=%lld T=%lld D=%lld", (long long)B, (long long)T, (long long)D);
  if (W < 1 || W > 8) return set_error(DYNCONV_ERR_UNSUPPORTED, "W=%lld not supported (1..8)", (long long)W);
  if (T > (int64_t)INT32_MAX / 2 || D > (int64_t)INT32_MAX / 16)
    return set_error(DYNCONV_ERR_SHAPE, "T or D too large");
  return DYNCONV_OK;
}

// ---------------------------------------------------------------- host-visible error word
// A kernel whose bounded wait gives up returns early and leaves its outputs
// incomplete.  Besides the device word that dynconv_check_device reads, it stores the
// wait site into this device's word of a small pinned, mapped host array, so the next
// call of this library on the device sees it without synchronising and returns
// DYNCONV_ERR_TIMEOUT.  The array is allocated, and every module's copy of the pointer
// set, on the device's first kernel-launching call that is not being captured into a
// CUDA graph (it synchronises once); until then only dynconv_check_device reports.

constexpr int kMaxDevices = 64;
std::mutex g_wire_mutex;
std::atomic<unsigned int*> g_host_words{nullptr};  // [kMaxDevices], pinned and mapped
std::atomic<int> g_wired[kMaxDevices];

bool capturing(cudaStream_t st) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess) {
    cudaGetLastError();
    return true;  // unknown: treat as capturing (no synchronous calls)
  }
  return cs != cudaStreamCaptureStatusNone;
}

void wire_host_error_word(cudaStream_t st) {
  if (t_no_alloc_scope) return;  // the no-allocation entry point allocates nothing, not even this
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return;
  if (g_wired[dev].load(std::memory_order_acquire)) return;
  if (capturing(st)) return;
  std::lock_guard<std::mutex> lock(g_wire_mutex);
  if (g_wired[dev].load(std::memory_order_relaxed)) return;
  unsigned int* words = g_host_words.load(std::memory_order_acquire);
  if (!words) {
    void* p = nullptr;
    if (cudaHostAlloc(&p, kMaxDevices * sizeof(unsigned int), cudaHostAllocMapped | cudaHostAllocPortable) !=
        cudaSuccess) {
      cudaGetLastError();
      return;
    }
    memset(p, 0, kMaxDevices * sizeof(unsigned int));
    words = static_cast<unsigned int*>(p);
    g_host_words.store(words, std::memory_order_release);
  }
  void* dp = nullptr;
  if (cudaHostGetDevicePointer(&dp, words, 0) != cudaSuccess || !dp) {
    cudaGetLastError();
    return;
  }
  unsigned int* mine = static_cast<unsigned int*>(dp) + dev;
  if (lr_tc_error_word_wire(mine) || lr_bwd_tm_error_word_wire(mine) || hw_tma_error_word_wire(mine) ||
      selftest_error_word_wire(mine)) {
    cudaGetLastError();
    return;
  }
  g_wired[dev].store(1, std::memory_order_release);
}

// DYNCONV_ERR_TIMEOUT if a kernel launched earlier on the current device gave up a
// wait since the last report (reported once; the device words of the same event are
// read and cleared here too, unless the stream is being captured).
int report_earlier_timeout(cudaStream_t st) {
  unsigned int* words = g_host_words.load(std::memory_order_acquire);
  if (!words) return DYNCONV_OK;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return DYNCONV_OK;
  if (*reinterpret_cast<volatile unsigned int*>(words + dev) == 0) return DYNCONV_OK;
  const unsigned int site = __atomic_exchange_n(words + dev, 0u, __ATOMIC_ACQ_REL);
  if (site == 0) return DYNCONV_OK;
  if (!capturing(st)) {
    (void)lr_tc_error_word();
    (void)lr_bwd_tm_error_word();
    (void)selftest_error_word();
    (void)hw_tma_error_word();
  }
  return set_error(DYNCONV_ERR_TIMEOUT,
                   "a kernel launched earlier on device %d gave up a bounded wait (site %u): the outputs of that "
                   "call are incomplete",
                   dev, site);
}

// First step of every kernel-launching entry point.
int op_entry(cudaStream_t st) {
  wire_host_error_word(st);
  return report_earlier_timeout(st);
}

int log2_exact(int64_t v) {
  int l = 0;
  while ((int64_t(1) << l) < v) ++l;
  return (int64_t(1) << l) == v ? l : -1;
}

}  // namespace
}  // namespace dynconv

using namespace dynconv;

extern "C" {

int dynconv_abi_version(void) { return DYNCONV_ABI_VERSION; }

const char* dynconv_status_string(int status) {
  switch (status) {
    case DYNCONV_OK: return "ok";
    case DYNCONV_ERR_SHAPE: return "bad shape";
    case DYNCONV_ERR_ALIGN: return "misaligned pointer";
    case DYNCONV_ERR_UNSUPPORTED: return "unsupported configuration";
    case DYNCONV_ERR_CUDA: return "CUDA error";
    case DYNCONV_ERR_TIMEOUT: return "device-side wait timed out";
    case DYNCONV_ERR_WORKSPACE: return "workspace missing or too small";
    case DYNCONV_ERR_ARGUMENT: return "null tensor argument";
    default: return "unknown status";
  }
}

const char* dynconv_last_error(void) { return g_last_error; }

uint64_t dynconv_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int dynconv_check_device(void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_status(e, "cudaStreamSynchronize");
  // the host-visible word holds the same events: cleared here, so the next call does
  // not report them again
  if (unsigned int* words = g_host_words.load(std::memory_order_acquire)) {
    int dev = -1;
    if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kMaxDevices)
      __atomic_exchange_n(words + dev, 0u, __ATOMIC_ACQ_REL);
  }
  // every word is read (and so cleared) before the first non-zero one is reported
  const unsigned int words[4] = {lr_tc_error_word(), lr_bwd_tm_error_word(), selftest_error_word(),
                                 hw_tma_error_word()};
  static const char* const kFile[4] = {"lowrank forward", "lowrank backward", "self-test", "headwise"};
  for (unsigned int v : words)
    if (v == 0xFFFFFFFFu) return set_error(DYNCONV_ERR_CUDA, "could not read the device error word");
  for (int i = 0; i < 4; ++i)
    if (words[i] != 0)
      return set_error(DYNCONV_ERR_TIMEOUT, "a device-side bounded wait gave up (%s kernel, site %u)", kFile[i],
                       words[i]);
  return DYNCONV_OK;
}

int dynconv_hw_fwd(const void* x, const void* weight, const void* static_w, void* y, int64_t B, int64_t T, int64_t D,
                   int64_t H, int64_t W, int dtype, int residual, void* stream) {
  int s;
  if ((s = op_entry((cudaStream_t)stream))) return s;
  if ((s = check_dtype(dtype))) return s;
  if ((s = check_common(B, T, D, W))) return s;
  if (H <= 0 || D % H != 0) return set_error(DYNCONV_ERR_SHAPE, "D=%lld must be divisible by H=%lld", (long long)D, (long long)H);
  const int l2 = log2_exact(D / H);
  if (l2 < 0) return set_error(DYNCONV_ERR_UNSUPPORTED, "head_size %lld is not a power of two", (long long)(D / H));
  if (B * T == 0) return DYNCONV_OK;
  if (!x || !weight || !y) return set_error(DYNCONV_ERR_ARGUMENT, "hw_fwd: null x/weight/y");
  const void* ptrs[] = {x, weight, static_w, y};
  if (hw_tma_supported(D, H, (int)W, l2, dtype, ptrs, 4))
    return hw_tma_fwd_launch(x, weight, static_w, y, B, T, D, H, (int)W, l2, residual, (cudaStream_t)stream);
  return hw_fwd_launch(x, weight, static_w, y, B, T, D, H, (int)W, l2, dtype, residual, (cudaStream_t)stream);
}

size_t dynconv_hw_bwd_workspace_bytes(int64_t B, int64_t T, int64_t D, int64_t H, int64_t W, int dtype,
                                      int has_static) {
  if (!has_static || B * T == 0) return 0;
  // Sized for either path (pointer alignment can only move a call to the
  // register-ring kernels, and both fit the larger of the two).
  int64_t rows = hw_partial_rows(B, T, D, dtype);
  const int l2 = (H > 0 && D % H == 0) ? log2_exact(D / H) : -1;
  if (l2 >= 0 && hw_tma_supported(D, H, (int)W, l2, dtype, nullptr, 0)) {
    const int64_t r2 = hw_tma_partial_rows(B, T, D, l2);
    if (r2 > rows) rows = r2;
  }
  return align_up((size_t)rows * (size_t)W * (size_t)D * sizeof(float));
}

int dynconv_hw_bwd(const void* x, const void* weight, const void* static_w, const void* dy, void* dx, void* dweight,
                   void* dstatic_w, float* dstatic_w_f32, void* workspace, size_t workspace_bytes, int64_t B,
                   int64_t T, int64_t D, int64_t H, int64_t W, int dtype, int residual, void* stream) {
  int s;
  if ((s = op_entry((cudaStream_t)stream))) return s;
  if ((s = check_dtype(dtype))) return s;
  if ((s = check_common(B, T, D, W))) return s;
  if (H <= 0 || D % H != 0) return set_error(DYNCONV_ERR_SHAPE, "D=%lld must be divisible by H=%lld", (long long)D, (long long)H);
  const int l2 = log2_exact(D / H);
  if (l2 < 0) return set_error(DYNCONV_ERR_UNSUPPORTED, "head_size %lld is not a power of two", (long long)(D / H));
  cudaStream_t st = (cudaStream_t)stream;
  const bool has_static = static_w != nullptr;
  if (has_static && !dstatic_w_f32) return set_error(DYNCONV_ERR_ARGUMENT, "hw_bwd: dstatic_w_f32 required with static_w");
  if (B * T == 0) {
    if (has_static) {
      if (cudaMemsetAsync(dstatic_w_f32, 0, (size_t)W * D * sizeof(float), st) != cudaSuccess)
        return set_error(DYNCONV_ERR_CUDA, "memset");
      if (dstatic_w) return cast_f32_launch(dstatic_w_f32, dstatic_w, W * D, dtype, st);
    }
    return DYNCONV_OK;
  }
  if (!x || !weight || !dy || !dx || !dweight) return set_error(DYNCONV_ERR_ARGUMENT, "hw_bwd: null tensor");
  float* part = nullptr;
  if (has_static) {
    const size_t need = dynconv_hw_bwd_workspace_bytes(B, T, D, H, W, dtype, 1);
    if (!workspace || workspace_bytes < need)
      return set_error(DYNCONV_ERR_WORKSPACE, "hw_bwd: workspace %zu < %zu bytes", workspace_bytes, need);
    part = (float*)workspace;
  }
  const void* ptrs[] = {x, weight, static_w, dy, dx, dweight};
  if (hw_tma_supported(D, H, (int)W, l2, dtype, ptrs, 6)) {
    if ((s = hw_tma_bwd_launch(x, weight, static_w, dy, dx, dweight, part, B, T, D, H, (int)W, l2, residual, st)))
      return s;
    if (has_static)
      return reduce_partials_launch(part, hw_tma_partial_rows(B, T, D, l2), W * D, dstatic_w_f32, dstatic_w, dtype,
                                    st);
    return DYNCONV_OK;
  }
  if ((s = hw_bwd_launch(x, weight, static_w, dy, dx, dweight, part, B, T, D, H, (int)W, l2, dtype, residual, st)))
    return s;
  if (has_static)
    return reduce_partials_launch(part, hw_partial_rows(B, T, D, dtype), W * D, dstatic_w_f32, dstatic_w, dtype, st);
  return DYNCONV_OK;
}

static int lr_checks(int64_t B, int64_t T, int64_t D, int64_t R, int64_t W, int dtype) {
  int s;
  if ((s = check_dtype(dtype))) return s;
  if ((s = check_common(B, T, D, W))) return s;
  if (R < 1 || R > 64) return set_error(DYNCONV_ERR_UNSUPPORTED, "R=%lld not supported (1..64)", (long long)R);
  return DYNCONV_OK;
}

static int check_groups(int64_t G) {
  if (G < 1 || G > kMaxGroups)
    return set_error(DYNCONV_ERR_SHAPE, "G=%lld channel groups outside 1..%d", (long long)G, kMaxGroups);
  return DYNCONV_OK;
}

size_t dynconv_lr_fwd_grouped_workspace_bytes(int64_t B, int64_t T, int64_t D, int64_t R, int64_t W, int64_t G,
                                              int dtype, int has_static) {
  const int Rk = (int)R + (has_static ? 1 : 0);
  if (B * T == 0 || G < 1 || G > kMaxGroups || !lr_tc_supported(D, Rk, (int)W, dtype, nullptr, 0, (int)G)) return 0;
  return lr_tc_fwd_workspace(B, T, Rk, (int)G);
}

size_t dynconv_lr_fwd_workspace_bytes(int64_t B, int64_t T, int64_t D, int64_t R, int64_t W, int dtype,
                                      int has_static) {
  return dynconv_lr_fwd_grouped_workspace_bytes(B, T, D, R, W, 1, dtype, has_static);
}

int dynconv_lr_fwd_grouped(const void* x, const void* z, const void* U, const void* static_w, void* y,
                           void* workspace, size_t workspace_bytes, int64_t B, int64_t T, int64_t D, int64_t R,
                           int64_t W, int64_t G, int dtype, int residual, void* stream) {
  int s;
  if ((s = op_entry((cudaStream_t)stream))) return s;
  if ((s = lr_checks(B, T, D, R, W, dtype))) return s;
  if ((s = check_groups(G))) return s;
  const int Rk = (int)R + (static_w ? 1 : 0);
  if (Rk > 64) return set_error(DYNCONV_ERR_UNSUPPORTED, "R_kernel=%d > 64", Rk);
  if (B * T == 0) return DYNCONV_OK;
  if (!x || !z || !U || !y) return set_error(DYNCONV_ERR_ARGUMENT, "lr_fwd: null tensor");
  cudaStream_t st = (cudaStream_t)stream;
  const void* ptrs[] = {x, z, U, static_w, y, workspace};
  if (lr_tc_supported(D, Rk, (int)W, dtype, ptrs, 6, (int)G)) {
    const size_t need = lr_tc_fwd_workspace(B, T, Rk, (int)G);
    if (!workspace || workspace_bytes < need)
      return set_error(DYNCONV_ERR_WORKSPACE, "lr_fwd: workspace %zu < %zu bytes", workspace_bytes, need);
    return lr_tc_fwd_launch(x, z, U, static_w, y, workspace, workspace_bytes, B, T, D, (int)G, (int)R, Rk, (int)W,
                            residual, st);
  }
  if (G > 1)
    return set_error(DYNCONV_ERR_UNSUPPORTED,
                     "lr_fwd_grouped: G=%lld groups need the tensor-core path (bf16, W <= 4, R_kernel <= 64, "
                     "D %% 128 == 0, 16-byte aligned tensors); call dynconv_lr_fwd per group",
                     (long long)G);
  return lr_fwd_simple_launch(x, z, U, static_w, y, B, T, D, (int)R, Rk, (int)W, dtype, residual, st);
}

int dynconv_lr_fwd(const void* x, const void* z, const void* U, const void* static_w, void* y, void* workspace,
                   size_t workspace_bytes, int64_t B, int64_t T, int64_t D, int64_t R, int64_t W, int dtype,
                   int residual, void* stream) {
  return dynconv_lr_fwd_grouped(x, z, U, static_w, y, workspace, workspace_bytes, B, T, D, R, W, 1, dtype, residual,
                                stream);
}

size_t dynconv_lr_bwd_grouped_workspace_bytes(int64_t B, int64_t T, int64_t D, int64_t R, int64_t W, int64_t G,
                                              int dtype, int has_static) {
  const int Rk = (int)R + (has_static ? 1 : 0);
  if (B * T == 0 || G < 1 || G > kMaxGroups) return 0;
  size_t tc = 0;
  if (lr_tc_bwd_supported(D, Rk, (int)W, dtype, nullptr, 0, (int)G)) tc = lr_tc_bwd_workspace(B, T, D, Rk, (int)W, (int)G);
  if (G > 1) return tc;
  // Sized for whichever path dynconv_lr_bwd will take (pointer alignment aside,
  // which only ever moves a call onto the simple path; both fit the max).
  const size_t simple = align_up((size_t)lr_simple_partial_rows(B, T) * (size_t)Rk * (size_t)W * (size_t)D * sizeof(float));
  return simple > tc ? simple : tc;
}

size_t dynconv_lr_bwd_workspace_bytes(int64_t B, int64_t T, int64_t D, int64_t R, int64_t W, int dtype,
                                      int has_static) {
  return dynconv_lr_bwd_grouped_workspace_bytes(B, T, D, R, W, 1, dtype, has_static);
}

// dU_f32 [G][Rk][W*D] -> dU [G][R][W*D] and dstatic_w [G][W][D] (either may be null).
static int cast_grouped(const float* dU_f32, void* dU, void* dsw, int64_t G, int64_t R, int Rk, int64_t W, int64_t D,
                        int dtype, cudaStream_t st) {
  int s;
  const int64_t wd = W * D;
  const size_t esz = dtype == DYNCONV_DTYPE_BF16 ? 2 : 4;
  for (int64_t g = 0; g < G; ++g) {
    const float* src = dU_f32 + g * Rk * wd;
    if (dU && (s = cast_f32_launch(src, (char*)dU + (size_t)(g * R * wd) * esz, R * wd, dtype, st))) return s;
    if (Rk > R && dsw && (s = cast_f32_launch(src + R * wd, (char*)dsw + (size_t)(g * wd) * esz, wd, dtype, st)))
      return s;
  }
  return DYNCONV_OK;
}

int dynconv_lr_bwd_grouped(const void* x, const void* z, const void* U, const void* static_w, const void* dy,
                           void* dx, void* dz, void* dU, void* dstatic_w, float* dU_f32, void* workspace,
                           size_t workspace_bytes, int64_t B, int64_t T, int64_t D, int64_t R, int64_t W, int64_t G,
                           int dtype, int residual, const void* z_packed, void* stream) {
  int s;
  if ((s = op_entry((cudaStream_t)stream))) return s;
  if ((s = lr_checks(B, T, D, R, W, dtype))) return s;
  if ((s = check_groups(G))) return s;
  const bool has_static = static_w != nullptr;
  const int Rk = (int)R + (has_static ? 1 : 0);
  if (Rk > 64) return set_error(DYNCONV_ERR_UNSUPPORTED, "R_kernel=%d > 64", Rk);
  if (!dU_f32) return set_error(DYNCONV_ERR_ARGUMENT, "lr_bwd: dU_f32 required");
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t nacc = G * Rk * W * D;
  if (B * T == 0) {
    if (cudaMemsetAsync(dU_f32, 0, (size_t)nacc * sizeof(float), st) != cudaSuccess)
      return set_error(DYNCONV_ERR_CUDA, "memset");
    return cast_grouped(dU_f32, dU, has_static ? dstatic_w : nullptr, G, R, Rk, W, D, dtype, st);
  }
  if (!x || !z || !U || !dy || !dx || !dz) return set_error(DYNCONV_ERR_ARGUMENT, "lr_bwd: null tensor");
  const void* ptrs[] = {x, z, U, static_w, dy, dx, dz, z_packed};
  const bool tc = lr_tc_bwd_supported(D, Rk, (int)W, dtype, ptrs, 8, (int)G);
  if (!tc && G > 1)
    return set_error(DYNCONV_ERR_UNSUPPORTED,
                     "lr_bwd_grouped: G=%lld groups need the tensor-core path (bf16, W <= 4, R_kernel <= 32, "
                     "D %% 128 == 0, G*D/128 <= SM count, 16-byte aligned tensors); call dynconv_lr_bwd per group",
                     (long long)G);
  const size_t need = dynconv_lr_bwd_grouped_workspace_bytes(B, T, D, R, W, G, dtype, has_static);
  if (!workspace || workspace_bytes < need)
    return set_error(DYNCONV_ERR_WORKSPACE, "lr_bwd: workspace %zu < %zu bytes", workspace_bytes, need);
  if (tc)
    return lr_tc_bwd_launch(x, z, U, static_w, dy, dx, dz, dU_f32, dU, dstatic_w, workspace, workspace_bytes, B, T, D,
                            (int)G, (int)R, Rk, (int)W, residual, z_packed, st);
  float* part = (float*)workspace;
  if ((s = lr_bwd_simple_launch(x, z, U, static_w, dy, dx, dz, part, B, T, D, (int)R, Rk, (int)W, dtype, residual, st)))
    return s;
  const int P = (int)lr_simple_partial_rows(B, T);
  if ((s = reduce_partials_launch(part, P, nacc, dU_f32, nullptr, dtype, st))) return s;
  return cast_grouped(dU_f32, dU, has_static ? dstatic_w : nullptr, 1, R, Rk, W, D, dtype, st);
}

int dynconv_lr_bwd_grouped_dp(const void* x, const void* z, const void* U, const void* static_w, const void* dy,
                              void* dx, void* dz, void* dU, void* dstatic_w, float* dU_f32, void* workspace,
                              size_t workspace_bytes, int64_t B, int64_t T, int64_t D, int64_t R, int64_t W, int64_t G,
                              int dtype, int residual, const void* z_packed, void* comm, void* stream) {
  int s;
  if ((s = op_entry((cudaStream_t)stream))) return s;
  if ((s = lr_checks(B, T, D, R, W, dtype))) return s;
  if ((s = check_groups(G))) return s;
  const bool has_static = static_w != nullptr;
  const int Rk = (int)R + (has_static ? 1 : 0);
  if (!dU_f32) return set_error(DYNCONV_ERR_ARGUMENT, "lr_bwd_dp: dU_f32 required");
  if (!x || !z || !U || !dy || !dx || !dz) return set_error(DYNCONV_ERR_ARGUMENT, "lr_bwd_dp: null tensor");
  lrtc::DpPeers peers;
  if (!comm_peers(comm, &peers)) return set_error(DYNCONV_ERR_ARGUMENT, "lr_bwd_dp: communicator missing or not connected");
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != comm_device(comm))
    return set_error(DYNCONV_ERR_ARGUMENT, "lr_bwd_dp: the communicator belongs to device %d, current is %d",
                     comm_device(comm), dev);
  const void* ptrs[] = {x, z, U, static_w, dy, dx, dz, z_packed};
  if (B * T == 0 || !lr_tc_bwd_supported(D, Rk, (int)W, dtype, ptrs, 8, (int)G))
    return set_error(DYNCONV_ERR_UNSUPPORTED,
                     "lr_bwd_dp: the fused data-parallel backward needs the tensor-core path (bf16, W <= 4, "
                     "R_kernel <= 32, B*T > 0, 16-byte aligned tensors); all-reduce dU_f32 of dynconv_lr_bwd_grouped "
                     "instead");
  const size_t need = dynconv_lr_bwd_grouped_workspace_bytes(B, T, D, R, W, G, dtype, has_static);
  if (!workspace || workspace_bytes < need)
    return set_error(DYNCONV_ERR_WORKSPACE, "lr_bwd_dp: workspace %zu < %zu bytes", workspace_bytes, need);
  return lr_tm_bwd_launch(x, z, U, static_w, dy, dx, dz, dU_f32, dU, dstatic_w, workspace, workspace_bytes, B, T, D,
                          (int)G, (int)R, Rk, (int)W, residual, &peers, z_packed, (cudaStream_t)stream);
}

int dynconv_lr_bwd(const void* x, const void* z, const void* U, const void* static_w, const void* dy, void* dx,
                   void* dz, void* dU, void* dstatic_w, float* dU_f32, void* workspace, size_t workspace_bytes,
                   int64_t B, int64_t T, int64_t D, int64_t R, int64_t W, int dtype, int residual, void* stream) {
  return dynconv_lr_bwd_grouped(x, z, U, static_w, dy, dx, dz, dU, dstatic_w, dU_f32, workspace, workspace_bytes, B,
                                T, D, R, W, 1, dtype, residual, nullptr, stream);
}

int dynconv_cast_f32(const float* src, void* dst, int64_t n, int dtype, void* stream) {
  int s;
  if ((s = op_entry((cudaStream_t)stream))) return s;
  if ((s = check_dtype(dtype))) return s;
  if (n < 0) return set_error(DYNCONV_ERR_SHAPE, "n < 0");
  if (n > 0 && (!src || !dst)) return set_error(DYNCONV_ERR_ARGUMENT, "cast: null pointer");
  return cast_f32_launch(src, dst, n, dtype, (cudaStream_t)stream);
}

int dynconv_umma_selftest(const void* A, const void* B, float* D, int M, int N, int K, int Nb, int a_major, int a_sbo,
                          int a_lbo, int b_major, int b_sbo, int b_lbo, int b_row_offset, int a_row_offset,
                          void* stream) {
  if (!A || !B || !D) return set_error(DYNCONV_ERR_ARGUMENT, "selftest: null pointer");
  return umma_selftest_launch(A, B, D, M, N, K, Nb, a_major, a_sbo, a_lbo, b_major, b_sbo, b_lbo, b_row_offset,
                              a_row_offset, (cudaStream_t)stream);
}

int dynconv_wait_selftest(uint64_t limit_ns, int* out, void* stream) {
  if (limit_ns == 0 || limit_ns > 100000000ull)
    return set_error(DYNCONV_ERR_ARGUMENT, "wait_selftest: limit %llu ns outside 1 ns .. 100 ms",
                     (unsigned long long)limit_ns);
  wire_host_error_word((cudaStream_t)stream);
  return wait_selftest_launch(limit_ns, out, (cudaStream_t)stream);
}

}  // extern "C"
