// dynconv_lr_fwd_noalloc: the low-rank forward with its scratch in a fixed
// device array of this library instead of a caller-provided workspace.
//
// Who needs it: callers that cannot allocate device memory at the point of the
// call -- a host-language binding (cgo, JNI, a plain C program) that has no
// access to PyTorch's caching allocator and must not call cudaMalloc on its hot
// path (cudaMalloc/cudaFree synchronise the device), or a serving process that
// reserves all its memory at start-up and forbids allocations afterwards.
//
// The scratch is the packed-z buffer of the bf16 tensor-core path
// ([R_kernel/8][B][T][8] bf16, 256-byte rounded; see z_pack_kernel in
// lowrank_tc.cu).  It lives in one static __device__ array per device and is
// found once per device with cudaGetSymbolAddress; the call then goes through
// dynconv_lr_fwd unchanged, so results are those of dynconv_lr_fwd.  Nothing in
// the scratch has to start at zero: z_pack_kernel writes every byte the forward
// kernel later reads (padding ranks included) before that kernel runs.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/dynconv.h"
#include "common.cuh"

namespace {

constexpr size_t kScratchBytes = DYNCONV_LR_FWD_NOALLOC_SCRATCH_BYTES;
static_assert(kScratchBytes % 256 == 0, "scratch size must keep 256-byte granularity");

__device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Address of this device's scratch array.  The first call per device does the
// set-up (it also makes the runtime load this module on that device); later
// calls only read the cached pointer.  Keyed by device ordinal: the library runs
// in each device's primary context only (ensure_context binds it), so one
// module instance -- one scratch address -- exists per device.
int scratch_for_current_device(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return dynconv::cuda_status(e, "lr_fwd_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return dynconv::set_error(DYNCONV_ERR_UNSUPPORTED, "lr_fwd_noalloc: device ordinal %d >= %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return dynconv::cuda_status(e, "lr_fwd_noalloc: cudaGetSymbolAddress");
    if (!p) return dynconv::set_error(DYNCONV_ERR_CUDA, "lr_fwd_noalloc: cudaGetSymbolAddress returned NULL");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return DYNCONV_OK;
}

}  // namespace

extern "C" int dynconv_lr_fwd_noalloc(const void* x, const void* z, const void* U, const void* static_w, void* y,
                                      int64_t B, int64_t T, int64_t D, int64_t R, int64_t W, int dtype, int residual,
                                      void* stream) {
  // Size check first: it needs neither the device nor the tensors.
  const size_t need = dynconv_lr_fwd_workspace_bytes(B, T, D, R, W, dtype, static_w != nullptr);
  if (need > kScratchBytes)
    return dynconv::set_error(DYNCONV_ERR_WORKSPACE,
                              "lr_fwd_noalloc: B=%lld T=%lld R=%lld needs %zu scratch bytes, above the fixed %zu; "
                              "use dynconv_lr_fwd with a caller workspace",
                              (long long)B, (long long)T, (long long)R, need, kScratchBytes);
  void* scratch = nullptr;
  int s = scratch_for_current_device(&scratch);
  if (s) return s;
  const dynconv::NoAllocScope no_alloc;  // no pinned error-word array either
  return dynconv_lr_fwd(x, z, U, static_w, y, scratch, kScratchBytes, B, T, D, R, W, dtype, residual, stream);
}
