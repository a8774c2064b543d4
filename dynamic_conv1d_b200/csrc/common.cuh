// common.cuh -- shared device/host helpers of libdynconv (sm_100a only).
//
// * element access for bf16 / fp32 tensors (16-byte vector loads, RNE stores)
// * the device error word that bounded waits set when they give up
// * thin inline-PTX wrappers for mbarrier, TMA (cp.async.bulk.tensor) and the
//   5th-generation tensor core (tcgen05: TMEM alloc, mma, commit, ld)
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/dynconv.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ != 1000)
#error "libdynconv is written for sm_100a (B200) only"
#endif

namespace dynconv {

// ----------------------------------------------------------------- host side

// Records `msg` as the calling thread's last error and returns `status`.
int set_error(int status, const char* fmt, ...);
// While one exists on the calling thread, the library allocates nothing of its own
// (the no-allocation entry point holds one around its call).
struct NoAllocScope {
  NoAllocScope();
  ~NoAllocScope();
  NoAllocScope(const NoAllocScope&) = delete;
  NoAllocScope& operator=(const NoAllocScope&) = delete;
};
// Wraps a CUDA runtime status: DYNCONV_OK or DYNCONV_ERR_CUDA with the CUDA message.
int cuda_status(cudaError_t e, const char* what);
// Number of SMs of the current device (cached per device).
int sm_count();

// Makes the current device's primary context current on the calling thread
// (cudaSetDevice does so since CUDA 12), once per thread and device.  Driver-API
// calls such as cuTensorMapEncodeTiled need a current context, and a thread that
// has made no runtime call yet -- autograd's backward worker, say -- has none.
int ensure_context();

// Encodes a tiled, no-swizzle, zero-fill bf16 TMA descriptor (cuTensorMapEncodeTiled,
// reached through the runtime's driver entry point).  `strides_bytes` has rank-1
// entries (dimension 0 is dense).  DYNCONV_OK or DYNCONV_ERR_CUDA.
int encode_tensor_map_bf16(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims,
                           const cuuint64_t* strides_bytes, const cuuint32_t* box);

// Counts kernel launches (dynconv_launch_count) -- call once per launch.
void note_launch(int n = 1);

#define DYNCONV_CHECK_LAUNCH(what)                                  \
  do {                                                              \
    cudaError_t e__ = cudaGetLastError();                           \
    if (e__ != cudaSuccess) return ::dynconv::cuda_status(e__, what); \
    ::dynconv::note_launch();                                       \
  } while (0)

// --------------------------------------------------------------- device side

// Set to a nonzero site code by a bounded wait that gave up.  Without relocatable
// device code a __device__ variable cannot be shared between translation units,
// so every .cu file that waits on mbarriers gets its own copy (internal linkage)
// and exports a host accessor with DYNCONV_DEFINE_ERROR_ACCESSOR, which
// dynconv_check_device() polls.
static __device__ unsigned int g_device_error;

// Host-visible copy of the error word: this device's word in pinned, mapped host
// memory, which the host reads at the next library call without synchronising (the
// call then reports DYNCONV_ERR_TIMEOUT).  The host wires it once per device (the
// accessor's _wire function); until then it is null and only g_device_error is set.
static __device__ unsigned int* g_host_error;

// Records that a bounded wait gave up at `site`: the device word (first site wins)
// and, once wired, the host-visible word (a plain store over the bus, then a system
// fence; any nonzero site will do, so racing writers need no atomics).
__device__ __forceinline__ void record_device_error(unsigned int site) {
  atomicCAS(&g_device_error, 0u, site);
  unsigned int* h = g_host_error;
  if (h) {
    *reinterpret_cast<volatile unsigned int*>(h) = site;
    __threadfence_system();
  }
}

#define DYNCONV_DEFINE_ERROR_ACCESSOR(fn)                                      \
  unsigned int fn() {                                                          \
    unsigned int v = 0;                                                        \
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess)    \
      return 0xFFFFFFFFu;                                                      \
    if (v != 0) {                                                              \
      const unsigned int z = 0;                                                \
      cudaMemcpyToSymbol(g_device_error, &z, sizeof(z));                       \
    }                                                                          \
    return v;                                                                  \
  }                                                                            \
  int fn##_wire(unsigned int* host_word) {                                     \
    return cudaMemcpyToSymbol(g_host_error, &host_word, sizeof(host_word)) ==  \
                   cudaSuccess                                                 \
               ? 0                                                             \
               : -1;                                                           \
  }

enum DeviceErrorSite : unsigned int {
  kErrNone = 0,
  kErrWaitProducer = 1,
  kErrWaitMma = 2,
  kErrWaitEpilogue = 3,
  kErrWaitTail = 4,
};

template <typename T>
struct Elem;

template <>
struct Elem<__nv_bfloat16> {
  static constexpr int kVec = 8;  // elements per 16-byte vector
  __device__ __forceinline__ static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

template <>
struct Elem<float> {
  static constexpr int kVec = 4;
  __device__ __forceinline__ static float to_f(float v) { return v; }
  __device__ __forceinline__ static float from_f(float v) { return v; }
};

// Loads N consecutive elements starting at p into float registers.  When the
// span is 16-byte aligned (checked at run time; uniform across a warp in all
// call sites) it is read as 16-byte vectors, otherwise element by element.
template <typename T, int N>
__device__ __forceinline__ void load_span(const T* __restrict__ p, float (&out)[N]) {
  constexpr int kBytes = N * (int)sizeof(T);
  if (kBytes % 16 == 0 && ((reinterpret_cast<uintptr_t>(p) & 15) == 0)) {
    constexpr int kV = 16 / (int)sizeof(T);
#pragma unroll
    for (int i = 0; i < N; i += kV) {
      uint4 u = __ldg(reinterpret_cast<const uint4*>(p + i));
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < kV; ++j) out[i + j] = Elem<T>::to_f(e[j]);
    }
  } else if (kBytes % 8 == 0 && ((reinterpret_cast<uintptr_t>(p) & 7) == 0)) {
    constexpr int kV = 8 / (int)sizeof(T);
#pragma unroll
    for (int i = 0; i < N; i += kV) {
      uint2 u = __ldg(reinterpret_cast<const uint2*>(p + i));
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < kV; ++j) out[i + j] = Elem<T>::to_f(e[j]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = Elem<T>::to_f(p[i]);
  }
}

template <typename T, int N>
__device__ __forceinline__ void store_span(T* __restrict__ p, const float (&v)[N]) {
  constexpr int kBytes = N * (int)sizeof(T);
  if (kBytes % 16 == 0 && ((reinterpret_cast<uintptr_t>(p) & 15) == 0)) {
    constexpr int kV = 16 / (int)sizeof(T);
#pragma unroll
    for (int i = 0; i < N; i += kV) {
      uint4 u;
      T* e = reinterpret_cast<T*>(&u);
#pragma unroll
      for (int j = 0; j < kV; ++j) e[j] = Elem<T>::from_f(v[i + j]);
      *reinterpret_cast<uint4*>(p + i) = u;
    }
  } else if (kBytes % 8 == 0 && ((reinterpret_cast<uintptr_t>(p) & 7) == 0)) {
    constexpr int kV = 8 / (int)sizeof(T);
#pragma unroll
    for (int i = 0; i < N; i += kV) {
      uint2 u;
      T* e = reinterpret_cast<T*>(&u);
#pragma unroll
      for (int j = 0; j < kV; ++j) e[j] = Elem<T>::from_f(v[i + j]);
      *reinterpret_cast<uint2*>(p + i) = u;
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) p[i] = Elem<T>::from_f(v[i]);
  }
}

// ------------------------------------------------------------ PTX wrappers

// Packed fp32 pair arithmetic (sm_100 f32x2 instructions, round to nearest even).
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}


__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Rounds a dynamic shared-memory base up to 1024 bytes.  The offset is added to
// the __shared__ pointer itself (no integer round trip), so the compiler keeps
// the shared address space and emits LDS/STS rather than generic loads/stores.
__device__ __forceinline__ uint8_t* align_smem_1024(uint8_t* base) {
  const uint32_t a = smem_u32(base);
  return base + ((1024u - (a & 1023u)) & 1023u);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Arrives `count` times at once (count >= 1).
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// As mbar_try_wait, but the thread may be suspended for up to `suspend_ns` while
// the phase is incomplete (it resumes as soon as the phase completes), so a waiting
// warp does not spend issue slots spinning.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity, uint32_t suspend_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(suspend_ns)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Upper bound on the wall time one mbarrier phase may take (every phase in these
// kernels completes in micro- to milliseconds).  A wait that runs out records
// `site` in g_device_error, raises the CTA's abort flag and returns false, so the
// kernel unwinds instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 1500000000ull;  // 1.5 s
constexpr uint32_t kWaitSuspendNs = 1000000u;       // longest single suspension, 1 ms

// Slow path of mbar_wait, kept out of line so that the many wait sites of a
// warp-specialised kernel stay small in the instruction cache.
static __device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, unsigned int site,
                                                   volatile int* abort_flag, uint64_t limit_ns = kWaitLimitNs) {
  if (*abort_flag) return false;
  const uint64_t t0 = globaltimer_ns();
  const uint32_t suspend = limit_ns < kWaitSuspendNs ? (uint32_t)limit_ns : kWaitSuspendNs;
  for (;;) {
    if (mbar_try_wait_suspend(bar, parity, suspend)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > limit_ns) break;
  }
  record_device_error(site);
  *abort_flag = 1;
  return false;
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int site,
                                          volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;  // fast path: phase complete (the try may suspend briefly)
  return mbar_wait_slow(bar, parity, site, abort_flag);
}

// TMA tiled 3-D load into shared memory, completion counted on `bar`.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                            int c1, int c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
      : "memory");
}

// TMA tiled 4-D load into shared memory, completion counted on `bar`.
__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "l"(policy)
      : "memory");
}

// TMA tiled 3-D store from shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* smem_src, int c0, int c1,
                                             int c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group.L2::cache_hint [%0, {%2, %3, %4}], [%1], %5;" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
      : "memory");
}

// Untiled bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(gmem_src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Named barrier over `count` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ------------------------------------------------------------------ tcgen05

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]; kind::f16 (bf16 inputs, fp32 accumulate).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]; kind::f16.  A is K-major in TMEM: lane m
// holds row m, column c packs elements (2c, 2c+1) of that row (low half first).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// As umma_f16 / umma_f16_ts with a compile-time accumulate flag (no predicate
// computation between back-to-back MMAs of an issuing thread).
template <int ACC>
__device__ __forceinline__ void umma_f16_c(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "n"(ACC)
      : "memory");
}

template <int ACC>
__device__ __forceinline__ void umma_f16_ts_c(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "n"(ACC)
      : "memory");
}

// 32 lanes x 8 consecutive 32-bit columns from registers; lane i of the warp writes row (base lane + i).
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

__device__ __forceinline__ void tmem_st4(uint32_t taddr, const uint32_t (&v)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(v[0]), "r"(v[1]),
               "r"(v[2]), "r"(v[3])
               : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Arrives once on `bar` when every previously issued tcgen05.mma of this thread completes.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns; lane i of the warp gets row (base lane + i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 8 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 4 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, float (&v)[4]) {
  uint32_t r[4];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor, SWIZZLE_NONE ("interleaved") canonical layout.
// lbo: byte stride between 8-element core-matrix groups along K;
// sbo: byte stride between core-matrix groups along M/N.  Both K-major and
// MN-major operands use this pairing in the no-swizzle mode.
__device__ __forceinline__ uint64_t make_smem_desc(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  // base offset 0, lbo mode 0, layout type 0 (SWIZZLE_NONE)
  return d;
}

// Shared-memory matrix descriptor, 128-byte swizzle (the layout a TMA load with
// CU_TENSOR_MAP_SWIZZLE_128B writes: 16-byte chunk c of 128-byte row r sits at
// chunk c ^ (r % 8); the pattern repeats every 1024 bytes, so the start address
// must be 1024-aligned).  MN-major operand: lbo = byte stride between 64-element
// atoms along M/N, sbo = byte stride between groups of 8 rows along K.
__device__ __forceinline__ uint64_t make_smem_desc_sw128(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = make_smem_desc(smem_addr, lbo, sbo);
  d |= (uint64_t)2 << 61;  // layout type SWIZZLE_128B
  return d;
}

// Byte offset of element (mn, k) in a 128-byte-swizzled MN-major operand whose
// 64-element atoms are `lbo` bytes apart (rows of 128 bytes, 8-row groups 1024 apart).
__host__ __device__ __forceinline__ uint32_t mnmajor_sw128_off(int mn, int k, uint32_t lbo) {
  const uint32_t c = (uint32_t)(mn & 63);
  return (uint32_t)(mn >> 6) * lbo + (uint32_t)(k >> 3) * 1024u + (uint32_t)(k & 7) * 128u +
         ((((c >> 3) ^ (uint32_t)(k & 7)) & 7u) << 4) + (c & 7u) * 2u;
}

// bf16 pair helpers: pack two floats (round to nearest even; exact for values
// that are already bf16) and the correctly rounded product of two bf16 pairs.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&p);
}

__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 D.
__host__ __device__ constexpr uint32_t make_idesc_bf16(int M, int N, int a_mn_major, int b_mn_major) {
  return (1u << 4)                          // D format: F32
         | (1u << 7)                        // A format: BF16
         | (1u << 10)                       // B format: BF16
         | ((uint32_t)a_mn_major << 15)     // A major (0 = K, 1 = MN)
         | ((uint32_t)b_mn_major << 16)     // B major
         | ((uint32_t)(N >> 3) << 17)       // N / 8
         | ((uint32_t)(M >> 4) << 24);      // M / 16
}

// Byte offset of element (mn, k) in a no-swizzle K-major operand.
__host__ __device__ __forceinline__ uint32_t kmajor_off(int mn, int k, uint32_t sbo, uint32_t lbo) {
  return (uint32_t)(mn & 7) * 16u + (uint32_t)(mn >> 3) * sbo + (uint32_t)(k & 7) * 2u + (uint32_t)(k >> 3) * lbo;
}

// Byte offset of element (mn, k) in a no-swizzle MN-major operand.
__host__ __device__ __forceinline__ uint32_t mnmajor_off(int mn, int k, uint32_t sbo, uint32_t lbo) {
  return (uint32_t)(mn & 7) * 2u + (uint32_t)(mn >> 3) * sbo + (uint32_t)(k & 7) * 16u + (uint32_t)(k >> 3) * lbo;
}

}  // namespace dynconv
