// reduce.cu -- deterministic second-pass reductions and float32 -> dtype casts.
//
// The backward kernels never use floating-point atomics for the shared gradients
// (dstatic_w, dU): each producer writes a float32 partial row into the workspace
// and this pass sums the P partial rows in a fixed order (p = 0 .. P-1), so the
// result is bit-identical from run to run.  The reference accumulates the same
// sums with fp32 atomics (headwise.py:157, lowrank.py:137).
#include "common.cuh"

namespace dynconv {

// out_f32[i] = sum_p part[p*n + i] (p ascending); optionally also cast into out (dtype T).
// One element per thread; the partial rows are loaded eight at a time ahead of the
// (still ascending) additions, so the load latencies overlap.
template <typename T>
__global__ void __launch_bounds__(256) reduce_partials_kernel(const float* __restrict__ part, int P, int64_t n,
                                                              float* __restrict__ out_f32, T* __restrict__ out) {
  constexpr int kAhead = 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float acc = 0.f;
    int p = 0;
    for (; p + kAhead <= P; p += kAhead) {
      float v[kAhead];
#pragma unroll
      for (int j = 0; j < kAhead; ++j) v[j] = __ldg(part + (int64_t)(p + j) * n + i);
#pragma unroll
      for (int j = 0; j < kAhead; ++j) acc += v[j];
    }
    for (; p < P; ++p) acc += __ldg(part + (int64_t)p * n + i);
    if (out_f32) out_f32[i] = acc;
    if (out) out[i] = Elem<T>::from_f(acc);
  }
}

template <typename T>
__global__ void __launch_bounds__(256) cast_f32_kernel(const float* __restrict__ src, T* __restrict__ dst, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = Elem<T>::from_f(src[i]);
}

static unsigned reduce_grid(int64_t n) {
  int64_t g = (n + 255) / 256;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (unsigned)g;
}

int reduce_partials_launch(const float* part, int P, int64_t n, float* out_f32, void* out, int dtype,
                           cudaStream_t st) {
  if (n <= 0) return DYNCONV_OK;
  if (dtype == DYNCONV_DTYPE_BF16)
    reduce_partials_kernel<__nv_bfloat16><<<reduce_grid(n), 256, 0, st>>>(part, P, n, out_f32, (__nv_bfloat16*)out);
  else
    reduce_partials_kernel<float><<<reduce_grid(n), 256, 0, st>>>(part, P, n, out_f32, (float*)out);
  DYNCONV_CHECK_LAUNCH("reduce_partials_kernel");
  return DYNCONV_OK;
}

int cast_f32_launch(const float* src, void* dst, int64_t n, int dtype, cudaStream_t st) {
  if (n <= 0) return DYNCONV_OK;
  int64_t g = (n + 255) / 256;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (g > cap) g = cap;
  if (dtype == DYNCONV_DTYPE_BF16)
    cast_f32_kernel<__nv_bfloat16><<<(unsigned)g, 256, 0, st>>>(src, (__nv_bfloat16*)dst, n);
  else
    cast_f32_kernel<float><<<(unsigned)g, 256, 0, st>>>(src, (float*)dst, n);
  DYNCONV_CHECK_LAUNCH("cast_f32_kernel");
  return DYNCONV_OK;
}

}  // namespace dynconv
