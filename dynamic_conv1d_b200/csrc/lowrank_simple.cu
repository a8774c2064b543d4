// lowrank_simple.cu -- CUDA-core lowrank kernels for the float32 path and for
// shapes outside the tensor-core kernels' envelope (W > 4, R_kernel > 64 or odd D).
//
// Reference behaviour: lowrank.py:24-67 (forward), lowrank.py:86-140 (dU/dz),
// lowrank.py:158-205 (dx); oracle reference.py:23-39.  The reference's float32
// path uses IEEE-precision dots (lowrank.py:61,133,192); these kernels compute
// every product and sum in float32 FMA, so they match it to float32 rounding.
//
// The static filter is folded in as rank R (z_ext[..., R] = 1, U_ext[R] = static_w)
// by index arithmetic, never materialised in HBM (the reference pads/cats,
// lowrank.py:222-226).  All reductions have a fixed order: dz by warp shuffles and
// one shared-memory pass per token; dU by per-chunk partial rows summed in
// reduce.cu.
#include "common.cuh"

namespace dynconv {

namespace {

// z_ext[t, r] for the folded static rank
template <typename T>
__device__ __forceinline__ float zext(const T* __restrict__ zrow, int r, int R) {
  return r < R ? Elem<T>::to_f(zrow[r]) : 1.f;
}

// U_ext[r, w, d]
template <typename T>
__device__ __forceinline__ float uext(const T* __restrict__ U, const T* __restrict__ sw, int r, int w, int d, int R,
                                      int D, int W) {
  return r < R ? Elem<T>::to_f(U[((size_t)r * W + w) * D + d]) : Elem<T>::to_f(sw[(size_t)w * D + d]);
}

}  // namespace

// y[b,t,d]; one thread per (token, channel)
template <typename T>
__global__ void __launch_bounds__(256) lr_fwd_simple_kernel(const T* __restrict__ x, const T* __restrict__ z,
                                                            const T* __restrict__ U, const T* __restrict__ sw,
                                                            T* __restrict__ y, int Tlen, int D, int R, int Rk, int W,
                                                            int residual) {
  const int d = blockIdx.y * blockDim.x + threadIdx.x;
  const int64_t tok = blockIdx.x;  // b*T + t
  if (d >= D) return;
  const int t = (int)(tok % Tlen);
  const T* zrow = z + tok * R;
  float acc = 0.f;
  for (int w = 0; w < W; ++w) {
    if (t - w < 0) break;
    float k = 0.f;
    for (int r = 0; r < Rk; ++r) k = fmaf(zext(zrow, r, R), uext(U, sw, r, w, d, R, D, W), k);
    acc = fmaf(k, Elem<T>::to_f(x[(tok - w) * D + d]), acc);
  }
  if (residual) acc += Elem<T>::to_f(x[tok * D + d]);
  y[tok * D + d] = Elem<T>::from_f(acc);
}

// dx[b,t,d] = sum_w dy[t+w,d] * K[t+w,w,d]  (+ dy[t,d])
template <typename T>
__global__ void __launch_bounds__(256) lr_dx_simple_kernel(const T* __restrict__ z, const T* __restrict__ U,
                                                           const T* __restrict__ sw, const T* __restrict__ dy,
                                                           T* __restrict__ dx, int Tlen, int D, int R, int Rk, int W,
                                                           int residual) {
  const int d = blockIdx.y * blockDim.x + threadIdx.x;
  const int64_t tok = blockIdx.x;
  if (d >= D) return;
  const int t = (int)(tok % Tlen);
  float acc = 0.f;
  for (int w = 0; w < W; ++w) {
    if (t + w >= Tlen) break;
    const T* zrow = z + (tok + w) * R;
    float k = 0.f;
    for (int r = 0; r < Rk; ++r) k = fmaf(zext(zrow, r, R), uext(U, sw, r, w, d, R, D, W), k);
    acc = fmaf(k, Elem<T>::to_f(dy[(tok + w) * D + d]), acc);
  }
  if (residual) acc += Elem<T>::to_f(dy[tok * D + d]);
  dx[tok * D + d] = Elem<T>::from_f(acc);
}

// dz[b,t,r] = sum_{w,d} dy[t,d] x[t-w,d] U[r,w,d], r < R; one block (256 threads) per token.
constexpr int kMaxRk = 64;
template <typename T>
__global__ void __launch_bounds__(256) lr_dz_simple_kernel(const T* __restrict__ x, const T* __restrict__ U,
                                                           const T* __restrict__ dy, T* __restrict__ dz, int Tlen,
                                                           int D, int R, int W) {
  const int64_t tok = blockIdx.x;
  const int t = (int)(tok % Tlen);
  float acc[kMaxRk];
#pragma unroll
  for (int r = 0; r < kMaxRk; ++r) acc[r] = 0.f;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    const float g = Elem<T>::to_f(dy[tok * D + d]);
    for (int w = 0; w < W && t - w >= 0; ++w) {
      const float p = g * Elem<T>::to_f(x[(tok - w) * D + d]);
#pragma unroll
      for (int r = 0; r < kMaxRk; ++r)
        if (r < R) acc[r] = fmaf(p, Elem<T>::to_f(U[((size_t)r * W + w) * D + d]), acc[r]);
    }
  }
  __shared__ float red[8][kMaxRk];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int r = 0; r < kMaxRk; ++r) {
    if (r < R) {
      float v = acc[r];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0) red[warp][r] = v;
    }
  }
  __syncthreads();
  if (threadIdx.x < R) {
    float v = 0.f;
    for (int wp = 0; wp < (int)(blockDim.x >> 5); ++wp) v += red[wp][threadIdx.x];
    dz[tok * R + threadIdx.x] = Elem<T>::from_f(v);
  }
}

// part[chunk][r][w*D + d] = sum_{tok in chunk} z_ext[tok,r] dy[tok,d] x[tok-w,d]
// grid: (ceil(D/256), Rk*W, nchunks)
template <typename T>
__global__ void __launch_bounds__(256) lr_du_simple_kernel(const T* __restrict__ x, const T* __restrict__ z,
                                                           const T* __restrict__ dy, float* __restrict__ part,
                                                           int64_t ntok, int Tlen, int D, int R, int Rk, int W,
                                                           int chunk) {
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  const int r = blockIdx.y / W, w = blockIdx.y % W;
  const int64_t c = blockIdx.z;
  if (d >= D) return;
  const int64_t tbeg = c * chunk;
  const int64_t tend = min(tbeg + (int64_t)chunk, ntok);
  float acc = 0.f;
  for (int64_t tok = tbeg; tok < tend; ++tok) {
    const int t = (int)(tok % Tlen);
    if (t - w < 0) continue;
    const float zz = r < R ? Elem<T>::to_f(z[tok * R + r]) : 1.f;
    acc = fmaf(zz * Elem<T>::to_f(dy[tok * D + d]), Elem<T>::to_f(x[(tok - w) * D + d]), acc);
  }
  part[(c * Rk + r) * (int64_t)W * D + (int64_t)w * D + d] = acc;
}

namespace {
constexpr int kDuChunk = 256;
}

int64_t lr_simple_partial_rows(int64_t B, int64_t T) { return (B * T + kDuChunk - 1) / kDuChunk; }

int lr_fwd_simple_launch(const void* x, const void* z, const void* U, const void* sw, void* y, int64_t B, int64_t T,
                         int64_t D, int R, int Rk, int W, int dtype, int residual, cudaStream_t st) {
  dim3 grid((unsigned)(B * T), (unsigned)((D + 255) / 256));
  if (dtype == DYNCONV_DTYPE_BF16)
    lr_fwd_simple_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        (const __nv_bfloat16*)x, (const __nv_bfloat16*)z, (const __nv_bfloat16*)U, (const __nv_bfloat16*)sw,
        (__nv_bfloat16*)y, (int)T, (int)D, R, Rk, W, residual);
  else
    lr_fwd_simple_kernel<float><<<grid, 256, 0, st>>>((const float*)x, (const float*)z, (const float*)U,
                                                      (const float*)sw, (float*)y, (int)T, (int)D, R, Rk, W, residual);
  DYNCONV_CHECK_LAUNCH("lr_fwd_simple_kernel");
  return DYNCONV_OK;
}

// dx, dz, and the fp32 dU partial rows (to be summed by reduce_partials_launch).
int lr_bwd_simple_launch(const void* x, const void* z, const void* U, const void* sw, const void* dy, void* dx,
                         void* dz, float* part, int64_t B, int64_t T, int64_t D, int R, int Rk, int W, int dtype,
                         int residual, cudaStream_t st) {
  if (R > kMaxRk) return set_error(DYNCONV_ERR_UNSUPPORTED, "R=%d > %d", R, kMaxRk);
  const int64_t ntok = B * T;
  dim3 gdx((unsigned)ntok, (unsigned)((D + 255) / 256));
  dim3 gdu((unsigned)((D + 255) / 256), (unsigned)(Rk * W), (unsigned)lr_simple_partial_rows(B, T));
  if (dtype == DYNCONV_DTYPE_BF16) {
    using T16 = __nv_bfloat16;
    lr_dx_simple_kernel<T16><<<gdx, 256, 0, st>>>((const T16*)z, (const T16*)U, (const T16*)sw, (const T16*)dy,
                                                  (T16*)dx, (int)T, (int)D, R, Rk, W, residual);
    lr_dz_simple_kernel<T16><<<(unsigned)ntok, 256, 0, st>>>((const T16*)x, (const T16*)U, (const T16*)dy, (T16*)dz,
                                                            (int)T, (int)D, R, W);
    lr_du_simple_kernel<T16><<<gdu, 256, 0, st>>>((const T16*)x, (const T16*)z, (const T16*)dy, part, ntok, (int)T,
                                                  (int)D, R, Rk, W, kDuChunk);
  } else {
    lr_dx_simple_kernel<float><<<gdx, 256, 0, st>>>((const float*)z, (const float*)U, (const float*)sw,
                                                    (const float*)dy, (float*)dx, (int)T, (int)D, R, Rk, W, residual);
    lr_dz_simple_kernel<float><<<(unsigned)ntok, 256, 0, st>>>((const float*)x, (const float*)U, (const float*)dy,
                                                              (float*)dz, (int)T, (int)D, R, W);
    lr_du_simple_kernel<float><<<gdu, 256, 0, st>>>((const float*)x, (const float*)z, (const float*)dy, part, ntok,
                                                    (int)T, (int)D, R, Rk, W, kDuChunk);
  }
  DYNCONV_CHECK_LAUNCH("lr_bwd_simple kernels");
  note_launch(2);  // three kernels above, one counted by the check
  return DYNCONV_OK;
}

}  // namespace dynconv
