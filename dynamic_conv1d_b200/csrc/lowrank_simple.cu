// lowrank_simple.cu -- CUDA-core lowrank kernels for the float32 path and for
// shapes outside the tensor-core kernels' envelope (W > 4; R_kernel > 32 in the
// backward, > 64 in the forward; D not a multiple of 8; unaligned tensors).
//
// Reference behaviour: lowrank.py:24-67 (forward), lowrank.py:86-140 (dU/dz),
// lowrank.py:158-205 (dx); oracle reference.py:23-39.  The reference's float32
// path uses IEEE-precision dots (lowrank.py:61,133,192); these kernels compute
// every product and sum in float32 FMA, so they match it to float32 rounding.
//
// The static filter is folded in as rank R (z_ext[..., R] = 1, U_ext[R] = static_w)
// by index arithmetic, never materialised in HBM (the reference pads/cats,
// lowrank.py:222-226).  The operands of a tile are staged in shared memory, so U is
// read once per tile and dy / x once per group of 8 ranks.  All reductions have a
// fixed order: dz within a block (channel chunks in order, slices in order); dU by
// per-chunk partial rows summed in reduce.cu.
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

constexpr int kMaxRk = 64;  // R_kernel bound of these kernels (dz keeps 8 ranks per warp x 8 warps)

}  // namespace

// The bf16 path rounds the products dy * x_shift to bf16 before the dz / dU sums, as
// the reference's bf16 kernel does (lowrank.py:127-129); the float32 path keeps them.
template <typename T>
__device__ __forceinline__ float round_p(float v) {
  if constexpr (sizeof(T) == 2) return __bfloat162float(__float2bfloat16_rn(v));
  else return v;
}

// ---------------------------------------------------------------------------- y and dx
// y[tok, d]  = sum_w K_w(tok) x[tok - w, d] (+ x[tok, d])           (DX = false)
// dx[tok, d] = sum_w K_w(tok + w) dy[tok + w, d] (+ dy[tok, d])      (DX = true)
// with K_w(s)[d] = sum_r z_ext[s, r] U_ext[r, w, d] (lowrank.py:24-67, 158-205).  A block
// owns 64 channels x 64 tokens: the U_ext block [Rk][W][64] and the tile's z_ext rows are
// staged in shared memory once (fp32), so U is read once per tile instead of once per
// token.  Thread (channel c, token subgroup) computes 4 consecutive tokens at a time: per
// rank it loads the W values U[r][.][c] and the z values of its tokens once and does
// 4 x W multiply-adds with them.
constexpr int kKxCh = 64, kKxTok = 64, kKxGrp = 4;

template <typename T, bool DX, int W>
__global__ void __launch_bounds__(256) lr_kx_tiled_kernel(const T* __restrict__ xin, const T* __restrict__ z,
                                                          const T* __restrict__ U, const T* __restrict__ sw,
                                                          T* __restrict__ out, int64_t ntok, int Tlen, int D, int R,
                                                          int Rk, int residual) {
  extern __shared__ float smf[];
  float* us = smf;                       // [Rk][W][kKxCh]
  float* zs = us + Rk * W * kKxCh;       // [kKxTok + W - 1][Rk]
  const int d0 = blockIdx.x * kKxCh;
  const int64_t k0 = (int64_t)blockIdx.y * kKxTok;
  for (int i = threadIdx.x; i < Rk * W * kKxCh; i += blockDim.x) {
    const int cc = i % kKxCh, rw = i / kKxCh, w = rw % W, r = rw / W, d = d0 + cc;
    us[i] = d < D ? uext(U, sw, r, w, d, R, D, W) : 0.f;
  }
  const int nz = kKxTok + (DX ? W - 1 : 0);
  for (int i = threadIdx.x; i < nz * Rk; i += blockDim.x) {
    const int row = i / Rk, r = i % Rk;
    const int64_t k = k0 + row;
    zs[i] = k < ntok ? zext(z + k * R, r, R) : 0.f;
  }
  __syncthreads();
  const int c = threadIdx.x % kKxCh, sub = threadIdx.x / kKxCh;
  const int d = d0 + c;
  if (d >= D) return;
  constexpr int NZ = DX ? kKxGrp + W - 1 : kKxGrp;  // z rows a group of tokens reads
  for (int j0 = sub * kKxGrp; j0 < kKxTok; j0 += (256 / kKxCh) * kKxGrp) {
    if (k0 + j0 >= ntok) break;
    // K[tt][w] = K_w(token j0 + tt (+ w for dx)), summed over r in order
    float K[kKxGrp][W];
#pragma unroll
    for (int tt = 0; tt < kKxGrp; ++tt)
#pragma unroll
      for (int w = 0; w < W; ++w) K[tt][w] = 0.f;
    for (int r = 0; r < Rk; ++r) {
      float u[W], zr[NZ];
#pragma unroll
      for (int w = 0; w < W; ++w) u[w] = us[(r * W + w) * kKxCh + c];
#pragma unroll
      for (int i = 0; i < NZ; ++i) zr[i] = zs[(j0 + i) * Rk + r];
#pragma unroll
      for (int tt = 0; tt < kKxGrp; ++tt)
#pragma unroll
        for (int w = 0; w < W; ++w) K[tt][w] = fmaf(zr[DX ? tt + w : tt], u[w], K[tt][w]);
    }
    int t = (int)((k0 + j0) % Tlen);  // position of the group's first token in its sequence
#pragma unroll
    for (int tt = 0; tt < kKxGrp; ++tt, t = (t + 1 == Tlen) ? 0 : t + 1) {
      const int64_t tok = k0 + j0 + tt;
      if (tok < ntok) {
        float acc = 0.f;
#pragma unroll
        for (int w = 0; w < W; ++w) {
          if (DX ? (t + w >= Tlen) : (t - w < 0)) break;
          acc = fmaf(K[tt][w], Elem<T>::to_f(xin[(DX ? tok + w : tok - w) * D + d]), acc);
        }
        if (residual) acc += Elem<T>::to_f(xin[tok * D + d]);
        out[tok * D + d] = Elem<T>::from_f(acc);
      }
    }
  }
}

// ---------------------------------------------------------------------------- dz
// dz[tok, r] = sum_{w,d} P_w[tok, d] U[r, w, d],  P_w = dy[tok, d] x[tok - w, d], r < R
// (lowrank.py:86-140).  A block owns 32 tokens and walks D in 32-channel chunks: dy, x
// (with the W-1 rows before the tile) and the U chunk [R][W][32] are staged in shared
// memory, the products P once per chunk.  Warp (rank group g, channel slice sl) accumulates
// ranks 8g .. 8g + 7 of the 32 tokens (lane = token) over its slice of the chunk's channels,
// reading the ranks as two float4s from the U chunk stored [W][channel][rank] (a broadcast
// within the warp); with R <= 32 the 8 warps split the channels instead of idling.  The
// slices' sums are added in slice order at the end.  U is read once per 32 tokens.
constexpr int kDzTok = 32, kDzCh = 32, kDzPad = kDzCh + 1;

template <typename T, int W>
__global__ void __launch_bounds__(256) lr_dz_tiled_kernel(const T* __restrict__ x, const T* __restrict__ U,
                                                          const T* __restrict__ dy, T* __restrict__ dz, int64_t ntok,
                                                          int Tlen, int D, int R) {
  extern __shared__ float smf[];
  const int RP = (R + 7) / 8 * 8 + 4;             // a channel's ranks: whole float4 pairs, + 4 against bank conflicts
  float* us = smf;                                // [W][kDzCh][RP]
  float* ps = us + W * kDzCh * RP;                // [W][kDzTok][kDzPad]
  float* dys = ps + W * kDzTok * kDzPad;          // [kDzTok][kDzPad]
  float* xs = dys + kDzTok * kDzPad;              // [kDzTok + W - 1][kDzPad]
  float* red = xs + (kDzTok + W - 1) * kDzPad;    // [8 warps][kDzTok][8 ranks]
  __shared__ int tpos[kDzTok];                    // position of each token in its sequence
  const int64_t k0 = (int64_t)blockIdx.x * kDzTok;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int NG = R <= 8 ? 1 : R <= 16 ? 2 : R <= 32 ? 4 : 8;  // rank groups (of 8)
  const int NS = 8 / NG;                                       // channel slices per group
  const int rg = warp % NG, sl = warp / NG;
  const int cc_lo = sl * (kDzCh / NS), cc_hi = cc_lo + kDzCh / NS;
  if (threadIdx.x < kDzTok) tpos[threadIdx.x] = (int)((k0 + threadIdx.x) % Tlen);
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int dc0 = 0; dc0 < D; dc0 += kDzCh) {
    __syncthreads();  // the previous chunk's reads are done
    for (int i = threadIdx.x; i < kDzTok * kDzCh; i += blockDim.x) {
      const int row = i / kDzCh, cc = i % kDzCh, d = dc0 + cc;
      const int64_t k = k0 + row;
      dys[row * kDzPad + cc] = (k < ntok && d < D) ? Elem<T>::to_f(dy[k * D + d]) : 0.f;
    }
    for (int i = threadIdx.x; i < (kDzTok + W - 1) * kDzCh; i += blockDim.x) {
      const int row = i / kDzCh, cc = i % kDzCh, d = dc0 + cc;
      const int64_t k = k0 - (W - 1) + row;
      xs[row * kDzPad + cc] = (k >= 0 && k < ntok && d < D) ? Elem<T>::to_f(x[k * D + d]) : 0.f;
    }
    const int RQ = (R + 7) / 8 * 8;
    for (int i = threadIdx.x; i < RQ * W * kDzCh; i += blockDim.x) {
      const int cc = i % kDzCh, rw = i / kDzCh, w = rw % W, r = rw / W, d = dc0 + cc;
      us[(w * kDzCh + cc) * RP + r] = (d < D && r < R) ? Elem<T>::to_f(U[((size_t)r * W + w) * D + d]) : 0.f;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < W * kDzTok * kDzCh; i += blockDim.x) {
      const int cc = i % kDzCh, j = (i / kDzCh) % kDzTok, w = i / (kDzCh * kDzTok);
      const int64_t tok = k0 + j;
      float p = 0.f;
      if (tok < ntok && tpos[j] - w >= 0)
        p = round_p<T>(dys[j * kDzPad + cc] * xs[(j + W - 1 - w) * kDzPad + cc]);
      ps[(w * kDzTok + j) * kDzPad + cc] = p;
    }
    __syncthreads();
    if (8 * rg < R) {
      for (int w = 0; w < W; ++w) {
        const float* pr = ps + (w * kDzTok + lane) * kDzPad;
        const float* ur = us + (w * kDzCh) * RP + 8 * rg;
#pragma unroll 4
        for (int cc = cc_lo; cc < cc_hi; ++cc) {
          const float p = pr[cc];
          const float4 u0 = *reinterpret_cast<const float4*>(ur + cc * RP);
          const float4 u1 = *reinterpret_cast<const float4*>(ur + cc * RP + 4);
          acc[0] = fmaf(p, u0.x, acc[0]);
          acc[1] = fmaf(p, u0.y, acc[1]);
          acc[2] = fmaf(p, u0.z, acc[2]);
          acc[3] = fmaf(p, u0.w, acc[3]);
          acc[4] = fmaf(p, u1.x, acc[4]);
          acc[5] = fmaf(p, u1.y, acc[5]);
          acc[6] = fmaf(p, u1.z, acc[6]);
          acc[7] = fmaf(p, u1.w, acc[7]);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) red[(warp * kDzTok + lane) * 8 + i] = acc[i];
  __syncthreads();
  const int64_t tok = k0 + lane;
  if (sl == 0 && tok < ntok) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = 8 * rg + i;
      if (r < R) {
        float v = 0.f;
        for (int s2 = 0; s2 < NS; ++s2) v += red[((rg + NG * s2) * kDzTok + lane) * 8 + i];
        dz[tok * R + r] = Elem<T>::from_f(v);
      }
    }
  }
}

// ---------------------------------------------------------------------------- dU
// part[chunk][r][w*D + d] = sum_{tok in chunk} z_ext[tok, r] P_w[tok, d]  (lowrank.py:126-137,
// without the atomics).  Thread = channel; block (channel block, 8 ranks, token chunk).  The
// thread walks its chunk once, keeping the last W x values in registers, and accumulates
// [8 ranks][W taps]; dy and x are read once per group of 8 ranks.
constexpr int kDuChunk = 256;

template <typename T, int W>
__global__ void __launch_bounds__(128) lr_du_tiled_kernel(const T* __restrict__ x, const T* __restrict__ z,
                                                          const T* __restrict__ dy, float* __restrict__ part,
                                                          int64_t ntok, int Tlen, int D, int R, int Rk) {
  __shared__ float zsh[kDuChunk][8];  // z_ext of the chunk's tokens, this block's 8 ranks
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  const int r0 = blockIdx.y * 8;
  const int64_t c = blockIdx.z;
  const int64_t tbeg = c * kDuChunk;
  const int64_t tend = min(tbeg + (int64_t)kDuChunk, ntok);
  for (int i = threadIdx.x; i < kDuChunk * 8; i += blockDim.x) {
    const int j = i / 8, r = r0 + i % 8;
    const int64_t tok = tbeg + j;
    zsh[j][i % 8] = (tok < tend && r < Rk) ? (r < R ? Elem<T>::to_f(z[tok * R + r]) : 1.f) : 0.f;
  }
  __syncthreads();
  if (d >= D) return;
  float acc[8][W];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int w = 0; w < W; ++w) acc[i][w] = 0.f;
  // xw[w] = x[tok - w, d] once token tok is loaded; before the first token it holds the
  // chunk's look-behind x[tbeg - 1 - w] (values from another batch row are masked below)
  float xw[W];
#pragma unroll
  for (int w = 0; w < W; ++w) xw[w] = tbeg - 1 - w >= 0 ? Elem<T>::to_f(x[(tbeg - 1 - w) * D + d]) : 0.f;
  int t = (int)(tbeg % Tlen);
#pragma unroll 4
  for (int64_t tok = tbeg; tok < tend; ++tok) {
#pragma unroll
    for (int w = W - 1; w > 0; --w) xw[w] = xw[w - 1];
    xw[0] = Elem<T>::to_f(x[tok * D + d]);
    const float g = Elem<T>::to_f(dy[tok * D + d]);
    float p[W];
#pragma unroll
    for (int w = 0; w < W; ++w) p[w] = t - w >= 0 ? round_p<T>(g * xw[w]) : 0.f;
    const float* zr = zsh[tok - tbeg];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float zz = zr[i];  // 0 for ranks >= R_kernel (never stored)
#pragma unroll
      for (int w = 0; w < W; ++w) acc[i][w] = fmaf(zz, p[w], acc[i][w]);
    }
    if (++t == Tlen) t = 0;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = r0 + i;
    if (r < Rk) {
#pragma unroll
      for (int w = 0; w < W; ++w) part[(c * Rk + r) * (int64_t)W * D + (int64_t)w * D + d] = acc[i][w];
    }
  }
}

int64_t lr_simple_partial_rows(int64_t B, int64_t T) { return (B * T + kDuChunk - 1) / kDuChunk; }

namespace {

template <typename K>
int set_smem(K kern, size_t bytes, const char* what) {
  if (bytes <= 48 * 1024) return DYNCONV_OK;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return cuda_status(e, what);
  }
  return DYNCONV_OK;
}

template <typename E, bool DX, int W>
int launch_kx_w(const void* xin, const void* z, const void* U, const void* sw, void* out, int64_t B, int64_t Tlen,
                int64_t D, int R, int Rk, int residual, cudaStream_t st) {
  const int64_t ntok = B * Tlen;
  const size_t smem = ((size_t)Rk * W * kKxCh + (size_t)(kKxTok + W - 1) * Rk) * sizeof(float);
  auto kern = lr_kx_tiled_kernel<E, DX, W>;
  if (int s = set_smem(kern, smem, "cudaFuncSetAttribute(lr_kx_tiled)")) return s;
  dim3 grid((unsigned)((D + kKxCh - 1) / kKxCh), (unsigned)((ntok + kKxTok - 1) / kKxTok));
  kern<<<grid, 256, smem, st>>>((const E*)xin, (const E*)z, (const E*)U, (const E*)sw, (E*)out, ntok, (int)Tlen, (int)D,
                                R, Rk, residual);
  DYNCONV_CHECK_LAUNCH(DX ? "lr_kx_tiled_kernel(dx)" : "lr_kx_tiled_kernel(y)");
  return DYNCONV_OK;
}

template <typename E, bool DX>
int launch_kx(const void* xin, const void* z, const void* U, const void* sw, void* out, int64_t B, int64_t Tlen,
              int64_t D, int R, int Rk, int W, int residual, cudaStream_t st) {
  switch (W) {
    case 1: return launch_kx_w<E, DX, 1>(xin, z, U, sw, out, B, Tlen, D, R, Rk, residual, st);
    case 2: return launch_kx_w<E, DX, 2>(xin, z, U, sw, out, B, Tlen, D, R, Rk, residual, st);
    case 3: return launch_kx_w<E, DX, 3>(xin, z, U, sw, out, B, Tlen, D, R, Rk, residual, st);
    case 4: return launch_kx_w<E, DX, 4>(xin, z, U, sw, out, B, Tlen, D, R, Rk, residual, st);
    case 5: return launch_kx_w<E, DX, 5>(xin, z, U, sw, out, B, Tlen, D, R, Rk, residual, st);
    case 6: return launch_kx_w<E, DX, 6>(xin, z, U, sw, out, B, Tlen, D, R, Rk, residual, st);
    case 7: return launch_kx_w<E, DX, 7>(xin, z, U, sw, out, B, Tlen, D, R, Rk, residual, st);
    case 8: return launch_kx_w<E, DX, 8>(xin, z, U, sw, out, B, Tlen, D, R, Rk, residual, st);
    default: return set_error(DYNCONV_ERR_UNSUPPORTED, "W=%d not supported (1..8)", W);
  }
}

template <typename E, int W>
int launch_dz_w(const void* x, const void* U, const void* dy, void* dz, int64_t B, int64_t Tlen, int64_t D, int R,
                cudaStream_t st) {
  const int64_t ntok = B * Tlen;
  const size_t smem = ((size_t)((R + 7) / 8 * 8 + 4) * W * kDzCh + (size_t)W * kDzTok * kDzPad +
                       (size_t)kDzTok * kDzPad + (size_t)(kDzTok + W - 1) * kDzPad + (size_t)8 * kDzTok * 8) *
                      sizeof(float);
  auto kern = lr_dz_tiled_kernel<E, W>;
  if (int s = set_smem(kern, smem, "cudaFuncSetAttribute(lr_dz_tiled)")) return s;
  kern<<<(unsigned)((ntok + kDzTok - 1) / kDzTok), 256, smem, st>>>((const E*)x, (const E*)U, (const E*)dy, (E*)dz,
                                                                    ntok, (int)Tlen, (int)D, R);
  DYNCONV_CHECK_LAUNCH("lr_dz_tiled_kernel");
  return DYNCONV_OK;
}

template <typename E>
int launch_dz(const void* x, const void* U, const void* dy, void* dz, int64_t B, int64_t Tlen, int64_t D, int R, int W,
              cudaStream_t st) {
  switch (W) {
    case 1: return launch_dz_w<E, 1>(x, U, dy, dz, B, Tlen, D, R, st);
    case 2: return launch_dz_w<E, 2>(x, U, dy, dz, B, Tlen, D, R, st);
    case 3: return launch_dz_w<E, 3>(x, U, dy, dz, B, Tlen, D, R, st);
    case 4: return launch_dz_w<E, 4>(x, U, dy, dz, B, Tlen, D, R, st);
    case 5: return launch_dz_w<E, 5>(x, U, dy, dz, B, Tlen, D, R, st);
    case 6: return launch_dz_w<E, 6>(x, U, dy, dz, B, Tlen, D, R, st);
    case 7: return launch_dz_w<E, 7>(x, U, dy, dz, B, Tlen, D, R, st);
    case 8: return launch_dz_w<E, 8>(x, U, dy, dz, B, Tlen, D, R, st);
    default: return set_error(DYNCONV_ERR_UNSUPPORTED, "W=%d not supported (1..8)", W);
  }
}

template <typename E, int W>
int launch_du_w(const void* x, const void* z, const void* dy, float* part, int64_t B, int64_t Tlen, int64_t D, int R,
                int Rk, cudaStream_t st) {
  const int64_t ntok = B * Tlen;
  dim3 grid((unsigned)((D + 127) / 128), (unsigned)((Rk + 7) / 8), (unsigned)lr_simple_partial_rows(B, Tlen));
  lr_du_tiled_kernel<E, W><<<grid, 128, 0, st>>>((const E*)x, (const E*)z, (const E*)dy, part, ntok, (int)Tlen, (int)D, R,
                                                 Rk);
  DYNCONV_CHECK_LAUNCH("lr_du_tiled_kernel");
  return DYNCONV_OK;
}

template <typename E>
int launch_du(const void* x, const void* z, const void* dy, float* part, int64_t B, int64_t Tlen, int64_t D, int R,
              int Rk, int W, cudaStream_t st) {
  switch (W) {
    case 1: return launch_du_w<E, 1>(x, z, dy, part, B, Tlen, D, R, Rk, st);
    case 2: return launch_du_w<E, 2>(x, z, dy, part, B, Tlen, D, R, Rk, st);
    case 3: return launch_du_w<E, 3>(x, z, dy, part, B, Tlen, D, R, Rk, st);
    case 4: return launch_du_w<E, 4>(x, z, dy, part, B, Tlen, D, R, Rk, st);
    case 5: return launch_du_w<E, 5>(x, z, dy, part, B, Tlen, D, R, Rk, st);
    case 6: return launch_du_w<E, 6>(x, z, dy, part, B, Tlen, D, R, Rk, st);
    case 7: return launch_du_w<E, 7>(x, z, dy, part, B, Tlen, D, R, Rk, st);
    case 8: return launch_du_w<E, 8>(x, z, dy, part, B, Tlen, D, R, Rk, st);
    default: return set_error(DYNCONV_ERR_UNSUPPORTED, "W=%d not supported (1..8)", W);
  }
}

}  // namespace

int lr_fwd_simple_launch(const void* x, const void* z, const void* U, const void* sw, void* y, int64_t B, int64_t T,
                         int64_t D, int R, int Rk, int W, int dtype, int residual, cudaStream_t st) {
  if (Rk > kMaxRk) return set_error(DYNCONV_ERR_UNSUPPORTED, "R_kernel=%d > %d", Rk, kMaxRk);
  if (dtype == DYNCONV_DTYPE_BF16)
    return launch_kx<__nv_bfloat16, false>(x, z, U, sw, y, B, T, D, R, Rk, W, residual, st);
  return launch_kx<float, false>(x, z, U, sw, y, B, T, D, R, Rk, W, residual, st);
}

// dx, dz, and the fp32 dU partial rows (to be summed by reduce_partials_launch).
int lr_bwd_simple_launch(const void* x, const void* z, const void* U, const void* sw, const void* dy, void* dx,
                         void* dz, float* part, int64_t B, int64_t T, int64_t D, int R, int Rk, int W, int dtype,
                         int residual, cudaStream_t st) {
  if (Rk > kMaxRk) return set_error(DYNCONV_ERR_UNSUPPORTED, "R_kernel=%d > %d", Rk, kMaxRk);
  int s;
  if (dtype == DYNCONV_DTYPE_BF16) {
    using T16 = __nv_bfloat16;
    if ((s = launch_kx<T16, true>(dy, z, U, sw, dx, B, T, D, R, Rk, W, residual, st))) return s;
    if ((s = launch_dz<T16>(x, U, dy, dz, B, T, D, R, W, st))) return s;
    return launch_du<T16>(x, z, dy, part, B, T, D, R, Rk, W, st);
  }
  if ((s = launch_kx<float, true>(dy, z, U, sw, dx, B, T, D, R, Rk, W, residual, st))) return s;
  if ((s = launch_dz<float>(x, U, dy, dz, B, T, D, R, W, st))) return s;
  return launch_du<float>(x, z, dy, part, B, T, D, R, Rk, W, st);
}

}  // namespace dynconv
