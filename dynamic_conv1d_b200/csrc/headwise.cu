// headwise.cu -- headwise dynamic short convolution, forward and backward.
//
// Reference behaviour: headwise.py:24-91 (forward kernel) and headwise.py:105-215
// (backward kernel) of OliverSieberling/dynamic-conv1d, oracle reference.py:5-20.
//
// Design (B200): both directions are pure HBM streams (no contraction worth a
// tensor core), so each thread owns VEC consecutive channels (one 16-byte vector)
// and walks a run of L consecutive timesteps of one batch row.  The W-1 previous
// x rows (forward, backward dweight) and the W-1 following dy rows (backward dx)
// live in a register ring, so every row is read from HBM once per thread; the
// W-1 halo rows at the start of a run are re-read by the neighbouring run of the
// same block and are served by L1/L2.
//
//   block = 32 (channel vectors, one warp) x 8 (runs)   -> 32*VEC channels x 8*L steps
//   grid  = ceil(D / (32*VEC)) x (B * ceil(T / (8*L)))
//
// Backward reductions:
//   dweight[b,t,h,w] = sum_{d in head h} dy[b,t,d] x[b,t-w,d]  -- in-thread sum over
//       the head's channels of this vector, then xor-shuffles across the G = hs/VEC
//       lanes of a head (no shared memory, no atomics);
//   dstatic_w[w,d]   = sum_{b,t} dy x_shift -- per-thread fp32 sums, a fixed-order
//       reduction over the 8 runs of the block in shared memory, one fp32 partial
//       row per block in the workspace, then a fixed-order second pass
//       (reduce_partials in reduce.cu).  Deterministic; the reference uses fp32
//       atomics here (headwise.py:157).
#include "common.cuh"

namespace dynconv {

constexpr int kRunsPerBlock = 8;

template <typename T, int VEC, int K, int W>
__global__ void __launch_bounds__(256) hw_fwd_kernel(const T* __restrict__ x, const T* __restrict__ wgt,
                                                     const T* __restrict__ sw, T* __restrict__ y, int Tlen,
                                                     int D, int H, int log2hs, int L, int nTB, int residual) {
  constexpr int HPT = VEC / K;  // heads touched by this thread's channel vector
  constexpr int CH = (HPT * W >= 16) ? 2 : 4;
  const int cg = blockIdx.x * 32 + threadIdx.x;
  const int d0 = cg * VEC;
  const int b = blockIdx.y / nTB;
  const int t0 = (blockIdx.y % nTB) * (kRunsPerBlock * L) + threadIdx.y * L;
  const int t1 = min(t0 + L, Tlen);
  if (d0 >= D || t0 >= Tlen) return;

  const size_t rowD = (size_t)D;
  const size_t rowHW = (size_t)H * W;
  const T* xb = x + (size_t)b * Tlen * rowD + d0;
  T* yb = y + (size_t)b * Tlen * rowD + d0;
  const int h0 = d0 >> log2hs;
  const T* wb = wgt + ((size_t)b * Tlen * H + h0) * W;

  float s[W][VEC];
#pragma unroll
  for (int w = 0; w < W; ++w) {
    if (sw != nullptr) {
      load_span<T, VEC>(sw + (size_t)w * D + d0, s[w]);
    } else {
#pragma unroll
      for (int c = 0; c < VEC; ++c) s[w][c] = 0.f;
    }
  }

  // xw[j] holds x at step (t - (W-1) + j) relative to the chunk start t.
  float xw[W - 1 + CH][VEC];
#pragma unroll
  for (int j = 0; j < W - 1; ++j) {
    const int tt = t0 - (W - 1) + j;
    if (tt >= 0) {
      load_span<T, VEC>(xb + (size_t)tt * rowD, xw[j]);
    } else {
#pragma unroll
      for (int c = 0; c < VEC; ++c) xw[j][c] = 0.f;
    }
  }

  for (int t = t0; t < t1; t += CH) {
    float wv[CH][HPT * W];
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      const int tt = t + i;
      if (tt < t1) {
        load_span<T, VEC>(xb + (size_t)tt * rowD, xw[W - 1 + i]);
        load_span<T, HPT * W>(wb + (size_t)tt * rowHW, wv[i]);
      } else {
#pragma unroll
        for (int c = 0; c < VEC; ++c) xw[W - 1 + i][c] = 0.f;
#pragma unroll
        for (int c = 0; c < HPT * W; ++c) wv[i][c] = 0.f;
      }
    }
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      const int tt = t + i;
      if (tt < t1) {
        float out[VEC];
#pragma unroll
        for (int c = 0; c < VEC; ++c) {
          float acc = 0.f;
#pragma unroll
          for (int w = 0; w < W; ++w) acc = fmaf(wv[i][(c / K) * W + w] + s[w][c], xw[W - 1 + i - w][c], acc);
          if (residual) acc += xw[W - 1 + i][c];
          out[c] = acc;
        }
        store_span<T, VEC>(yb + (size_t)tt * rowD, out);
      }
    }
#pragma unroll
    for (int j = 0; j < W - 1; ++j) {
#pragma unroll
      for (int c = 0; c < VEC; ++c) xw[j][c] = xw[j + CH][c];
    }
  }
}

template <typename T, int VEC, int K, int W>
__global__ void __launch_bounds__(256) hw_bwd_kernel(const T* __restrict__ x, const T* __restrict__ wgt,
                                                     const T* __restrict__ sw, const T* __restrict__ dy,
                                                     T* __restrict__ dx, T* __restrict__ dw,
                                                     float* __restrict__ dsw_part, int Tlen, int D, int H,
                                                     int log2hs, int L, int nTB, int residual) {
  constexpr int HPT = VEC / K;
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int cg = blockIdx.x * 32 + tx;
  const int d0 = cg * VEC;
  const bool active = d0 < D;
  const int b = blockIdx.y / nTB;
  const int tb = blockIdx.y % nTB;
  const int t0 = tb * (kRunsPerBlock * L) + ty * L;
  const int t1 = min(t0 + L, Tlen);  // may be <= t0: empty run (still joins shuffles / barriers)
  // threads per head along the warp (only > 1 when a head spans several vectors)
  const int hs = 1 << log2hs;
  const int G = (hs > VEC) ? (hs / VEC) : 1;

  const size_t rowD = (size_t)D;
  const size_t rowHW = (size_t)H * W;
  const int dsafe = active ? d0 : 0;
  const T* xb = x + (size_t)b * Tlen * rowD + dsafe;
  const T* dyb = dy + (size_t)b * Tlen * rowD + dsafe;
  T* dxb = dx + (size_t)b * Tlen * rowD + dsafe;
  const int h0 = dsafe >> log2hs;
  const T* wb = wgt + ((size_t)b * Tlen * H + h0) * W;
  T* dwb = dw + ((size_t)b * Tlen * H + h0) * W;

  float s[W][VEC];
#pragma unroll
  for (int w = 0; w < W; ++w) {
    if (sw != nullptr && active) {
      load_span<T, VEC>(sw + (size_t)w * D + d0, s[w]);
    } else {
#pragma unroll
      for (int c = 0; c < VEC; ++c) s[w][c] = 0.f;
    }
  }

  float dsa[W][VEC];  // dstatic_w partial sums of this thread
  float dxa[W][VEC];  // dx accumulators, slot (tok - t0) mod W
  float xw[W][VEC];   // x ring, slot (tok - t0) mod W
#pragma unroll
  for (int w = 0; w < W; ++w) {
#pragma unroll
    for (int c = 0; c < VEC; ++c) {
      dsa[w][c] = 0.f;
      dxa[w][c] = 0.f;
      xw[w][c] = 0.f;
    }
  }
  // Look-behind rows t0-W+1 .. t0-1 go to slots 1 .. W-1.
#pragma unroll
  for (int j = 1; j < W; ++j) {
    const int tt = t0 - W + j;
    if (active && tt >= 0 && tt < Tlen && t0 < t1) load_span<T, VEC>(xb + (size_t)tt * rowD, xw[j]);
  }

  const int s_end = (t1 > t0) ? (t1 + W - 1) : t0;  // rows t0 .. t1+W-2 contribute to dx[t0 .. t1-1]
  for (int sb = t0; sb < s_end; sb += W) {
#pragma unroll
    for (int i = 0; i < W; ++i) {
      const int srow = sb + i;
      if (srow < s_end) {  // uniform across the warp (same run)
        float g[VEC], wv[HPT * W];
        const bool row_ok = active && srow < Tlen;
        if (row_ok) {
          load_span<T, VEC>(dyb + (size_t)srow * rowD, g);
          load_span<T, HPT * W>(wb + (size_t)srow * rowHW, wv);
        } else {
#pragma unroll
          for (int c = 0; c < VEC; ++c) g[c] = 0.f;
#pragma unroll
          for (int c = 0; c < HPT * W; ++c) wv[c] = 0.f;
        }
        if (srow < t1) {
          if (row_ok) {
            load_span<T, VEC>(xb + (size_t)srow * rowD, xw[i]);
          } else {
#pragma unroll
            for (int c = 0; c < VEC; ++c) xw[i][c] = 0.f;
          }
          // dweight and dstatic_w for row srow
          float hsum[HPT * W];
#pragma unroll
          for (int k = 0; k < HPT * W; ++k) hsum[k] = 0.f;
#pragma unroll
          for (int w = 0; w < W; ++w) {
#pragma unroll
            for (int c = 0; c < VEC; ++c) {
              const float p = g[c] * xw[(i - w + W) % W][c];
              dsa[w][c] += p;
              hsum[(c / K) * W + w] += p;
            }
          }
          for (int off = 1; off < G; off <<= 1) {
#pragma unroll
            for (int k = 0; k < HPT * W; ++k) hsum[k] += __shfl_xor_sync(0xffffffffu, hsum[k], off);
          }
          if (row_ok && (G == 1 || (tx & (G - 1)) == 0)) store_span<T, HPT * W>(dwb + (size_t)srow * rowHW, hsum);
          if (residual) {
#pragma unroll
            for (int c = 0; c < VEC; ++c) dxa[i][c] += g[c];
          }
        }
        // dx[srow - k] += dy[srow] * (weight[srow, h, k] + static_w[k])
#pragma unroll
        for (int k = 0; k < W; ++k) {
          const int tt = srow - k;
          if (tt >= t0 && tt < t1) {
#pragma unroll
            for (int c = 0; c < VEC; ++c) dxa[(i - k + W) % W][c] = fmaf(g[c], wv[(c / K) * W + k] + s[k][c], dxa[(i - k + W) % W][c]);
          }
        }
        // token srow-(W-1) is complete
        const int tdone = srow - (W - 1);
        if (tdone >= t0 && tdone < t1) {
          if (active) store_span<T, VEC>(dxb + (size_t)tdone * rowD, dxa[(i + 1) % W]);
#pragma unroll
          for (int c = 0; c < VEC; ++c) dxa[(i + 1) % W][c] = 0.f;
        }
      }
    }
  }

  if (dsw_part != nullptr) {
    // fixed-order reduction of the 8 runs of this block (one tap at a time),
    // then one partial row per block and tap
    __shared__ float red[kRunsPerBlock][32 * VEC];
    const int tid = ty * 32 + tx;
    float* part = dsw_part + (size_t)(b * nTB + tb) * W * rowD;
#pragma unroll
    for (int w = 0; w < W; ++w) {
#pragma unroll
      for (int c = 0; c < VEC; ++c) red[ty][tx * VEC + c] = dsa[w][c];
      __syncthreads();
      for (int dl = tid; dl < 32 * VEC; dl += 32 * kRunsPerBlock) {
        const int d = blockIdx.x * 32 * VEC + dl;
        if (d < D) {
          float acc = 0.f;
#pragma unroll
          for (int r = 0; r < kRunsPerBlock; ++r) acc += red[r][dl];
          part[(size_t)w * rowD + d] = acc;
        }
      }
      __syncthreads();
    }
  }
}

// ------------------------------------------------------------------ dispatch

namespace {

constexpr int kHwRun = 32;  // steps per thread run

struct HwGeom {
  dim3 grid, block;
  int nTB;
};

HwGeom hw_geom(int64_t B, int64_t T, int64_t D, int vec) {
  HwGeom g;
  const int64_t ncg = (D + vec - 1) / vec;
  g.nTB = (int)((T + kRunsPerBlock * kHwRun - 1) / (kRunsPerBlock * kHwRun));
  g.block = dim3(32, kRunsPerBlock);
  g.grid = dim3((unsigned)((ncg + 31) / 32), (unsigned)(B * g.nTB));
  return g;
}

template <typename E, int VEC, int K>
int launch_hw_fwd_w(const void* x, const void* w, const void* sw, void* y, int64_t B, int64_t T, int64_t D,
                    int64_t H, int W, int log2hs, int residual, cudaStream_t st) {
  HwGeom g = hw_geom(B, T, D, VEC);
#define DYNCONV_HWF(WW)                                                                                       \
  case WW:                                                                                                    \
    hw_fwd_kernel<E, VEC, K, WW><<<g.grid, g.block, 0, st>>>(                                                 \
        (const E*)x, (const E*)w, (const E*)sw, (E*)y, (int)T, (int)D, (int)H, log2hs, kHwRun, g.nTB, residual); \
    break;
  switch (W) {
    DYNCONV_HWF(1) DYNCONV_HWF(2) DYNCONV_HWF(3) DYNCONV_HWF(4)
    DYNCONV_HWF(5) DYNCONV_HWF(6) DYNCONV_HWF(7) DYNCONV_HWF(8)
    default: return set_error(DYNCONV_ERR_UNSUPPORTED, "W=%d not supported (1..8)", W);
  }
#undef DYNCONV_HWF
  DYNCONV_CHECK_LAUNCH("hw_fwd_kernel");
  return DYNCONV_OK;
}

template <typename E, int VEC, int K>
int launch_hw_bwd_w(const void* x, const void* w, const void* sw, const void* dy, void* dx, void* dw,
                    float* part, int64_t B, int64_t T, int64_t D, int64_t H, int W, int log2hs, int residual,
                    cudaStream_t st) {
  HwGeom g = hw_geom(B, T, D, VEC);
#define DYNCONV_HWB(WW)                                                                                  \
  case WW:                                                                                               \
    hw_bwd_kernel<E, VEC, K, WW><<<g.grid, g.block, 0, st>>>(                                            \
        (const E*)x, (const E*)w, (const E*)sw, (const E*)dy, (E*)dx, (E*)dw, part, (int)T, (int)D, (int)H, \
        log2hs, kHwRun, g.nTB, residual);                                                                \
    break;
  switch (W) {
    DYNCONV_HWB(1) DYNCONV_HWB(2) DYNCONV_HWB(3) DYNCONV_HWB(4)
    DYNCONV_HWB(5) DYNCONV_HWB(6) DYNCONV_HWB(7) DYNCONV_HWB(8)
    default: return set_error(DYNCONV_ERR_UNSUPPORTED, "W=%d not supported (1..8)", W);
  }
#undef DYNCONV_HWB
  DYNCONV_CHECK_LAUNCH("hw_bwd_kernel");
  return DYNCONV_OK;
}

// Picks the vector width and the in-thread head span K = min(hs, VEC).
template <typename E>
int hw_dispatch(bool fwd, const void* x, const void* w, const void* sw, const void* dy, void* dx_or_y,
                void* dw, float* part, int64_t B, int64_t T, int64_t D, int64_t H, int W, int log2hs,
                int residual, cudaStream_t st) {
  constexpr int V = Elem<E>::kVec;
  const int hs = 1 << log2hs;
  const bool vec_ok = (D % V) == 0;
  if (vec_ok) {
    if (hs >= V) {
      if (hs / V > 32) return set_error(DYNCONV_ERR_UNSUPPORTED, "head_size %d > %d not supported", hs, 32 * V);
      return fwd ? launch_hw_fwd_w<E, V, V>(x, w, sw, dx_or_y, B, T, D, H, W, log2hs, residual, st)
                 : launch_hw_bwd_w<E, V, V>(x, w, sw, dy, dx_or_y, dw, part, B, T, D, H, W, log2hs, residual, st);
    }
    if (hs == 1)
      return fwd ? launch_hw_fwd_w<E, V, 1>(x, w, sw, dx_or_y, B, T, D, H, W, log2hs, residual, st)
                 : launch_hw_bwd_w<E, V, 1>(x, w, sw, dy, dx_or_y, dw, part, B, T, D, H, W, log2hs, residual, st);
    if (hs == 2)
      return fwd ? launch_hw_fwd_w<E, V, 2>(x, w, sw, dx_or_y, B, T, D, H, W, log2hs, residual, st)
                 : launch_hw_bwd_w<E, V, 2>(x, w, sw, dy, dx_or_y, dw, part, B, T, D, H, W, log2hs, residual, st);
    if (hs == 4 && V > 4)
      return fwd ? launch_hw_fwd_w<E, V, (V > 4 ? 4 : V)>(x, w, sw, dx_or_y, B, T, D, H, W, log2hs, residual, st)
                 : launch_hw_bwd_w<E, V, (V > 4 ? 4 : V)>(x, w, sw, dy, dx_or_y, dw, part, B, T, D, H, W, log2hs,
                                                            residual, st);
    return set_error(DYNCONV_ERR_UNSUPPORTED, "head_size %d", hs);
  }
  // D not a multiple of the vector width: one channel per thread.
  if (hs > 32) return set_error(DYNCONV_ERR_UNSUPPORTED, "head_size %d > 32 with D %% %d != 0", hs, V);
  return fwd ? launch_hw_fwd_w<E, 1, 1>(x, w, sw, dx_or_y, B, T, D, H, W, log2hs, residual, st)
             : launch_hw_bwd_w<E, 1, 1>(x, w, sw, dy, dx_or_y, dw, part, B, T, D, H, W, log2hs, residual, st);
}

}  // namespace

int hw_partial_rows(int64_t B, int64_t T, int64_t D, int dtype) {
  const int vec = dtype == DYNCONV_DTYPE_BF16 ? Elem<__nv_bfloat16>::kVec : Elem<float>::kVec;
  return (int)(B * hw_geom(B, T, D, vec).nTB);
}

int hw_fwd_launch(const void* x, const void* w, const void* sw, void* y, int64_t B, int64_t T, int64_t D,
                  int64_t H, int W, int log2hs, int dtype, int residual, cudaStream_t st) {
  if (dtype == DYNCONV_DTYPE_BF16)
    return hw_dispatch<__nv_bfloat16>(true, x, w, sw, nullptr, y, nullptr, nullptr, B, T, D, H, W, log2hs, residual, st);
  return hw_dispatch<float>(true, x, w, sw, nullptr, y, nullptr, nullptr, B, T, D, H, W, log2hs, residual, st);
}

int hw_bwd_launch(const void* x, const void* w, const void* sw, const void* dy, void* dx, void* dw, float* part,
                  int64_t B, int64_t T, int64_t D, int64_t H, int W, int log2hs, int dtype, int residual,
                  cudaStream_t st) {
  if (dtype == DYNCONV_DTYPE_BF16)
    return hw_dispatch<__nv_bfloat16>(false, x, w, sw, dy, dx, dw, part, B, T, D, H, W, log2hs, residual, st);
  return hw_dispatch<float>(false, x, w, sw, dy, dx, dw, part, B, T, D, H, W, log2hs, residual, st);
}

}  // namespace dynconv
