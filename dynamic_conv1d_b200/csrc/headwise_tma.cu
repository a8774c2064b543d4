// headwise_tma.cu -- headwise dynamic short convolution, bf16, TMA-staged
// persistent kernels (forward and backward).
//
// Reference behaviour: headwise.py:24-91 (forward kernel) and headwise.py:105-215
// (backward kernel) of OliverSieberling/dynamic-conv1d; oracle reference.py:5-20.
//
// Both directions stream HBM (no contraction worth a tensor core).  A tile is
// 256 channels x TR timesteps of one batch row; a CTA keeps one 256-channel block
// for a contiguous range of tiles (grid = n_dblk x n_groups, about one CTA per SM):
//
//   warp NC (producer, one lane): TMA loads of the tile's x rows (with the W-1
//       look-behind rows; zero fill for t < 0 and t >= T), and for the backward the
//       dy and weight rows with their W-1 look-ahead rows, into an S-stage ring
//       (full / empty mbarriers, every wait bounded);
//   warps 0..NC-1 (compute): lane l owns the 16-byte vector of channels 8l..8l+7,
//       warp c owns rows c*RPT .. c*RPT+RPT-1 of the tile; every operand comes from
//       shared memory, outputs go straight to HBM as 16-byte stores (a warp writes
//       512 contiguous bytes per row).
//
// Backward reductions:
//   dweight[b,t,h,w] = sum_{d in head h} dy[b,t,d] x[b,t-w,d]: in-thread over the
//       thread's channels of the head, then xor shuffles over the hs/8 lanes of a
//       head (hs >= 8); no shared memory, no atomics;
//   dstatic_w[w,d] = sum_{b,t} dy x_shift: per-thread fp32 sums over all of the
//       CTA's tiles (its channel block is fixed), a fixed-order sum over the NC
//       compute warps in shared memory at the end, one fp32 partial row per CTA,
//       then the fixed-order second pass reduce_partials (reduce.cu).  The
//       reference accumulates with fp32 atomics (headwise.py:157).
#include "common.cuh"

namespace dynconv {

DYNCONV_DEFINE_ERROR_ACCESSOR(hw_tma_error_word)

namespace {

constexpr int kCB = 256;  // channels per tile (32 lanes x 8)
constexpr int kNC = 8;    // compute warps
constexpr int kHwThreads = 32 * (kNC + 1);
constexpr int kSmemCap = 200 * 1024;

// Per-instantiation geometry.  K = min(head_size, 8): a thread's 8 channels span
// HPT = 8 / K heads.
template <int K, int W, bool BWD>
struct HwGeo {
  static constexpr int HPT = 8 / K;
  static constexpr int TR = BWD ? 16 : (K == 8 ? 64 : 16);
  static constexpr int RPT = TR / kNC;
  static_assert(RPT * kNC == TR, "rows per tile must split over the compute warps");
  static constexpr int ROWS_X = TR + W - 1;           // x rows t0-(W-1) .. t0+TR-1
  static constexpr int ROWS_A = BWD ? TR + W - 1 : TR;  // dy / weight rows t0 .. t0+ROWS_A-1
  static constexpr int WB_MAX = (kCB / K) * W;         // weight elements per row (hs = K at most)
  static constexpr int X_BYTES = ROWS_X * kCB * 2;
  static constexpr int DY_BYTES = BWD ? ROWS_A * kCB * 2 : 0;
  static constexpr int W_BYTES = ROWS_A * WB_MAX * 2;
  static constexpr int STAGE = ((X_BYTES + DY_BYTES + W_BYTES) + 127) / 128 * 128;
  static constexpr int S = (kSmemCap / STAGE) < 4 ? (kSmemCap / STAGE) : 4;
  static_assert(S >= 2, "stage ring too shallow");
  static constexpr int RED_BYTES = kNC * W * kCB * 4;  // dstatic_w reduction (reuses the ring)
  static_assert(!BWD || RED_BYTES <= S * STAGE, "reduction buffer must fit in the ring");
  static constexpr int SMEM = S * STAGE + 1024 + 256;  // + alignment slack + barriers
};

struct HwSplit {
  int n_dblk, n_groups, tiles_row, n_tiles;
};

// N bf16 from/to an address aligned to A bytes, in A-byte pieces.
template <int N, int A>
__device__ __forceinline__ void ld_bf16(const __nv_bfloat16* p, __nv_bfloat16 (&v)[N]) {
  static_assert((2 * N) % A == 0, "piece size");
  if constexpr (A == 16) {
#pragma unroll
    for (int i = 0; i < N / 8; ++i) reinterpret_cast<uint4*>(v)[i] = reinterpret_cast<const uint4*>(p)[i];
  } else if constexpr (A == 8) {
#pragma unroll
    for (int i = 0; i < N / 4; ++i) reinterpret_cast<uint2*>(v)[i] = reinterpret_cast<const uint2*>(p)[i];
  } else if constexpr (A == 4) {
#pragma unroll
    for (int i = 0; i < N / 2; ++i) reinterpret_cast<uint32_t*>(v)[i] = reinterpret_cast<const uint32_t*>(p)[i];
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = p[i];
  }
}

template <int N, int A>
__device__ __forceinline__ void st_bf16(__nv_bfloat16* p, const __nv_bfloat16 (&v)[N]) {
  static_assert((2 * N) % A == 0, "piece size");
  if constexpr (A == 16) {
#pragma unroll
    for (int i = 0; i < N / 8; ++i) reinterpret_cast<uint4*>(p)[i] = reinterpret_cast<const uint4*>(v)[i];
  } else if constexpr (A == 8) {
#pragma unroll
    for (int i = 0; i < N / 4; ++i) reinterpret_cast<uint2*>(p)[i] = reinterpret_cast<const uint2*>(v)[i];
  } else if constexpr (A == 4) {
#pragma unroll
    for (int i = 0; i < N / 2; ++i) reinterpret_cast<uint32_t*>(p)[i] = reinterpret_cast<const uint32_t*>(v)[i];
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) p[i] = v[i];
  }
}

constexpr int pow2_align(int bytes) { return (bytes % 16 == 0) ? 16 : (bytes % 8 == 0) ? 8 : (bytes % 4 == 0) ? 4 : 2; }

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

// Weights of the thread's heads for one row: wt[j][w] for the head of channel
// group j (j < HPT; HPT = 1 when the 8 channels share one head).
template <int K, int W>
__device__ __forceinline__ void load_row_weights(const __nv_bfloat16* wrow, int lane, int log2hs, float (&wt)[8 / K][W]) {
  constexpr int HPT = 8 / K;
  constexpr int N = HPT * W;
  __align__(16) __nv_bfloat16 v[N];
  if constexpr (K == 8) {
    const int hl = (8 * lane) >> log2hs;  // local head of the block
    ld_bf16<N, pow2_align(2 * W)>(wrow + hl * W, v);
  } else {
    ld_bf16<N, pow2_align(2 * N)>(wrow + lane * N, v);
  }
#pragma unroll
  for (int j = 0; j < HPT; ++j)
#pragma unroll
    for (int w = 0; w < W; ++w) wt[j][w] = __bfloat162float(v[j * W + w]);
}

template <int K, int W, bool BWD>
__global__ void __launch_bounds__(kHwThreads, 1)
    hw_tma_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap dymap,
                  const __grid_constant__ CUtensorMap wmap, const __nv_bfloat16* __restrict__ sw,
                  __nv_bfloat16* __restrict__ out, __nv_bfloat16* __restrict__ dw, float* __restrict__ part,
                  HwSplit sp, int T, int D, int H, int log2hs, int wb, int wchunks, int residual) {
  using G = HwGeo<K, W, BWD>;
  constexpr int HPT = G::HPT, TR = G::TR, RPT = G::RPT, S = G::S;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + S * G::STAGE);
  uint64_t* empty_bar = full_bar + S;
  volatile int* abort_flag_p = reinterpret_cast<volatile int*>(empty_bar + S);
  volatile int& abort_flag = *abort_flag_p;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dblk = blockIdx.x, g = blockIdx.y;
  const int d0 = dblk * kCB;
  const int j0 = (int)((int64_t)g * sp.n_tiles / sp.n_groups);
  const int j1 = (int)((int64_t)(g + 1) * sp.n_tiles / sp.n_groups);
  const int n = j1 - j0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kNC);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kNC) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tensormap(&xmap);
      prefetch_tensormap(&wmap);
      if constexpr (BWD) prefetch_tensormap(&dymap);
      const uint64_t pol = policy_evict_normal();
      const uint32_t bytes = G::X_BYTES + G::DY_BYTES + G::ROWS_A * wb * 2;
      for (int k = 0; k < n; ++k) {
        const int s = k % S;
        if (!mbar_wait(&empty_bar[s], ((k / S) & 1) ^ 1, kErrWaitProducer, &abort_flag)) break;
        const int tile = j0 + k, b = tile / sp.tiles_row, t0 = (tile % sp.tiles_row) * TR;
        uint8_t* st = smem + s * G::STAGE;
        mbar_arrive_expect_tx(&full_bar[s], bytes);
        tma_load_3d(st, &xmap, &full_bar[s], d0, t0 - (W - 1), b, pol);
        if constexpr (BWD) tma_load_3d(st + G::X_BYTES, &dymap, &full_bar[s], d0, t0, b, pol);
        uint8_t* wdst = st + G::X_BYTES + G::DY_BYTES;
        if (wchunks == 0) tma_load_3d(wdst, &wmap, &full_bar[s], dblk * wb, t0, b, pol);
        else tma_load_4d(wdst, &wmap, &full_bar[s], 0, dblk * wchunks, t0, b, pol);
      }
    }
    return;
  }

  // -------------------------------------------------------------- compute
  const int dch = d0 + 8 * lane;
  const bool dok = dch < D;
  const int r0 = warp * RPT;
  float s_w[W][8];
#pragma unroll
  for (int w = 0; w < W; ++w) {
    if (sw != nullptr && dok) {
      unpack8(*reinterpret_cast<const uint4*>(sw + (size_t)w * D + dch), s_w[w]);
    } else {
#pragma unroll
      for (int c = 0; c < 8; ++c) s_w[w][c] = 0.f;
    }
  }
  float acc_sw[BWD ? W : 1][8];
#pragma unroll
  for (int w = 0; w < (BWD ? W : 1); ++w)
#pragma unroll
    for (int c = 0; c < 8; ++c) acc_sw[w][c] = 0.f;

  bool dead = false;
  for (int k = 0; k < n; ++k) {
    const int s = k % S;
    if (!mbar_wait(&full_bar[s], (k / S) & 1, kErrWaitEpilogue, &abort_flag)) {
      dead = true;
      break;
    }
    const int tile = j0 + k, b = tile / sp.tiles_row, t0 = (tile % sp.tiles_row) * TR;
    const uint8_t* st = smem + s * G::STAGE;
    const __nv_bfloat16* xs = reinterpret_cast<const __nv_bfloat16*>(st) + 8 * lane;
    const __nv_bfloat16* ws = reinterpret_cast<const __nv_bfloat16*>(st + G::X_BYTES + G::DY_BYTES);

    if constexpr (!BWD) {
      // x rows r0 .. r0+RPT+W-2 of the tile (step t0 - (W-1) + i)
      float xr[RPT + W - 1][8];
#pragma unroll
      for (int i = 0; i < RPT + W - 1; ++i) unpack8(*reinterpret_cast<const uint4*>(xs + (r0 + i) * kCB), xr[i]);
#pragma unroll
      for (int rr = 0; rr < RPT; ++rr) {
        const int t = t0 + r0 + rr;
        float wt[HPT][W];
        load_row_weights<K, W>(ws + (r0 + rr) * wb, lane, log2hs, wt);
        float y[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          float v = residual ? xr[rr + W - 1][c] : 0.f;
#pragma unroll
          for (int w = 0; w < W; ++w) v = fmaf(wt[c / K][w] + s_w[w][c], xr[rr + W - 1 - w][c], v);
          y[c] = v;
        }
        if (dok && t < T) *reinterpret_cast<uint4*>(out + ((size_t)b * T + t) * D + dch) = pack8(y);
      }
    } else {
      const __nv_bfloat16* dys = reinterpret_cast<const __nv_bfloat16*>(st + G::X_BYTES) + 8 * lane;
      // dy rows r0 .. r0+RPT+W-2 (step t0 + i); x rows r0 .. r0+RPT+W-2 (step t0 - (W-1) + i),
      // kept packed (bf16) and unpacked where used
      uint4 dyp[RPT + W - 1], xp[RPT + W - 1];
#pragma unroll
      for (int i = 0; i < RPT + W - 1; ++i) {
        dyp[i] = *reinterpret_cast<const uint4*>(dys + (r0 + i) * kCB);
        xp[i] = *reinterpret_cast<const uint4*>(xs + (r0 + i) * kCB);
      }
      // dx[t] = sum_w (weight[t+w, h, w] + static_w[w]) * dy[t+w]  (+ dy[t]).  Weight row
      // j (step t0 + r0 + j) is read once and feeds dx rows j - w.
      float dxv[RPT][8];
#pragma unroll
      for (int rr = 0; rr < RPT; ++rr) {
        if (residual) unpack8(dyp[rr], dxv[rr]);
        else {
#pragma unroll
          for (int c = 0; c < 8; ++c) dxv[rr][c] = 0.f;
        }
      }
#pragma unroll
      for (int j = 0; j < RPT + W - 1; ++j) {
        float wt[HPT][W], dyf[8];
        load_row_weights<K, W>(ws + (r0 + j) * wb, lane, log2hs, wt);
        unpack8(dyp[j], dyf);
#pragma unroll
        for (int w = 0; w < W; ++w) {
          const int rr = j - w;
          if (rr >= 0 && rr < RPT) {
#pragma unroll
            for (int c = 0; c < 8; ++c) dxv[rr][c] = fmaf(wt[c / K][w] + s_w[w][c], dyf[c], dxv[rr][c]);
          }
        }
      }
#pragma unroll
      for (int rr = 0; rr < RPT; ++rr) {
        const int t = t0 + r0 + rr;
        // P_w = dy[t] * x[t-w]: dweight (per head) and dstatic_w (per channel)
        float pw[W][8], dyf[8];
        unpack8(dyp[rr], dyf);
#pragma unroll
        for (int w = 0; w < W; ++w) {
          float xf[8];
          unpack8(xp[rr + W - 1 - w], xf);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            pw[w][c] = dyf[c] * xf[c];
            acc_sw[w][c] += pw[w][c];
          }
        }
        const bool row_ok = t < T;
        if (dok && row_ok) *reinterpret_cast<uint4*>(out + ((size_t)b * T + t) * D + dch) = pack8(dxv[rr]);
        if constexpr (K == 8) {
          float hsum[W];
#pragma unroll
          for (int w = 0; w < W; ++w) {
            float v = 0.f;
#pragma unroll
            for (int c = 0; c < 8; ++c) v += pw[w][c];
            hsum[w] = v;
          }
          const int gl = 1 << (log2hs - 3);  // lanes per head
          for (int o = 1; o < gl; o <<= 1)
#pragma unroll
            for (int w = 0; w < W; ++w) hsum[w] += __shfl_xor_sync(0xffffffffu, hsum[w], o);
          if (dok && row_ok && (lane & (gl - 1)) == 0) {
            __align__(16) __nv_bfloat16 v[W];
#pragma unroll
            for (int w = 0; w < W; ++w) v[w] = __float2bfloat16_rn(hsum[w]);
            const int h = dch >> log2hs;
            st_bf16<W, pow2_align(2 * W)>(dw + (((size_t)b * T + t) * H + h) * W, v);
          }
        } else {
          __align__(16) __nv_bfloat16 v[HPT * W];
#pragma unroll
          for (int j = 0; j < HPT; ++j)
#pragma unroll
            for (int w = 0; w < W; ++w) {
              float a = 0.f;
#pragma unroll
              for (int c = 0; c < K; ++c) a += pw[w][j * K + c];
              v[j * W + w] = __float2bfloat16_rn(a);
            }
          if (dok && row_ok) {
            const int h0 = dch / K;
            st_bf16<HPT * W, pow2_align(2 * HPT * W)>(dw + (((size_t)b * T + t) * H + h0) * W, v);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[s]);
  }

  if constexpr (BWD) {
    if (part != nullptr) {
      // Fixed-order sum of the compute warps' dstatic_w partials, one row per CTA.
      // Every TMA load into the ring has completed (each was waited on above,
      // or the CTA is aborting), so the ring is free to reuse.
      named_bar_sync(1, kNC * 32);
      float* red = reinterpret_cast<float*>(smem);  // [kNC][W][kCB]
#pragma unroll
      for (int w = 0; w < W; ++w)
#pragma unroll
        for (int c = 0; c < 8; ++c) red[(warp * W + w) * kCB + 8 * lane + c] = acc_sw[w][c];
      named_bar_sync(1, kNC * 32);
      for (int i = threadIdx.x; i < W * kCB; i += kNC * 32) {
        const int w = i / kCB, c = i % kCB;
        float v = 0.f;
        for (int q = 0; q < kNC; ++q) v += red[(q * W + w) * kCB + c];
        if (d0 + c < D) part[((size_t)g * W + w) * D + d0 + c] = v;
      }
    }
  }
  (void)dead;
}

HwSplit hw_split(int64_t B, int64_t T, int64_t D, int TR) {
  HwSplit sp;
  sp.n_dblk = (int)((D + kCB - 1) / kCB);
  sp.tiles_row = (int)((T + TR - 1) / TR);
  sp.n_tiles = (int)(B * sp.tiles_row);
  int g = sm_count() / sp.n_dblk;
  if (g < 1) g = 1;
  if (g > sp.n_tiles) g = sp.n_tiles;
  sp.n_groups = g;
  return sp;
}

int hw_tr(int K, bool bwd) { return bwd ? 16 : (K == 8 ? 64 : 16); }

template <int K, int W, bool BWD>
int launch_hw_tma(const void* x, const void* wgt, const void* sw, const void* dy, void* out, void* dw, float* part,
                  int64_t B, int64_t T, int64_t D, int64_t H, int log2hs, int residual, cudaStream_t st) {
  using G = HwGeo<K, W, BWD>;
  const HwSplit sp = hw_split(B, T, D, G::TR);
  const int hs = 1 << log2hs;
  const int wb = (kCB / hs) * W;  // weight elements per tile row (hs <= 256)
  const int64_t HW = H * W;
  CUtensorMap xmap, dymap, wmap;
  int s;
  {
    const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)T, (cuuint64_t)B};
    const cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)T * D * 2};
    const cuuint32_t box_x[3] = {kCB, (cuuint32_t)G::ROWS_X, 1};
    if ((s = encode_tensor_map_bf16(&xmap, x, 3, dims, strides, box_x))) return s;
    if constexpr (BWD) {
      const cuuint32_t box_a[3] = {kCB, (cuuint32_t)G::ROWS_A, 1};
      if ((s = encode_tensor_map_bf16(&dymap, dy, 3, dims, strides, box_a))) return s;
    } else {
      dymap = xmap;  // unused
    }
  }
  int wchunks = 0;
  if (wb <= 256) {
    const cuuint64_t dims[3] = {(cuuint64_t)HW, (cuuint64_t)T, (cuuint64_t)B};
    const cuuint64_t strides[2] = {(cuuint64_t)HW * 2, (cuuint64_t)T * HW * 2};
    const cuuint32_t box[3] = {(cuuint32_t)wb, (cuuint32_t)G::ROWS_A, 1};
    if ((s = encode_tensor_map_bf16(&wmap, wgt, 3, dims, strides, box))) return s;
  } else {
    wchunks = wb / 256;
    const cuuint64_t dims[4] = {256, (cuuint64_t)(HW / 256), (cuuint64_t)T, (cuuint64_t)B};
    const cuuint64_t strides[3] = {512, (cuuint64_t)HW * 2, (cuuint64_t)T * HW * 2};
    const cuuint32_t box[4] = {256, (cuuint32_t)wchunks, (cuuint32_t)G::ROWS_A, 1};
    if ((s = encode_tensor_map_bf16(&wmap, wgt, 4, dims, strides, box))) return s;
  }
  auto kern = hw_tma_kernel<K, W, BWD>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return cuda_status(e, "cudaFuncSetAttribute(hw_tma_kernel)");
  }
  dim3 grid(sp.n_dblk, sp.n_groups);
  kern<<<grid, kHwThreads, G::SMEM, st>>>(xmap, dymap, wmap, (const __nv_bfloat16*)sw, (__nv_bfloat16*)out,
                                          (__nv_bfloat16*)dw, part, sp, (int)T, (int)D, (int)H, log2hs, wb, wchunks,
                                          residual);
  DYNCONV_CHECK_LAUNCH(BWD ? "hw_tma_kernel(bwd)" : "hw_tma_kernel(fwd)");
  return DYNCONV_OK;
}

template <bool BWD>
int hw_tma_dispatch(const void* x, const void* wgt, const void* sw, const void* dy, void* out, void* dw, float* part,
                    int64_t B, int64_t T, int64_t D, int64_t H, int W, int log2hs, int residual, cudaStream_t st) {
  const int K = log2hs >= 3 ? 8 : (1 << log2hs);
#define DYNCONV_HWT(KK, WW)                                                                                       \
  if (K == KK && W == WW)                                                                                         \
    return launch_hw_tma<KK, WW, BWD>(x, wgt, sw, dy, out, dw, part, B, T, D, H, log2hs, residual, st);
  DYNCONV_HWT(1, 1) DYNCONV_HWT(1, 2) DYNCONV_HWT(1, 3) DYNCONV_HWT(1, 4)
  DYNCONV_HWT(2, 1) DYNCONV_HWT(2, 2) DYNCONV_HWT(2, 3) DYNCONV_HWT(2, 4)
  DYNCONV_HWT(4, 1) DYNCONV_HWT(4, 2) DYNCONV_HWT(4, 3) DYNCONV_HWT(4, 4)
  DYNCONV_HWT(8, 1) DYNCONV_HWT(8, 2) DYNCONV_HWT(8, 3) DYNCONV_HWT(8, 4)
#undef DYNCONV_HWT
  return set_error(DYNCONV_ERR_UNSUPPORTED, "headwise TMA path: head_size %d, W %d", 1 << log2hs, W);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

// Envelope of the TMA path: bf16, W <= 4, D % 8 == 0, head_size <= 256, a tile
// row of weights ((256 / head_size) * W elements) a multiple of 16 bytes (and of
// 256 elements, with H*W too, when it exceeds one 256-element TMA box), 16-byte
// aligned tensors.  Everything else runs the register-ring kernels of headwise.cu.
bool hw_tma_supported(int64_t D, int64_t H, int W, int log2hs, int dtype, const void* const* ptrs, int nptrs) {
  if (dtype != DYNCONV_DTYPE_BF16 || W < 1 || W > 4 || D % 8 != 0 || log2hs > 8) return false;
  const int64_t wb = (int64_t)(kCB >> log2hs) * W;
  const int64_t HW = H * W;
  if (wb % 8 != 0 || HW % 8 != 0) return false;
  if (wb > 256 && (wb % 256 != 0 || HW % 256 != 0)) return false;
  for (int i = 0; i < nptrs; ++i)
    if (ptrs[i] && !aligned16(ptrs[i])) return false;
  return true;
}

int hw_tma_partial_rows(int64_t B, int64_t T, int64_t D, int log2hs) {
  return hw_split(B, T, D, hw_tr(log2hs >= 3 ? 8 : 1, true)).n_groups;
}

int hw_tma_fwd_launch(const void* x, const void* w, const void* sw, void* y, int64_t B, int64_t T, int64_t D, int64_t H,
                      int W, int log2hs, int residual, cudaStream_t st) {
  return hw_tma_dispatch<false>(x, w, sw, nullptr, y, nullptr, nullptr, B, T, D, H, W, log2hs, residual, st);
}

int hw_tma_bwd_launch(const void* x, const void* w, const void* sw, const void* dy, void* dx, void* dw, float* part,
                      int64_t B, int64_t T, int64_t D, int64_t H, int W, int log2hs, int residual, cudaStream_t st) {
  return hw_tma_dispatch<true>(x, w, sw, dy, dx, dw, part, B, T, D, H, W, log2hs, residual, st);
}

}  // namespace dynconv
