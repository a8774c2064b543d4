// headwise_tma.cu -- headwise dynamic short convolution, bf16, TMA-staged
// persistent kernels (forward and backward).
//
// Reference behaviour: headwise.py:24-91 (forward kernel) and headwise.py:105-215
// (backward kernel) of OliverSieberling/dynamic-conv1d; oracle reference.py:5-20.
//
// Both directions stream HBM (no contraction worth a tensor core).  A tile is
// 128 channels x TR timesteps of one batch row; a CTA keeps one 128-channel block
// for a contiguous range of tiles (grid = n_dblk x n_groups, two CTAs per SM):
//
//   warp NC (producer, one lane): TMA loads of the tile's x rows (with the W-1
//       look-behind rows; zero fill for t < 0 and t >= T), and for the backward the
//       dy and weight rows with their W-1 look-ahead rows, into an S-stage ring
//       (full / empty mbarriers, every wait bounded);
//   warps 0..NC-1 (compute): lane l owns the 8-byte vector of channels 4l..4l+3,
//       warp c owns rows c*RPT .. c*RPT+RPT-1 of the tile; every operand comes from
//       shared memory, outputs go straight to HBM as 8-byte stores (a warp writes
//       256 contiguous bytes per row).  Four channels per lane keep the per-thread
//       state (static_w, the dstatic_w sums, the row window) small enough for two
//       CTAs -- sixteen compute warps -- per SM.
//
// Backward reductions:
//   dweight[b,t,h,w] = sum_{d in head h} dy[b,t,d] x[b,t-w,d]: in-thread over the
//       thread's channels of the head, then xor shuffles over the hs/4 lanes of a
//       head (hs >= 4); no shared memory, no atomics;
//   dstatic_w[w,d] = sum_{b,t} dy x_shift: per-thread fp32 sums over all of the
//       CTA's tiles (its channel block is fixed), a fixed-order sum over the NC
//       compute warps in shared memory at the end, one fp32 partial row per CTA,
//       then the fixed-order second pass reduce_partials (reduce.cu).  The
//       reference accumulates with fp32 atomics (headwise.py:157).
#include "common.cuh"

namespace dynconv {

DYNCONV_DEFINE_ERROR_ACCESSOR(hw_tma_error_word)

namespace {

constexpr int kVec = 4;            // channels per lane (one 8-byte vector)
constexpr int kCB = 32 * kVec;     // channels per tile
constexpr int kNC = 8;             // compute warps
constexpr int kHwThreads = 32 * (kNC + 1);
constexpr int kCtasPerSm = 2;
constexpr int kSmemCap = 100 * 1024;  // per CTA (two per SM)

// Per-instantiation geometry.  K = min(head_size, kVec): a thread's kVec channels
// span HPT = kVec / K heads.
template <int K, int W, bool BWD>
struct HwGeo {
  static constexpr int HPT = kVec / K;
  static constexpr int TR = K == kVec ? (BWD ? 32 : 64) : 16;
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

using VecT = uint2;  // kVec bf16
static_assert(sizeof(VecT) == 2 * kVec, "vector type");

__device__ __forceinline__ void unpackv2(const VecT& u, float2 (&f)[kVec / 2]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < kVec / 2; ++i) f[i] = __bfloat1622float2(h[i]);
}

__device__ __forceinline__ VecT packv2(const float2 (&f)[kVec / 2]) {
  VecT u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < kVec / 2; ++i) h[i] = __floats2bfloat162_rn(f[i].x, f[i].y);
  return u;
}

// Lane-to-channel maps.  Default: lane l owns channels 4l..4l+3 of the 128-channel
// block (one 8-byte vector).  SPLIT (head_size 1 only): lane l owns channels
// 2l, 2l+1, 64+2l, 65+2l, so that its heads' weights (2 heads x W taps per pair)
// sit at a 16-byte lane stride in shared memory -- the 32-byte stride of the
// default map makes those reads 2-way bank-conflicted.
template <bool SPLIT>
__device__ __forceinline__ int lane_ch(int lane, int c) {
  return SPLIT ? ((c >> 1) * 64 + 2 * lane + (c & 1)) : (kVec * lane + c);
}

// The lane's kVec channels of one row (row = first channel of the block).
template <bool SPLIT>
__device__ __forceinline__ VecT ld_lane(const __nv_bfloat16* row, int lane) {
  if constexpr (SPLIT) {
    VecT v;
    v.x = *reinterpret_cast<const uint32_t*>(row + 2 * lane);
    v.y = *reinterpret_cast<const uint32_t*>(row + 64 + 2 * lane);
    return v;
  } else {
    return *reinterpret_cast<const VecT*>(row + kVec * lane);
  }
}

template <bool SPLIT>
__device__ __forceinline__ void st_lane(__nv_bfloat16* row, int lane, VecT v) {
  if constexpr (SPLIT) {
    *reinterpret_cast<uint32_t*>(row + 2 * lane) = v.x;
    *reinterpret_cast<uint32_t*>(row + 64 + 2 * lane) = v.y;
  } else {
    *reinterpret_cast<VecT*>(row + kVec * lane) = v;
  }
}

// dweight of one head and row: v[w] holds this lane's partial over its channels;
// the 2^LG lanes of the head (consecutive, aligned) sum them and write the W taps
// to dst (row_ok: this lane's row and channels are inside the tensor).  For W = 4
// and W = 2 the first levels are a reduce-scatter (each lane keeps half of the
// taps and sends the other half), so a head of 8 lanes costs 4 shuffles instead
// of 12; every lane writes the taps it ends up owning.  LG is a compile-time
// constant, so the whole butterfly is straight-line code.
template <int W, int LG>
__device__ __forceinline__ void head_reduce_store(float (&v)[W], int lane, bool row_ok, __nv_bfloat16* dst) {
  constexpr unsigned kAll = 0xffffffffu;
  constexpr int G = 1 << LG;  // lanes per head
  if constexpr (W == 4 && LG >= 1) {
    // level 1 (lanes l, l^1): the odd lane keeps taps 2,3, the even lane taps 0,1
    const bool up1 = lane & 1;
    float k0 = up1 ? v[2] : v[0], k1 = up1 ? v[3] : v[1];
    const float s0 = up1 ? v[0] : v[2], s1 = up1 ? v[1] : v[3];
    k0 += __shfl_xor_sync(kAll, s0, 1);
    k1 += __shfl_xor_sync(kAll, s1, 1);
    if constexpr (LG == 1) {
      if (row_ok) *reinterpret_cast<__nv_bfloat162*>(dst + (up1 ? 2 : 0)) = __floats2bfloat162_rn(k0, k1);
    } else {
      // level 2 (lanes l, l^2): keep one tap
      const bool up2 = lane & 2;
      float k = up2 ? k1 : k0;
      k += __shfl_xor_sync(kAll, up2 ? k0 : k1, 2);
#pragma unroll
      for (int o = 4; o < G; o <<= 1) k += __shfl_xor_sync(kAll, k, o);
      if (row_ok && (lane & (G - 1)) < 4) dst[(up1 ? 2 : 0) + (up2 ? 1 : 0)] = __float2bfloat16_rn(k);
    }
  } else if constexpr (W == 2 && LG >= 1) {
    const bool up1 = lane & 1;
    float k = up1 ? v[1] : v[0];
    k += __shfl_xor_sync(kAll, up1 ? v[0] : v[1], 1);
#pragma unroll
    for (int o = 2; o < G; o <<= 1) k += __shfl_xor_sync(kAll, k, o);
    if (row_ok && (lane & (G - 1)) < 2) dst[up1 ? 1 : 0] = __float2bfloat16_rn(k);
  } else {
#pragma unroll
    for (int o = 1; o < G; o <<= 1)
#pragma unroll
      for (int w = 0; w < W; ++w) v[w] += __shfl_xor_sync(kAll, v[w], o);
    if (row_ok && (lane & (G - 1)) == 0) {
      __align__(8) __nv_bfloat16 o[W];
#pragma unroll
      for (int w = 0; w < W; ++w) o[w] = __float2bfloat16_rn(v[w]);
      st_bf16<W, pow2_align(2 * W)>(dst, o);
    }
  }
}

// Weights of the thread's heads for one row: wt[j][w] for the head of channel
// group j (j < HPT; HPT = 1 when the lane's channels share one head).
template <int K, int W, bool SPLIT>
__device__ __forceinline__ void load_row_weights(const __nv_bfloat16* wrow, int lane, int log2hs,
                                                 float (&wt)[kVec / K][W]) {
  constexpr int HPT = kVec / K;
  constexpr int N = HPT * W;
  __align__(16) __nv_bfloat16 v[N];
  if constexpr (SPLIT) {  // K == 1: heads 2l, 2l+1 and 64+2l, 65+2l
    __nv_bfloat16(&lo)[2 * W] = *reinterpret_cast<__nv_bfloat16(*)[2 * W]>(v);
    __nv_bfloat16(&hi)[2 * W] = *reinterpret_cast<__nv_bfloat16(*)[2 * W]>(v + 2 * W);
    ld_bf16<2 * W, pow2_align(4 * W)>(wrow + 2 * lane * W, lo);
    ld_bf16<2 * W, pow2_align(4 * W)>(wrow + (64 + 2 * lane) * W, hi);
  } else if constexpr (K == kVec) {
    const int hl = (kVec * lane) >> log2hs;  // local head of the block
    ld_bf16<N, pow2_align(2 * W)>(wrow + hl * W, v);
  } else {
    ld_bf16<N, pow2_align(2 * N)>(wrow + lane * N, v);
  }
#pragma unroll
  for (int j = 0; j < HPT; ++j)
#pragma unroll
    for (int w = 0; w < W; ++w) wt[j][w] = __bfloat162float(v[j * W + w]);
}

template <int K, int W, bool BWD, bool SPLIT, int LG>
__global__ void __launch_bounds__(kHwThreads, kCtasPerSm)
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
      int b = j0 / sp.tiles_row, t0 = (j0 % sp.tiles_row) * TR;
      for (int k = 0; k < n; ++k, t0 += TR) {
        if (t0 >= T) {
          t0 = 0;
          ++b;
        }
        const int s = k % S;
        if (!mbar_wait(&empty_bar[s], ((k / S) & 1) ^ 1, kErrWaitProducer, &abort_flag)) break;
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
  // Channel pairs (c = 2p, 2p+1) are computed with packed fp32 instructions
  // (fma/add/mul .rn.f32x2): each lane of a pair rounds exactly like the scalar op.
  constexpr int P = kVec / 2;
  const int dch = d0 + lane_ch<SPLIT>(lane, 0);  // first channel of the lane (SPLIT: D % 128 == 0)
  const bool dok = dch < D;
  const int r0 = warp * RPT;
  float2 s2[W][P];
#pragma unroll
  for (int w = 0; w < W; ++w) {
    if (sw != nullptr && dok) {
      unpackv2(ld_lane<SPLIT>(sw + (size_t)w * D + d0, lane), s2[w]);
    } else {
#pragma unroll
      for (int q = 0; q < P; ++q) s2[w][q] = make_float2(0.f, 0.f);
    }
  }
  float2 acc_sw[BWD ? W : 1][P];
#pragma unroll
  for (int w = 0; w < (BWD ? W : 1); ++w)
#pragma unroll
    for (int q = 0; q < P; ++q) acc_sw[w][q] = make_float2(0.f, 0.f);

  // (b, t0) of the current tile, advanced incrementally
  int b = j0 / sp.tiles_row, t0 = (j0 % sp.tiles_row) * TR;
  bool dead = false;
  for (int k = 0; k < n; ++k) {
    const int s = k % S;
    if (!mbar_wait(&full_bar[s], (k / S) & 1, kErrWaitEpilogue, &abort_flag)) {
      dead = true;
      break;
    }
    const uint8_t* st = smem + s * G::STAGE;
    const __nv_bfloat16* xs = reinterpret_cast<const __nv_bfloat16*>(st);
    const __nv_bfloat16* ws = reinterpret_cast<const __nv_bfloat16*>(st + G::X_BYTES + G::DY_BYTES);

    if constexpr (!BWD) {
      // x rows r0 .. r0+RPT+W-2 of the tile (step t0 - (W-1) + i)
      float2 xr[RPT + W - 1][P];
#pragma unroll
      for (int i = 0; i < RPT + W - 1; ++i) unpackv2(ld_lane<SPLIT>(xs + (r0 + i) * kCB, lane), xr[i]);
#pragma unroll
      for (int rr = 0; rr < RPT; ++rr) {
        const int t = t0 + r0 + rr;
        float wt[HPT][W];
        load_row_weights<K, W, SPLIT>(ws + (r0 + rr) * wb, lane, log2hs, wt);
        float2 y[P];
#pragma unroll
        for (int q = 0; q < P; ++q) {
          y[q] = residual ? xr[rr + W - 1][q] : make_float2(0.f, 0.f);
#pragma unroll
          for (int w = 0; w < W; ++w) {
            const float2 coef = add2(make_float2(wt[(2 * q) / K][w], wt[(2 * q + 1) / K][w]), s2[w][q]);
            y[q] = fma2(coef, xr[rr + W - 1 - w][q], y[q]);
          }
        }
        if (dok && t < T) st_lane<SPLIT>(out + ((size_t)b * T + t) * D + d0, lane, packv2(y));
      }
    } else {
      const __nv_bfloat16* dys = reinterpret_cast<const __nv_bfloat16*>(st + G::X_BYTES);
      if constexpr (K == kVec) {
        // One pass over the warp's input rows i = 0 .. RPT+W-2 (dy and weight row r0 + i,
        // step t0 + r0 + i), every row loaded once:
        //   dx[t] = sum_w (weight[t+w, h, w] + static_w[w]) * dy[t+w]  (+ dy[t]): input row
        //       i adds its tap-w term to the pending dx row i - w (a ring of W rows, row rr
        //       in slot rr % W); row i - (W-1) is then complete and stored;
        //   P_w = dy[t] * x[t-w] for output row i (i < RPT): dstatic_w sums (per channel)
        //       and dweight (summed over the head's channels), with x from a ring of the
        //       last W x rows (x row r0 + k in slot k % W).
        // Every sum sees its terms in the order of the per-row loop below (residual, then
        // taps w = 0 .. W-1; rows in order), so both paths round alike.
        float2 dxa[W][P], xw[W][P];
#pragma unroll
        for (int k2 = 0; k2 < W - 1; ++k2) unpackv2(ld_lane<SPLIT>(xs + (r0 + k2) * kCB, lane), xw[k2 % W]);
#pragma unroll
        for (int i = 0; i < RPT + W - 1; ++i) {
          float2 dyr[P];
          unpackv2(ld_lane<SPLIT>(dys + (r0 + i) * kCB, lane), dyr);
          float wt[HPT][W];
          load_row_weights<K, W, SPLIT>(ws + (r0 + i) * wb, lane, log2hs, wt);
          if (i < RPT) {
#pragma unroll
            for (int q = 0; q < P; ++q) dxa[i % W][q] = residual ? dyr[q] : make_float2(0.f, 0.f);
          }
#pragma unroll
          for (int w = 0; w < W; ++w) {
            const int rr = i - w;
            if (rr >= 0 && rr < RPT) {
#pragma unroll
              for (int q = 0; q < P; ++q) {
                const float2 coef = add2(make_float2(wt[0][w], wt[0][w]), s2[w][q]);
                dxa[rr % W][q] = fma2(coef, dyr[q], dxa[rr % W][q]);
              }
            }
          }
          if (i >= W - 1 && i - (W - 1) < RPT) {
            const int t = t0 + r0 + i - (W - 1);
            if (dok && t < T) st_lane<SPLIT>(out + ((size_t)b * T + t) * D + d0, lane, packv2(dxa[(i - (W - 1)) % W]));
          }
          if (i < RPT) {
            const int t = t0 + r0 + i;
            const bool row_ok = dok && t < T;
            // x row r0 + i + W - 1 (step t) joins the ring; x[t - w] is in slot (i + W - 1 - w) % W
            unpackv2(ld_lane<SPLIT>(xs + (r0 + i + W - 1) * kCB, lane), xw[(i + W - 1) % W]);
#pragma unroll
            for (int w = 0; w < W; ++w)
#pragma unroll
              for (int q = 0; q < P; ++q) acc_sw[w][q] = fma2(dyr[q], xw[(i + W - 1 - w) % W][q], acc_sw[w][q]);
            // one head per lane: sum the lane's channels, then over the hs/4 lanes of the head
            float hsum[W];
#pragma unroll
            for (int w = 0; w < W; ++w) {
              const float2(&xr)[P] = xw[(i + W - 1 - w) % W];
              float2 a = mul2(dyr[0], xr[0]);
#pragma unroll
              for (int q = 1; q < P; ++q) a = fma2(dyr[q], xr[q], a);
              hsum[w] = a.x + a.y;
            }
            head_reduce_store<W, LG>(hsum, lane, row_ok, dw + (((size_t)b * T + t) * H + (dch >> log2hs)) * W);
          }
        }
      } else {
        // head_size 1 or 2 (several heads per lane, 16-row tiles): every row of the warp's
        // window in registers, then a per-row loop.
        // dy rows r0 .. r0+RPT+W-2 (step t0 + i); x rows r0 .. r0+RPT+W-2 (step t0 - (W-1) + i)
        float2 dyf[RPT + W - 1][P], xf[RPT + W - 1][P];
#pragma unroll
        for (int i = 0; i < RPT + W - 1; ++i) {
          unpackv2(ld_lane<SPLIT>(dys + (r0 + i) * kCB, lane), dyf[i]);
          unpackv2(ld_lane<SPLIT>(xs + (r0 + i) * kCB, lane), xf[i]);
        }
        // dx[t] = sum_w (weight[t+w, h, w] + static_w[w]) * dy[t+w]  (+ dy[t]).  Weight row
        // j (step t0 + r0 + j) is read once and feeds dx rows j - w.
        float2 dxv[RPT][P];
#pragma unroll
        for (int rr = 0; rr < RPT; ++rr)
#pragma unroll
          for (int q = 0; q < P; ++q) dxv[rr][q] = residual ? dyf[rr][q] : make_float2(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < RPT + W - 1; ++j) {
          float wt[HPT][W];
          load_row_weights<K, W, SPLIT>(ws + (r0 + j) * wb, lane, log2hs, wt);
#pragma unroll
          for (int w = 0; w < W; ++w) {
            const int rr = j - w;
            if (rr >= 0 && rr < RPT) {
#pragma unroll
              for (int q = 0; q < P; ++q) {
                const float2 coef = add2(make_float2(wt[(2 * q) / K][w], wt[(2 * q + 1) / K][w]), s2[w][q]);
                dxv[rr][q] = fma2(coef, dyf[j][q], dxv[rr][q]);
              }
            }
          }
        }
#pragma unroll
        for (int rr = 0; rr < RPT; ++rr) {
          const int t = t0 + r0 + rr;
          const bool row_ok = dok && t < T;
          if (row_ok) st_lane<SPLIT>(out + ((size_t)b * T + t) * D + d0, lane, packv2(dxv[rr]));
          // P_w = dy[t] * x[t-w]: dstatic_w (per channel, fused multiply-add) and
          // dweight (HPT heads per lane, K channels each)
#pragma unroll
          for (int w = 0; w < W; ++w)
#pragma unroll
            for (int q = 0; q < P; ++q) acc_sw[w][q] = fma2(dyf[rr][q], xf[rr + W - 1 - w][q], acc_sw[w][q]);
          __align__(16) __nv_bfloat16 v[HPT * W];
#pragma unroll
          for (int w = 0; w < W; ++w)
#pragma unroll
            for (int q = 0; q < P; ++q) {
              const float2 pr = mul2(dyf[rr][q], xf[rr + W - 1 - w][q]);
              if constexpr (K == 1) {
                v[(2 * q) * W + w] = __float2bfloat16_rn(pr.x);
                v[(2 * q + 1) * W + w] = __float2bfloat16_rn(pr.y);
              } else {
                v[q * W + w] = __float2bfloat16_rn(pr.x + pr.y);
              }
            }
          if (row_ok) {
            __nv_bfloat16* drow = dw + ((size_t)b * T + t) * H * W;
            if constexpr (SPLIT) {
              __nv_bfloat16(&lo)[2 * W] = *reinterpret_cast<__nv_bfloat16(*)[2 * W]>(v);
              __nv_bfloat16(&hi)[2 * W] = *reinterpret_cast<__nv_bfloat16(*)[2 * W]>(v + 2 * W);
              st_bf16<2 * W, pow2_align(4 * W)>(drow + (size_t)(d0 + 2 * lane) * W, lo);
              st_bf16<2 * W, pow2_align(4 * W)>(drow + (size_t)(d0 + 64 + 2 * lane) * W, hi);
            } else {
              st_bf16<HPT * W, pow2_align(2 * HPT * W)>(drow + (size_t)(dch / K) * W, v);
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[s]);
    t0 += TR;
    if (t0 >= T) {
      t0 = 0;
      ++b;
    }
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
        for (int q = 0; q < P; ++q) {
          red[(warp * W + w) * kCB + lane_ch<SPLIT>(lane, 2 * q)] = acc_sw[w][q].x;
          red[(warp * W + w) * kCB + lane_ch<SPLIT>(lane, 2 * q + 1)] = acc_sw[w][q].y;
        }
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
  int g = kCtasPerSm * sm_count() / sp.n_dblk;
  if (g < 1) g = 1;
  if (g > sp.n_tiles) g = sp.n_tiles;
  sp.n_groups = g;
  return sp;
}

int hw_tr(int K, bool bwd) { return K == kVec ? (bwd ? 32 : 64) : 16; }

template <int K, int W, bool BWD, bool SPLIT, int LG>
int launch_hw_tma(const void* x, const void* wgt, const void* sw, const void* dy, void* out, void* dw, float* part,
                  int64_t B, int64_t T, int64_t D, int64_t H, int log2hs, int residual, cudaStream_t st) {
  using G = HwGeo<K, W, BWD>;
  const HwSplit sp = hw_split(B, T, D, G::TR);
  const int hs = 1 << log2hs;
  const int wb = (kCB / hs) * W;  // weight elements per tile row (hs <= kCB)
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
    // rows wider than one 256-element box: 128-element chunks as a 4-D box
    wchunks = wb / 128;
    const cuuint64_t dims[4] = {128, (cuuint64_t)(HW / 128), (cuuint64_t)T, (cuuint64_t)B};
    const cuuint64_t strides[3] = {256, (cuuint64_t)HW * 2, (cuuint64_t)T * HW * 2};
    const cuuint32_t box[4] = {128, (cuuint32_t)wchunks, (cuuint32_t)G::ROWS_A, 1};
    if ((s = encode_tensor_map_bf16(&wmap, wgt, 4, dims, strides, box))) return s;
  }
  auto kern = hw_tma_kernel<K, W, BWD, SPLIT, LG>;
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

// Backward with head_size >= kVec: lanes per head 2^LG = head_size / kVec as a
// compile-time constant (head_size 4..128).
template <int W, bool BWD>
int launch_hw_tma_lg(const void* x, const void* wgt, const void* sw, const void* dy, void* out, void* dw, float* part,
                     int64_t B, int64_t T, int64_t D, int64_t H, int log2hs, int residual, cudaStream_t st) {
  switch (log2hs - 2) {
    case 0: return launch_hw_tma<kVec, W, BWD, false, 0>(x, wgt, sw, dy, out, dw, part, B, T, D, H, log2hs, residual, st);
    case 1: return launch_hw_tma<kVec, W, BWD, false, 1>(x, wgt, sw, dy, out, dw, part, B, T, D, H, log2hs, residual, st);
    case 2: return launch_hw_tma<kVec, W, BWD, false, 2>(x, wgt, sw, dy, out, dw, part, B, T, D, H, log2hs, residual, st);
    case 3: return launch_hw_tma<kVec, W, BWD, false, 3>(x, wgt, sw, dy, out, dw, part, B, T, D, H, log2hs, residual, st);
    case 4: return launch_hw_tma<kVec, W, BWD, false, 4>(x, wgt, sw, dy, out, dw, part, B, T, D, H, log2hs, residual, st);
    case 5: return launch_hw_tma<kVec, W, BWD, false, 5>(x, wgt, sw, dy, out, dw, part, B, T, D, H, log2hs, residual, st);
    default: return set_error(DYNCONV_ERR_UNSUPPORTED, "headwise TMA path: head_size %d", 1 << log2hs);
  }
}

template <bool BWD>
int hw_tma_dispatch(const void* x, const void* wgt, const void* sw, const void* dy, void* out, void* dw, float* part,
                    int64_t B, int64_t T, int64_t D, int64_t H, int W, int log2hs, int residual, cudaStream_t st) {
  const int K = log2hs >= 2 ? 4 : (1 << log2hs);
#define DYNCONV_HWT(KK, WW)                                                                                       \
  if (K == KK && W == WW) {                                                                                       \
    if (KK == 1 && D % kCB == 0)                                                                                  \
      return launch_hw_tma<KK, WW, BWD, KK == 1, 0>(x, wgt, sw, dy, out, dw, part, B, T, D, H, log2hs, residual, st); \
    if (KK == kVec && BWD) return launch_hw_tma_lg<WW, BWD>(x, wgt, sw, dy, out, dw, part, B, T, D, H, log2hs,     \
                                                             residual, st);                                        \
    return launch_hw_tma<KK, WW, BWD, false, 0>(x, wgt, sw, dy, out, dw, part, B, T, D, H, log2hs, residual, st);  \
  }
  DYNCONV_HWT(1, 1) DYNCONV_HWT(1, 2) DYNCONV_HWT(1, 3) DYNCONV_HWT(1, 4)
  DYNCONV_HWT(2, 1) DYNCONV_HWT(2, 2) DYNCONV_HWT(2, 3) DYNCONV_HWT(2, 4)
  DYNCONV_HWT(4, 1) DYNCONV_HWT(4, 2) DYNCONV_HWT(4, 3) DYNCONV_HWT(4, 4)
#undef DYNCONV_HWT
  return set_error(DYNCONV_ERR_UNSUPPORTED, "headwise TMA path: head_size %d, W %d", 1 << log2hs, W);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

// Envelope of the TMA path: bf16, W <= 4, D % 8 == 0, head_size <= 128, a tile
// row of weights ((128 / head_size) * W elements) a multiple of 16 bytes (and of
// 128 elements, with H*W too, when it exceeds one 256-element TMA box), 16-byte
// aligned tensors.  Everything else runs the register-ring kernels of headwise.cu.
bool hw_tma_supported(int64_t D, int64_t H, int W, int log2hs, int dtype, const void* const* ptrs, int nptrs) {
  if (dtype != DYNCONV_DTYPE_BF16 || W < 1 || W > 4 || D % 8 != 0 || log2hs > 7) return false;
  const int64_t wb = (int64_t)(kCB >> log2hs) * W;
  const int64_t HW = H * W;
  if (wb % 8 != 0 || HW % 8 != 0) return false;
  if (wb > 256 && (wb % 128 != 0 || HW % 128 != 0)) return false;
  for (int i = 0; i < nptrs; ++i)
    if (ptrs[i] && !aligned16(ptrs[i])) return false;
  return true;
}

int hw_tma_partial_rows(int64_t B, int64_t T, int64_t D, int log2hs) {
  return hw_split(B, T, D, hw_tr(log2hs >= 2 ? kVec : 1, true)).n_groups;
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
