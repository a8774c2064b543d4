// lowrank_tc.cu -- tcgen05 (5th-generation tensor core) lowrank kernels, bf16.
//
// Reference behaviour: lowrank.py:24-67 (forward kernel, Triton tl.dot with
// K = R_kernel), lowrank.py:214-249 (static-rank fold + launch); oracle
// reference.py:23-39.
//
// Forward data flow per work item (128 channels x 64 timesteps of one batch row):
//
//   HBM x  --TMA (3-D box, zero fill for t<0 / t>=T)--> smem x tile [67 rows][128 ch]
//   HBM z_pack --TMA (4-D box)--> smem z tile, already in the K-major MMA layout
//        (z_pack = z_ext as [R_kernel/8][B][T][8] bf16 with the static rank = 1.0,
//         written once per call by z_pack_kernel; z rows are 2R bytes, which TMA
//         cannot tile directly when R is odd)
//   smem U (per 128-channel block, static_w folded as rank R)   [K-major, per tap]
//   tcgen05.mma (M = 128 channels, N = 64 timesteps, K = R_kernel) per tap w
//        -> TMEM acc_w[ch][t] = sum_r U[r,w,ch] z[t,r]      (the dynamic weights;
//                                                            never written to HBM)
//   epilogue warps: y[t,ch] = sum_w acc_w[ch][t] * x[t-w,ch] (+ x[t,ch])
//        -> per-warp smem y sub-tile [16 steps][32 ch] -> TMA store issued by the warp
//
// Warp roles (576 threads, one CTA per SM, persistent over a contiguous range
// of work items):  warp 0 producer, warp 1 TMEM owner + MMA issuer (one lane),
// warps 2..17 epilogue (four warps per TMEM lane quarter, one per 16-step quarter
// of the tile).
// Pipelines: S-stage x/z ring (full/empty mbarriers), double-buffered TMEM
// accumulators (acc_full via tcgen05.commit / acc_empty), a double-buffered y
// sub-tile per epilogue warp (the warp's own TMA store bulk groups), so the
// epilogue warps never synchronise with one another.  Every mbarrier wait is
// bounded (common.cuh).
#include <mutex>

#include "common.cuh"

namespace dynconv {

DYNCONV_DEFINE_ERROR_ACCESSOR(lr_tc_error_word)

int reduce_partials_launch(const float* part, int P, int64_t n, float* out_f32, void* out, int dtype, cudaStream_t st);
int cast_f32_launch(const float* src, void* dst, int64_t n, int dtype, cudaStream_t st);

namespace {

constexpr int kBT = 64;         // timesteps per work item (MMA N)
constexpr int kBD = 128;        // channels per work item (MMA M)
constexpr int kStages = 4;      // x/z pipeline depth (forward, R_kernel <= 32)
constexpr int kEpiWarps = 16;   // forward epilogue warps: four per TMEM lane quarter
constexpr int kEpiSteps = kBT / (kEpiWarps / 4);  // timesteps per epilogue warp and tile
constexpr int kFwdThreads = 64 + 32 * kEpiWarps;


// --------------------------------------------------------------- tensor maps

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 3-D bf16 map over a [B][T][D] tensor: dims (D, T, B), box (box_d, box_t, 1).
int make_btd_map(CUtensorMap* map, const void* base, int64_t B, int64_t T, int64_t D, int box_d, int box_t) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(DYNCONV_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (int s = ensure_context()) return s;
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)T * D * 2};
  cuuint32_t box[3] = {(cuuint32_t)box_d, (cuuint32_t)box_t, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(DYNCONV_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return DYNCONV_OK;
}

// 4-D bf16 map over z_pack [RKP/8][B][T][8]: dims (8, T, B, RKP/8), box (8, rows, 1, RKP/8).
// The box lands in shared memory as [RKP/8][rows][8]: the no-swizzle K-major layout
// (16-byte rows, 8-rank chunks `rows * 16` bytes apart).  Rows past T read as zero.
int make_zpack_map(CUtensorMap* map, const void* base, int64_t B, int64_t T, int rkp, int rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(DYNCONV_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (int s = ensure_context()) return s;
  cuuint64_t dims[4] = {8, (cuuint64_t)T, (cuuint64_t)B, (cuuint64_t)(rkp / 8)};
  cuuint64_t strides[3] = {16, (cuuint64_t)T * 16, (cuuint64_t)B * T * 16};
  cuuint32_t box[4] = {8, (cuuint32_t)rows, 1, (cuuint32_t)(rkp / 8)};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(DYNCONV_ERR_CUDA, "cuTensorMapEncodeTiled(z_pack) failed (%d)", (int)r);
  return DYNCONV_OK;
}

// z_pack[c][b][t][e] = z_ext[b, t, 8c + e]: z for ranks < R, 1.0 at rank R when the
// static filter is fused (the reference's F.pad(z, (0, 1), value=1.0),
// lowrank.py:224), 0 up to RKP.  One thread per (8-rank chunk, token): consecutive
// threads write consecutive 16-byte chunks.
__global__ void __launch_bounds__(256) z_pack_kernel(const __nv_bfloat16* __restrict__ z,
                                                     __nv_bfloat16* __restrict__ zp, int64_t ntok, int R, int rkp,
                                                     int has_static) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= ntok * (rkp / 8)) return;
  const int c = (int)(i / ntok);
  const int64_t tok = i - (int64_t)c * ntok;
  const __nv_bfloat16* zr = z + tok * R;
  __align__(16) __nv_bfloat16 v[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int r = 8 * c + e;
    v[e] = r < R ? zr[r] : __float2bfloat16_rn((r == R && has_static) ? 1.f : 0.f);
  }
  *reinterpret_cast<uint4*>(zp + i * 8) = *reinterpret_cast<const uint4*>(v);
}

size_t zpack_bytes(int64_t B, int64_t T, int rkp) { return ((size_t)B * T * rkp * 2 + 255) / 256 * 256; }

int z_pack_launch(const void* z, void* zp, int64_t B, int64_t T, int R, int rkp, bool has_static, cudaStream_t st) {
  const int64_t ntok = B * T;
  const int64_t nthreads = ntok * (rkp / 8);
  z_pack_kernel<<<(unsigned)((nthreads + 255) / 256), 256, 0, st>>>((const __nv_bfloat16*)z, (__nv_bfloat16*)zp,
                                                                   ntok, R, rkp, has_static ? 1 : 0);
  DYNCONV_CHECK_LAUNCH("z_pack_kernel");
  return DYNCONV_OK;
}

// ------------------------------------------------------------- work split
//
// CTA (dblk, g) of a grid of n_dblk x n_groups owns channel block dblk (128
// channels) for the contiguous range of 64-step tiles [j0, j1) of group g, tiles
// numbered b * tiles_row + t0 / 64.  A fixed channel block per CTA means the U
// block is loaded once, and the CTAs of one tile (one per channel block) run in
// step -- which the backward's cross-CTA dz reduction relies on.
struct TileSplit {
  int n_dblk, n_groups, tiles_row, n_tiles;
};

TileSplit tile_split(int64_t B, int64_t T, int64_t D) {
  TileSplit sp;
  sp.n_dblk = (int)((D + kBD - 1) / kBD);
  sp.tiles_row = (int)((T + kBT - 1) / kBT);
  sp.n_tiles = (int)(B * sp.tiles_row);
  int ng = sm_count() / sp.n_dblk;
  if (ng < 1) ng = 1;
  if (ng > sp.n_tiles) ng = sp.n_tiles;
  sp.n_groups = ng;
  return sp;
}

// ------------------------------------------------------------- smem layout

template <int W, int RKP>
struct FwdSmem {
  static constexpr int kS = RKP <= 32 ? kStages : 3;  // pipeline depth (shared memory bound)
  static constexpr int kXRows = kBT + W - 1;
  static constexpr uint32_t kXBytes = (uint32_t)kXRows * kBD * 2;        // TMA box bytes
  static constexpr uint32_t kXStride = (kXBytes + 1023u) / 1024u * 1024u;
  static constexpr uint32_t kZBytes = (uint32_t)kBT * RKP * 2;           // K-major, 64 rows x RKP
  static constexpr uint32_t kYWarpBytes = kEpiSteps * 32 * 2;  // one epilogue warp's y sub-tile [steps][32 ch]
  static constexpr uint32_t kUTap = (uint32_t)kBD * RKP * 2;
  static constexpr uint32_t kOffX = 0;
  static constexpr uint32_t kOffZ = kOffX + kS * kXStride;
  static constexpr uint32_t kOffY = kOffZ + kS * kZBytes;  // [kEpiWarps][2 buffers][kYWarpBytes]
  static constexpr uint32_t kOffU = kOffY + kEpiWarps * 2 * kYWarpBytes;
  static constexpr uint32_t kTotal = kOffU + W * kUTap + 1024;  // + alignment slack
  // K-major operand strides
  static constexpr uint32_t kZLbo = kBT * 16;          // next 8-rank chunk of z
  static constexpr uint32_t kZSbo = 128;               // next 8 timesteps
  static constexpr uint32_t kULbo = 128;               // next 8-rank chunk of U
  static constexpr uint32_t kUSbo = (RKP / 8) * 128;   // next 8 channels
};

// Loads U_ext for channel block dblk into smem: one [128 ch x RKP] K-major block per
// tap (rank R = static_w when present, zero padding up to RKP).  The NT calling
// threads each read up to ceil(W*RKP*16 / NT) 16-byte vectors (8 channels of one
// (rank, tap) row; D % 8 == 0 on this path, so a vector never straddles the end
// of D), all loads issued before any store so their latencies overlap.
template <int W, int RKP, int NT>
__device__ void load_u_block(uint8_t* us, const __nv_bfloat16* __restrict__ U, const __nv_bfloat16* __restrict__ sw,
                             int dblk, int D, int R, int tid) {
  constexpr uint32_t kUTap = (uint32_t)kBD * RKP * 2;
  constexpr uint32_t kUSbo = (RKP / 8) * 128;
  constexpr int NV = W * RKP * (kBD / 8);
  constexpr int PER = (NV + NT - 1) / NT;
  const int d0 = dblk * kBD;
  uint4 u[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = tid + i * NT;
    u[i] = make_uint4(0, 0, 0, 0);
    if (e < NV) {
      const int v8 = e % (kBD / 8);  // 8-channel group
      const int r = (e / (kBD / 8)) % RKP;
      const int w = e / ((kBD / 8) * RKP);
      const int d = d0 + v8 * 8;
      if (d < D) {
        if (r < R) u[i] = __ldg(reinterpret_cast<const uint4*>(U + ((size_t)r * W + w) * D + d));
        else if (r == R && sw != nullptr) u[i] = __ldg(reinterpret_cast<const uint4*>(sw + (size_t)w * D + d));
      }
    }
  }
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = tid + i * NT;
    if (e < NV) {
      const int v8 = e % (kBD / 8);
      const int r = (e / (kBD / 8)) % RKP;
      const int w = e / ((kBD / 8) * RKP);
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u[i]);
#pragma unroll
      for (int k = 0; k < 8; ++k)
        *reinterpret_cast<__nv_bfloat16*>(us + w * kUTap + kmajor_off(v8 * 8 + k, r, kUSbo, 128)) = h[k];
    }
  }
}

// ------------------------------------------------------------- forward kernel

template <int W, int RKP>
__global__ void __launch_bounds__(kFwdThreads, 1)
    lr_fwd_tc_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap ymap,
                     const __grid_constant__ CUtensorMap zmap, const __nv_bfloat16* __restrict__ U,
                     const __nv_bfloat16* __restrict__ sw, TileSplit sp, int T, int D, int R, int residual) {
  using L = FwdSmem<W, RKP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  constexpr int S = L::kS;
  __shared__ uint64_t full_bar[S], empty_bar[S], accf_bar[2], acce_bar[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dblk = blockIdx.x % sp.n_dblk;
  const int g = blockIdx.x / sp.n_dblk;
  const int j0 = (int)((int64_t)sp.n_tiles * g / sp.n_groups);
  const int n = (int)((int64_t)sp.n_tiles * (g + 1) / sp.n_groups) - j0;
  const int d0 = dblk * kBD;
  constexpr uint32_t kAccCols = W * kBT;
  constexpr uint32_t kTmemCols = (2 * kAccCols <= 256) ? 256 : 512;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);  // one arrive.expect_tx; the x and z TMA loads complete the bytes
      mbar_init(&empty_bar[s], kEpiWarps);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf_bar[a], 1);
      mbar_init(&acce_bar[a], kEpiWarps);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&xmap);
    prefetch_tensormap(&ymap);
    prefetch_tensormap(&zmap);
  }
  __syncthreads();  // barriers initialised: the producer starts its loads at once
  uint32_t tmem = 0;
  if (warp != 0) {
    // U block of this CTA's channels (MMA A operand), loaded once by all but the
    // producer, then the TMEM allocation.
    constexpr int kNonProducer = kFwdThreads - 32;
    load_u_block<W, RKP, kNonProducer>(smem + L::kOffU, U, sw, dblk, D, R, threadIdx.x - 32);
    fence_proxy_async_smem();
    if (warp == 1) {
      tmem_alloc(&tmem_slot, kTmemCols);
      tmem_relinquish();
    }
    tc_fence_before();
    named_bar_sync(2, kNonProducer);
    tc_fence_after();
    tmem = tmem_slot;
  }

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      for (int k = 0; k < n; ++k) {
        const int s = k % S;
        if (!mbar_wait(&empty_bar[s], ((k / S) & 1) ^ 1, kErrWaitProducer, &abort_flag)) break;
        const int tile = j0 + k, b = tile / sp.tiles_row, t0 = (tile % sp.tiles_row) * kBT;
        mbar_arrive_expect_tx(&full_bar[s], L::kXBytes + L::kZBytes);
        tma_load_3d(smem + L::kOffX + s * L::kXStride, &xmap, &full_bar[s], d0, t0 - (W - 1), b, pol);
        tma_load_4d(smem + L::kOffZ + s * L::kZBytes, &zmap, &full_bar[s], 0, t0, b, 0, pol);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc = make_idesc_bf16(kBD, kBT, 0, 0);
    uint8_t* us = smem + L::kOffU;
    for (int k = 0; k < n; ++k) {
      const int s = k % S, a = k & 1;
      if (!mbar_wait(&full_bar[s], (k / S) & 1, kErrWaitMma, &abort_flag)) break;
      if (!mbar_wait(&acce_bar[a], ((k >> 1) & 1) ^ 1, kErrWaitMma, &abort_flag)) break;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t zb = smem_u32(smem + L::kOffZ + s * L::kZBytes);
        const uint32_t ub = smem_u32(us);
#pragma unroll
        for (int w = 0; w < W; ++w) {
#pragma unroll
          for (int ks = 0; ks < RKP / 16; ++ks) {
            const uint64_t ad = make_smem_desc(ub + w * L::kUTap + ks * 2 * L::kULbo, L::kULbo, L::kUSbo);
            const uint64_t bd = make_smem_desc(zb + ks * 2 * L::kZLbo, L::kZLbo, L::kZSbo);
            umma_f16(tmem + a * kAccCols + w * kBT, ad, bd, idesc, ks > 0 ? 1u : 0u);
          }
        }
        umma_commit(&accf_bar[a]);
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int e = warp - 2;            // 0..kEpiWarps-1
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int part = e >> 2;           // which kEpiSteps-step part of the tile
    const int ch = q * 32 + lane;      // channel within the block (= TMEM lane)
    const uint64_t pol_y = policy_evict_first();
    bool dead = false;  // a bounded wait gave up: skip the work, keep arriving
    for (int k = 0; k < n; ++k) {
      const int s = k % S, a = k & 1;
      const int tile = j0 + k, b = tile / sp.tiles_row, t0 = (tile % sp.tiles_row) * kBT;
      // this warp's y buffer (k & 1) is free once its store of item k-2 has read it
      if (lane == 0 && !dead) bulk_wait_group_read<1>();
      __syncwarp();
      if (!dead) dead = !mbar_wait(&full_bar[s], (k / S) & 1, kErrWaitEpilogue, &abort_flag);
      if (!dead) dead = !mbar_wait(&accf_bar[a], (k >> 1) & 1, kErrWaitEpilogue, &abort_flag);
      tc_fence_after();
      __nv_bfloat16* ys = reinterpret_cast<__nv_bfloat16*>(smem + L::kOffY + (e * 2 + a) * L::kYWarpBytes);
      if (!dead) {
        const __nv_bfloat16* xs = reinterpret_cast<const __nv_bfloat16*>(smem + L::kOffX + s * L::kXStride);
        // x window: xr[j] = x at step (tok0 - (W-1) + j); smem row of step t is (t - t0) + (W-1)
        float xr[16 + W - 1];
        const int tok0 = part * kEpiSteps;
#pragma unroll
        for (int j = 0; j < W - 1; ++j) xr[j] = __bfloat162float(xs[(tok0 + j) * kBD + ch]);
#pragma unroll
        for (int c = 0; c < kEpiSteps / 16; ++c) {
          const int tb = tok0 + c * 16;
          float acc[W][16];
#pragma unroll
          for (int w = 0; w < W; ++w)
            tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + a * kAccCols + w * kBT + tb, acc[w]);
#pragma unroll
          for (int j = 0; j < 16; ++j) xr[W - 1 + j] = __bfloat162float(xs[(tb + j + W - 1) * kBD + ch]);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float yv = 0.f;
#pragma unroll
            for (int w = 0; w < W; ++w) yv = fmaf(acc[w][j], xr[W - 1 + j - w], yv);
            if (residual) yv += xr[W - 1 + j];
            ys[(c * 16 + j) * 32 + lane] = __float2bfloat16_rn(yv);
          }
#pragma unroll
          for (int j = 0; j < W - 1; ++j) xr[j] = xr[16 + j];
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&acce_bar[a]);
        mbar_arrive(&empty_bar[s]);
        if (!dead) {
          tma_store_3d(&ymap, ys, d0 + q * 32, t0 + part * kEpiSteps, b, pol_y);
          bulk_commit_group();
        }
      }
    }
    if (lane == 0) bulk_wait_group<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

template <int W, int RKP>
int launch_fwd(const void* x, const void* z, const void* U, const void* sw, void* y, void* ws, int64_t B, int64_t T,
               int64_t D, int R, int residual, cudaStream_t st) {
  using L = FwdSmem<W, RKP>;
  static_assert(L::kTotal <= 232448 - 512, "forward shared memory budget (227 KB per CTA)");
  CUtensorMap xmap, ymap, zmap;
  int s;
  if ((s = make_btd_map(&xmap, x, B, T, D, kBD, kBT + W - 1))) return s;
  if ((s = make_btd_map(&ymap, y, B, T, D, 32, kEpiSteps))) return s;  // per-warp [steps][32 ch] stores
  if ((s = make_zpack_map(&zmap, ws, B, T, RKP, kBT))) return s;
  if ((s = z_pack_launch(z, ws, B, T, R, RKP, sw != nullptr, st))) return s;
  const TileSplit sp = tile_split(B, T, D);
  const int grid = sp.n_dblk * sp.n_groups;
  const int smem = (int)L::kTotal;
  cudaError_t e = cudaFuncSetAttribute(lr_fwd_tc_kernel<W, RKP>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) {
    cudaGetLastError();  // do not leave the failure pending for the next launch check
    return cuda_status(e, "cudaFuncSetAttribute(lr_fwd_tc)");
  }
  lr_fwd_tc_kernel<W, RKP><<<grid, kFwdThreads, smem, st>>>(xmap, ymap, zmap, (const __nv_bfloat16*)U,
                                                            (const __nv_bfloat16*)sw, sp, (int)T, (int)D, R, residual);
  DYNCONV_CHECK_LAUNCH("lr_fwd_tc_kernel");
  return DYNCONV_OK;
}

template <int RKP>
int launch_fwd_w(int W, const void* x, const void* z, const void* U, const void* sw, void* y, void* ws, int64_t B,
                 int64_t T, int64_t D, int R, int residual, cudaStream_t st) {
  switch (W) {
    case 1: return launch_fwd<1, RKP>(x, z, U, sw, y, ws, B, T, D, R, residual, st);
    case 2: return launch_fwd<2, RKP>(x, z, U, sw, y, ws, B, T, D, R, residual, st);
    case 3: return launch_fwd<3, RKP>(x, z, U, sw, y, ws, B, T, D, R, residual, st);
    case 4: return launch_fwd<4, RKP>(x, z, U, sw, y, ws, B, T, D, R, residual, st);
    default: return set_error(DYNCONV_ERR_UNSUPPORTED, "tensor-core path: W=%d", W);
  }
}


// ============================================================== backward
//
// One fused pass over dy and x per work item (128 channels x 64 timesteps):
//
//   MMA-1  acc1_w[ch][t] = sum_r U[r,w,ch] z[t+w,r]    M=128 ch, N=32 t (two halves), K=R_kernel
//          A = U^T held in TMEM for the whole kernel; B = the z tile read from row w
//          (the no-swizzle K-major layout is linear in rows).
//   epilogue: dx[t,ch] = sum_w acc1_w[ch][t] dy[t+w,ch] (+ dy)   -> HBM (bf16)
//             P_w[t,ch] = bf16(dy[t,ch] x[t-w,ch])   (rounded to bf16 as the reference
//             does before its dots, lowrank.py:128) -> smem, and transposed -> TMEM
//   MMA-2  dU_w[ch][r] += sum_t P_w[t,ch] z[t,r]       M=128 ch, N=R_kernel, K=64 t
//          A = P^T from TMEM (R_kernel <= 16; else from smem), B = z (MN-major view);
//          accumulated in TMEM over all items of the CTA, one partial block per CTA;
//          after a grid-wide count (cooperative launch) every CTA sums a slice of the
//          partials in group order and writes dU_f32, dU and dstatic_w itself.
//   MMA-3  dz[t][r]     = sum_{w,ch} P_w[t,ch] U[r,w,ch] M=64 t,  N=R_kernel, K=128*W
//          A = P (smem, MN-major view), B = U (smem); partial over this CTA's 128
//          channels, written to the workspace.  After its last tile every CTA of a
//          token group publishes its partials (one fence + counter), waits for the
//          group's other channel-block CTAs (co-resident: cooperative launch) and
//          sums a 1/n_dblk slice of the group's dz in channel-block order:
//          deterministic, and the reduction work is spread evenly.
//
// Why operands live where they do: one tcgen05.mma costs about one pass of its
// shared-memory operands at ~128 B/clock (a 128x16 bf16 A operand alone is 4 KB),
// so the A operands that are either constant (U) or produced lane-per-channel by
// the epilogue (P^T) are kept in TMEM and only the small B operands are read from
// shared memory.  MMA-3 needs P with timesteps as rows, so it reads P from shared
// memory; it runs on its own issuing warp (M = 64 MMAs from two issuers overlap).
//
// Warps: 0 producer (TMA), 1 MMA-1/MMA-2 issuer + TMEM owner, 2 MMA-3 issuer,
// 3..18 epilogue (four per TMEM lane quarter, one per 8-step piece of each half).
// Grid = n_dblk x n_groups CTAs: CTA (dblk, g) owns channel block dblk for a
// contiguous range of 64-step tiles, so the CTAs sharing a tile's dz run in step
// and the dz partial working set stays small and L2-resident.

constexpr int kBwdStages = 2;
constexpr int kZRows = 72;  // z rows t0 .. t0+71 (64 + W-1 look-ahead, rounded up to whole core matrices)
constexpr int kBwdCtl = 3;       // control warps
constexpr int kBwdEpi = 16;      // epilogue warps
constexpr int kBwdPiece = 8;     // timesteps per epilogue warp and half
constexpr int kBwdThreads = 32 * (kBwdCtl + kBwdEpi);

__host__ __device__ constexpr uint32_t round1024(uint32_t v) { return (v + 1023u) / 1024u * 1024u; }

template <int W, int RKP, int NP>
struct BwdSmem {
  static constexpr int kRows = kBT + W - 1;
  static constexpr uint32_t kTileBytes = (uint32_t)kRows * kBD * 2;
  static constexpr uint32_t kTileStride = round1024(kTileBytes);
  static constexpr uint32_t kZBytes = (uint32_t)kZRows * RKP * 2;
  static constexpr uint32_t kZStride = (kZBytes + 127u) / 128u * 128u;
  static constexpr uint32_t kUTap = (uint32_t)kBD * RKP * 2;
  static constexpr uint32_t kPTap = (uint32_t)kBT * kBD * 2;
  static constexpr uint32_t kOffU = 0;
  static constexpr uint32_t kOffDy = round1024(kOffU + W * kUTap);
  static constexpr uint32_t kOffX = kOffDy + kBwdStages * kTileStride;
  static constexpr uint32_t kOffZ = kOffX + kBwdStages * kTileStride;
  static constexpr uint32_t kOffP = round1024(kOffZ + kBwdStages * kZStride);
  static constexpr uint32_t kTotal = kOffP + NP * W * kPTap + 1024;
  // no-swizzle operand strides (bytes)
  static constexpr uint32_t kUChunk = (RKP / 8) * 128;  // U: next 8 channels (K-major sbo / MN-major lbo)
  static constexpr uint32_t kZChunk = kZRows * 16;      // z: next 8 ranks
  static constexpr uint32_t kPChunk = (kBT / 8) * 128;  // P: next 8 channels
  // TMEM columns
  static constexpr bool kPT = (RKP == 16);                  // P^T for MMA-2 held in TMEM
  static constexpr uint32_t kColA1 = 0;                     // 2 halves x W taps x 32 steps
  static constexpr uint32_t kColUA = 64 * W;                // U^T: W taps x RKP/2 (bf16 pairs)
  static constexpr uint32_t kColPT = kColUA + W * RKP / 2;  // P^T: W taps x 32 (64 steps, bf16 pairs)
  static constexpr uint32_t kColDU = kColPT + (kPT ? 32 * W : 0);
  static constexpr uint32_t kColDZ = kColDU + W * RKP;      // 2 x RKP, M = 64 layout
  static constexpr uint32_t kCols = kColDZ + 2 * RKP;
  static constexpr uint32_t kAlloc = kCols <= 256 ? 256 : 512;
  static_assert(kCols <= 512, "TMEM budget");
};

template <int N>
__device__ __forceinline__ void tmem_ld_n(uint32_t taddr, float (&v)[N]) {
  static_assert(N == 4 || N == 8 || N == 16, "");
  if constexpr (N == 4) tmem_ld4(taddr, v);
  else if constexpr (N == 8) tmem_ld8(taddr, v);
  else tmem_ld16(taddr, v);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&p);
}

template <int W, int RKP, int NP>
__global__ void __launch_bounds__(kBwdThreads, 1)
    lr_bwd_tc_kernel(const __grid_constant__ CUtensorMap dymap, const __grid_constant__ CUtensorMap xmap,
                     const __grid_constant__ CUtensorMap zmap, const __nv_bfloat16* __restrict__ U,
                     const __nv_bfloat16* __restrict__ sw, __nv_bfloat16* __restrict__ dx,
                     __nv_bfloat16* __restrict__ dz, float* __restrict__ dzp, int* __restrict__ grp_done,
                     float* __restrict__ dUp, float* __restrict__ dU_f32, __nv_bfloat16* __restrict__ dU,
                     __nv_bfloat16* __restrict__ dsw, TileSplit sp, int T, int D, int R, int Rk, int residual) {
  using L = BwdSmem<W, RKP, NP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  __shared__ uint64_t full_bar[kBwdStages], empty_bar[kBwdStages], a1f_bar[2], a1e_bar[2], pf_bar[NP], pe_bar[NP],
      pte_bar, dzf_bar[2], dze_bar[2], du_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  __shared__ int grp_ok;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dblk = blockIdx.x % sp.n_dblk;
  const int g = blockIdx.x / sp.n_dblk;
  const int j0 = (int)((int64_t)sp.n_tiles * g / sp.n_groups);
  const int j1 = (int)((int64_t)sp.n_tiles * (g + 1) / sp.n_groups);
  const int n = j1 - j0;
  const int d0 = dblk * kBD;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kBwdStages; ++s) {
      mbar_init(&full_bar[s], 1);  // one arrive.expect_tx; the dy, x and z TMA loads complete the bytes
      mbar_init(&empty_bar[s], 1);
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(&a1f_bar[h], 1);
      mbar_init(&a1e_bar[h], kBwdEpi);
      mbar_init(&dzf_bar[h], 1);
      mbar_init(&dze_bar[h], kBwdEpi);
    }
    for (int p = 0; p < NP; ++p) {
      mbar_init(&pf_bar[p], kBwdEpi);
      mbar_init(&pe_bar[p], L::kPT ? 1 : 2);  // MMA-3 (and MMA-2 when it reads P from smem)
    }
    mbar_init(&pte_bar, 1);
    mbar_init(&du_bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&dymap);
    prefetch_tensormap(&xmap);
    prefetch_tensormap(&zmap);
  }
  __syncthreads();  // barriers initialised: the producer starts its loads at once
  uint32_t tmem = 0;
  if (warp != 0) {
    // Everything but the producer: U block of this CTA's channels in smem (MMA-3 B
    // operand; ranks >= R zero, rank R = static_w), TMEM allocation, then U^T in
    // TMEM (MMA-1 A operand: lane = channel, column c of tap w = ranks (2c, 2c+1),
    // which are adjacent in the K-major smem copy).
    constexpr int kNonProducer = kBwdThreads - 32;
    load_u_block<W, RKP, kNonProducer>(smem + L::kOffU, U, sw, dblk, D, R, threadIdx.x - 32);
    fence_proxy_async_smem();
    if (warp == 1) {
      tmem_alloc(&tmem_slot, L::kAlloc);
      tmem_relinquish();
    }
    tc_fence_before();
    named_bar_sync(2, kNonProducer);
    tc_fence_after();
    tmem = tmem_slot;
    if (warp >= kBwdCtl && ((warp - kBwdCtl) >> 2) == 0) {  // one warp per lane quarter
      const int q = warp & 3, ch = q * 32 + lane;
      const uint8_t* us = smem + L::kOffU;
#pragma unroll
      for (int w = 0; w < W; ++w) {
#pragma unroll
        for (int c0 = 0; c0 < RKP / 2; c0 += 8) {
          uint32_t v[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            v[i] = *reinterpret_cast<const uint32_t*>(us + w * L::kUTap + kmajor_off(ch, 2 * (c0 + i), L::kUChunk, 128));
          tmem_st8(tmem + ((uint32_t)(q * 32) << 16) + L::kColUA + w * (RKP / 2) + c0, v);
        }
      }
      tmem_st_wait();
    }
    tc_fence_before();
    named_bar_sync(2, kNonProducer);
    tc_fence_after();
  }

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // Stage k % 2 is released by the commit after the MMAs of tile k-2 that read it.
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      for (int k = 0; k < n; ++k) {
        const int s = k % kBwdStages;
        if (!mbar_wait(&empty_bar[s], ((k / kBwdStages) & 1) ^ 1, kErrWaitProducer, &abort_flag)) break;
        const int tile = j0 + k, b = tile / sp.tiles_row, t0 = (tile % sp.tiles_row) * kBT;
        mbar_arrive_expect_tx(&full_bar[s], 2 * L::kTileBytes + L::kZBytes);
        tma_load_3d(smem + L::kOffDy + s * L::kTileStride, &dymap, &full_bar[s], d0, t0, b, pol);
        tma_load_3d(smem + L::kOffX + s * L::kTileStride, &xmap, &full_bar[s], d0, t0 - (W - 1), b, pol);
        tma_load_4d(smem + L::kOffZ + s * L::kZStride, &zmap, &full_bar[s], 0, t0, b, 0, pol);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA-1 / MMA-2 issuer
    const uint32_t pb0 = smem_u32(smem + L::kOffP);
    const uint32_t idesc1 = make_idesc_bf16(kBD, 32, 0, 0);
    const uint32_t idesc2 = make_idesc_bf16(kBD, RKP, 0, 1);
    bool ok = true;
    auto mma2 = [&](int j) -> bool {
      const int p = j % NP, sj = j % kBwdStages;
      if (!mbar_wait(&pf_bar[p], (j / NP) & 1, kErrWaitMma, &abort_flag)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t zb = smem_u32(smem + L::kOffZ + sj * L::kZStride);
#pragma unroll
        for (int w = 0; w < W; ++w) {
#pragma unroll
          for (int ks = 0; ks < kBT / 16; ++ks) {  // K = timesteps
            const uint64_t bd = make_smem_desc(zb + ks * 256, 128, L::kZChunk);
            const uint32_t acc = (j == 0 && ks == 0) ? 0u : 1u;
            if constexpr (L::kPT) {
              umma_f16_ts(tmem + L::kColDU + w * RKP, tmem + L::kColPT + w * 32 + ks * 8, bd, idesc2, acc);
            } else {
              const uint64_t ad = make_smem_desc(pb0 + p * W * L::kPTap + w * L::kPTap + ks * 256, 128, L::kPChunk);
              umma_f16(tmem + L::kColDU + w * RKP, ad, bd, idesc2, acc);
            }
          }
        }
        if constexpr (L::kPT) umma_commit(&pte_bar);
        else umma_commit(&pe_bar[p]);
        umma_commit(&empty_bar[sj]);
      }
      __syncwarp();
      return true;
    };
    for (int k = 0; k < n && ok; ++k) {
      const int s = k % kBwdStages;
      if (!mbar_wait(&full_bar[s], (k / kBwdStages) & 1, kErrWaitMma, &abort_flag)) break;
      const uint32_t zb = smem_u32(smem + L::kOffZ + s * L::kZStride);
      for (int h = 0; h < 2 && ok; ++h) {
        if (!mbar_wait(&a1e_bar[h], (k & 1) ^ 1, kErrWaitMma, &abort_flag)) { ok = false; break; }
        tc_fence_after();
        if (lane == 0) {
#pragma unroll
          for (int w = 0; w < W; ++w) {
#pragma unroll
            for (int ks = 0; ks < RKP / 16; ++ks) {  // z rows from 32h + w
              const uint64_t bd = make_smem_desc(zb + (32 * h + w) * 16 + ks * 2 * L::kZChunk, L::kZChunk, 128);
              umma_f16_ts(tmem + L::kColA1 + h * 32 * W + w * 32, tmem + L::kColUA + w * (RKP / 2) + ks * 8, bd,
                          idesc1, ks > 0 ? 1u : 0u);
            }
          }
          umma_commit(&a1f_bar[h]);
        }
        __syncwarp();
      }
      if (ok && k >= 1) ok = mma2(k - 1);
    }
    if (ok && n >= 1) ok = mma2(n - 1);
    if (lane == 0) umma_commit(&du_bar);
    __syncwarp();
  } else if (warp == 2) {
    // ------------------------------------------------------------ MMA-3 issuer
    const uint32_t ub = smem_u32(smem + L::kOffU), pb0 = smem_u32(smem + L::kOffP);
    const uint32_t idesc3 = make_idesc_bf16(64, RKP, 1, 1);
    for (int j = 0; j < n; ++j) {
      const int p = j % NP;
      if (!mbar_wait(&pf_bar[p], (j / NP) & 1, kErrWaitMma, &abort_flag)) break;
      if (!mbar_wait(&dze_bar[j & 1], ((j >> 1) & 1) ^ 1, kErrWaitMma, &abort_flag)) break;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t pb = pb0 + p * W * L::kPTap;
#pragma unroll
        for (int w = 0; w < W; ++w) {
#pragma unroll
          for (int ks = 0; ks < kBD / 16; ++ks) {  // K = (tap, channel)
            const uint64_t ad = make_smem_desc(pb + w * L::kPTap + ks * 2 * L::kPChunk, L::kPChunk, 128);
            const uint64_t bd = make_smem_desc(ub + w * L::kUTap + ks * 2 * L::kUChunk, L::kUChunk, 128);
            umma_f16(tmem + L::kColDZ + (j & 1) * RKP, ad, bd, idesc3, (w == 0 && ks == 0) ? 0u : 1u);
          }
        }
        umma_commit(&dzf_bar[j & 1]);
        umma_commit(&pe_bar[p]);
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int e = warp - kBwdCtl;
    const int q = warp & 3;   // TMEM lane quarter this warp may access
    const int pp = e >> 2;    // 8-step piece of each 32-step half
    const int ch = q * 32 + lane;
    const bool dok = d0 + ch < D;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    bool dead = false;
    constexpr int PC = kBwdPiece;

    // dz partial of tile j (M = 64 layout: lanes 0..15 of quarter q hold steps 16q..16q+15;
    // the four warps of a quarter take RKP/4 columns each) -> workspace
    auto dz_readout = [&](int j) {
      const int tile = j0 + j;
      if (!dead) dead = !mbar_wait(&dzf_bar[j & 1], (j >> 1) & 1, kErrWaitEpilogue, &abort_flag);
      tc_fence_after();
      constexpr int NC = RKP / 4;
      float v[NC];
      const int c0 = pp * NC;
      if (!dead) {
        tmem_ld_n<NC>(tmem + lane_base + L::kColDZ + (j & 1) * RKP + c0, v);
        tmem_ld_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dze_bar[j & 1]);
      if (!dead && lane < 16) {
        float* dst = dzp + (((size_t)dblk * sp.n_tiles + tile) * kBT + 16 * q + lane) * RKP + c0;
#pragma unroll
        for (int i = 0; i < NC; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
      }
    };

    for (int k = 0; k < n; ++k) {
      const int s = k % kBwdStages, p = k % NP;
      const int tile = j0 + k, b = tile / sp.tiles_row, t0 = (tile % sp.tiles_row) * kBT;
      if (!dead) dead = !mbar_wait(&full_bar[s], (k / kBwdStages) & 1, kErrWaitEpilogue, &abort_flag);
      const __nv_bfloat16* dys = reinterpret_cast<const __nv_bfloat16*>(smem + L::kOffDy + s * L::kTileStride);
      const __nv_bfloat16* xs = reinterpret_cast<const __nv_bfloat16*>(smem + L::kOffX + s * L::kTileStride);
      uint8_t* pbuf = smem + L::kOffP + p * W * L::kPTap;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (!dead) dead = !mbar_wait(&a1f_bar[h], k & 1, kErrWaitEpilogue, &abort_flag);
        tc_fence_after();
        if (!dead) {
          const int tb = 32 * h + PC * pp;
          float acc[W][PC];
#pragma unroll
          for (int w = 0; w < W; ++w) tmem_ld_n<PC>(tmem + lane_base + L::kColA1 + h * 32 * W + w * 32 + PC * pp, acc[w]);
          float dyr[PC + W - 1], xr[PC + W - 1];
#pragma unroll
          for (int j = 0; j < PC + W - 1; ++j) {
            dyr[j] = __bfloat162float(dys[(tb + j) * kBD + ch]);  // dy at step tb + j
            xr[j] = __bfloat162float(xs[(tb + j) * kBD + ch]);    // x at step tb - (W-1) + j
          }
          tmem_ld_wait();
          __nv_bfloat16* dxc = dx + ((size_t)b * T + t0 + tb) * D + d0 + ch;
#pragma unroll
          for (int j = 0; j < PC; ++j) {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < W; ++w) v = fmaf(acc[w][j], dyr[j + w], v);
            if (residual) v += dyr[j];
            if (dok && t0 + tb + j < T) dxc[(size_t)j * D] = __float2bfloat16_rn(v);
          }
          // P^T in TMEM is single-buffered: wait for the MMA-2 of the previous tile
          if (L::kPT && h == 0) dead = !mbar_wait(&pte_bar, (k & 1) ^ 1, kErrWaitEpilogue, &abort_flag);
          // the P buffer is needed from the first P store on (with one buffer, the
          // previous tile's MMA-2/3 overlap this tile's first dx half)
          if (!dead && h == 0) dead = !mbar_wait(&pe_bar[p], ((k / NP) & 1) ^ 1, kErrWaitEpilogue, &abort_flag);
          if (!dead) {
#pragma unroll
            for (int w = 0; w < W; ++w) {
              uint32_t pk[PC / 2];
#pragma unroll
              for (int i = 0; i < PC / 2; ++i)
                pk[i] = pack_bf16x2(dyr[2 * i] * xr[2 * i + W - 1 - w], dyr[2 * i + 1] * xr[2 * i + W - w]);
              *reinterpret_cast<uint4*>(pbuf + w * L::kPTap + kmajor_off(ch, tb, L::kPChunk, 128)) =
                  make_uint4(pk[0], pk[1], pk[2], pk[3]);
              if constexpr (L::kPT) tmem_st4(tmem + lane_base + L::kColPT + w * 32 + tb / 2, pk);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a1e_bar[h]);
      }
      fence_proxy_async_smem();
      if constexpr (L::kPT) tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pf_bar[p]);
      if (k >= 1) dz_readout(k - 1);
    }
    if (n >= 1) dz_readout(n - 1);
    // dU partial of this CTA: TMEM (lane = channel) -> dUp[g][r][w*D + d0 + ch]
    if (!dead) dead = !mbar_wait(&du_bar, 0, kErrWaitTail, &abort_flag);
    tc_fence_after();
    if (!dead) {
      // the four warps of a lane quarter split the W * RKP / 16 column chunks
      for (int cidx = pp; cidx < W * (RKP / 16); cidx += 4) {
        const int w = cidx / (RKP / 16), rc = cidx % (RKP / 16);
        float v[16];
        tmem_ld16(tmem + lane_base + L::kColDU + w * RKP + rc * 16, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int r = rc * 16 + i;
          if (r < Rk && dok) dUp[((size_t)g * Rk + r) * W * D + (size_t)w * D + d0 + ch] = v[i];
        }
      }
    }
  }

  // ---------------------------------------------------------------- dz reduction
  // Publish this CTA's dz partials (CTA barrier, then one cumulative gpu-scope
  // fence), wait for the other channel-block CTAs of the group, then sum this
  // CTA's 1/n_dblk slice of the group's (step, rank) pairs in channel-block order.
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(&grp_done[g], 1);
    atomicAdd(&grp_done[sp.n_groups], 1);  // grid-wide count, waited on before the dU reduction
    bool ok = !abort_flag;
    if (ok) {
      const volatile int* gd = grp_done + g;
      const uint64_t tstart = globaltimer_ns();
      while (*gd < sp.n_dblk) {
        if (globaltimer_ns() - tstart > kWaitLimitNs) {
          atomicCAS(&g_device_error, 0u, (unsigned)kErrWaitTail);
          ok = false;
          break;
        }
      }
    }
    __threadfence();
    grp_ok = ok ? 1 : 0;
  }
  __syncthreads();
  if (grp_ok) {
    const int64_t nsteps = (int64_t)n * kBT;
    const int64_t lo = nsteps * dblk / sp.n_dblk, hi = nsteps * (dblk + 1) / sp.n_dblk;
    constexpr int RQ = RKP / 4;  // float4 groups per step
    for (int64_t e2 = lo * RQ + threadIdx.x; e2 < hi * RQ; e2 += blockDim.x) {
      const int64_t st = e2 / RQ;
      const int rq = (int)(e2 % RQ);
      const int tile = j0 + (int)(st / kBT), tok = (int)(st % kBT);
      const int b = tile / sp.tiles_row, t = (tile % sp.tiles_row) * kBT + tok;
      float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 16
      for (int k2 = 0; k2 < sp.n_dblk; ++k2) {  // all partial loads in flight, summed in order
        const float4 f =
            __ldcg(reinterpret_cast<const float4*>(dzp + (((size_t)k2 * sp.n_tiles + tile) * kBT + tok) * RKP) + rq);
        a4.x += f.x;
        a4.y += f.y;
        a4.z += f.z;
        a4.w += f.w;
      }
      if (t < T) {
        __nv_bfloat16* dst = dz + ((size_t)b * T + t) * R;
        const float av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (4 * rq + i < R) dst[4 * rq + i] = __float2bfloat16_rn(av[i]);
      }
    }
  }

  // ---------------------------------------------------------------- dU reduction
  // Every CTA published its dU partial with the counts above; once the whole grid
  // has (cooperative launch: all CTAs are resident), CTA i sums its 1/grid slice of
  // the [Rk][W*D] accumulator over the groups in group order (deterministic) and
  // writes dU_f32, and the bf16 dU rows / dstatic_w row when they are requested.
  __syncthreads();
  if (threadIdx.x == 0) {
    bool ok = grp_ok != 0;
    if (ok) {
      const volatile int* gd = grp_done + sp.n_groups;
      const uint64_t tstart = globaltimer_ns();
      while (*gd < (int)gridDim.x) {
        if (globaltimer_ns() - tstart > kWaitLimitNs) {
          atomicCAS(&g_device_error, 0u, (unsigned)kErrWaitTail);
          ok = false;
          break;
        }
      }
    }
    __threadfence();
    grp_ok = ok ? 1 : 0;
  }
  __syncthreads();
  if (grp_ok) {
    const int64_t wd = (int64_t)W * D;
    const int64_t n4 = (int64_t)Rk * wd / 4;  // W*D % 4 == 0 (D % 8 == 0)
    const int64_t lo = n4 * blockIdx.x / gridDim.x, hi = n4 * (blockIdx.x + 1) / gridDim.x;
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
      float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
      for (int gg = 0; gg < sp.n_groups; ++gg) {
        const float4 f = __ldcg(reinterpret_cast<const float4*>(dUp) + (size_t)gg * n4 + i);
        a4.x += f.x;
        a4.y += f.y;
        a4.z += f.z;
        a4.w += f.w;
      }
      reinterpret_cast<float4*>(dU_f32)[i] = a4;
      const int64_t e0 = 4 * i;
      const int r = (int)(e0 / wd);
      __nv_bfloat16* dst = r < R ? (dU ? dU + e0 : nullptr) : (dsw ? dsw + (e0 - (int64_t)R * wd) : nullptr);
      if (dst) {
        dst[0] = __float2bfloat16_rn(a4.x);
        dst[1] = __float2bfloat16_rn(a4.y);
        dst[2] = __float2bfloat16_rn(a4.z);
        dst[3] = __float2bfloat16_rn(a4.w);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, L::kAlloc);
}

struct BwdWorkspace {
  float* dzp;
  int* cnt;
  float* dUp;
  void* zp;
  size_t bytes;
};

static size_t al256(size_t v) { return (v + 255) / 256 * 256; }

BwdWorkspace bwd_workspace(void* base, int64_t B, int64_t T, int64_t D, int Rk, int W) {
  const TileSplit sp = tile_split(B, T, D);
  const int rkp = Rk <= 16 ? 16 : 32;
  BwdWorkspace w;
  const size_t dzp = al256((size_t)sp.n_dblk * sp.n_tiles * kBT * rkp * sizeof(float));
  const size_t cnt = al256((size_t)(sp.n_groups + 1) * sizeof(int));  // group counts + grid count
  const size_t dUp = al256((size_t)sp.n_groups * Rk * W * D * sizeof(float));
  const size_t zp = zpack_bytes(B, T, rkp);
  uint8_t* p = (uint8_t*)base;
  w.dzp = (float*)p;
  w.cnt = (int*)(p ? p + dzp : nullptr);
  w.dUp = (float*)(p ? p + dzp + cnt : nullptr);
  w.zp = p ? p + dzp + cnt + dUp : nullptr;
  w.bytes = dzp + cnt + dUp + zp;
  return w;
}

template <int W, int RKP>
int launch_bwd(const void* x, const void* z, const void* U, const void* sw, const void* dy, void* dx, void* dz,
               float* dU_f32, void* dU, void* dsw, void* wsp, int64_t B, int64_t T, int64_t D, int R, int Rk,
               int residual, cudaStream_t st) {
  constexpr int NP = RKP == 16 ? 2 : 1;
  using L = BwdSmem<W, RKP, NP>;
  static_assert(L::kTotal <= 232448 - 512, "backward shared memory budget (227 KB per CTA)");
  CUtensorMap dymap, xmap, zmap;
  int s;
  const TileSplit sp = tile_split(B, T, D);
  BwdWorkspace ws = bwd_workspace(wsp, B, T, D, Rk, W);
  if ((s = make_btd_map(&dymap, dy, B, T, D, kBD, kBT + W - 1))) return s;
  if ((s = make_btd_map(&xmap, x, B, T, D, kBD, kBT + W - 1))) return s;
  if ((s = make_zpack_map(&zmap, ws.zp, B, T, RKP, kZRows))) return s;
  if ((s = z_pack_launch(z, ws.zp, B, T, R, RKP, sw != nullptr, st))) return s;
  cudaError_t e = cudaMemsetAsync(ws.cnt, 0, (size_t)(sp.n_groups + 1) * sizeof(int), st);
  if (e != cudaSuccess) return cuda_status(e, "cudaMemsetAsync(group counters)");
  const int smem = (int)L::kTotal;
  e = cudaFuncSetAttribute(lr_bwd_tc_kernel<W, RKP, NP>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return cuda_status(e, "cudaFuncSetAttribute(lr_bwd_tc)");
  }
  // Cooperative launch: the CTAs of a token group wait for one another before
  // the dz reduction, so the whole grid must be co-resident (grid <= SM count,
  // one CTA per SM; lr_tc_bwd_supported checks the first bound).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(sp.n_dblk * sp.n_groups));
  cfg.blockDim = dim3(kBwdThreads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, lr_bwd_tc_kernel<W, RKP, NP>, dymap, xmap, zmap, (const __nv_bfloat16*)U,
                         (const __nv_bfloat16*)sw, (__nv_bfloat16*)dx, (__nv_bfloat16*)dz, ws.dzp, ws.cnt, ws.dUp,
                         dU_f32, (__nv_bfloat16*)dU, (__nv_bfloat16*)(sw ? dsw : nullptr), sp, (int)T, (int)D, R, Rk,
                         residual);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return cuda_status(e, "cudaLaunchKernelEx(lr_bwd_tc_kernel)");
  }
  DYNCONV_CHECK_LAUNCH("lr_bwd_tc_kernel");
  return DYNCONV_OK;
}

template <int RKP>
int launch_bwd_w(int W, const void* x, const void* z, const void* U, const void* sw, const void* dy, void* dx,
                 void* dz, float* dU_f32, void* dU, void* dsw, void* ws, int64_t B, int64_t T, int64_t D, int R,
                 int Rk, int residual, cudaStream_t st) {
  switch (W) {
    case 1: return launch_bwd<1, RKP>(x, z, U, sw, dy, dx, dz, dU_f32, dU, dsw, ws, B, T, D, R, Rk, residual, st);
    case 2: return launch_bwd<2, RKP>(x, z, U, sw, dy, dx, dz, dU_f32, dU, dsw, ws, B, T, D, R, Rk, residual, st);
    case 3: return launch_bwd<3, RKP>(x, z, U, sw, dy, dx, dz, dU_f32, dU, dsw, ws, B, T, D, R, Rk, residual, st);
    case 4: return launch_bwd<4, RKP>(x, z, U, sw, dy, dx, dz, dU_f32, dU, dsw, ws, B, T, D, R, Rk, residual, st);
    default: return set_error(DYNCONV_ERR_UNSUPPORTED, "tensor-core backward: W=%d", W);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

// Tensor-core path envelope: bf16, W <= 4, R_kernel <= 64, D % 8 == 0 (TMA row
// pitch), 16-byte aligned activations (TMA base).  Everything else runs the
// CUDA-core kernels of lowrank_simple.cu.
bool lr_tc_bwd_supported(int64_t D, int Rk, int W, int dtype, const void* const* ptrs, int nptrs) {
  if (dtype != DYNCONV_DTYPE_BF16 || W < 1 || W > 4 || Rk < 1 || Rk > 32 || D % 8 != 0) return false;
  if ((D + kBD - 1) / kBD > sm_count()) return false;  // the cooperative grid must fit on the GPU
  for (int i = 0; i < nptrs; ++i)
    if (ptrs[i] && !aligned16(ptrs[i])) return false;
  return encode_fn() != nullptr || nptrs == 0;
}

bool lr_tc_supported(int64_t D, int Rk, int W, int dtype, const void* const* ptrs, int nptrs) {
  if (dtype != DYNCONV_DTYPE_BF16 || W < 1 || W > 4 || Rk < 1 || Rk > 64 || D % 8 != 0) return false;
  for (int i = 0; i < nptrs; ++i)
    if (ptrs[i] && !aligned16(ptrs[i])) return false;
  return encode_fn() != nullptr || nptrs == 0;
}

size_t lr_tc_bwd_workspace(int64_t B, int64_t T, int64_t D, int Rk, int W) {
  return bwd_workspace(nullptr, B, T, D, Rk, W).bytes;
}

size_t lr_tc_fwd_workspace(int64_t B, int64_t T, int Rk) { return zpack_bytes(B, T, (Rk + 15) / 16 * 16); }

int lr_tc_fwd_launch(const void* x, const void* z, const void* U, const void* sw, void* y, void* ws, size_t ws_bytes,
                     int64_t B, int64_t T, int64_t D, int R, int Rk, int W, int residual, cudaStream_t st) {
  if (!ws || ws_bytes < lr_tc_fwd_workspace(B, T, Rk))
    return set_error(DYNCONV_ERR_WORKSPACE, "lr_fwd (tensor core): workspace too small");
  const int rkp = (Rk + 15) / 16 * 16;
  switch (rkp) {
    case 16: return launch_fwd_w<16>(W, x, z, U, sw, y, ws, B, T, D, R, residual, st);
    case 32: return launch_fwd_w<32>(W, x, z, U, sw, y, ws, B, T, D, R, residual, st);
    case 48: return launch_fwd_w<48>(W, x, z, U, sw, y, ws, B, T, D, R, residual, st);
    case 64: return launch_fwd_w<64>(W, x, z, U, sw, y, ws, B, T, D, R, residual, st);
    default: return set_error(DYNCONV_ERR_UNSUPPORTED, "R_kernel=%d", Rk);
  }
}

int lr_tc_bwd_launch(const void* x, const void* z, const void* U, const void* sw, const void* dy, void* dx, void* dz,
                     float* dU_f32, void* dU, void* dsw, void* ws, size_t ws_bytes, int64_t B, int64_t T, int64_t D,
                     int R, int Rk, int W, int residual, cudaStream_t st) {
  if (ws_bytes < lr_tc_bwd_workspace(B, T, D, Rk, W))
    return set_error(DYNCONV_ERR_WORKSPACE, "lr_bwd (tensor core): workspace too small");
  if (Rk <= 16) return launch_bwd_w<16>(W, x, z, U, sw, dy, dx, dz, dU_f32, dU, dsw, ws, B, T, D, R, Rk, residual, st);
  return launch_bwd_w<32>(W, x, z, U, sw, dy, dx, dz, dU_f32, dU, dsw, ws, B, T, D, R, Rk, residual, st);
}

}  // namespace dynconv
