// lowrank_tc.cu -- tcgen05 (5th-generation tensor core) lowrank kernels, bf16.
//
// Reference behaviour: lowrank.py:24-67 (forward kernel, Triton tl.dot with
// K = R_kernel), lowrank.py:214-249 (static-rank fold + launch); oracle
// reference.py:23-39.
//
// Forward data flow per work item (128 channels x 64 timesteps of one batch row):
//
//   HBM x  --TMA (3-D box, zero fill for t<0 / t>=T)--> smem x tile [67 rows][128 ch]
//   HBM z  --producer warp (plain loads, static rank = 1.0)--> smem z tile, K-major
//   smem U (per 128-channel block, static_w folded as rank R)   [K-major, per tap]
//   tcgen05.mma (M = 128 channels, N = 64 timesteps, K = R_kernel) per tap w
//        -> TMEM acc_w[ch][t] = sum_r U[r,w,ch] z[t,r]      (the dynamic weights;
//                                                            never written to HBM)
//   epilogue warps: y[t,ch] = sum_w acc_w[ch][t] * x[t-w,ch] (+ x[t,ch])
//        -> smem y tile -> TMA store
//
// Warp roles (320 threads, one CTA per SM, persistent over a contiguous range
// of work items):  warp 0 producer, warp 1 TMEM owner + MMA issuer (one lane),
// warps 2..9 epilogue (two warps per TMEM lane quarter, one per 32-step half).
// Pipelines: S-stage x/z ring (full/empty mbarriers), double-buffered TMEM
// accumulators (acc_full via tcgen05.commit / acc_empty), double-buffered y tile
// (TMA store bulk groups).  Every mbarrier wait is bounded (common.cuh).
#include <mutex>

#include "common.cuh"

namespace dynconv {

DYNCONV_DEFINE_ERROR_ACCESSOR(lr_tc_error_word)

namespace {

constexpr int kBT = 64;         // timesteps per work item (MMA N)
constexpr int kBD = 128;        // channels per work item (MMA M)
constexpr int kStages = 4;      // x/z pipeline depth
constexpr int kEpiWarps = 8;    // epilogue warps
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

// ------------------------------------------------------------- work split

struct WorkSplit {
  int n_dblk;       // 128-channel blocks
  int tiles_row;    // 64-step tiles per batch row
  int64_t n_items;  // n_dblk * B * tiles_row, d-block major
};

__host__ __device__ inline void item_coords(const WorkSplit& w, int64_t item, int& dblk, int& b, int& t0) {
  const int64_t tiles = w.n_items / w.n_dblk;  // B * tiles_row
  dblk = (int)(item / tiles);
  const int64_t tile = item % tiles;
  b = (int)(tile / w.tiles_row);
  t0 = (int)(tile % w.tiles_row) * kBT;
}

// ------------------------------------------------------------- smem layout

template <int W, int RKP>
struct FwdSmem {
  static constexpr int kXRows = kBT + W - 1;
  static constexpr uint32_t kXBytes = (uint32_t)kXRows * kBD * 2;        // TMA box bytes
  static constexpr uint32_t kXStride = (kXBytes + 1023u) / 1024u * 1024u;
  static constexpr uint32_t kZBytes = (uint32_t)kBT * RKP * 2;           // K-major, 64 rows x RKP
  static constexpr uint32_t kYBytes = (uint32_t)kBT * kBD * 2;
  static constexpr uint32_t kUTap = (uint32_t)kBD * RKP * 2;
  static constexpr uint32_t kOffX = 0;
  static constexpr uint32_t kOffZ = kOffX + kStages * kXStride;
  static constexpr uint32_t kOffY = kOffZ + kStages * kZBytes;
  static constexpr uint32_t kOffU = kOffY + 2 * kYBytes;
  static constexpr uint32_t kTotal = kOffU + W * kUTap + 1024;  // + alignment slack
  // K-major operand strides
  static constexpr uint32_t kZLbo = kBT * 16;          // next 8-rank chunk of z
  static constexpr uint32_t kZSbo = 128;               // next 8 timesteps
  static constexpr uint32_t kULbo = 128;               // next 8-rank chunk of U
  static constexpr uint32_t kUSbo = (RKP / 8) * 128;   // next 8 channels
};

// Loads U_ext for channel block dblk into smem (K-major, one [128 x RKP] block per tap).
template <int W, int RKP>
__device__ void load_u_block(uint8_t* us, const __nv_bfloat16* __restrict__ U, const __nv_bfloat16* __restrict__ sw,
                             int dblk, int D, int R, int lane, int nthreads) {
  using L = FwdSmem<W, RKP>;
  const int d0 = dblk * kBD;
  for (int e = lane; e < W * RKP * kBD; e += nthreads) {
    const int d = e % kBD;
    const int r = (e / kBD) % RKP;
    const int w = e / (kBD * RKP);
    __nv_bfloat16 v = __float2bfloat16_rn(0.f);
    if (d0 + d < D) {
      if (r < R) v = U[((size_t)r * W + w) * D + d0 + d];
      else if (r == R && sw != nullptr) v = sw[(size_t)w * D + d0 + d];
    }
    *reinterpret_cast<__nv_bfloat16*>(us + w * L::kUTap + kmajor_off(d, r, L::kUSbo, L::kULbo)) = v;
  }
}

// Writes the z tile (64 timesteps x RKP ranks, K-major) for rows t0.. of batch b.
template <int W, int RKP>
__device__ void load_z_tile(uint8_t* zs, const __nv_bfloat16* __restrict__ z, int b, int t0, int T, int R,
                            bool has_static, int lane) {
  using L = FwdSmem<W, RKP>;
  for (int j = lane; j < kBT; j += 32) {
    const int t = t0 + j;
    const bool ok = t < T;
    const __nv_bfloat16* zr = z + ((size_t)b * T + (ok ? t : 0)) * R;
#pragma unroll
    for (int c = 0; c < RKP / 8; ++c) {
      __align__(16) __nv_bfloat16 v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int r = c * 8 + k;
        float f = 0.f;
        if (ok) {
          if (r < R) f = __bfloat162float(zr[r]);
          else if (r == R && has_static) f = 1.f;
        }
        v[k] = __float2bfloat16_rn(f);
      }
      *reinterpret_cast<uint4*>(zs + kmajor_off(j, c * 8, L::kZSbo, L::kZLbo)) = *reinterpret_cast<uint4*>(v);
    }
  }
}

// ------------------------------------------------------------- forward kernel

template <int W, int RKP>
__global__ void __launch_bounds__(kFwdThreads, 1)
    lr_fwd_tc_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap ymap,
                     const __nv_bfloat16* __restrict__ z, const __nv_bfloat16* __restrict__ U,
                     const __nv_bfloat16* __restrict__ sw, WorkSplit ws, int T, int D, int R, int residual) {
  using L = FwdSmem<W, RKP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full_bar[kStages], empty_bar[kStages], accf_bar[2], acce_bar[2], u_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t G = gridDim.x;
  const int64_t it0 = ws.n_items * blockIdx.x / G, it1 = ws.n_items * (blockIdx.x + 1) / G;
  const bool has_static = sw != nullptr;
  constexpr uint32_t kAccCols = W * kBT;
  constexpr uint32_t kTmemCols = (2 * kAccCols <= 256) ? 256 : 512;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kEpiWarps);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf_bar[a], 1);
      mbar_init(&acce_bar[a], kEpiWarps);
    }
    mbar_init(&u_bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&xmap);
    prefetch_tensormap(&ymap);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    const uint64_t pol = policy_evict_first();
    for (int64_t i = it0; i < it1; ++i) {
      const int k = (int)(i - it0), s = k % kStages;
      if (!mbar_wait(&empty_bar[s], ((k / kStages) & 1) ^ 1, kErrWaitProducer, &abort_flag)) break;
      int dblk, b, t0;
      item_coords(ws, i, dblk, b, t0);
      load_z_tile<W, RKP>(smem + L::kOffZ + s * L::kZBytes, z, b, t0, T, R, has_static, lane);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_expect_tx(&full_bar[s], L::kXBytes);
        tma_load_3d(smem + L::kOffX + s * L::kXStride, &xmap, &full_bar[s], dblk * kBD, t0 - (W - 1), b, pol);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc = make_idesc_bf16(kBD, kBT, 0, 0);
    uint8_t* us = smem + L::kOffU;
    int cur = -1;
    uint32_t u_phase = 0;
    for (int64_t i = it0; i < it1; ++i) {
      const int k = (int)(i - it0), s = k % kStages, a = k & 1;
      int dblk, b, t0;
      item_coords(ws, i, dblk, b, t0);
      if (dblk != cur) {
        if (cur >= 0) {  // wait until the MMAs that read the old U block are done
          if (lane == 0) umma_commit(&u_bar);
          __syncwarp();
          if (!mbar_wait(&u_bar, u_phase, kErrWaitMma, &abort_flag)) break;
          u_phase ^= 1;
        }
        load_u_block<W, RKP>(us, U, sw, dblk, D, R, lane, 32);
        fence_proxy_async_smem();
        __syncwarp();
        cur = dblk;
      }
      if (!mbar_wait(&full_bar[s], (k / kStages) & 1, kErrWaitMma, &abort_flag)) break;
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
    const int e = warp - 2;            // 0..7
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int half = e >> 2;           // which 32-step half of the tile
    const int ch = q * 32 + lane;      // channel within the block (= TMEM lane)
    const int et = e * 32 + lane;      // 0..255
    const uint64_t pol_y = policy_evict_first();
    bool dead = false;  // a bounded wait gave up: keep joining the named barriers, skip the work
    for (int64_t i = it0; i < it1; ++i) {
      const int k = (int)(i - it0), s = k % kStages, a = k & 1;
      int dblk, b, t0;
      item_coords(ws, i, dblk, b, t0);
      // y buffer `a` is free once the store issued two items ago has read it
      if (et == 0 && !dead) bulk_wait_group_read<1>();
      named_bar_sync(1, 32 * kEpiWarps);
      if (!dead) dead = !mbar_wait(&full_bar[s], (k / kStages) & 1, kErrWaitEpilogue, &abort_flag);
      if (!dead) dead = !mbar_wait(&accf_bar[a], (k >> 1) & 1, kErrWaitEpilogue, &abort_flag);
      tc_fence_after();
      __nv_bfloat16* ys = reinterpret_cast<__nv_bfloat16*>(smem + L::kOffY + a * L::kYBytes);
      if (!dead) {
        const __nv_bfloat16* xs = reinterpret_cast<const __nv_bfloat16*>(smem + L::kOffX + s * L::kXStride);
        // x window: xr[j] = x at step (tok0 - (W-1) + j); smem row of step t is (t - t0) + (W-1)
        float xr[16 + W - 1];
        const int tok0 = half * 32;
#pragma unroll
        for (int j = 0; j < W - 1; ++j) xr[j] = __bfloat162float(xs[(tok0 + j) * kBD + ch]);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
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
            ys[(tb + j) * kBD + ch] = __float2bfloat16_rn(yv);
          }
#pragma unroll
          for (int j = 0; j < W - 1; ++j) xr[j] = xr[16 + j];
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&acce_bar[a]);
        mbar_arrive(&empty_bar[s]);
      }
      fence_proxy_async_smem();
      named_bar_sync(1, 32 * kEpiWarps);
      if (et == 0 && !dead) {
        tma_store_3d(&ymap, ys, dblk * kBD, t0, b, pol_y);
        bulk_commit_group();
      }
    }
    if (et == 0) bulk_wait_group<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

template <int W, int RKP>
int launch_fwd(const void* x, const void* z, const void* U, const void* sw, void* y, int64_t B, int64_t T, int64_t D,
               int R, int residual, cudaStream_t st) {
  using L = FwdSmem<W, RKP>;
  CUtensorMap xmap, ymap;
  int s;
  if ((s = make_btd_map(&xmap, x, B, T, D, kBD, kBT + W - 1))) return s;
  if ((s = make_btd_map(&ymap, y, B, T, D, kBD, kBT))) return s;
  WorkSplit ws;
  ws.n_dblk = (int)((D + kBD - 1) / kBD);
  ws.tiles_row = (int)((T + kBT - 1) / kBT);
  ws.n_items = (int64_t)ws.n_dblk * B * ws.tiles_row;
  const int grid = (int)std::min<int64_t>(ws.n_items, sm_count());
  const int smem = (int)L::kTotal;
  cudaError_t e = cudaFuncSetAttribute(lr_fwd_tc_kernel<W, RKP>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(lr_fwd_tc)");
  lr_fwd_tc_kernel<W, RKP><<<grid, kFwdThreads, smem, st>>>(xmap, ymap, (const __nv_bfloat16*)z,
                                                            (const __nv_bfloat16*)U, (const __nv_bfloat16*)sw, ws,
                                                            (int)T, (int)D, R, residual);
  DYNCONV_CHECK_LAUNCH("lr_fwd_tc_kernel");
  return DYNCONV_OK;
}

template <int RKP>
int launch_fwd_w(int W, const void* x, const void* z, const void* U, const void* sw, void* y, int64_t B, int64_t T,
                 int64_t D, int R, int residual, cudaStream_t st) {
  switch (W) {
    case 1: return launch_fwd<1, RKP>(x, z, U, sw, y, B, T, D, R, residual, st);
    case 2: return launch_fwd<2, RKP>(x, z, U, sw, y, B, T, D, R, residual, st);
    case 3: return launch_fwd<3, RKP>(x, z, U, sw, y, B, T, D, R, residual, st);
    case 4: return launch_fwd<4, RKP>(x, z, U, sw, y, B, T, D, R, residual, st);
    default: return set_error(DYNCONV_ERR_UNSUPPORTED, "tensor-core path: W=%d", W);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

// Tensor-core path envelope: bf16, W <= 4, R_kernel <= 64, D % 8 == 0 (TMA row
// pitch), 16-byte aligned activations (TMA base).  Everything else runs the
// CUDA-core kernels of lowrank_simple.cu.
bool lr_tc_bwd_supported(int64_t D, int Rk, int W, int dtype, const void* const* ptrs, int nptrs) {
  (void)D; (void)Rk; (void)W; (void)dtype; (void)ptrs; (void)nptrs;
  return false;
}

bool lr_tc_supported(int64_t D, int Rk, int W, int dtype, const void* const* ptrs, int nptrs) {
  if (dtype != DYNCONV_DTYPE_BF16 || W < 1 || W > 4 || Rk < 1 || Rk > 64 || D % 8 != 0) return false;
  for (int i = 0; i < nptrs; ++i)
    if (ptrs[i] && !aligned16(ptrs[i])) return false;
  return encode_fn() != nullptr || nptrs == 0;
}

size_t lr_tc_bwd_workspace(int64_t B, int64_t T, int64_t D, int Rk, int W) {
  (void)B; (void)T; (void)D; (void)Rk; (void)W;
  return 0;
}

int lr_tc_fwd_launch(const void* x, const void* z, const void* U, const void* sw, void* y, int64_t B, int64_t T,
                     int64_t D, int R, int Rk, int W, int residual, cudaStream_t st) {
  const int rkp = (Rk + 15) / 16 * 16;
  switch (rkp) {
    case 16: return launch_fwd_w<16>(W, x, z, U, sw, y, B, T, D, R, residual, st);
    case 32: return launch_fwd_w<32>(W, x, z, U, sw, y, B, T, D, R, residual, st);
    case 48: return launch_fwd_w<48>(W, x, z, U, sw, y, B, T, D, R, residual, st);
    case 64: return launch_fwd_w<64>(W, x, z, U, sw, y, B, T, D, R, residual, st);
    default: return set_error(DYNCONV_ERR_UNSUPPORTED, "R_kernel=%d", Rk);
  }
}

int lr_tc_bwd_launch(const void*, const void*, const void*, const void*, const void*, void*, void*, float*, void*,
                     void*, void*, size_t, int64_t, int64_t, int64_t, int, int, int, int, cudaStream_t) {
  return set_error(DYNCONV_ERR_UNSUPPORTED, "tensor-core lowrank backward not built");
}

}  // namespace dynconv
