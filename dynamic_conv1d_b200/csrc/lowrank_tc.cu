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
//   smem U (per 128-channel block, static_w folded as rank R)   [MN-major, per tap]
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

#include "lowrank_tc.cuh"

namespace dynconv {

DYNCONV_DEFINE_ERROR_ACCESSOR(lr_tc_error_word)

namespace lrtc {

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

int make_btd_map(CUtensorMap* map, const void* base, int64_t B, int64_t T, int64_t D, int box_d, int box_t,
                 int swizzle_bytes) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(DYNCONV_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (swizzle_bytes != 0 && box_d * 2 != swizzle_bytes)
    return set_error(DYNCONV_ERR_SHAPE, "swizzled map: box of %d channels != %d bytes", box_d, swizzle_bytes);
  if (int s = ensure_context()) return s;
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)T * D * 2};
  cuuint32_t box[3] = {(cuuint32_t)box_d, (cuuint32_t)box_t, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                  : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                  : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                        : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(DYNCONV_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return DYNCONV_OK;
}

int make_zpack_map(CUtensorMap* map, const void* base, int64_t B, int64_t T, int rkp, int rows, int G) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(DYNCONV_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (int s = ensure_context()) return s;
  cuuint64_t dims[4] = {8, (cuuint64_t)T, (cuuint64_t)B, (cuuint64_t)(G * rkp / 8)};
  cuuint64_t strides[3] = {16, (cuuint64_t)T * 16, (cuuint64_t)B * T * 16};
  cuuint32_t box[4] = {8, (cuuint32_t)rows, 1, (cuuint32_t)(rkp / 8)};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(DYNCONV_ERR_CUDA, "cuTensorMapEncodeTiled(z_pack) failed (%d)", (int)r);
  return DYNCONV_OK;
}

// z_pack[g*RKP/8 + c][b][t][e] = z_ext_g[b, t, 8c + e]: group g's z (columns
// g*R .. g*R+R-1 of a [B][T][G*R] row) for ranks < R, 1.0 at rank R when the static
// filter is fused (the reference's F.pad(z, (0, 1), value=1.0), lowrank.py:224), 0 up
// to RKP.  One thread per (8-rank chunk, token): consecutive threads write
// consecutive 16-byte chunks.
__global__ void __launch_bounds__(256) z_pack_kernel(const __nv_bfloat16* __restrict__ z,
                                                     __nv_bfloat16* __restrict__ zp, int64_t ntok, int R, int rkp,
                                                     int has_static, int G) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= ntok * (G * rkp / 8)) return;
  const int cc = (int)(i / ntok);
  const int64_t tok = i - (int64_t)cc * ntok;
  const int g = cc / (rkp / 8), c = cc - g * (rkp / 8);
  const __nv_bfloat16* zr = z + tok * (int64_t)(G * R) + g * R;
  __align__(16) __nv_bfloat16 v[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int r = 8 * c + e;
    v[e] = r < R ? zr[r] : __float2bfloat16_rn((r == R && has_static) ? 1.f : 0.f);
  }
  *reinterpret_cast<uint4*>(zp + i * 8) = *reinterpret_cast<const uint4*>(v);
}

size_t zpack_bytes(int64_t B, int64_t T, int rkp, int G) {
  return ((size_t)B * T * rkp * G * 2 + 255) / 256 * 256;
}

int z_pack_launch(const void* z, void* zp, int64_t B, int64_t T, int R, int rkp, bool has_static, cudaStream_t st,
                  int G) {
  const int64_t ntok = B * T;
  const int64_t nthreads = ntok * (G * rkp / 8);
  z_pack_kernel<<<(unsigned)((nthreads + 255) / 256), 256, 0, st>>>((const __nv_bfloat16*)z, (__nv_bfloat16*)zp,
                                                                   ntok, R, rkp, has_static ? 1 : 0, G);
  DYNCONV_CHECK_LAUNCH("z_pack_kernel");
  return DYNCONV_OK;
}

}  // namespace lrtc

namespace {

using namespace lrtc;

constexpr int kStages = 4;      // x/z pipeline depth (forward, R_kernel <= 32)
constexpr int kEpiWarps = 16;   // forward epilogue warps: four per TMEM lane quarter
constexpr int kEpiSteps = kBT / (kEpiWarps / 4);  // timesteps per epilogue warp and tile
constexpr int kFwdThreads = 64 + 32 * kEpiWarps;

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
  static constexpr uint32_t kULbo = 128;               // U (MN-major): next 8-rank chunk
  static constexpr uint32_t kUSbo = (RKP / 8) * 128;   // U (MN-major): next 8 channels
};

// ------------------------------------------------------------- forward kernel

template <int W, int RKP>
__global__ void __launch_bounds__(kFwdThreads, 1)
    lr_fwd_tc_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap ymap,
                     const __grid_constant__ CUtensorMap zmap, const __nv_bfloat16* __restrict__ U,
                     const __nv_bfloat16* __restrict__ sw, TileSplit sp, ChanGroups cg, int T, int R, int residual) {
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
  const int grp = dblk / cg.nd;  // channel group of this CTA's block
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
    load_u_mn<W, RKP, kNonProducer>(smem + L::kOffU, U + (size_t)grp * R * W * cg.Dg,
                                    sw ? sw + (size_t)grp * W * cg.Dg : nullptr, (dblk - grp * cg.nd) * kBD, cg.Dg, R,
                                    threadIdx.x - 32);
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
        tma_load_4d(smem + L::kOffZ + s * L::kZBytes, &zmap, &full_bar[s], 0, t0, b, grp * (RKP / 8), pol);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc = make_idesc_bf16(kBD, kBT, 1, 0);  // A = U^T (MN-major: channels), B = z (K-major)
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
          // two steps at a time with packed f32x2 arithmetic (each lane rounds like the scalar op)
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            float2 y2 = mul2(make_float2(acc[0][j], acc[0][j + 1]), make_float2(xr[W - 1 + j], xr[W + j]));
#pragma unroll
            for (int w = 1; w < W; ++w)
              y2 = fma2(make_float2(acc[w][j], acc[w][j + 1]), make_float2(xr[W - 1 + j - w], xr[W + j - w]), y2);
            if (residual) y2 = add2(y2, make_float2(xr[W - 1 + j], xr[W + j]));
            // lane pairs swap halves so that each lane stores one whole 32-bit word: the even
            // lane channels (l, l+1) of step j, the odd lane channels (l-1, l) of step j+1
            const uint32_t mine = pack_bf16x2(y2.x, y2.y);  // (step j, step j+1) of channel `lane`
            const uint32_t other = __shfl_xor_sync(0xffffffffu, mine, 1);
            const uint32_t word = (lane & 1) ? __byte_perm(other, mine, 0x7632) : __byte_perm(mine, other, 0x5410);
            *reinterpret_cast<uint32_t*>(ys + (c * 16 + j + (lane & 1)) * 32 + (lane & ~1)) = word;
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

// x, y: [B][T][G*D]; z: [B][T][G*R]; U: [G][R][W*D]; sw: [G][W][D] or null.
template <int W, int RKP>
int launch_fwd(const void* x, const void* z, const void* U, const void* sw, void* y, void* ws, int64_t B, int64_t T,
               int64_t D, int G, int R, int residual, cudaStream_t st) {
  using L = FwdSmem<W, RKP>;
  static_assert(L::kTotal <= 232448 - 512, "forward shared memory budget (227 KB per CTA)");
  const int64_t Dt = (int64_t)G * D;
  CUtensorMap xmap, ymap, zmap;
  int s;
  if ((s = make_btd_map(&xmap, x, B, T, Dt, kBD, kBT + W - 1))) return s;
  if ((s = make_btd_map(&ymap, y, B, T, Dt, 32, kEpiSteps))) return s;  // per-warp [steps][32 ch] stores
  if ((s = make_zpack_map(&zmap, ws, B, T, RKP, kBT, G))) return s;
  if ((s = z_pack_launch(z, ws, B, T, R, RKP, sw != nullptr, st, G))) return s;
  const TileSplit sp = tile_split(B, T, Dt);
  const ChanGroups cg = chan_groups(D, G);
  const int grid = sp.n_dblk * sp.n_groups;
  const int smem = (int)L::kTotal;
  cudaError_t e = cudaFuncSetAttribute(lr_fwd_tc_kernel<W, RKP>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) {
    cudaGetLastError();  // do not leave the failure pending for the next launch check
    return cuda_status(e, "cudaFuncSetAttribute(lr_fwd_tc)");
  }
  lr_fwd_tc_kernel<W, RKP><<<grid, kFwdThreads, smem, st>>>(xmap, ymap, zmap, (const __nv_bfloat16*)U,
                                                            (const __nv_bfloat16*)sw, sp, cg, (int)T, R, residual);
  DYNCONV_CHECK_LAUNCH("lr_fwd_tc_kernel");
  return DYNCONV_OK;
}

template <int RKP>
int launch_fwd_w(int W, const void* x, const void* z, const void* U, const void* sw, void* y, void* ws, int64_t B,
                 int64_t T, int64_t D, int G, int R, int residual, cudaStream_t st) {
  switch (W) {
    case 1: return launch_fwd<1, RKP>(x, z, U, sw, y, ws, B, T, D, G, R, residual, st);
    case 2: return launch_fwd<2, RKP>(x, z, U, sw, y, ws, B, T, D, G, R, residual, st);
    case 3: return launch_fwd<3, RKP>(x, z, U, sw, y, ws, B, T, D, G, R, residual, st);
    case 4: return launch_fwd<4, RKP>(x, z, U, sw, y, ws, B, T, D, G, R, residual, st);
    default: return set_error(DYNCONV_ERR_UNSUPPORTED, "tensor-core path: W=%d", W);
  }
}

}  // namespace

// Tensor-core forward envelope: bf16, W <= 4, R_kernel <= 64, D % 8 == 0 (TMA row
// pitch; D % 128 == 0 with G > 1 channel groups), 16-byte aligned activations (TMA
// base).  Everything else runs the CUDA-core kernels of lowrank_simple.cu.
bool lr_tc_supported(int64_t D, int Rk, int W, int dtype, const void* const* ptrs, int nptrs, int G) {
  if (dtype != DYNCONV_DTYPE_BF16 || W < 1 || W > 4 || Rk < 1 || Rk > 64 || D % 8 != 0) return false;
  if (G < 1 || (G > 1 && D % kBD != 0)) return false;
  for (int i = 0; i < nptrs; ++i)
    if (ptrs[i] && !aligned16(ptrs[i])) return false;
  return encode_fn() != nullptr || nptrs == 0;
}

size_t lr_tc_fwd_workspace(int64_t B, int64_t T, int Rk, int G) {
  return zpack_bytes(B, T, (Rk + 15) / 16 * 16, G);
}

int lr_tc_fwd_launch(const void* x, const void* z, const void* U, const void* sw, void* y, void* ws, size_t ws_bytes,
                     int64_t B, int64_t T, int64_t D, int G, int R, int Rk, int W, int residual, cudaStream_t st) {
  if (!ws || ws_bytes < lr_tc_fwd_workspace(B, T, Rk, G))
    return set_error(DYNCONV_ERR_WORKSPACE, "lr_fwd (tensor core): workspace too small");
  const int rkp = (Rk + 15) / 16 * 16;
  switch (rkp) {
    case 16: return launch_fwd_w<16>(W, x, z, U, sw, y, ws, B, T, D, G, R, residual, st);
    case 32: return launch_fwd_w<32>(W, x, z, U, sw, y, ws, B, T, D, G, R, residual, st);
    case 48: return launch_fwd_w<48>(W, x, z, U, sw, y, ws, B, T, D, G, R, residual, st);
    case 64: return launch_fwd_w<64>(W, x, z, U, sw, y, ws, B, T, D, G, R, residual, st);
    default: return set_error(DYNCONV_ERR_UNSUPPORTED, "R_kernel=%d", Rk);
  }
}

}  // namespace dynconv
