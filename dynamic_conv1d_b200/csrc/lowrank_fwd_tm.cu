// lowrank_fwd_tm.cu -- tcgen05 forward of the lowrank dynamic convolution, bf16,
// time-major.
//
// Reference behaviour: lowrank.py:24-67 (forward kernel, Triton tl.dot with
// K = R_kernel), lowrank.py:214-249 (static-rank fold + launch); oracle
// reference.py:23-39.
//
//   Wt_w[t,ch] = sum_r z_ext[t,r] U_ext[r,w,ch]          (dynamic weights, never in HBM)
//   y[t,ch]    = sum_w Wt_w[t,ch] x[t-w,ch]  (+ x[t,ch] if residual)
//
// Orientation: tensor-memory lane = timestep.  A tile is 128 steps x 128
// channels of one batch row, handled as four 32-channel chunks.  Per chunk, one
// MMA per tap writes D[t][ch] = Wt_w[t,ch] (M = 128 steps, N = 32 channels,
// K = R_kernel; A = the z tile, K-major; B = U tap w, MN-major), and each
// epilogue thread owns one step: it reads its x rows t-w (16 bytes = 8 channels
// per load, conflict-free in the 128-byte-swizzled TMA tile) and writes y rows
// with 16-byte stores.
//
// Warps: 0 producer (TMA: z per tile, x per 64-channel half tile into a ring),
// 1/2 weight MMAs of chunk parity 0/1 (warp 1 owns TMEM), 3..18 the epilogue in
// two teams of eight (team = chunk parity; a warp has 32 steps of its TMEM lane
// quarter and 16 channels of the chunk).  Four weight buffers in tensor memory
// (4 x 128 columns), so the MMAs of the next two chunks of a team run while it
// works.  Every wait is bounded (common.cuh).
#include "lowrank_tc.cuh"

namespace dynconv {

DYNCONV_DEFINE_ERROR_ACCESSOR(lr_fwd_tm_error_word)

namespace {

using namespace lrtc;

constexpr int kTT = 128;          // steps per tile
constexpr int kCh = 32;           // channels per chunk
constexpr int kRowsX = kTT + 3;   // rows of an x box (W - 1 <= 3 halo rows)
constexpr int kZR = 128;          // z rows per tile
constexpr int kCtl = 3;           // producer + two MMA issuers
constexpr int kEpi = 16;          // epilogue warps
constexpr int kThreads = 32 * (kCtl + kEpi);
constexpr int kNWB = 4;           // weight buffers (4 x 128 tensor-memory columns)

template <int W, int RKP>
struct FtCfg {
  static constexpr uint32_t kBox = (uint32_t)kRowsX * 128;  // one 64-channel box, 128-byte rows
  static constexpr uint32_t kBoxStride = round1024(kBox);
  static constexpr uint32_t kUcg = (RKP / 8) * 128;         // U: next 8 channels
  static constexpr uint32_t kUTap = 16 * kUcg;              // U: next tap
  static constexpr uint32_t kLZ = kZR * 16;                 // z: next 8 ranks
  static constexpr uint32_t kZBytes = (RKP / 8) * kLZ;
  static constexpr uint32_t kUBytes = W * kUTap;
  static constexpr uint32_t kStage = 32 * 16 * 2;  // one warp's y sub-tile [32 steps][16 ch]
  static constexpr uint32_t kStageAll = kEpi * 2 * kStage;
  // ring depth: what is left of 227 KB after U, two z tiles and the y sub-tiles
  static constexpr int S0 = (int)((232448u - 2048u - kUBytes - 2 * kZBytes - kStageAll) / kBoxStride);
  static constexpr int S = S0 > 8 ? 8 : S0;
  static constexpr uint32_t kOffRing = 0;
  static constexpr uint32_t kOffU = kOffRing + S * kBoxStride;
  static constexpr uint32_t kOffZ = kOffU + kUBytes;
  static constexpr uint32_t kOffStage = (kOffZ + 2 * kZBytes + 255u) / 256u * 256u;  // 32-byte swizzle
  static constexpr uint32_t kTotal = kOffStage + kStageAll + 1024;  // + alignment slack
  static_assert(S >= 3, "forward ring too shallow");
  static_assert(kTotal <= 232448 - 512, "shared-memory budget (227 KB per CTA, static part aside)");
};

__device__ __forceinline__ float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

struct FtSplit {
  int n_dblk, tiles_row, n_tiles;
  int64_t n_units;  // n_dblk * n_tiles, split evenly over the grid
};

// Walks a CTA's units in order without divisions: (channel block, tile) and the
// tile's batch row b and first step t0.
struct UnitCursor {
  int dblk, tile, b, t0;
  __device__ __forceinline__ void init(int64_t u, const FtSplit& sp) {
    dblk = (int)(u / sp.n_tiles);
    tile = (int)(u - (int64_t)dblk * sp.n_tiles);
    b = tile / sp.tiles_row;
    t0 = (tile - b * sp.tiles_row) * kTT;
  }
  // advance one unit; true when the channel block changed
  __device__ __forceinline__ bool next(const FtSplit& sp) {
    ++tile;
    t0 += kTT;
    if (t0 >= sp.tiles_row * kTT) {
      t0 = 0;
      ++b;
    }
    if (tile == sp.n_tiles) {
      tile = 0;
      b = 0;
      ++dblk;
      return true;
    }
    return false;
  }
};

// U_ext block of channels [dlb, dlb + 128) of one group as 8 x 8 blocks
// [tap][ch/8][r/8][8 r][8 ch] -- the MN-major B operand (N = channels, K = ranks).
template <int W, int RKP, int NT>
__device__ void load_u_ft(uint8_t* us, const __nv_bfloat16* __restrict__ U, const __nv_bfloat16* __restrict__ sw,
                          int dlb, int Dg, int R, int tid) {
  constexpr int NV = W * RKP * (kBD / 8);
  for (int e = tid; e < NV; e += NT) {
    const int c8 = e % (kBD / 8);
    const int r = (e / (kBD / 8)) % RKP;
    const int w = e / ((kBD / 8) * RKP);
    const int d = dlb + 8 * c8;
    uint4 u = make_uint4(0, 0, 0, 0);
    if (d < Dg) {
      if (r < R) u = __ldg(reinterpret_cast<const uint4*>(U + ((size_t)r * W + w) * Dg + d));
      else if (r == R && sw != nullptr) u = __ldg(reinterpret_cast<const uint4*>(sw + (size_t)w * Dg + d));
    }
    *reinterpret_cast<uint4*>(us + ((w * 16 + c8) * (RKP / 8) + r / 8) * 128 + (r % 8) * 16) = u;
  }
}

// Work split: unit u = dblk * n_tiles + tile (channel block major); CTA i owns
// units [u0, u1) with u0 = n_units * i / grid.  A CTA's range is contiguous, so it
// crosses into the next channel block at most a few times (it reloads U there).
template <int W, int RKP>
__global__ void __launch_bounds__(kThreads, 1)
    lr_fwd_tm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap zmap,
                     const __grid_constant__ CUtensorMap ymap, const __nv_bfloat16* __restrict__ U,
                     const __nv_bfloat16* __restrict__ sw, FtSplit sp, ChanGroups cg, int T, int D, int R,
                     int residual) {
  using L = FtCfg<W, RKP>;
  constexpr int S = L::S;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  __shared__ uint64_t xfull[S], xempty[S], zfull[2], zempty[2], wfull[kNWB], wempty[kNWB], ufree, uready;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t u0 = sp.n_units * blockIdx.x / gridDim.x;
  const int64_t u1 = sp.n_units * (blockIdx.x + 1) / gridDim.x;
  const int n = (int)(u1 - u0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], kEpi);  // both teams read every half tile
    }
    for (int b2 = 0; b2 < 2; ++b2) {
      mbar_init(&zfull[b2], 1);
      mbar_init(&zempty[b2], 2);  // both MMA issuers
    }
    for (int c = 0; c < kNWB; ++c) {
      mbar_init(&wfull[c], 1);
      mbar_init(&wempty[c], kEpi / 2);
    }
    mbar_init(&ufree, 2);      // both MMA issuers are done with the old U block
    mbar_init(&uready, kEpi);  // every epilogue warp has stored its part of the new one
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&xmap);
    prefetch_tensormap(&zmap);
    prefetch_tensormap(&ymap);
  }
  __syncthreads();
  if (warp == 1) {
    tmem_alloc(&tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const uint64_t pol_z = policy_evict_normal();  // z rows are read by every channel block
      int hs = 0;
      UnitCursor uc;
      uc.init(u0, sp);
      for (int k = 0; k < n; ++k, uc.next(sp)) {
        const int b = uc.b, t0 = uc.t0;
        const int d0 = uc.dblk * kBD, grp = uc.dblk / cg.nd;
        if (!mbar_wait(&zempty[k & 1], ((k >> 1) & 1) ^ 1, kErrWaitProducer, &abort_flag)) break;
        mbar_arrive_expect_tx(&zfull[k & 1], L::kZBytes);
        tma_load_4d(smem + L::kOffZ + (k & 1) * L::kZBytes, &zmap, &zfull[k & 1], 0, t0, b, grp * (RKP / 8), pol_z);
        bool ok = true;
        for (int half = 0; half < 2; ++half, ++hs) {
          const int s = hs % S;
          if (!mbar_wait(&xempty[s], ((hs / S) & 1) ^ 1, kErrWaitProducer, &abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&xfull[s], L::kBox);
          tma_load_3d(smem + L::kOffRing + s * L::kBoxStride, &xmap, &xfull[s], d0 + 64 * half, t0 - 3, b, pol);
        }
        if (!ok) break;
      }
    }
    __syncwarp();
  } else {
    if (warp == 1 || warp == 2) {
      // ---------------------------------------------------------- weight MMAs (chunk parity tau)
      const int tau = warp - 1;
      const uint32_t idesc = make_idesc_bf16(kTT, kCh, 0, 1);  // A = z (K-major), B = U (MN-major)
      const uint32_t ub = smem_u32(smem + L::kOffU);
      const uint32_t zb0 = smem_u32(smem + L::kOffZ);
      int useg = 0;  // U segments started
      UnitCursor uc;
      uc.init(u0, sp);
      for (int k = 0; k < n; ++k) {
        if (k > 0 && uc.next(sp)) {
          // new channel block: the U buffer is free once this issuer's MMAs so far are done
          if (lane == 0) umma_commit(&ufree);
          __syncwarp();
          ++useg;
        }
        if (!mbar_wait(&uready, useg & 1, kErrWaitMma, &abort_flag)) break;
        if (!mbar_wait(&zfull[k & 1], (k >> 1) & 1, kErrWaitMma, &abort_flag)) break;
        const uint32_t zb = zb0 + (k & 1) * L::kZBytes;
        bool ok = true;
        for (int j = tau; j < 4; j += 2) {
          const int c = 4 * k + j, wb = c % kNWB;
          if (!mbar_wait(&wempty[wb], ((c / kNWB) & 1) ^ 1, kErrWaitMma, &abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
#pragma unroll
            for (int w = 0; w < W; ++w) {
#pragma unroll
              for (int ks = 0; ks < RKP / 16; ++ks) {
                const uint64_t ad = make_smem_desc(zb + ks * 2 * L::kLZ, L::kLZ, 128);
                const uint64_t bd = make_smem_desc(ub + w * L::kUTap + 4 * j * L::kUcg + ks * 256, 128, L::kUcg);
                umma_f16(tmem + wb * 128 + w * kCh, ad, bd, idesc, ks > 0 ? 1u : 0u);
              }
            }
            umma_commit(&wfull[wb]);
            if (j + 2 >= 4) umma_commit(&zempty[k & 1]);
          }
          __syncwarp();
        }
        if (!ok) break;
      }
    } else {
      // ---------------------------------------------------------- epilogue
      const int e = warp - kCtl;   // 0..15
      const int q = warp & 3;      // TMEM lane quarter = 32-step quarter of the tile
      const int tau = e >> 3;      // team: chunks of this parity
      const int h = (e >> 2) & 1;  // 16-channel half of the chunk
      const int t = 32 * q + lane;
      const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16);
      const uint64_t pol_y = policy_evict_first();
      bool dead = false;
      int useg = 0;
      int m = 0;  // chunks this warp has handled
      UnitCursor uc;
      uc.init(u0, sp);
      for (int k = 0; k < n; ++k) {
        const bool new_block = k == 0 || uc.next(sp);
        const int dblk = uc.dblk;
        if (new_block) {
          // U block of a new channel block (the first one, or a reload once both
          // issuers have finished every MMA that reads the old block)
          if (k > 0) {
            if (!dead) dead = !mbar_wait(&ufree, useg & 1, kErrWaitEpilogue, &abort_flag);
            ++useg;
          }
          if (!dead) {
            const int grp = dblk / cg.nd, dl0 = dblk * kBD - grp * cg.Dg;
            load_u_ft<W, RKP, 32 * kEpi>(smem + L::kOffU, U + (size_t)grp * R * W * cg.Dg,
                                         sw ? sw + (size_t)grp * W * cg.Dg : nullptr, dl0, cg.Dg, R, 32 * e + lane);
            fence_proxy_async_smem();
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&uready);
        }
        const int b = uc.b, t0 = uc.t0;
        const int d0 = dblk * kBD;
        for (int j = tau; j < 4; j += 2, ++m) {
          const int c = 4 * k + j, wb = c % kNWB, hs = 2 * k + (j >> 1), s = hs % S;
          if (!dead) dead = !mbar_wait(&wfull[wb], (c / kNWB) & 1, kErrWaitEpilogue, &abort_flag);
          if (!dead) dead = !mbar_wait(&xfull[s], (hs / S) & 1, kErrWaitEpilogue, &abort_flag);
          tc_fence_after();
          // this warp's y sub-tile buffer (m & 1) is free once its store of chunk m-2 has read it
          uint8_t* const stg = smem + L::kOffStage + (e * 2 + (m & 1)) * L::kStage;
          if (lane == 0 && !dead) bulk_wait_group_read<1>();
          __syncwarp();
          if (!dead) {
            const uint8_t* xs = smem + L::kOffRing + s * L::kBoxStride;
            const uint32_t wcol = ta + wb * 128 + 16 * h;  // this warp's 16 channels, tap 0
            // weights in four batches (8-channel group cgi, 4-channel half hh), each
            // tensor-memory load issued one step ahead of its use
            float wa[W][4], wb2[W][4];
            auto ld_w = [&](float (&v)[W][4], int cgi, int hh) {
#pragma unroll
              for (int w = 0; w < W; ++w) tmem_ld4(wcol + w * kCh + cgi * 8 + 4 * hh, v[w]);
            };
            // y[t] for 4 channels = sum_w Wt_w[t] x[t-w] (+ x[t]) -> two bf16 pairs
            auto y4 = [&](const float (&v)[W][4], const uint4 (&xr)[W], int hh, uint32_t& p0, uint32_t& p1) {
              // packed f32x2 arithmetic on channel pairs (each lane rounds like the scalar op)
              const uint32_t* d = reinterpret_cast<const uint32_t*>(&xr[0]) + 2 * hh;
              float2 a0, a1;
              {
                const float2 x0 = make_float2(bf_lo(d[0]), bf_hi(d[0])), x1 = make_float2(bf_lo(d[1]), bf_hi(d[1]));
                const float2 w0 = make_float2(v[0][0], v[0][1]), w1 = make_float2(v[0][2], v[0][3]);
                a0 = residual ? fma2(w0, x0, x0) : mul2(w0, x0);
                a1 = residual ? fma2(w1, x1, x1) : mul2(w1, x1);
              }
#pragma unroll
              for (int w = 1; w < W; ++w) {
                const uint32_t* dw = reinterpret_cast<const uint32_t*>(&xr[w]) + 2 * hh;
                a0 = fma2(make_float2(v[w][0], v[w][1]), make_float2(bf_lo(dw[0]), bf_hi(dw[0])), a0);
                a1 = fma2(make_float2(v[w][2], v[w][3]), make_float2(bf_lo(dw[1]), bf_hi(dw[1])), a1);
              }
              p0 = pack_bf16x2(a0.x, a0.y);
              p1 = pack_bf16x2(a1.x, a1.y);
            };
            ld_w(wa, 0, 0);
            // both 8-channel groups' x rows t-W+1 .. t, loaded before any store
            uint4 xr[2][W];
#pragma unroll
            for (int cgi = 0; cgi < 2; ++cgi) {
              const int cc = (j & 1) * 4 + 2 * h + cgi;  // 16-byte chunk within the half tile's 128-byte row
#pragma unroll
              for (int w = 0; w < W; ++w) {
                const int r = t - w + 3;
                xr[cgi][w] = *reinterpret_cast<const uint4*>(xs + r * 128 + ((cc ^ (r & 7)) << 4));
              }
            }
            uint32_t pk[2][4];
#pragma unroll
            for (int cgi = 0; cgi < 2; ++cgi) {
              tmem_ld_wait();  // batch (cgi, 0) in wa
              ld_w(wb2, cgi, 1);
              y4(wa, xr[cgi], 0, pk[cgi][0], pk[cgi][1]);
              tmem_ld_wait();  // batch (cgi, 1) in wb2
              if (cgi == 0) ld_w(wa, 1, 0);
              y4(wb2, xr[cgi], 1, pk[cgi][2], pk[cgi][3]);
            }
#pragma unroll
            for (int cgi = 0; cgi < 2; ++cgi)  // rows of the [32 steps][16 ch] sub-tile, 32-byte swizzle
              *reinterpret_cast<uint4*>(stg + lane * 32 + ((cgi ^ ((lane >> 2) & 1)) << 4)) =
                  make_uint4(pk[cgi][0], pk[cgi][1], pk[cgi][2], pk[cgi][3]);
          }
          fence_proxy_async_smem();  // the y sub-tile, for the TMA store
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&wempty[wb]);
            mbar_arrive(&xempty[s]);
            if (!dead) {
              tma_store_3d(&ymap, stg, d0 + 32 * j + 16 * h, t0 + 32 * q, b, pol_y);  // clipped at T and D
              bulk_commit_group();
            }
          }
        }
      }
      if (lane == 0) bulk_wait_group<0>();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// x, y: [B][T][G*D]; z: [B][T][G*R]; U: [G][R][W*D]; sw: [G][W][D] or null.
template <int W, int RKP>
int launch_ft(const void* x, const void* z, const void* U, const void* sw, void* y, void* ws, int64_t B, int64_t T,
              int64_t D, int G, int R, int residual, cudaStream_t st) {
  using L = FtCfg<W, RKP>;
  const int64_t Dt = (int64_t)G * D;
  CUtensorMap xmap, zmap;
  int s;
  if ((s = make_btd_map(&xmap, x, B, T, Dt, 64, kRowsX, 128))) return s;
  CUtensorMap ymap;
  if ((s = make_btd_map(&ymap, y, B, T, Dt, 16, 32, 32))) return s;  // per-warp [32 steps][16 ch] stores
  if ((s = make_zpack_map(&zmap, ws, B, T, RKP, kZR, G))) return s;
  if ((s = z_pack_launch(z, ws, B, T, R, RKP, sw != nullptr, st, G))) return s;
  FtSplit sp;
  sp.n_dblk = (int)((Dt + kBD - 1) / kBD);
  sp.tiles_row = (int)((T + kTT - 1) / kTT);
  sp.n_tiles = (int)(B * sp.tiles_row);
  sp.n_units = (int64_t)sp.n_dblk * sp.n_tiles;
  const ChanGroups cg = chan_groups(D, G);
  const int64_t grid = sp.n_units < sm_count() ? sp.n_units : sm_count();
  const int smem = (int)L::kTotal;
  cudaError_t e = cudaFuncSetAttribute(lr_fwd_tm_kernel<W, RKP>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) {
    cudaGetLastError();  // do not leave the failure pending for the next launch check
    return cuda_status(e, "cudaFuncSetAttribute(lr_fwd_tm)");
  }
  lr_fwd_tm_kernel<W, RKP><<<(unsigned)grid, kThreads, smem, st>>>(
      xmap, zmap, ymap, (const __nv_bfloat16*)U, (const __nv_bfloat16*)sw, sp, cg, (int)T, (int)Dt, R, residual);
  DYNCONV_CHECK_LAUNCH("lr_fwd_tm_kernel");
  return DYNCONV_OK;
}

template <int RKP>
int launch_ft_w(int W, const void* x, const void* z, const void* U, const void* sw, void* y, void* ws, int64_t B,
                int64_t T, int64_t D, int G, int R, int residual, cudaStream_t st) {
  switch (W) {
    case 1: return launch_ft<1, RKP>(x, z, U, sw, y, ws, B, T, D, G, R, residual, st);
    case 2: return launch_ft<2, RKP>(x, z, U, sw, y, ws, B, T, D, G, R, residual, st);
    case 3: return launch_ft<3, RKP>(x, z, U, sw, y, ws, B, T, D, G, R, residual, st);
    case 4: return launch_ft<4, RKP>(x, z, U, sw, y, ws, B, T, D, G, R, residual, st);
    default: return set_error(DYNCONV_ERR_UNSUPPORTED, "tensor-core path: W=%d", W);
  }
}

}  // namespace

// Time-major tensor-core forward; the workspace holds z_pack (lr_tc_fwd_workspace).
int lr_tm_fwd_launch(const void* x, const void* z, const void* U, const void* sw, void* y, void* ws, int64_t B,
                     int64_t T, int64_t D, int G, int R, int Rk, int W, int residual, cudaStream_t st) {
  const int rkp = (Rk + 15) / 16 * 16;
  switch (rkp) {
    case 16: return launch_ft_w<16>(W, x, z, U, sw, y, ws, B, T, D, G, R, residual, st);
    case 32: return launch_ft_w<32>(W, x, z, U, sw, y, ws, B, T, D, G, R, residual, st);
    case 48: return launch_ft_w<48>(W, x, z, U, sw, y, ws, B, T, D, G, R, residual, st);
    case 64: return launch_ft_w<64>(W, x, z, U, sw, y, ws, B, T, D, G, R, residual, st);
    default: return set_error(DYNCONV_ERR_UNSUPPORTED, "R_kernel=%d", Rk);
  }
}

}  // namespace dynconv
