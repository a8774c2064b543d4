// lowrank_bwd_tm.cu -- fused tcgen05 backward of the lowrank dynamic convolution,
// bf16, time-major.
//
// Reference behaviour: the dU/dz kernel (lowrank.py:86-140) and the dx kernel
// (lowrank.py:158-205), launched by _LowrankDynamicConvolutionFn.backward
// (lowrank.py:252-299); oracle reference.py:23-39.  One pass over dy and x computes
// dx, dz, dU and dstatic_w (the reference reads dy twice, in two kernels).
//
// Math, per step t and channel ch (z_ext = z plus the static rank, U_ext likewise):
//   Wt_w[t,ch] = sum_r z_ext[t,r] U_ext[r,w,ch]                      (dynamic weights)
//   dx[t,ch]   = sum_w dy[t+w,ch] Wt_w[t+w,ch]  (+ dy[t,ch] if residual)
//   P_w[t,ch]  = bf16(dy[t,ch] x[t-w,ch])      (bf16 product, as lowrank.py:128)
//   dU[r,w,ch] = sum_t z_ext[t,r] P_w[t,ch]     dz[t,r] = sum_{w,ch} P_w[t,ch] U_ext[r,w,ch]
//
// Orientation: tensor-memory lane = timestep.  A tile is 128 steps (the M = 128
// of the weight and dz MMAs) x 128 channels, handled as four 32-channel chunks.
// The weight MMA of tap w reads the z tile from row w, so it writes
// D[t][ch] = Wt_w[t+w, ch] -- the weight that dx[t] needs -- with no transpose:
// each epilogue thread owns one step and reads its dy and x rows (16 bytes = 8
// channels per load, conflict-free in the 128-byte-swizzled TMA tiles).
//
// Per chunk (32 channels x 128 steps):
//   weight MMA  D[t][ch] per tap, M = 128, N = 32, K = R_kernel       (A = z rows t+w,
//               K-major; B = U tap w, MN-major)
//   epilogue    dx -> HBM (16-byte stores), P_w -> shared memory in 8 x 8 blocks laid
//               out [step/8][tap][ch/8][8 steps][8 ch]
//   dz MMA      D[t][r] += P_w[t][ch] U[r,w,ch], M = 128, N = R_kernel, K = 16 (tap, ch)
//               per instruction (A = P read K-major)
//   dU MMA      D[(w,ch)][r] += P_w[t][ch] z[t][r], M = 128 = 4 taps x 32 channels,
//               N = R_kernel, K = 16 steps per instruction (A = the same P read MN-major,
//               B = z MN-major); one accumulator per chunk position, kept in tensor
//               memory over every tile of the CTA
// 40 MMAs per 8192 (step, channel) pairs at R_kernel <= 16.
//
// Warps: 0 producer (TMA: z per tile, dy and x per 64-channel half tile into a
// ring), 1 weight MMAs + TMEM owner, 2/3 dz MMAs and 4/5 dU MMAs of chunk parity
// 0/1 (separate dz accumulators, summed at readout), 6..21 the epilogue in two teams of eight (team = chunk parity; a warp has 32 steps of its
// TMEM lane quarter and 16 channels of the chunk).  The dz partial of this CTA's
// 128 channels goes to the workspace and is summed across channel blocks after a
// grid-wide count (cooperative launch), as is dU across token groups.  Every wait
// is bounded (common.cuh); a wait that gives up marks the CTA dead and the kernel
// unwinds, still arriving on the barriers it owns.
#include "lowrank_tc.cuh"

namespace dynconv {

DYNCONV_DEFINE_ERROR_ACCESSOR(lr_bwd_tm_error_word)

namespace {

using namespace lrtc;

constexpr int kTT = 128;               // steps per tile
constexpr int kCh = 32;                // channels per chunk
constexpr int kRowsXY = kTT + 3;       // rows of a dy / x box (W - 1 <= 3 halo rows)
constexpr int kZR = 136;               // z rows per tile (128 + W - 1, padded)
constexpr int kCtl = 6;                // producer + five MMA issuers
constexpr int kEpi = 16;               // epilogue warps
constexpr int kThreads = 32 * (kCtl + kEpi);

template <int W, int RKP>
struct TmCfg {
  static constexpr int S = RKP == 16 ? 3 : 2;     // ring of dy/x half tiles (64 channels)
  static constexpr int NWB = RKP == 16 ? 3 : 2;   // weight buffers in tensor memory
  static constexpr uint32_t kBox = (uint32_t)kRowsXY * 128;  // one 64-channel box, 128-byte rows
  static constexpr uint32_t kBoxStride = round1024(kBox);
  static constexpr uint32_t kSlot = 2 * kBoxStride;        // dy box, then x box
  static constexpr uint32_t kPBuf = 4u * kTT * kCh * 2;    // 4 taps x 128 steps x 32 channels
  static constexpr uint32_t kUcg = (RKP / 8) * 128;        // U: next 8 channels
  static constexpr uint32_t kUTap = 16 * kUcg;             // U: next tap
  static constexpr uint32_t kLZ = kZR * 16;                // z: next 8 ranks
  static constexpr uint32_t kZBytes = (RKP / 8) * kLZ;
  static constexpr uint32_t kOffRing = 0;
  static constexpr uint32_t kOffP = kOffRing + S * kSlot;
  static constexpr uint32_t kOffU = kOffP + 2 * kPBuf;
  static constexpr uint32_t kOffZ = kOffU + W * kUTap;
  static constexpr uint32_t kStage = 32 * 16 * 2;                  // one warp's dx sub-tile [32 steps][16 ch]
  static constexpr uint32_t kOffStage = (kOffZ + 2 * kZBytes + 255u) / 256u * 256u;  // 32-byte swizzle: 256-aligned
  static constexpr uint32_t kTotal = kOffStage + kEpi * 2 * kStage + 1024;  // + alignment slack
  // tensor-memory columns
  static constexpr uint32_t kColW = 0;               // NWB buffers x (4 taps x 32 channels)
  static constexpr uint32_t kColDZ = NWB * 128;      // [team][tile buffer] x RKP
  static constexpr uint32_t kColDU = kColDZ + 4 * RKP;  // [chunk position] x RKP
  static_assert(kColDU + 4 * RKP <= 512, "tensor-memory budget");
  static_assert(kTotal <= 232448 - 512, "shared-memory budget (227 KB per CTA, static part aside)");
};

template <int N>
__device__ __forceinline__ void tmem_ld_n(uint32_t taddr, float (&v)[N]) {
  static_assert(N == 4 || N == 8 || N == 16, "");
  if constexpr (N == 4) tmem_ld4(taddr, v);
  else if constexpr (N == 8) tmem_ld8(taddr, v);
  else tmem_ld16(taddr, v);
}

// bf16 pair -> two floats (exact)
__device__ __forceinline__ float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

struct TmSplit {
  int n_dblk, n_groups, tiles_row, n_tiles;
};

inline TmSplit tm_split(int64_t B, int64_t T, int64_t D) {
  TmSplit sp;
  sp.n_dblk = (int)((D + kBD - 1) / kBD);
  sp.tiles_row = (int)((T + kTT - 1) / kTT);
  sp.n_tiles = (int)(B * sp.tiles_row);
  int ng = sm_count() / sp.n_dblk;
  if (ng < 1) ng = 1;
  if (ng > sp.n_tiles) ng = sp.n_tiles;
  sp.n_groups = ng;
  return sp;
}

template <int W, int RKP>
__global__ void __launch_bounds__(kThreads, 1)
    lr_bwd_tm_kernel(const __grid_constant__ CUtensorMap dymap, const __grid_constant__ CUtensorMap xmap,
                     const __grid_constant__ CUtensorMap zmap, const __grid_constant__ CUtensorMap dxmap,
                     const __nv_bfloat16* __restrict__ U, const __nv_bfloat16* __restrict__ sw,
                     __nv_bfloat16* __restrict__ dz, float* __restrict__ dzp, int* __restrict__ grp_done,
                     float* __restrict__ dUp, float* __restrict__ dU_f32, __nv_bfloat16* __restrict__ dU,
                     __nv_bfloat16* __restrict__ dsw, TmSplit sp, ChanGroups cg, int T, int D, int R, int Rk,
                     int residual, const __grid_constant__ DpPeers peers) {
  // D: channels of an activation row (G * Dg); cg.Dg: channels of one group's U
  using L = TmCfg<W, RKP>;
  constexpr int S = L::S, NWB = L::NWB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  __shared__ uint64_t rfull[S], rempty[S], zfull[2], zempty[2], wfull[NWB], wempty[NWB], pfull[2], pempty[2],
      dzfull[2], dzempty[2], du_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  __shared__ int grp_ok;
  __shared__ unsigned long long dp_epoch_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dblk = blockIdx.x % sp.n_dblk;
  const int g = blockIdx.x / sp.n_dblk;
  const int j0 = (int)((int64_t)sp.n_tiles * g / sp.n_groups);
  const int j1 = (int)((int64_t)sp.n_tiles * (g + 1) / sp.n_groups);
  const int n = j1 - j0;
  const int d0 = dblk * kBD;         // first channel in the activation row
  const int grp = dblk / cg.nd;      // channel group of this CTA's block
  const int dl0 = d0 - grp * cg.Dg;  // first channel within the group

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&rfull[s], 1);
      mbar_init(&rempty[s], kEpi);  // both teams read every half tile
    }
    for (int b2 = 0; b2 < 2; ++b2) {
      mbar_init(&zfull[b2], 1);
      mbar_init(&zempty[b2], 3);    // the weight MMAs and both dU issuers of the tile
      mbar_init(&pfull[b2], kEpi / 2);
      mbar_init(&pempty[b2], 2);    // the dz and the dU MMAs of the chunk
      mbar_init(&dzfull[b2], 2);    // both dz issuers
      mbar_init(&dzempty[b2], kEpi);
    }
    for (int c = 0; c < NWB; ++c) {
      mbar_init(&wfull[c], 1);
      mbar_init(&wempty[c], kEpi / 2);
    }
    mbar_init(&du_bar, 2);
    abort_flag = 0;
    // data-parallel call counter and the float4s each source has delivered so far (calls
    // may differ in size); read before any CTA of this launch advances them
    dp_epoch_s = peers.world > 1 ? *reinterpret_cast<volatile unsigned long long*>(peers.epoch) : 0ull;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&dymap);
    prefetch_tensormap(&xmap);
    prefetch_tensormap(&zmap);
    prefetch_tensormap(&dxmap);
  }
  __syncthreads();  // barriers initialised: the producer starts its loads at once
  const unsigned long long dp_epoch = dp_epoch_s;
  uint32_t tmem = 0;
  if (warp != 0) {
    constexpr int kNonProducer = kThreads - 32;
    load_u_mn<W, RKP, kNonProducer>(smem + L::kOffU, U + (size_t)grp * R * W * cg.Dg,
                                    sw ? sw + (size_t)grp * W * cg.Dg : nullptr, dl0, cg.Dg, R, threadIdx.x - 32);
    fence_proxy_async_smem();
    if (warp == 1) {
      tmem_alloc(&tmem_slot, 512);
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
      const uint64_t pol_z = policy_evict_normal();  // z rows are read by every channel block
      int hs = 0;
      for (int k = 0; k < n; ++k) {
        const int tile = j0 + k, b = tile / sp.tiles_row, t0 = (tile % sp.tiles_row) * kTT;
        if (!mbar_wait(&zempty[k & 1], ((k >> 1) & 1) ^ 1, kErrWaitProducer, &abort_flag)) break;
        mbar_arrive_expect_tx(&zfull[k & 1], L::kZBytes);
        tma_load_4d(smem + L::kOffZ + (k & 1) * L::kZBytes, &zmap, &zfull[k & 1], 0, t0, b, grp * (RKP / 8), pol_z);
        bool ok = true;
        for (int half = 0; half < 2; ++half, ++hs) {
          const int s = hs % S;
          if (!mbar_wait(&rempty[s], ((hs / S) & 1) ^ 1, kErrWaitProducer, &abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* slot = smem + L::kOffRing + s * L::kSlot;
          mbar_arrive_expect_tx(&rfull[s], 2 * L::kBox);
          tma_load_3d(slot, &dymap, &rfull[s], d0 + 64 * half, t0, b, pol);                      // rows t0 .. t0+130
          tma_load_3d(slot + L::kBoxStride, &xmap, &rfull[s], d0 + 64 * half, t0 - 3, b, pol);  // t0-3 .. t0+127
        }
        if (!ok) break;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ weight MMAs
    const uint32_t idesc = make_idesc_bf16(kTT, kCh, 0, 1);  // A = z (K-major), B = U (MN-major)
    const uint32_t ub = smem_u32(smem + L::kOffU);
    const uint32_t zb0 = smem_u32(smem + L::kOffZ);
    for (int k = 0; k < n; ++k) {
      if (!mbar_wait(&zfull[k & 1], (k >> 1) & 1, kErrWaitMma, &abort_flag)) break;
      const uint32_t zb = zb0 + (k & 1) * L::kZBytes;
      bool ok = true;
      for (int j = 0; j < 4; ++j) {
        const int c = 4 * k + j, wb = c % NWB;
        if (!mbar_wait(&wempty[wb], ((c / NWB) & 1) ^ 1, kErrWaitMma, &abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
#pragma unroll
          for (int w = 0; w < W; ++w) {
#pragma unroll
            for (int ks = 0; ks < RKP / 16; ++ks) {
              const uint64_t ad = make_smem_desc(zb + w * 16 + ks * 2 * L::kLZ, L::kLZ, 128);
              const uint64_t bd = make_smem_desc(ub + w * L::kUTap + 4 * j * L::kUcg + ks * 256, 128, L::kUcg);
              umma_f16(tmem + L::kColW + wb * 128 + w * kCh, ad, bd, idesc, ks > 0 ? 1u : 0u);
            }
          }
          umma_commit(&wfull[wb]);
          if (j == 3) umma_commit(&zempty[k & 1]);
        }
        __syncwarp();
      }
      if (!ok) break;
    }
  } else if (warp >= 2 && warp <= 5) {
    // ------------------------------------------------------------ dz (warps 2/3) and dU (4/5) MMAs of
    // chunk parity tau: separate issuers, so a chunk's 16 MMAs go out in two parallel streams
    const bool is_dz = warp < 4;
    const int tau = (warp - 2) & 1;
    const uint32_t idesc = is_dz ? make_idesc_bf16(kTT, RKP, 0, 0)   // dz: A = P (K-major), B = U (K-major)
                                 : make_idesc_bf16(kTT, RKP, 1, 1);  // dU: A = P (MN-major), B = z (MN-major)
    const uint32_t pb = smem_u32(smem + L::kOffP + tau * L::kPBuf);
    const uint32_t ub = smem_u32(smem + L::kOffU);
    const uint32_t zb0 = smem_u32(smem + L::kOffZ);
    int m = 0;
    for (int k = 0; k < n; ++k) {
      bool ok = true;
      for (int j = tau; j < 4; j += 2, ++m) {
        if (!mbar_wait(&pfull[tau], m & 1, kErrWaitMma, &abort_flag) ||
            (j == tau && is_dz && !mbar_wait(&dzempty[k & 1], ((k >> 1) & 1) ^ 1, kErrWaitMma, &abort_flag)) ||
            (j == tau && !is_dz && !mbar_wait(&zfull[k & 1], (k >> 1) & 1, kErrWaitMma, &abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          if (is_dz) {
            const uint32_t dacc = tmem + L::kColDZ + (tau * 2 + (k & 1)) * RKP;
#pragma unroll
            for (int w = 0; w < W; ++w) {
#pragma unroll
              for (int h2 = 0; h2 < 2; ++h2) {
                const uint64_t ad = make_smem_desc(pb + (w * 4 + 2 * h2) * 128, 128, 2048);
                const uint64_t bd = make_smem_desc(ub + w * L::kUTap + (4 * j + 2 * h2) * L::kUcg, L::kUcg, 128);
                umma_f16(dacc, ad, bd, idesc, (j == tau && w == 0 && h2 == 0) ? 0u : 1u);
              }
            }
            umma_commit(&pempty[tau]);
            if (j == tau + 2) umma_commit(&dzfull[k & 1]);
          } else {
            const uint32_t uacc = tmem + L::kColDU + j * RKP;
            const uint32_t zb = zb0 + (k & 1) * L::kZBytes;
#pragma unroll
            for (int s8 = 0; s8 < kTT / 16; ++s8) {
              const uint64_t ad = make_smem_desc(pb + s8 * 4096, 2048, 128);
              const uint64_t bd = make_smem_desc(zb + s8 * 256, 128, L::kLZ);
              umma_f16(uacc, ad, bd, idesc, (k == 0 && s8 == 0) ? 0u : 1u);
            }
            umma_commit(&pempty[tau]);
            if (j == tau + 2) umma_commit(&zempty[k & 1]);
          }
        }
        __syncwarp();
      }
      if (!ok) break;
    }
    if (!is_dz && lane == 0) umma_commit(&du_bar);
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int e = warp - kCtl;   // 0..15
    const int q = warp & 3;      // TMEM lane quarter = 32-step quarter of the tile
    const int tau = e >> 3;      // team: chunks of this parity
    const int h = (e >> 2) & 1;  // 16-channel half of the chunk
    const int sub = e >> 2;      // 0..3: column slice of the dz readout, chunk position of the dU readout
    const int t = 32 * q + lane;  // step within the tile
    const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16);
    uint8_t* const pbuf = smem + L::kOffP + tau * L::kPBuf + (t >> 3) * 2048 + (t & 7) * 16;
    bool dead = false;

    // dz partial of tile kk (both parities' accumulators added) -> workspace
    auto dz_readout = [&](int kk) {
      const int tile = j0 + kk;
      if (!dead) dead = !mbar_wait(&dzfull[kk & 1], (kk >> 1) & 1, kErrWaitEpilogue, &abort_flag);
      tc_fence_after();
      constexpr int NC = RKP / 4;
      float v[NC], v2[NC];
      const int c0 = sub * NC;
      if (!dead) {
        const uint32_t a0 = ta + L::kColDZ + (kk & 1) * RKP + c0;
        tmem_ld_n<NC>(a0, v);
        tmem_ld_n<NC>(a0 + 2 * RKP, v2);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < NC; ++c) v[c] += v2[c];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dzempty[kk & 1]);
      if (!dead) {
        float* dst = dzp + (((size_t)dblk * sp.n_tiles + tile) * kTT + t) * RKP + c0;
#pragma unroll
        for (int c = 0; c < NC; c += 4) *reinterpret_cast<float4*>(dst + c) = make_float4(v[c], v[c + 1], v[c + 2], v[c + 3]);
      }
    };

    const uint64_t pol_dx = policy_evict_first();
    int m = 0;
    for (int k = 0; k < n; ++k) {
      const int tile = j0 + k, b = tile / sp.tiles_row, t0 = (tile % sp.tiles_row) * kTT;
      for (int j = tau; j < 4; j += 2, ++m) {
        const int c = 4 * k + j, wb = c % NWB, hs = 2 * k + (j >> 1), s = hs % S;
        if (!dead) dead = !mbar_wait(&wfull[wb], (c / NWB) & 1, kErrWaitEpilogue, &abort_flag);
        if (!dead) dead = !mbar_wait(&rfull[s], (hs / S) & 1, kErrWaitEpilogue, &abort_flag);
        tc_fence_after();
        // this warp's dx sub-tile buffer (m & 1) is free once its store of chunk m-2 has read it
        uint8_t* const stg = smem + L::kOffStage + (e * 2 + (m & 1)) * L::kStage;
        if (lane == 0 && !dead) bulk_wait_group_read<1>();
        __syncwarp();
        const uint8_t* dys = smem + L::kOffRing + s * L::kSlot;
        const uint8_t* xs = dys + L::kBoxStride;
        // ---- dx (needs the weights and dy): first, while the MMAs of this team's previous
        // chunk may still be reading its P buffer
        if (!dead) {
          const uint32_t wcol = ta + L::kColW + wb * 128 + 16 * h;  // this warp's 16 channels, tap 0
          // The weights arrive in four batches (8-channel group cgi, 4-channel half hh) of
          // W x 4 values.  Each batch's tensor-memory load is issued one step ahead, so
          // its latency overlaps the dy loads or the previous batch's dx.
          float wa[W][4], wb2[W][4];
          auto ld_w = [&](float (&v)[W][4], int cgi, int hh) {
#pragma unroll
            for (int w = 0; w < W; ++w) tmem_ld4(wcol + w * kCh + cgi * 8 + 4 * hh, v[w]);
          };
          // dx[t] for 4 channels = sum_w Wt_w[t+w] dy[t+w] (+ dy[t]) -> two bf16 pairs
          auto dx4 = [&](const float (&v)[W][4], const uint4 (&dyr)[W], int hh, uint32_t& p0, uint32_t& p1) {
            // packed f32x2 arithmetic on channel pairs (each lane rounds like the scalar op)
            const uint32_t* d = reinterpret_cast<const uint32_t*>(&dyr[0]) + 2 * hh;
            float2 a0, a1;
            {
              const float2 x0 = make_float2(bf_lo(d[0]), bf_hi(d[0])), x1 = make_float2(bf_lo(d[1]), bf_hi(d[1]));
              const float2 w0 = make_float2(v[0][0], v[0][1]), w1 = make_float2(v[0][2], v[0][3]);
              a0 = residual ? fma2(w0, x0, x0) : mul2(w0, x0);
              a1 = residual ? fma2(w1, x1, x1) : mul2(w1, x1);
            }
#pragma unroll
            for (int w = 1; w < W; ++w) {
              const uint32_t* dw = reinterpret_cast<const uint32_t*>(&dyr[w]) + 2 * hh;
              a0 = fma2(make_float2(v[w][0], v[w][1]), make_float2(bf_lo(dw[0]), bf_hi(dw[0])), a0);
              a1 = fma2(make_float2(v[w][2], v[w][3]), make_float2(bf_lo(dw[1]), bf_hi(dw[1])), a1);
            }
            p0 = pack_bf16x2(a0.x, a0.y);
            p1 = pack_bf16x2(a1.x, a1.y);
          };
          ld_w(wa, 0, 0);
          // both 8-channel groups' dy rows t .. t+W-1, loaded before any store
          uint4 dyr[2][W];
#pragma unroll
          for (int cgi = 0; cgi < 2; ++cgi) {
            const int cc = (j & 1) * 4 + 2 * h + cgi;  // 16-byte chunk within the half tile's 128-byte row
#pragma unroll
            for (int w = 0; w < W; ++w) {
              const int r = t + w;
              dyr[cgi][w] = *reinterpret_cast<const uint4*>(dys + r * 128 + ((cc ^ (r & 7)) << 4));
            }
          }
          uint32_t pk[2][4];
#pragma unroll
          for (int cgi = 0; cgi < 2; ++cgi) {
            tmem_ld_wait();          // batch (cgi, 0) in wa
            ld_w(wb2, cgi, 1);
            dx4(wa, dyr[cgi], 0, pk[cgi][0], pk[cgi][1]);
            tmem_ld_wait();          // batch (cgi, 1) in wb2
            if (cgi == 0) ld_w(wa, 1, 0);
            dx4(wb2, dyr[cgi], 1, pk[cgi][2], pk[cgi][3]);
          }
#pragma unroll
          for (int cgi = 0; cgi < 2; ++cgi)  // rows of the [32 steps][16 ch] sub-tile, 32-byte swizzle
            *reinterpret_cast<uint4*>(stg + lane * 32 + ((cgi ^ ((lane >> 2) & 1)) << 4)) =
                make_uint4(pk[cgi][0], pk[cgi][1], pk[cgi][2], pk[cgi][3]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&wempty[wb]);  // the weights are in registers: the buffer is free
        // ---- P_w[t] = bf16(dy[t] * x[t-w]) -> block (t/8, w, cgc) of the team's P buffer, once
        // the MMAs of the team's previous chunk are done with it
        if (!dead) dead = !mbar_wait(&pempty[tau], (m & 1) ^ 1, kErrWaitEpilogue, &abort_flag);
        if (!dead) {
          // every load of the section first (the compiler cannot move a load above a store
          // into the same shared memory), then the products and the stores
          uint4 d0v[2], xr[2][W];
#pragma unroll
          for (int cgi = 0; cgi < 2; ++cgi) {
            const int cc = (j & 1) * 4 + 2 * h + cgi;
            d0v[cgi] = *reinterpret_cast<const uint4*>(dys + t * 128 + ((cc ^ (t & 7)) << 4));
#pragma unroll
            for (int w = 0; w < W; ++w) {
              const int r = t - w + 3;
              xr[cgi][w] = *reinterpret_cast<const uint4*>(xs + r * 128 + ((cc ^ (r & 7)) << 4));
            }
          }
#pragma unroll
          for (int cgi = 0; cgi < 2; ++cgi) {
#pragma unroll
            for (int w = 0; w < W; ++w)
              *reinterpret_cast<uint4*>(pbuf + (w * 4 + 2 * h + cgi) * 128) =
                  make_uint4(mul_bf16x2(d0v[cgi].x, xr[cgi][w].x), mul_bf16x2(d0v[cgi].y, xr[cgi][w].y),
                             mul_bf16x2(d0v[cgi].z, xr[cgi][w].z), mul_bf16x2(d0v[cgi].w, xr[cgi][w].w));
          }
        }
        fence_proxy_async_smem();  // P and the dx sub-tile, for the MMAs and the TMA store
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&pfull[tau]);
          mbar_arrive(&rempty[s]);
          if (!dead) {
            tma_store_3d(&dxmap, stg, d0 + 32 * j + 16 * h, t0 + 32 * q, b, pol_dx);  // clipped at T and D
            bulk_commit_group();
          }
        }
        if (j == tau && k >= 1) dz_readout(k - 1);  // the previous tile's dz, once this team has moved on
      }
    }
    if (n >= 1) dz_readout(n - 1);
    if (lane == 0) bulk_wait_group<0>();
    // dU partial of this CTA: lane (w, ch) of chunk position `sub` -> dUp[g][grp][r][w*Dg + d]
    if (!dead) dead = !mbar_wait(&du_bar, 0, kErrWaitTail, &abort_flag);
    tc_fence_after();
    if (!dead && q < W) {
      float v[RKP];
      if constexpr (RKP == 16) {
        tmem_ld16(ta + L::kColDU + sub * RKP, v);
      } else {
        float v0[16], v1[16];
        tmem_ld16(ta + L::kColDU + sub * RKP, v0);
        tmem_ld16(ta + L::kColDU + sub * RKP + 16, v1);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          v[i] = v0[i];
          v[16 + i] = v1[i];
        }
      }
      tmem_ld_wait();
      const int dlc = dl0 + kCh * sub + lane;
      if (dlc < cg.Dg) {
#pragma unroll
        for (int r = 0; r < RKP; ++r)
          if (r < Rk) dUp[(((size_t)g * cg.G + grp) * Rk + r) * W * cg.Dg + (size_t)q * cg.Dg + dlc] = v[r];
      }
    }
  }

  // ---------------------------------------------------------------- tail
  // Publish this CTA's dz and dU partials (CTA barrier, then one cumulative gpu-scope
  // fence) on two counters: its token group's and the grid's.  Single rank: wait for
  // the group's other channel-block CTAs (co-resident: cooperative launch), reduce dz,
  // then wait for the grid and reduce dU.  Data parallel: wait for the grid at once,
  // reduce dU and post this rank's sums to every peer, reduce dz while they travel,
  // and only then wait for the peers' sums.
  const bool dp = peers.world > 1;
  const int par = (int)(dp_epoch & 1);
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(&grp_done[g], 1);
    atomicAdd(&grp_done[sp.n_groups], 1);
    grp_ok = abort_flag ? 0 : 1;
  }
  // bounded wait (thread 0) until *cnt reaches target; grp_ok = 0 on time-out
  auto wait_count = [&](const int* cnt, int target) {
    if (threadIdx.x == 0) {
      bool ok = grp_ok != 0;
      if (ok) {
        const volatile int* c = cnt;
        const uint64_t tstart = globaltimer_ns();
        while (*c < target) {
          if (globaltimer_ns() - tstart > kWaitLimitNs) {
            record_device_error(kErrWaitTail);
            ok = false;
            break;
          }
        }
      }
      __threadfence();
      grp_ok = ok ? 1 : 0;
    }
    __syncthreads();
  };

  // dz: this CTA's share of the group's (step, channel group) pairs, summed over the
  // channel blocks in order: deterministic, evenly spread
  auto dz_reduce = [&]() {
    if (!grp_ok) return;
    const int64_t npairs = (int64_t)n * kTT * cg.G;
    const int64_t lo = npairs * dblk / sp.n_dblk, hi = npairs * (dblk + 1) / sp.n_dblk;
    constexpr int RQ = RKP / 4;  // float4 groups per step
    const int RG = cg.G * R;     // dz row width
    for (int64_t e2 = lo * RQ + threadIdx.x; e2 < hi * RQ; e2 += blockDim.x) {
      const int64_t sg = e2 / RQ;
      const int rq = (int)(e2 % RQ);
      const int64_t st = sg / cg.G;
      const int go = (int)(sg - st * cg.G);
      const int tile = j0 + (int)(st / kTT), tok = (int)(st % kTT);
      const int b = tile / sp.tiles_row, t = (tile % sp.tiles_row) * kTT + tok;
      if (t >= T) continue;
      float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f);
      const int kb = go * cg.nd;
#pragma unroll 4
      for (int k2 = kb; k2 < kb + cg.nd; ++k2) {  // partial loads in flight, summed in order
        const float4 f =
            __ldcg(reinterpret_cast<const float4*>(dzp + (((size_t)k2 * sp.n_tiles + tile) * kTT + tok) * RKP) + rq);
        a4.x += f.x;
        a4.y += f.y;
        a4.z += f.z;
        a4.w += f.w;
      }
      __nv_bfloat16* dst = dz + ((size_t)b * T + t) * RG + go * R;
      const float av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (4 * rq + c < R) dst[4 * rq + c] = __float2bfloat16_rn(av[c]);
    }
  };

  if (!dp) {
    wait_count(grp_done + g, sp.n_dblk);
    dz_reduce();
  }
  wait_count(grp_done + sp.n_groups, (int)gridDim.x);

  // dU: CTA i sums its 1/grid slice of the [G][Rk][W*Dg] accumulator over the token
  // groups in group order (deterministic) and writes dU_f32, and the bf16 dU rows /
  // dstatic_w rows when they are requested.
  const int64_t wd = (int64_t)W * cg.Dg;
  const int64_t per_g = (int64_t)Rk * wd;  // one group's [Rk][W*Dg] block
  const int64_t n4 = cg.G * per_g / 4;     // W*Dg % 4 == 0 (Dg % 8 == 0)
  const int64_t lo = n4 * blockIdx.x / gridDim.x, hi = n4 * (blockIdx.x + 1) / gridDim.x;
  // The final value of element i: fp32 sum, bf16 dU row or dstatic_w row
  auto finish = [&](int64_t i, float4 a4) {
    reinterpret_cast<float4*>(dU_f32)[i] = a4;
    const int64_t e0 = 4 * i;
    const int go = (int)(e0 / per_g);
    const int64_t rem = e0 - go * per_g;
    const int r = (int)(rem / wd);
    const int64_t col = rem - (int64_t)r * wd;
    __nv_bfloat16* dst = r < R ? (dU ? dU + ((int64_t)go * R + r) * wd + col : nullptr)
                               : (dsw ? dsw + (int64_t)go * wd + col : nullptr);
    if (dst) {
      dst[0] = __float2bfloat16_rn(a4.x);
      dst[1] = __float2bfloat16_rn(a4.y);
      dst[2] = __float2bfloat16_rn(a4.z);
      dst[3] = __float2bfloat16_rn(a4.w);
    }
  };
  if (grp_ok) {
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
      float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
      for (int gg = 0; gg < sp.n_groups; ++gg) {
        const float4 f = __ldcg(reinterpret_cast<const float4*>(dUp) + (size_t)gg * n4 + i);
        a4.x += f.x;
        a4.y += f.y;
        a4.z += f.z;
        a4.w += f.w;
      }
      if (!dp) {
        finish(i, a4);
      } else {
        // this rank's sum of element i -> slot [par][rank] of every rank's landing buffer
        const int64_t off = ((int64_t)par * peers.world + peers.rank) * peers.cap / 4 + i;
        for (int p2 = 0; p2 < peers.world; ++p2) reinterpret_cast<float4*>(peers.land[p2])[off] = a4;
      }
    }
  }
  if (dp) {
    // Publish: every thread's peer stores, then one system-scope fence per thread,
    // the CTA barrier, and this call's number in flag [rank][this CTA] of every rank.
    // While the stores travel, reduce dz (the grid-wide wait above covers the token
    // group's).  Then wait until flag [src][this CTA] shows this call for every
    // source -- CTA i of every rank owns the same slice [lo, hi) -- and sum the world
    // sources in rank order: the same order on every rank, so all ranks hold
    // bit-identical results.
    const unsigned long long call = dp_epoch + 1;
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0 && grp_ok)
      for (int p2 = 0; p2 < peers.world; ++p2)
        reinterpret_cast<volatile unsigned long long*>(peers.flags[p2])[peers.rank * kMaxDpCtas + blockIdx.x] = call;
    dz_reduce();
    __syncthreads();
    if (threadIdx.x == 0) {
      bool ok = grp_ok != 0;
      const uint64_t tstart = globaltimer_ns();
      for (int src = 0; ok && src < peers.world; ++src) {
        const volatile unsigned long long* f = peers.flags[peers.rank] + src * kMaxDpCtas + blockIdx.x;
        while (*f < call) {
          if (globaltimer_ns() - tstart > kWaitLimitNs) {
            record_device_error(kErrWaitTail);
            ok = false;
            break;
          }
        }
      }
      __threadfence_system();
      grp_ok = ok ? 1 : 0;
    }
    __syncthreads();
    if (grp_ok) {
      const float4* own = reinterpret_cast<const float4*>(peers.land[peers.rank]);
      for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int src = 0; src < peers.world; ++src) {
          const float4 f = __ldcg(own + ((int64_t)par * peers.world + src) * peers.cap / 4 + i);
          a4.x += f.x;
          a4.y += f.y;
          a4.z += f.z;
          a4.w += f.w;
        }
        finish(i, a4);
      }
      // one CTA advances the call count; every CTA of this launch read it at the start
      if (blockIdx.x == 0 && threadIdx.x == 0) *peers.epoch = call;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

struct TmWorkspace {
  float* dzp;
  int* cnt;
  float* dUp;
  void* zp;
  size_t bytes;
};

size_t al256(size_t v) { return (v + 255) / 256 * 256; }

int rkp_of(int Rk) { return Rk <= 16 ? 16 : 32; }

// D: channels per group; the activation rows hold G * D.
TmWorkspace tm_workspace(void* base, int64_t B, int64_t T, int64_t D, int Rk, int W, int G) {
  const TmSplit sp = tm_split(B, T, (int64_t)G * D);
  const int rkp = rkp_of(Rk);
  TmWorkspace w;
  const size_t dzp = al256((size_t)sp.n_dblk * sp.n_tiles * kTT * rkp * sizeof(float));
  const size_t cnt = al256((size_t)(sp.n_groups + 1) * sizeof(int));  // group counts + grid count
  const size_t dUp = al256((size_t)sp.n_groups * G * Rk * W * D * sizeof(float));
  const size_t zp = zpack_bytes(B, T, rkp, G);
  uint8_t* p = (uint8_t*)base;
  w.dzp = (float*)p;
  w.cnt = (int*)(p ? p + dzp : nullptr);
  w.dUp = (float*)(p ? p + dzp + cnt : nullptr);
  w.zp = p ? p + dzp + cnt + dUp : nullptr;
  w.bytes = dzp + cnt + dUp + zp;
  return w;
}

// x, dy, dx: [B][T][G*D]; z, dz: [B][T][G*R]; U, dU: [G][R][W*D]; sw, dsw: [G][W][D];
// dU_f32: [G][Rk][W*D].
template <int W, int RKP>
int launch_tm(const void* x, const void* z, const void* U, const void* sw, const void* dy, void* dx, void* dz,
              float* dU_f32, void* dU, void* dsw, void* wsp, int64_t B, int64_t T, int64_t D, int G, int R, int Rk,
              int residual, const DpPeers& peers, const void* zp_in, cudaStream_t st) {
  using L = TmCfg<W, RKP>;
  CUtensorMap dymap, xmap, zmap;
  int s;
  const int64_t Dt = (int64_t)G * D;
  const TmSplit sp = tm_split(B, T, Dt);
  const ChanGroups cg = chan_groups(D, G);
  TmWorkspace ws = tm_workspace(wsp, B, T, D, Rk, W, G);
  if ((s = make_btd_map(&dymap, dy, B, T, Dt, 64, kRowsXY, 128))) return s;
  if ((s = make_btd_map(&xmap, x, B, T, Dt, 64, kRowsXY, 128))) return s;
  CUtensorMap dxmap;
  if ((s = make_btd_map(&dxmap, dx, B, T, Dt, 16, 32, 32))) return s;  // per-warp [32 steps][16 ch] stores
  // z packed by the forward (same z) is read as it is; otherwise pack it here
  const void* zp = zp_in ? zp_in : ws.zp;
  if ((s = make_zpack_map(&zmap, zp, B, T, RKP, kZR, G))) return s;
  if (!zp_in && (s = z_pack_launch(z, ws.zp, B, T, R, RKP, sw != nullptr, st, G))) return s;
  cudaError_t e = cudaMemsetAsync(ws.cnt, 0, (size_t)(sp.n_groups + 1) * sizeof(int), st);
  if (e != cudaSuccess) return cuda_status(e, "cudaMemsetAsync(group counters)");
  const int smem = (int)L::kTotal;
  e = cudaFuncSetAttribute(lr_bwd_tm_kernel<W, RKP>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return cuda_status(e, "cudaFuncSetAttribute(lr_bwd_tm)");
  }
  // Cooperative launch: the CTAs of a token group wait for one another before
  // the dz reduction, so the whole grid must be co-resident (grid <= SM count,
  // one CTA per SM; lr_tc_bwd_supported checks the first bound).
  if (peers.world > 1 && sp.n_dblk * sp.n_groups > kMaxDpCtas)  // one flag per CTA and source
    return set_error(DYNCONV_ERR_UNSUPPORTED, "lr_bwd_dp: grid of %d CTAs > %d", sp.n_dblk * sp.n_groups, kMaxDpCtas);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(sp.n_dblk * sp.n_groups));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, lr_bwd_tm_kernel<W, RKP>, dymap, xmap, zmap, dxmap, (const __nv_bfloat16*)U,
                         (const __nv_bfloat16*)sw, (__nv_bfloat16*)dz, ws.dzp, ws.cnt, ws.dUp,
                         dU_f32, (__nv_bfloat16*)dU, (__nv_bfloat16*)(sw ? dsw : nullptr), sp, cg, (int)T, (int)Dt,
                         R, Rk, residual, peers);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return cuda_status(e, "cudaLaunchKernelEx(lr_bwd_tm_kernel)");
  }
  DYNCONV_CHECK_LAUNCH("lr_bwd_tm_kernel");
  return DYNCONV_OK;
}

template <int RKP>
int launch_tm_w(int W, const void* x, const void* z, const void* U, const void* sw, const void* dy, void* dx,
                void* dz, float* dU_f32, void* dU, void* dsw, void* ws, int64_t B, int64_t T, int64_t D, int G, int R,
                int Rk, int residual, const DpPeers& pr, const void* zp, cudaStream_t st) {
  switch (W) {
    case 1: return launch_tm<1, RKP>(x, z, U, sw, dy, dx, dz, dU_f32, dU, dsw, ws, B, T, D, G, R, Rk, residual, pr, zp, st);
    case 2: return launch_tm<2, RKP>(x, z, U, sw, dy, dx, dz, dU_f32, dU, dsw, ws, B, T, D, G, R, Rk, residual, pr, zp, st);
    case 3: return launch_tm<3, RKP>(x, z, U, sw, dy, dx, dz, dU_f32, dU, dsw, ws, B, T, D, G, R, Rk, residual, pr, zp, st);
    case 4: return launch_tm<4, RKP>(x, z, U, sw, dy, dx, dz, dU_f32, dU, dsw, ws, B, T, D, G, R, Rk, residual, pr, zp, st);
    default: return set_error(DYNCONV_ERR_UNSUPPORTED, "tensor-core backward: W=%d", W);
  }
}

}  // namespace

// Tensor-core backward envelope: bf16, W <= 4, R_kernel <= 32, D % 8 == 0 (TMA row
// pitch; D % 128 == 0 with G > 1 channel groups), 16-byte aligned activations (TMA
// base), grid co-resident.  Everything else runs the CUDA-core kernels of
// lowrank_simple.cu (G = 1 only).
bool lr_tc_bwd_supported(int64_t D, int Rk, int W, int dtype, const void* const* ptrs, int nptrs, int G) {
  if (dtype != DYNCONV_DTYPE_BF16 || W < 1 || W > 4 || Rk < 1 || Rk > 32 || D % 8 != 0) return false;
  if (G < 1 || (G > 1 && D % kBD != 0)) return false;
  if (((int64_t)G * D + kBD - 1) / kBD > sm_count()) return false;  // the cooperative grid must fit on the GPU
  for (int i = 0; i < nptrs; ++i)
    if (ptrs[i] && !aligned16(ptrs[i])) return false;
  return encode_fn() != nullptr || nptrs == 0;
}

size_t lr_tm_bwd_workspace(int64_t B, int64_t T, int64_t D, int Rk, int W, int G) {
  return tm_workspace(nullptr, B, T, D, Rk, W, G).bytes;
}

size_t lr_tc_bwd_workspace(int64_t B, int64_t T, int64_t D, int Rk, int W, int G) {
  return lr_tm_bwd_workspace(B, T, D, Rk, W, G);
}

// peers == nullptr: single-GPU result.  Otherwise dU_f32 / dU / dstatic_w receive the
// sum over the peers' ranks, reduced inside the kernel over peer memory.  zp: z already
// packed by the forward ([G*RKP/8][B][T][8]), or nullptr to pack it here.
int lr_tm_bwd_launch(const void* x, const void* z, const void* U, const void* sw, const void* dy, void* dx, void* dz,
                     float* dU_f32, void* dU, void* dsw, void* ws, size_t ws_bytes, int64_t B, int64_t T, int64_t D,
                     int G, int R, int Rk, int W, int residual, const DpPeers* peers, const void* zp,
                     cudaStream_t st) {
  if (ws_bytes < lr_tm_bwd_workspace(B, T, D, Rk, W, G))
    return set_error(DYNCONV_ERR_WORKSPACE, "lr_bwd (tensor core): workspace too small");
  DpPeers pr = {};
  pr.world = 1;
  if (peers) {
    pr = *peers;
    if ((int64_t)G * (Rk) * W * D > pr.cap)
      return set_error(DYNCONV_ERR_WORKSPACE, "lr_bwd (data parallel): communicator holds %lld floats, the call needs %lld",
                       (long long)pr.cap, (long long)((int64_t)G * Rk * W * D));
  }
  if (Rk <= 16)
    return launch_tm_w<16>(W, x, z, U, sw, dy, dx, dz, dU_f32, dU, dsw, ws, B, T, D, G, R, Rk, residual, pr, zp, st);
  return launch_tm_w<32>(W, x, z, U, sw, dy, dx, dz, dU_f32, dU, dsw, ws, B, T, D, G, R, Rk, residual, pr, zp, st);
}

int lr_tc_bwd_launch(const void* x, const void* z, const void* U, const void* sw, const void* dy, void* dx, void* dz,
                     float* dU_f32, void* dU, void* dsw, void* ws, size_t ws_bytes, int64_t B, int64_t T, int64_t D,
                     int G, int R, int Rk, int W, int residual, const void* zp, cudaStream_t st) {
  return lr_tm_bwd_launch(x, z, U, sw, dy, dx, dz, dU_f32, dU, dsw, ws, ws_bytes, B, T, D, G, R, Rk, W, residual,
                          nullptr, zp, st);
}

}  // namespace dynconv
