// lowrank_bwd_tc.cu -- fused tcgen05 backward of the lowrank dynamic convolution, bf16.
//
// Reference behaviour: the dU/dz kernel (lowrank.py:86-140) and the dx kernel
// (lowrank.py:158-205), launched by _LowrankDynamicConvolutionFn.backward
// (lowrank.py:252-299); oracle reference.py:23-39.  One pass over dy and x computes
// dx, dz, dU and dstatic_w (the reference reads dy twice, in two kernels).
//
// Math, per channel ch and step t (z_ext = z plus the static rank, U_ext likewise):
//   Wt_w[t,ch] = sum_r z_ext[t,r] U_ext[r,w,ch]                      (dynamic weights)
//   dx[t,ch]   = sum_w dy[t+w,ch] Wt_w[t+w,ch]  (+ dy[t,ch] if residual)
//   P_w[t,ch]  = bf16(dy[t,ch] x[t-w,ch])      (bf16 product, as lowrank.py:128)
//   dU_w[ch,r] = sum_t P_w[t,ch] z_ext[t,r]     dz[t,r] = sum_{w,ch} P_w[t,ch] U_ext[r,w,ch]
//
// Orientation: tensor-memory lane = channel (the M = 128 dimension of every MMA
// but the dz one), so each epilogue thread owns one channel and walks time in
// registers.  dy and x arrive from HBM as [t][ch] rows; they are turned into
// lane-per-channel float32 columns by the tensor core itself -- an MMA with the
// 16 x 16 identity as B reads a 16-row block of the TMA tile as an MN-major A
// operand and writes D[ch][j] = block[j][ch] to tensor memory (one product per
// output, exact).  So the epilogue reads dy and x with tcgen05.ld, 16 values per
// instruction, instead of 2-byte shared-memory loads, and the tensor core, idle
// otherwise, does the transposition.
//
// Work unit: a quarter (16 steps x 128 channels) of a 64-step tile.  Per quarter:
//   transposes   dyT/xT blocks (16 steps each) into a 4-slot tensor-memory ring; a
//                quarter reads dy blocks i, i+1 (steps t..t+18) and x blocks i, i+1
//                (steps t-16..t+15), so each block is transposed once and shared
//                by two quarters;
//   MMA-1        acc_w[ch][j] = sum_r U^T[ch,r] z_ext[t+j+w, r]   M=128, N=16, K=R_kernel
//                (A = U^T held in tensor memory, B = z rows from t+w);
//   epilogue     dx (f32x2 FMAs) -> HBM (each warp writes 64-byte rows);
//                P_w as bf16 pairs (mul.rn.bf16x2) -> shared memory (dz MMA) and,
//                at R_kernel = 16, tensor memory (dU MMA);
//   MMA-2        dU_w[ch][r] += sum_j P_w[t+j, ch] z_ext[t+j, r]  M=128, N=R_kernel, K=16,
//                accumulated in tensor memory over every quarter of the CTA;
//   MMA-3        (per tile) dz[t][r] = sum_{w,ch} P_w[t,ch] U_ext[r,w,ch]   M=64, K=128*W,
//                partial over this CTA's 128 channels -> workspace, then a fixed-order
//                cross-CTA sum (see the end of the kernel).
//
// Warps: 0 producer (TMA: z tile per tile, dy+x blocks per quarter into a ring),
// 1 transposes + MMA-1 + TMEM owner, 2 MMA-2 + MMA-3, 3..18 epilogue in two teams
// of eight (team = quarter parity; a team has two warps per TMEM lane quarter,
// one per 8-step half of the quarter), so two quarters are in flight.  Every wait
// is bounded (common.cuh); a wait that gives up marks the CTA dead and the kernel
// unwinds, still arriving on the barriers it owns.
#include "lowrank_tc.cuh"

namespace dynconv {

DYNCONV_DEFINE_ERROR_ACCESSOR(lr_bwd_error_word)

namespace {

using namespace lrtc;

constexpr int kQ = 16;                 // steps per quarter
constexpr int kQPT = kBT / kQ;         // quarters per tile
constexpr int kBlkPT = kQPT + 1;       // transposed blocks per tile and tensor
constexpr int kZRows = 72;             // z rows t0 .. t0+71 (64 + W-1, whole core matrices)
constexpr int kCtl = 8;                // control warps (producer + seven MMA issuers)
constexpr int kEpi = 8;                // epilogue warps: two teams of four (one per TMEM lane quarter)
constexpr int kThreads = 32 * (kCtl + kEpi);


template <int W, int RKP>
struct BwdCfg {
  static constexpr int kRKP = RKP;
  static constexpr bool kPT = false;        // MMA-2 reads P from shared memory
  static constexpr int NP = 2;              // P buffers (MMA-3 of one tile overlaps the next)
  static constexpr int S = (RKP == 16) ? 8 : 4;  // shared-memory ring of (dy, x) block pairs
  static constexpr int kTRing = (RKP == 16) ? 8 : 4;  // tensor-memory block ring (dyT / xT slots)
  // shared memory (bytes from the 1024-aligned base)
  static constexpr uint32_t kHalf = kQ * 128;     // 16 rows x 64 channels (one swizzle atom column)
  static constexpr uint32_t kBlk = 2 * kHalf;     // 128 channels
  static constexpr uint32_t kSlot = 2 * kBlk;     // dy block, then x block
  static constexpr uint32_t kUTap = (uint32_t)kBD * RKP * 2;
  static constexpr uint32_t kZBytes = (uint32_t)kZRows * RKP * 2;
  static constexpr uint32_t kZStride = (kZBytes + 127u) / 128u * 128u;
  static constexpr uint32_t kPTap = (uint32_t)kBT * kBD * 2;
  static constexpr uint32_t kOffRing = 0;
  static constexpr uint32_t kOffP = kOffRing + S * kSlot;
  static constexpr uint32_t kOffU = kOffP + NP * W * kPTap;
  static constexpr uint32_t kOffZ = round1024(kOffU + W * kUTap);
  static constexpr uint32_t kDxWarp = kQ * 32 * 2;  // [16 steps][32 ch] bf16 sub-tile (dx transpose)
  static constexpr uint32_t kOffDx = kOffZ + 2 * kZStride;
  static constexpr uint32_t kOffI = kOffDx + kEpi * kDxWarp;
  static constexpr uint32_t kTotal = kOffI + 512 + 1024;  // + alignment slack
  // operand strides
  static constexpr uint32_t kUChunk = (RKP / 8) * 128;  // U: next 8 channels
  static constexpr uint32_t kZChunk = kZRows * 16;      // z: next 8 ranks
  static constexpr uint32_t kPChunk = (kBT / 8) * 128;  // P: next 8 channels
  // tensor-memory columns
  static constexpr uint32_t kAcc = W * kQ;             // one team's weights (W taps x 16 steps)
  static constexpr uint32_t kColAcc = 0;
  static constexpr uint32_t kColDyT = 2 * kAcc;
  static constexpr uint32_t kColXT = kColDyT + kTRing * kQ;

  static constexpr uint32_t kPTSlot = W * 8;           // P^T of one quarter: W taps x 16 steps (bf16 pairs)
  static constexpr uint32_t kColPT = kColXT + kTRing * kQ;
  static constexpr uint32_t kColDU = kColPT + (kPT ? 4 * kPTSlot : 0);
  static constexpr uint32_t kColDZ = kColDU + W * RKP;  // 2 buffers x 2 MMA-3 accumulators x RKP, M = 64 layout
  static constexpr uint32_t kCols = kColDZ + 4 * RKP;
  static_assert(kCols <= 512, "tensor-memory budget");
  static_assert(kTotal <= 232448 - 1024, "shared-memory budget (227 KB per CTA, static part aside)");
};

template <int N>
__device__ __forceinline__ void tmem_ld_n(uint32_t taddr, float (&v)[N]) {
  static_assert(N == 4 || N == 8 || N == 16, "");
  if constexpr (N == 4) tmem_ld4(taddr, v);
  else if constexpr (N == 8) tmem_ld8(taddr, v);
  else tmem_ld16(taddr, v);
}

// MMA-3 of one tile for taps [WLO, WHI): K = (tap, channel) steps into one
// accumulator.  ad0 / bd0: descriptors of the tile's P buffer and of U at tap 0,
// channel 0; every other operand is a compile-time offset (16-byte units).
template <int WLO, int WHI, class L>
__device__ __forceinline__ void issue_mma3(uint32_t dacc, uint64_t ad0, uint64_t bd0, uint32_t idesc) {
  // first K-step of the first tap overwrites the accumulator; the loop stays rolled
  // (the issue rate of one thread, not its instruction count, bounds this stream)
  umma_f16_c<0>(dacc, ad0 + (uint64_t)((WLO * L::kPTap) >> 4), bd0 + (uint64_t)((WLO * L::kUTap) >> 4), idesc);
#pragma unroll 1
  for (int s = 1; s < (WHI - WLO) * (kBD / 16); ++s) {
    const int w = WLO + s / (kBD / 16), ks = s % (kBD / 16);
    const uint64_t ad = ad0 + (uint64_t)((w * L::kPTap + ks * 2 * L::kPChunk) >> 4);
    const uint64_t bd = bd0 + (uint64_t)((w * L::kUTap + ks * 2 * L::kUChunk) >> 4);
    umma_f16_c<1>(dacc, ad, bd, idesc);
  }
}

// MMA-2 of one quarter for taps [WLO, WHI): A = P^T of the quarter (tensor memory
// at R_kernel = 16, else the P buffer), B = the quarter's z rows.
template <int WLO, int WHI, class L>
__device__ __forceinline__ void issue_mma2(uint32_t du, uint32_t pt, uint64_t ad0, uint64_t bd, uint32_t idesc,
                                           bool accumulate) {
#pragma unroll
  for (int w = WLO; w < WHI; ++w) {
    if constexpr (L::kPT) {
      if (accumulate) umma_f16_ts_c<1>(du + w * L::kRKP, pt + w * 8, bd, idesc);
      else umma_f16_ts_c<0>(du + w * L::kRKP, pt + w * 8, bd, idesc);
    } else {
      const uint64_t ad = ad0 + (uint64_t)((w * L::kPTap) >> 4);
      if (accumulate) umma_f16_c<1>(du + w * L::kRKP, ad, bd, idesc);
      else umma_f16_c<0>(du + w * L::kRKP, ad, bd, idesc);
    }
  }
}

template <int W, int RKP>
__global__ void __launch_bounds__(kThreads, 1)
    lr_bwd_tc_kernel(const __grid_constant__ CUtensorMap dymap, const __grid_constant__ CUtensorMap xmap,
                     const __grid_constant__ CUtensorMap zmap, const __nv_bfloat16* __restrict__ U,
                     const __nv_bfloat16* __restrict__ sw, __nv_bfloat16* __restrict__ dx, __nv_bfloat16* __restrict__ dz, float* __restrict__ dzp, int* __restrict__ grp_done,
                     float* __restrict__ dUp, float* __restrict__ dU_f32, __nv_bfloat16* __restrict__ dU,
                     __nv_bfloat16* __restrict__ dsw, TileSplit sp, ChanGroups cg, int T, int D, int R, int Rk,
                     int residual, int tma4) {
  // D: channels of an activation row (G * Dg); cg.Dg: channels of one group's U
  using L = BwdCfg<W, RKP>;
  constexpr int S = L::S, NP = L::NP, kTRing = L::kTRing;
  constexpr int kW0 = (W + 1) / 2;  // taps [0, kW0) go to the first issuer of a split stream
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  __shared__ uint64_t rfull[S], rempty[S], zfull[2], zempty[2], tfull[kTRing], tfree[kTRing], accfull[2],
      accempty[2], pf[4], ptempty[4], pe[NP], dzf[2], dze[2], du_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  __shared__ int grp_ok;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dblk = blockIdx.x % sp.n_dblk;
  const int g = blockIdx.x / sp.n_dblk;
  const int j0 = (int)((int64_t)sp.n_tiles * g / sp.n_groups);
  const int j1 = (int)((int64_t)sp.n_tiles * (g + 1) / sp.n_groups);
  const int n = j1 - j0;
  const int nq = n * kQPT;
  const int d0 = dblk * kBD;           // first channel in the activation row
  const int grp = dblk / cg.nd;        // channel group of this CTA's block
  const int dl0 = d0 - grp * cg.Dg;    // first channel within the group

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&rfull[s], 1);
      mbar_init(&rempty[s], 1);
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(&zfull[h], 1);
      mbar_init(&zempty[h], 4);  // last weight MMAs (two issuers) and last dU MMAs (two issuers) of the tile
      mbar_init(&accfull[h], 1);
      mbar_init(&accempty[h], 4);
    }
    for (int c = 0; c < kTRing; ++c) {
      mbar_init(&tfull[c], 1);
      mbar_init(&tfree[c], 8);  // two quarters x 4 warps per block
    }
    for (int c = 0; c < 4; ++c) {
      mbar_init(&pf[c], 4);
      mbar_init(&ptempty[c], 2);
    }
    for (int p = 0; p < NP; ++p) mbar_init(&pe[p], L::kPT ? 2 : 4);
    for (int h = 0; h < 2; ++h) {
      mbar_init(&dzf[h], 2);
      mbar_init(&dze[h], kEpi);
    }
    mbar_init(&du_bar, 2);
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
    // Everything but the producer: U block in shared memory (dz MMA B operand),
    // the 16x16 identity (transpose B operand), TMEM allocation, U^T in TMEM.
    constexpr int kNonProducer = kThreads - 32;
    const int tid = threadIdx.x - 32;
    load_u_block<W, RKP, kNonProducer>(smem + L::kOffU, U + (size_t)grp * R * W * cg.Dg,
                                       sw ? sw + (size_t)grp * W * cg.Dg : nullptr, dblk - grp * cg.nd, cg.Dg, R, tid);
    if (tid < kQ * kQ) {
      const int nn = tid >> 4, kk = tid & 15;
      *reinterpret_cast<__nv_bfloat16*>(smem + L::kOffI + kmajor_off(nn, kk, 128, 256)) =
          __float2bfloat16_rn(nn == kk ? 1.f : 0.f);
    }
    fence_proxy_async_smem();
    if (warp == 1) {
      tmem_alloc(&tmem_slot, 512);
      tmem_relinquish();
    }
    tc_fence_before();
    named_bar_sync(2, kNonProducer);
    tc_fence_after();
    tmem = tmem_slot;
    tc_fence_before();
    named_bar_sync(2, kNonProducer);
    tc_fence_after();
  }

  // Each MMA stream has its own issuing warp: one warp sustains about one
  // tcgen05.mma per ~130 cycles, the tensor core several times that.
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      for (int k = 0; k < n; ++k) {
        const int tile = j0 + k, b = tile / sp.tiles_row, t0 = (tile % sp.tiles_row) * kBT;
        if (!mbar_wait(&zempty[k & 1], ((k >> 1) & 1) ^ 1, kErrWaitProducer, &abort_flag)) break;
        mbar_arrive_expect_tx(&zfull[k & 1], L::kZBytes);
        tma_load_4d(smem + L::kOffZ + (k & 1) * L::kZStride, &zmap, &zfull[k & 1], 0, t0, b, grp * (RKP / 8), pol);
        bool ok = true;
        for (int bb = 0; bb < kBlkPT; ++bb) {
          const int nb = kBlkPT * k + bb, m = nb % S;
          if (!mbar_wait(&rempty[m], ((nb / S) & 1) ^ 1, kErrWaitProducer, &abort_flag)) { ok = false; break; }
          uint8_t* slot = smem + L::kOffRing + m * L::kSlot;
          mbar_arrive_expect_tx(&rfull[m], L::kSlot);
          // dy block bb: steps t0 + 16bb ..; x block bb: steps t0 - 16 + 16bb .. (zero fill outside [0, T))
          if (tma4) {  // both 64-channel halves in one box
            tma_load_4d(slot, &dymap, &rfull[m], 0, t0 + kQ * bb, d0 / 64, b, pol);
            tma_load_4d(slot + L::kBlk, &xmap, &rfull[m], 0, t0 - kQ + kQ * bb, d0 / 64, b, pol);
          } else {
            tma_load_3d(slot, &dymap, &rfull[m], d0, t0 + kQ * bb, b, pol);
            tma_load_3d(slot + L::kHalf, &dymap, &rfull[m], d0 + 64, t0 + kQ * bb, b, pol);
            tma_load_3d(slot + L::kBlk, &xmap, &rfull[m], d0, t0 - kQ + kQ * bb, b, pol);
            tma_load_3d(slot + L::kBlk + L::kHalf, &xmap, &rfull[m], d0 + 64, t0 - kQ + kQ * bb, b, pol);
          }
        }
        if (!ok) break;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ transposes (+ TMEM owner)
    // Block nb of the stream (kBlkPT per tile) -> TMEM ring slot nb % kTRing.
    const uint32_t ib = smem_u32(smem + L::kOffI);
    const uint32_t idesc_t = make_idesc_bf16(kBD, kQ, 1, 0);  // A MN-major (swizzled tile), B = I (K-major)
    const uint64_t bd_i = make_smem_desc(ib, 256, 128);
    const uint64_t ad_ring = make_smem_desc_sw128(smem_u32(smem + L::kOffRing), L::kHalf, 1024);
    const int nblk = n * kBlkPT;
    for (int nb = 0; nb < nblk; ++nb) {
      const int m = nb % S, c = nb % kTRing;
      if (!mbar_wait(&rfull[m], (nb / S) & 1, kErrWaitMma, &abort_flag)) break;
      if (!mbar_wait(&tfree[c], ((nb / kTRing) & 1) ^ 1, kErrWaitMma, &abort_flag)) break;
      tc_fence_after();
      if (lane == 0) {
        const uint64_t ad = ad_ring + (uint64_t)((m * L::kSlot) >> 4);
        umma_f16_c<0>(tmem + L::kColDyT + c * kQ, ad, bd_i, idesc_t);
        umma_f16_c<0>(tmem + L::kColXT + c * kQ, ad + (uint64_t)(L::kBlk >> 4), bd_i, idesc_t);
        umma_commit(&rempty[m]);
        umma_commit(&tfull[c]);
      }
      __syncwarp();
    }
  } else if (warp == 2 || warp == 3) {
    // ------------------------------------------------------------ MMA-1 (weights) of one team's quarters
    // Before issuing it also waits for everything else the team's epilogue needs for
    // the quarter -- the two transposed blocks, a free P buffer -- so accfull alone
    // tells the epilogue that the quarter is ready.
    const int team = warp - 2;
    const uint32_t idesc1 = make_idesc_bf16(kBD, kQ, 0, 0);  // A = U^T (K-major, shared), B = z (K-major)
    const uint64_t ud1 = make_smem_desc(smem_u32(smem + L::kOffU), 128, L::kUChunk);
    const uint64_t zdesc0 = make_smem_desc(smem_u32(smem + L::kOffZ), L::kZChunk, 128);
    const uint32_t acc = tmem + L::kColAcc + team * L::kAcc;
    for (int Q = team; Q < nq; Q += 2) {
      const int k = Q / kQPT, i = Q % kQPT, p = k % NP;
      const int nbA = kBlkPT * k + i;
      if (i < 2 && !mbar_wait(&zfull[k & 1], (k >> 1) & 1, kErrWaitMma, &abort_flag)) break;
      if (!mbar_wait(&accempty[team], ((Q >> 1) & 1) ^ 1, kErrWaitMma, &abort_flag)) break;
      if (!mbar_wait(&tfull[nbA % kTRing], (nbA / kTRing) & 1, kErrWaitMma, &abort_flag)) break;
      if (!mbar_wait(&tfull[(nbA + 1) % kTRing], ((nbA + 1) / kTRing) & 1, kErrWaitMma, &abort_flag)) break;
      if (i < 2 && !mbar_wait(&pe[p], ((k / NP) & 1) ^ 1, kErrWaitMma, &abort_flag)) break;
      tc_fence_after();
      if (lane == 0) {
        // z rows from 16i + w of stage k & 1 (descriptor start address in 16-byte units)
        const uint64_t zd = zdesc0 + (uint64_t)(((k & 1) * L::kZStride + (uint32_t)(kQ * i) * 16u) >> 4);
#pragma unroll
        for (int w = 0; w < W; ++w) {
#pragma unroll
          for (int ks = 0; ks < RKP / 16; ++ks)
            if (ks == 0)
              umma_f16_c<0>(acc + w * kQ, ud1 + (uint64_t)((w * L::kUTap) >> 4), zd + (uint64_t)((w * 16) >> 4), idesc1);
            else
              umma_f16_c<1>(acc + w * kQ, ud1 + (uint64_t)((w * L::kUTap + ks * 256) >> 4),
                            zd + (uint64_t)((w * 16 + ks * 2 * L::kZChunk) >> 4), idesc1);
        }
        umma_commit(&accfull[team]);
        if (i >= kQPT - 2) umma_commit(&zempty[k & 1]);  // this issuer's last read of z tile k
      }
      __syncwarp();
    }
  } else if (warp == 4 || warp == 5) {
    // ------------------------------------------------------------ MMA-2 (dU) for a subset of the taps
    const bool lo = warp == 4;
    const uint64_t pd0 = make_smem_desc(smem_u32(smem + L::kOffP), 128, L::kPChunk);
    const uint64_t zd0 = make_smem_desc(smem_u32(smem + L::kOffZ), 128, L::kZChunk);  // K = steps, N = ranks
    const uint32_t idesc2 = make_idesc_bf16(kBD, RKP, 0, 1);  // A = P^T (K-major), B = z (MN-major)
    for (int Q = 0; Q < nq; ++Q) {
      const int k = Q / kQPT, i = Q % kQPT, p = k % NP;
      if (!mbar_wait(&pf[Q & 3], (Q >> 2) & 1, kErrWaitMma, &abort_flag)) break;
      tc_fence_after();
      if (lane == 0) {
        const uint64_t bd = zd0 + (uint64_t)(((k & 1) * L::kZStride + (uint32_t)(kQ * i) * 16u) >> 4);
        const uint64_t ad0 = pd0 + (uint64_t)((p * W * L::kPTap + (uint32_t)i * 2u * 128u) >> 4);
        const uint32_t pt = tmem + L::kColPT + (Q & 3) * L::kPTSlot;
        if (lo) issue_mma2<0, kW0, L>(tmem + L::kColDU, pt, ad0, bd, idesc2, Q > 0);
        else issue_mma2<kW0, W, L>(tmem + L::kColDU, pt, ad0, bd, idesc2, Q > 0);
        if constexpr (L::kPT) umma_commit(&ptempty[Q & 3]);
        if (i == kQPT - 1) {
          umma_commit(&zempty[k & 1]);
          if constexpr (!L::kPT) umma_commit(&pe[p]);  // P buffer p read by this issuer for the last time
        }
      }
      __syncwarp();
    }
    if (lane == 0) umma_commit(&du_bar);
    __syncwarp();
  } else if (warp == 6 || warp == 7) {
    // ------------------------------------------------------------ MMA-3 (dz) for a subset of the taps,
    // into this issuer's own accumulator (the epilogue adds the two)
    const int half = warp - 6;
    const uint64_t pd0 = make_smem_desc(smem_u32(smem + L::kOffP), L::kPChunk, 128);
    const uint64_t ud0 = make_smem_desc(smem_u32(smem + L::kOffU), L::kUChunk, 128);
    const uint32_t idesc3 = make_idesc_bf16(64, RKP, 1, 1);  // A = P (MN-major), B = U (MN-major)
    const uint32_t dacc0 = tmem + L::kColDZ + half * RKP;
    for (int k = 0; k < n; ++k) {
      const int p = k % NP;
      bool ok = true;
      for (int i = 0; i < kQPT && ok; ++i) ok = mbar_wait(&pf[(kQPT * k + i) & 3], ((kQPT * k + i) >> 2) & 1, kErrWaitMma, &abort_flag);
      if (!ok) break;
      if (!mbar_wait(&dze[k & 1], ((k >> 1) & 1) ^ 1, kErrWaitMma, &abort_flag)) break;
      tc_fence_after();
      if (lane == 0) {
        const uint64_t ad0 = pd0 + (uint64_t)((p * W * L::kPTap) >> 4);
        const uint32_t dacc = dacc0 + (k & 1) * 2 * RKP;
        if (half == 0) issue_mma3<0, kW0, L>(dacc, ad0, ud0, idesc3);
        else issue_mma3<kW0, W, L>(dacc, ad0, ud0, idesc3);
        umma_commit(&dzf[k & 1]);
        umma_commit(&pe[p]);
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int e = warp - kCtl;      // 0..7
    const int q = warp & 3;         // TMEM lane quarter this warp may access
    const int team = e >> 2;        // quarters of this parity
    const int ch = q * 32 + lane;
    const bool dok = d0 + ch < D;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const uint32_t ta = tmem + lane_base;
    uint8_t* const pch = smem + L::kOffP + kmajor_off(ch, 0, L::kPChunk, 128);  // this channel's P column
    __nv_bfloat16* const st = reinterpret_cast<__nv_bfloat16*>(smem + L::kOffDx + e * L::kDxWarp);
    const int ccol = d0 + q * 32 + (lane & 3) * 8;  // first channel of this lane's 16-byte dx pieces
    bool dead = false;

    // dz partial of tile kk (M = 64 layout: lanes 0..15 of quarter q hold steps
    // 16q..16q+15; the two warps of a lane quarter take RKP/2 columns each; the two
    // MMA-3 accumulators are added) -> workspace
    auto dz_readout = [&](int kk) {
      const int tile = j0 + kk;
      if (!dead) dead = !mbar_wait(&dzf[kk & 1], (kk >> 1) & 1, kErrWaitEpilogue, &abort_flag);
      tc_fence_after();
      constexpr int NC = RKP / 2;
      constexpr int NACC = W > 1 ? 2 : 1;
      float v[NC], v2[NC];
      const int c0 = team * NC;
      if (!dead) {
        const uint32_t dzc = ta + L::kColDZ + (kk & 1) * 2 * RKP + c0;
        tmem_ld_n<NC>(dzc, v);
        if constexpr (NACC > 1) tmem_ld_n<NC>(dzc + RKP, v2);
        tmem_ld_wait();
        if constexpr (NACC > 1) {
#pragma unroll
          for (int c = 0; c < NC; ++c) v[c] += v2[c];
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dze[kk & 1]);
      if (!dead && lane < 16) {
        float* dst = dzp + (((size_t)dblk * sp.n_tiles + tile) * kBT + 16 * q + lane) * RKP + c0;
#pragma unroll
        for (int c = 0; c < NC; c += 4) *reinterpret_cast<float4*>(dst + c) = make_float4(v[c], v[c + 1], v[c + 2], v[c + 3]);
      }
    };

    int k = 0, i = team, tile = j0;
    int b = tile / sp.tiles_row, t0 = (tile % sp.tiles_row) * kBT;
    for (int Q = team, it = 0; Q < nq; Q += 2, ++it) {
      const int p = k % NP;
      const int nbA = kBlkPT * k + i, cA = nbA % kTRing, cB = (nbA + 1) % kTRing;
      if (!dead) dead = !mbar_wait(&accfull[team], it & 1, kErrWaitEpilogue, &abort_flag);
      tc_fence_after();
      // acc[w][j]: weights of tap w at step 16i + j0h + j; dy(m): dy at step 16i + m (m < 20);
      // xv(m): x at step 16i - 4 + m (m < 20).  Quarter-relative rows: dy block i holds
      // rows 0..15, dy block i+1 rows 16..31; x block i rows -16..-1, x block i+1 rows 0..15.
      float acc[W][8], dyA[16], dyB[4], xA[4], xB[16];
      if (!dead) {
        tmem_ld16(ta + L::kColDyT + cA * kQ, dyA);
        tmem_ld4(ta + L::kColDyT + cB * kQ, dyB);
        tmem_ld4(ta + L::kColXT + cA * kQ + 12, xA);
        tmem_ld16(ta + L::kColXT + cB * kQ, xB);
#pragma unroll
        for (int w = 0; w < W; ++w) tmem_ld8(ta + L::kColAcc + team * L::kAcc + w * kQ, acc[w]);
        tmem_ld_wait();
      }
      auto dyv = [&](int m) -> float { return m < 16 ? dyA[m] : dyB[m - 16]; };
      auto xv = [&](int m) -> float { return m < 4 ? xA[m] : xB[m - 4]; };
      // dx[j] = sum_w acc_w[j] dy[j+w] (+ dy[j]) for steps j0h .. j0h+7 -> shared sub-tile
      auto dx_half = [&](int j0h) {
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          const int j = j0h + jj;
          float v = residual ? fmaf(acc[0][jj], dyv(j), dyv(j)) : acc[0][jj] * dyv(j);
#pragma unroll
          for (int w = 1; w < W; ++w) v = fmaf(acc[w][jj], dyv(j + w), v);
          st[j * 32 + lane] = __float2bfloat16_rn(v);
        }
      };
      if (!dead) {
        dx_half(0);
#pragma unroll
        for (int w = 0; w < W; ++w) tmem_ld8(ta + L::kColAcc + team * L::kAcc + w * kQ + 8, acc[w]);
        tmem_ld_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&accempty[team]);
        mbar_arrive_cnt(&tfree[cA], i == 0 ? 2u : 1u);
        mbar_arrive_cnt(&tfree[cB], i == kQPT - 1 ? 2u : 1u);
      }
      if (!dead) {
        dx_half(8);
        __syncwarp();
        // the warp's [16 steps][32 ch] sub-tile, read back as 16-byte row pieces: lane l
        // stores channels ccol.. of steps l/4 and l/4 + 8 (64 contiguous bytes per 4 lanes)
        if (ccol < D) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int r = (lane >> 2) + 8 * h, t = t0 + kQ * i + r;
            const uint4 v = *reinterpret_cast<const uint4*>(st + r * 32 + (lane & 3) * 8);
            if (t < T) *reinterpret_cast<uint4*>(dx + ((size_t)b * T + t) * D + ccol) = v;
          }
        }
        __syncwarp();  // the sub-tile is rewritten by the next quarter
        // ---- P_w = bf16(dy * x_{t-w}) as (step, step+1) pairs -> shared memory (dz and dU MMAs)
        uint32_t dy2[kQ / 2];
#pragma unroll
        for (int pp = 0; pp < kQ / 2; ++pp) dy2[pp] = pack_bf16x2(dyv(2 * pp), dyv(2 * pp + 1));
        uint8_t* pbuf = pch + p * W * L::kPTap + (2 * i) * 128;
        // tap w pairs step (2pp, 2pp+1) of dy with x rows (2pp-w, 2pp+1-w), i.e. xv pair
        // m = 2pp + 4 - w: even taps use even m, odd taps odd m -- one parity at a time
#pragma unroll
        for (int par = 0; par < 2; ++par) {
          uint32_t xp[10];  // xp[c] = (xv(2c + par), xv(2c + par + 1))
#pragma unroll
          for (int c = 0; c < 10; ++c) {
            const int m = 2 * c + par;
            xp[c] = (m >= 4 - (W - 1) && m <= 18) ? pack_bf16x2(xv(m), xv(m + 1)) : 0u;
          }
#pragma unroll
          for (int w = par; w < W; w += 2) {
            uint32_t pk[8];
#pragma unroll
            for (int pp = 0; pp < 8; ++pp) pk[pp] = mul_bf16x2(dy2[pp], xp[(2 * pp + 4 - w - par) >> 1]);
            *reinterpret_cast<uint4*>(pbuf + w * L::kPTap) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            *reinterpret_cast<uint4*>(pbuf + w * L::kPTap + 128) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pf[Q & 3]);
      if (i == team + 2 && k >= 1) dz_readout(k - 1);  // after this team's last quarter of tile k
      // next quarter of this team
      i += 2;
      if (i >= kQPT) {
        i -= kQPT;
        ++k;
        ++tile;
        t0 += kBT;
        if (t0 >= (int)((int64_t)sp.tiles_row * kBT)) {
          t0 = 0;
          ++b;
        }
      }
    }
    if (n >= 1) dz_readout(n - 1);
    // dU partial of this CTA: TMEM (lane = channel) -> dUp[g][grp][r][w*Dg + dl0 + ch]
    if (!dead) dead = !mbar_wait(&du_bar, 0, kErrWaitTail, &abort_flag);
    tc_fence_after();
    if (!dead) {
      for (int cidx = team; cidx < W * (RKP / 16); cidx += 2) {
        const int w = cidx / (RKP / 16), rc = cidx % (RKP / 16);
        float v[16];
        tmem_ld16(ta + L::kColDU + w * RKP + rc * 16, v);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const int r = rc * 16 + c;
          if (r < Rk && dok)
            dUp[(((size_t)g * cg.G + grp) * Rk + r) * W * cg.Dg + (size_t)w * cg.Dg + dl0 + ch] = v[c];
        }
      }
    }
  }

  // ---------------------------------------------------------------- dz reduction
  // Publish this CTA's dz partials (CTA barrier, then one cumulative gpu-scope
  // fence), wait for the other channel-block CTAs of the group (co-resident:
  // cooperative launch), then sum this CTA's 1/n_dblk slice of the group's
  // (step, rank) pairs in channel-block order: deterministic, evenly spread.
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
    // (step, channel group) pairs of the token group, split evenly over its CTAs;
    // group go's dz sums the partials of its own channel blocks
    const int64_t npairs = (int64_t)n * kBT * cg.G;
    const int64_t lo = npairs * dblk / sp.n_dblk, hi = npairs * (dblk + 1) / sp.n_dblk;
    constexpr int RQ = RKP / 4;  // float4 groups per step
    const int RG = cg.G * R;     // dz row width
    for (int64_t e2 = lo * RQ + threadIdx.x; e2 < hi * RQ; e2 += blockDim.x) {
      const int64_t sg = e2 / RQ;
      const int rq = (int)(e2 % RQ);
      const int64_t st = sg / cg.G;
      const int go = (int)(sg - st * cg.G);
      const int tile = j0 + (int)(st / kBT), tok = (int)(st % kBT);
      const int b = tile / sp.tiles_row, t = (tile % sp.tiles_row) * kBT + tok;
      float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f);
      const int kb = go * cg.nd;
#pragma unroll 4
      for (int k2 = kb; k2 < kb + cg.nd; ++k2) {  // partial loads in flight, summed in order
        const float4 f =
            __ldcg(reinterpret_cast<const float4*>(dzp + (((size_t)k2 * sp.n_tiles + tile) * kBT + tok) * RKP) + rq);
        a4.x += f.x;
        a4.y += f.y;
        a4.z += f.z;
        a4.w += f.w;
      }
      if (t < T) {
        __nv_bfloat16* dst = dz + ((size_t)b * T + t) * RG + go * R;
        const float av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (4 * rq + c < R) dst[4 * rq + c] = __float2bfloat16_rn(av[c]);
      }
    }
  }

  // ---------------------------------------------------------------- dU reduction
  // Once the whole grid has published its dU partial (the grid-wide count above),
  // CTA i sums its 1/grid slice of the [Rk][W*D] accumulator over the groups in
  // group order (deterministic) and writes dU_f32, and the bf16 dU rows /
  // dstatic_w row when they are requested.
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
    const int64_t wd = (int64_t)W * cg.Dg;
    const int64_t per_g = (int64_t)Rk * wd;  // one group's [Rk][W*Dg] block
    const int64_t n4 = cg.G * per_g / 4;     // W*Dg % 4 == 0 (Dg % 8 == 0)
    const int64_t lo = n4 * blockIdx.x / gridDim.x, hi = n4 * (blockIdx.x + 1) / gridDim.x;
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
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

struct BwdWorkspace {
  float* dzp;
  int* cnt;
  float* dUp;
  void* zp;
  size_t bytes;
};

size_t al256(size_t v) { return (v + 255) / 256 * 256; }

int rkp_of(int Rk) { return Rk <= 16 ? 16 : 32; }

// D: channels per group; the activation rows hold G * D.
BwdWorkspace bwd_workspace(void* base, int64_t B, int64_t T, int64_t D, int Rk, int W, int G) {
  const TileSplit sp = tile_split(B, T, (int64_t)G * D);
  const int rkp = rkp_of(Rk);
  BwdWorkspace w;
  const size_t dzp = al256((size_t)sp.n_dblk * sp.n_tiles * kBT * rkp * sizeof(float));
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
int launch_bwd(const void* x, const void* z, const void* U, const void* sw, const void* dy, void* dx, void* dz,
               float* dU_f32, void* dU, void* dsw, void* wsp, int64_t B, int64_t T, int64_t D, int G, int R, int Rk,
               int residual, cudaStream_t st) {
  using L = BwdCfg<W, RKP>;
  CUtensorMap dymap, xmap, zmap;
  int s;
  const int64_t Dt = (int64_t)G * D;
  const TileSplit sp = tile_split(B, T, Dt);
  const ChanGroups cg = chan_groups(D, G);
  BwdWorkspace ws = bwd_workspace(wsp, B, T, D, Rk, W, G);
  const int tma4 = Dt % 64 == 0 ? 1 : 0;
  if (tma4) {
    if ((s = make_btd4_map(&dymap, dy, B, T, Dt, kQ))) return s;
    if ((s = make_btd4_map(&xmap, x, B, T, Dt, kQ))) return s;
  } else {
    if ((s = make_btd_map(&dymap, dy, B, T, Dt, 64, kQ, 128))) return s;
    if ((s = make_btd_map(&xmap, x, B, T, Dt, 64, kQ, 128))) return s;
  }
  if ((s = make_zpack_map(&zmap, ws.zp, B, T, RKP, kZRows, G))) return s;
  if ((s = z_pack_launch(z, ws.zp, B, T, R, RKP, sw != nullptr, st, G))) return s;
  cudaError_t e = cudaMemsetAsync(ws.cnt, 0, (size_t)(sp.n_groups + 1) * sizeof(int), st);
  if (e != cudaSuccess) return cuda_status(e, "cudaMemsetAsync(group counters)");
  const int smem = (int)L::kTotal;
  e = cudaFuncSetAttribute(lr_bwd_tc_kernel<W, RKP>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return cuda_status(e, "cudaFuncSetAttribute(lr_bwd_tc)");
  }
  // Cooperative launch: the CTAs of a token group wait for one another before
  // the dz reduction, so the whole grid must be co-resident (grid <= SM count,
  // one CTA per SM; lr_tc_bwd_supported checks the first bound).
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
  e = cudaLaunchKernelEx(&cfg, lr_bwd_tc_kernel<W, RKP>, dymap, xmap, zmap, (const __nv_bfloat16*)U,
                         (const __nv_bfloat16*)sw, (__nv_bfloat16*)dx, (__nv_bfloat16*)dz, ws.dzp, ws.cnt, ws.dUp, dU_f32,
                         (__nv_bfloat16*)dU, (__nv_bfloat16*)(sw ? dsw : nullptr), sp, cg, (int)T, (int)Dt, R, Rk,
                         residual, tma4);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return cuda_status(e, "cudaLaunchKernelEx(lr_bwd_tc_kernel)");
  }
  DYNCONV_CHECK_LAUNCH("lr_bwd_tc_kernel");
  return DYNCONV_OK;
}

template <int RKP>
int launch_bwd_w(int W, const void* x, const void* z, const void* U, const void* sw, const void* dy, void* dx,
                 void* dz, float* dU_f32, void* dU, void* dsw, void* ws, int64_t B, int64_t T, int64_t D, int G, int R,
                 int Rk, int residual, cudaStream_t st) {
  switch (W) {
    case 1: return launch_bwd<1, RKP>(x, z, U, sw, dy, dx, dz, dU_f32, dU, dsw, ws, B, T, D, G, R, Rk, residual, st);
    case 2: return launch_bwd<2, RKP>(x, z, U, sw, dy, dx, dz, dU_f32, dU, dsw, ws, B, T, D, G, R, Rk, residual, st);
    case 3: return launch_bwd<3, RKP>(x, z, U, sw, dy, dx, dz, dU_f32, dU, dsw, ws, B, T, D, G, R, Rk, residual, st);
    case 4: return launch_bwd<4, RKP>(x, z, U, sw, dy, dx, dz, dU_f32, dU, dsw, ws, B, T, D, G, R, Rk, residual, st);
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

size_t lr_tm_bwd_workspace(int64_t B, int64_t T, int64_t D, int Rk, int W, int G);
int lr_tm_bwd_launch(const void* x, const void* z, const void* U, const void* sw, const void* dy, void* dx, void* dz,
                     float* dU_f32, void* dU, void* dsw, void* ws, size_t ws_bytes, int64_t B, int64_t T, int64_t D,
                     int G, int R, int Rk, int W, int residual, const DpPeers* peers, cudaStream_t st);

size_t lr_tc_bwd_workspace(int64_t B, int64_t T, int64_t D, int Rk, int W, int G) {
  return lr_tm_bwd_workspace(B, T, D, Rk, W, G);
}

int lr_tc_bwd_launch(const void* x, const void* z, const void* U, const void* sw, const void* dy, void* dx, void* dz,
                     float* dU_f32, void* dU, void* dsw, void* ws, size_t ws_bytes, int64_t B, int64_t T, int64_t D,
                     int G, int R, int Rk, int W, int residual, cudaStream_t st) {
  return lr_tm_bwd_launch(x, z, U, sw, dy, dx, dz, dU_f32, dU, dsw, ws, ws_bytes, B, T, D, G, R, Rk, W, residual,
                          nullptr, st);
}

int lr_tc_bwd_launch_quarters(const void* x, const void* z, const void* U, const void* sw, const void* dy, void* dx, void* dz,
                     float* dU_f32, void* dU, void* dsw, void* ws, size_t ws_bytes, int64_t B, int64_t T, int64_t D,
                     int G, int R, int Rk, int W, int residual, cudaStream_t st) {
  if (ws_bytes < bwd_workspace(nullptr, B, T, D, Rk, W, G).bytes)
    return set_error(DYNCONV_ERR_WORKSPACE, "lr_bwd (tensor core): workspace too small");
  if (Rk <= 16)
    return launch_bwd_w<16>(W, x, z, U, sw, dy, dx, dz, dU_f32, dU, dsw, ws, B, T, D, G, R, Rk, residual, st);
  return launch_bwd_w<32>(W, x, z, U, sw, dy, dx, dz, dU_f32, dU, dsw, ws, B, T, D, G, R, Rk, residual, st);
}

}  // namespace dynconv
