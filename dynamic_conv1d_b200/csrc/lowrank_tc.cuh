// lowrank_tc.cuh -- pieces shared by the tcgen05 lowrank forward (lowrank_tc.cu)
// and backward (lowrank_bwd_tm.cu) kernels, bf16 only.
//
// Forward work split: a tile is 128 channels (one channel block, the MMA M
// dimension) x 64 timesteps of one batch row.  CTA (dblk, g) of a grid of
// n_dblk x n_groups owns channel block dblk for the contiguous range of tiles
// [j0, j1) of group g, tiles numbered b * tiles_row + t0 / 64, so its U block is
// loaded once.  (The backward uses 128-step tiles; lowrank_bwd_tm.cu.)
//
// z_pack: z rows are 2R bytes (30 at R = 15), which TMA cannot tile (row pitch
// not a multiple of 16 bytes), so z plus the static rank is first packed as
// [R_kernel/8][B][T][8] bf16 -- a 4-D box of that lands in shared memory in the
// no-swizzle K-major operand layout.
#pragma once

#include "common.cuh"

namespace dynconv {
namespace lrtc {

constexpr int kBT = 64;   // timesteps per tile
constexpr int kBD = 128;  // channels per tile (MMA M, TMEM lanes)

struct TileSplit {
  int n_dblk, n_groups, tiles_row, n_tiles;
};

inline TileSplit tile_split(int64_t B, int64_t T, int64_t D) {
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

// Channel groups: G independent convolutions side by side in one activation row
// ([B][T][G*Dg] -- the query, key and value slices of a fused QKV projection),
// each with its own z slice ([B][T][G*R]) and its own U / static_w.  Group g owns
// channel blocks [g*nd, (g+1)*nd); with G > 1, Dg % 128 == 0, so no 128-channel
// block straddles two groups and a block's global first channel is dblk * 128.
struct ChanGroups {
  int G;   // number of groups (1 = the plain op)
  int nd;  // channel blocks per group, ceil(Dg / 128)
  int Dg;  // channels per group
};

inline ChanGroups chan_groups(int64_t D, int G) { return ChanGroups{G, (int)((D + kBD - 1) / kBD), (int)D}; }

// Data-parallel peers of the fused backward (dp_comm.cu): every rank's landing
// buffer [2 parities][world sources][cap floats] and flags [world sources][kMaxDpCtas]
// (one per source CTA: the last call that CTA delivered its slice for) mapped into
// this process (peer memory over NVLink, plain loads and stores), and this rank's
// device-side call counter.  world == 1: no cross-GPU reduction.
constexpr int kMaxWorld = 8;
constexpr int kMaxDpCtas = 256;  // the backward's grid is at most one CTA per SM
struct DpPeers {
  int world, rank;
  int64_t cap;                                   // floats per (parity, source) slot
  float* land[kMaxWorld];                        // rank p's landing buffer
  unsigned long long* flags[kMaxWorld];          // rank p's flags [source][CTA]
  unsigned long long* epoch;                     // this rank's count of completed calls
};

__host__ __device__ constexpr uint32_t round1024(uint32_t v) { return (v + 1023u) / 1024u * 1024u; }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// cuTensorMapEncodeTiled through the runtime's driver entry point (nullptr when
// the driver does not provide it).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn();

// 3-D bf16 map over a [B][T][D] tensor: dims (D, T, B), box (box_d, box_t, 1).
// swizzle_bytes 0 (none), 32, 64 or 128: box_d * 2 must equal it, and the shared-memory
// side must be aligned to 8 x swizzle_bytes (16-byte chunk c of row r sits at chunk
// c ^ ((r >> k) & mask), the pattern TMA and the MMA descriptors share).
int make_btd_map(CUtensorMap* map, const void* base, int64_t B, int64_t T, int64_t D, int box_d, int box_t,
                 int swizzle_bytes = 0);

// 4-D bf16 map over z_pack [G*RKP/8][B][T][8]: dims (8, T, B, G*RKP/8), box (8, rows, 1,
// RKP/8); group g's box starts at coordinate g*RKP/8 of the last dimension.  The box
// lands as [RKP/8][rows][8] (16-byte rows, 8-rank chunks rows*16 bytes apart); rows
// past T read as zero.
int make_zpack_map(CUtensorMap* map, const void* base, int64_t B, int64_t T, int rkp, int rows, int G = 1);

size_t zpack_bytes(int64_t B, int64_t T, int rkp, int G = 1);
// z [B][T][G*R] -> z_pack [G*RKP/8][B][T][8] (static rank and zero padding per group).
int z_pack_launch(const void* z, void* zp, int64_t B, int64_t T, int R, int rkp, bool has_static, cudaStream_t st,
                  int G = 1);

// U_ext block of channels [dlb, dlb + 128) of one group into shared memory as 8 x 8
// blocks [tap][ch/8][r/8][8 r][8 ch] (a 16-byte row = 8 channels of one rank): the
// MN-major operand "M or N = channels, K = ranks" (sbo = (RKP/8) * 128 between
// 8-channel groups, lbo = 128 between 8-rank groups), and also the K-major operand
// "K = channels, N = ranks" of the backward's dz MMA.  Rank R is static_w when
// given, zero up to RKP; channels past Dg are zero.  Consecutive threads fill
// consecutive 16-byte rows (rank-fastest), so the stores are bank-conflict-free;
// each thread issues all its 16-byte loads before its stores.
template <int W, int RKP, int NT>
__device__ void load_u_mn(uint8_t* us, const __nv_bfloat16* __restrict__ U, const __nv_bfloat16* __restrict__ sw,
                          int dlb, int Dg, int R, int tid) {
  constexpr int NV = W * RKP * (kBD / 8);
  constexpr int PER = (NV + NT - 1) / NT;
  uint4 u[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = tid + i * NT;
    u[i] = make_uint4(0, 0, 0, 0);
    if (e < NV) {
      const int r = e % RKP, c8 = (e / RKP) % (kBD / 8), w = e / (RKP * (kBD / 8));
      const int d = dlb + 8 * c8;
      if (d < Dg) {
        if (r < R) u[i] = __ldg(reinterpret_cast<const uint4*>(U + ((size_t)r * W + w) * Dg + d));
        else if (r == R && sw != nullptr) u[i] = __ldg(reinterpret_cast<const uint4*>(sw + (size_t)w * Dg + d));
      }
    }
  }
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = tid + i * NT;
    if (e < NV) {
      const int r = e % RKP, c8 = (e / RKP) % (kBD / 8), w = e / (RKP * (kBD / 8));
      *reinterpret_cast<uint4*>(us + ((w * 16 + c8) * (RKP / 8) + r / 8) * 128 + (r % 8) * 16) = u[i];
    }
  }
}

}  // namespace lrtc
}  // namespace dynconv
