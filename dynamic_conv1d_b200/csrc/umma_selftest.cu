// umma_selftest.cu -- a single-CTA tcgen05.mma check of the shared-memory
// descriptor encodings (no-swizzle K-major and MN-major operands, arbitrary
// SBO/LBO, row-shifted K-major A or B), of the 128-byte-swizzled MN-major A operand
// (the layout a SWIZZLE_128B TMA load writes) and of the TMEM accumulator layout
// for M = 64 and M = 128, as used by the lowrank tensor-core kernels.
// Exposed through dynconv_umma_selftest() for the GPU unit tests only.
#include "common.cuh"

namespace dynconv {

DYNCONV_DEFINE_ERROR_ACCESSOR(selftest_error_word)

__global__ void __launch_bounds__(128) umma_selftest_kernel(const __nv_bfloat16* __restrict__ A,
                                                            const __nv_bfloat16* __restrict__ Bm,
                                                            float* __restrict__ Dout, int M, int N, int K, int Nb,
                                                            int a_major, uint32_t a_sbo, uint32_t a_lbo, int b_major,
                                                            uint32_t b_sbo, uint32_t b_lbo, int b_off, int a_off,
                                                            uint32_t a_bytes, uint32_t ncols) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  uint8_t* As = smem;
  uint8_t* Bs = smem + (a_bytes + 1023u) / 1024u * 1024u;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const bool a_tmem = (a_major == 2);  // A staged in TMEM after the D columns
  if (!a_tmem) {
    // A has M + a_off rows; the MMA reads rows a_off .. a_off + M - 1
    for (int i = tid; i < (M + a_off) * K; i += blockDim.x) {
      const int m = i / K, k = i % K;
      const uint32_t off = a_major == 3 ? mnmajor_sw128_off(m, k, a_lbo)
                           : a_major   ? mnmajor_off(m, k, a_sbo, a_lbo)
                                       : kmajor_off(m, k, a_sbo, a_lbo);
      *reinterpret_cast<__nv_bfloat16*>(As + off) = A[i];
    }
  }
  for (int i = tid; i < K * Nb; i += blockDim.x) {
    const int k = i / Nb, n = i % Nb;
    const uint32_t off = b_major ? mnmajor_off(n, k, b_sbo, b_lbo) : kmajor_off(n, k, b_sbo, b_lbo);
    *reinterpret_cast<__nv_bfloat16*>(Bs + off) = Bm[i];
  }
  fence_proxy_async_smem();
  if (tid == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, ncols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_slot;
  const uint32_t a_col = (uint32_t)N;  // A columns follow the N accumulator columns
  if (a_tmem) {
    // M == 128: warp w writes rows 32w..32w+31, K/2 packed columns per row, 8 at a time
    const int m = 32 * warp + lane;
    for (int c0 = 0; c0 < K / 2; c0 += 8) {
      uint32_t v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const __nv_bfloat162 p2 = __halves2bfloat162(A[(size_t)m * K + 2 * (c0 + j)], A[(size_t)m * K + 2 * (c0 + j) + 1]);
        v[j] = *reinterpret_cast<const uint32_t*>(&p2);
      }
      tmem_st8(tbase + ((uint32_t)(32 * warp) << 16) + a_col + (uint32_t)c0, v);
    }
    tmem_st_wait();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }

  if (tid == 0) {
    const uint32_t idesc = make_idesc_bf16(M, N, a_tmem ? 0 : (a_major ? 1 : 0), b_major);
    const uint32_t a0 = smem_u32(As) + (uint32_t)a_off * 16u, b0 = smem_u32(Bs) + (uint32_t)b_off * 16u;
    for (int ks = 0; ks < K / 16; ++ks) {
      const uint64_t bd = make_smem_desc(b0 + (uint32_t)ks * 2u * b_lbo, b_lbo, b_sbo);
      if (a_tmem) {
        umma_f16_ts(tbase, tbase + a_col + (uint32_t)ks * 8u, bd, idesc, ks > 0 ? 1u : 0u);
      } else {
        const uint64_t ad = a_major == 3 ? make_smem_desc_sw128(a0 + (uint32_t)ks * 2u * a_sbo, a_lbo, a_sbo)
                                         : make_smem_desc(a0 + (uint32_t)ks * 2u * a_lbo, a_lbo, a_sbo);
        umma_f16(tbase, ad, bd, idesc, ks > 0 ? 1u : 0u);
      }
    }
    umma_commit(&bar);
  }
  const bool ok = mbar_wait(&bar, 0, kErrWaitMma, &abort_flag);
  tc_fence_after();
  if (ok) {
    for (int c0 = 0; c0 < N; c0 += 16) {
      float v[16];
      tmem_ld16(tbase + ((uint32_t)(32 * warp) << 16) + (uint32_t)c0, v);
      tmem_ld_wait();
      int m = -1;
      if (M == 128) m = 32 * warp + lane;
      else if (lane < 16) m = 16 * warp + lane;
      if (m >= 0) {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (c0 + j < N) Dout[(size_t)m * N + c0 + j] = v[j];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, ncols);
}

static uint32_t span_bytes(int major, int mn_extent, int k_extent, uint32_t sbo, uint32_t lbo) {
  const uint32_t last = major ? mnmajor_off(mn_extent - 1, k_extent - 1, sbo, lbo)
                              : kmajor_off(mn_extent - 1, k_extent - 1, sbo, lbo);
  // the MMA reads whole 16-byte rows of the last core matrix
  return ((last + 16u + 127u) / 128u) * 128u + 128u;
}

int umma_selftest_launch(const void* A, const void* B, float* D, int M, int N, int K, int Nb, int a_major, int a_sbo,
                         int a_lbo, int b_major, int b_sbo, int b_lbo, int b_off, int a_off, cudaStream_t st) {
  if (!(M == 64 || M == 128)) return set_error(DYNCONV_ERR_SHAPE, "selftest: M must be 64 or 128");
  if (N < 16 || N > 256 || N % 16 != 0) return set_error(DYNCONV_ERR_SHAPE, "selftest: N in 16..256, multiple of 16");
  if (K < 16 || K % 16 != 0) return set_error(DYNCONV_ERR_SHAPE, "selftest: K multiple of 16");
  if (Nb < N + b_off) return set_error(DYNCONV_ERR_SHAPE, "selftest: Nb < N + b_row_offset");
  if (b_off != 0 && (b_major != 0 || b_sbo != 128))
    return set_error(DYNCONV_ERR_SHAPE, "selftest: row offset needs K-major B with SBO = 128");
  if (a_off < 0 || b_off < 0 || a_off > 64 || (a_off != 0 && (a_major != 0 || a_sbo != 128)))
    return set_error(DYNCONV_ERR_SHAPE, "selftest: A row offset (0..64) needs K-major A with SBO = 128");
  if ((a_sbo | a_lbo | b_sbo | b_lbo) & 15) return set_error(DYNCONV_ERR_ALIGN, "selftest: strides must be 16-byte multiples");
  if (a_major == 2 && (M != 128 || N + K / 2 > 256))
    return set_error(DYNCONV_ERR_SHAPE, "selftest: A in TMEM needs M = 128 and N + K/2 <= 256");
  if (a_major == 3 && (a_sbo != 1024 || a_lbo % 1024 != 0 || a_lbo < (K + 7) / 8 * 1024))
    return set_error(DYNCONV_ERR_SHAPE, "selftest: swizzled A needs SBO = 1024 and LBO a multiple of 1024 past its rows");
  const uint32_t abytes = a_major == 2   ? 128u
                          : a_major == 3 ? (uint32_t)((M + 63) / 64) * (uint32_t)a_lbo
                                         : span_bytes(a_major, M + a_off, K, (uint32_t)a_sbo, (uint32_t)a_lbo);
  const uint32_t bbytes = span_bytes(b_major, Nb, K, (uint32_t)b_sbo, (uint32_t)b_lbo);
  const uint32_t smem = (abytes + 1023u) / 1024u * 1024u + bbytes;
  if (smem > 200 * 1024) return set_error(DYNCONV_ERR_SHAPE, "selftest: operands need %u bytes of smem", smem);
  uint32_t ncols = 32;
  while (ncols < (uint32_t)N + (a_major == 2 ? (uint32_t)K / 2 : 0u)) ncols <<= 1;
  // Reserve the whole shared memory so any descriptor walk stays inside this CTA's window.
  const int smem_alloc = 220 * 1024;
  cudaError_t e = cudaFuncSetAttribute(umma_selftest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_alloc);
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(umma_selftest)");
  umma_selftest_kernel<<<1, 128, smem_alloc, st>>>((const __nv_bfloat16*)A, (const __nv_bfloat16*)B, D, M, N, K, Nb,
                                                   a_major, (uint32_t)a_sbo, (uint32_t)a_lbo, b_major, (uint32_t)b_sbo,
                                                   (uint32_t)b_lbo, b_off, a_off, abytes, ncols);
  DYNCONV_CHECK_LAUNCH("umma_selftest_kernel");
  return DYNCONV_OK;
}

// A wait that nobody ends: one CTA waits on an mbarrier that no thread arrives on,
// through the same bounded slow path the kernels use, with a short limit.  The
// wait gives up, records its site in this file's device error word, raises the
// CTA's abort flag and returns; the kernel then exits normally.  Exercises the
// timeout path end to end (dynconv_check_device reports DYNCONV_ERR_TIMEOUT).
__global__ void __launch_bounds__(32) wait_selftest_kernel(uint64_t limit_ns, int* out) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncwarp();
  bool ok = mbar_try_wait(&bar, 0);
  if (!ok) ok = mbar_wait_slow(&bar, 0, kErrWaitTail, &abort_flag, limit_ns);
  if (threadIdx.x == 0 && out) out[0] = ok ? 1 : 0;
}

int wait_selftest_launch(uint64_t limit_ns, int* out, cudaStream_t st) {
  wait_selftest_kernel<<<1, 32, 0, st>>>(limit_ns, out);
  DYNCONV_CHECK_LAUNCH("wait_selftest_kernel");
  return DYNCONV_OK;
}

}  // namespace dynconv
