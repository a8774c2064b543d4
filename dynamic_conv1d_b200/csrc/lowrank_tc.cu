// lowrank_tc.cu -- tcgen05 (5th-gen tensor core) lowrank kernels for bf16.
#include "common.cuh"

namespace dynconv {

DYNCONV_DEFINE_ERROR_ACCESSOR(lr_tc_error_word)

bool lr_tc_supported(int64_t D, int Rk, int W, int dtype, const void* const* ptrs, int nptrs) {
  (void)D; (void)Rk; (void)W; (void)dtype; (void)ptrs; (void)nptrs;
  return false;
}

size_t lr_tc_bwd_workspace(int64_t B, int64_t T, int64_t D, int Rk, int W) {
  (void)B; (void)T; (void)D; (void)Rk; (void)W;
  return 0;
}

int lr_tc_fwd_launch(const void*, const void*, const void*, const void*, void*, int64_t, int64_t, int64_t, int, int,
                     int, int, cudaStream_t) {
  return set_error(DYNCONV_ERR_UNSUPPORTED, "tensor-core lowrank forward not built");
}

int lr_tc_bwd_launch(const void*, const void*, const void*, const void*, const void*, void*, void*, float*, void*,
                     void*, void*, size_t, int64_t, int64_t, int64_t, int, int, int, int, cudaStream_t) {
  return set_error(DYNCONV_ERR_UNSUPPORTED, "tensor-core lowrank backward not built");
}

}  // namespace dynconv
