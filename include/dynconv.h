/*
 * dynconv.h -- C ABI of the B200 (sm_100a) dynamic short convolution library
 * (libdynconv.so).  Drop-in boundary for the GPU half of the reference project
 * OliverSieberling/dynamic-conv1d: each entry point replaces one kernel launch
 * site (or launch group) of the reference's autograd Functions.
 *
 * Conventions
 *   - All tensors are caller-allocated device buffers, dense row-major
 *     ("contiguous" in PyTorch terms).  The library never allocates or frees them.
 *   - `dtype` is a dynconv_dtype; every floating tensor of one call shares it,
 *     except the explicitly float* accumulators.
 *   - `stream` is a cudaStream_t passed as void* (0 = legacy default stream).
 *     Calls are asynchronous: no host synchronisation.
 *   - Return value: DYNCONV_OK (0) or a dynconv_status error code; the message of
 *     the last failing call on the calling thread is dynconv_last_error().
 *   - Shapes: x,y,dx,dy [B,T,D]; headwise weight [B,T,H,W]; lowrank z [B,T,R],
 *     U [R, W*D] (viewed as [R][W][D]); static_w [W,D].  W in 1..8.
 *   - Contexts: the library works in the primary context of the current device
 *     (the one the CUDA runtime and PyTorch use).  On a thread with no current
 *     context it makes that primary context current.  Contexts created with
 *     cuCtxCreate are not supported: device pointers, streams and the per-device
 *     state below (the noalloc scratch address, cached SM counts) all belong to
 *     the primary context.
 *   - Errors on the device: the tensor-core kernels bound every wait (1.5 s).  A
 *     wait that gives up makes its kernel return early, leaving that call's
 *     outputs incomplete, and sets a device error word; the call itself has
 *     already returned DYNCONV_OK.  It is reported in two ways: (1) the next
 *     kernel-launching call on the same device that starts after the kernel gave
 *     up returns DYNCONV_ERR_TIMEOUT without launching anything (it reads a word
 *     of pinned, mapped host memory that the kernel also wrote; no
 *     synchronisation), once; (2) dynconv_check_device synchronises the stream
 *     and reports it.  Use (2) once per step to learn of it before the outputs
 *     are used.  The pinned word is set up on a device's first kernel-launching
 *     call that is not being captured into a CUDA graph (that call synchronises
 *     once); before that only (2) reports.  dynconv_lr_fwd_noalloc never sets
 *     it up (it allocates nothing), but reports through it once it exists.
 */
#ifndef DYNCONV_H_
#define DYNCONV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with hidden default visibility; everything declared
 * here is exported. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define DYNCONV_ABI_VERSION 1

typedef enum dynconv_dtype {
  DYNCONV_DTYPE_BF16 = 0,
  DYNCONV_DTYPE_F32 = 1
} dynconv_dtype;

typedef enum dynconv_status {
  DYNCONV_OK = 0,
  DYNCONV_ERR_SHAPE = 1,       /* inconsistent or out-of-range sizes            */
  DYNCONV_ERR_ALIGN = 2,       /* a pointer is not aligned as the kernel needs  */
  DYNCONV_ERR_UNSUPPORTED = 3, /* valid for the reference, not for this build   */
  DYNCONV_ERR_CUDA = 4,        /* a CUDA runtime/driver call failed             */
  DYNCONV_ERR_TIMEOUT = 5,     /* a bounded device-side wait gave up            */
  DYNCONV_ERR_WORKSPACE = 6,   /* workspace missing or too small                */
  DYNCONV_ERR_ARGUMENT = 7     /* null pointer where a tensor is required       */
} dynconv_status;

/* Library identity and diagnostics. */
int dynconv_abi_version(void);
const char* dynconv_status_string(int status);
const char* dynconv_last_error(void);
/* Synchronises `stream`, then reads and clears the device error word that
 * bounded waits inside the tensor-core kernels set when they give up (and the
 * pinned host-visible copy of it, so the next call does not report the same
 * event).  Returns DYNCONV_OK, DYNCONV_ERR_TIMEOUT or DYNCONV_ERR_CUDA. */
int dynconv_check_device(void* stream);
/* Number of kernels this library has launched in this process (all devices,
 * all threads).  Diagnostic only; no reference counterpart. */
uint64_t dynconv_launch_count(void);

/* ---------------------------------------------------------------- headwise */

/* y = sum_w (weight[b,t,d/hs,w] + static_w[w,d]) * x[b,t-w,d]  (+ x if residual)
 * Replaces the causal_conv1d_fwd_kernel launch in
 * _HeadwiseDynamicConvolutionFn.forward (headwise.py:220-254; launch :234-248).
 * static_w may be NULL.  hs = D/H must be a power of two. */
int dynconv_hw_fwd(const void* x, const void* weight, const void* static_w, void* y,
                   int64_t B, int64_t T, int64_t D, int64_t H, int64_t W,
                   int dtype, int residual, void* stream);

/* Workspace for dynconv_hw_bwd (bytes; 0 when static_w is absent). */
size_t dynconv_hw_bwd_workspace_bytes(int64_t B, int64_t T, int64_t D, int64_t H, int64_t W,
                                      int dtype, int has_static);

/* Backward of dynconv_hw_fwd for upstream gradient dy.
 * Replaces the causal_conv1d_bwd_kernel launch and the dstatic cast in
 * _HeadwiseDynamicConvolutionFn.backward (headwise.py:257-309; launch :283-300).
 * Writes dx [B,T,D] and dweight [B,T,H,W] (no power-of-two padding of W).
 * With static_w != NULL: the float32 sum over (b,t) of dy*x_shift is written to
 * dstatic_w_f32 [W,D] (required) and, when dstatic_w != NULL, also cast to
 * `dtype` into dstatic_w.  The reduction is deterministic (fixed-order two-pass). */
int dynconv_hw_bwd(const void* x, const void* weight, const void* static_w, const void* dy,
                   void* dx, void* dweight, void* dstatic_w, float* dstatic_w_f32,
                   void* workspace, size_t workspace_bytes,
                   int64_t B, int64_t T, int64_t D, int64_t H, int64_t W,
                   int dtype, int residual, void* stream);

/* ----------------------------------------------------------------- lowrank */

/* Workspace for dynconv_lr_fwd (bytes; may be 0). */
size_t dynconv_lr_fwd_workspace_bytes(int64_t B, int64_t T, int64_t D, int64_t R, int64_t W,
                                      int dtype, int has_static);

/* y = sum_w ((z@U).view(B,T,W,D)[b,t,w,d] + static_w[w,d]) * x[b,t-w,d] (+ x)
 * Replaces the static-rank fold (F.pad / torch.cat, lowrank.py:222-226) and the
 * causal_conv1d_fwd_kernel launch (lowrank.py:230-242) of
 * _LowrankDynamicConvolutionFn.forward.  static_w is folded in as rank R
 * (R_kernel = R + 1); U is never concatenated.  The bf16 tensor-core path packs
 * z_ext (z plus the static rank) into the workspace, [R_kernel/8][B][T][8], so
 * TMA can place it in the MMA operand layout.  Any R >= 1 with R_kernel <= 64 is
 * accepted (the reference needs R_kernel a power of two >= 16). */
int dynconv_lr_fwd(const void* x, const void* z, const void* U, const void* static_w, void* y,
                   void* workspace, size_t workspace_bytes,
                   int64_t B, int64_t T, int64_t D, int64_t R, int64_t W,
                   int dtype, int residual, void* stream);

/* Fixed size of the scratch array that dynconv_lr_fwd_noalloc uses (8 MiB per
 * device): enough for B*T <= 262144 tokens at R_kernel <= 16, 131072 at <= 32. */
#define DYNCONV_LR_FWD_NOALLOC_SCRATCH_BYTES ((size_t)8 << 20)

/* dynconv_lr_fwd without a caller workspace: no counterpart in the reference.
 * For callers that cannot allocate device memory at the call -- a host-language
 * binding (cgo, JNI, plain C) with no access to PyTorch's caching allocator that
 * must not call cudaMalloc on its hot path (cudaMalloc/cudaFree synchronise the
 * device), or a server that reserves all memory at start-up.  Allocates nothing:
 * the scratch is a static device array of DYNCONV_LR_FWD_NOALLOC_SCRATCH_BYTES
 * bytes inside the library, one per device; nothing in it has to start at zero.
 * Same arguments and results as dynconv_lr_fwd otherwise.
 *   - The first call on each device (with that device current) does a one-time
 *     set-up: it looks up the scratch address, which also loads the library's
 *     module on that device.  Make that first call before any stream capture.
 *     The address is cached per device ordinal, for the device's primary context
 *     (the only kind of context the library supports).
 *   - Sizes whose workspace (dynconv_lr_fwd_workspace_bytes) exceeds the scratch
 *     are rejected with DYNCONV_ERR_WORKSPACE; use dynconv_lr_fwd for those.
 *   - All calls on one device share the one scratch array: two calls that can
 *     overlap (different streams, or host threads without ordering between them)
 *     race on it.  Issue them on one stream, or order them. */
int dynconv_lr_fwd_noalloc(const void* x, const void* z, const void* U, const void* static_w, void* y,
                           int64_t B, int64_t T, int64_t D, int64_t R, int64_t W,
                           int dtype, int residual, void* stream);

/* Workspace for dynconv_lr_bwd (bytes). */
size_t dynconv_lr_bwd_workspace_bytes(int64_t B, int64_t T, int64_t D, int64_t R, int64_t W,
                                      int dtype, int has_static);

/* Backward of dynconv_lr_fwd.  Replaces the dU/dz and dx kernel launches, the
 * float32 dU zero-init and the cast/split of _LowrankDynamicConvolutionFn.backward
 * (lowrank.py:252-299; launches :266-292).
 * Writes dx [B,T,D], dz [B,T,R] and the float32 accumulator dU_f32 [R_kernel, W*D]
 * (rows 0..R-1 = dU, row R = dstatic_w when static_w != NULL; required).  When dU
 * (and dstatic_w) are non-NULL, the accumulator is also cast to `dtype` into
 * dU [R, W*D] and dstatic_w [W,D].  Pass dU = dstatic_w = NULL to all-reduce
 * dU_f32 across data-parallel ranks first and cast afterwards with dynconv_cast_f32. */
int dynconv_lr_bwd(const void* x, const void* z, const void* U, const void* static_w, const void* dy,
                   void* dx, void* dz, void* dU, void* dstatic_w, float* dU_f32,
                   void* workspace, size_t workspace_bytes,
                   int64_t B, int64_t T, int64_t D, int64_t R, int64_t W,
                   int dtype, int residual, void* stream);

/* ------------------------------------------------------ grouped (Q/K/V) lowrank */

/* G low-rank convolutions that share B, T, D, R, W -- the query, key and value
 * convolutions of one attention layer (reference README.md:86-105, three
 * LowRankDynamicShortConvolution modules) -- in one launch of each kernel.  No
 * reference counterpart as one call: it replaces G calls of dynconv_lr_fwd /
 * dynconv_lr_bwd, with the same results per group.
 *   x, y, dy, dx : [B, T, G*D]  group g owns channels [g*D, (g+1)*D) of each row --
 *                  the layout of a fused QKV projection's output, so q, k and v
 *                  are read in place, with no split or copy
 *   z, dz        : [B, T, G*R]  group g's z in columns [g*R, (g+1)*R)
 *   U, dU        : [G, R, W*D]
 *   static_w, dstatic_w : [G, W, D] (optional, as for the single op)
 *   dU_f32       : [G, R_kernel, W*D], group g's rows as dynconv_lr_bwd's dU_f32
 * With G > 1 the call needs the tensor-core path: bf16, W <= 4, R_kernel <= 64
 * (forward) / <= 32 (backward), D % 128 == 0, G*D/128 <= the SM count (backward),
 * 16-byte aligned tensors; anything else returns DYNCONV_ERR_UNSUPPORTED (call
 * the single op per group).  G = 1 is exactly dynconv_lr_fwd / dynconv_lr_bwd.
 * G in 1..16. */
size_t dynconv_lr_fwd_grouped_workspace_bytes(int64_t B, int64_t T, int64_t D, int64_t R, int64_t W, int64_t G,
                                              int dtype, int has_static);
int dynconv_lr_fwd_grouped(const void* x, const void* z, const void* U, const void* static_w, void* y,
                           void* workspace, size_t workspace_bytes,
                           int64_t B, int64_t T, int64_t D, int64_t R, int64_t W, int64_t G,
                           int dtype, int residual, void* stream);
size_t dynconv_lr_bwd_grouped_workspace_bytes(int64_t B, int64_t T, int64_t D, int64_t R, int64_t W, int64_t G,
                                              int dtype, int has_static);
/* z_packed: NULL, or the workspace of the dynconv_lr_fwd_grouped call that produced y from
 * this same z (same B, T, R, G and static_w presence, z unchanged since): on the tensor-core
 * path that workspace holds z packed for the MMAs, and the backward reads it instead of
 * packing z again (one launch fewer).  16-byte aligned. */
int dynconv_lr_bwd_grouped(const void* x, const void* z, const void* U, const void* static_w, const void* dy,
                           void* dx, void* dz, void* dU, void* dstatic_w, float* dU_f32,
                           void* workspace, size_t workspace_bytes,
                           int64_t B, int64_t T, int64_t D, int64_t R, int64_t W, int64_t G,
                           int dtype, int residual, const void* z_packed, void* stream);

/* ------------------------------------------- data parallel (fused all-reduce) */

/* A communicator for the fused data-parallel backward: one per rank (one process
 * per GPU, world 2..8 on one node), made once, before any stream capture.  No
 * reference counterpart: it replaces the NCCL all-reduce of the float32
 * shared-gradient buffer that the reference's caller would run after backward.
 *   1. dynconv_comm_create(world, rank, max_floats, &comm, blob) on each rank, with
 *      that rank's GPU current: allocates this rank's landing buffer
 *      (2 x world x max_floats floats) and flags, and writes a blob of
 *      dynconv_comm_blob_bytes() bytes (CUDA IPC handles, device UUID, rank);
 *   2. exchange the blobs (any host channel, e.g. torch.distributed), in rank order;
 *   3. dynconv_comm_connect(comm, blobs) on each rank: maps every peer's buffers
 *      (refuses two ranks on one GPU);
 *   4. dynconv_lr_bwd_grouped_dp(...) on every rank, the same number of calls, in the
 *      same order: dU_f32 (and dU / dstatic_w when given) receive the SUM over all
 *      ranks, reduced inside the backward kernel over peer memory (NVLink stores,
 *      bounded waits: a rank that never arrives makes the others' kernels return
 *      and dynconv_check_device report DYNCONV_ERR_TIMEOUT);
 *   5. dynconv_comm_destroy(comm) once no rank will call again.
 * max_floats: a multiple of 4, at least G * R_kernel * W * D of every call. */
size_t dynconv_comm_blob_bytes(void);
int dynconv_comm_create(int world, int rank, int64_t max_floats, void** comm, void* blob);
int dynconv_comm_connect(void* comm, const void* blobs);
int dynconv_comm_destroy(void* comm);
/* dynconv_lr_bwd_grouped, with the shared gradients summed over the communicator's
 * ranks.  Tensor-core path only (bf16, W <= 4, R_kernel <= 32, 16-byte aligned);
 * otherwise DYNCONV_ERR_UNSUPPORTED. */
int dynconv_lr_bwd_grouped_dp(const void* x, const void* z, const void* U, const void* static_w, const void* dy,
                              void* dx, void* dz, void* dU, void* dstatic_w, float* dU_f32,
                              void* workspace, size_t workspace_bytes,
                              int64_t B, int64_t T, int64_t D, int64_t R, int64_t W, int64_t G,
                              int dtype, int residual, const void* z_packed, void* comm, void* stream);

/* dst[i] = (dtype) src[i], i < n, round-to-nearest-even.  Used after the
 * data-parallel all-reduce of the float32 shared-gradient buffers (replaces
 * dU_fp32.to(U.dtype), lowrank.py:294, and dstatic_accum.to(...), headwise.py:305). */
int dynconv_cast_f32(const float* src, void* dst, int64_t n, int dtype, void* stream);

/* ------------------------------------------------------------- diagnostics */

/* One tcgen05.mma (kind::f16, bf16 in, fp32 accumulate) sequence on operands
 * staged into the canonical no-swizzle shared-memory layouts used by the
 * lowrank kernels, for the unit tests of descriptor encodings.  No reference
 * counterpart.  A: logical [M][K] bf16 row-major; B: logical [K][Nb] bf16
 * row-major (Nb >= N + b_row_offset); D: [M][N] float32 = A @ B[:, off:off+N].
 * a_major/b_major: 0 = K-major, 1 = MN-major (a_major 2: A staged K-major in
 * tensor memory, M = 128); *_sbo/*_lbo: byte strides of the staged layout;
 * b_row_offset shifts a K-major B by whole rows (16 B each); a_row_offset does
 * the same for a K-major A given with M + a_row_offset rows (D = A[off:off+M] @ B). */
int dynconv_umma_selftest(const void* A, const void* B, float* D,
                          int M, int N, int K, int Nb,
                          int a_major, int a_sbo, int a_lbo,
                          int b_major, int b_sbo, int b_lbo, int b_row_offset,
                          int a_row_offset, void* stream);

/* Test hook for the fault-containment path (no reference counterpart): launches one
 * CTA that waits on an mbarrier no thread ever arrives on, through the kernels'
 * bounded-wait code, with a limit of limit_ns (1 ns .. 100 ms).  The wait gives up,
 * sets the device error word and the kernel returns; a following
 * dynconv_check_device() reports DYNCONV_ERR_TIMEOUT once and clears the word.
 * out (device int, may be NULL) receives 0 when the wait gave up. */
int dynconv_wait_selftest(uint64_t limit_ns, int* out, void* stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* DYNCONV_H_ */
