/*
 * b2msl.h — C ABI of the B200 (sm_100a) hot-path kernels that replace the
 * Metal template path of triton-msl (FlashAttention forward, fast matmul with
 * bias/activation epilogue, row-reduction family).
 *
 * Conventions (all entry points):
 *  - Plain device pointers and sizes; strides are in ELEMENTS, like the stride
 *    arguments the reference's Triton kernels receive.
 *  - `stream` is a cudaStream_t (NULL = legacy default stream). Every call is
 *    stream-ordered and asynchronous; nothing synchronises the host.
 *  - The library never allocates device memory on these paths; scratch space,
 *    where a path needs it, is passed in (`workspace`, sized by
 *    b2_query_workspace()).
 *  - Return 0 on success or a negative B2_E* status. Validation happens before
 *    any launch, so a failed call has launched nothing. The reference raises
 *    MetalNonRecoverableError instead of producing wrong numbers
 *    (triton_msl/errors.py:82-102); this ABI returns B2_EINVAL/B2_EUNSUPPORTED
 *    and the message is available from b2_last_error() on the same thread.
 *  - Device-side waits are bounded; a wedged pipeline sets a bit in the
 *    device status word (b2_device_status) instead of hanging.
 */
#ifndef B2MSL_H_
#define B2MSL_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* status codes */
#define B2_OK 0
#define B2_EINVAL (-1)       /* bad shape / stride / pointer / dtype combination */
#define B2_EUNSUPPORTED (-2) /* valid request this build does not implement */
#define B2_ELAUNCH (-3)      /* CUDA runtime error while launching */
#define B2_ETIMEOUT (-4)     /* a bounded device wait expired (see b2_device_status) */

/* element types */
#define B2_F32 0
#define B2_F16 1
#define B2_BF16 2
#define B2_I64 3

/* GEMM epilogue activations (reference op table: triton_msl/codegen/_lowerer_templates.py:1733-1748) */
#define B2_ACT_NONE 0
#define B2_ACT_RELU 1
#define B2_ACT_GELU 2      /* exact erf GELU */
#define B2_ACT_GELU_TANH 3 /* tanh-approximated GELU */
#define B2_ACT_SILU 4
#define B2_ACT_SOFTMAX 5   /* softmax over each output row (fused matmul -> row softmax,
                              reference _lowerer_templates.py:1515-1728); needs N <= 256 */

/* Epilogue op codes (b2_gemm_epilogue): each op maps the running fp32 value
 * x of an output element; a and b are the op's two constants, bias[n] the
 * column bias. Reference op tables: triton_msl/codegen/_lowerer_templates.py:1733-1748. */
#define B2_EPI_ADD 1        /* x + a */
#define B2_EPI_SUB 2        /* x - a */
#define B2_EPI_RSUB 3       /* a - x */
#define B2_EPI_MUL 4        /* x * a */
#define B2_EPI_DIV 5        /* x / a */
#define B2_EPI_RDIV 6       /* a / x */
#define B2_EPI_ADD_BIAS 7   /* x + bias[n] */
#define B2_EPI_MUL_BIAS 8   /* x * bias[n] */
#define B2_EPI_MAX 9        /* max(x, a), NaN-propagating (tl.maximum) */
#define B2_EPI_MIN 10       /* min(x, a), NaN-propagating (tl.minimum) */
#define B2_EPI_MAXNUM 11    /* max(x, a), NaN-quiet (IEEE maxNum) */
#define B2_EPI_MINNUM 12    /* min(x, a), NaN-quiet */
#define B2_EPI_CLAMP 13     /* min(max(x, a), b), NaN-propagating (torch.clamp) */
#define B2_EPI_CLAMPNUM 14  /* min(max(x, a), b), NaN-quiet */
#define B2_EPI_NEG 15
#define B2_EPI_EXP 16
#define B2_EPI_EXP2 17
#define B2_EPI_LOG 18
#define B2_EPI_LOG2 19
#define B2_EPI_SQRT 20
#define B2_EPI_RSQRT 21
#define B2_EPI_SIN 22
#define B2_EPI_COS 23
#define B2_EPI_ERF 24
#define B2_EPI_TANH 25
#define B2_EPI_FLOOR 26
#define B2_EPI_CEIL 27
#define B2_EPI_ABS 28
#define B2_EPI_RELU 29      /* NaN-propagating, like torch.relu */
#define B2_EPI_GELU 30      /* exact erf GELU */
#define B2_EPI_GELU_TANH 31
#define B2_EPI_SILU 32
#define B2_EPI_SIGMOID 33
#define B2_EPI_FMA 34       /* x * a + b */
#define B2_EPI_MAX_OPS 16

/* row operations (b2_row_op) */
#define B2_ROW_SOFTMAX 0
#define B2_ROW_LAYERNORM 1
#define B2_ROW_RMSNORM 2
#define B2_ROW_SUM 3
#define B2_ROW_MAX 4
#define B2_ROW_ARGMAX 5
#define B2_ROW_MIN 6
#define B2_ROW_ARGMIN 7

/* Library version, e.g. "b2msl 0.1.0 sm_100a". */
const char* b2_version(void);

/* Last error message of the calling thread ("" if none). */
const char* b2_last_error(void);

/* Kernel family the calling thread's last successful call launched
 * ("fa_sm100", "fa_simt", "gemm_sm100" (128x256 tiles), "gemm_sm100_n128"
 * (128x128 tiles), "gemm_sm100_pair" (256x256 tiles on CTA pairs), "gemm_sm100_splitk", "gemm_sm100_tf32x3", "gemm_simt",
 * "row_reduce", "row_split", "row_memset"). Introspection for tests and benchmarks; the reference's
 * equivalent is its TRITON_MSL_PATH_LOG lowering-path log
 * (triton_msl/codegen/msl_emitter.py:523-538). */
const char* b2_last_kernel(void);

/*
 * FlashAttention forward: o = softmax(sm_scale * q @ k^T [+ causal mask]) @ v.
 *
 * Replaces the reference FA entry: the @triton.jit kernel `_flash_attn_fwd`
 * (tests/test_flash_attention.py:35-118) lowered to the simdgroup template
 * `make_flash_attention_kernel_simdgroup` (triton_msl/codegen/_msl_templates.py:1833-2070),
 * whose buffer ABI is (Q, K, V, Out, 16 strides in the order
 * q.zhmk, k.zhnk, v.zhnk, o.zhmk, Z, H, N_CTX) (_msl_templates.py:2108-2121).
 * Here Z=B, N_CTX=S; strides[16] is that same 16-stride list in elements.
 * q, k, v and o share `dtype` (B2_F32, B2_F16 or B2_BF16); accumulation is
 * fp32. The causal mask keeps key j for query i iff j <= i; rows with no
 * unmasked key produce zeros (reference oracle nan_to_num, tests/test_flash_attention.py:124-135).
 */
int b2_fa_fwd(const void* q, const void* k, const void* v, void* o,
              int64_t B, int64_t H, int64_t S, int64_t D,
              const int64_t strides[16], float sm_scale, int causal, int dtype,
              void* stream);

/*
 * GEMM with fused epilogue: C = act(alpha * (A @ B) + bias[None, :]).
 *
 * Replaces the fast-matmul template `make_simdgroup_matmul_kernel_fast`
 * (triton_msl/codegen/_msl_templates.py:4134-4255) dispatched by
 * `dispatch_fast_matmul` (triton_msl/autotuning/_fast_matmul_dispatch.py:27-158)
 * and the staged epilogue template (_lowerer_templates.py:1515-1855). Stride
 * arguments follow the reference's `mm` kernel (tests/test_fast_matmul_parity.py:14-27):
 * strides[6] = {s_am, s_ak, s_bk, s_bn, s_cm, s_cn} in elements.
 * in_dtype applies to A and B; bias (may be NULL) has bias_dtype; C has out_dtype.
 * fp32 inputs: given the workspace b2_query_workspace(0, M, N, K, B2_F32)
 * reports (on sm_100 GPUs), the tensor cores compute the product as 3xTF32
 * (x = hi + lo, A.B = hi.hi + hi.lo + lo.hi; no input rounding to TF32
 * alone; the tensor core's fp32 accumulation adds an error that grows with K,
 * measured 2.5e-5 * max|C| at K=2048); with no workspace, fp32 FMA.
 * fp16/bf16 inputs: shapes with at least one full wave of 256x256 output
 * tiles and at most 4e12 FLOP run on CTA pairs (two SMs per tile, M=256
 * tensor-core MMAs; a last wave that fills at most half of the pairs runs as
 * 256x128 half tiles); the others on one SM per 128x256 or 128x128 tile,
 * whichever leaves fewer SMs idle for the work; when even narrow tiles would fill at most half the SMs and K >= 512,
 * the K loop is split across CTAs (split-K) given the workspace
 * b2_query_workspace reports, with fp32 partial sums reduced in a fixed order
 * before the epilogue (without the workspace the unsplit kernel runs).
 * workspace/ws_bytes: scratch as reported by b2_query_workspace (may be NULL/0
 * when that reports 0, or to force the FMA path for fp32).
 */
int b2_gemm(const void* A, const void* Bm, const void* bias, void* C,
            int64_t M, int64_t N, int64_t K, const int64_t strides[6],
            float alpha, int act, int in_dtype, int bias_dtype, int out_dtype,
            void* workspace, size_t ws_bytes, void* stream);

/*
 * GEMM with a general fused epilogue: C = f_n(...f_1(A @ B)) with fp32 math,
 * f_i given by codes[i] (B2_EPI_*) and the constants args[2i], args[2i+1];
 * 0 <= n_ops <= B2_EPI_MAX_OPS. The accumulator enters the chain unscaled and
 * without bias (use B2_EPI_MUL / B2_EPI_ADD_BIAS). Replaces the reference's
 * fused epilogue lowering of an ordered op chain on the dot result
 * (_emit_matmul_epilogue_loop, triton_msl/codegen/_lowerer_templates.py:1749-1855,
 * op tables :1733-1748), which the reference applies only to single-strip
 * (N <~ 200) matmuls; here any shape, on the same kernels and path selection
 * as b2_gemm (tensor cores, split-K, CUDA cores). Other arguments as b2_gemm.
 */
int b2_gemm_epilogue(const void* A, const void* Bm, const void* bias, void* C,
                     int64_t M, int64_t N, int64_t K, const int64_t strides[6],
                     const int32_t* codes, const float* args, int n_ops,
                     int in_dtype, int bias_dtype, int out_dtype,
                     void* workspace, size_t ws_bytes, void* stream);

/*
 * Row operation over x[rows, cols] (row stride ld_x elements, unit column stride).
 *
 * Replaces the reference row family: the TG-cached softmax / LayerNorm
 * templates (triton_msl/codegen/_lowerer_templates.py:992-1320), the generic
 * tt.reduce lowering for sum/max/argmax (_lowerer_reduce.py:773-1333) and the
 * prebuilt make_row_reduce_kernel / make_softmax_kernel / make_rms_norm_kernel /
 * make_layer_norm_kernel ABIs (_msl_templates.py:259-449, 888-1090).
 *   SOFTMAX:   out[r, :] = softmax(x[r, :])                       (out like x)
 *   LAYERNORM: out = (x - mean) * rsqrt(var + eps) * w + b      (w, b may be NULL)
 *   RMSNORM:   out = x * rsqrt(mean(x^2) + eps) * w               (w may be NULL)
 *   SUM/MAX/MIN: out[r] = reduce(x[r, :])        (out has x's dtype, NaN propagates)
 *   ARGMAX/ARGMIN: out[r] = int64 index; ties -> lowest index; a NaN counts as
 *              the extreme value (first NaN wins), matching torch.argmax.
 * w and b have x's dtype. ld_out is the output row stride (elements) for the
 * row-shaped outputs and ignored for the per-row scalars.
 * workspace: scratch for the split-row path used when rows are few and long;
 * size from b2_query_workspace (0 for most shapes).
 */
int b2_row_op(int op, const void* x, const void* w, const void* b, void* out,
              int64_t rows, int64_t cols, int64_t ld_x, int64_t ld_out,
              float eps, int dtype, void* workspace, size_t ws_bytes,
              void* stream);

/*
 * Row sum / max / min / argmax / argmin over x[rows, cols] (row stride ld_x,
 * unit column stride) that allocates nothing and takes no workspace.
 *
 * No counterpart in the reference: it is an addition for callers that cannot
 * allocate device memory when they reduce -- code inside a custom allocator or
 * an out-of-memory handler, or a host runtime that forbids cudaMalloc after
 * start-up. It always runs the split-row kernels: results are identical to
 * b2_row_op's wherever b2_row_op takes its split-row path (few long rows) and
 * differ only by fp32 summation order elsewhere; indices are exact.
 *  - Scratch is a fixed 256 KiB array in the library's device image, held on
 *    every GPU that loads the library until the process exits. It holds
 *    rows * ceil(cols / 65536) <= 16384 partial results; larger requests fail
 *    with B2_EINVAL (use b2_row_op with a workspace for those).
 *  - The first call on a device looks up the array's device address with that
 *    device current; make that first call before any stream capture. A
 *    successful lookup is kept for the life of the process (so a
 *    cudaDeviceReset, or a non-primary driver context made current, is not
 *    supported afterwards); a failed one returns B2_ELAUNCH and is retried by
 *    the next call.
 *  - `stream` must belong to the current device (B2_EINVAL otherwise).
 *  - All calls share the one array: calls whose kernels overlap on the GPU
 *    (different streams, or different host threads, same device) race.
 *    Every scratch slot a call reads is written by the same call first, so
 *    nothing needs clearing between calls.
 * out: int64 indices for argmax/argmin, else x's dtype. cols must be > 0.
 */
int b2_row_reduce_noalloc(int op, const void* x, void* out, int64_t rows, int64_t cols,
                          int64_t ld_x, int dtype, void* stream);

/*
 * Reduction over the middle axis of a contiguous x[outer, R, inner]:
 * out[o, i] = reduce over r of x[o, r, i] (torch's sum / amax / amin / argmax /
 * argmin along a dimension that is not the last one: x viewed as
 * [prod(dims before), size(dim), prod(dims after)]). Replaces the reference's
 * generic tt.reduce lowering for non-last axes (triton_msl/codegen/_lowerer_reduce.py:773-1010,
 * fuzzed as 2d_sum_ax0 / 3d_sum_ax0 in tests/test_fuzz_reduce.py:88-139).
 * op: B2_ROW_SUM / MAX / MIN / ARGMAX / ARGMIN (NaN and tie rules as b2_row_op);
 * out: x's dtype, or int64 indices in [0, R) for argmax/argmin. workspace: size
 * from b2_query_workspace(3, outer, R, inner, 0) (splits R across CTAs when the
 * output is small); without it one pass runs.
 */
int b2_reduce_axis(int op, const void* x, void* out, int64_t outer, int64_t R, int64_t inner,
                   int dtype, void* workspace, size_t ws_bytes, void* stream);

/* Scratch bytes a call with these arguments needs (0 = none).
 * kind: 0 = b2_gemm (a0=M, a1=N, a2=K, a3=in_dtype),
 *       1 = b2_row_op (a0=op, a1=rows, a2=cols, a3=dtype),
 *       2 = b2_fa_fwd (always 0),
 *       3 = b2_reduce_axis (a0=outer, a1=R, a2=inner). */
size_t b2_query_workspace(int kind, int64_t a0, int64_t a1, int64_t a2, int64_t a3);

/* OR of the device status bits written by bounded waits on `device` since the
 * last clear (0 = no wait expired). Synchronises that device. clear != 0 resets it. */
int b2_device_status(int device, int clear, uint32_t* status_out);

/* Device status bits (b2_device_status). */
#define B2_STATUS_TIMEOUT_TMA 0x1u  /* a consumer gave up waiting for a TMA fill */
#define B2_STATUS_TIMEOUT_MMA 0x2u  /* a waiter gave up on a tensor-core commit */
#define B2_STATUS_TIMEOUT_EPI 0x4u  /* a waiter gave up on the epilogue / softmax warps */
#define B2_STATUS_TIMEOUT_SLOT 0x8u /* the TMA producer gave up waiting for a free stage */

/*
 * Failure-path test of the bounded device waits (no counterpart in the
 * reference; its fast-path failure contract is "return False and take the
 * generic path", triton_msl/autotuning/_fast_matmul_dispatch.py:152-158).
 * Launches the tensor-core GEMM on fp16 A[M,K] (row-major) and B given as
 * [N,K] (row-major), C fp16 [M,N], with its TMA producer told to load
 * nothing and every wait limited to wait_limit_ns (<= 1 s). The MMA warp's
 * wait for the first operand stage runs out, the CTA abort flag stops the
 * other roles, TMEM is freed and the kernel returns; C is left unwritten.
 * A later b2_device_status() then reports B2_ETIMEOUT with
 * B2_STATUS_TIMEOUT_TMA set. Returns the launch status (B2_OK when queued).
 */
int b2_test_stalled_gemm(const void* A, const void* Bm, void* C, int64_t M, int64_t N, int64_t K,
                         uint64_t wait_limit_ns, void* stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}  // extern "C"
#endif

#endif  /* B2MSL_H_ */
