/*
 * pmkl_b200.h -- C ABI of the B200 (sm_100a) causal-attention and
 * warp-softmax library (libpmkl_b200.so).
 *
 * This is the drop-in boundary for pmkl's hot path.  Every pointer argument
 * is a DEVICE pointer owned by the caller; the library never allocates device
 * memory on these entry points and never synchronises: work is enqueued on the
 * caller's CUDA stream (`stream`, a cudaStream_t; NULL = legacy default
 * stream) and the call returns once it is enqueued.
 *
 * Every entry point returns PMKL_OK (0) on success or a negative pmkl_status;
 * pmkl_status_string() names it.  Argument errors are detected on the host
 * before anything is launched, mirroring the reference's CHECK_FAIL
 * (pmkl/core/utils/exception.h:121-129) and TORCH_CHECK
 * (pmkl_pytorch_ext/fused_self_attention.cpp:140-141) checks.
 */
#ifndef PMKL_B200_H_
#define PMKL_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PMKL_B200_VERSION 100 /* 1.0.0 */

/* Element types.  The reference dispatches float, double, half and bfloat16
 * (fused_self_attention.cpp:152-156); double is rejected here. */
typedef enum pmkl_dtype {
    PMKL_DTYPE_F32 = 0,
    PMKL_DTYPE_F16 = 1,
    PMKL_DTYPE_BF16 = 2,
} pmkl_dtype;

typedef enum pmkl_status {
    PMKL_OK = 0,
    PMKL_ERR_INVALID_SHAPE = -1,   /* negative / inconsistent sizes, size limits */
    PMKL_ERR_INVALID_DTYPE = -2,   /* unknown or unsupported dtype combination */
    PMKL_ERR_NULL_POINTER = -3,    /* a required pointer is NULL for a non-empty problem */
    PMKL_ERR_MISALIGNED = -4,      /* a pointer breaks the alignment the chosen kernel needs */
    PMKL_ERR_UNSUPPORTED = -5,     /* valid arguments this build has no kernel for */
    PMKL_ERR_NO_DEVICE = -6,       /* no CUDA device, or not an sm_100 device */
    PMKL_ERR_LAUNCH = -7,          /* the CUDA runtime rejected the launch */
    PMKL_ERR_DEVICE_TIMEOUT = -8,  /* a kernel gave up on a bounded wait (see pmkl_device_error) */
    PMKL_ERR_WORKSPACE = -9,       /* workspace smaller than the call needs */
} pmkl_status;

/* Kernel selection for pmkl_causal_attention_fwd_ex. */
typedef enum pmkl_attention_kernel {
    PMKL_ATTN_AUTO = 0,    /* tcgen05 path when it applies, else the SIMT path */
    PMKL_ATTN_SIMT = 1,    /* generic CUDA-core kernel: any dtype, head size 1..256 */
    PMKL_ATTN_TCGEN05 = 2, /* tensor-core kernel: fp16/bf16, head size 64 or 128 */
    PMKL_ATTN_TCGEN05_SIMPLE = 3, /* one query tile per CTA, non-persistent (comparison only) */
} pmkl_attention_kernel;

/*
 * Fused (causal) self-attention forward.
 *
 * Replaces pmkl::nlp::causal_attention_forward<scalar_t, BLOCK_M, HIDDEN_SIZE>
 * (pmkl/nlp/causal_attention.h:258-288) and the compute behind
 * fused_self_attention_fw (pmkl_pytorch_ext/fused_self_attention.cpp:139-173).
 *
 *   q, k, v, o : [batch, heads, seq, hidden], contiguous, element type `dtype`
 *                for q/k/v and `out_dtype` for o.
 *   m, l       : [batch, heads, seq], element type `out_dtype`.
 *                m = row max of the scaled, masked scores  s = scale * q.k
 *                l = sum over keys of exp(s - m)
 *                o = softmax(s) v
 *                (semantics of fused_self_attention.cpp:38-61 and
 *                 causal_attention.h:200-255).
 *   is_causal  : key j is visible to query i only when j <= i.
 *   scale      : score scale; pass 0 (or any value <= 0) for 1/sqrt(hidden),
 *                the value the reference hard-codes (causal_attention.h:192).
 *   dtype      : PMKL_DTYPE_F32, _F16 or _BF16.
 *   out_dtype  : dtype (the reference's behaviour: outputs in v's dtype,
 *                fused_self_attention.cpp:148-150) or PMKL_DTYPE_F32.
 *
 * Any seq >= 0 is accepted (the reference kernel needs seq % 32 == 0,
 * causal_attention.h:267; its CPU path takes any seq).  An empty problem
 * returns PMKL_OK without launching (causal_attention.h:270).
 */
int pmkl_causal_attention_fwd(const void *q, const void *k, const void *v, void *o, void *m, void *l,
                              int batch, int heads, int seq, int hidden, int dtype, int out_dtype,
                              int is_causal, float scale, void *stream);

/* As pmkl_causal_attention_fwd, with an explicit kernel choice (tests and
 * benchmarks use it to run one path on purpose).  PMKL_ATTN_TCGEN05 returns
 * PMKL_ERR_UNSUPPORTED when that kernel does not cover the arguments. */
int pmkl_causal_attention_fwd_ex(const void *q, const void *k, const void *v, void *o, void *m, void *l,
                                 int batch, int heads, int seq, int hidden, int dtype, int out_dtype,
                                 int is_causal, float scale, int kernel, void *stream);

/*
 * As pmkl_causal_attention_fwd_ex for strided and grouped-query inputs, so that
 * callers with other layouts (e.g. [batch, seq, heads, hidden] views, or K/V
 * with fewer heads) need no copy; the reference makes its inputs contiguous
 * (fused_self_attention.cpp:160-162) and takes equal head counts only (:141).
 *
 *   q, o       : [batch, heads, seq, hidden] elements at
 *                b * s[0] + h * s[1] + row * s[2] + col (s = q_strides /
 *                o_strides, element strides; the hidden dimension is
 *                contiguous).
 *   k, v       : the same with kv_heads heads (k_strides / v_strides); query
 *                head h reads K/V head h / (heads / kv_heads).  kv_heads must
 *                divide heads (kv_heads == heads: ordinary attention; 1:
 *                multi-query).
 *   m, l       : contiguous [batch, heads, seq], as in the forward.
 *   a NULL strides pointer means that tensor is contiguous.
 * The tensor-core kernel runs when the pointers are 16-byte aligned and every
 * stride is a multiple of 16 bytes (fp32 o: of 4 elements); otherwise the
 * CUDA-core kernel.  Negative strides and a kv_heads that does not divide heads
 * give PMKL_ERR_INVALID_SHAPE.  PMKL_ATTN_TCGEN05_SIMPLE accepts contiguous,
 * equal-head inputs only.
 */
int pmkl_causal_attention_fwd_strided(const void *q, const void *k, const void *v, void *o, void *m, void *l,
                                      int batch, int heads, int kv_heads, int seq, int hidden,
                                      const int64_t *q_strides, const int64_t *k_strides, const int64_t *v_strides,
                                      const int64_t *o_strides, int dtype, int out_dtype, int is_causal, float scale,
                                      int kernel, void *stream);

/* The kernel pmkl_causal_attention_fwd_ex would run for these arguments:
 * PMKL_ATTN_TCGEN05 (the persistent two-tile tensor-core kernel),
 * PMKL_ATTN_TCGEN05_SIMPLE, PMKL_ATTN_SIMT, or a negative pmkl_status.  Needs
 * a current sm_100 device.  No reference counterpart (diagnostic). */
int pmkl_attention_selected_kernel(const void *q, const void *k, const void *v, const void *o, int hidden, int dtype,
                                   int out_dtype, int kernel);

/*
 * Fused (causal) self-attention backward.
 *
 * Replaces fused_self_attention_bw (pmkl_pytorch_ext/fused_self_attention.cpp:
 * 175-215), whose math is pmkl_cpu::host_self_attention_backward (:66-135);
 * the reference has no GPU backward.  Gradients of o with respect to q, k, v
 * given dout = dL/do and the forward's row statistics m, l as the caller
 * passes them (used as given: p = exp(scale q.k - m) / l, as :91 does):
 *   dv = P^T dout,  dS = P * (dout v^T - delta),  delta_i = sum_j P_ij (dout_i . v_j),
 *   dq = scale dS k,  dk = scale dS^T q.
 *
 *   dout, q, k, v, dq, dk, dv : [batch, heads, seq, hidden], contiguous, `dtype`.
 *   m, l                      : [batch, heads, seq], `dtype` (the forward's
 *                               outputs, which the reference returns in v's dtype).
 *   scale                     : as in the forward (<= 0: 1/sqrt(hidden), the
 *                               reference's fixed value, :90).
 *   workspace                 : device scratch of at least
 *                               pmkl_causal_attention_bwd_workspace_size(...)
 *                               bytes, 256-byte aligned; its contents on entry
 *                               do not matter.  Not used after the call's work
 *                               completes on `stream`.
 *
 * dq, dk, dv are written, not accumulated (the reference zero-fills them first,
 * :186-188, so the results agree).  Accumulation is fp32; 16-bit outputs are
 * rounded once.  fp16/bf16 with hidden 64 or 128 and 16-byte aligned pointers
 * run on the tensor cores; everything else on the CUDA-core path.
 */
int pmkl_causal_attention_bwd(const void *dout, const void *q, const void *k, const void *v, const void *m,
                              const void *l, void *dq, void *dk, void *dv, int batch, int heads, int seq,
                              int hidden, int dtype, int is_causal, float scale, void *workspace,
                              size_t workspace_bytes, void *stream);

/* As pmkl_causal_attention_bwd with an explicit kernel choice: PMKL_ATTN_AUTO,
 * PMKL_ATTN_SIMT, PMKL_ATTN_TCGEN05 (PMKL_ERR_UNSUPPORTED when the tensor-core
 * path does not cover the arguments), or PMKL_ATTN_TCGEN05_SIMPLE: the
 * tensor-core gradient kernels with the per-row term delta taken the long way
 * (a forward writing fp32 O, m, l, then a row-statistics kernel) instead of
 * from the persistent forward's epilogue (comparison only). */
int pmkl_causal_attention_bwd_ex(const void *dout, const void *q, const void *k, const void *v, const void *m,
                                 const void *l, void *dq, void *dk, void *dv, int batch, int heads, int seq,
                                 int hidden, int dtype, int is_causal, float scale, void *workspace,
                                 size_t workspace_bytes, int kernel, void *stream);

/*
 * As pmkl_causal_attention_bwd_ex for strided and grouped-query tensors, the
 * backward of pmkl_causal_attention_fwd_strided: views (e.g. [batch, seq,
 * heads, hidden] tensors seen as [batch, heads, seq, hidden]) are read and the
 * gradients written in place, with no copies; the reference makes its inputs
 * contiguous (fused_self_attention.cpp:160-162, :179) and takes equal head
 * counts only (:178-180).
 *
 *   dout, q, dq : [batch, heads, seq, hidden] at b * s[0] + h * s[1] + row * s[2]
 *                 + col (element strides dout_strides, q_strides, dq_strides;
 *                 the hidden dimension contiguous).
 *   k, v, dk, dv: the same with kv_heads heads; query head h reads K/V head
 *                 h / (heads / kv_heads), and dk, dv are the sums over those
 *                 query heads (formed in fp32, rounded once).
 *   m, l        : contiguous [batch, heads, seq].
 *   a NULL strides pointer means that tensor is contiguous.
 * Workspace as for pmkl_causal_attention_bwd with the query heads
 * (pmkl_causal_attention_bwd_workspace_size(batch, heads, ...)).  The
 * tensor-core path runs when the pointers are 16-byte aligned and every stride
 * is a multiple of 16 bytes; otherwise the CUDA-core path.  kv_heads that does
 * not divide heads or negative strides give PMKL_ERR_INVALID_SHAPE;
 * PMKL_ATTN_TCGEN05_SIMPLE accepts contiguous, equal-head tensors only.
 */
int pmkl_causal_attention_bwd_strided(const void *dout, const void *q, const void *k, const void *v, const void *m,
                                      const void *l, void *dq, void *dk, void *dv, int batch, int heads, int kv_heads,
                                      int seq, int hidden, const int64_t *dout_strides, const int64_t *q_strides,
                                      const int64_t *k_strides, const int64_t *v_strides, const int64_t *dq_strides,
                                      const int64_t *dk_strides, const int64_t *dv_strides, int dtype, int is_causal,
                                      float scale, void *workspace, size_t workspace_bytes, int kernel, void *stream);

/* Workspace bytes pmkl_causal_attention_bwd needs for these sizes (0 for an
 * empty problem): on the tensor-core path the per-row statistics, 8 bytes per
 * row at a row pitch of seq rounded up to 128; on the CUDA-core path 4 bytes
 * per row.  No reference counterpart: the reference's CPU backward needs no
 * scratch. */
size_t pmkl_causal_attention_bwd_workspace_size(int batch, int heads, int seq, int hidden, int dtype);

/* The same for pmkl_causal_attention_bwd_ex with a given kernel choice:
 * PMKL_ATTN_TCGEN05_SIMPLE's long route also holds the forward's fp32 O, m, l
 * (4 (hidden + 2) bytes more per row); 0 for an unknown choice.  No reference
 * counterpart. */
size_t pmkl_causal_attention_bwd_workspace_size_ex(int batch, int heads, int seq, int hidden, int dtype, int kernel);

/* Size of the library's static device scratch used by
 * pmkl_causal_attention_bwd_static (64 MiB).  The array is a global of the
 * library's device code, so every device on which the library's module is
 * loaded holds it until the process exits, whichever entry points the caller
 * uses. */
#define PMKL_BWD_STATIC_SCRATCH_BYTES ((size_t)64 << 20)

/*
 * pmkl_causal_attention_bwd without a caller workspace and without any device
 * allocation: the scratch is a statically allocated __device__ array of
 * PMKL_BWD_STATIC_SCRATCH_BYTES (256-byte aligned) inside libpmkl_b200.  The
 * first call on a device looks up the array's device address
 * (cudaGetSymbolAddress, with that device current) and keeps it; a failed
 * lookup returns PMKL_ERR_LAUNCH and is tried again on the next call.  Make
 * that first call on each device before any stream capture.  No cudaMalloc,
 * cudaFree or allocator call happens on this path.  Same arguments (minus the workspace), results
 * and status codes as pmkl_causal_attention_bwd; a problem whose
 * pmkl_causal_attention_bwd_workspace_size() exceeds the scratch (more than
 * 8 Mi rows of batch x heads x seq rounded up to 128 on the tensor-core path,
 * e.g. 512 (batch, head) slices of 16384 rows) is rejected with
 * PMKL_ERR_WORKSPACE before anything is launched.  Nothing in the scratch
 * has to start at zero: every byte a kernel reads is written earlier in the
 * same call.
 *
 * The scratch is shared by every call on a device: two calls whose work
 * overlaps in time (different streams, or different host threads without
 * ordering between their streams) race on it and give undefined results.
 * Issue such calls on one stream, or order them.
 *
 * No reference counterpart: an addition of this library (the reference's
 * backward is a host loop that needs no scratch).
 */
int pmkl_causal_attention_bwd_static(const void *dout, const void *q, const void *k, const void *v, const void *m,
                                     const void *l, void *dq, void *dk, void *dv, int batch, int heads, int seq,
                                     int hidden, int dtype, int is_causal, float scale, void *stream);

/*
 * Row-wise softmax / log-softmax.
 *
 * Replaces pmkl::norm::warp_softmax_forward<output_t, input_t, acc_t,
 * is_log_softmax> (pmkl/norm/warp_softmax.h:159-201).  Same argument meaning:
 * `rows` rows of `elements` values, consecutive rows `stride` elements apart;
 * dst uses the same row stride.  Accumulation is fp32 (acc_t = float).
 * 0 <= elements <= 1024 as in the reference (warp_softmax.h:162); elements == 0
 * returns without launching.  Rows whose exp-sum is zero produce NaN
 * (warp_softmax.h:147-148).
 */
int pmkl_warp_softmax_fwd(void *dst, const void *src, int elements, int stride, int rows, int in_dtype,
                          int out_dtype, int is_log, void *stream);

/* Human-readable name of a pmkl_status value (static storage). */
const char *pmkl_status_string(int status);

/* PMKL_B200_VERSION of the loaded library. */
int pmkl_version(void);

/* Waits for `stream` (NULL = legacy default stream).  The C++ shim calls it
 * after each launch to keep the reference launcher's synchronous behaviour
 * (pmkl/core/launcher/cuda_launcher.h:334, stream_sync).  Returns PMKL_OK,
 * or PMKL_ERR_LAUNCH when the stream reports an error. */
int pmkl_stream_synchronize(void *stream);

/*
 * Device-side error word of the current device: bit 0 set when a kernel gave
 * up on a bounded wait and returned early (its outputs are then undefined).
 * This call synchronises the device.  Returns PMKL_OK when the word is zero,
 * PMKL_ERR_DEVICE_TIMEOUT when it is set (and clears it when `clear` != 0),
 * or PMKL_ERR_LAUNCH when the runtime reports an error.  No reference
 * counterpart: the reference's launcher only checks launch errors
 * (pmkl/core/launcher/cuda_launcher.h:297-335).
 */
int pmkl_device_error(int clear);

/*
 * Bounded-wait self-test: launches `ctas` CTAs of a diagnostic kernel whose
 * one waiting thread per CTA waits on an mbarrier that nothing ever arrives
 * on, with a limit of `limit_ns` (100 us .. 2 s, the limit every kernel of
 * this library uses).  It goes through the same steps as an attention kernel
 * that gives up: the wait runs out, the CTA's abort flag is raised, issued
 * tensor-core work is drained, tensor memory is freed and the device error
 * word is set (read with pmkl_device_error).  A CTA that finds the word
 * already set skips its work, as every tensor-core kernel does.  `out`
 * (device memory, 2 * ctas values, 8-byte aligned) receives per CTA the
 * outcome (0 completed, 1 ran out, 2 skipped) and the nanoseconds waited.
 * Nothing faults, traps or hangs.  Diagnostic only; no reference counterpart
 * (the reference checks errors on the host only,
 * pmkl/core/utils/exception.h:121-129).
 */
int pmkl_wait_selftest(int ctas, unsigned long long limit_ns, unsigned long long *out, void *stream);

/*
 * Tensor-core self-test: runs the tile primitives of the tcgen05 kernel in
 * isolation on one CTA and writes fp32 results for comparison with a host
 * matrix product.  Diagnostic only; no reference counterpart.
 *   which == 0:  c[128 x 128] = a[128 x hidden] * b[128 x hidden]^T
 *                (both operands K-major, the Q.K^T form)
 *   which == 1:  c[128 x hidden] = a[128 x 128] * b[128 x hidden]
 *                (a staged through tensor memory, b MN-major: the P.V form)
 * a, b: fp16/bf16 (`dtype`), row-major, contiguous; hidden is 64 or 128.
 */
int pmkl_tc_selftest(int which, const void *a, const void *b, float *c, int hidden, int dtype, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* PMKL_B200_H_ */
