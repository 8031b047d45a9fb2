/*
 * mamba3_b200.h -- C ABI of the B200 (sm_100a) Mamba-3 single-token decode.
 *
 * One entry point per GPU routine of the reference's kernel package
 * (michaelYZh/mamba3-fused-triton-kernel, src/kernels/*.py).  The reference
 * binds those routines from Python; the Python package in this repository
 * binds these symbols through ctypes with the same argument meaning.
 *
 * Conventions shared by every entry point:
 *   - All pointers are device pointers on the CURRENT device, owned by the
 *     caller.  Nothing here allocates or frees memory, synchronises the host
 *     or starts threads.  Work is enqueued on `stream` (0 = legacy default).
 *   - Strides and sizes are in ELEMENTS, not bytes.
 *   - The carried state (ssm_state / h, bx_prev, angle_state) is updated IN
 *     PLACE and must be contiguous with a 16-byte aligned base.  A strided
 *     state is rejected (M3_ERR_ALIGN) rather than copied, because a copy
 *     would break the in-place contract.
 *   - Arguments are validated on the host before any launch; an invalid call
 *     returns a non-zero status and enqueues nothing.  Device code never traps.
 *   - Calls of the entry points other than m3_mimo_step_static are safe to
 *     capture in a CUDA graph after one eager call on the device (the first
 *     call sets kernel attributes).  This header states nothing about
 *     capturing m3_mimo_step_static.
 */
#ifndef MAMBA3_B200_H
#define MAMBA3_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t / CUstream. */
typedef struct CUstream_st *m3_stream_t;

/* Status codes. */
enum {
  M3_OK = 0,
  M3_ERR_NULL = 1,   /* a required pointer is NULL                         */
  M3_ERR_SHAPE = 2,  /* inconsistent or unsupported sizes                  */
  M3_ERR_RANK = 3,   /* unsupported mimo_rank (supported: 1, 2, 4, 8)      */
  M3_ERR_DTYPE = 4,  /* unsupported dtype code                             */
  M3_ERR_ALIGN = 5,  /* state not contiguous / not 16-byte aligned         */
  M3_ERR_LAUNCH = 6, /* the CUDA launch itself failed                      */
  M3_ERR_DEVICE = 7, /* no usable CUDA device                              */
  M3_ERR_UNSUPPORTED = 8, /* valid layer the single-launch step does not take */
  M3_ERR_SCRATCH = 9      /* needs more than the library's static scratch     */
};

/* Element type codes. */
enum { M3_F32 = 0, M3_BF16 = 1 };

/* Geometry of one Mamba-3 layer (src/models/mamba3.py:87-114).
 * d_inner must equal nheads * headdim; ngroups must be 1 (the reference
 * decode path expands one B/C group over all heads, mamba3.py:209-210).
 * d_state must be a multiple of 4 and at most 256; num_rope_angles <=
 * d_state / 2 (the first 2*num_rope_angles state entries are rotated). */
typedef struct m3_dims {
  int32_t batch;           /* B                                  */
  int32_t nheads;          /* H                                  */
  int32_t headdim;         /* P                                  */
  int32_t d_state;         /* D                                  */
  int32_t mimo_rank;       /* R (1 for SISO)                     */
  int32_t num_rope_angles; /* A (full-fused entry points only)   */
  int32_t ngroups;         /* G, must be 1                       */
  int32_t d_inner;         /* H * P                              */
  float A_floor;           /* full-fused entry points only       */
} m3_dims;

/* Arguments of the state-update-only entry points (precomputed B/C/dt).
 * Shapes follow the reference kernels:
 *   x, z, y        (B, H, P)        any strides; x/z/y may be bf16
 *   B_proj, C_proj SISO (B, H, D), MIMO (B, R, H, D)   any strides, f32
 *   ADT, DT, trap  (B, H)           any strides, f32
 *   D_skip         (H,)             any stride,  f32
 *   mimo_x, mimo_o (H, R, P)        any strides, f32 (MIMO only)
 *   h, bx_prev     SISO (B, H, P, D), MIMO (B, H, D)  contiguous f32, in place
 * z == NULL selects the un-gated routines; the *_fused entry points require
 * z and multiply y by silu(z). */
typedef struct m3_ssm_args {
  const void *x;  int64_t x_sb, x_sh, x_sp;  int32_t x_dtype;
  const void *z;  int64_t z_sb, z_sh, z_sp;  int32_t z_dtype;
  void *y;        int64_t y_sb, y_sh, y_sp;  int32_t y_dtype;
  const float *B_proj; int64_t B_sb, B_sr, B_sh, B_sd;
  const float *C_proj; int64_t C_sb, C_sr, C_sh, C_sd;
  const float *ADT;    int64_t adt_sb, adt_sh;
  const float *DT;     int64_t dt_sb, dt_sh;
  const float *trap;   int64_t trap_sb, trap_sh;
  const float *D_skip; int64_t D_sh;
  const float *mimo_x; int64_t mx_sh, mx_sr, mx_sp;
  const float *mimo_o; int64_t mo_sh, mo_sr, mo_sp;
  float *h;
  float *bx_prev;
} m3_ssm_args;

/* Arguments of the full-step fused entry points.
 *   zx           (B, d_in_proj) row stride zx_stride_b, unit column stride;
 *                the raw in_proj output [z | x | B | C | dd_dt | dd_A |
 *                trap | angle] (mamba3.py:165-179); f32 or bf16
 *   dt_bias, D   (H,)          param_dtype
 *   B_norm_w, C_norm_w (D,)    param_dtype
 *   B_bias, C_bias (H, R, D)   param_dtype, contiguous
 *   mimo_x, mimo_o (H, R, P)   param_dtype, contiguous (MIMO only)
 *   ssm_state    SISO (B, H, P, D), MIMO (B, H, D)   contiguous f32, in place
 *   bx_prev      same shape as ssm_state                 contiguous f32, in place
 *   angle_state  (B, H, A)                               contiguous f32, in place
 *   y            (B, H*P) row stride y_stride_b; silu(z)-gated output;
 *                f32 or bf16 (bf16 rounds to nearest even, like .to(bf16)) */
typedef struct m3_full_args {
  const void *zx;  int64_t zx_stride_b; int32_t zx_dtype;
  int32_t param_dtype;
  const void *dt_bias, *D, *B_norm_w, *C_norm_w, *B_bias, *C_bias, *mimo_x, *mimo_o;
  float *ssm_state;
  float *bx_prev;
  float *angle_state;
  void *y; int64_t y_stride_b; int32_t y_dtype;
} m3_full_args;

/* Replaces mamba3_siso_decode_triton (src/kernels/siso_decode.py:136-187). */
int m3_siso_decode(const m3_dims *dims, const m3_ssm_args *args, m3_stream_t stream);

/* Replaces mamba3_mimo_decode_triton (src/kernels/mimo_decode.py:394-457);
 * mimo_rank in {1, 2, 4, 8}, else M3_ERR_RANK (the reference raises
 * ValueError, mimo_decode.py:426-430). */
int m3_mimo_decode(const m3_dims *dims, const m3_ssm_args *args, m3_stream_t stream);

/* Replaces mamba3_siso_decode_fused_triton (src/kernels/siso_decode_fused.py:143-193). */
int m3_siso_decode_fused(const m3_dims *dims, const m3_ssm_args *args, m3_stream_t stream);

/* Replaces mamba3_mimo_decode_fused_triton (src/kernels/mimo_decode_fused.py:114-170);
 * lifts the reference's R == 4 restriction (mimo_decode_fused.py:144). */
int m3_mimo_decode_fused(const m3_dims *dims, const m3_ssm_args *args, m3_stream_t stream);

/* Replaces mamba3_siso_full_fused_triton (src/kernels/fused_full_decode.py:228-289). */
int m3_siso_full_fused(const m3_dims *dims, const m3_full_args *args, m3_stream_t stream);

/* Replaces mamba3_mimo_full_fused_triton (src/kernels/fused_full_decode.py:569-636);
 * lifts the reference's R == 4 restriction (fused_full_decode.py:600). */
int m3_mimo_full_fused(const m3_dims *dims, const m3_full_args *args, m3_stream_t stream);

/* Prefill of MIMO layers: dims->batch sequences of seq_len tokens each, the
 * full step of m3_mimo_full_fused applied token after token with the carried
 * state kept on chip (replaces the sequential loop of Mamba3.forward,
 * src/models/mamba3.py:242-304).  zx rows (in_proj outputs) and y rows are
 * b * seq_len + t at zx_stride_b / y_stride_b; the state arrays hold
 * dims->batch rows, read once and written once.  M3_ERR_UNSUPPORTED for
 * shapes the streamed kernel does not take (then step token by token). */
int m3_mimo_prefill(const m3_dims *dims, const m3_full_args *args, int32_t seq_len, m3_stream_t stream);

/* Prefill of SISO layers: the full step of m3_siso_full_fused applied token
 * after token to dims->batch sequences of seq_len tokens, with each head's
 * (headdim, d_state) state tile kept on chip from the first token to the
 * last (replaces the sequential loop of Mamba3.forward,
 * src/models/mamba3.py:242-304, for is_mimo=False).  Row layout as
 * m3_mimo_prefill; M3_ERR_UNSUPPORTED for shapes the kernel does not take. */
int m3_siso_prefill(const m3_dims *dims, const m3_full_args *args, int32_t seq_len, m3_stream_t stream);

/* Small-batch fp32 linear layer of the decode step's projections (in_proj /
 * out_proj, nn.Linear without bias, src/models/mamba3.py:115,158, called at
 * src/models/inference.py:489,553):  C[m, n] = sum_k A[m, k] * W[n, k].
 * A: (M, K) row stride lda, W: (N, K) row stride ldw, C: (M, N) row stride
 * ldc; fp32, 16-byte aligned bases, K, lda, ldw multiples of 4.  Tuned for
 * M (the batch) up to a few hundred; fp32 accumulation. */
int m3_linear_f32(const float *A, int64_t lda, const float *W, int64_t ldw, float *C, int64_t ldc,
                  int32_t M, int32_t N, int32_t K, m3_stream_t stream);

/* bf16 linear layer of the decode step's projections on the tensor cores
 * (tcgen05, fp32 accumulation); same operation and call sites as
 * m3_linear_f32:  C[m, n] = sum_k A[m, k] * W[n, k].  A: (M, K) bf16 row
 * stride lda, W: (N, K) bf16 row stride ldw, C: (M, N) row stride ldc in
 * c_dtype (M3_BF16, rounded to nearest, or M3_F32).  16-byte aligned bases,
 * K >= 64, K, lda, ldw multiples of 8.  Pairs of SMs (tcgen05.mma
 * .cta_group::2) share each batch tile.  When the call splits K, the pairs
 * add their partial tiles into an fp32 accumulator in `workspace` (16-byte
 * aligned, at least m3_linear_bf16_workspace_bytes(M, N, K) bytes,
 * M3_ERR_SHAPE otherwise; NULL / 0 when that is 0), which must be ZEROED
 * before its first use and is left at zero by every call (zero it again
 * after a call that reported M3_DEVERR_TIMEOUT); calls sharing a workspace
 * must not overlap on the GPU.  M3_ERR_UNSUPPORTED when the driver offers
 * no tensor-map encoder. */
int m3_linear_bf16(const void *A, int64_t lda, const void *W, int64_t ldw, void *C, int64_t ldc, int32_t M,
                   int32_t N, int32_t K, int32_t c_dtype, void *workspace, int64_t workspace_bytes,
                   m3_stream_t stream);

/* Workspace bytes m3_linear_bf16 needs for this shape on the current device
 * (0 when it does not split K); negative for an invalid shape. */
int64_t m3_linear_bf16_workspace_bytes(int32_t M, int32_t N, int32_t K);

/* fp32 linear layer of the decode step's projections for batches beyond the
 * small-batch kernel's (same operation and call sites as m3_linear_f32,
 * src/models/mamba3.py:115,158 called at src/models/inference.py:489,553),
 * on the tensor cores in split precision: each fp32 operand is given as a
 * TF32 head and its remainder (m3_split_tf32), and every k step issues the
 * three tcgen05.mma (kind::tf32) products hi.hi + hi.lo + lo.hi, which
 * carry about as many significant bits as fp32 (the dropped lo.lo term is
 * ~2^-22 relative); accumulation in fp32.
 *   C[m, n] = sum_k (A_hi + A_lo)[m, k] * (W_hi + W_lo)[n, k]
 * A_hi / A_lo: (M, K) row stride lda; W_hi / W_lo: (N, K) row stride ldw;
 * C: (M, N) fp32 row stride ldc.  16-byte aligned bases, K >= 32, K, lda and
 * ldw multiples of 4.  No workspace.  M3_ERR_UNSUPPORTED when the driver
 * offers no tensor-map encoder. */
int m3_linear_f32_tc(const float *A_hi, const float *A_lo, int64_t lda, const float *W_hi, const float *W_lo,
                     int64_t ldw, float *C, int64_t ldc, int32_t M, int32_t N, int32_t K, m3_stream_t stream);

/* bf16 linear layer of the decode step's projections for small decode
 * batches (M <= 64 rows: a GPU's share of a strongly scaled batch, or a
 * single-stream decode), same operation and call sites as m3_linear_bf16.
 * At these sizes the call is a stream of the weight, which this kernel reads
 * once from HBM through the tensor cores (mma.sync bf16, fp32 accumulation;
 * K split across the warps of a CTA and summed in a fixed order, so results
 * are deterministic).  A: (M, K) bf16 row stride lda, W: (N, K) bf16 row
 * stride ldw, C: (M, N) row stride ldc in c_dtype (M3_BF16 rounded to
 * nearest, or M3_F32).  A and W 16-byte aligned; K, lda, ldw multiples of 8;
 * C 4-byte aligned.  M3_ERR_SHAPE for M > 64.  No workspace. */
int m3_linear_bf16_skinny(const void *A, int64_t lda, const void *W, int64_t ldw, void *C, int64_t ldc, int32_t M,
                          int32_t N, int32_t K, int32_t c_dtype, m3_stream_t stream);

/* The operand split m3_linear_f32_tc takes: hi = x with the 13 low mantissa
 * bits cleared (exactly a TF32 value), lo = x - hi (exact in fp32).
 * x: (rows, cols) row stride ldx; hi, lo: row stride ld; 16-byte aligned,
 * cols, ldx, ld multiples of 4.  No reference counterpart (the reference's
 * projections are plain fp32 nn.Linear calls). */
int m3_split_tf32(const float *x, int64_t ldx, float *hi, float *lo, int64_t ld, int32_t rows, int32_t cols,
                  m3_stream_t stream);

/* Arguments of the single-launch decode step (m3_mimo_step).
 *   dtype        M3_F32 or M3_BF16: u, both projection weights, the per-head
 *                parameters (as in m3_full_args), out and the workspace's
 *                intermediates; accumulation is fp32
 *   u            (B, d_model) row stride u_stride_b
 *   in_proj_w    (d_in_proj, d_model) row stride in_proj_stride
 *   out_proj_w   (d_model, d_inner) row stride out_proj_stride
 *   ssm_state, bx_prev, angle_state   as in m3_full_args, in place
 *   out          (B, d_model) row stride out_stride_b; device memory or pinned
 *                host memory (the kernel's stores then go straight to the host)
 *   workspace    device scratch of at least m3_mimo_step_workspace_bytes,
 *                256-byte aligned, ZEROED ONCE before its first use and then
 *                left to the library (it holds the in_proj output, the gated
 *                output and two grid-barrier words, a base and an arrival
 *                counter, that are never reset: each launch advances the
 *                base past its own arrivals).  After a launch on it reports
 *                M3_DEVERR_TIMEOUT the words no longer agree, every later
 *                launch on it times out as well, and the workspace must be
 *                zeroed again before its next use.  One workspace per
 *                concurrently running launch.
 * d_model, row strides and the weights' row strides multiples of 4; u and
 * the weights 16-byte (f32) / 8-byte (bf16) aligned. */
typedef struct m3_step_args {
  int32_t d_model;
  int32_t dtype;
  const void *u;           int64_t u_stride_b;
  const void *in_proj_w;   int64_t in_proj_stride;
  const void *out_proj_w;  int64_t out_proj_stride;
  const void *dt_bias, *D, *B_norm_w, *C_norm_w, *B_bias, *C_bias, *mimo_x, *mimo_o;
  float *ssm_state;
  float *bx_prev;
  float *angle_state;
  void *out;               int64_t out_stride_b;
  void *workspace;         int64_t workspace_bytes;
} m3_step_args;

/* Workspace bytes m3_mimo_step needs for this layer and batch, or the
 * negated status (-M3_ERR_*) when the call would be rejected;
 * -M3_ERR_UNSUPPORTED for a valid layer outside the single-launch kernel's
 * range (nheads not a multiple of 8, headdim > 128, d_state > 128, d_model
 * or d_inner not a multiple of 4), which the three-launch path serves. */
int64_t m3_mimo_step_workspace_bytes(const m3_dims *dims, int32_t d_model, int32_t dtype);

/* The whole decode step of one MIMO layer in ONE launch: in_proj, the
 * full-step fused update and out_proj (the sequence of
 * Mamba3Decoder._step_triton_full_fused, src/models/inference.py:476-559,
 * whose projections are nn.Linear without bias, src/models/mamba3.py:
 * 115,158).  A cooperative launch (all CTAs resident) with two grid-wide
 * barriers; no counterpart kernel in the reference, whose step is three
 * launches. */
int m3_mimo_step(const m3_dims *dims, const m3_step_args *args, m3_stream_t stream);

/* Workspace bytes m3_siso_step needs for this layer and batch (dims with
 * mimo_rank 1), or the negated status; -M3_ERR_UNSUPPORTED for a valid
 * layer outside the kernel's range (headdim > 1024, d_model or d_inner not a
 * multiple of 4). */
int64_t m3_siso_step_workspace_bytes(const m3_dims *dims, int32_t d_model, int32_t dtype);

/* The whole decode step of one SISO layer (is_mimo=False) in ONE launch:
 * in_proj, the full-step fused SISO update (m3_siso_full_fused) and
 * out_proj, the sequence of Mamba3Decoder._step_triton_full_fused
 * (src/models/inference.py:476-559) for SISO layers.  Same arguments,
 * workspace rules and grid barriers as m3_mimo_step; the state is the SISO
 * layout (batch, nheads, headdim, d_state), B_bias / C_bias are (nheads,
 * d_state), and mimo_x / mimo_o are not read (may be NULL).  Each (batch
 * row, head) state tile is updated by one CTA.  For callers that want one
 * launch per step (eager decoding, where each launch costs host time);
 * replayed from a CUDA graph the three launches measured faster on B200
 * (18.9 against 24.6 us a step for the d256 layer at batch 1), so the
 * Python decoder keeps them for SISO layers. */
int m3_siso_step(const m3_dims *dims, const m3_step_args *args, m3_stream_t stream);

/* Bytes of the library's own device scratch array behind m3_mimo_step_static
 * (held on every GPU that loads the library until the process exits). */
#define M3_STEP_STATIC_SCRATCH_BYTES (4 * 1024 * 1024)

/* m3_mimo_step for callers that cannot allocate device memory: a plugin
 * handed device buffers by a host framework without access to its
 * allocator, a serving thread that must not call cudaMalloc (it can
 * synchronise the device and take milliseconds), a process whose device
 * footprint is fixed after start-up.  Same arguments and results as
 * m3_mimo_step, except that args->workspace must be NULL and
 * args->workspace_bytes 0: the workspace is a device array inside the
 * library, M3_STEP_STATIC_SCRATCH_BYTES long.  A layer and batch needing
 * more (m3_mimo_step_workspace_bytes) return M3_ERR_SCRATCH; like every call
 * that m3_mimo_step would reject, it enqueues nothing and leaves the array
 * as it was.  Allocates nothing.  The first call on a device looks up the
 * array's device address (once, with that device current); make that first
 * call before any stream capture.  Each call clears the array's barrier
 * words on `stream` before its launch; every call on a device shares the
 * array, so calls that overlap on the GPU race and must be serialised by
 * the caller.  No counterpart in the reference. */
int m3_mimo_step_static(const m3_dims *dims, const m3_step_args *args, m3_stream_t stream);

/* Residual add + RMSNorm between the blocks of a stack (x <- x +
 * mixer(RMSNorm(x)), src/models/mamba3.py:412-421 with RMSNorm :26-36):
 *   x_out = x + o            (o may be NULL: x_out = x; x_out may be NULL)
 *   xn    = x_out / sqrt(mean(x_out^2) + eps) * w   (xn may be NULL)
 * x, o, x_out, xn: (M, N) rows of `dtype` (f32 or bf16; the add rounds to
 * dtype like torch's add), w: (N,) f32.  N <= 8192.  One launch. */
int m3_residual_rmsnorm(int32_t dtype, const void *x, int64_t ldx, const void *o, int64_t ldo,
                        const float *w, void *x_out, int64_t ldxo, void *xn, int64_t ldn,
                        int32_t M, int32_t N, float eps, m3_stream_t stream);

/* Device-side error word of the library's kernels: 0, or a bit mask of
 * M3_DEVERR_* raised by a kernel that gave up a bounded wait (the kernel
 * then skipped its remaining work and returned).  The outputs and the state
 * a launch that raised it was updating are undefined (a prefill may have
 * stored the output rows of finished chunks while leaving the state as it
 * was), and m3_mimo_step's workspace must be zeroed again.  Synchronises
 * the device.
 * `reset` != 0 clears the word.  Returns -1 if it cannot be read.
 * Diagnostics only; no counterpart in the reference. */
enum { M3_DEVERR_TIMEOUT = 1 };
int m3_device_error(int reset);

/* Self test of the bounded waits: launches one CTA that waits on a barrier
 * nothing completes, with a short bound, and returns.  Afterwards
 * m3_device_error reports M3_DEVERR_TIMEOUT.  Diagnostics only; no
 * counterpart in the reference. */
int m3_selftest_wait_timeout(m3_stream_t stream);

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int m3_version(void);

/* Static, NUL-terminated description of a status code. */
const char *m3_status_string(int status);

#ifdef __cplusplus
}
#endif

#endif /* MAMBA3_B200_H */
