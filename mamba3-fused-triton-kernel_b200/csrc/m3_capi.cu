// extern "C" entry points declared in include/mamba3_b200.h.
//
// Each entry point validates its arguments on the host, fills the kernel
// parameter block and enqueues exactly one kernel on the caller's stream.
// No allocation, no synchronisation, no device-side traps.
#include <cstdint>

#include "m3_kernels.cuh"
#include "m3_step.cuh"

namespace {

using m3::KParams;

constexpr int kVersion = 10400;  // 1.4.0
constexpr int kMaxHeaddim = 4096;

bool dtype_ok(int32_t dt) { return dt == M3_F32 || dt == M3_BF16; }
bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Sizes shared by every entry point.  batch == 0 is a valid empty call.
int check_dims(const m3_dims *d, bool mimo) {
  if (!d) return M3_ERR_NULL;
  if (d->batch < 0 || d->nheads <= 0 || d->headdim <= 0 || d->d_state <= 0) return M3_ERR_SHAPE;
  if (d->headdim > kMaxHeaddim) return M3_ERR_SHAPE;
  if (d->d_state % 4 != 0 || d->d_state > 256) return M3_ERR_SHAPE;
  if (mimo) {
    const int r = d->mimo_rank;
    if (r != 1 && r != 2 && r != 4 && r != 8) return M3_ERR_RANK;
  }
  return M3_OK;
}

int check_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) {
    cudaGetLastError();
    return M3_ERR_DEVICE;
  }
  return M3_OK;
}

int launch_status(cudaError_t e) { return e == cudaSuccess ? M3_OK : M3_ERR_LAUNCH; }

int ssm_entry(const m3_dims *d, const m3_ssm_args *a, m3_stream_t stream, bool mimo, bool gated) {
  int st = check_dims(d, mimo);
  if (st != M3_OK) return st;
  if (!a) return M3_ERR_NULL;
  if (!a->x || !a->y || !a->B_proj || !a->C_proj || !a->ADT || !a->DT || !a->trap || !a->D_skip ||
      !a->h || !a->bx_prev)
    return M3_ERR_NULL;
  if (mimo && (!a->mimo_x || !a->mimo_o)) return M3_ERR_NULL;
  if (gated && !a->z) return M3_ERR_NULL;
  if (!dtype_ok(a->x_dtype) || !dtype_ok(a->y_dtype) || (gated && !dtype_ok(a->z_dtype)))
    return M3_ERR_DTYPE;
  if (!aligned16(a->h) || !aligned16(a->bx_prev)) return M3_ERR_ALIGN;
  if (d->batch == 0) return M3_OK;
  st = check_device();
  if (st != M3_OK) return st;

  KParams kp = {};
  kp.B = d->batch; kp.H = d->nheads; kp.P = d->headdim; kp.D = d->d_state;
  kp.R = mimo ? d->mimo_rank : 1;
  kp.heads_per_cta = m3::mimo_heads_per_cta(kp.H);
  kp.x = a->x; kp.x_sb = a->x_sb; kp.x_sh = a->x_sh; kp.x_sp = a->x_sp; kp.x_dt = a->x_dtype;
  kp.z = gated ? a->z : nullptr;
  kp.z_sb = a->z_sb; kp.z_sh = a->z_sh; kp.z_sp = a->z_sp; kp.z_dt = a->z_dtype;
  kp.y = a->y; kp.y_sb = a->y_sb; kp.y_sh = a->y_sh; kp.y_sp = a->y_sp; kp.y_dt = a->y_dtype;
  kp.Bp = a->B_proj; kp.B_sb = a->B_sb; kp.B_sr = a->B_sr; kp.B_sh = a->B_sh; kp.B_sd = a->B_sd;
  kp.Cp = a->C_proj; kp.C_sb = a->C_sb; kp.C_sr = a->C_sr; kp.C_sh = a->C_sh; kp.C_sd = a->C_sd;
  kp.adt = a->ADT; kp.adt_sb = a->adt_sb; kp.adt_sh = a->adt_sh;
  kp.dt = a->DT; kp.dt_sb = a->dt_sb; kp.dt_sh = a->dt_sh;
  kp.trap = a->trap; kp.tr_sb = a->trap_sb; kp.tr_sh = a->trap_sh;
  kp.Dsk = a->D_skip; kp.D_sh = a->D_sh;
  kp.smx = a->mimo_x; kp.mx_sh = a->mx_sh; kp.mx_sr = a->mx_sr; kp.mx_sp = a->mx_sp;
  kp.smo = a->mimo_o; kp.mo_sh = a->mo_sh; kp.mo_sr = a->mo_sr; kp.mo_sp = a->mo_sp;
  kp.h = a->h; kp.bx = a->bx_prev;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return launch_status(mimo ? m3::launch_mimo(kp, false, s) : m3::launch_siso(kp, false, s));
}

// Validation and kernel parameters of a full-step call; M3_OK with *empty
// set when the batch is empty (nothing to launch).
int full_params(const m3_dims *d, const m3_full_args *a, bool mimo, m3::KParams *out, bool *empty) {
  *empty = false;
  int st = check_dims(d, mimo);
  if (st != M3_OK) return st;
  if (!a) return M3_ERR_NULL;
  if (d->ngroups != 1) return M3_ERR_SHAPE;
  if (d->d_inner != d->nheads * d->headdim) return M3_ERR_SHAPE;
  if (d->num_rope_angles <= 0 || 2 * d->num_rope_angles > d->d_state) return M3_ERR_SHAPE;
  const int R = mimo ? d->mimo_rank : 1;
  const int64_t d_in_proj = 2LL * d->d_inner + 2LL * d->d_state * R + 3LL * d->nheads + d->num_rope_angles;
  if (a->zx_stride_b < d_in_proj) return M3_ERR_SHAPE;
  if (a->y_stride_b < (int64_t)d->d_inner) return M3_ERR_SHAPE;
  if (!a->zx || !a->dt_bias || !a->D || !a->B_norm_w || !a->C_norm_w || !a->B_bias || !a->C_bias ||
      !a->ssm_state || !a->bx_prev || !a->angle_state || !a->y)
    return M3_ERR_NULL;
  if (mimo && (!a->mimo_x || !a->mimo_o)) return M3_ERR_NULL;
  if (!dtype_ok(a->zx_dtype) || !dtype_ok(a->param_dtype) || !dtype_ok(a->y_dtype)) return M3_ERR_DTYPE;
  if (!aligned16(a->ssm_state) || !aligned16(a->bx_prev)) return M3_ERR_ALIGN;
  if ((reinterpret_cast<uintptr_t>(a->angle_state) & 3u) != 0) return M3_ERR_ALIGN;
  if (d->batch == 0) {
    *empty = true;
    return M3_OK;
  }
  st = check_device();
  if (st != M3_OK) return st;

  KParams &kp = *out;
  kp = KParams{};
  kp.B = d->batch; kp.H = d->nheads; kp.P = d->headdim; kp.D = d->d_state; kp.R = R;
  kp.A = d->num_rope_angles; kp.A_floor = d->A_floor;
  kp.d_inner = d->d_inner; kp.d_bc = d->d_state * R;
  kp.heads_per_cta = m3::mimo_heads_per_cta(kp.H);
  kp.zx = a->zx; kp.zx_sb = a->zx_stride_b; kp.zx_dt = a->zx_dtype; kp.par_dt = a->param_dtype;
  kp.dt_bias = a->dt_bias; kp.Dp = a->D; kp.wB = a->B_norm_w; kp.wC = a->C_norm_w;
  kp.bB = a->B_bias; kp.bC = a->C_bias; kp.mx = a->mimo_x; kp.mo = a->mimo_o;
  kp.h = a->ssm_state; kp.bx = a->bx_prev; kp.ang = a->angle_state;
  kp.y = a->y; kp.y_sb = a->y_stride_b; kp.y_sh = d->headdim; kp.y_sp = 1; kp.y_dt = a->y_dtype;
  return M3_OK;
}

int full_entry(const m3_dims *d, const m3_full_args *a, m3_stream_t stream, bool mimo) {
  KParams kp;
  bool empty = false;
  const int st = full_params(d, a, mimo, &kp, &empty);
  if (st != M3_OK || empty) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return launch_status(mimo ? m3::launch_mimo(kp, true, s) : m3::launch_siso(kp, true, s));
}

bool aligned_to(const void *p, unsigned a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }
int64_t round_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

// Workspace layout of the single-launch step: barrier counters, the in_proj
// output (row stride rounded up to 4 elements), the gated output.
struct StepLayout {
  int64_t ldzx, zx_off, y_off, bytes;
};

StepLayout step_layout(const m3_dims *d, int64_t d_in_proj, int es) {
  StepLayout L;
  L.ldzx = round_up(d_in_proj, 4);
  L.zx_off = m3::kStepBarBytes;
  L.y_off = L.zx_off + round_up((int64_t)d->batch * L.ldzx * es, 256);
  L.bytes = L.y_off + round_up((int64_t)d->batch * d->d_inner * es, 256);
  return L;
}

// Shape checks of the single-launch step (MIMO or SISO layer);
// M3_ERR_UNSUPPORTED for a valid layer the kernel does not take.
int check_step_dims(const m3_dims *d, int32_t d_model, int32_t dtype, bool mimo) {
  int st = check_dims(d, mimo);
  if (st != M3_OK) return st;
  if (!dtype_ok(dtype)) return M3_ERR_DTYPE;
  if (d->ngroups != 1 || d->d_inner != d->nheads * d->headdim || d_model <= 0) return M3_ERR_SHAPE;
  if (d->num_rope_angles <= 0 || 2 * d->num_rope_angles > d->d_state) return M3_ERR_SHAPE;
  if (!mimo && d->mimo_rank != 1) return M3_ERR_SHAPE;
  if (d_model % 4 != 0 || d->d_inner % 4 != 0) return M3_ERR_UNSUPPORTED;
  if (mimo && (d->nheads % 8 != 0 || d->headdim > 128 || d->d_state > 128)) return M3_ERR_UNSUPPORTED;
  if (!mimo && d->headdim > 1024) return M3_ERR_UNSUPPORTED;
  return M3_OK;
}

// Append an L2 prefetch range (trimmed to 16-byte boundaries; at most
// kMaxPrefetchChunks 4 KB chunks in all, one per thread of the grid).
void add_prefetch(m3::StepParams &sp, const void *p, int64_t bytes) {
  constexpr int64_t kChunk = 4096, kMaxPrefetchChunks = 148 * 256;
  if (!p || bytes <= 0 || sp.n_prefetch >= m3::kStepMaxPrefetch) return;
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uintptr_t lo = (a + 15) & ~uintptr_t(15);
  const uintptr_t hi = (a + (uintptr_t)bytes) & ~uintptr_t(15);
  if (hi <= lo) return;
  const int first = sp.pf_first[sp.n_prefetch];
  int64_t len = (int64_t)(hi - lo);
  if (first + (len + kChunk - 1) / kChunk > kMaxPrefetchChunks) len = (kMaxPrefetchChunks - first) * kChunk;
  if (len <= 0) return;
  sp.pf_ptr[sp.n_prefetch] = reinterpret_cast<const void *>(lo);
  sp.pf_bytes[sp.n_prefetch] = len;
  sp.pf_first[sp.n_prefetch + 1] = first + (int)((len + kChunk - 1) / kChunk);
  ++sp.n_prefetch;
}

int64_t step_workspace_bytes(const m3_dims *d, int32_t d_model, int32_t dtype, bool mimo) {
  const int st = check_step_dims(d, d_model, dtype, mimo);
  if (st != M3_OK) return -(int64_t)st;
  const int64_t d_in_proj = 2LL * d->d_inner + 2LL * d->d_state * d->mimo_rank + 3LL * d->nheads + d->num_rope_angles;
  return step_layout(d, d_in_proj, dtype == M3_BF16 ? 2 : 4).bytes;
}

// Every check m3_mimo_step / m3_siso_step makes before it enqueues
// anything; *empty is set for a batch of zero rows (nothing to launch).
int step_check(const m3_dims *d, const m3_step_args *a, bool *empty, bool mimo) {
  *empty = false;
  if (!d || !a) return M3_ERR_NULL;
  int st = check_step_dims(d, a->d_model, a->dtype, mimo);
  if (st != M3_OK) return st;
  if (!a->u || !a->in_proj_w || !a->out_proj_w || !a->dt_bias || !a->D || !a->B_norm_w || !a->C_norm_w ||
      !a->B_bias || !a->C_bias || (mimo && (!a->mimo_x || !a->mimo_o)) || !a->ssm_state || !a->bx_prev ||
      !a->angle_state || !a->out || !a->workspace)
    return M3_ERR_NULL;
  const int es = a->dtype == M3_BF16 ? 2 : 4;
  const int R = d->mimo_rank;
  const int64_t d_in_proj = 2LL * d->d_inner + 2LL * d->d_state * R + 3LL * d->nheads + d->num_rope_angles;
  if (a->u_stride_b < a->d_model || a->in_proj_stride < a->d_model || a->out_proj_stride < d->d_inner ||
      a->out_stride_b < a->d_model)
    return M3_ERR_SHAPE;
  const StepLayout L = step_layout(d, d_in_proj, es);
  if (a->workspace_bytes < L.bytes) return M3_ERR_SHAPE;
  const unsigned va = (unsigned)(4 * es);  // a 4-element vector
  if (a->u_stride_b % 4 || a->in_proj_stride % 4 || a->out_proj_stride % 4) return M3_ERR_ALIGN;
  if (!aligned_to(a->u, va) || !aligned_to(a->in_proj_w, va) || !aligned_to(a->out_proj_w, va) ||
      !aligned_to(a->B_bias, va) || !aligned_to(a->C_bias, va) || !aligned_to(a->workspace, 256) ||
      !aligned16(a->ssm_state) || !aligned16(a->bx_prev) || !aligned_to(a->angle_state, 4))
    return M3_ERR_ALIGN;
  if (d->batch == 0) {
    *empty = true;
    return M3_OK;
  }
  st = check_device();
  if (st != M3_OK) return st;
  int dev = 0, coop = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) != cudaSuccess || !coop) {
    cudaGetLastError();
    return M3_ERR_DEVICE;
  }
  return M3_OK;
}

int step_entry(const m3_dims *d, const m3_step_args *a, m3_stream_t stream, bool mimo) {
  bool empty = false;
  const int st = step_check(d, a, &empty, mimo);
  if (st != M3_OK || empty) return st;
  const int es = a->dtype == M3_BF16 ? 2 : 4;
  const int R = mimo ? d->mimo_rank : 1;
  const int64_t d_in_proj = 2LL * d->d_inner + 2LL * d->d_state * R + 3LL * d->nheads + d->num_rope_angles;
  const StepLayout L = step_layout(d, d_in_proj, es);

  char *ws = static_cast<char *>(a->workspace);
  m3::StepParams sp = {};
  KParams &kp = sp.kp;
  kp.B = d->batch; kp.H = d->nheads; kp.P = d->headdim; kp.D = d->d_state; kp.R = R;
  kp.A = d->num_rope_angles; kp.A_floor = d->A_floor;
  kp.d_inner = d->d_inner; kp.d_bc = d->d_state * R;
  kp.heads_per_cta = mimo ? m3::mimo_heads_per_cta(kp.H) : 1;
  kp.zx = ws + L.zx_off; kp.zx_sb = L.ldzx; kp.zx_dt = a->dtype; kp.par_dt = a->dtype;
  kp.dt_bias = a->dt_bias; kp.Dp = a->D; kp.wB = a->B_norm_w; kp.wC = a->C_norm_w;
  kp.bB = a->B_bias; kp.bC = a->C_bias; kp.mx = mimo ? a->mimo_x : nullptr; kp.mo = mimo ? a->mimo_o : nullptr;
  kp.h = a->ssm_state; kp.bx = a->bx_prev; kp.ang = a->angle_state;
  kp.y = ws + L.y_off; kp.y_sb = d->d_inner; kp.y_sh = d->headdim; kp.y_sp = 1; kp.y_dt = a->dtype;
  sp.g_in = {a->u, a->u_stride_b, a->in_proj_w, a->in_proj_stride, ws + L.zx_off, L.ldzx,
             d->batch, (int)d_in_proj, a->d_model};
  sp.g_out = {ws + L.y_off, d->d_inner, a->out_proj_w, a->out_proj_stride, a->out, a->out_stride_b,
              d->batch, a->d_model, d->d_inner};
  sp.bar = reinterpret_cast<unsigned *>(ws);

  const int64_t S = (int64_t)d->batch * d->nheads * (mimo ? 1 : d->headdim) * d->d_state * 4;
  add_prefetch(sp, a->out_proj_w, ((int64_t)(a->d_model - 1) * a->out_proj_stride + d->d_inner) * es);
  add_prefetch(sp, a->ssm_state, S);
  add_prefetch(sp, a->bx_prev, S);
  add_prefetch(sp, a->angle_state, (int64_t)d->batch * d->nheads * d->num_rope_angles * 4);
  if (mimo) {
    add_prefetch(sp, a->mimo_x, (int64_t)d->nheads * R * d->headdim * es);
    add_prefetch(sp, a->mimo_o, (int64_t)d->nheads * R * d->headdim * es);
  }
  add_prefetch(sp, a->B_bias, (int64_t)d->nheads * R * d->d_state * es);
  add_prefetch(sp, a->C_bias, (int64_t)d->nheads * R * d->d_state * es);
  add_prefetch(sp, a->B_norm_w, (int64_t)d->d_state * es);
  add_prefetch(sp, a->C_norm_w, (int64_t)d->d_state * es);
  add_prefetch(sp, a->dt_bias, (int64_t)d->nheads * es);
  add_prefetch(sp, a->D, (int64_t)d->nheads * es);
  add_prefetch(sp, a->in_proj_w, ((d_in_proj - 1) * a->in_proj_stride + a->d_model) * es);
  return launch_status(mimo ? m3::launch_mimo_step(sp, reinterpret_cast<cudaStream_t>(stream))
                            : m3::launch_siso_step(sp, reinterpret_cast<cudaStream_t>(stream)));
}

}  // namespace

namespace m3 {
int step_validate(const m3_dims *d, const m3_step_args *a, bool *empty) { return step_check(d, a, empty, true); }
}  // namespace m3

extern "C" {

int m3_siso_decode(const m3_dims *dims, const m3_ssm_args *args, m3_stream_t stream) {
  return ssm_entry(dims, args, stream, false, false);
}

int m3_mimo_decode(const m3_dims *dims, const m3_ssm_args *args, m3_stream_t stream) {
  return ssm_entry(dims, args, stream, true, false);
}

int m3_siso_decode_fused(const m3_dims *dims, const m3_ssm_args *args, m3_stream_t stream) {
  return ssm_entry(dims, args, stream, false, true);
}

int m3_mimo_decode_fused(const m3_dims *dims, const m3_ssm_args *args, m3_stream_t stream) {
  return ssm_entry(dims, args, stream, true, true);
}

int m3_siso_full_fused(const m3_dims *dims, const m3_full_args *args, m3_stream_t stream) {
  return full_entry(dims, args, stream, false);
}

int m3_mimo_prefill(const m3_dims *dims, const m3_full_args *args, int32_t seq_len, m3_stream_t stream) {
  if (seq_len < 0) return M3_ERR_SHAPE;
  KParams kp;
  bool empty = false;
  const int st = full_params(dims, args, true, &kp, &empty);
  if (st != M3_OK || empty || seq_len == 0) return st;
  kp.L = seq_len;
  bool taken = false;
  const cudaError_t e = m3::launch_mimo_prefill(kp, reinterpret_cast<cudaStream_t>(stream), &taken);
  if (!taken) return M3_ERR_UNSUPPORTED;
  return launch_status(e);
}

int m3_siso_prefill(const m3_dims *dims, const m3_full_args *args, int32_t seq_len, m3_stream_t stream) {
  if (seq_len < 0) return M3_ERR_SHAPE;
  KParams kp;
  bool empty = false;
  const int st = full_params(dims, args, false, &kp, &empty);
  if (st != M3_OK || empty || seq_len == 0) return st;
  kp.L = seq_len;
  bool taken = false;
  const cudaError_t e = m3::launch_siso_prefill(kp, reinterpret_cast<cudaStream_t>(stream), &taken);
  if (!taken) return M3_ERR_UNSUPPORTED;
  return launch_status(e);
}

int m3_mimo_full_fused(const m3_dims *dims, const m3_full_args *args, m3_stream_t stream) {
  return full_entry(dims, args, stream, true);
}

int m3_linear_f32(const float *A, int64_t lda, const float *W, int64_t ldw, float *C, int64_t ldc, int32_t M,
                  int32_t N, int32_t K, m3_stream_t stream) {
  if (!A || !W || !C) return M3_ERR_NULL;
  if (M < 0 || N <= 0 || K <= 0 || lda < K || ldw < K || ldc < N) return M3_ERR_SHAPE;
  if (K % 4 || lda % 4 || ldw % 4) return M3_ERR_ALIGN;
  if (!aligned16(A) || !aligned16(W) || (reinterpret_cast<uintptr_t>(C) & 3u)) return M3_ERR_ALIGN;
  if (M == 0) return M3_OK;
  const int st = check_device();
  if (st != M3_OK) return st;
  return launch_status(
      m3::launch_linear_small_m(A, lda, W, ldw, C, ldc, M, N, K, reinterpret_cast<cudaStream_t>(stream)));
}

int64_t m3_linear_bf16_workspace_bytes(int32_t M, int32_t N, int32_t K) {
  if (M < 0 || N <= 0 || K < 64) return -M3_ERR_SHAPE;
  return m3::gemm_bf16_workspace_bytes(M, N, K);
}

int m3_linear_bf16(const void *A, int64_t lda, const void *W, int64_t ldw, void *C, int64_t ldc, int32_t M,
                   int32_t N, int32_t K, int32_t c_dtype, void *workspace, int64_t workspace_bytes,
                   m3_stream_t stream) {
  if (!A || !W || !C) return M3_ERR_NULL;
  if (!dtype_ok(c_dtype)) return M3_ERR_DTYPE;
  if (M < 0 || N <= 0 || K < 64 || lda < K || ldw < K || ldc < N) return M3_ERR_SHAPE;
  if (K % 8 || lda % 8 || ldw % 8) return M3_ERR_ALIGN;
  if (!aligned16(A) || !aligned16(W) || !aligned16(C)) return M3_ERR_ALIGN;
  if (M == 0) return M3_OK;
  const int st = check_device();
  if (st != M3_OK) return st;
  if (!m3::gemm_bf16_supported(A, lda, W, ldw, C, ldc, M, N, K)) return M3_ERR_UNSUPPORTED;
  const int64_t need = m3::gemm_bf16_workspace_bytes(M, N, K);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need)) return M3_ERR_SHAPE;
  if (need > 0 && !aligned16(workspace)) return M3_ERR_ALIGN;
  return launch_status(m3::launch_gemm_bf16(A, lda, W, ldw, C, ldc, M, N, K, c_dtype == M3_BF16,
                                            static_cast<float *>(workspace), reinterpret_cast<cudaStream_t>(stream)));
}

int m3_linear_f32_tc(const float *A_hi, const float *A_lo, int64_t lda, const float *W_hi, const float *W_lo,
                     int64_t ldw, float *C, int64_t ldc, int32_t M, int32_t N, int32_t K, m3_stream_t stream) {
  if (!A_hi || !A_lo || !W_hi || !W_lo || !C) return M3_ERR_NULL;
  if (M < 0 || N <= 0 || K < 32 || lda < K || ldw < K || ldc < N) return M3_ERR_SHAPE;
  if (K % 4 || lda % 4 || ldw % 4) return M3_ERR_ALIGN;
  if (!aligned16(A_hi) || !aligned16(A_lo) || !aligned16(W_hi) || !aligned16(W_lo) || !aligned16(C))
    return M3_ERR_ALIGN;
  if (M == 0) return M3_OK;
  const int st = check_device();
  if (st != M3_OK) return st;
  if (!m3::gemm_tf32x3_supported(A_hi, A_lo, lda, W_hi, W_lo, ldw, C, ldc, M, N, K)) return M3_ERR_UNSUPPORTED;
  return launch_status(m3::launch_gemm_tf32x3(A_hi, A_lo, lda, W_hi, W_lo, ldw, C, ldc, M, N, K,
                                              reinterpret_cast<cudaStream_t>(stream)));
}

int m3_linear_bf16_skinny(const void *A, int64_t lda, const void *W, int64_t ldw, void *C, int64_t ldc, int32_t M,
                          int32_t N, int32_t K, int32_t c_dtype, m3_stream_t stream) {
  if (!A || !W || !C) return M3_ERR_NULL;
  if (!dtype_ok(c_dtype)) return M3_ERR_DTYPE;
  if (M < 0 || M > m3::kSkinnyMaxRows || N <= 0 || K <= 0 || lda < K || ldw < K || ldc < N) return M3_ERR_SHAPE;
  if (K % 8 || lda % 8 || ldw % 8) return M3_ERR_ALIGN;
  if (!aligned16(A) || !aligned16(W) || (reinterpret_cast<uintptr_t>(C) & 3u)) return M3_ERR_ALIGN;
  if (c_dtype == M3_BF16 && (reinterpret_cast<uintptr_t>(C) & 1u)) return M3_ERR_ALIGN;
  if (M == 0) return M3_OK;
  const int st = check_device();
  if (st != M3_OK) return st;
  if (!m3::gemm_skinny_supported(A, lda, W, ldw, C, ldc, M, N, K)) return M3_ERR_UNSUPPORTED;
  return launch_status(m3::launch_gemm_skinny(A, lda, W, ldw, C, ldc, M, N, K, c_dtype == M3_BF16,
                                              reinterpret_cast<cudaStream_t>(stream)));
}

int m3_split_tf32(const float *x, int64_t ldx, float *hi, float *lo, int64_t ld, int32_t rows, int32_t cols,
                  m3_stream_t stream) {
  if (!x || !hi || !lo) return M3_ERR_NULL;
  if (rows < 0 || cols < 0 || ldx < cols || ld < cols) return M3_ERR_SHAPE;
  if (cols % 4 || ldx % 4 || ld % 4) return M3_ERR_ALIGN;
  if (!aligned16(x) || !aligned16(hi) || !aligned16(lo)) return M3_ERR_ALIGN;
  if (rows == 0 || cols == 0) return M3_OK;
  const int st = check_device();
  if (st != M3_OK) return st;
  return launch_status(m3::launch_tf32_split(x, ldx, hi, lo, ld, rows, cols, reinterpret_cast<cudaStream_t>(stream)));
}

int m3_residual_rmsnorm(int32_t dtype, const void *x, int64_t ldx, const void *o, int64_t ldo, const float *w,
                        void *x_out, int64_t ldxo, void *xn, int64_t ldn, int32_t M, int32_t N, float eps,
                        m3_stream_t stream) {
  if (!x || (xn && !w) || (!x_out && !xn)) return M3_ERR_NULL;
  if (!dtype_ok(dtype)) return M3_ERR_DTYPE;
  if (M < 0 || N <= 0 || N > m3::residual_rmsnorm_max_width() || ldx < N || (o && ldo < N) ||
      (x_out && ldxo < N) || (xn && ldn < N))
    return M3_ERR_SHAPE;
  if (M == 0) return M3_OK;
  const int st = check_device();
  if (st != M3_OK) return st;
  return launch_status(m3::launch_residual_rmsnorm(dtype, x, o, w, x_out, xn, M, N, ldx, ldo, ldxo, ldn, eps,
                                                   reinterpret_cast<cudaStream_t>(stream)));
}

int64_t m3_mimo_step_workspace_bytes(const m3_dims *dims, int32_t d_model, int32_t dtype) {
  if (!dims) return -(int64_t)M3_ERR_NULL;
  return step_workspace_bytes(dims, d_model, dtype, true);
}

int m3_mimo_step(const m3_dims *dims, const m3_step_args *args, m3_stream_t stream) {
  return step_entry(dims, args, stream, true);
}

int64_t m3_siso_step_workspace_bytes(const m3_dims *dims, int32_t d_model, int32_t dtype) {
  if (!dims) return -(int64_t)M3_ERR_NULL;
  return step_workspace_bytes(dims, d_model, dtype, false);
}

int m3_siso_step(const m3_dims *dims, const m3_step_args *args, m3_stream_t stream) {
  return step_entry(dims, args, stream, false);
}

int m3_device_error(int reset) {
  const int a = m3::siso_device_error(reset != 0);
  const int b = m3::mimo_device_error(reset != 0);
  const int c = m3::step_device_error(reset != 0);
  const int d = m3::mimo_stream_device_error(reset != 0);
  const int e = m3::gemm_device_error(reset != 0);
  const int f = m3::siso_prefill_device_error(reset != 0);
  if (a < 0 || b < 0 || c < 0 || d < 0 || e < 0 || f < 0) return -1;
  return a | b | c | d | e | f;
}

int m3_selftest_wait_timeout(m3_stream_t stream) {
  const int st = check_device();
  if (st != M3_OK) return st;
  return launch_status(m3::launch_wait_timeout_probe(reinterpret_cast<cudaStream_t>(stream)));
}

int m3_version(void) { return kVersion; }

const char *m3_status_string(int status) {
  switch (status) {
    case M3_OK: return "ok";
    case M3_ERR_NULL: return "a required pointer is NULL";
    case M3_ERR_SHAPE: return "inconsistent or unsupported sizes";
    case M3_ERR_RANK: return "unsupported mimo_rank (supported: 1, 2, 4, 8)";
    case M3_ERR_DTYPE: return "unsupported dtype code";
    case M3_ERR_ALIGN: return "state must be contiguous with a 16-byte aligned base";
    case M3_ERR_LAUNCH: return "CUDA kernel launch failed";
    case M3_ERR_DEVICE: return "no usable CUDA device";
    case M3_ERR_UNSUPPORTED: return "layer outside the single-launch step kernel's range";
    case M3_ERR_SCRATCH: return "workspace larger than the library's static scratch (M3_STEP_STATIC_SCRATCH_BYTES)";
    default: return "unknown status";
  }
}

}  // extern "C"
