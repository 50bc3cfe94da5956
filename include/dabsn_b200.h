/*
 * dabsn_b200 — C ABI of the B200 (sm_100a) kernels for the DABSN scan + read
 * hot path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (cudaStream_t passed as void*), launches asynchronously on that stream and
 * returns a status code (DABSN_OK = 0).  The compute entry points allocate no
 * device memory: the caller (the Python glue in dabsn_b200/, or any other
 * host) owns every buffer.  The one allocating call is dabsn_tp_alloc, which
 * creates the IPC-shareable exchange buffers of tensor parallelism.  Activation tensors are row-major and contiguous, in FP32
 * (dtype = DABSN_F32) or BF16 (dtype = DABSN_BF16); parameters, recurrent
 * state, statistics and gradients of parameters are FP32.
 *
 * Each entry point replaces one implementation the reference library binds for
 * this path (paths inside BleedingXiko/dabsn v0.1.8).
 */
#ifndef DABSN_B200_H_
#define DABSN_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DABSN_F32 0
#define DABSN_BF16 1

/* status codes */
#define DABSN_OK 0
#define DABSN_ERR_SHAPE 1
#define DABSN_ERR_DTYPE 2
#define DABSN_ERR_LAUNCH 3
#define DABSN_ERR_UNSUPPORTED 4
#define DABSN_ERR_TIMEOUT 5

/* Per-unit ([H]) and scalar ([1]) FP32 parameters of the recurrent core, in
 * the order of the reference operator schema (batched_runtime.py:1507-1531). */
typedef struct dabsn_core_params {
  const float* beta;
  const float* log_kappa;
  const float* logit_recover;
  const float* k_s;
  const float* k_y;
  const float* k_b;
  const float* k_n;
  const float* k_bias;
  const float* r_s;
  const float* r_y;
  const float* r_b;
  const float* r_n;
  const float* r_bias;
  const float* logit_c_decay;
  const float* k_c;
  const float* r_c;
  const float* logit_alpha;
  const float* log_lambda;
  const float* logit_c_suppress;
} dabsn_core_params;

/* Library version string and the message of the last failed call (per host
 * thread). */
const char* dabsn_version(void);
const char* dabsn_last_error(void);

/* Status word of the bounded device-side waits on the current device: 0 when
 * no wait has timed out, else the code of the kernel that gave up (1 core scan
 * forward, 2 core scan reverse).  Synchronises the device; reset != 0 clears
 * it.  Diagnostics only: the reference has no device-side waits. */
int dabsn_device_status(int reset);

/* Forward of the registered `dabsn::core_scan_batched` operator.
 * Replaces: src/dabsn/kernels/batched_runtime.py:1098-1205
 * (`_batched_forward_tapes`, the CUDA kernel bound by
 * src/dabsn/kernels/triton.py:275-311 `_registered_cuda_core_scan`).
 *   Wx, Wgx      [B,T,H] activations
 *   rec          [2H,H]  cat(Ug, A) in the activation dtype
 *   init_b/e/c   [B,H]   FP32 initial budget / energy / saturation
 *   U            [B,T,2H] out: (y, budget after the step)
 *   nov, plast, expr, write, energy, sat, gate  [B,T,H] out tapes
 *   fin_b/e/c    [B,H]   out: final state (activation dtype)              */
int dabsn_core_scan_fwd(int dtype, int64_t B, int64_t T, int64_t H, const void* Wx,
                        const void* Wgx, const void* rec, const dabsn_core_params* params,
                        const float* init_b, const float* init_e, const float* init_c, void* U,
                        void* nov, void* plast, void* expr, void* write, void* energy, void* sat,
                        void* gate, void* fin_b, void* fin_e, void* fin_c, void* stream);

/* Reverse of `dabsn::core_scan_batched`.
 * Replaces: src/dabsn/kernels/batched_runtime.py:1333-1504
 * (`DABSNCoreScanBatched.backward`, the autograd formula registered at
 * :1630-1634), whose per-step math is `_backward_step` (:299-466).
 *   U, energy, sat, gate, plast, expr  saved forward tapes
 *   gU [B,T,2H], gnov/gp/gay/gwrite/ge/gc [B,T,H], gfin_b/e/c [B,H]:
 *        FP32 upstream gradients; NULL means zero.
 *   gWx, gWgx, day [B,T,H] out (activation dtype): gradients of Wx and Wgx and
 *        the expression adjoint; grad[Ug;A] = [gWgx, day]^T y is left to a
 *        library GEMM.
 *   g_init_b/e/c [B,H] out FP32; partial [B,19,H] out FP32 per-sequence sums
 *        of the 16 per-unit and 3 scalar parameter gradients.               */
int dabsn_core_scan_bwd(int dtype, int64_t B, int64_t T, int64_t H, const void* U,
                        const void* energy, const void* sat, const void* gate, const void* plast,
                        const void* expr, const void* rec, const dabsn_core_params* params,
                        const float* init_b, const float* init_c, const float* gU,
                        const float* gnov, const float* gp, const float* gay, const float* gwrite,
                        const float* ge, const float* gc, const float* gfin_b,
                        const float* gfin_e, const float* gfin_c, void* gWx, void* gWgx, void* day,
                        float* g_init_b, float* g_init_e, float* g_init_c, float* partial,
                        void* stream);


/* Grid-wide variants of the core scan for wide states (BF16 only; H a
 * multiple of 16 with H/16 <= the SM count, up to 32 sequences per call).
 * Same mathematics and tensors as dabsn_core_scan_fwd / _bwd; they replace
 * the same reference functions (batched_runtime.py:1098-1205 and :1333-1504),
 * which the reference runs at these widths as a per-step cuBLAS GEMM plus a
 * compiled pointwise kernel replayed from CUDA graphs.  The caller passes
 * `scratch` of at least dabsn_core_scan_wide_scratch_bytes(H) device bytes
 * (exchange buffer + grid-barrier counter; reset by the call).  The kernel
 * is a cooperative launch of H/16 (or H/8) co-resident CTAs.  The reverse
 * reads the tapes' gradients gU ... gc in `grad_dtype` (DABSN_F32, or
 * DABSN_BF16: the tapes' own dtype, as autograd delivers them).  In
 * dabsn_core_scan_wide_bwd, bit i of `row_bcast` (0 gnov, 1 gp, 2 gay,
 * 3 gwrite, 4 ge, 5 gc) marks that gradient as one value per (sequence,
 * step), a [B, T] array applied to every unit. */
size_t dabsn_core_scan_wide_scratch_bytes(int64_t H);
int dabsn_core_scan_wide_fwd(int64_t B, int64_t T, int64_t H, const void* Wx, const void* Wgx,
                             const void* rec, const dabsn_core_params* params,
                             const float* init_b, const float* init_e, const float* init_c,
                             void* U, void* nov, void* plast, void* expr, void* write,
                             void* energy, void* sat, void* gate, void* fin_b, void* fin_e,
                             void* fin_c, void* scratch, size_t scratch_bytes, void* stream);
int dabsn_core_scan_wide_bwd(int64_t B, int64_t T, int64_t H, const void* U, const void* energy,
                             const void* sat, const void* gate, const void* plast,
                             const void* expr, const void* rec, const dabsn_core_params* params,
                             const float* init_b, const float* init_c, int grad_dtype,
                             unsigned row_bcast, const void* gU, const void* gnov, const void* gp,
                             const void* gay, const void* gwrite, const void* ge,
                             const void* gc,
                             const float* gfin_b, const float* gfin_e, const float* gfin_c,
                             void* gWx, void* gWgx, void* day, float* g_init_b, float* g_init_e,
                             float* g_init_c, float* partial, void* scratch,
                             size_t scratch_bytes, void* stream);

/* dabsn::permanent_delta_scan (permanent.py:56-110, 384-431): the delta-rule
 * scan r_t = S k_t, S += beta_t (v_t - r_t) k_t^T over S [h x h] (zero at
 * t = 0), k, v, r [B,T,h], beta [B,T], h <= 128, FP32 or BF16 (FP32 state).
 * `ckpt` (optional forward output, dabsn_delta_ckpt_floats floats) receives S
 * every 64 steps and at the end; the reverse needs it and the forward's r.
 * g = dL/dr FP32; dk, dv, dbeta in the input dtype. */
size_t dabsn_delta_ckpt_floats(int64_t B, int64_t T, int64_t h);
int dabsn_permanent_delta_fwd(int dtype, int64_t B, int64_t T, int64_t h, const void* k,
                              const void* v, const void* beta, void* out, float* ckpt,
                              void* stream);
int dabsn_permanent_delta_bwd(int dtype, int64_t B, int64_t T, int64_t h, const void* k,
                              const void* v, const void* beta, const void* recon, const float* g,
                              const float* ckpt, void* dk, void* dv, void* dbeta, void* stream);

/* dabsn::local_field_gather (local_field.py:208-240): out [B,N,K,D] =
 * x[b, patch[n,k], :] for x [B,C,D], patch int64 [N,K] with values < C.
 * dabsn_local_field_scatter: grad_x [B,C,D] from grad_out [B,N,K,D], summing
 * per cell c the slots listed in order[offsets[c] .. offsets[c+1]] (the flat
 * slot indices n*K + k sorted by source cell; offsets int64 [C+1]). */
int dabsn_local_field_gather(int dtype, int64_t B, int64_t C, int64_t N, int64_t K, int64_t D,
                             const void* x, const int64_t* patch, void* out, void* stream);
int dabsn_local_field_scatter(int dtype, int64_t B, int64_t C, int64_t N, int64_t K, int64_t D,
                              const void* grad_out, const int64_t* order, const int64_t* offsets,
                              void* grad_x, void* stream);

/* Readout + mean cross-entropy without materialised logits (replaces
 * ChunkedLinearCrossEntropy / chunked_linear_cross_entropy,
 * runtime/loss.py:52-231, for BF16 hidden and weight): hidden [rows, D],
 * weight [V, D] BF16 (16-byte aligned, D a multiple of 8), bias FP32 [V] or
 * NULL, targets int64 [rows].  Forward: lse and tgt_logit FP32 [rows]
 * (workspace: dabsn_linear_ce_workspace_floats floats); the loss is
 * mean(lse - tgt_logit) over rows whose target != ignore_index.  Reverse:
 * dlogits workspace BF16 [rows, dabsn_linear_ce_ld(V)], dhidden BF16
 * [rows, D], dweight FP32 [V, D] written (accumulate 0) or added to
 * (accumulate 1); scale (one FP32 device value) = dL/dloss / valid rows.
 * The caller may run the reverse over row chunks (pointers offset to the
 * chunk's first row, the workspace sized for the chunk), accumulating dweight,
 * to bound the workspace as the reference's chunk budget bounds its logits.
 * round_bf16 rounds the logits to BF16 before the softmax (autocast). */
int64_t dabsn_linear_ce_ld(int64_t V);
size_t dabsn_linear_ce_workspace_floats(int64_t rows, int64_t V);
int dabsn_linear_ce_fwd(int64_t rows, int64_t V, int64_t D, const void* hidden,
                        const void* weight, const float* bias, const int64_t* targets,
                        int ignore_index, int round_bf16, float* lse, float* tgt_logit,
                        float* workspace, void* stream);
int dabsn_linear_ce_bwd(int64_t rows, int64_t V, int64_t D, const void* hidden,
                        const void* weight, const float* bias, const int64_t* targets,
                        int ignore_index, int round_bf16, const float* lse, const float* scale,
                        void* dlogits, void* dhidden, float* dweight, int accumulate,
                        void* stream);

/* Tensor parallel over state units (replaces the per-step loop of
 * TensorParallelDABSNCore.forward_from_state, core.py:609-874, and its
 * autograd through _GatherHiddenRecurrent, core.py:525-600): the grid-wide
 * scan spread over P <= 8 GPUs of one node, BF16.  Rank `rank` owns units
 * [ubase, ubase + Hl) (all ranks the same Hl): its Wx/Wgx/tapes/gradients are
 * [B,T,Hl], init/finals [B,Hl], parameters its slices, `rec` its rows
 * [Ug[units]; A[units]] ([2Hl, H]) forward and the full [Ug; A] ([2H, H])
 * backward.  `peer_bufs` holds every rank's exchange buffer (P device
 * pointers, dabsn_tp_buffer_bytes(H) bytes each, from dabsn_tp_alloc and
 * opened with dabsn_tp_ipc_open; zero-initialised once, never reset):
 * each step the ranks store their slices into all buffers and meet at a
 * bounded cross-GPU barrier on the buffers' counters.  `base` is the count
 * the counters held before this call (0 for the first call on fresh buffers,
 * then the previous call's *next_base); every rank makes the same sequence of
 * calls.  A timed-out barrier records status 3 (forward) or 4 (reverse). */
size_t dabsn_tp_buffer_bytes(int64_t H);
int dabsn_tp_alloc(size_t bytes, void** ptr);
int dabsn_tp_free(void* ptr);
int dabsn_tp_ipc_handle(void* ptr, void* handle);      /* 64-byte CUDA IPC handle */
int dabsn_tp_ipc_open(const void* handle, void** ptr);
int dabsn_tp_ipc_close(void* ptr);
int dabsn_core_scan_tp_fwd(int64_t B, int64_t T, int64_t H, int64_t Hl, int64_t ubase, int P,
                           int rank, void* const* peer_bufs, uint32_t base, uint32_t* next_base,
                           const void* Wx, const void* Wgx, const void* rec,
                           const dabsn_core_params* params, const float* init_b,
                           const float* init_e, const float* init_c, void* U, void* nov,
                           void* plast, void* expr, void* write, void* energy, void* sat,
                           void* gate, void* fin_b, void* fin_e, void* fin_c, void* stream);
int dabsn_core_scan_tp_bwd(int64_t B, int64_t T, int64_t H, int64_t Hl, int64_t ubase, int P,
                           int rank, void* const* peer_bufs, uint32_t base, uint32_t* next_base,
                           const void* U, const void* energy, const void* sat, const void* gate,
                           const void* plast, const void* expr, const void* rec_full,
                           const dabsn_core_params* params, const float* init_b,
                           const float* init_c, int grad_dtype, const void* gU,
                           const void* gnov, const void* gp, const void* gay,
                           const void* gwrite, const void* ge, const void* gc,
                           const float* gfin_b,
                           const float* gfin_e, const float* gfin_c, void* gWx, void* gWgx,
                           void* day, float* g_init_b, float* g_init_e, float* g_init_c,
                           float* partial, void* stream);

/* Forward wide scan that allocates nothing.  No counterpart in the reference:
 * it exists for callers that cannot allocate device memory when they run the
 * scan (allocator or memory-pool callbacks, host frameworks that own every
 * allocation, runtimes that forbid cudaMalloc after start-up).  Same
 * arguments and results as dabsn_core_scan_wide_fwd without `scratch`: the
 * scratch is a static device array of DABSN_WIDE_NOALLOC_SCRATCH_BYTES that
 * each GPU loading the library holds until exit, so H is limited to
 * DABSN_WIDE_NOALLOC_MAX_H (larger H returns DABSN_ERR_UNSUPPORTED).  The
 * first call on a device (and the first after a cudaDeviceReset) looks up the
 * array's device address (make it before any stream capture).  All calls share the array: calls that overlap on the
 * GPU (other streams, other host threads) race and must be serialised by the
 * caller.  The call clears the barrier counter on `stream` itself. */
#define DABSN_WIDE_NOALLOC_MAX_H 2048
#define DABSN_WIDE_NOALLOC_SCRATCH_BYTES (2 * 32 * 2 * DABSN_WIDE_NOALLOC_MAX_H * 2 + 256)
int dabsn_core_scan_wide_fwd_noalloc(int64_t B, int64_t T, int64_t H, const void* Wx,
                                     const void* Wgx, const void* rec,
                                     const dabsn_core_params* params, const float* init_b,
                                     const float* init_e, const float* init_c, void* U,
                                     void* nov, void* plast, void* expr, void* write,
                                     void* energy, void* sat, void* gate, void* fin_b,
                                     void* fin_e, void* fin_c, void* stream);

/* Mean cross-entropy over materialised logits [rows][ld] (FP32 or BF16,
 * `dtype`), one pass each way.  Forward writes per row the log-sum-exp and
 * the target's logit (FP32; 0 for rows whose target is ignore_index; NaN, and
 * device status code 7, for a target outside [0, V)).  Reverse writes
 * dlogits [rows][V] in the logits' dtype: scale * (softmax - onehot) for
 * valid rows, 0 for ignored ones, with `scale` one FP32 value on the device.
 * Replaces: src/dabsn/runtime/loss.py:187-231
 * (`chunked_cross_entropy_from_logits`: FP32 upcast of the logits, in chunks
 * above the element budget, then logsumexp / gather and autograd). */
int dabsn_ce_logits_fwd(int dtype, int64_t rows, int64_t V, int64_t ld, const void* logits,
                        const int64_t* targets, int64_t ignore_index, float* lse,
                        float* tgt_logit, void* stream);
int dabsn_ce_logits_bwd(int dtype, int64_t rows, int64_t V, int64_t ld, const void* logits,
                        const int64_t* targets, int64_t ignore_index, const float* lse,
                        const float* scale, void* dlogits, void* stream);

/* The core's input projections on the tcgen05 GEMM (BF16, FP32 accumulation):
 * Wx = x W^T and Wgx = x Wg^T + bias_g (bias rounded to BF16 first, as
 * autocast casts it), x [M][D] with row stride ldx, W and Wg [H][D], outputs
 * [M][H]; one launch.  Reverse: dx = dWx W + dWgx Wg [M][D] (skipped when dx
 * is null), dW = dWx^T x and dWg = dWgx^T x [H][D].  D and H multiples of 8,
 * operands 16-byte aligned.
 * Replaces: src/dabsn/core.py:280-283 (`self.W(inputs)`, `self.Wg(inputs)`,
 * two nn.Linear calls, cuBLAS under autocast) and their autograd. */
int dabsn_input_proj_fwd(int64_t M, int64_t D, int64_t H, const void* x, int64_t ldx,
                         const void* W, const void* Wg, const float* bias_g, void* Wx, void* Wgx,
                         void* stream);
int dabsn_input_proj_bwd(int64_t M, int64_t D, int64_t H, const void* x, int64_t ldx,
                         const void* W, const void* Wg, const void* gWx, const void* gWgx,
                         void* dx, void* dW, void* dWg, void* stream);

/* Gradient of the recurrent matrices over all M = B*T steps on the tcgen05
 * GEMM: grad Ug = dWgx^T y, grad A = dA^T y ([H][H] BF16), with y [M][H] of
 * row stride ldy (the y half of the U tape), dWgx and dA [M][H].
 * Replaces: src/dabsn/kernels/batched_runtime.py:1474-1481 (one cuBLAS
 * matmul of [dWgx, dA]^T and y in the activation dtype). */
int dabsn_rec_grad(int64_t M, int64_t H, const void* y, int64_t ldy, const void* gWgx,
                   const void* day, void* gUg, void* gA, void* stream);

/* The read's output projection and long-channel term on the tcgen05 GEMM:
 * out [M][H] FP32 = bf16(y W0^T + b W1^T + r W2^T + bf16(bias)) +
 * (*add_scale) * addend, with W = [W0 W1 W2] ([H][3H] BF16), y / b / r
 * [M][H] BF16 of row strides ldy / ldb / ldr (y and b read in place from
 * the U tape), addend [M][H] FP32, add_scale one FP32 value on the device.
 * Reverse: dy, db, dr = gout W_i ([M][H] BF16) and dW = gout^T [y b r]
 * ([H][3H] BF16) for gout [M][H] BF16.
 * Replaces: src/dabsn/read.py:435-438 (`out(torch.cat([y, budget,
 * retrieved]))`, an nn.Linear on a concatenated copy, cuBLAS under
 * autocast, plus `long_gain * long`). */
int dabsn_read_out_fwd(int64_t M, int64_t H, const void* y, int64_t ldy, const void* bud,
                       int64_t ldb, const void* ret, int64_t ldr, const void* W,
                       const float* bias, const float* addend, const float* add_scale,
                       float* out, void* stream);
int dabsn_read_out_bwd(int64_t M, int64_t H, const void* y, int64_t ldy, const void* bud,
                       int64_t ldb, const void* ret, int64_t ldr, const void* W,
                       const void* gout, void* dy, void* dbud, void* dret, void* dW,
                       void* stream);

/* Row glue of the projections' reverse passes (replaces the elementwise and
 * reduction work autograd runs around read.py:435-438 and core.py:278-307
 * under autocast).  Rows are processed in blocks of 64;
 * dabsn_glue_blocks(R) = the number of blocks.
 * dabsn_read_out_grad_prep: grad FP32 [R, H] (the gradient of the read's
 *   FP32 output), long_channel FP32 [R, H], long_gain FP32 [1] ->
 *   grad_bf16 BF16 [R, H] (the GEMMs' operand), dlong FP32 [R, H] =
 *   long_gain * grad, colpart FP32 [blocks, H] (column sums of grad_bf16 per
 *   block: summed, the bias gradient), dotpart FP32 [blocks] (per-block sums
 *   of grad * long_channel: summed, the gain's gradient).  H a multiple of 8.
 * dabsn_colsum_bf16: x BF16 [R, H] -> colpart FP32 [blocks, H]. */
int64_t dabsn_glue_blocks(int64_t R);
int dabsn_read_out_grad_prep(int64_t R, int64_t H, const float* grad, const float* long_channel,
                             const float* long_gain, void* grad_bf16, float* dlong,
                             float* colpart, float* dotpart, void* stream);
int dabsn_colsum_bf16(int64_t R, int64_t H, const void* x, float* colpart, void* stream);

/* Fused long-memory channel, forward: the expected / retention / long
 * recurrences and their elementwise glue in one pass.
 * Replaces: src/dabsn/kernels/long.py:492-579 (`fused_long_scan_from_state`:
 * three `dabsn::linear_recurrence` launches of the Triton kernel at
 * long.py:106-148 plus ATen glue); loop form at src/dabsn/read.py:597-640.
 *   write, plasticity [B,T,H] activations
 *   logits [4] FP32: logit_retain, logit_expect_retain, logit_retention_decay,
 *          logit_retention_strength
 *   init   [3,B,H] FP32 (long, expected, retention) or NULL for (0, 0, 1)
 *   out    [B,T,H] FP32 long-memory sequence
 *   ckpt   [B, ceil(T/dabsn_long_chunk()), 3, H] FP32 chunk checkpoints for
 *          the reverse pass, or NULL (inference)
 *   fin    [3,B,H] FP32 final (long, expected, retention) or NULL           */
int dabsn_long_chunk(void);
int dabsn_long_fwd(int dtype, int64_t B, int64_t T, int64_t H, const void* write,
                   const void* plasticity, const float* logits, const float* init, float* out,
                   float* ckpt, float* fin, void* stream);

/* Fused long-memory channel, reverse.
 * Replaces: the autograd of the three `dabsn::linear_recurrence` calls
 * (src/dabsn/kernels/long.py:425-430 and the Triton reverse kernel at
 * long.py:150-212, which stores a [B,T,H] scratch tape) plus the glue.
 *   gout [B,T,H] FP32 upstream gradient of out; gfin [3,B,H] or NULL
 *   dwrite, dplast [B,T,H] out (activation dtype)
 *   ginit [3,B,H] out FP32 or NULL; partial [B*H,4] out FP32 per-element
 *          gradients of the four logits (sum them).                         */
int dabsn_long_bwd(int dtype, int64_t B, int64_t T, int64_t H, const void* write,
                   const void* plasticity, const float* logits, const float* ckpt,
                   const float* gout, const float* gfin, void* dwrite, void* dplast, float* ginit,
                   float* partial, void* stream);

/* Exact three-way admitted read, forward.
 * Replaces: src/dabsn/kernels/compact_admitted.py:16-143
 * (`dense_bmm_three_way_read_exact` under the query-chunked
 * `dabsn::admitted_three_way_read_compact_dense_bmm`), reached from
 * src/dabsn/kernels/triton.py:314-406 (`cuda_compact_three_way_read`).
 *   mode 0 = seq (causal), 1 = field; total_steps = T of the full sequence
 *   query [B,T,H], bank_keys/bank_writes/next_writes [B,N,H],
 *   cocktail [B,T,4], bank_cocktail [B,N,4], bank_key_bias/bank_admission
 *   [B,N] (activation dtype); scale [1] FP32; bank_idx [B,N] int64;
 *   bank_valid [B,N] bool; gains [4] FP32 (short, pad, induct, cocktail)
 *   out [B,T,H] activation dtype; streams [B,T,3,H] FP32 and lse [B,T,3]
 *   FP32 are saved for the reverse pass.                                    */
int dabsn_read_fwd(int dtype, int64_t B, int64_t T, int64_t N, int64_t H, int mode,
                   int64_t total_steps, const void* query, const void* bank_keys,
                   const void* bank_writes, const void* next_writes, const void* cocktail,
                   const void* bank_cocktail, const void* bank_key_bias,
                   const void* bank_admission, const float* scale, const int64_t* bank_idx,
                   const uint8_t* bank_valid, const float* gains, void* out, float* streams,
                   float* lse, void* stream);

/* Exact three-way admitted read, reverse.
 * Replaces: the autograd of `dense_bmm_three_way_read_exact` (bmm / softmax
 * backward over saved [B,T,N] weights; compact_admitted.py:40-80) and the
 * analytic formula at src/dabsn/kernels/admitted.py:126-239.
 *   gout [B,T,H] FP32; u3 [B,T,3] out FP32 (gout . stream, for the gains);
 *   dquery [B,T,H], dkeys/dwrites/dnext [B,N,H] out (activation dtype);
 *   dcocktail [B,T,4], dbias [B,N] (gradient of key_bias and of admission),
 *   dbank_cocktail [B,N,4], partial [B,ceil(T/32),2] (d scale, d cocktail
 *   gain) out FP32.                                                         */
int dabsn_read_bwd(int dtype, int64_t B, int64_t T, int64_t N, int64_t H, int mode,
                   int64_t total_steps, const void* query, const void* bank_keys,
                   const void* bank_writes, const void* next_writes, const void* cocktail,
                   const void* bank_cocktail, const void* bank_key_bias,
                   const void* bank_admission, const float* scale, const int64_t* bank_idx,
                   const uint8_t* bank_valid, const float* gains, const float* streams,
                   const float* lse, const float* gout, float* u3, void* dquery,
                   float* dcocktail, void* dkeys, void* dwrites, void* dnext, float* dbias,
                   float* dbank_cocktail, float* partial, void* stream);

/* Read admission and admitted bank (replaces the glue of
 * DABSNRead._unified_forward, read.py:152-303, with the admission score of
 * _AdmittedReadParameters.admission, read.py:58-72).
 * dabsn_admission_fwd: expression, novelty, plasticity, energy, saturation
 *   [B,T,H] (dtype code); params FP32 [8] = p_gain, novelty_gain, null_bias,
 *   adm_p_gain, adm_novelty_gain, adm_saturation_gain, adm_energy_gain,
 *   adm_bias; window FP32 [1] = softplus(admit_window); mode 0 seq (causal
 *   prefix max) / 1 field (whole-sequence max).  Out: query [B,T,H] in
 *   query_dtype (FP32 or BF16: the read's compute dtype), key_bias,
 *   admission FP32 [B,T], cocktail FP32 [B,T,4], stats FP32 [B,T,8] (saved
 *   for the backward; stats[6] is the expression norm), order int64 [B,T]
 *   (members, then the rest, each ascending), counts int64 [B], inv int32
 *   [B,T] (bank slot of a member, -1 otherwise).
 * dabsn_bank_gather: the first n entries of `order`: bank writes and next
 *   writes (write dtype), keys (normalised writes, key_dtype FP32 or BF16),
 *   cocktails, biases, admissions FP32, positions int64, valid flags (bool),
 *   key norms FP32.
 * dabsn_admission_bwd: gradients (any may be NULL) of query, cocktail,
 *   keys, writes, next writes, bank cocktail, bank bias, bank admission ->
 *   d expression and d write (dtype code), d_means FP32 [B,T,4] (per-unit
 *   gradient of plasticity, novelty, energy, saturation) and param_part FP32
 *   [B,T,8] (per-token terms of the 8 parameter gradients).  The [.,.,H]
 *   gradients (query, keys, writes, next writes) are all in grad_dtype (BF16
 *   only with BF16 activations); the rest are FP32.  Query and keys are
 *   recomputed from expression, write, stats and key_norm. */
int dabsn_admission_fwd(int dtype, int64_t B, int64_t T, int64_t H, int mode,
                        const void* expression, const void* novelty, const void* plasticity,
                        const void* energy, const void* saturation, const float* params,
                        const float* window, int query_dtype, void* query, float* key_bias,
                        float* admission, float* cocktail, float* stats, int64_t* order,
                        int64_t* counts, int* inv, void* stream);
int dabsn_bank_gather(int dtype, int64_t B, int64_t T, int64_t H, int64_t n, const void* write,
                      const float* key_bias, const float* admission, const float* cocktail,
                      const int64_t* order, const int64_t* counts, void* bank_writes,
                      int key_dtype, void* bank_keys, void* next_writes, float* bank_cocktail,
                      float* bank_bias, float* bank_admission, int64_t* bank_idx,
                      void* bank_valid, float* key_norm, void* stream);
int dabsn_admission_bwd(int dtype, int64_t B, int64_t T, int64_t H, int64_t n,
                        const void* expression, const void* write, const float* stats,
                        const float* cocktail, const float* params, const int* inv,
                        const float* key_norm, int grad_dtype, const void* d_query,
                        const float* d_cocktail, const void* d_keys, const void* d_writes,
                        const void* d_next, const float* d_bank_cocktail,
                        const float* d_bank_bias, const float* d_bank_admission,
                        void* d_expression, void* d_write, float* d_means, float* param_part,
                        void* stream);

/* Three-way admitted read for wide states (BF16 only, H a multiple of 8,
 * meant for H > 256).  Replaces the same reference functions as
 * dabsn_read_fwd / _bwd (compact_admitted.py:16-143 through triton.py:314-406),
 * as a chain of tensor-core GEMMs and two row-softmax kernels.
 *   query, bank_keys, bank_writes, next_writes BF16 [B,T,H] / [B,N,H];
 *   cocktail [B,T,4] and bank_cocktail [B,N,4] BF16; bank_key_bias and
 *   bank_admission FP32 [B,N]; scale FP32 [1]; gains FP32 [4].
 * Forward: out BF16 [B,T,H]; compat BF16 [B,T,dabsn_read_wide_ld(N)]
 * (bf16(q.k), saved for the backward); lse FP32 [B,T,3].
 * Backward: gout BF16 [B,T,H]; u3 [B,T,3] (gout . stream), dquery,
 * dkeys, dwrites, dnext BF16; dcocktail [B,T,4], dbias [B,N], dbank_cocktail
 * [B,N,4], rowpart [B,T,2] (d scale, d cocktail gain) FP32.
 * `workspace` holds at least dabsn_read_wide_fwd_workspace /
 * _bwd_workspace bytes of device memory (16-byte aligned). */
int64_t dabsn_read_wide_ld(int64_t N);
size_t dabsn_read_wide_fwd_workspace(int64_t B, int64_t T, int64_t N);
size_t dabsn_read_wide_bwd_workspace(int64_t B, int64_t T, int64_t N);
int dabsn_read_wide_fwd(int64_t B, int64_t T, int64_t N, int64_t H, int mode,
                        int64_t total_steps, const void* query, const void* bank_keys,
                        const void* bank_writes, const void* next_writes, const void* cocktail,
                        const void* bank_cocktail, const float* bank_key_bias,
                        const float* bank_admission, const float* scale,
                        const int64_t* bank_idx, const uint8_t* bank_valid, const float* gains,
                        void* out, void* compat, float* lse, void* workspace,
                        size_t workspace_bytes, void* stream);
int dabsn_read_wide_bwd(int64_t B, int64_t T, int64_t N, int64_t H, int mode,
                        int64_t total_steps, const void* query, const void* bank_keys,
                        const void* bank_writes, const void* next_writes, const void* cocktail,
                        const void* bank_cocktail, const float* bank_key_bias,
                        const float* bank_admission, const float* scale,
                        const int64_t* bank_idx, const uint8_t* bank_valid, const float* gains,
                        const void* compat, const float* lse, const void* gout, float* u3,
                        void* dquery, float* dcocktail, void* dkeys, void* dwrites,
                        void* dnext, float* dbias, float* dbank_cocktail, float* rowpart,
                        void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DABSN_B200_H_ */
