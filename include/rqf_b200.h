/*
 * rqf_b200.h — C ABI of the B200 (sm_100a) backend for the RQF complex
 * linear-recurrence scan family.
 *
 * Every entry point takes raw device pointers, sizes and a CUDA stream, never
 * allocates or frees device memory, and returns an int status (RQF_OK == 0).
 * Complex tensors are interleaved re/im float32 (the memory layout of a
 * contiguous torch.complex64 tensor, i.e. torch.view_as_real).  Per-channel
 * coefficients (c1, c2, tap0, tap1) are complex (F,) vectors.
 *
 * Gradients follow PyTorch's conjugate-Wirtinger convention, e.g.
 *   grad_c1 = sum_{b,t} conj(y[t-1]) * g[t],   grad_u = conj(c2) * g.
 *
 * Two memory layouts are served:
 *   BTF  (batch, time, filters): filters innermost — the layout of
 *        rqf_models/ops/chunked_scan_kernel.py:_triton_chunked_scan (:340)
 *        and _triton_chunked_scan_prospective (:506).  No permutes are made.
 *   FBT  (filters, batch, time): time innermost — the layout of
 *        rqf_models/ops/fbt_scan_kernel.py:fbt_prospective_scan (:332),
 *        fbt_recompute_scan (:667) and the selective kernels
 *        rqf_models/ops/selective_scan_kernel.py (:491, :517).
 *
 * Saved context.  Forward kernels write one complex "carry" per (row, tile):
 * the recurrence state entering that tile.  Backward kernels recompute the
 * states from those carries instead of reading a saved output.  The caller
 * owns the carry buffer (rqf_*_carry_count complex entries) between forward
 * and backward.
 *
 * Scratch.  Forward and full-BPTT backward kernels chain tiles of a row with a
 * decoupled look-back; they need a caller-provided scratch buffer of
 * rqf_*_scratch_bytes() bytes (16-byte aligned), which the entry point clears
 * with cudaMemsetAsync on the given stream before the launch.  Scratch may be
 * reused by the next call on the same stream.
 *
 * Errors.  A look-back wait is bounded; when it runs out the kernel latches
 * RQF_ERR_LOOKBACK_TIMEOUT into a per-device error word and returns.  Read it
 * with rqf_read_device_error (synchronises the stream).
 */
#ifndef RQF_B200_H
#define RQF_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *rqf_stream_t; /* identical to cudaStream_t */

enum rqf_status {
  RQF_OK = 0,
  RQF_ERR_SHAPE = 1,            /* negative / inconsistent sizes            */
  RQF_ERR_ALIGN = 2,            /* pointer alignment requirement violated   */
  RQF_ERR_LOOKBACK_TIMEOUT = 3, /* bounded cross-tile wait gave up          */
  RQF_ERR_LAUNCH = 4,           /* CUDA launch / memset error               */
  RQF_ERR_ARGUMENT = 5,         /* null pointer or unsupported option       */
  RQF_ERR_CAPACITY = 6,         /* size beyond a fixed internal maximum     */
  RQF_ERR_PIPELINE_TIMEOUT = 7  /* bounded tensor-core pipeline wait gave up */
};

/* ---- library information -------------------------------------------- */
int rqf_abi_version(void);
const char *rqf_status_string(int status);

/* Copy (and optionally clear) the device error word of the current device.
 * Synchronises `stream`. */
int rqf_read_device_error(int *out_code, int clear, rqf_stream_t stream);

/* Diagnostic: run one look-back wait on a predecessor flag that nothing ever
 * publishes, so the bounded wait runs out (about 0.3 s), latches
 * RQF_ERR_LOOKBACK_TIMEOUT in the device error word and the kernel returns —
 * the failure path of every cross-tile wait, without faulting or hanging the
 * GPU.  `scratch` needs 256 bytes.  Read the result with
 * rqf_read_device_error. */
int rqf_selftest_lookback_timeout(void *scratch, rqf_stream_t stream);

/* ---- sizes of saved context and scratch ------------------------------ */
/* BTF kernels: rows = batch * filters.  Two kernel families share the
 * buffers: a streaming one (tiles of 1..8 x 128 steps, re-read from L2 in a
 * second pass, entry states saved per 128-step sub-tile) for few chains of
 * batch x 32 channels, and a tile-resident one
 * (tiles of 1..4 x 64 steps held in shared memory, entry states saved per
 * 64-step sub-tile) for many.  rqf_btf_num_tiles gives the 64-step sub-tiles
 * along time (an upper bound on the tiles of either family); size buffers
 * with rqf_btf_carry_count / _scratch_bytes.
 * Every (B,T,F) scan entry point takes `path`, per call: 0 = automatic
 * (streaming below 48 chains of batch x 32 channels), 1 = streaming, 2 =
 * tile-resident; anything else is RQF_ERR_ARGUMENT.  A backward must be given
 * the path its forward was given, since the saved entry states of the two
 * families differ (the automatic choice depends only on batch and filters,
 * so it agrees by itself). */
int64_t rqf_btf_num_tiles(int64_t time);
int64_t rqf_btf_carry_count(int64_t batch, int64_t time, int64_t filters);
size_t rqf_btf_scratch_bytes(int64_t batch, int64_t time, int64_t filters);
/* FBT kernels: rows = filters * batch, tiles of 2048 samples along time.  The
 * saved context ("carries", complex64) holds one entry state per thread (256)
 * of every tile plus one marker element: the forward fills it and the
 * backward replays each thread's states from it (rqf_fbt_carry_count; 1/8 of
 * the (F,B,T) tensor's size; 0 for rejected shapes).  The scratch size is
 * SIZE_MAX for shapes that the FBT entry points reject (RQF_ERR_SHAPE). */
int64_t rqf_fbt_num_tiles(int64_t time);
int64_t rqf_fbt_carry_count(int64_t filters, int64_t batch, int64_t time);
size_t rqf_fbt_scratch_bytes(int64_t filters, int64_t batch, int64_t time);

/* ---- diagonal scan, (B,T,F) layout ----------------------------------- *
 * Replaces rqf_models/ops/chunked_scan_kernel.py:_chunked_scan_forward_raw
 * (:217) / _chunked_scan_kernel (:60):  y[t] = c1*y[t-1] + c2*u[t], y[-1]=0.
 * u is complex (B,T,F) or, with u_is_real != 0, float32 (B,T,F) — the real
 * input that rqf_models/ops/scan.py:sequential_scan (:290, :366) promotes to
 * complex before the kernel; the result is identical. */
int rqf_chunked_scan_forward(const float *c1, const float *c2, const void *u,
                             int u_is_real, float *y, float *carries,
                             void *scratch, int64_t batch, int64_t time,
                             int64_t filters, int path, rqf_stream_t stream);

/* Magnitude |y[t]| of the same scan, for no-grad consumers: replaces
 * rqf_models/ops/triton_scan_kernel.py:_sequential_scan_forward_abs_raw_block_f
 * (:507) and _sequential_scan_real_forward_abs_raw_block_f (:1531), reached
 * from rqf_models/ops/scan.py:sequential_scan_abs (:381-432).  y_abs is
 * float32 (B,T,F); no carries are saved (there is no backward); scratch as
 * rqf_btf_scratch_bytes. */
int rqf_chunked_scan_abs_forward(const float *c1, const float *c2, const void *u,
                                 int u_is_real, float *y_abs, void *scratch,
                                 int64_t batch, int64_t time, int64_t filters,
                                 int path, rqf_stream_t stream);

/* Replaces chunked_scan_kernel.py:_chunked_scan_backward_raw (:252) /
 * _chunked_scan_backward_kernel (:122): g[t] = gy[t] + conj(c1) g[t+1];
 * grad_u = conj(c2) g (real part only when u_is_real);
 * grad_c1 = sum conj(y[t-1]) g[t];  grad_c2 = sum conj(u[t]) g[t].
 * y[t-1] is recomputed from `carries`; grad_c1/grad_c2 are overwritten. */
int rqf_chunked_scan_backward(const float *c1, const float *c2, const void *u,
                              int u_is_real, const float *carries,
                              const float *grad_y, void *grad_u, float *grad_c1,
                              float *grad_c2, void *scratch, int64_t batch,
                              int64_t time, int64_t filters, int path,
                              rqf_stream_t stream);

/* ---- multi-oscillator scan with C-weight reduction, (B,T,F) layout --- *
 * Replaces rqf_models/ops/triton_scan_kernel.py:_triton_sequential_scan_multi_osc
 * (:2499; forward _sequential_scan_multi_osc_forward_raw :1935, backward
 * _sequential_scan_multi_osc_backward_raw :2280), its real-input and
 * parallel variants (:3071, :4106) and magnitude epilogues (:2019, :2688),
 * reached from rqf_models/backbones/rqf/block.py:_scan_standard_multi_osc
 * (:737):
 *   x_s[t] = c1_s x_s[t-1] + c2_s u[t, s / n],   s < filters * n,
 *   out[t, f] = sum_{k<n} cw_{f n + k} x_{f n + k}[t],
 * n = num_osc (a power of two <= 32, else RQF_ERR_SHAPE).  c1, c2, cw are
 * complex (filters * n); u is complex, or float32 with u_is_real,
 * (B,T,filters); out is complex (B,T,filters), or float32 |out| with out_abs
 * (then carries may be null: nothing is saved).  Size carries and scratch
 * with rqf_multi_osc_carry_count / _scratch_bytes. */
int rqf_multi_osc_forward(const float *c1, const float *c2, const float *cw,
                          const void *u, int u_is_real, void *out, int out_abs,
                          float *carries, void *scratch, int64_t batch,
                          int64_t time, int64_t filters, int64_t num_osc,
                          rqf_stream_t stream);

/* g_s[t] = conj(c1_s) g_s[t+1] + conj(cw_s) grad_out[t, f];
 * grad_u[t, f] = sum_k conj(c2_s) g_s[t] (its real part when u_is_real);
 * grad_c1_s = sum conj(x_s[t-1]) g_s[t], grad_c2_s = sum conj(u[t, f]) g_s[t],
 * grad_cw_s = sum conj(x_s[t]) grad_out[t, f] (complex: the reference's real
 * (filters*n, 2) C-weight gradient is its real view).  The three coefficient
 * gradients are overwritten. */
int rqf_multi_osc_backward(const float *c1, const float *c2, const float *cw,
                           const void *u, int u_is_real, const float *carries,
                           const float *grad_out, void *grad_u, float *grad_c1,
                           float *grad_c2, float *grad_cw, void *scratch,
                           int64_t batch, int64_t time, int64_t filters,
                           int64_t num_osc, rqf_stream_t stream);
int64_t rqf_multi_osc_carry_count(int64_t batch, int64_t time, int64_t filters,
                                  int64_t num_osc);
size_t rqf_multi_osc_scratch_bytes(int64_t batch, int64_t time, int64_t filters,
                                   int64_t num_osc);

/* ---- two-tap prospective scan, (B,T,F) layout ------------------------ *
 * Replaces chunked_scan_kernel.py:_chunked_prospective_forward_raw (:442) /
 * _chunked_prospective_kernel (:374):
 *   y[t] = c1*y[t-1] + tap0*x[t] + tap1*x[t-1],  x[-1] = 0. */
int rqf_chunked_prospective_forward(const float *c1, const float *tap0,
                                    const float *tap1, const float *x, float *y,
                                    float *carries, void *scratch,
                                    int64_t batch, int64_t time,
                                    int64_t filters, int path, rqf_stream_t stream);

/* Replaces _ChunkedProspectiveScanFunction.backward
 * (chunked_scan_kernel.py:489-503), fused into one kernel:
 *   grad_x[t] = conj(tap0) g[t] + conj(tap1) g[t+1];  grad_c1, grad_tap0,
 *   grad_tap1 = sums of conj(y[t-1]) g, conj(x[t]) g, conj(x[t-1]) g. */
int rqf_chunked_prospective_backward(
    const float *c1, const float *tap0, const float *tap1, const float *x,
    const float *carries, const float *grad_y, float *grad_x, float *grad_c1,
    float *grad_tap0, float *grad_tap1, void *scratch, int64_t batch,
    int64_t time, int64_t filters, int path, rqf_stream_t stream);

/* ---- two-tap prospective scan, (F,B,T) layout ------------------------ *
 * Replaces fbt_scan_kernel.py:_fbt_prospective_kernel (:34) and
 * _fbt_recompute_forward_kernel (:360).  Writes split-ReLU(y) when
 * fuse_act != 0 (relu(Re y) + i relu(Im y)), else the raw state y. */
int rqf_fbt_prospective_forward(const float *c1, const float *tap0,
                                const float *tap1, const float *z, float *out,
                                float *carries, void *scratch, int64_t filters,
                                int64_t batch, int64_t time, int fuse_act,
                                rqf_stream_t stream);

/* Pure RQF block forward with the complex skip connection fused:
 *   out = act(y) + skip  (rqf_models/backbones/rqf/pure.py:_forward_fbt_stack
 *   :535, h = out + h), y the two-tap scan above.  skip may be NULL (then this
 *   is rqf_fbt_prospective_forward).  The backward is
 *   rqf_fbt_prospective_backward on the output cotangent; the skip's
 *   cotangent is that same cotangent. */
int rqf_fbt_block_forward(const float *c1, const float *tap0, const float *tap1,
                          const float *z, const float *skip, float *out, float *carries,
                          void *scratch, int64_t filters, int64_t batch, int64_t time,
                          int fuse_act, rqf_stream_t stream);

/* Replaces fbt_scan_kernel.py:_fbt_prospective_backward_kernel (:113) and
 * _fbt_recompute_backward_kernel (:439).  grad_out is the cotangent of the
 * forward's output (of the split-ReLU output when fuse_act != 0; the mask is
 * sign(y) > 0 per component, recomputed).  Writes grad_z and overwrites
 * grad_c1 / grad_tap0 / grad_tap1 (complex (F,)). */
int rqf_fbt_prospective_backward(const float *c1, const float *tap0,
                                 const float *tap1, const float *z,
                                 const float *carries, const float *grad_out,
                                 float *grad_z, float *grad_c1,
                                 float *grad_tap0, float *grad_tap1,
                                 void *scratch, int64_t filters, int64_t batch,
                                 int64_t time, int fuse_act,
                                 rqf_stream_t stream);

/* ---- first block over a rank-1 input ---------------------------------- *
 * The first Pure RQF block when the input projection has one channel
 * (pure.py:_forward_fbt_stack :510-534 with input_dims = 1, the waveform
 * models): its drive z = u x + beta (u = W w_in, beta = W b_in) and skip
 * h0 = w x + bb (w = w_in, bb = b_in) are made inside the (F,B,T) row scan
 * from x (batch, time) float32 instead of being read from HBM.  The forward
 * equals rqf_lowrank_drive followed by rqf_fbt_block_forward on its z and h0
 * (the same operations), writes out = act(y) (+ h0) and the (F,B,T) saved
 * context.  The backward replays from that context and, instead of grad_z,
 * returns its row sums gzx = [sum gz x, sum gz] and gsx = [sum g x, sum g]
 * (complex (F, 2), over batch and time; gsx nullable; the plain sums only
 * with with_sum), which is what the block's weight and input-projection
 * cotangents need (rqf_rowdot of grad_z and of the output cotangent).
 * beta, w, bb nullable (no w: no skip).  Both need the persistent row
 * kernels and T a multiple of 4: rqf_fbt_rank1_supported; otherwise
 * RQF_ERR_SHAPE. */
int rqf_fbt_rank1_supported(int64_t filters, int64_t batch, int64_t time);
size_t rqf_fbt_rank1_scratch_bytes(int64_t filters, int64_t batch, int64_t time);
int rqf_fbt_rank1_forward(const float *u, const float *beta, const float *w, const float *bb,
                          const float *x, const float *c1, const float *tap0, const float *tap1,
                          float *out, float *carries, int64_t filters, int64_t batch,
                          int64_t time, int fuse_act, rqf_stream_t stream);
int rqf_fbt_rank1_backward(const float *u, const float *beta, const float *x, const float *c1,
                           const float *tap0, const float *tap1, const float *carries,
                           const float *grad_out, float *gzx, float *gsx, float *grad_c1,
                           float *grad_tap0, float *grad_tap1, void *scratch, int64_t filters,
                           int64_t batch, int64_t time, int fuse_act, int with_sum,
                           rqf_stream_t stream);
/* The TBPTT(1) surrogate of the same block (the gradients of
 * rqf_fbt_tbptt1_backward_wsum, rqf_models/backbones/rqf/pure.py:184-187 with
 * the lag source the same projection as z): no adjoint recursion, d = the
 * masked output cotangent, grad_z = conj(tap0) d, the lag cotangent
 * conj(tap1) d[t+1].  gzx = [sum gz x, sum gz] (the input projection's
 * term), gwx = [sum gsum x, sum gsum] with gsum = grad_z + the lag cotangent
 * (the weight cotangent's), gsx = [sum g x, sum g] (nullable); the plain
 * sums only with with_sum.  Same context, shapes and errors as
 * rqf_fbt_rank1_backward. */
int rqf_fbt_rank1_tbptt_backward(const float *u, const float *beta, const float *x,
                                 const float *c1, const float *tap0, const float *tap1,
                                 const float *carries, const float *grad_out, float *gzx,
                                 float *gwx, float *gsx, float *grad_c1, float *grad_tap0,
                                 float *grad_tap1, void *scratch, int64_t filters, int64_t batch,
                                 int64_t time, int fuse_act, int with_sum, rqf_stream_t stream);

/* ---- TBPTT(1) two-tap surrogate backward ----------------------------- *
 * The forward value of the reference's TBPTT(1) path equals the exact scan
 * (rqf_models/backbones/rqf/block.py:_scan_two_tap_with_grad_mode :904-954),
 * so the forward is rqf_chunked_prospective_forward (layout 0, BTF) or
 * rqf_fbt_prospective_forward (layout 1, FBT).  This replaces the pointwise
 * autograd of the one-step rebuild  C1*h[t-1].detach() + tap0*z[t] +
 * tap1*zw[t-1]  (block.py:946-954) with one kernel, no temporal scan:
 *   g        = grad_out (masked by split-ReLU'(y) when fuse_act; layout 1
 *              only: the BTF forward has no fused activation, so layout 0
 *              with fuse_act returns RQF_ERR_ARGUMENT)
 *   grad_z   = conj(tap0) g[t]
 *   grad_zw  = conj(tap1) g[t+1]  (cotangent of the lag source zw = z values)
 *   grad_c1  = sum conj(y[t-1]) g[t], grad_tap0 = sum conj(z[t]) g[t],
 *   grad_tap1 = sum conj(z[t-1]) g[t].
 * dims = {batch, time, filters} for layout 0, {filters, batch, time} for 1;
 * path as the (B,T,F) forward's (layout 0; ignored for layout 1). */
int rqf_tbptt1_two_tap_backward(int layout, const float *c1, const float *tap0,
                                const float *tap1, const float *z,
                                const float *carries, const float *grad_out,
                                float *grad_z, float *grad_zw, float *grad_c1,
                                float *grad_tap0, float *grad_tap1,
                                void *scratch, int64_t d0, int64_t d1,
                                int64_t d2, int fuse_act, int path,
                                rqf_stream_t stream);
/* The same (F,B,T) backward writing grad_zsum = grad_z + grad_zw in place of
 * grad_zw: the operand of the weight cotangent when both taps come from one
 * projection (the lag source zw is the same W h as z, pure.py:184-187, so
 * grad W = (grad_z + grad_zw) h^H), which saves the caller an element-wise
 * pass.  grad_z is still written (the input cotangent W^H grad_z needs it). */
int rqf_fbt_tbptt1_backward_wsum(const float *c1, const float *tap0, const float *tap1,
                                 const float *z, const float *carries, const float *grad_out,
                                 float *grad_z, float *grad_zsum, float *grad_c1,
                                 float *grad_tap0, float *grad_tap1, void *scratch,
                                 int64_t filters, int64_t batch, int64_t time, int fuse_act,
                                 rqf_stream_t stream);

/* ---- selective (input-dependent ZOH) scan, (F,B,T) layout ------------ *
 * Replaces rqf_models/ops/selective_scan_kernel.py:selective_forward (:491) /
 * _forward (:155) and selective_backward (:517) / _backward (:250) /
 * _group_reduce (:465).  The options mirror the reference's 12-tuple
 * (rqf_models/backbones/rqf/selective.py:249-262); the inputs mirror
 * SelectiveScanInputs (rqf_models/ops/selective_scan.py:10-23). */
typedef struct {
  int has_gamma, has_warp, has_write, log_shift;
  float gamma_scale, warp_scale;
  int prospective, gamma_horizon, write_sigmoid;
  float write_max, write_bias;
  int bound_warp;
} rqf_selective_options;

typedef struct {
  const float *gamma_logits; /* (F,B,T), or NULL without gamma control */
  const float *warp_logits;  /* (num_groups,B,T), or NULL without warp  */
  const float *write_logits; /* (F,B,T), or NULL without write control */
  const float *bias, *theta; /* (F,) */
  const int64_t *groups;     /* (F,) warp group per channel, or NULL  */
  const float *minimum, *span, *step, *horizon, *theta_minimum, *theta_maximum; /* (F,) */
  int64_t num_groups;
} rqf_selective_inputs;

int64_t rqf_selective_num_tiles(int64_t time);
int64_t rqf_selective_carry_count(int64_t filters, int64_t batch, int64_t time);
size_t rqf_selective_scratch_bytes(int64_t filters, int64_t batch, int64_t time, int has_warp);

/* Writes raw (may be NULL) and split-ReLU(raw) `act` (may be NULL) as
 * complex (F,B,T), and the per-tile entry states into `carries`. */
int rqf_selective_forward(const float *z, const rqf_selective_inputs *inputs,
                          const rqf_selective_options *options, float *raw, float *act,
                          float *carries, int64_t filters, int64_t batch, int64_t time,
                          rqf_stream_t stream);

/* grad_raw / grad_act: cotangents of raw and act (either may be NULL).
 * Outputs as selective_backward: dz (total drive cotangent in full BPTT, the
 * spatial part in TBPTT(1)), dzw (TBPTT(1) only: total, for the weight; may
 * be NULL otherwise), dgamma (F,B,T) / dwarp (num_groups,B,T) / dwrite (F,B,T)
 * logit cotangents (NULL when the controller is off), dbias / dtheta (F,). */
int rqf_selective_backward(const float *z, const rqf_selective_inputs *inputs,
                           const rqf_selective_options *options, const float *carries,
                           const float *grad_raw, const float *grad_act, int truncated,
                           float *dz, float *dzw, float *dgamma, float *dwarp, float *dwrite,
                           float *dbias, float *dtheta, void *scratch, int64_t filters,
                           int64_t batch, int64_t time, rqf_stream_t stream);

/* ---- selective scan, bf16 storage mode -------------------------------- *
 * No counterpart in the reference, whose selective kernel requires fp32
 * logits and complex64 activations (rqf_models/ops/selective_scan.py:187-198):
 * the storage mode of the selective benchmark configuration ("bf16
 * activations, fp32 complex state").  Same arguments and arithmetic as rqf_selective_forward /
 * _backward, except that the three logit pointers of `inputs` address bf16
 * (2-byte) elements, raw / act are written as interleaved bf16 pairs
 * (F,B,T,2), and the logit cotangents dgamma / dwarp / dwrite are written in
 * bf16.  z, the carries, the output cotangents, dz / dzw and dbias / dtheta
 * stay fp32, and so does every value inside the kernels (bf16 inputs are
 * widened exactly; outputs are rounded to nearest-even once). */
int rqf_selective_forward_bf16(const float *z, const rqf_selective_inputs *inputs,
                               const rqf_selective_options *options, void *raw, void *act,
                               float *carries, int64_t filters, int64_t batch, int64_t time,
                               rqf_stream_t stream);
int rqf_selective_backward_bf16(const float *z, const rqf_selective_inputs *inputs,
                                const rqf_selective_options *options, const float *carries,
                                const float *grad_raw, const float *grad_act, int truncated,
                                float *dz, float *dzw, void *dgamma, void *dwarp, void *dwrite,
                                float *dbias, float *dtheta, void *scratch, int64_t filters,
                                int64_t batch, int64_t time, rqf_stream_t stream);

/* ---- allocation-free variant of rqf_fbt_prospective_backward --------- *
 * No counterpart in the reference.  For callers that cannot allocate device
 * memory — e.g. code running inside a framework allocator's callback, a
 * real-time loop that forbids cudaMalloc after start-up, or a host language
 * binding that only hands over tensors it already owns — so they cannot
 * provide the `scratch` buffer the other backward entry point needs.
 *
 * Same arguments and results as rqf_fbt_prospective_backward without
 * `scratch`: the scratch lives in a fixed 4 MiB __device__ array inside this
 * library (every GPU that loads the library holds it until process exit).
 * Shapes are validated first (RQF_ERR_SHAPE, as the regular entry point);
 * valid shapes whose scratch (rqf_fbt_scratch_bytes) exceeds 4 MiB are
 * rejected with RQF_ERR_CAPACITY.  The first call on a device looks up the array's
 * device address on that device (cudaGetSymbolAddress, once per device), so
 * make the first call on each device outside any stream capture.  The cached
 * address lives as long as the device's context: a process that calls
 * cudaDeviceReset on a device after using this entry point there must not
 * call it on that device again.  All calls
 * share the one array and it keeps the last call's contents (the part that
 * must start at zero is cleared on every call), so calls whose GPU work
 * overlaps — on different streams, or from different host threads without
 * ordering — race on it and must be serialised by the caller.  Allocates
 * nothing: no cudaMalloc, cudaFree or allocating library routine. */
int rqf_fbt_prospective_backward_noalloc(const float *c1, const float *tap0, const float *tap1,
                                         const float *z, const float *carries,
                                         const float *grad_out, float *grad_z, float *grad_c1,
                                         float *grad_tap0, float *grad_tap1, int64_t filters,
                                         int64_t batch, int64_t time, int fuse_act,
                                         rqf_stream_t stream);

/* ---- complex projection GEMM of the Pure RQF block (tensor cores) ---- *
 * Replaces the complex GEMM torch.matmul(W, h.reshape(d_model, batch*time))
 * of rqf_models/backbones/rqf/pure.py:223 (PureRQFBlock._forward_fbt) and its
 * input cotangent W^H gz (autograd of the same matmul; the reference runs both
 * as cuBLAS fp32 complex GEMMs):
 *
 *   out[j, n] = sum_k op(W)[j, k] * x[k, n]  (+ acc[j, n])        complex64
 *
 * conj_transpose = 0: op(W) = W with W (m x k);  = 1: op(W) = W^H with W
 * (k x m).  x is (k x n) with n contiguous ((F,B,T) activations, n = B*T);
 * out and acc (nullable; may alias out) are (m x n).  Arithmetic: split TF32
 * on the tensor cores (each fp32 operand split into two TF32 parts, three
 * TF32 products per fp32 product, fp32 accumulation), fp32-comparable.
 * Requirements: n even, x / out / acc 16-byte aligned, n < 2^30.
 * `workspace` needs rqf_projection_workspace_bytes(m, k) bytes (16-byte
 * aligned); it holds the split copy of op(W) and is free again when the
 * launch completes.  The pipeline's waits are bounded: on expiry the kernel
 * latches RQF_ERR_PIPELINE_TIMEOUT in the device error word. */
size_t rqf_projection_workspace_bytes(int64_t m, int64_t k);
/* Diagnostic: where the first expired wait of the projection pipeline gave
 * up since the last clear (0 none, 1 producer, 2 transform, 3/4 MMA issuer,
 * 5 epilogue, 6 shutdown drain, 7 block-scan link record, 8 block-scan
 * backward ring load); -1 on a CUDA error.  Synchronous. */
int rqf_projection_timeout_site(int clear);
int rqf_projection(const float *w, const float *x, const float *acc, float *out, int64_t m,
                   int64_t k, int64_t n, int conj_transpose, void *workspace,
                   rqf_stream_t stream);

/* Pure RQF block forward in one launch: the projection of pure.py:223 with
 * the block's scan, activation and skip connection (pure.py:529-535) run in
 * the GEMM's epilogue, tile by tile, while the tensor cores work on the next
 * tile.  Equal to rqf_projection (conj_transpose = 0, acc = NULL) into z
 * followed by rqf_fbt_block_forward(c1, tap0, tap1, z, skip, out, carries):
 *
 *   z   = W x                       complex (filters, batch*time), written
 *   out = act(y) + skip             y the two-tap scan of z along time
 *   carries                         every 8-sample group's entry state, the
 *                                   saved context of the (F,B,T) row kernels
 *
 * so rqf_fbt_prospective_backward and rqf_tbptt1_two_tap_backward (layout 1)
 * take its z and carries unchanged.  W is (filters x k), x (k x batch*time)
 * with time contiguous, skip (nullable) and out (filters, batch, time);
 * carries holds rqf_fbt_carry_count(filters, batch, time) complex values.
 * The scan's state crosses the GEMM's 128-sample tiles through link records
 * in the workspace (rqf_projection_block_scan_workspace_bytes; 0 for shapes
 * this entry rejects): every tile waits, bounded, for the tile before it.
 * Requirements: time a multiple of 128, batch * time < 2^30, k > 0, x / z /
 * out / skip / carries / workspace 16-byte aligned, out distinct from x, z
 * and skip, z distinct from x and skip (RQF_ERR_ARGUMENT). */
size_t rqf_projection_block_scan_workspace_bytes(int64_t filters, int64_t k, int64_t batch,
                                                 int64_t time);
int rqf_projection_block_scan(const float *w, const float *x, const float *c1, const float *tap0,
                              const float *tap1, const float *skip, float *z, float *out,
                              float *carries, void *workspace, int64_t filters, int64_t k,
                              int64_t batch, int64_t time, int fuse_act, rqf_stream_t stream);

/* The backward of two stacked Pure RQF blocks meeting at one launch: the
 * input cotangent of the upper block's projection (autograd of pure.py:223)
 * with the lower block's scan VJP (fbt_scan_kernel.py:_FBTRecompute /
 * _FBTProspectiveScan backward, :575-689 and :245-329) run in the GEMM's
 * epilogue, tile by tile from the end of each batch row.  Equal to
 * rqf_projection(w, gz_above, acc, grad_out, conj_transpose = 1) followed by
 * rqf_fbt_prospective_backward(c1, tap0, tap1, z, carries, grad_out):
 *
 *   grad_out = W^H gz_above + acc        the lower block's output cotangent
 *   grad_z, grad_c1, grad_tap0, grad_tap1   the lower block's scan VJP of it
 *
 * W is (k x filters), the upper block's weight; gz_above (k, batch, time)
 * its z cotangent; acc (nullable) the skip's cotangent (filters, batch,
 * time); c1 / tap0 / tap1, z and carries the lower block's coefficients and
 * saved context from any (F,B,T) forward of this library (each saves every
 * 8-sample group's entry state and the marker after them; a context without
 * the marker latches RQF_ERR_ARGUMENT in the device error word).
 * The coefficient gradients are summed per (row, tile) in the workspace and
 * reduced in a fixed order in double.  Requirements as for
 * rqf_projection_block_scan; the outputs distinct from every input. */
size_t rqf_projection_block_scan_backward_workspace_bytes(int64_t filters, int64_t k,
                                                          int64_t batch, int64_t time);
int rqf_projection_block_scan_backward(const float *w, const float *gz_above, const float *acc,
                                       const float *c1, const float *tap0, const float *tap1,
                                       const float *z, const float *carries, float *grad_out,
                                       float *grad_z, float *grad_c1, float *grad_tap0,
                                       float *grad_tap1, void *workspace, int64_t filters,
                                       int64_t k, int64_t batch, int64_t time, int fuse_act,
                                       rqf_stream_t stream);

/* Weight cotangent of the same projection (autograd of pure.py:223's matmul
 * with respect to W; cuBLAS fp32 in the reference):
 *
 *   gw[j, i] = sum_n gz[j, n] * conj(x[i, n])                      complex64
 *
 * gz (m x n) and x (k x n) with n contiguous; gw (m x k).  Split TF32 on the
 * tensor cores, the n reduction split over CTAs and the fp32 partial tiles
 * summed in a fixed order (deterministic).  Requirements as rqf_projection;
 * `workspace` needs rqf_projection_weight_grad_workspace_bytes(m, k, n) bytes
 * on the current device (the split count follows its SM count). */
size_t rqf_projection_weight_grad_workspace_bytes(int64_t m, int64_t k, int64_t n);
int rqf_projection_weight_grad(const float *gz, const float *x, float *gw, int64_t m, int64_t k,
                               int64_t n, void *workspace, rqf_stream_t stream);

/* The same two GEMMs with a real left operand, for the readout's hidden layer
 * (train.py:ComplexReadoutClassifier :74-136: Linear(2F, H) on [Re h; Im h],
 * whose cotangent g is real): x (k x n) real in rqf_projection_real,
 *
 *   out[j, n] = sum_k op(W)[j, k] * x[k, n] (+ acc[j, n])          complex64
 *
 * and gz (m x n) real in rqf_projection_weight_grad_real,
 *
 *   gw[j, i] = sum_n gz[j, n] * conj(x[i, n])                      complex64.
 *
 * Half the tensor-core work of the complex forms, which would multiply the
 * zero imaginary parts.  n must be a multiple of 4 (the real rows' TMA
 * pitch); the rest as rqf_projection / rqf_projection_weight_grad, with
 * workspace sizes from rqf_projection_workspace_bytes and
 * rqf_projection_weight_grad_real_workspace_bytes. */
int rqf_projection_real(const float *w, const float *x, const float *acc, float *out, int64_t m,
                        int64_t k, int64_t n, int conj_transpose, void *workspace,
                        rqf_stream_t stream);
size_t rqf_projection_weight_grad_real_workspace_bytes(int64_t m, int64_t k, int64_t n);
int rqf_projection_weight_grad_real(const float *gz, const float *x, float *gw, int64_t m,
                                    int64_t k, int64_t n, void *workspace, rqf_stream_t stream);

/* The readout hidden layer's forward GEMM, W1 [Re x; Im x] = Re(W x) with W
 * = W1[:, :F] - i W1[:, F:] (train.py:ComplexReadoutClassifier :126-136):
 *
 *   out[j, n] = Re sum_k w[j, k] * x[k, n]                          float32 (m x n)
 *
 * w (m x k) and x (k x n) complex64.  x is split into its Re and Im planes in
 * shared memory, so the tensor cores do the real product only (half the work
 * of rqf_projection, whose imaginary part the readout discards).  n a
 * multiple of 4; `workspace` needs rqf_projection_real_out_workspace_bytes(m,
 * k) bytes. */
size_t rqf_projection_real_out_workspace_bytes(int64_t m, int64_t k);
int rqf_projection_real_out(const float *w, const float *x, float *out, int64_t m, int64_t k,
                            int64_t n, void *workspace, rqf_stream_t stream);

/* First block over a low-rank input projection (pure.py:_forward_fbt_stack
 * :522-534: proj = w_in @ x_cf (+ b_in), h = proj.to(complex64), then the
 * first block's z = W @ h).  With I = input_dims <= 4:
 *
 *   z[f, n] = sum_i u[f, i] x[i, n] + beta[f]        complex64, (F, N)
 *   h[f, n] = sum_i w_in[f, i] x[i, n] + b_in[f]     complex64, imaginary 0
 *
 * u = W w_in (F x I complex), beta = W b_in (F complex); x (I x N) real with
 * N contiguous and even.  beta, b_in and h may be null (h null: z only).
 * One HBM-bound pass replaces the F x F projection GEMM of the first block.
 * z and h 16-byte aligned, x 8-byte aligned. */
int rqf_lowrank_drive(const float *u, const float *beta, const float *w_in, const float *b_in,
                      const float *x, float *z, float *h, int64_t f, int64_t n, int i,
                      rqf_stream_t stream);

/* Row dots of a complex (F x N) matrix against I <= 4 real rows, for the
 * first block's cotangents (gW = (gz x^T) w_in^T, grad w_in = Re(W^H (gz x^T)
 * + g x^T), and the bias terms from the row sums):
 *
 *   out[f, j] = sum_n a[f, n] x[j, n]   (j < I);   out[f, I] = sum_n a[f, n]  (with_sum)
 *
 * out complex (F x (I + with_sum)).  Fixed-order reduction (per-chunk partials
 * in double, summed in chunk order): deterministic.  `workspace` needs
 * rqf_rowdot_workspace_bytes(f, n, i, with_sum) bytes.  a 16-byte aligned, x
 * 8-byte aligned, N even, F <= 65535. */
size_t rqf_rowdot_workspace_bytes(int64_t f, int64_t n, int i, int with_sum);
int rqf_rowdot(const float *a, const float *x, float *out, void *workspace, int64_t f, int64_t n,
               int i, int with_sum, rqf_stream_t stream);

/* Hidden layer of the mean-pooled readout (train.py:ComplexReadoutClassifier
 * :74-136, Linear -> ReLU per step, logits mean-pooled over time), given the
 * real part Re z (float32, H x B x T, T contiguous) of the projection of the
 * encoder state (rqf_projection_real_out):
 *
 *   pooled[h, b] = (1/T) sum_t relu(Re z[h, b, t] + bias[h])      float32 (H x B)
 *   mask[(h B + b) W + t/32] bit t%32 = (Re z + bias > 0),  W = ceil(T/32)
 *
 * bias may be null.  One pass over Re z; fixed-order reduction. */
int rqf_readout_relu_pool(const float *z, const float *bias, uint32_t *mask, float *pooled,
                          int64_t h, int64_t batch, int64_t time, rqf_stream_t stream);
/* Its backward: g[h, b, t] = mask ? scale[h, b] : 0 (float32, the real
 * input of rqf_projection_real and rqf_projection_weight_grad_real; scale =
 * gpool / T) and counts[h, b] = number of set mask bits (float32; may be
 * null). */
int rqf_readout_relu_pool_backward(const uint32_t *mask, const float *scale, float *gc,
                                   float *counts, int64_t h, int64_t batch, int64_t time,
                                   rqf_stream_t stream);

/* The per-step readout's hidden layer (train.py:ComplexReadoutClassifier
 * :74-136, Linear -> ReLU at every step, for per-step logits): in place on
 * the real part z (float32, H x B x T, T contiguous) of the projection,
 * z = relu(z + bias[h]) and the mask bits of rqf_readout_relu_pool (bias may
 * be null).  Its backward: g = mask ? gy : 0 (float32, like gy) and
 * rowsum[h, b] = sum_t g (nullable; in double, fixed order), the bias's
 * cotangent before the sum over the batch. */
int rqf_readout_bias_relu(float *z, const float *bias, uint32_t *mask, int64_t h, int64_t batch,
                          int64_t time, rqf_stream_t stream);
int rqf_readout_bias_relu_backward(const float *gy, const uint32_t *mask, float *g, float *rowsum,
                                   int64_t h, int64_t batch, int64_t time, rqf_stream_t stream);

/* The per-timestep classification loss of the TBPTT(1) recipe
 * (train.py:per_step_cross_entropy :663-674: cross_entropy over the
 * (batch*time, classes) view, batch row b's label for each of its time
 * steps, label smoothing, mean), on the logits as the readout's output GEMM
 * writes them: float32 (classes, batch*time), sample b*time + t.  labels
 * int64 (batch), each in [0, classes) (else RQF_ERR_ARGUMENT is latched for
 * rqf_read_device_error and class 0 used).  loss: one float32; the sum is
 * taken per block in double and then over blocks in a fixed order.
 * `scratch` needs rqf_per_step_cross_entropy_scratch_bytes (8-byte aligned).
 * The backward writes grad_logits (classes, batch*time) for the upstream
 * gradient *grad_loss (a device scalar): (softmax - (1 - eps) onehot(y) -
 * eps / classes) * grad_loss / (batch*time). */
size_t rqf_per_step_cross_entropy_scratch_bytes(int64_t batch, int64_t time);
int rqf_per_step_cross_entropy(const float *logits, const int64_t *labels, float *loss,
                               void *scratch, int64_t classes, int64_t batch, int64_t time,
                               float label_smoothing, rqf_stream_t stream);
int rqf_per_step_cross_entropy_backward(const float *logits, const int64_t *labels,
                                        const float *grad_loss, float *grad_logits,
                                        int64_t classes, int64_t batch, int64_t time,
                                        float label_smoothing, rqf_stream_t stream);

/* ---- RQF filter-bank coefficients (rqf_models/backbones/rqf/filter.py) -- *
 * Replaces RQF.compute_two_tap_coefficients (filter.py:510-664) with the
 * parameter reads it makes (the tau / gamma / freq properties, :402-449):
 * every discretization that has a two-tap form (Euler and ZOH prospective,
 * FOH prospective and not), tau mode (rho = 1), gamma mode (rho = 1/gamma),
 * an explicit prospective_tau (rho = tau_p / tau), the dynamic gamma clamp
 * (clamp_gamma, :594-598), and both leaf parametrizations:
 *
 *   log space     (param_space 0): theta_leaf = log_theta, gamma_leaf = log_gamma,
 *                                  gamma = e^gamma_leaf, freq = e^theta_leaf / (2 pi tau)
 *   sigmoid space (param_space 1): theta_leaf = freq_param, gamma_leaf = gamma_param,
 *                                  gamma = min_gamma + (max_gamma - min_gamma) sig(gamma_leaf),
 *                                  freq = min_freq + (max_freq - min_freq) sig(theta_leaf)
 *
 * tau = e^log_tau per filter (log_tau may be NULL: the scalar opts->tau).
 * Outputs c1, tap0, tap1 complex64 (n,) — Euler's real taps with zero
 * imaginary parts; computed in double from the fp32 leaves.  phi = (e^a-1)/a
 * and psi = (e^a-1-a)/a^2 take the reference's 4th-order Taylor forms below
 * |a| = 1e-4 and 1e-3.  bilinear has no two-tap form, and Euler / ZOH without
 * prospective input are single-tap (RQF_ERR_ARGUMENT, as the reference raises).
 *
 * The backward takes complex cotangents (each may be NULL) and writes the
 * real gradients of the leaves it is given outputs for (each may be NULL):
 * grad p = sum over outputs of Re(conj(d out / d p) * grad_out), through every
 * branch above (the clamp's derivative follows the selected operand, as
 * torch.clamp's does). */
enum { RQF_DISC_EULER = 0, RQF_DISC_ZOH = 1, RQF_DISC_FOH = 2 };

typedef struct {
  const float *theta_leaf;      /* log_theta or freq_param, (n,)           */
  const float *gamma_leaf;      /* log_gamma or gamma_param, (n,)          */
  const float *log_tau;         /* (n,) or NULL                            */
  const float *min_gamma, *max_gamma, *min_freq, *max_freq; /* sigmoid (n,) */
  const float *prospective_tau; /* (n,) seconds, or NULL (mode decides rho) */
} rqf_coeff_leaves;

typedef struct {
  int discretization; /* RQF_DISC_*                                       */
  int prospective;    /* 1: prospective taps; 0: FOH non-prospective taps */
  int gamma_mode;     /* 0: tau mode; 1: gamma mode (ignored with tau_p)  */
  int param_space;    /* 0: log leaves; 1: sigmoid leaves                 */
  int clamp_gamma;
  double dt;
  double tau;         /* used when leaves->log_tau is NULL                */
} rqf_coeff_options;

int rqf_filter_two_tap_coefficients(const rqf_coeff_leaves *leaves, const rqf_coeff_options *opts,
                                    float *c1, float *tap0, float *tap1, int64_t n,
                                    rqf_stream_t stream);
int rqf_filter_two_tap_coefficients_backward(const rqf_coeff_leaves *leaves,
                                             const rqf_coeff_options *opts, const float *grad_c1,
                                             const float *grad_tap0, const float *grad_tap1,
                                             float *grad_theta_leaf, float *grad_gamma_leaf,
                                             float *grad_log_tau, float *grad_prospective_tau,
                                             int64_t n, rqf_stream_t stream);

/* The log-space ZOH tau-mode case with one scalar tau (the Pure RQF paper
 * recipe, and this backend's encoder): the general producer with
 * {RQF_DISC_ZOH, prospective, tau mode, log space, no clamp}:
 *
 *   a = (dt/tau) (-gamma + i theta (1 - gamma)),  gamma = e^lg, theta = e^lt
 *   c1 = e^a,  tap0 = gamma ((dt/tau) (e^a - 1)/a + c1),  tap1 = -gamma c1 */
int rqf_two_tap_coefficients(const float *log_theta, const float *log_gamma, float *c1, float *tap0,
                             float *tap1, int64_t n, double dt, double tau, rqf_stream_t stream);
int rqf_two_tap_coefficients_backward(const float *log_theta, const float *log_gamma,
                                      const float *grad_c1, const float *grad_tap0,
                                      const float *grad_tap1, float *grad_log_theta,
                                      float *grad_log_gamma, int64_t n, double dt, double tau,
                                      rqf_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* RQF_B200_H */
