/*
 * hdcmamba_b200 -- C ABI of the B200 (sm_100a) kernels for HdcMamba-9v3's layer forward.
 *
 * Every entry point takes plain device pointers, element strides and sizes, and
 * a cudaStream_t; none allocates device memory.  Kernels are launched
 * asynchronously on `stream`.  Return value: 0 on success, a negative HDC_E*
 * code for a rejected argument (nothing launched), or a positive cudaError_t
 * from the launch.  hdc_error_string() describes the last error of the calling
 * thread.
 *
 * dtype codes: HDC_F32 (fp32 activations) or HDC_BF16 (bf16 activations).
 * Unless stated otherwise, activations are in `dtype`, norm/conv/gn parameters
 * in `dtype`, and decay / state tensors in fp32.
 *
 * Each declaration names the reference code it replaces (N01N9/hdcmamba,
 * file:line).  The reference is Python + Triton; its "FFI" for this path is the
 * Triton launch `kernel[grid](...)`, so the arguments below follow those
 * launches' pointer / stride / size arguments.
 */
#ifndef HDCMAMBA_B200_H
#define HDCMAMBA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* hdc_stream_t; /* == cudaStream_t */

enum { HDC_F32 = 0, HDC_BF16 = 1 };
enum { HDC_ACT_NONE = 0, HDC_ACT_SILU = 1 };
enum {
  HDC_OK = 0,
  HDC_E_DTYPE = -1,    /* unsupported dtype code */
  HDC_E_SHAPE = -2,    /* a size is out of the supported range */
  HDC_E_ALIGN = -3,    /* a pointer / stride breaks the 16-byte vector rule */
  HDC_E_NULL = -4,     /* a required pointer is NULL */
  HDC_E_WORKSPACE = -5 /* workspace too small */
};

/* Library version and the compute capability it was built for (100 = sm_100a). */
int hdc_version(void);
int hdc_built_arch(void);
const char* hdc_error_string(void);
/* Number of kernel launches this library has issued in the process (all devices). */
long long hdc_launch_count(void);

/*
 * LayerNorm over D, then causal depthwise conv1d of width 4 over L, optional SiLU.
 * Replaces _fused_norm_conv_fwd_kernel (hdcmamba/model.py:22-72) as launched by
 * FusedNormConv1dFunction.forward (hdcmamba/model.py:128-146).
 *   x, out    : [B, L, D] contiguous, dtype.  out must not alias x.
 *   norm_w/b  : [D]; conv_w : [D, 4] (tap k multiplies row t-3+k); conv_b : [D].
 *   halo      : NULL, or [B, 3, D] rows that precede x[:, 0] (sequence-parallel
 *               segments); NULL means rows before t=0 are zeros, whose
 *               LayerNorm is norm_b (hdcmamba/model.py:47-57).
 *   mean,rstd : NULL, or [B, L] bf16 per-row statistics (hdcmamba/model.py:67-68).
 *   act       : HDC_ACT_NONE (the reference) or HDC_ACT_SILU.
 * D must be a multiple of 8 (bf16) / 4 (fp32), D <= 4096 (bf16) / 2048 (fp32); pointers
 * 16-byte aligned.
 */
int hdc_ln_conv_fwd(int dtype, const void* x, const void* norm_w, const void* norm_b,
                    const void* conv_w, const void* conv_b, const void* halo, void* out,
                    void* mean, void* rstd, int64_t B, int64_t L, int64_t D, float eps, int act,
                    hdc_stream_t stream);
/*
 * hdc_ln_conv_fwd for a sequence-parallel segment whose halo arrives from another GPU (no
 * single-launch counterpart in the reference, which has no sequence parallelism): the CTAs
 * that read the halo first wait (bounded, acquire at system scope) until the uint32 *halo_flag
 * reaches the generation *halo_gen, so no separate wait kernel precedes the launch.  halo,
 * halo_flag and halo_gen are required.  A wait that times out records code 43 in
 * hdc_device_error() and the kernel goes on (its output is then invalid).
 */
int hdc_ln_conv_fwd_halo_flag(int dtype, const void* x, const void* norm_w, const void* norm_b,
                              const void* conv_w, const void* conv_b, const void* halo, void* out,
                              void* mean, void* rstd, int64_t B, int64_t L, int64_t D, float eps, int act,
                              const uint32_t* halo_flag, const uint32_t* halo_gen, hdc_stream_t stream);

/*
 * Backward of hdc_ln_conv_fwd (no activation): the reference's
 * _fused_norm_conv_bwd_kernel + FusedNormConv1dFunction.backward (hdcmamba/model.py:74-124,
 * 148-166), with its formulas: dx through the LayerNorm backward on the forward's bf16
 * mean / rstd ([B*L] bf16 from hdc_ln_conv_fwd); d_conv_w[d][k] = sum_t go[t] *
 * xhat[t-3+k] * nw (no norm-bias term, nothing from the rows before the sequence);
 * d_norm_b = sum_t dn[t] over real rows; d_conv_b = sum_t go[t].  Parameter gradients are
 * summed in fp32 (per CTA, then over the CTAs in a fixed order) and stored in dtype:
 * d_norm_w / d_norm_b / d_conv_b [D], d_conv_w [D, 4].  grad_out, x, dx: [B, L, D]
 * contiguous.  D a multiple of 4, at most 2048; pointers 16-byte aligned; workspace of
 * hdc_ln_conv_bwd_workspace_bytes(B, L, D) bytes.
 */
size_t hdc_ln_conv_bwd_workspace_bytes(int64_t B, int64_t L, int64_t D);
int hdc_ln_conv_bwd(int dtype, const void* grad_out, const void* x, const void* mean, const void* rstd,
                    const void* norm_w, const void* conv_w, void* dx, void* dnorm_w, void* dnorm_b,
                    void* dconv_w, void* dconv_b, void* workspace, size_t workspace_bytes, int64_t B,
                    int64_t L, int64_t D, hdc_stream_t stream);

/*
 * Diagonal SSM chunk statistics (pass 1 of the chunked scan).
 * Replaces _ssm_intra_v2's last_state / chunk_decay outputs (hdcmamba/model.py:175-198,
 * launched at 345-350).  For batch b and chunk n (C steps), per channel j < ds:
 *   stats[((b*N)+n)*2*ds + j]      = bf16(h at the chunk end, started from 0)
 *   stats[((b*N)+n)*2*ds + ds + j] = bf16(sum of dt_s*A over the chunk)
 * (fp32 storage holding bf16-rounded values).
 *   projs     : row (b, t) starts at projs + b*proj_sb + t*proj_st; columns
 *               [0,ds) dt, [ds,2ds) x, [2ds,3ds) b (hdcmamba/model.py:189-191).
 *   A_log     : [ds], dtype.
 * L must be a multiple of C; ds a power of two in [16, 256].
 */
int hdc_ssm_chunk_stats(int dtype, const void* projs, int64_t proj_sb, int64_t proj_st,
                        const void* A_log, float* stats, int64_t B, int64_t L, int64_t ds,
                        int64_t C, hdc_stream_t stream);

/*
 * Diagonal SSM outputs (pass 2): exclusive prefix over chunk statistics, then
 * y = bf16(bf16(y_intra) + G_n * exp(cum_log)).
 * Replaces _ssm_scan_v2 + _ssm_inter_v2 (hdcmamba/model.py:200-233, launched 352-363).
 *   stats     : [B, n_prev + N, 2*ds] from hdc_ssm_chunk_stats; the first n_prev
 *               chunks precede this segment (sequence-parallel: earlier ranks),
 *               stats_sb = (n_prev+N)*2*ds is the batch stride in floats.
 *   y         : element (b, t, j) at y + b*y_sb + t*y_st + j, dtype.
 */
int hdc_ssm_scan_out(int dtype, const void* projs, int64_t proj_sb, int64_t proj_st,
                     const void* A_log, const float* stats, int64_t stats_sb, int64_t n_prev,
                     void* y, int64_t y_sb, int64_t y_st, int64_t B, int64_t L, int64_t ds,
                     int64_t C, hdc_stream_t stream);

/*
 * The whole diagonal-SSM chunked scan in one call: hdc_ssm_chunk_stats into the caller's
 * stats ([B, L/C, 2*ds] fp32 scratch), then hdc_ssm_scan_out with n_prev = 0.
 * Replaces the three SSM kernels of hdcmamba/model.py:175-233 (launched 345-363).  The two
 * passes are enqueued back to back, so the output pass may start its loads and local scans
 * while the statistics pass finishes (it waits for that pass before reading stats).
 */
int hdc_ssm_scan_fwd(int dtype, const void* projs, int64_t proj_sb, int64_t proj_st,
                     const void* A_log, float* stats, void* y, int64_t y_sb, int64_t y_st,
                     int64_t B, int64_t L, int64_t ds, int64_t C, hdc_stream_t stream);

/*
 * hdc_ssm_scan_out with the statistics stored in blocks of block_chunks chunks, block i
 * at stats + i*block_stride (batch b of a block at + b*stats_sb): the rank-major layout of
 * per-rank statistics gathered under sequence parallelism, read in place.  Chunk m of
 * batch b is at stats + (m / block_chunks)*block_stride + b*stats_sb +
 * (m % block_chunks)*2*ds.  Same prefix order and results as hdc_ssm_scan_out.
 * wait_mask != 0: the statistics of earlier ranks arrive from other GPUs; every CTA first
 * stages its chunk's inputs, then waits (bounded, acquire at system scope) until each
 * uint32 flag wait_flags[s] with bit s of wait_mask set reaches *wait_gen (code 45 in
 * hdc_device_error() on a timeout).  wait_mask == 0: no wait (flags may be NULL).
 */
int hdc_ssm_scan_out_blocked(int dtype, const void* projs, int64_t proj_sb, int64_t proj_st,
                             const void* A_log, const float* stats, int64_t stats_sb,
                             int64_t block_chunks, int64_t block_stride, int64_t n_prev, void* y,
                             int64_t y_sb, int64_t y_st, int64_t B, int64_t L, int64_t ds, int64_t C,
                             const uint32_t* wait_flags, uint32_t wait_mask,
                             const uint32_t* wait_gen, hdc_stream_t stream);

/*
 * The whole diagonal-SSM chunked scan (hdc_ssm_chunk_stats + hdc_ssm_scan_out, n_prev = 0)
 * without any device allocation by the caller or the library.  No counterpart in the
 * reference.  For callers that cannot allocate device memory (a host that only hands the
 * library the tensors it owns, or code that must not call cudaMalloc at that point):
 * the chunk statistics live in a fixed device array of hdc_ssm_noalloc_capacity() fp32
 * values (4 MiB, reserved on every GPU that loads the library until process exit), so
 * B * (L / C) * 2 * ds must not exceed it (HDC_E_WORKSPACE otherwise).  The first call
 * on a device looks the array's address up (cudaGetSymbolAddress); make it before any
 * stream capture.  Calls share the array: every value read is rewritten by the same
 * call, but calls that overlap on the GPU race.
 */
int hdc_ssm_scan_fwd_noalloc(int dtype, const void* projs, int64_t proj_sb, int64_t proj_st,
                             const void* A_log, void* y, int64_t y_sb, int64_t y_st, int64_t B,
                             int64_t L, int64_t ds, int64_t C, hdc_stream_t stream);
int64_t hdc_ssm_noalloc_capacity(void);

/*
 * Slot memory: size in bytes of the fp32 workspace hdc_slot_scan_fwd needs.
 */
size_t hdc_slot_workspace_bytes(int64_t B, int64_t L, int64_t H, int64_t hd, int64_t C);

/*
 * Slot memory: chunked decayed linear attention with a (bd x bd) fp32 state per
 * (batch, head), bd = max(64, pow2(hd)).
 * Replaces _slot_all_fused (hdcmamba/model.py:236-272, launched at 365-371).
 *   q, k, v   : element (b, t, h, d) at ptr + b*in_sb + t*in_st + h*hd + d (dtype);
 *               for the Block these are column slices of projs.
 *   gamma     : [H] per-head decay in dtype (gamma_buf.to(x.dtype), model.py:335),
 *               used when log_a is NULL.
 *   log_a     : NULL, or fp32 per-step log decay, element (b,t,h) at
 *               log_a + (b*L + t)*H + h (the per-step generalisation).
 *   y         : element (b, t, h, d) at y + b*y_sb + h*y_sh + t*y_st + d (dtype).
 *   rows      : rows of each chunk a launch covers (the reference's slot_block_c
 *               when smaller than C, hdcmamba/model.py:17); rows == C normally.
 *   state_in  : NULL or fp32 [B*H, bd, bd] initial state; state_out: NULL or
 *               fp32 [B*H, bd, bd] state after the last chunk.
 *   workspace : hdc_slot_workspace_bytes(...) bytes of device memory.
 * bf16 activations run the tcgen05 tensor-core kernel; fp32 runs the CUDA-core kernel.
 */
int hdc_slot_scan_fwd(int dtype, const void* q, const void* k, const void* v, int64_t in_sb,
                      int64_t in_st, const void* gamma, const float* log_a, void* y, int64_t y_sb,
                      int64_t y_sh, int64_t y_st, const float* state_in, float* state_out,
                      void* workspace, size_t workspace_bytes, int64_t B, int64_t L, int64_t H,
                      int64_t hd, int64_t C, int64_t rows, hdc_stream_t stream);

/*
 * Slot memory scan with the GroupNorm * sigmoid(gate) epilogue fused in: writes
 *   out(b,t,h,:) = bf16( GroupNorm_h(y(b,t,h,:)) * sigmoid(gate(b,t,h,:)) )
 * with y the hdc_slot_scan_fwd output (rounded to bf16 first, as the reference stores
 * y_slot) and the GroupNorm of the reference gate kernel (eps 1e-5, the padded-lane
 * variance term for head_dim < 64).  Together replaces _slot_all_fused and the slot half
 * of _fused_gnorm_gate_cat_kernel (hdcmamba/model.py:236-293) for the corrected launch
 * strides; for the Block, out = combined + d_state with out_sh = head_dim.
 *   gate element (b,t,h,d) at gate + b*gate_sb + t*gate_st + h*hd + d;
 *   out  element (b,t,h,d) at out + b*out_sb + h*out_sh + t*out_st + d.
 * bf16 only, tcgen05 path only (head_dim <= 64 and a multiple of 8, chunk 64/128/256);
 * other shapes return HDC_E_SHAPE.
 */
int hdc_slot_gate_fwd(int dtype, const void* q, const void* k, const void* v, int64_t in_sb,
                      int64_t in_st, const void* gamma, const float* log_a, const void* gate,
                      int64_t gate_sb, int64_t gate_st, const void* gn_w, const void* gn_b, void* out,
                      int64_t out_sb, int64_t out_sh, int64_t out_st, const float* state_in,
                      float* state_out, void* workspace, size_t workspace_bytes, int64_t B, int64_t L,
                      int64_t H, int64_t hd, int64_t C, hdc_stream_t stream);

/*
 * Slot memory state only: the fp32 state after the whole sequence, started from zero
 * (state_out [B*H, 64, 64]), and the product of all chunk decays (decay_out [B*H]), with
 * no outputs.  The sequence-parallel runner exchanges these per rank and folds them into
 * the next rank's state_in (hdc_slot_scan_fwd / hdc_slot_gate_fwd).  Same chunk recurrence
 * as _slot_all_fused's `running` (hdcmamba/model.py:252, 271-272).  bf16, tcgen05 path only.
 * On return `workspace` also holds every segment's local state, which
 * hdc_slot_gate_carry_fwd reuses.
 */
int hdc_slot_state_fwd(int dtype, const void* k, const void* v, int64_t in_sb, int64_t in_st,
                       const void* gamma, const float* log_a, float* state_out, float* decay_out,
                       void* workspace, size_t workspace_bytes, int64_t B, int64_t L, int64_t H,
                       int64_t hd, int64_t C, hdc_stream_t stream);

/*
 * hdc_slot_gate_fwd for one rank's part of a sequence under sequence parallelism: the
 * entering state is folded from the n_prev earlier parts, R <- D_s R + R_s for s = 0 ..
 * n_prev-1 (R from zero), where part s has R_s at prev_state + s*prev_stride (fp32
 * [B*H, 64, 64]) and D_s at prev_decay + s*prev_stride (fp32 [B*H]): the gathered
 * state_out / decay_out of hdc_slot_state_fwd on the earlier ranks.  prev_state must be
 * 16-byte aligned and prev_stride a multiple of 4 (HDC_E_ALIGN otherwise).  `workspace` must be
 * the one that this rank's hdc_slot_state_fwd over the same k, v and shape filled (its
 * segment states are reused; only the output pass runs).  No single-launch counterpart in
 * the reference: it replaces _slot_all_fused's carry of `running` across chunks
 * (hdcmamba/model.py:252, 271-272) across ranks.
 * wait_mask != 0: prev_state / prev_decay arrive from other GPUs; the kernel waits (bounded,
 * acquire at system scope) until each uint32 flag wait_flags[s] with bit s of wait_mask set
 * reaches *wait_gen before it reads them -- at chunk 256 after the first chunk's S and P, so
 * the wait overlaps them (code 44 in hdc_device_error() on a timeout).  wait_mask == 0: no wait.
 */
int hdc_slot_gate_carry_fwd(int dtype, const void* q, const void* k, const void* v, int64_t in_sb,
                            int64_t in_st, const void* gamma, const float* log_a, const void* gate,
                            int64_t gate_sb, int64_t gate_st, const void* gn_w, const void* gn_b,
                            void* out, int64_t out_sb, int64_t out_sh, int64_t out_st,
                            const float* prev_state, const float* prev_decay, int64_t prev_stride,
                            int64_t n_prev, float* state_out, void* workspace, size_t workspace_bytes,
                            int64_t B, int64_t L, int64_t H, int64_t hd, int64_t C,
                            const uint32_t* wait_flags, uint32_t wait_mask,
                            const uint32_t* wait_gen, hdc_stream_t stream);

/*
 * hdc_slot_scan_fwd with the kernel family chosen per call (tests / cross-checks): path 0 =
 * automatic (tcgen05 for bf16 with feature width 64, chunk 64/128/256, 8-aligned head_dim
 * and row-contiguous inputs; CUDA cores otherwise), 1 = always the CUDA-core kernel, 2 =
 * require tcgen05 (HDC_E_SHAPE when it cannot be used).  *path_used (host int, may be NULL)
 * receives 1 when the tcgen05 kernels ran, 0 for the CUDA-core kernels.  No state is kept
 * between calls.  Same reference code as hdc_slot_scan_fwd (hdcmamba/model.py:236-272).
 */
int hdc_slot_scan_fwd_path(int dtype, const void* q, const void* k, const void* v, int64_t in_sb,
                           int64_t in_st, const void* gamma, const float* log_a, void* y, int64_t y_sb,
                           int64_t y_sh, int64_t y_st, const float* state_in, float* state_out,
                           void* workspace, size_t workspace_bytes, int64_t B, int64_t L, int64_t H,
                           int64_t hd, int64_t C, int64_t rows, int path, int* path_used,
                           hdc_stream_t stream);

/*
 * Device-side error word of the tcgen05 kernels: 0, or the code of a bounded wait
 * (mbarrier) that timed out after ~2 s.  Synchronous; reset != 0 clears it.
 * Returns -1 if the word could not be read.
 */
int hdc_device_error(int reset);

/*
 * GroupNorm over each head of y_slot, times sigmoid(gate), concatenated after y_ssm.
 * Replaces _fused_gnorm_gate_cat_kernel (hdcmamba/model.py:274-295, launched at 375-380);
 * the stride arguments mirror that launch, so the reference's literal strides
 * (shipped quirks) and corrected strides are both expressible.
 *   y_slot element (b,h,l,d): y_slot + (b*H+h)*slot_s_bh + (l/slot_rows)*slot_s_n
 *                             + (l%slot_rows)*slot_s_c + d
 *   y_ssm  element (b,l,j)  : y_ssm + b*ssm_s_b + l*ssm_s_l + j
 *   gate   element (b,l,h,d): gate + b*gate_s_b + l*gate_s_l + h*hd + d
 *   out    element (b,l,c)  : out + b*out_s_b + l*out_s_l + c, c in [0, ds+H*hd)
 *   gn_w, gn_b : [H*hd] (dtype).  eps = 1e-5 (hdcmamba/model.py:291).
 */
int hdc_gate_cat_fwd(int dtype, const void* y_slot, int64_t slot_s_bh, int64_t slot_s_n,
                     int64_t slot_s_c, int64_t slot_rows, const void* y_ssm, int64_t ssm_s_b,
                     int64_t ssm_s_l, const void* gate, int64_t gate_s_b, int64_t gate_s_l,
                     const void* gn_w, const void* gn_b, void* out, int64_t out_s_b,
                     int64_t out_s_l, int64_t B, int64_t L, int64_t H, int64_t hd, int64_t ds,
                     hdc_stream_t stream);

/*
 * Row LayerNorm without affine, fp32 statistics, result in dtype (in place allowed).
 * Replaces F.layer_norm(combined.float(), (ds+dm,)).to(x.dtype) (hdcmamba/model.py:382).
 *   in/out : [rows, width] contiguous.
 */
int hdc_row_layernorm(int dtype, const void* in, void* out, int64_t rows, int64_t width,
                      float eps, hdc_stream_t stream);

/*
 * Row LayerNorm with the elementwise affine of nn.LayerNorm: (x - mean) * rstd * weight +
 * bias in fp32, result in dtype (in place allowed).  Replaces HdcMamba9v3Model.norm_final
 * (hdcmamba/model.py:400, 404) and the LM wrapper's final LayerNorm (train.py:121, 135).
 *   in/out : [rows, width] contiguous;  weight, bias : [width] in dtype.
 */
int hdc_row_layernorm_affine(int dtype, const void* in, const void* weight, const void* bias,
                             void* out, int64_t rows, int64_t width, float eps,
                             hdc_stream_t stream);

/*
 * Recurrent single-token decode (no reference counterpart: the reference's generation
 * re-runs the whole prefix).  The state continues the chunked prefill one row at a time
 * with the prefill's formulas and rounding points (bf16 activations: the tcgen05 path's;
 * fp32: the CUDA-core path and the gate kernel's):
 * hdc_ln_conv_step: x [B, D] -> out [B, D]; window fp32 [B, 3, D] holds the normalised
 *   rows t-3, t-2, t-1 and is shifted in place.
 * hdc_ssm_step: one step of the diagonal SSM from projs rows [B, >=3ds] (batch stride
 *   proj_sb); h / cum / G fp32 [B, ds] are the chunk-local state, its summed log decay and
 *   the carry of the earlier chunks; *pos (device int32, the row index within the chunk of
 *   C rows) == C-1 folds the chunk into G.  y element (b, j) at y + b*y_sb + j.
 * hdc_ssm_carry_fwd: G after the N chunks whose statistics (hdc_ssm_chunk_stats, fp32
 *   [B, N, 2ds]) are given, folded in chunk order.
 * hdc_slot_step: row i of the current chunk of the slot scan, fused with GroupNorm(head) *
 *   sigmoid(gate); one CTA per (batch, head).  q / k / v / gate: [B, H*hd] rows of projs
 *   (batch stride proj_sb); R / U fp32 [B*H, 64, 64] (state at the chunk start, update of
 *   the chunk so far); k_cache / v_cache [B*H, C, 64] in dtype (the chunk's phi(k) / v rows);
 *   out element (b, h, d) at out + b*out_sb + h*hd + d.  The row index i is read from the
 *   device int32 *pos (0 <= i < C; otherwise nothing is written and hdc_device_error
 *   reports 51).  hd <= 64, C <= 256.  The position lives on the device so that a decode
 *   step can be replayed as a CUDA graph.
 */
int hdc_ln_conv_step(int dtype, const void* x, const void* norm_w, const void* norm_b, const void* conv_w,
                     const void* conv_b, float* window, void* out, int64_t B, int64_t D, float eps,
                     hdc_stream_t stream);
int hdc_ssm_step(int dtype, const void* projs, int64_t proj_sb, const void* A_log, float* h, float* cum,
                 float* G, void* y, int64_t y_sb, int64_t B, int64_t ds, const int32_t* pos, int64_t C,
                 hdc_stream_t stream);
int hdc_ssm_carry_fwd(int dtype, const float* stats, int64_t B, int64_t N, int64_t ds, float* G,
                      hdc_stream_t stream);
int hdc_slot_step(int dtype, const void* q, const void* k, const void* v, const void* gate, int64_t proj_sb,
                  const void* gamma, const void* gn_w, const void* gn_b, float* R, float* U, void* k_cache,
                  void* v_cache, void* out, int64_t out_sb, int64_t B, int64_t H, int64_t hd, int64_t C,
                  const int32_t* pos, hdc_stream_t stream);

/*
 * Peer-memory exchange for sequence parallelism (one process per GPU, NVLink / NVSwitch).
 * No reference counterpart: it replaces the all-gathers of the sequence-parallel runner
 * with direct peer stores where the data flow is one-directional (rank r needs the carries
 * of ranks < r and the halo rows of rank r-1).  Every wait is bounded (~2 s) and reports a
 * timeout through hdc_device_error().
 *
 * hdc_peer_alloc / hdc_peer_free: a zeroed device mailbox (cudaMalloc) that can be shared.
 * hdc_ipc_handle / hdc_ipc_open / hdc_ipc_close: CUDA IPC handle (hdc_ipc_handle_bytes()
 *   bytes) of a mailbox, and its mapping in another process of the same node.
 * hdc_peer_put: for every target t with bit t of mask set, copy `bytes` from src (local,
 *   16-byte aligned) to dst_base[t] + dst_off, then store *gen (a device counter) as a
 *   uint32 flag at dst_base[t] + flag_off with release semantics at system scope.
 *   dst_base is a device array of `world` mailbox base addresses as mapped in this process.
 *   The copy to each target is split over up to 64 CTAs (8 KB slices); `counters` is a
 *   caller-owned device array of `world` uint32, zero before the call and left zero after it,
 *   through which the CTA finishing a target's last slice raises its flag.  Puts that may
 *   run concurrently (different streams) need separate counter arrays.
 * hdc_peer_wait: wait until flags[s] has reached *gen (wrap-safe >=) for every bit s of mask
 *   (acquire, system scope).
 * hdc_peer_wait_for: hdc_peer_wait with the caller's limit per flag (1 ns .. 2 s; HDC_E_SHAPE
 *   otherwise); on timeout the wait records code 41 in hdc_device_error() and returns.
 * hdc_peer_gen_bump: *gen += 1 (once per forward on every rank).
 * hdc_peer_barrier: store *gen into slot `rank` of the uint32 array at base[s] + bar_off of
 *   every rank s, then wait until all `world` slots of local_bar have reached *gen.
 */
int hdc_peer_alloc(size_t bytes, void** dev_ptr);
int hdc_peer_free(void* dev_ptr);
int hdc_ipc_handle_bytes(void);
int hdc_ipc_handle(const void* dev_ptr, void* handle_out);
int hdc_ipc_open(const void* handle, void** dev_ptr);
int hdc_ipc_close(void* dev_ptr);
int hdc_peer_put(const void* src, size_t bytes, const uint64_t* dst_base, uint64_t dst_off,
                 uint64_t flag_off, uint32_t mask, int world, const uint32_t* gen,
                 uint32_t* counters, hdc_stream_t stream);
int hdc_peer_wait(const uint32_t* flags, uint32_t mask, const uint32_t* gen, hdc_stream_t stream);
int hdc_peer_wait_for(const uint32_t* flags, uint32_t mask, const uint32_t* gen, uint64_t timeout_ns,
                      hdc_stream_t stream);
int hdc_peer_gen_bump(uint32_t* gen, hdc_stream_t stream);
int hdc_peer_barrier(const uint64_t* base, uint64_t bar_off, int world, int rank,
                     const uint32_t* local_bar, const uint32_t* gen, hdc_stream_t stream);

/*
 * Tracing (no counterpart in the reference, which times whole forwards with
 * time.perf_counter, benchmark.py:165-192): enqueue on `stream` a one-thread kernel that
 * stores the device's %globaltimer (ns) into buf[index].  Stamps taken between the
 * launches of a CUDA graph time each op on the device in stream order
 * (hdcmamba_b200/trace.py).  buf: device array of at least index + 1 entries.
 */
int hdc_trace_stamp(unsigned long long* buf, long long index, hdc_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* HDCMAMBA_B200_H */
