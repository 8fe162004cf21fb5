/*
 * lizard_cuda.h — C ABI of the B200 (sm_100a) backend for Lizard's two
 * attention branches: chunked gated linear attention (GLA) and sliding-window
 * softmax attention with sink logits (SWA).
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * passed as void*. The library never allocates or frees device memory: the
 * caller owns every buffer, including the opaque "saved" buffer that carries
 * forward state into the backward pass and the backward workspace. Sizes of
 * those two buffers come from the *_bytes queries below. All work is enqueued
 * on the given stream; no call synchronises the host.
 *
 * Return value: LZ_OK (0) or an LZ_ERR_* code; lz_last_error_string() then
 * holds a message for the calling thread. Bad shapes, null or misaligned
 * pointers are reported as errors, never by aborting or trapping.
 *
 * Tensor layouts (row-major, contiguous, "BH" = batch*heads, b-major):
 *   fq, fk     bf16 [BH, L, F]      feature-mapped queries / keys (F = NF)
 *   v, y, dy   bf16 [BH, L, D]      values / output / output grad (D = ND)
 *   log_gamma  fp32 [B, L] when gate_per_head == 0 (one gate shared by the H
 *              heads of a batch row), fp32 [BH, L] when gate_per_head == 1
 *   q, k       bf16 [BH, L, D]      already-rotated queries / keys for SWA
 *   q_lo, k_lo bf16 [BH, L, D]      optional residuals: q = q + q_lo, k = k + k_lo
 *              (pass null for both when the caller's data is bf16)
 *   meta       fp32 [n_meta]        sink logits (n_meta may be 0)
 */
#ifndef LIZARD_CUDA_H_
#define LIZARD_CUDA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LZ_ABI_VERSION 3

enum {
  LZ_OK = 0,
  LZ_ERR_INVALID_ARGUMENT = 1, /* bad shape, null pointer, bad alignment */
  LZ_ERR_UNSUPPORTED = 2,      /* valid but outside this build's limits  */
  LZ_ERR_CUDA = 3,             /* a CUDA launch or runtime call failed   */
  LZ_ERR_WORKSPACE = 4         /* workspace / saved buffer too small     */
};

/* Output dtype selector for gradient buffers. */
enum { LZ_DTYPE_F32 = 0, LZ_DTYPE_BF16 = 1 };

/* ABI revision of the loaded library; equals LZ_ABI_VERSION it was built with. */
int lz_abi_version(void);

/* Message for the last failing call on this host thread ("" if none). */
const char* lz_last_error_string(void);

/* Number of kernels this library has launched in this process (all devices).
 * Lets a caller count device launches inside a timed region. */
uint64_t lz_launch_count(void);

/* Every wait inside the tensor-core kernels is bounded (about 2 s); a wait
 * that gives up records where in this per-device flag and the kernel unwinds
 * instead of hanging. Reads the flag of the current device into *site
 * (0 = no wait ever timed out). Synchronous. */
int lz_device_timeout_flag(unsigned int* site);

/* Clears that flag on the current device, after the caller has read and
 * handled a timeout: until it is cleared, the waits of the affected kernels
 * return at once. No counterpart in the reference (its Triton kernels have no
 * bounded waits). Synchronous. */
int lz_device_timeout_clear(void);

/* Test switch for the bounded-wait path on the current device (no counterpart
 * in the reference): with on != 0, lz_swa_decode arms the barrier of its
 * ring-buffer copy but issues no copy, so the wait runs out after about 2 s,
 * lz_device_timeout_flag reports the site, and the call writes nothing. Off by
 * default; leave it off outside tests. */
int lz_test_withhold_decode_ring_copy(int on);

/* ------------------------------------------------------------------------ */
/* GLA                                                                      */
/* ------------------------------------------------------------------------ */

/* Bytes of the opaque buffer lz_gla_fwd fills for lz_gla_bwd.
 * Replaces the tensors _GLA.forward keeps with ctx.save_for_backward
 * (src/kernels/gla.py:220-232 of the reference): fp32 y and den, the
 * cumulative log gate G, the per-chunk states S (bf16) and z (fp32). */
size_t lz_gla_saved_bytes(int B, int H, int L, int F, int D, int chunk);

/* Bytes of scratch lz_gla_bwd needs (delta, dS, dz, dG, and the per-chunk
 * increments when the chunk-parallel schedule is planned). */
size_t lz_gla_bwd_workspace_bytes(int B, int H, int L, int F, int D, int chunk);

/* Bytes of scratch lz_gla_fwd needs: 0 when the sequential walk is planned
 * for this shape, else the per-chunk increments and states of the
 * chunk-parallel schedule. No counterpart in the reference, whose forward
 * allocates its state tensors itself (src/kernels/gla.py:221-222). */
size_t lz_gla_fwd_workspace_bytes(int B, int H, int L, int F, int D, int chunk);

/* Schedule of the GLA kernels, process-wide: 0 = chosen per shape (default),
 * 1 = sequential walk over the chunks of each head (state kept on chip),
 * 2 = chunk-parallel (every chunk's state increment at once, then a scan over
 * chunks, then every chunk's output at once). Both give the same results
 * within bf16 rounding. Returns the previous setting, or -LZ_ERR_INVALID_ARGUMENT
 * for a value outside 0..2 (the setting is then unchanged). The workspace queries
 * depend on it: do not change it between a query and the call it sizes.
 * No counterpart in the reference; a hook for tests and tuning. */
int lz_gla_set_schedule(int schedule);

/* Chunk outputs of the chunk-parallel schedule on the tensor cores (1, the
 * default: F in {128, 256} with D = 64, or F = D = 128) or on the warp-MMA
 * kernel (0). Returns the previous setting. A hook for tests and tuning,
 * process-wide; y is the same with and without a saved buffer either way. */
int lz_gla_set_split_out_tc(int on);

/* Selects the walk schedule's tensor-core forward for F = D = 128: two
 * sequences per SM with 64-token chunks (1) or one sequence per SM with
 * 128-token chunks (0, the default). Both save the same 128-token chunk states
 * for the backward. Returns the previous setting. A hook for tests and tuning,
 * process-wide; do not change it between a forward and its backward. */
int lz_gla_set_fwd_tc64(int on);

/* L2 prefetch in the tensor-core per-chunk gradient kernel (F = D = 128 and
 * F = D = 64): each CTA sends the operands of the CTA one SM count further on
 * to L2 while it computes (1, the default) or not (0). Results are identical
 * either way. Returns the previous setting. A hook for tests and tuning,
 * process-wide. No counterpart in the reference. */
int lz_gla_set_bwd_prefetch(int on);

/* Forward of gla(fq, fk, v, log_gamma, chunk).
 * Replaces gla() + _GLA.forward of the reference (src/kernels/gla.py:259-263
 * and 213-234): G = cumsum(log_gamma) is computed on the device, chunk by
 * chunk. y is bf16. When saved is non-null the forward also fills it for the
 * backward; y is bit-identical either way. workspace may be null when
 * lz_gla_fwd_workspace_bytes returns 0.
 * chunk is the reference's chunk length argument; the kernels use 64-token
 * chunks and accept any chunk >= 1 (results agree within bf16 tolerance). */
int lz_gla_fwd(const void* fq, const void* fk, const void* v,
               const float* log_gamma, int gate_per_head,
               void* y, void* saved, size_t saved_bytes,
               void* workspace, size_t workspace_bytes,
               int B, int H, int L, int F, int D, int chunk, void* stream);

/* Backward of gla(). Replaces _GLA.backward (src/kernels/gla.py:236-256)
 * including the torch-side delta, dg and the cumsum/expand backward of
 * gla.py:260-262: it writes dfq, dfk [BH,L,F], dv [BH,L,D] in grad_dtype and
 * dlog_gamma (fp32, same shape as log_gamma). */
int lz_gla_bwd(const void* fq, const void* fk, const void* v,
               const float* log_gamma, int gate_per_head,
               const void* saved, size_t saved_bytes, const void* dy,
               void* dfq, void* dfk, void* dv, int grad_dtype,
               float* dlog_gamma, void* workspace, size_t workspace_bytes,
               int B, int H, int L, int F, int D, int chunk, void* stream);

/* Grouped-query forms (GQA): fk [B*Hkv, L, F] and v [B*Hkv, L, D] with
 * H % Hkv == 0; query head h reads key/value head h / (H / Hkv). In the
 * reference's caller fk = hedgehog(repeat_interleave(k)) and v is
 * repeat_interleaved (src/lizard_attention.py:73-85), so every head of a group
 * sees the same fk and v: these entries take them once. fq, y, log_gamma, the
 * saved buffer and the forward workspace keep H heads (the sizes above); the
 * backward workspace is lz_gla_bwd_gqa_workspace_bytes (it adds fp32 room for
 * the per-head dfk and dv). dfk and dv are [B*Hkv, L, *], each the sum over its
 * group of query heads in a fixed order (the autograd of repeat_interleave).
 * lz_gla_fwd / lz_gla_bwd are these with Hkv = H. */
size_t lz_gla_bwd_gqa_workspace_bytes(int B, int H, int Hkv, int L, int F, int D, int chunk);
/* Forward workspace of lz_gla_fwd_gqa. training != 0 when a saved buffer is
 * passed. Without one and with a gate shared by the heads (gate_per_head = 0),
 * the chunk-parallel schedule keeps one state per key/value head (the query
 * heads of a group have identical states), so the workspace is sized for Hkv
 * heads. 0 when the sequential walk is planned. */
size_t lz_gla_fwd_gqa_workspace_bytes(int B, int H, int Hkv, int L, int F, int D, int chunk,
                                      int gate_per_head, int training);
int lz_gla_fwd_gqa(const void* fq, const void* fk, const void* v,
                   const float* log_gamma, int gate_per_head,
                   void* y, void* saved, size_t saved_bytes,
                   void* workspace, size_t workspace_bytes,
                   int B, int H, int Hkv, int L, int F, int D, int chunk, void* stream);
int lz_gla_bwd_gqa(const void* fq, const void* fk, const void* v,
                   const float* log_gamma, int gate_per_head,
                   const void* saved, size_t saved_bytes, const void* dy,
                   void* dfq, void* dfk, void* dv, int grad_dtype,
                   float* dlog_gamma, void* workspace, size_t workspace_bytes,
                   int B, int H, int Hkv, int L, int F, int D, int chunk, void* stream);

/* ------------------------------------------------------------------------ */
/* GLA, sequence-parallel segments                                          */
/* ------------------------------------------------------------------------ */
/* A long sequence split over P ranks: rank r owns tokens [r*Ls, (r+1)*Ls)
 * of every head (fq, fk, v, y, dy are that rank's [BH, Ls, *] slices and
 * log_gamma its [B or BH, Ls] slice; Ls a multiple of 64 except on the last
 * rank). Each rank runs its segment in its own gate frame and only a summary
 * per rank crosses ranks (one all_gather; the transport is the caller's):
 *   summary (fp32) = state [BH,F,D] | zstate [BH,F] | logdecay [BH]
 *   seed    (fp32) = state [BH,F,D] | zstate [BH,F]
 * Forward:  seg_fwd_begin -> gather summaries -> seg_combine(reverse=0)
 *           -> seg_fwd_end(seed; null on rank 0).
 * Backward: seg_bwd_begin -> gather -> seg_combine(reverse=1)
 *           -> seg_bwd_end(dseed; null on the last rank)
 *           -> gather each rank's dlog_gamma[:, 0] -> seg_gate_offset.
 * The reference has no sequence-parallel path; these entry points restate its
 * state recurrence (src/kernels/gla.py:44-57 forward, 118-132 backward) across
 * segments. The workspace must be the same buffer from a begin call to the
 * matching end call. */

/* Workspace bytes of the segment calls (one buffer serves both directions). */
size_t lz_gla_seg_workspace_bytes(int B, int H, int L, int F, int D);

/* Floats of one rank's summary. */
size_t lz_gla_seg_summary_floats(int B, int H, int F, int D);

/* Forward, part 1: per-chunk state increments of the segment (kept in the
 * workspace) and the summary: the state after the segment from a zero start,
 * its normaliser and the segment's total log decay per head. */
int lz_gla_seg_fwd_begin(const void* fk, const void* v, const float* log_gamma,
                         int gate_per_head, float* summary, void* workspace,
                         size_t workspace_bytes, int B, int H, int L, int F, int D,
                         void* stream);

/* Forward, part 2: the states of every chunk from the seed (the state
 * entering the segment; null = zero) and y; fills saved as lz_gla_fwd does. */
int lz_gla_seg_fwd_end(const void* fq, const void* fk, const void* v,
                       const float* log_gamma, int gate_per_head, const float* seed,
                       void* y, void* saved, size_t saved_bytes, void* workspace,
                       size_t workspace_bytes, int B, int H, int L, int F, int D,
                       void* stream);

/* Backward, part 1: per-chunk state-gradient increments and the summary: the
 * gradient w.r.t. the state entering the segment from the segment's own
 * outputs, and the total log decay. saved comes from lz_gla_seg_fwd_end. */
int lz_gla_seg_bwd_begin(const void* fq, const void* saved, size_t saved_bytes,
                         const void* dy, float* summary, void* workspace,
                         size_t workspace_bytes, int B, int H, int L, int F, int D,
                         void* stream);

/* Backward, part 2: dfq, dfk, dv and this segment's part of dlog_gamma (the
 * reverse cumsum restricted to the segment), from dseed (the gradient w.r.t.
 * the state leaving the segment; null = zero). seeded_forward: the forward's
 * seed was not null. */
int lz_gla_seg_bwd_end(const void* fq, const void* fk, const void* v, int gate_per_head,
                       const void* saved, size_t saved_bytes, const void* dy,
                       const float* dseed, int seeded_forward, void* dfq, void* dfk,
                       void* dv, int grad_dtype, float* dlog_gamma, void* workspace,
                       size_t workspace_bytes, int B, int H, int L, int F, int D,
                       void* stream);

/* seed of `rank` from the P gathered summaries ([P][summary floats]):
 * forward (reverse = 0) combines ranks 0..rank-1, backward (reverse = 1)
 * ranks rank+1..P-1, each step h = h * exp(logdecay_q) + state_q. */
int lz_gla_seg_combine(const float* summaries, int P, int rank, int reverse, float* seed,
                       int B, int H, int F, int D, void* stream);

/* dlog_gamma [rows, L] += the sum over ranks after `rank` of totals[q][row],
 * where totals [P][rows] holds every rank's dlog_gamma[row, 0]. */
int lz_gla_seg_gate_offset(float* dlog_gamma, const float* totals, int P, int rank,
                           int rows, int L, void* stream);

/* ------------------------------------------------------------------------ */
/* Hedgehog feature map (the GLA prologue)                                  */
/* ------------------------------------------------------------------------ */
/* f [R, 2 Fd] (bf16) = [softmax(x W^T), softmax(-x W^T)] per row, fused.
 * Replaces hedgehog() of the reference (src/lizard_attention.py:9-11) as the
 * layer calls it on each head's queries and keys before gla(); the reference
 * keeps the result in x's dtype and gla() then casts it to bf16.
 * x [R, Dh] in x_dtype (LZ_DTYPE_F32 or LZ_DTYPE_BF16), weight [Fd, Dh] fp32,
 * Dh <= 128, Fd <= 128. */
int lz_hedgehog_fwd(const void* x, int x_dtype, const float* weight, void* f, int R, int Dh,
                    int Fd, void* stream);

/* Bytes of scratch lz_hedgehog_bwd needs (per-CTA partial weight gradients). */
size_t lz_hedgehog_bwd_workspace_bytes(int R, int Dh, int Fd);

/* Backward of lz_hedgehog_fwd (the autograd of the reference's matmul,
 * softmax and concatenation): dx [R, Dh] and dweight [Fd, Dh] in fp32 from
 * df [R, 2 Fd] in df_dtype. dweight is reduced over rows in a fixed order. */
int lz_hedgehog_bwd(const void* x, int x_dtype, const float* weight, const void* df,
                    int df_dtype, float* dx, float* dweight, void* workspace,
                    size_t workspace_bytes, int R, int Dh, int Fd, void* stream);

/* Forward on the tensor cores (1, the default) or on the warp-MMA kernel (0)
 * for bf16 x with Dh = 64 and Fd = 128 (other shapes always take the latter).
 * Returns the previous setting; a hook for tests and tuning, process-wide. */
int lz_hedgehog_set_tc(int on);

/* Forwards of at most `rows` rows (R) take the warp-per-row kernel (a warp per
 * row, W staged per CTA; for decode-sized inputs); -1 restores the default
 * (fewer rows than one 64-row tile per SM), 0 sends every forward to the tiled
 * kernels. Returns the previous setting (-1 for the default); a hook for
 * tests and tuning, process-wide. */
long long lz_hedgehog_set_rows_max(long long rows);

/* SWA forwards (lz_swa_fwd_gqa and lz_swa_rope_fwd) and the dq and dk / dv
 * kernels of the backward on the tensor cores (1, the default: tcgen05
 * kernels for head dim 64 and windows up to 128) or on the 64-row
 * warp-MMA kernels (0). Returns the previous setting; a hook for tests and
 * tuning, process-wide. */
int lz_swa_set_tc(int on);

/* The same for x [B, Hx, L, Dh] at element strides (x_sb, x_sh, x_sl) with Dh
 * contiguous, e.g. a projection output [B, L, Hx * Dh] read in place as heads
 * (x_sb = L * Hx * Dh, x_sh = Dh, x_sl = Hx * Dh). R = B * Hx * L rows in
 * (batch, head, token) order; f, df and dx are contiguous [R, ...]. */
int lz_hedgehog_fwd_strided(const void* x, int x_dtype, long long x_sb, long long x_sh,
                            long long x_sl, int B, int Hx, int L, const float* weight, void* f,
                            int Dh, int Fd, void* stream);
int lz_hedgehog_bwd_strided(const void* x, int x_dtype, long long x_sb, long long x_sh,
                            long long x_sl, int B, int Hx, int L, const float* weight,
                            const void* df, int df_dtype, float* dx, float* dweight,
                            void* workspace, size_t workspace_bytes, int Dh, int Fd,
                            void* stream);

/* ------------------------------------------------------------------------ */
/* Rotary embedding for the SWA operands (no counterpart in the reference's   */
/* kernels: its caller rotates with torch ops, src/lizard_attention.py:87-88, */
/* and kernels.swa splits nothing)                                           */
/* ------------------------------------------------------------------------ */

/* r = x * cos + rotate_half(x) * sin (Llama's rotate-half RoPE), written as
 * hi = bf16(r) and, when lo is not null, lo = bf16(r - hi): the q / k and
 * q_lo / k_lo operands of lz_swa_fwd_gqa. x is [B, Hx, L, Dh] in x_dtype
 * (LZ_DTYPE_F32 or LZ_DTYPE_BF16) at element strides x_sb, x_sh, x_sl (Dh
 * contiguous), so a projection output [B, L, Hx * Dh] is read in place with
 * x_sb = L * Hx * Dh, x_sh = Dh, x_sl = Hx * Dh. cos and sin are [B, L, Dh]
 * in cs_dtype at strides cs_sb (0 broadcasts one table over the batch) and
 * cs_sl. hi and lo are contiguous [B, Hx, L, Dh] bf16. Dh must be even. */
int lz_rope_split(const void* x, int x_dtype, long long x_sb, long long x_sh, long long x_sl,
                  const void* cos, const void* sin, int cs_dtype, long long cs_sb,
                  long long cs_sl, void* hi, void* lo, int B, int Hx, int L, int Dh,
                  void* stream);

/* Gradient of lz_rope_split's r: dx = R^T dr, dr fp32 contiguous
 * [B, Hx, L, Dh], dx contiguous [B, Hx, L, Dh] in dx_dtype. */
int lz_rope_bwd(const float* dr, const void* cos, const void* sin, int cs_dtype,
                long long cs_sb, long long cs_sl, void* dx, int dx_dtype, int B, int Hx,
                int L, int Dh, void* stream);

/* ------------------------------------------------------------------------ */
/* Output blend of the two branches (no counterpart in the reference's        */
/* kernels: its caller does this with torch ops, src/lizard_attention.py:92-97) */
/* ------------------------------------------------------------------------ */

/* out[b, l, h * D + d] = float(y_gla[b, h, l, d]) + alpha * float(y_swa[b, h, l, d]),
 * stored in out_dtype (LZ_DTYPE_BF16 or LZ_DTYPE_F32): the blend, the cast to
 * the hidden dtype and the [B, H, L, D] -> [B, L, H * D] transpose the output
 * projection reads, in one pass. y_gla, y_swa bf16 [B*H, L, D]; alpha is a
 * device pointer to one fp32 value (alpha_blend in the compute dtype). The
 * product and the sum round once each, as the reference's torch ops do. */
int lz_blend_fwd(const void* y_gla, const void* y_swa, const float* alpha, void* out,
                 int out_dtype, int B, int H, int L, int D, void* stream);

/* Bytes of scratch lz_blend_bwd needs (per-block d alpha partials). */
size_t lz_blend_bwd_workspace_bytes(int B, int H, int L, int D);

/* Gradient of lz_blend_fwd for dout [B, L, H * D] in dout_dtype:
 * dy_gla = bf16(dout), dy_swa = bf16(alpha * dout) (both [B*H, L, D], the
 * dtype the GLA and SWA backward consume) and *dalpha = sum dout * y_swa (fp32,
 * reduced over per-block partials in a fixed order). */
int lz_blend_bwd(const void* dout, int dout_dtype, const void* y_swa, const float* alpha,
                 void* dy_gla, void* dy_swa, float* dalpha, void* workspace,
                 size_t workspace_bytes, int B, int H, int L, int D, void* stream);

/* ------------------------------------------------------------------------ */
/* SWA                                                                      */
/* ------------------------------------------------------------------------ */

/* Bytes of the opaque buffer lz_swa_fwd fills for lz_swa_bwd: the log-sum-exp
 * per row (the reference's lse, src/kernels/swa.py:145-155) and the output in
 * fp32, from which the backward forms delta. */
size_t lz_swa_saved_bytes(int B, int H, int L, int D);

/* Bytes of scratch lz_swa_bwd needs (delta per row, per-block sink partials). */
size_t lz_swa_bwd_workspace_bytes(int B, int H, int L, int D, int n_meta);

/* Forward of swa(q, k, v, meta, window). Replaces _SWA.forward
 * (src/kernels/swa.py:136-156): y = softmax over [i-window+1, i] with the
 * sink logits in the denominator, scale 1/sqrt(D). y is bf16. saved may be
 * null when no backward follows. With q_lo and k_lo the logits are
 * q.k + q.k_lo + q_lo.k (about 16 mantissa bits), for fp32 callers. */
int lz_swa_fwd(const void* q, const void* k, const void* v,
               const void* q_lo, const void* k_lo,
               const float* meta, int n_meta, int window,
               void* y, void* saved, size_t saved_bytes,
               int B, int H, int L, int D, void* stream);

/* Backward of swa(). Replaces _SWA.backward (src/kernels/swa.py:158-179)
 * including the torch-side delta and dmeta: writes dq, dk, dv [BH,L,D] in
 * grad_dtype and dmeta (fp32 [n_meta]). delta_i = sum_t P_it (dy_i . v_t) is
 * formed in fp32 inside the kernels, so y is not needed. q_lo / k_lo as in
 * the forward (both null or both set, the same as the forward call). */
int lz_swa_bwd(const void* q, const void* k, const void* v,
               const void* q_lo, const void* k_lo,
               const float* meta, int n_meta, int window,
               const void* saved, size_t saved_bytes,
               const void* dy, void* dq, void* dk, void* dv, int grad_dtype,
               float* dmeta, void* workspace, size_t workspace_bytes,
               int B, int H, int L, int D, void* stream);

/* Grouped-query forms (GQA): k, k_lo and v carry Hkv heads [B*Hkv, L, D],
 * H % Hkv == 0, and query head h attends with key/value head h / (H / Hkv).
 * This is the reference caller's repeat_interleave of K and V
 * (src/lizard_attention.py:73-76) without the copies. q, y, saved and the
 * workspace keep H heads (the same sizes as above); dk and dv are
 * [B*Hkv, L, D], each the sum over its group of query heads (the autograd
 * of repeat_interleave). lz_swa_fwd / lz_swa_bwd are these with Hkv = H. */
int lz_swa_fwd_gqa(const void* q, const void* k, const void* v,
                   const void* q_lo, const void* k_lo,
                   const float* meta, int n_meta, int window,
                   void* y, void* saved, size_t saved_bytes,
                   int B, int H, int Hkv, int L, int D, void* stream);
int lz_swa_bwd_gqa(const void* q, const void* k, const void* v,
                   const void* q_lo, const void* k_lo,
                   const float* meta, int n_meta, int window,
                   const void* saved, size_t saved_bytes,
                   const void* dy, void* dq, void* dk, void* dv, int grad_dtype,
                   float* dmeta, void* workspace, size_t workspace_bytes,
                   int B, int H, int Hkv, int L, int D, void* stream);

/* The SWA forward with RoPE inside: q [B, H, L, D], k and v [B, Hkv, L, D]
 * unrotated, all in x_dtype (LZ_DTYPE_F32 or LZ_DTYPE_BF16) at element strides
 * (batch, head, token) with D contiguous, so projection outputs are read in
 * place; cos / sin as for lz_rope_split. The kernel loads tiles of q, k, v
 * with TMA, rotates q and k in fp32 and splits them into bf16 value + residual
 * tiles in shared memory, then runs the forward of lz_swa_fwd_gqa: y (and
 * saved) equal lz_rope_split + lz_swa_fwd_gqa bit for bit. With the tensor-core
 * forward on (lz_swa_set_tc) and D = 64, window <= 128 that is a tcgen05
 * kernel (bf16 projections); otherwise the 64-row warp-MMA kernel. q_hi, q_lo
 * [B*H, L, D] and k_hi, k_lo [B*Hkv, L, D] (bf16, all null or all set) receive
 * the rotated operands that lz_swa_bwd_gqa takes. Returns LZ_ERR_UNSUPPORTED
 * without launching when D is not 32, 64 or 128, a stride or base is not
 * 16-byte aligned, the tiles do not fit in shared memory (fp32 at D = 128), or
 * the projections are fp32 at the tensor-core shape; rotate first then (the
 * two passes reach the same forward kernel). The reference rotates with torch
 * ops in its caller (src/lizard_attention.py:87-88). */
int lz_swa_rope_fwd(const void* q, const void* k, const void* v, int x_dtype,
                    long long q_sb, long long q_sh, long long q_sl,
                    long long k_sb, long long k_sh, long long k_sl,
                    long long v_sb, long long v_sh, long long v_sl,
                    const void* cos, const void* sin, int cs_dtype,
                    long long cs_sb, long long cs_sl,
                    const float* meta, int n_meta, int window,
                    void* y, void* saved, size_t saved_bytes,
                    void* q_hi, void* q_lo, void* k_hi, void* k_lo,
                    int B, int H, int Hkv, int L, int D, void* stream);

/* lz_swa_bwd for callers that cannot allocate (no counterpart in the
 * reference, whose kernels always allocate through torch). Some hosts give a
 * plugin only its input and output buffers, for example a serving runtime's
 * custom-op hook without a workspace request, so they cannot supply the
 * workspace of lz_swa_bwd. This variant takes the same arguments minus the
 * workspace and uses a fixed 4 MiB scratch array compiled into the library
 * (held on every GPU that loads it). It allocates nothing. It returns
 * LZ_ERR_UNSUPPORTED when lz_swa_bwd_workspace_bytes(B, H, L, D, n_meta)
 * exceeds 4 MiB (about B*H*L = 1,000,000 rows). All calls on a device share
 * the array; calls that overlap on the GPU race on it. The first call on a
 * device looks up the array's address and should come before any stream
 * capture; that address is kept for the device's primary context, so after a
 * cudaDeviceReset of the device this entry point must not be called again. */
int lz_swa_bwd_noalloc(const void* q, const void* k, const void* v,
                       const void* q_lo, const void* k_lo,
                       const float* meta, int n_meta, int window,
                       const void* saved, size_t saved_bytes,
                       const void* dy, void* dq, void* dk, void* dv, int grad_dtype,
                       float* dmeta, int B, int H, int L, int D, void* stream);

/* ------------------------------------------------------------------------ */
/* Recurrent decode (no counterpart in the reference, which has no cache: its */
/* layer recomputes the whole sequence, src/lizard_attention.py:78-97)        */
/* ------------------------------------------------------------------------ */

/* One GLA decode step for every sequence of the batch: with lg the new
 * token's log gate,
 *   S <- exp(lg) S + fk^T v,  z <- exp(lg) z + fk,  y = fq S / max(fq . z, FLT_MIN)
 * which equals the full-sequence gla() output at that position. fq bf16
 * [B*H, F]; fk bf16 [B*Hkv, F]; v bf16 [B*Hkv, D]; log_gamma fp32 [B] (gate
 * shared by the heads) or [B*H] (gate_per_head). state fp32 [B*Hs, F, D] and
 * zstate fp32 [B*Hs, F] are updated in place; y bf16 [B*H, D]. Hs, the state
 * head count, is H, or Hkv when the gate is shared by the heads: then the
 * H / Hkv query heads of a group read one state (they are identical in the
 * reference, which repeat_interleaves k and v). F <= 256, D % 4 == 0, D <= 256,
 * H / Hs in {1, 2, 4, 8, 16}. A zero state starts a sequence; the state after a
 * prompt is the summary of lz_gla_seg_fwd_begin over it (state | zstate). */
int lz_gla_decode(const void* fq, const void* fk, const void* v, const float* log_gamma,
                  int gate_per_head, float* state, float* zstate, void* y,
                  int B, int H, int Hkv, int Hs, int F, int D, void* stream);

/* One SWA decode step: rotates the new key k (Llama rotate-half RoPE with
 * cos / sin of the token's position) and writes it with v into slot
 * pos[b] % window of the rings k_ring / v_ring (fp32 [B*Hkv, window, D]), then
 * every query head attends (q rotated the same way) over the
 * min(pos[b] + 1, window) newest entries with the n_meta sink logits in the
 * denominator, scale 1/sqrt(D): the full-sequence swa() output at position
 * pos[b]. q [B, H, D], k, v [B, Hkv, D] in x_dtype at element strides
 * (batch, head) with D contiguous; cos, sin [B, D] in cs_dtype at batch
 * stride cs_sb (0 broadcasts); pos int32 [B] (tokens before the new one; the
 * caller advances it); y bf16 [B*H, D]. D even, D <= 256, window <= 1024. */
int lz_swa_decode(const void* q, const void* k, const void* v, int x_dtype,
                  long long q_sb, long long q_sh, long long k_sb, long long k_sh,
                  long long v_sb, long long v_sh, const void* cos, const void* sin,
                  int cs_dtype, long long cs_sb, float* k_ring, float* v_ring,
                  const int* pos, const float* meta, int n_meta, void* y,
                  int B, int H, int Hkv, int window, int D, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LIZARD_CUDA_H_ */
