// Layout of the opaque GLA "saved" buffer (forward -> backward) and of the
// backward workspace. Regions are 256-byte aligned inside the caller's buffer.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#include "common.cuh"

namespace lz {

struct GlaSaved {
  float* y32 = nullptr;  // [BH, L, D] fp32 output (delta = dy . y uses it)
  float* den = nullptr;  // [BH, L] row sums before the clamp
  float* g = nullptr;    // [BH, L] cumulative log gate G
  bf16* s = nullptr;     // [BH, NT, F, D] state entering each chunk (bf16)
  float* z = nullptr;    // [BH, NT, F] normaliser state entering each chunk
};

struct GlaWork {
  float* delta = nullptr;  // [BH, L]
  bf16* ds = nullptr;      // [BH, NT, F, D] state gradient leaving each chunk
  float* dz = nullptr;     // [BH, NT, F]
  float* dg = nullptr;     // [BH, L] gradient w.r.t. G
  float* dgt = nullptr;    // [BH, NT] sum of dg over each chunk
  // chunk-parallel schedule only (null for the sequential walk)
  float* inc = nullptr;    // [BH, NT, F, D] per-chunk increment Q^_n^T dY_n (fp32)
  float* incz = nullptr;   // [BH, NT, F]   per-chunk increment Q^_n^T delta_n
  float* lam = nullptr;    // [BH, NT]      log decay of each chunk, G_end - G_start
  // grouped keys / values only (fk, v with fewer heads than fq): per-query-head
  // gradients before the sum over each group
  float* gk = nullptr;     // [BH, L, F] fp32
  float* gv = nullptr;     // [BH, L, D] fp32
};

// Forward scratch of the chunk-parallel schedule.
struct GlaFwdWork {
  float* inc = nullptr;   // [BH, NT, F, D] per-chunk increment K~_n^T V_n (fp32)
  float* incz = nullptr;  // [BH, NT, F]   per-chunk increment sum_t K~_t
  float* lam = nullptr;   // [BH, NT]      log decay of each chunk
  float* gs = nullptr;    // [BH, NT]      G just before each chunk
  bf16* s = nullptr;      // [BH, NT, F, D] states when there is no saved buffer
  float* z = nullptr;     // [BH, NT, F]
};

// Schedule of a GLA call. The sequential walk keeps the running state on chip
// and moves the fewest bytes, but runs one chain of chunks per (batch*head,
// block) and so leaves most SMs idle when batch*heads is small. The
// chunk-parallel schedule computes every chunk's state increment at once,
// combines them with an elementwise scan over chunks and then forms every
// chunk's output at once, at the cost of fp32 increments through HBM/L2.
enum GlaSchedule { kScheduleAuto = 0, kScheduleWalk = 1, kScheduleSplit = 2 };
int gla_schedule_override();  // process-wide, set by lz_gla_set_schedule

constexpr long long kF128SplitHeads = 20;

inline bool gla_fwd_split(int B, int H, int L, int F, int D) {
  const int o = gla_schedule_override();
  if (o == kScheduleWalk) return false;
  if (o == kScheduleSplit) return true;
  if (L <= 64) return false;  // a single chunk: both schedules are the same work
  const long long BH = (long long)B * H;
  // F = D = 128: the tensor-core walk (one CTA per head) takes one chain's time
  // whatever BH is, the chunk-parallel kernels time that grows with BH * L;
  // they cross near 20 heads at L = 2048 ... 16384 (forward and backward)
  if (F == 128 && D == 128) return BH <= kF128SplitHeads;
  // F = 256 (the model's feature map): the warp-MMA walk splits the value
  // columns and waits on every chunk's loads; the chunk-parallel kernels were
  // 1.6-3x faster at config-5 shapes, and equal without shared states at B=32
  if (F > 128) return true;
  return BH * ((F + 63) / 64) * ((D + 63) / 64) <= 148;
}

inline bool gla_bwd_split(int B, int H, int L, int F, int D) {
  const int o = gla_schedule_override();
  if (o == kScheduleWalk) return false;
  if (o == kScheduleSplit) return true;
  if (L <= 64) return false;
  if (F == 128 && D == 128) return (long long)B * H <= kF128SplitHeads;
  return (long long)B * H * ((F + 63) / 64) * ((D + 63) / 64) <= 148;
}

inline size_t gla_nt(int L) { return (size_t)((L + 63) / 64); }

// Chunk length of the states in the saved buffer: 128 when the forward runs on
// the tensor-core kernel (F = D = 128, the walk schedule, 16-byte aligned
// inputs), whose states sit on 128-token boundaries; 64 otherwise. The forward
// and the backward both decide with this rule. The saved buffer is sized for
// 64-token chunks, which also holds the 128-token layout.
inline int gla_saved_chunk(int B, int H, int L, int F, int D, const void* fq, const void* fk,
                           const void* v) {
  if (F != 128 || D != 128 || gla_fwd_split(B, H, L, F, D)) return 64;
  return (aligned16(fq) && aligned16(fk) && aligned16(v)) ? 128 : 64;
}

inline size_t gla_saved_layout(int B, int H, int L, int F, int D, unsigned char* base,
                               GlaSaved* out) {
  const size_t BH = (size_t)B * H, NT = gla_nt(L);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  };
  const size_t o_y32 = take(BH * L * D * 4);
  const size_t o_den = take(BH * L * 4);
  const size_t o_g = take(BH * L * 4);
  const size_t o_s = take(BH * NT * F * D * 2);
  const size_t o_z = take(BH * NT * F * 4);
  if (out && base) {
    out->y32 = reinterpret_cast<float*>(base + o_y32);
    out->den = reinterpret_cast<float*>(base + o_den);
    out->g = reinterpret_cast<float*>(base + o_g);
    out->s = reinterpret_cast<bf16*>(base + o_s);
    out->z = reinterpret_cast<float*>(base + o_z);
  }
  return off;
}

inline size_t gla_work_layout(int B, int H, int L, int F, int D, bool split,
                              unsigned char* base, GlaWork* out, bool gqa = false) {
  const size_t BH = (size_t)B * H, NT = gla_nt(L);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  };
  const size_t o_delta = take(BH * L * 4);
  const size_t o_ds = take(BH * NT * F * D * 2);
  const size_t o_dz = take(BH * NT * F * 4);
  const size_t o_dg = take(BH * L * 4);
  const size_t o_dgt = take(BH * NT * 4);
  const size_t o_inc = split ? take(BH * NT * F * D * 4) : 0;
  const size_t o_incz = split ? take(BH * NT * F * 4) : 0;
  const size_t o_lam = split ? take(BH * NT * 4) : 0;
  const size_t o_gk = gqa ? take(BH * L * F * 4) : 0;
  const size_t o_gv = gqa ? take(BH * L * D * 4) : 0;
  if (out && base) {
    out->delta = reinterpret_cast<float*>(base + o_delta);
    out->ds = reinterpret_cast<bf16*>(base + o_ds);
    out->dz = reinterpret_cast<float*>(base + o_dz);
    out->dg = reinterpret_cast<float*>(base + o_dg);
    out->dgt = reinterpret_cast<float*>(base + o_dgt);
    if (split) {
      out->inc = reinterpret_cast<float*>(base + o_inc);
      out->incz = reinterpret_cast<float*>(base + o_incz);
      out->lam = reinterpret_cast<float*>(base + o_lam);
    }
    if (gqa) {
      out->gk = reinterpret_cast<float*>(base + o_gk);
      out->gv = reinterpret_cast<float*>(base + o_gv);
    }
  }
  return off;
}

// Hs: heads that carry states (H, or Hkv when a group of query heads shares
// one state: inference with a gate shared by the heads, gla_split.cu); 0 = H.
inline size_t gla_fwd_work_layout(int B, int H, int L, int F, int D, unsigned char* base,
                                  GlaFwdWork* out, int Hs = 0) {
  const size_t BH = (size_t)B * (Hs > 0 ? Hs : H), NT = gla_nt(L);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  };
  const size_t o_inc = take(BH * NT * F * D * 4);
  const size_t o_incz = take(BH * NT * F * 4);
  const size_t o_lam = take(BH * NT * 4);
  const size_t o_gs = take(BH * NT * 4);
  const size_t o_s = take(BH * NT * F * D * 2);
  const size_t o_z = take(BH * NT * F * 4);
  if (out && base) {
    out->inc = reinterpret_cast<float*>(base + o_inc);
    out->incz = reinterpret_cast<float*>(base + o_incz);
    out->lam = reinterpret_cast<float*>(base + o_lam);
    out->gs = reinterpret_cast<float*>(base + o_gs);
    out->s = reinterpret_cast<bf16*>(base + o_s);
    out->z = reinterpret_cast<float*>(base + o_z);
  }
  return off;
}

// Hkv: heads of fk and v (H % Hkv == 0; query head h reads head h / (H / Hkv)).
int gla_fwd(const bf16* fq, const bf16* fk, const bf16* v, const float* lg, int gph, bf16* y,
            const GlaSaved& sv, const GlaFwdWork& fw, int B, int H, int Hkv, int L, int F, int D,
            cudaStream_t stream);

// Chunk-parallel schedule (gla_split.cu).
int gla_fwd_split_run(const bf16* fq, const bf16* fk, const bf16* v, const float* lg, int gph,
                      bf16* y, const GlaSaved& sv, const GlaFwdWork& fw, int B, int H, int Hkv,
                      int L, int F, int D, cudaStream_t stream);
// Chunk outputs of the chunk-parallel schedule on the tensor cores (F in
// {128, 256} with D = 64, or F = D = 128; 16-byte aligned buffers):
// LZ_ERR_UNSUPPORTED without a launch otherwise. s_in / z_in: the scan's bf16
// states and fp32 normalisers per 64-token chunk of the state heads (sgrp query
// heads per state, 1 = one per query head). With sv.y32 set (training) it also
// writes sv.y32, sv.den and sv.g from the chunk start offsets gs.
int gla_out_tc(const bf16* fq, const bf16* fk, const bf16* v, const float* lg, int gph, int B,
               int H, int Hkv, int sgrp, int L, int F, int D, const bf16* s_in,
               const float* z_in, bf16* y, const GlaSaved& sv, const float* gs,
               cudaStream_t st);
int gla_bwd_split_states(const bf16* fq, const bf16* dy, const GlaSaved& sv, const GlaWork& wk,
                         int B, int H, int L, int F, int D, cudaStream_t stream);

// Sequence-parallel segments (gla_split.cu).
size_t gla_seg_summary_floats(int BH, int F, int D);
int gla_seg_fwd_begin(const bf16* fk, const bf16* v, const float* lg, int gph, float* summary,
                      const GlaFwdWork& fw, int B, int H, int L, int F, int D,
                      cudaStream_t stream);
int gla_seg_fwd_end(const bf16* fq, const bf16* fk, const bf16* v, const float* lg, int gph,
                    const float* seed, bf16* y, const GlaSaved& sv, const GlaFwdWork& fw, int B,
                    int H, int L, int F, int D, cudaStream_t stream);
int gla_seg_bwd_begin(const bf16* fq, const bf16* dy, const GlaSaved& sv, float* summary,
                      const GlaWork& wk, int B, int H, int L, int F, int D, cudaStream_t stream);
int gla_seg_bwd_end(const bf16* fq, const bf16* fk, const bf16* v, int gph, const GlaSaved& sv,
                    const bf16* dy, const float* dseed, int s_seeded, void* dfq, void* dfk,
                    void* dv, int gdt, float* dlg, const GlaWork& wk, int B, int H, int L, int F,
                    int D, cudaStream_t stream);
int gla_seg_combine(const float* summaries, int P, int rank, int reverse, float* seed, int BH,
                    int F, int D, cudaStream_t stream);
int gla_seg_gate_offset(float* dlg, const float* totals, int P, int rank, int rows, int L,
                        cudaStream_t stream);

// Per-chunk gradients and the log-gate gradient, once wk.ds / wk.dz / wk.delta
// hold the state gradients (s_seeded / ds_seeded: the state entering the first
// chunk / the gradient leaving the last chunk is not zero). fk and v carry Hkv
// heads; dfk and dv are written per query head ([B*H, L, *]) in gdt_kv.
int gla_bwd_tail(const bf16* fq, const bf16* fk, const bf16* v, int gph, const GlaSaved& sv,
                 const bf16* dy, void* dfq, void* dfk, void* dv, int gdt, int gdt_kv, float* dlg,
                 const GlaWork& wk, int B, int H, int Hkv, int L, int F, int D, int s_seeded,
                 int ds_seeded, cudaStream_t stream);

// Tensor-core backward for the 128-token chunk layout (gla_bwd_tc.cu).
int gla_bwd_tc_states(const bf16* fq, const bf16* dy, const GlaSaved& sv, const GlaWork& wk,
                      int B, int H, int L, cudaStream_t stream);
int gla_bwd_tc_chunks(const bf16* fq, const bf16* fk, const bf16* v, const bf16* dy,
                      const GlaSaved& sv, const GlaWork& wk, void* dfq, void* dfk, void* dv,
                      int gdt, int gdt_kv, int B, int H, int Hkv, int L, int s_seeded,
                      int ds_seeded, cudaStream_t stream, bool narrow = false);
// The chunk-parallel schedule's tensor-core kernels (chunk outputs, and the
// F = D = 64 chunk gradients) are on unless a test switched them off.
bool gla_split_out_tc_enabled();

// fk and v carry Hkv heads (H % Hkv == 0); dfk and dv are [B*Hkv, L, *], each
// the sum over its group of query heads (wk.gk / wk.gv hold the per-head terms).
int gla_bwd(const bf16* fq, const bf16* fk, const bf16* v, const float* lg, int gph,
            const GlaSaved& sv, const bf16* dy, void* dfq, void* dfk, void* dv, int gdt,
            float* dlg, const GlaWork& wk, int B, int H, int Hkv, int L, int F, int D,
            cudaStream_t stream);

}  // namespace lz
