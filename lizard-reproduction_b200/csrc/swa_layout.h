// Layout of the SWA saved buffer (log-sum-exp and fp32 output per row) and of
// the backward workspace. Both are per query row (B * H * L rows) also when the
// keys and values carry fewer heads (Hkv, GQA).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#include "common.cuh"

namespace lz {

constexpr int kMaxMeta = 32;  // most sink logits one call accepts

struct SwaWork {
  float* delta = nullptr;    // [BH, L]
  float* partial = nullptr;  // [BH * ceil(L/64), n_meta] sink-gradient partials
};

struct SwaSaved {
  float* lse = nullptr;  // [BH, L] log of the softmax denominator (sinks included)
  float* y32 = nullptr;  // [BH, L, D] fp32 output; delta = dy . y32 in the backward
};

inline size_t swa_saved_layout(int B, int H, int L, int D, unsigned char* base, SwaSaved* out) {
  const size_t rows = (size_t)B * H * L;
  const size_t o_y32 = align_up(rows * 4, 256);
  const size_t total = align_up(o_y32 + rows * (size_t)D * 4, 256);
  if (out && base) {
    out->lse = reinterpret_cast<float*>(base);
    out->y32 = reinterpret_cast<float*>(base + o_y32);
  }
  return total;
}

inline size_t swa_work_layout(int B, int H, int L, int n_meta, unsigned char* base,
                              SwaWork* out) {
  const size_t rows = (size_t)B * H * L;
  const size_t nblocks = (size_t)B * H * ((L + 63) / 64);
  const size_t o_delta = 0;
  const size_t o_part = align_up(rows * 4, 256);
  const size_t total = align_up(o_part + nblocks * (size_t)(n_meta > 0 ? n_meta : 1) * 4, 256);
  if (out && base) {
    out->delta = reinterpret_cast<float*>(base + o_delta);
    out->partial = reinterpret_cast<float*>(base + o_part);
  }
  return total;
}

// Arguments of the SWA forward with RoPE inside (lz_swa_rope_fwd).
struct SwaRopeArgs {
  const void *q, *k, *v;  // unrotated, x_dtype, element strides (batch, head, token)
  int x_dtype;
  long long q_sb, q_sh, q_sl, k_sb, k_sh, k_sl, v_sb, v_sh, v_sl;
  const void *cos, *sin;  // [B or broadcast, L, D], cs_dtype
  int cs_dtype;
  long long cs_sb, cs_sl;
  const float* meta;
  int n_meta, window;
  bf16* y;
  bf16 *q_hi, *q_lo, *k_hi, *k_lo;  // optional rotated operands for the backward
  int B, H, Hkv, L, D;
};

// LZ_ERR_UNSUPPORTED (without launching) when the TMA tiles cannot take the
// shape or strides.
int swa_rope_fwd(const SwaRopeArgs& a, const SwaSaved& sv, cudaStream_t st);

// The tensor-core forwards (swa_tc.cu): head dim 64, windows up to 128 (the
// fused rotation for bf16 projections); LZ_ERR_UNSUPPORTED without launching
// for anything else or when
// switched off (lz_swa_set_tc), and the callers then take the 64-row kernels.
bool swa_tc_enabled();
int swa_rope_fwd_tc(const SwaRopeArgs& a, const SwaSaved& sv, cudaStream_t st);
int swa_fwd_tc(const bf16* q, const bf16* k, const bf16* v, const bf16* ql, const bf16* kl,
               const float* meta, int n_meta, int W, bf16* y, const SwaSaved& sv, int B, int H,
               int Hkv, int L, int D, cudaStream_t st);

// dq and dk, dv of the backward on the tensor cores (same shapes as the forward).
int swa_bwd_dq_tc(const bf16* q, const bf16* k, const bf16* v, const bf16* ql, const bf16* kl,
                  const bf16* dy, const float* lse, const float* delta, int W, void* dq, int gdt,
                  int B, int H, int Hkv, int L, int D, cudaStream_t st);
int swa_bwd_dkv_tc(const bf16* q, const bf16* k, const bf16* v, const bf16* ql, const bf16* kl,
                   const bf16* dy, const float* lse, const float* delta, int W, void* dk,
                   void* dv, int gdt, int B, int H, int Hkv, int L, int D, cudaStream_t st);

int swa_fwd(const bf16* q, const bf16* k, const bf16* v, const bf16* ql, const bf16* kl,
            const float* meta, int n_meta, int W, bf16* y, const SwaSaved& sv, int B, int H,
            int Hkv, int L, int D, cudaStream_t st);

int swa_bwd(const bf16* q, const bf16* k, const bf16* v, const bf16* ql, const bf16* kl,
            const float* meta, int n_meta, int W, const SwaSaved& sv, const bf16* dy, void* dq,
            void* dk, void* dv, int gdt, float* dmeta, const SwaWork& wk, int B, int H, int Hkv,
            int L, int D, cudaStream_t st);

}  // namespace lz
