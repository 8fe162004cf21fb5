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
};

inline size_t gla_nt(int L) { return (size_t)((L + 63) / 64); }

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

inline size_t gla_work_layout(int B, int H, int L, int F, int D, unsigned char* base,
                              GlaWork* out) {
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
  if (out && base) {
    out->delta = reinterpret_cast<float*>(base + o_delta);
    out->ds = reinterpret_cast<bf16*>(base + o_ds);
    out->dz = reinterpret_cast<float*>(base + o_dz);
    out->dg = reinterpret_cast<float*>(base + o_dg);
  }
  return off;
}

int gla_fwd(const bf16* fq, const bf16* fk, const bf16* v, const float* lg, int gph, bf16* y,
            const GlaSaved& sv, int B, int H, int L, int F, int D, cudaStream_t stream);

int gla_bwd(const bf16* fq, const bf16* fk, const bf16* v, const float* lg, int gph,
            const GlaSaved& sv, const bf16* dy, void* dfq, void* dfk, void* dv, int gdt,
            float* dlg, const GlaWork& wk, int B, int H, int L, int F, int D,
            cudaStream_t stream);

}  // namespace lz
