// Layout of the SWA saved buffer (log-sum-exp per row) and backward workspace.
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

inline size_t swa_saved_bytes(int B, int H, int L) {
  return align_up((size_t)B * H * L * 4, 256);
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

int swa_fwd(const bf16* q, const bf16* k, const bf16* v, const bf16* ql, const bf16* kl,
            const float* meta, int n_meta, int W, bf16* y, float* lse, int B, int H, int L, int D,
            cudaStream_t st);

int swa_bwd(const bf16* q, const bf16* k, const bf16* v, const bf16* ql, const bf16* kl,
            const float* meta, int n_meta, int W, const float* lse, const bf16* dy, void* dq,
            void* dk, void* dv, int gdt, float* dmeta, const SwaWork& wk, int B, int H, int L,
            int D, cudaStream_t st);

}  // namespace lz
