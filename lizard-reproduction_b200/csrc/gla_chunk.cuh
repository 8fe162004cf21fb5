// Output of one 64-token GLA chunk for one value slice, shared by the
// sequential walk (gla_fwd.cu) and the chunk-parallel schedule (gla_split.cu).
//
//   a_it  = bf16((fq_i . fk_t) * exp(G_i - G_t)), t <= i      (gla.py:85-90)
//   Q~_i  = bf16(fq_i * exp(G_i - start))                      (gla.py:84)
//   num_i = Q~_i S + sum_t a_it v_t,  den_i = Q~_i . z + sum_t a_it  (gla.py:86-95)
//   y_i   = num_i / max(den_i, FLT_MIN)                        (gla.py:96)
//
// 4 warps, warp w owns rows 16w..16w+15 of the chunk. sG holds the cumulative
// log gate of the chunk's rows and `start` the value just before the chunk,
// both in the same frame (global or chunk-local). The caller has synchronised
// after staging the tiles; nothing in shared memory is written here.
#pragma once

#include "common.cuh"

namespace lz {

template <int FP, int DV>
__device__ __forceinline__ void gla_chunk_output(
    const bf16* sQ, const bf16* sK, const bf16* sV, const bf16* sS, const float* sZ,
    const float* sG, float start, int nvalid, bool with_state, size_t row_base, int D, int d0,
    bf16* __restrict__ y, float* __restrict__ y32, float* __restrict__ den_rows) {
  constexpr int LDQ = FP + 8, LDV = DV + 8;
  constexpr int NTV = DV / 8;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, cq = lane & 3;
  const int i0 = 16 * warp + gq, i1 = i0 + 8;
  const float gi0 = sG[i0], gi1 = sG[i1];

  // (a) intra-chunk scores s = fq fk^T for this warp's 16 rows
  float sacc[8][4];
#pragma unroll
  for (int c = 0; c < 8; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) sacc[c][e] = 0.f;
#pragma unroll 2
  for (int k0 = 0; k0 < FP; k0 += 16) {
    uint32_t a[4];
    lda_rm(a, sQ, LDQ, 16 * warp, k0);
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t bb[4];
      ldb_nk(bb, sK, LDQ, 16 * np, k0);
      mma16816(sacc[2 * np], a, bb[0], bb[1]);
      mma16816(sacc[2 * np + 1], a, bb[2], bb[3]);
    }
  }
  // (b) causal decay, bf16 rounding; the row sum uses the rounded weights
  float den0 = 0.f, den1 = 0.f;
  uint32_t af[4][4];
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    const int t = 8 * nt + 2 * cq;
    const float gt0 = sG[t], gt1 = sG[t + 1];
    const float w00 = (t <= i0 && i0 < nvalid) ? sacc[nt][0] * __expf(gi0 - gt0) : 0.f;
    const float w01 = (t + 1 <= i0 && i0 < nvalid) ? sacc[nt][1] * __expf(gi0 - gt1) : 0.f;
    const float w10 = (t <= i1 && i1 < nvalid) ? sacc[nt][2] * __expf(gi1 - gt0) : 0.f;
    const float w11 = (t + 1 <= i1 && i1 < nvalid) ? sacc[nt][3] * __expf(gi1 - gt1) : 0.f;
    const uint32_t p0 = pack_bf16(w00, w01), p1 = pack_bf16(w10, w11);
    den0 += bf16_lo(p0) + bf16_hi(p0);
    den1 += bf16_lo(p1) + bf16_hi(p1);
    af[nt >> 1][(nt & 1) * 2 + 0] = p0;
    af[nt >> 1][(nt & 1) * 2 + 1] = p1;
  }
  // (c) o = a V
  float oacc[NTV][4];
#pragma unroll
  for (int c = 0; c < NTV; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) oacc[c][e] = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int np = 0; np < NTV / 2; ++np) {
      uint32_t bb[4];
      ldb_kn(bb, sV, LDV, 16 * j, 16 * np);
      mma16816(oacc[2 * np], af[j], bb[0], bb[1]);
      mma16816(oacc[2 * np + 1], af[j], bb[2], bb[3]);
    }
  }
  // (d) inter-chunk: o += Q~ S, den += Q~ . z
  if (with_state) {
    const float qs0 = __expf(gi0 - start), qs1 = __expf(gi1 - start);
#pragma unroll 2
    for (int k0 = 0; k0 < FP; k0 += 16) {
      uint32_t a[4];
      lda_rm(a, sQ, LDQ, 16 * warp, k0);
      a[0] = pack_bf16(bf16_lo(a[0]) * qs0, bf16_hi(a[0]) * qs0);
      a[1] = pack_bf16(bf16_lo(a[1]) * qs1, bf16_hi(a[1]) * qs1);
      a[2] = pack_bf16(bf16_lo(a[2]) * qs0, bf16_hi(a[2]) * qs0);
      a[3] = pack_bf16(bf16_lo(a[3]) * qs1, bf16_hi(a[3]) * qs1);
      const int f = k0 + 2 * cq;
      const float z0 = sZ[f], z1 = sZ[f + 1], z8 = sZ[f + 8], z9 = sZ[f + 9];
      den0 += bf16_lo(a[0]) * z0 + bf16_hi(a[0]) * z1 + bf16_lo(a[2]) * z8 + bf16_hi(a[2]) * z9;
      den1 += bf16_lo(a[1]) * z0 + bf16_hi(a[1]) * z1 + bf16_lo(a[3]) * z8 + bf16_hi(a[3]) * z9;
#pragma unroll
      for (int np = 0; np < NTV / 2; ++np) {
        uint32_t bb[4];
        ldb_kn(bb, sS, LDV, k0, 16 * np);
        mma16816(oacc[2 * np], a, bb[0], bb[1]);
        mma16816(oacc[2 * np + 1], a, bb[2], bb[3]);
      }
    }
  }
  // (e) normalise and store
  den0 = quad_sum(den0);
  den1 = quad_sum(den1);
  const float inv0 = 1.f / fmaxf(den0, kTiny), inv1 = 1.f / fmaxf(den1, kTiny);
  const size_t row0 = (row_base + i0) * D, row1 = (row_base + i1) * D;
  const bool pair = (D & 1) == 0;
#pragma unroll
  for (int nt = 0; nt < NTV; ++nt) {
    const int d = d0 + 8 * nt + 2 * cq;
    if (d >= D) continue;
    const float y00 = oacc[nt][0] * inv0, y01 = oacc[nt][1] * inv0;
    const float y10 = oacc[nt][2] * inv1, y11 = oacc[nt][3] * inv1;
    if (i0 < nvalid) {
      if (pair) {
        *reinterpret_cast<__nv_bfloat162*>(y + row0 + d) = __floats2bfloat162_rn(y00, y01);
        if (y32) *reinterpret_cast<float2*>(y32 + row0 + d) = make_float2(y00, y01);
      } else {
        y[row0 + d] = __float2bfloat16_rn(y00);
        if (d + 1 < D) y[row0 + d + 1] = __float2bfloat16_rn(y01);
        if (y32) {
          y32[row0 + d] = y00;
          if (d + 1 < D) y32[row0 + d + 1] = y01;
        }
      }
    }
    if (i1 < nvalid) {
      if (pair) {
        *reinterpret_cast<__nv_bfloat162*>(y + row1 + d) = __floats2bfloat162_rn(y10, y11);
        if (y32) *reinterpret_cast<float2*>(y32 + row1 + d) = make_float2(y10, y11);
      } else {
        y[row1 + d] = __float2bfloat16_rn(y10);
        if (d + 1 < D) y[row1 + d + 1] = __float2bfloat16_rn(y11);
        if (y32) {
          y32[row1 + d] = y10;
          if (d + 1 < D) y32[row1 + d + 1] = y11;
        }
      }
    }
  }
  if (den_rows && cq == 0) {
    if (i0 < nvalid) den_rows[i0] = den0;
    if (i1 < nvalid) den_rows[i1] = den1;
  }
}

}  // namespace lz
