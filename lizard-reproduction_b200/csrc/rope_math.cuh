// Element helpers for rows handled 8 elements at a time: 8 consecutive row
// elements in fp32 from 16-byte loads, their bf16 packing and value + residual
// parts, and the rotate-half RoPE of the fused operand passes (the SWA
// forwards with RoPE inside).
#pragma once

#include "common.cuh"

namespace lz {

// 8 consecutive elements of a row as fp32 (16-byte loads; p 16-byte aligned).
__device__ __forceinline__ void load8(const bf16* p, float (&x)[8]) {
  const uint4 w = *reinterpret_cast<const uint4*>(p);
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[2 * i] = bf16_lo(u[i]);
    x[2 * i + 1] = bf16_hi(u[i]);
  }
}
__device__ __forceinline__ void load8(const float* p, float (&x)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
}
// 8 consecutive row elements held as loaded (16 or 32 bytes), converted later:
// lets a thread put several rows' loads in flight in few registers.
template <typename T>
struct Raw8;
template <>
struct Raw8<bf16> {
  uint4 w;
  __device__ __forceinline__ void load(const bf16* p) { w = *reinterpret_cast<const uint4*>(p); }
  __device__ __forceinline__ void get(float (&x)[8]) const {
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[2 * i] = bf16_lo(u[i]);
      x[2 * i + 1] = bf16_hi(u[i]);
    }
  }
};
template <>
struct Raw8<float> {
  float4 a, b;
  __device__ __forceinline__ void load(const float* p) {
    a = *reinterpret_cast<const float4*>(p);
    b = *reinterpret_cast<const float4*>(p + 4);
  }
  __device__ __forceinline__ void get(float (&x)[8]) const {
    x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z,
    x[7] = b.w;
  }
};

__device__ __forceinline__ uint4 pack8(const float (&x)[8]) {
  return make_uint4(pack_bf16(x[0], x[1]), pack_bf16(x[2], x[3]), pack_bf16(x[4], x[5]),
                    pack_bf16(x[6], x[7]));
}
// x - bf16(x) (the residual part), given h = pack8(x)
__device__ __forceinline__ uint4 resid8(const float (&x)[8], uint4 h) {
  const uint32_t u[4] = {h.x, h.y, h.z, h.w};
  float r[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    r[2 * i] = x[2 * i] - bf16_lo(u[i]);
    r[2 * i + 1] = x[2 * i + 1] - bf16_hi(u[i]);
  }
  return pack8(r);
}
// Llama rotate-half RoPE of 8 column pairs (d, d + D/2): x1 / x2 the two
// halves, c / s the cos / sin entries of the same columns; each product and
// each sum rounded once (fp32).
__device__ __forceinline__ void rope8(const float (&x1)[8], const float (&x2)[8],
                                      const float (&c1)[8], const float (&c2)[8],
                                      const float (&s1)[8], const float (&s2)[8], float (&o1)[8],
                                      float (&o2)[8]) {
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    o1[u] = __fadd_rn(__fmul_rn(x1[u], c1[u]), -__fmul_rn(x2[u], s1[u]));
    o2[u] = __fadd_rn(__fmul_rn(x2[u], c2[u]), __fmul_rn(x1[u], s2[u]));
  }
}

}  // namespace lz
