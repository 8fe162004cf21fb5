// Shared device helpers for the Lizard sm_100a kernels: warp-level bf16 MMA
// fragments (mma.sync m16n8k16 + ldmatrix), global->shared tile staging with
// cp.async, error plumbing for the C ABI.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>

#include "../../include/lizard_cuda.h"

typedef __nv_bfloat16 bf16;

namespace lz {

// ---------------------------------------------------------------- host side
void set_error(const std::string& msg);
void clear_error();
void count_launches(uint64_t n);
int check_launch(const char* what);  // cudaGetLastError -> LZ_ERR_CUDA

#define LZ_REQUIRE(cond, code, msg)                                     \
  do {                                                                  \
    if (!(cond)) {                                                      \
      ::lz::set_error(std::string(__func__) + ": " + (msg));            \
      return (code);                                                    \
    }                                                                   \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline int ceil_div(int a, int b) { return (a + b - 1) / b; }
inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// float tiny = smallest normal fp32, the clamp on the GLA row sum
// (reference: TINY in src/kernels/gla.py:7, torch.finfo.tiny in
// src/lizard_attention.py:30).
constexpr float kTiny = 1.1754943508222875e-38f;
constexpr float kLog2e = 1.4426950408889634f;

// Key/value head read by query head row block bh = b * H + h when keys and
// values carry H / grp heads (grouped-query attention): b * (H / grp) + h / grp.
__host__ __device__ __forceinline__ int kv_head(int bh, int H, int grp) {
  const int b = bh / H;
  return b * (H / grp) + (bh - b * H) / grp;
}

// ------------------------------------------------------------ device side
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  // Zero-fills the 16 bytes when !valid (src-size 0).
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)),
               "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// D(16x8, f32) += A(16x16, bf16, row) * B(16x8, bf16, col)
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, "
      "{%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Fragment loaders. Tiles live in shared memory as bf16 rows of `ld`
// elements (ld*2 a multiple of 16 bytes). Lane l supplies one 16-byte row.
//
// A operand, 16(m) x 16(k), from a row-major [m][k] tile.
__device__ __forceinline__ void lda_rm(uint32_t (&a)[4], const bf16* t, int ld, int m0, int k0) {
  const int l = threadIdx.x & 31;
  const int row = m0 + (l & 7) + ((l >> 3) & 1) * 8;
  const int col = k0 + (l >> 4) * 8;
  ldsm_x4(a, smem_u32(t + row * ld + col));
}
// A operand 16(m) x 16(k) where the tile is stored transposed: X[k][m].
__device__ __forceinline__ void lda_tr(uint32_t (&a)[4], const bf16* t, int ld, int m0, int k0) {
  const int l = threadIdx.x & 31;
  const int j = l >> 3;
  const int row = k0 + (l & 7) + (j >> 1) * 8;
  const int col = m0 + (j & 1) * 8;
  ldsm_x4_t(a, smem_u32(t + row * ld + col));
}
// B operands for two adjacent 8-wide n tiles (n0..n0+15) x 16(k), from a
// tile stored as Y[n][k] (i.e. B = Y^T). b[0],b[1] -> n tile 0; b[2],b[3] -> 1.
__device__ __forceinline__ void ldb_nk(uint32_t (&b)[4], const bf16* t, int ld, int n0, int k0) {
  const int l = threadIdx.x & 31;
  const int j = l >> 3;
  const int row = n0 + (l & 7) + (j >> 1) * 8;
  const int col = k0 + (j & 1) * 8;
  ldsm_x4(b, smem_u32(t + row * ld + col));
}
// Same, from a row-major [k][n] tile.
__device__ __forceinline__ void ldb_kn(uint32_t (&b)[4], const bf16* t, int ld, int k0, int n0) {
  const int l = threadIdx.x & 31;
  const int j = l >> 3;
  const int row = k0 + (l & 7) + (j & 1) * 8;
  const int col = n0 + (j >> 1) * 8;
  ldsm_x4_t(b, smem_u32(t + row * ld + col));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float bf16_lo(uint32_t x) {
  return __uint_as_float(x << 16);
}
__device__ __forceinline__ float bf16_hi(uint32_t x) {
  return __uint_as_float(x & 0xffff0000u);
}
__device__ __forceinline__ float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// Stage rows [r0, r0+ROWS) x cols [0, COLS) of a row-major bf16 matrix with
// `ncols` valid columns and row stride `ld` into smem (row stride lds),
// zero-filling rows >= nrows and cols >= ncols. `vec` selects 16-byte
// cp.async (requires ncols % 8 == 0, ld % 8 == 0 and a 16-byte aligned base);
// otherwise element loads are used. Caller commits / waits.
template <int ROWS, int COLS, int NTHREADS>
__device__ __forceinline__ void stage_tile(bf16* s, int lds, const bf16* g, int ld, int r0,
                                           int nrows, int c0, int ncols, bool vec) {
  const int tid = threadIdx.x;
  if (vec) {
    constexpr int CPR = COLS / 8;  // 16-byte chunks per row
    for (int i = tid; i < ROWS * CPR; i += NTHREADS) {
      const int r = i / CPR, c = (i % CPR) * 8;
      const bool ok = (r0 + r < nrows) && (c0 + c < ncols);
      const bf16* src = ok ? g + (size_t)(r0 + r) * ld + c0 + c : g;
      cp_async16(s + r * lds + c, src, ok);
    }
  } else {
    for (int i = tid; i < ROWS * COLS; i += NTHREADS) {
      const int r = i / COLS, c = i % COLS;
      const bool ok = (r0 + r < nrows) && (c0 + c < ncols);
      s[r * lds + c] = ok ? g[(size_t)(r0 + r) * ld + c0 + c] : __float2bfloat16_rn(0.f);
    }
  }
}

template <typename T>
__device__ __forceinline__ void store_val(void* p, size_t i, float x);
template <>
__device__ __forceinline__ void store_val<float>(void* p, size_t i, float x) {
  static_cast<float*>(p)[i] = x;
}
template <>
__device__ __forceinline__ void store_val<bf16>(void* p, size_t i, float x) {
  static_cast<bf16*>(p)[i] = __float2bfloat16_rn(x);
}
__device__ __forceinline__ void store_grad(void* p, size_t i, float x, int dtype) {
  if (dtype == LZ_DTYPE_BF16)
    store_val<bf16>(p, i, x);
  else
    store_val<float>(p, i, x);
}

// Stores x0 (element i) and x1 (element i + 1, when has1) of a gradient row.
__device__ __forceinline__ void store_grad2(void* p, size_t i, float x0, float x1, bool has1,
                                            bool pair, int dtype) {
  if (pair && has1) {
    if (dtype == LZ_DTYPE_BF16)
      *reinterpret_cast<__nv_bfloat162*>(static_cast<bf16*>(p) + i) = __floats2bfloat162_rn(x0, x1);
    else
      *reinterpret_cast<float2*>(static_cast<float*>(p) + i) = make_float2(x0, x1);
  } else {
    store_grad(p, i, x0, dtype);
    if (has1) store_grad(p, i + 1, x1, dtype);
  }
}

// out[r] = sum_d a[r][d] * b[r][d] for the 64 rows of a block (0 for r >=
// nrows), a bf16 and b fp32, both [rows, D] row-major and already offset to
// the block's first row. 128 threads (4 warps x 16 rows). With vec (D % 4 == 0,
// a 8-byte and b 16-byte aligned) a row is split over 16 or 32 lanes that
// load 4 elements each; loads of several rows are in flight at once.
__device__ __forceinline__ void block_row_dots64(const bf16* __restrict__ a,
                                                 const float* __restrict__ b, int nrows, int D,
                                                 bool vec, float* out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (vec && D <= 128) {
    const int hw = D <= 64 ? 16 : 32;  // lanes per row
    const int sub = lane / hw, l = lane % hw;
#pragma unroll 4
    for (int rr = 0; rr < 16; rr += 32 / hw) {
      const int r = warp * 16 + rr + sub;
      float acc = 0.f;
      if (r < nrows) {
        for (int d = 4 * l; d < D; d += 4 * hw) {
          const uint2 x = *reinterpret_cast<const uint2*>(a + (size_t)r * D + d);
          const float4 w = *reinterpret_cast<const float4*>(b + (size_t)r * D + d);
          acc += bf16_lo(x.x) * w.x + bf16_hi(x.x) * w.y + bf16_lo(x.y) * w.z +
                 bf16_hi(x.y) * w.w;
        }
      }
      for (int o = hw / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (l == 0) out[r] = acc;
    }
  } else {
#pragma unroll 2
    for (int rr = 0; rr < 16; ++rr) {
      const int r = warp * 16 + rr;
      float acc = 0.f;
      if (r < nrows)
        for (int d = lane; d < D; d += 32)
          acc += __bfloat162float(a[(size_t)r * D + d]) * b[(size_t)r * D + d];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) out[r] = acc;
    }
  }
}

__device__ __forceinline__ float quad_sum(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  x += __shfl_xor_sync(0xffffffffu, x, 2);
  return x;
}

}  // namespace lz
