// Rotary position embedding fused with the bf16 hi / lo split of the SWA
// kernels' query and key operands.
//
// The reference's caller rotates q and k in the layer's compute dtype
// (src/lizard_attention.py:87-88, Llama's rotate-half form
// r = x * cos + rotate_half(x) * sin, rotate_half(x) = [-x2, x1]) and the SWA
// wrapper then splits each fp32 operand into bf16(r) and bf16(r - bf16(r)).
// Here one pass reads x (fp32 or bf16, any batch / head / token strides, so
// the projection output [B, L, H * Dh] is read in place as [B, H, L, Dh]) and
// cos / sin ([B, L, Dh], fp32 or bf16, batch stride 0 to broadcast) and writes
// both bf16 parts contiguous [B, H, L, Dh]. Products and the sum round once
// each, as the reference's separate torch multiplies and add do.
//
// Backward: dx = R^T dr,
//   dx[d]     = dr[d] cos[d] + dr[d + h] sin[d + h]
//   dx[d + h] = dr[d + h] cos[d + h] - dr[d] sin[d]      (d < h = Dh / 2),
// the autograd of the same expression; cos and sin take no gradient.
#include "common.cuh"

namespace lz {
namespace {

template <typename T>
__device__ __forceinline__ float ld(const T* p, size_t i);
template <>
__device__ __forceinline__ float ld<float>(const float* p, size_t i) { return p[i]; }
template <>
__device__ __forceinline__ float ld<bf16>(const bf16* p, size_t i) {
  return __bfloat162float(p[i]);
}

// One thread per (row, pair of adjacent rotation indices j, j + 1 < h):
// it reads x[j..j+1] and x[j+h..j+h+1] and writes four bf16 pairs.
template <typename XT, typename CT, int V>
__global__ void __launch_bounds__(256)
rope_split_kernel(const XT* __restrict__ x, long long sb, long long sh, long long sl,
                  const CT* __restrict__ cs, const CT* __restrict__ sn, long long csb,
                  long long csl, bf16* __restrict__ hi, bf16* __restrict__ lo, int Hx, int L,
                  int Dh, long long nitems) {
  const int half = Dh / 2, per_row = half / V;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < nitems;
       e += (long long)gridDim.x * blockDim.x) {
    const long long row = e / per_row;
    const int j = (int)(e - row * per_row) * V;
    const int l = (int)(row % L);
    const long long bh = row / L;
    const int h = (int)(bh % Hx), b = (int)(bh / Hx);
    const XT* xr = x + b * sb + h * sh + l * sl;
    const size_t cr = (size_t)(b * csb + l * csl);
    float r1[V], r2[V];
#pragma unroll
    for (int u = 0; u < V; ++u) {
      const float x1 = ld(xr, j + u), x2 = ld(xr, j + u + half);
      const float c1 = ld(cs, cr + j + u), s1 = ld(sn, cr + j + u);
      const float c2 = ld(cs, cr + j + u + half), s2 = ld(sn, cr + j + u + half);
      r1[u] = __fadd_rn(__fmul_rn(x1, c1), -__fmul_rn(x2, s1));
      r2[u] = __fadd_rn(__fmul_rn(x2, c2), __fmul_rn(x1, s2));
    }
    const size_t o = (size_t)row * Dh + j;
#pragma unroll
    for (int u = 0; u < V; ++u) {
      const bf16 a = __float2bfloat16_rn(r1[u]), c = __float2bfloat16_rn(r2[u]);
      hi[o + u] = a;
      hi[o + u + half] = c;
      if (lo) {
        lo[o + u] = __float2bfloat16_rn(r1[u] - __bfloat162float(a));
        lo[o + u + half] = __float2bfloat16_rn(r2[u] - __bfloat162float(c));
      }
    }
  }
}

template <typename CT, int V>
__global__ void __launch_bounds__(256)
rope_bwd_kernel(const float* __restrict__ dr, const CT* __restrict__ cs,
                const CT* __restrict__ sn, long long csb, long long csl, void* __restrict__ dx,
                int dx_dtype, int Hx, int L, int Dh, long long nitems) {
  const int half = Dh / 2, per_row = half / V;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < nitems;
       e += (long long)gridDim.x * blockDim.x) {
    const long long row = e / per_row;
    const int j = (int)(e - row * per_row) * V;
    const int l = (int)(row % L);
    const int b = (int)(row / L / Hx);
    const size_t cr = (size_t)(b * csb + l * csl);
    const size_t o = (size_t)row * Dh + j;
#pragma unroll
    for (int u = 0; u < V; ++u) {
      const float g1 = dr[o + u], g2 = dr[o + u + half];
      const float c1 = ld(cs, cr + j + u), s1 = ld(sn, cr + j + u);
      const float c2 = ld(cs, cr + j + u + half), s2 = ld(sn, cr + j + u + half);
      store_grad(dx, o + u, __fadd_rn(__fmul_rn(g1, c1), __fmul_rn(g2, s2)), dx_dtype);
      store_grad(dx, o + u + half, __fadd_rn(__fmul_rn(g2, c2), -__fmul_rn(g1, s1)), dx_dtype);
    }
  }
}

unsigned grid_for(long long nitems) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long want = (nitems + 255) / 256, cap = (long long)sms * 8;
  return (unsigned)(want < cap ? (want > 0 ? want : 1) : cap);
}

template <typename XT, typename CT>
int launch_split(const void* x, long long sb, long long sh, long long sl, const void* cs,
                 const void* sn, long long csb, long long csl, bf16* hi, bf16* lo, int B,
                 int Hx, int L, int Dh, cudaStream_t st) {
  const int half = Dh / 2;
  const long long rows = (long long)B * Hx * L;
  if (half % 2 == 0) {
    const long long n = rows * (half / 2);
    rope_split_kernel<XT, CT, 2><<<grid_for(n), 256, 0, st>>>(
        static_cast<const XT*>(x), sb, sh, sl, static_cast<const CT*>(cs),
        static_cast<const CT*>(sn), csb, csl, hi, lo, Hx, L, Dh, n);
  } else {
    const long long n = rows * half;
    rope_split_kernel<XT, CT, 1><<<grid_for(n), 256, 0, st>>>(
        static_cast<const XT*>(x), sb, sh, sl, static_cast<const CT*>(cs),
        static_cast<const CT*>(sn), csb, csl, hi, lo, Hx, L, Dh, n);
  }
  count_launches(1);
  return check_launch("rope_split_kernel");
}

template <typename CT>
int launch_bwd(const float* dr, const void* cs, const void* sn, long long csb, long long csl,
               void* dx, int dx_dtype, int B, int Hx, int L, int Dh, cudaStream_t st) {
  const int half = Dh / 2;
  const long long rows = (long long)B * Hx * L;
  if (half % 2 == 0) {
    const long long n = rows * (half / 2);
    rope_bwd_kernel<CT, 2><<<grid_for(n), 256, 0, st>>>(
        dr, static_cast<const CT*>(cs), static_cast<const CT*>(sn), csb, csl, dx, dx_dtype, Hx,
        L, Dh, n);
  } else {
    const long long n = rows * half;
    rope_bwd_kernel<CT, 1><<<grid_for(n), 256, 0, st>>>(
        dr, static_cast<const CT*>(cs), static_cast<const CT*>(sn), csb, csl, dx, dx_dtype, Hx,
        L, Dh, n);
  }
  count_launches(1);
  return check_launch("rope_bwd_kernel");
}

int check_rope(int B, int Hx, int L, int Dh, int cs_dtype) {
  LZ_REQUIRE(B >= 1 && Hx >= 1 && L >= 1, LZ_ERR_INVALID_ARGUMENT, "sizes must be positive");
  LZ_REQUIRE(Dh >= 2 && Dh % 2 == 0, LZ_ERR_INVALID_ARGUMENT,
             "the rotated head dim must be even");
  LZ_REQUIRE((long long)B * Hx * L * Dh < (1ll << 40), LZ_ERR_INVALID_ARGUMENT,
             "tensor too large");
  LZ_REQUIRE(cs_dtype == LZ_DTYPE_F32 || cs_dtype == LZ_DTYPE_BF16, LZ_ERR_INVALID_ARGUMENT,
             "cos / sin dtype must be LZ_DTYPE_F32 or LZ_DTYPE_BF16");
  return LZ_OK;
}

}  // namespace
}  // namespace lz

extern "C" int lz_rope_split(const void* x, int x_dtype, long long x_sb, long long x_sh,
                             long long x_sl, const void* cos, const void* sin, int cs_dtype,
                             long long cs_sb, long long cs_sl, void* hi, void* lo, int B, int Hx,
                             int L, int Dh, void* stream) {
  using namespace lz;
  clear_error();
  int rc = check_rope(B, Hx, L, Dh, cs_dtype);
  if (rc) return rc;
  LZ_REQUIRE(x && cos && sin && hi, LZ_ERR_INVALID_ARGUMENT, "null pointer");
  LZ_REQUIRE(x_dtype == LZ_DTYPE_F32 || x_dtype == LZ_DTYPE_BF16, LZ_ERR_INVALID_ARGUMENT,
             "x dtype must be LZ_DTYPE_F32 or LZ_DTYPE_BF16");
  auto st = static_cast<cudaStream_t>(stream);
  auto h = static_cast<bf16*>(hi);
  auto l = static_cast<bf16*>(lo);
  if (x_dtype == LZ_DTYPE_F32)
    return cs_dtype == LZ_DTYPE_F32
               ? launch_split<float, float>(x, x_sb, x_sh, x_sl, cos, sin, cs_sb, cs_sl, h, l, B,
                                            Hx, L, Dh, st)
               : launch_split<float, bf16>(x, x_sb, x_sh, x_sl, cos, sin, cs_sb, cs_sl, h, l, B,
                                           Hx, L, Dh, st);
  return cs_dtype == LZ_DTYPE_F32
             ? launch_split<bf16, float>(x, x_sb, x_sh, x_sl, cos, sin, cs_sb, cs_sl, h, l, B, Hx,
                                         L, Dh, st)
             : launch_split<bf16, bf16>(x, x_sb, x_sh, x_sl, cos, sin, cs_sb, cs_sl, h, l, B, Hx,
                                        L, Dh, st);
}

extern "C" int lz_rope_bwd(const float* dr, const void* cos, const void* sin, int cs_dtype,
                           long long cs_sb, long long cs_sl, void* dx, int dx_dtype, int B,
                           int Hx, int L, int Dh, void* stream) {
  using namespace lz;
  clear_error();
  int rc = check_rope(B, Hx, L, Dh, cs_dtype);
  if (rc) return rc;
  LZ_REQUIRE(dr && cos && sin && dx, LZ_ERR_INVALID_ARGUMENT, "null pointer");
  LZ_REQUIRE(dx_dtype == LZ_DTYPE_F32 || dx_dtype == LZ_DTYPE_BF16, LZ_ERR_INVALID_ARGUMENT,
             "dx dtype must be LZ_DTYPE_F32 or LZ_DTYPE_BF16");
  auto st = static_cast<cudaStream_t>(stream);
  return cs_dtype == LZ_DTYPE_F32
             ? launch_bwd<float>(dr, cos, sin, cs_sb, cs_sl, dx, dx_dtype, B, Hx, L, Dh, st)
             : launch_bwd<bf16>(dr, cos, sin, cs_sb, cs_sl, dx, dx_dtype, B, Hx, L, Dh, st);
}
