// The layer's output blend: out = to(x dtype)(float(y_gla) + alpha * float(y_swa)),
// written straight in the layout the output projection reads.
//
// The reference's caller (src/lizard_attention.py:92-97) upcasts both bf16
// branch outputs to the compute dtype, scales the SWA branch by alpha_blend,
// adds, casts to the hidden dtype and transposes [B, H, L, D] to
// [B, L, H * D] for o_proj: four to five elementwise passes. Here one pass
// reads both branches and writes the blended rows at (b, l, h); the product
// and the sum round once each, as the separate torch ops do.
//
// Backward, with g = d out as fp32 (the cast's gradient):
//   d y_gla = bf16(g), d y_swa = bf16(alpha * g)   (the GLA / SWA backward take bf16)
//   d alpha = sum g * float(y_swa), reduced over per-block partials in a fixed order.
#include "common.cuh"

namespace lz {
namespace {

constexpr int kRowsPerBlock = 32;  // rows of D elements per CTA (256 threads)

// Vector path: 8 elements (16 bytes of bf16) per thread, D % 8 == 0.
__global__ void __launch_bounds__(256)
blend_fwd_kernel(const bf16* __restrict__ yg, const bf16* __restrict__ ys,
                 const float* __restrict__ alpha_p, void* __restrict__ out, int out_dtype,
                 int H, int L, int D, long long rows) {
  const float alpha = *alpha_p;
  const int per_row = D / 8;
  const long long n = rows * per_row;
  for (long long e = blockIdx.x * 256ll + threadIdx.x; e < n; e += (long long)gridDim.x * 256) {
    const long long row = e / per_row;  // (b, h, l) row of the branch outputs
    const int c = (int)(e - row * per_row) * 8;
    const int l = (int)(row % L);
    const long long bh = row / L;
    const int h = (int)(bh % H);
    const long long b = bh / H;
    const uint4 ag = *reinterpret_cast<const uint4*>(yg + row * D + c);
    const uint4 as = *reinterpret_cast<const uint4*>(ys + row * D + c);
    const uint32_t wg[4] = {ag.x, ag.y, ag.z, ag.w}, ws[4] = {as.x, as.y, as.z, as.w};
    float r[8];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      r[2 * u] = __fadd_rn(bf16_lo(wg[u]), __fmul_rn(alpha, bf16_lo(ws[u])));
      r[2 * u + 1] = __fadd_rn(bf16_hi(wg[u]), __fmul_rn(alpha, bf16_hi(ws[u])));
    }
    const size_t o = ((size_t)(b * L + l) * H + h) * D + c;  // [B, L, H, D]
    if (out_dtype == LZ_DTYPE_BF16) {
      uint4 w;
      w.x = pack_bf16(r[0], r[1]);
      w.y = pack_bf16(r[2], r[3]);
      w.z = pack_bf16(r[4], r[5]);
      w.w = pack_bf16(r[6], r[7]);
      *reinterpret_cast<uint4*>(static_cast<bf16*>(out) + o) = w;
    } else {
      float4* p = reinterpret_cast<float4*>(static_cast<float*>(out) + o);
      p[0] = make_float4(r[0], r[1], r[2], r[3]);
      p[1] = make_float4(r[4], r[5], r[6], r[7]);
    }
  }
}

// Scalar path for any D.
__global__ void __launch_bounds__(256)
blend_fwd_scalar_kernel(const bf16* __restrict__ yg, const bf16* __restrict__ ys,
                        const float* __restrict__ alpha_p, void* __restrict__ out,
                        int out_dtype, int H, int L, int D, long long n) {
  const float alpha = *alpha_p;
  for (long long e = blockIdx.x * 256ll + threadIdx.x; e < n; e += (long long)gridDim.x * 256) {
    const long long row = e / D;
    const int c = (int)(e - row * D);
    const int l = (int)(row % L);
    const long long bh = row / L;
    const int h = (int)(bh % H);
    const long long b = bh / H;
    const float r = __fadd_rn(__bfloat162float(yg[e]), __fmul_rn(alpha, __bfloat162float(ys[e])));
    store_grad(out, ((size_t)(b * L + l) * H + h) * D + c, r, out_dtype);
  }
}

template <typename T>
__device__ __forceinline__ float load_f(const void* p, size_t i) {
  return static_cast<float>(static_cast<const T*>(p)[i]);
}
template <>
__device__ __forceinline__ float load_f<bf16>(const void* p, size_t i) {
  return __bfloat162float(static_cast<const bf16*>(p)[i]);
}

// One CTA per kRowsPerBlock rows of [B, H, L] order, 256 threads striding over
// their rows * D elements; writes dyg, dys and the block's d alpha partial.
template <typename GT>
__global__ void __launch_bounds__(256)
blend_bwd_kernel(const void* __restrict__ dout, const bf16* __restrict__ ys,
                 const float* __restrict__ alpha_p, bf16* __restrict__ dyg,
                 bf16* __restrict__ dys, float* __restrict__ partial, int H, int L, int D,
                 long long rows) {
  __shared__ float red[256];
  const float alpha = *alpha_p;
  const long long r0 = (long long)blockIdx.x * kRowsPerBlock;
  const int nr = (int)min((long long)kRowsPerBlock, rows - r0);
  float acc = 0.f;
  for (int e = threadIdx.x; e < nr * D; e += 256) {
    const long long row = r0 + e / D;
    const int c = e % D;
    const int l = (int)(row % L);
    const long long bh = row / L;
    const int h = (int)(bh % H);
    const long long b = bh / H;
    const float g = load_f<GT>(dout, ((size_t)(b * L + l) * H + h) * D + c);
    const size_t i = (size_t)row * D + c;
    dyg[i] = __float2bfloat16_rn(g);
    dys[i] = __float2bfloat16_rn(__fmul_rn(alpha, g));
    acc += g * __bfloat162float(ys[i]);
  }
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) partial[blockIdx.x] = red[0];
}

__global__ void __launch_bounds__(256)
blend_alpha_reduce_kernel(const float* __restrict__ partial, long long nblocks,
                          float* __restrict__ dalpha) {
  __shared__ float red[256];
  float s = 0.f;
  for (long long b = threadIdx.x; b < nblocks; b += 256) s += partial[b];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) *dalpha = red[0];
}

unsigned grid_cap(long long items) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long want = (items + 255) / 256, cap = (long long)sms * 8;
  return (unsigned)(want < cap ? (want > 0 ? want : 1) : cap);
}

long long blend_blocks(int B, int H, int L) {
  return ((long long)B * H * L + kRowsPerBlock - 1) / kRowsPerBlock;
}

int check_blend(int B, int H, int L, int D, int dtype) {
  LZ_REQUIRE(B >= 1 && H >= 1 && L >= 1 && D >= 1, LZ_ERR_INVALID_ARGUMENT,
             "sizes must be positive");
  LZ_REQUIRE((long long)B * H * L * D < (1ll << 40), LZ_ERR_INVALID_ARGUMENT, "too large");
  LZ_REQUIRE(dtype == LZ_DTYPE_F32 || dtype == LZ_DTYPE_BF16, LZ_ERR_INVALID_ARGUMENT,
             "dtype must be LZ_DTYPE_F32 or LZ_DTYPE_BF16");
  return LZ_OK;
}

}  // namespace
}  // namespace lz

extern "C" int lz_blend_fwd(const void* y_gla, const void* y_swa, const float* alpha, void* out,
                            int out_dtype, int B, int H, int L, int D, void* stream) {
  using namespace lz;
  clear_error();
  int rc = check_blend(B, H, L, D, out_dtype);
  if (rc) return rc;
  LZ_REQUIRE(y_gla && y_swa && alpha && out, LZ_ERR_INVALID_ARGUMENT, "null pointer");
  auto st = static_cast<cudaStream_t>(stream);
  const long long rows = (long long)B * H * L;
  const bool vec = D % 8 == 0 && aligned16(y_gla) && aligned16(y_swa) && aligned16(out);
  if (vec) {
    blend_fwd_kernel<<<grid_cap(rows * (D / 8)), 256, 0, st>>>(
        static_cast<const bf16*>(y_gla), static_cast<const bf16*>(y_swa), alpha, out, out_dtype,
        H, L, D, rows);
  } else {
    blend_fwd_scalar_kernel<<<grid_cap(rows * D), 256, 0, st>>>(
        static_cast<const bf16*>(y_gla), static_cast<const bf16*>(y_swa), alpha, out, out_dtype,
        H, L, D, rows * D);
  }
  count_launches(1);
  return check_launch("blend_fwd_kernel");
}

extern "C" size_t lz_blend_bwd_workspace_bytes(int B, int H, int L, int D) {
  (void)D;
  if (B < 1 || H < 1 || L < 1) return 0;
  return lz::align_up((size_t)lz::blend_blocks(B, H, L) * 4, 256);
}

extern "C" int lz_blend_bwd(const void* dout, int dout_dtype, const void* y_swa,
                            const float* alpha, void* dy_gla, void* dy_swa, float* dalpha,
                            void* workspace, size_t workspace_bytes, int B, int H, int L, int D,
                            void* stream) {
  using namespace lz;
  clear_error();
  int rc = check_blend(B, H, L, D, dout_dtype);
  if (rc) return rc;
  LZ_REQUIRE(dout && y_swa && alpha && dy_gla && dy_swa && dalpha && workspace,
             LZ_ERR_INVALID_ARGUMENT, "null pointer");
  const long long nb = blend_blocks(B, H, L);
  LZ_REQUIRE(workspace_bytes >= (size_t)nb * 4, LZ_ERR_WORKSPACE, "workspace too small");
  auto st = static_cast<cudaStream_t>(stream);
  const long long rows = (long long)B * H * L;
  float* partial = static_cast<float*>(workspace);
  if (dout_dtype == LZ_DTYPE_BF16)
    blend_bwd_kernel<bf16><<<(unsigned)nb, 256, 0, st>>>(
        dout, static_cast<const bf16*>(y_swa), alpha, static_cast<bf16*>(dy_gla),
        static_cast<bf16*>(dy_swa), partial, H, L, D, rows);
  else
    blend_bwd_kernel<float><<<(unsigned)nb, 256, 0, st>>>(
        dout, static_cast<const bf16*>(y_swa), alpha, static_cast<bf16*>(dy_gla),
        static_cast<bf16*>(dy_swa), partial, H, L, D, rows);
  count_launches(1);
  rc = check_launch("blend_bwd_kernel");
  if (rc) return rc;
  blend_alpha_reduce_kernel<<<1, 256, 0, st>>>(partial, nb, dalpha);
  count_launches(1);
  return check_launch("blend_alpha_reduce_kernel");
}
