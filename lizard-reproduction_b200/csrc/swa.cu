// Sliding-window softmax attention with sink logits ("meta tokens").
//
// y_i = sum_{t in [i-W+1, i]} exp(s_it) v_t / (sum_j exp(meta_j) + sum_t exp(s_it)),
// s_it = q_i . k_t / sqrt(D)                 (reference: src/lizard_attention.py:34-44)
//
// Forward: flash-style online softmax whose running max / sum start from the
// sinks (src/kernels/swa.py:34-38), so the sinks add to the denominator only.
// Backward: delta_i = dy_i . y_i (bf16 y, swa.py:164), dq per query block,
// dk/dv per key block, dmeta_j = -sum_i exp(meta_j - lse_i) delta_i
// (swa.py:175-176) reduced in a fixed order.
#include <mutex>

#include "common.cuh"
#include "swa_layout.h"

namespace lz {

namespace {
constexpr int kB = 64;  // query / key block rows
constexpr float kLn2 = 0.6931471805599453f;

std::mutex g_swa_mu;
template <typename Kern>
int ensure_smem_swa(Kern k, size_t bytes, bool* done) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(g_swa_mu);
  if (dev < 64 && !done[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) {
      set_error(std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
      return LZ_ERR_CUDA;
    }
    done[dev] = true;
  }
  return LZ_OK;
}

__device__ __forceinline__ bool in_window(int i, int t, int L, int W) {
  return t <= i && i - t < W && i < L;
}

// ---------------------------------------------------------------- forward
template <int DP>
__global__ void __launch_bounds__(128)
swa_fwd_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ v,
               const float* __restrict__ meta, int n_meta, int W, float scale_log2, int L, int D,
               int nqb, int vec, bf16* __restrict__ y, float* __restrict__ lse) {
  constexpr int LD = DP + 8, NTD = DP / 8;
  extern __shared__ __align__(128) unsigned char smem[];
  bf16* sQ = reinterpret_cast<bf16*>(smem);
  bf16* sK = sQ + kB * LD;  // 2 stages
  bf16* sV = sK + 2 * kB * LD;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, cq = lane & 3;
  const int qb = blockIdx.x % nqb, bh = blockIdx.x / nqb;
  const int q0 = qb * kB;
  const size_t base = (size_t)bh * L * D;

  // sinks seed the running max / sum (log2 domain)
  float ms = -1e30f;
  for (int j = 0; j < n_meta; ++j) ms = fmaxf(ms, meta[j] * kLog2e);
  float ls = 0.f;
  for (int j = 0; j < n_meta; ++j) ls += exp2f(meta[j] * kLog2e - ms);

  const int lo = max(q0 - W + 1, 0) / kB * kB;
  const int hi = min(q0 + kB, L);
  stage_tile<kB, DP, 128>(sQ, LD, q + base, D, q0, L, 0, D, vec);
  stage_tile<kB, DP, 128>(sK, LD, k + base, D, lo, L, 0, D, vec);
  stage_tile<kB, DP, 128>(sV, LD, v + base, D, lo, L, 0, D, vec);
  cp_async_commit();

  const int i0 = q0 + 16 * warp + gq, i1 = i0 + 8;
  float m0 = ms, m1 = ms, l0 = ls, l1 = ls;
  float o[NTD][4];
#pragma unroll
  for (int c = 0; c < NTD; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[c][e] = 0.f;
  uint32_t qa[DP / 16][4];

  int stage = 0;
  for (int kb = lo; kb < hi; kb += kB, stage ^= 1) {
    if (kb + kB < hi) {
      stage_tile<kB, DP, 128>(sK + (stage ^ 1) * kB * LD, LD, k + base, D, kb + kB, L, 0, D, vec);
      stage_tile<kB, DP, 128>(sV + (stage ^ 1) * kB * LD, LD, v + base, D, kb + kB, L, 0, D, vec);
      cp_async_commit();
      asm volatile("cp.async.wait_group 1;\n" ::);
    } else {
      cp_async_wait_all();
    }
    __syncthreads();
    if (kb == lo) {
#pragma unroll
      for (int kk = 0; kk < DP / 16; ++kk) lda_rm(qa[kk], sQ, LD, 16 * warp, 16 * kk);
    }
    const bf16* tK = sK + stage * kB * LD;
    const bf16* tV = sV + stage * kB * LD;
    float s[8][4];
#pragma unroll
    for (int c = 0; c < 8; ++c)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[c][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < DP / 16; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bb[4];
        ldb_nk(bb, tK, LD, 16 * np, 16 * kk);
        mma16816(s[2 * np], qa[kk], bb[0], bb[1]);
        mma16816(s[2 * np + 1], qa[kk], bb[2], bb[3]);
      }
    }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = kb + 8 * nt + 2 * cq + (e & 1);
        const int i = (e < 2) ? i0 : i1;
        const float x = in_window(i, t, L, W) ? s[nt][e] * scale_log2 : -INFINITY;
        s[nt][e] = x;
        if (e < 2) mx0 = fmaxf(mx0, x); else mx1 = fmaxf(mx1, x);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float al0 = exp2f(m0 - mn0), al1 = exp2f(m1 - mn1);
    float rs0 = 0.f, rs1 = 0.f;
    uint32_t pa[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = exp2f(s[nt][0] - mn0), p1 = exp2f(s[nt][1] - mn0);
      const float p2 = exp2f(s[nt][2] - mn1), p3 = exp2f(s[nt][3] - mn1);
      rs0 += p0 + p1;
      rs1 += p2 + p3;
      pa[nt >> 1][(nt & 1) * 2 + 0] = pack_bf16(p0, p1);
      pa[nt >> 1][(nt & 1) * 2 + 1] = pack_bf16(p2, p3);
    }
    rs0 = quad_sum(rs0);
    rs1 = quad_sum(rs1);
    l0 = l0 * al0 + rs0;
    l1 = l1 * al1 + rs1;
    m0 = mn0;
    m1 = mn1;
#pragma unroll
    for (int c = 0; c < NTD; ++c) {
      o[c][0] *= al0;
      o[c][1] *= al0;
      o[c][2] *= al1;
      o[c][3] *= al1;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int np = 0; np < NTD / 2; ++np) {
        uint32_t bb[4];
        ldb_kn(bb, tV, LD, 16 * j, 16 * np);
        mma16816(o[2 * np], pa[j], bb[0], bb[1]);
        mma16816(o[2 * np + 1], pa[j], bb[2], bb[3]);
      }
    }
    __syncthreads();
  }
  const float inv0 = 1.f / l0, inv1 = 1.f / l1;
#pragma unroll
  for (int nt = 0; nt < NTD; ++nt) {
    const int d = 8 * nt + 2 * cq;
    if (i0 < L) {
      if (d < D) y[base + (size_t)i0 * D + d] = __float2bfloat16_rn(o[nt][0] * inv0);
      if (d + 1 < D) y[base + (size_t)i0 * D + d + 1] = __float2bfloat16_rn(o[nt][1] * inv0);
    }
    if (i1 < L) {
      if (d < D) y[base + (size_t)i1 * D + d] = __float2bfloat16_rn(o[nt][2] * inv1);
      if (d + 1 < D) y[base + (size_t)i1 * D + d + 1] = __float2bfloat16_rn(o[nt][3] * inv1);
    }
  }
  if (lse && cq == 0) {
    if (i0 < L) lse[(size_t)bh * L + i0] = m0 * kLn2 + logf(l0);
    if (i1 < L) lse[(size_t)bh * L + i1] = m1 * kLn2 + logf(l1);
  }
}

// ------------------------------------------------------- backward: prep
// delta_i = dy_i . y_i; per-block partials of sum_i exp(meta_j - lse_i) delta_i.
constexpr int kPrepRows = 64;
__global__ void __launch_bounds__(256)
swa_bwd_prep_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ y,
                    const float* __restrict__ lse, const float* __restrict__ meta, int n_meta,
                    long long rows, int D, float* __restrict__ delta,
                    float* __restrict__ partial) {
  __shared__ float wpart[8][kMaxMeta];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float acc[kMaxMeta];
#pragma unroll
  for (int j = 0; j < kMaxMeta; ++j) acc[j] = 0.f;
  for (int r = warp; r < kPrepRows; r += 8) {
    const long long row = (long long)blockIdx.x * kPrepRows + r;
    if (row >= rows) break;
    float x = 0.f;
    for (int d = lane; d < D; d += 32)
      x += __bfloat162float(dy[row * D + d]) * __bfloat162float(y[row * D + d]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    if (lane == 0) {
      delta[row] = x;
      const float l = lse[row];
#pragma unroll
      for (int j = 0; j < kMaxMeta; ++j)
        if (j < n_meta) acc[j] += __expf(meta[j] - l) * x;
    }
  }
  if (lane == 0)
#pragma unroll
    for (int j = 0; j < kMaxMeta; ++j) wpart[warp][j] = acc[j];
  __syncthreads();
  if (threadIdx.x < n_meta) {
    float s = 0.f;
    for (int w = 0; w < 8; ++w) s += wpart[w][threadIdx.x];
    partial[(size_t)blockIdx.x * n_meta + threadIdx.x] = s;
  }
}

__global__ void swa_dmeta_kernel(const float* __restrict__ partial, int nblocks, int n_meta,
                                 float* __restrict__ dmeta) {
  const int j = threadIdx.x;
  if (j >= n_meta) return;
  float s = 0.f;
  for (int b = 0; b < nblocks; ++b) s += partial[(size_t)b * n_meta + j];
  dmeta[j] = -s;
}

// ------------------------------------------------------- backward: dq
template <int DP>
__global__ void __launch_bounds__(128)
swa_bwd_dq_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k,
                  const bf16* __restrict__ v, const bf16* __restrict__ dy,
                  const float* __restrict__ lse, const float* __restrict__ delta, int W,
                  float scale, int L, int D, int nqb, int vec, void* __restrict__ dq, int gdt) {
  constexpr int LD = DP + 8, NTD = DP / 8;
  extern __shared__ __align__(128) unsigned char smem[];
  bf16* sQ = reinterpret_cast<bf16*>(smem);
  bf16* sDy = sQ + kB * LD;
  bf16* sK = sDy + kB * LD;  // 2 stages
  bf16* sV = sK + 2 * kB * LD;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, cq = lane & 3;
  const int qb = blockIdx.x % nqb, bh = blockIdx.x / nqb;
  const int q0 = qb * kB;
  const size_t base = (size_t)bh * L * D;
  const int lo = max(q0 - W + 1, 0) / kB * kB;
  const int hi = min(q0 + kB, L);
  stage_tile<kB, DP, 128>(sQ, LD, q + base, D, q0, L, 0, D, vec);
  stage_tile<kB, DP, 128>(sDy, LD, dy + base, D, q0, L, 0, D, vec);
  stage_tile<kB, DP, 128>(sK, LD, k + base, D, lo, L, 0, D, vec);
  stage_tile<kB, DP, 128>(sV, LD, v + base, D, lo, L, 0, D, vec);
  cp_async_commit();
  const int i0 = q0 + 16 * warp + gq, i1 = i0 + 8;
  const float lse0 = i0 < L ? lse[(size_t)bh * L + i0] : 0.f;
  const float lse1 = i1 < L ? lse[(size_t)bh * L + i1] : 0.f;
  const float dl0 = i0 < L ? delta[(size_t)bh * L + i0] : 0.f;
  const float dl1 = i1 < L ? delta[(size_t)bh * L + i1] : 0.f;
  float acc[NTD][4];
#pragma unroll
  for (int c = 0; c < NTD; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[c][e] = 0.f;
  int stage = 0;
  for (int kb = lo; kb < hi; kb += kB, stage ^= 1) {
    if (kb + kB < hi) {
      stage_tile<kB, DP, 128>(sK + (stage ^ 1) * kB * LD, LD, k + base, D, kb + kB, L, 0, D, vec);
      stage_tile<kB, DP, 128>(sV + (stage ^ 1) * kB * LD, LD, v + base, D, kb + kB, L, 0, D, vec);
      cp_async_commit();
      asm volatile("cp.async.wait_group 1;\n" ::);
    } else {
      cp_async_wait_all();
    }
    __syncthreads();
    const bf16* tK = sK + stage * kB * LD;
    const bf16* tV = sV + stage * kB * LD;
    float s[8][4], dp[8][4];
#pragma unroll
    for (int c = 0; c < 8; ++c)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[c][e] = dp[c][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < DP / 16; ++kk) {
      uint32_t a[4], g[4];
      lda_rm(a, sQ, LD, 16 * warp, 16 * kk);
      lda_rm(g, sDy, LD, 16 * warp, 16 * kk);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bk[4], bv[4];
        ldb_nk(bk, tK, LD, 16 * np, 16 * kk);
        ldb_nk(bv, tV, LD, 16 * np, 16 * kk);
        mma16816(s[2 * np], a, bk[0], bk[1]);
        mma16816(s[2 * np + 1], a, bk[2], bk[3]);
        mma16816(dp[2 * np], g, bv[0], bv[1]);
        mma16816(dp[2 * np + 1], g, bv[2], bv[3]);
      }
    }
    uint32_t da[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      float x[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = kb + 8 * nt + 2 * cq + (e & 1);
        const int i = (e < 2) ? i0 : i1;
        const float p = in_window(i, t, L, W) ? __expf(s[nt][e] * scale - ((e < 2) ? lse0 : lse1)) : 0.f;
        x[e] = p * (dp[nt][e] - ((e < 2) ? dl0 : dl1));
      }
      da[nt >> 1][(nt & 1) * 2 + 0] = pack_bf16(x[0], x[1]);
      da[nt >> 1][(nt & 1) * 2 + 1] = pack_bf16(x[2], x[3]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int np = 0; np < NTD / 2; ++np) {
        uint32_t bb[4];
        ldb_kn(bb, tK, LD, 16 * j, 16 * np);
        mma16816(acc[2 * np], da[j], bb[0], bb[1]);
        mma16816(acc[2 * np + 1], da[j], bb[2], bb[3]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int nt = 0; nt < NTD; ++nt) {
    const int d = 8 * nt + 2 * cq;
    if (i0 < L) {
      if (d < D) store_grad(dq, base + (size_t)i0 * D + d, acc[nt][0] * scale, gdt);
      if (d + 1 < D) store_grad(dq, base + (size_t)i0 * D + d + 1, acc[nt][1] * scale, gdt);
    }
    if (i1 < L) {
      if (d < D) store_grad(dq, base + (size_t)i1 * D + d, acc[nt][2] * scale, gdt);
      if (d + 1 < D) store_grad(dq, base + (size_t)i1 * D + d + 1, acc[nt][3] * scale, gdt);
    }
  }
}

// ------------------------------------------------------- backward: dk, dv
// Works on transposed scores s^T = k q^T so every operand stays row-major.
template <int DP>
__global__ void __launch_bounds__(128)
swa_bwd_dkv_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k,
                   const bf16* __restrict__ v, const bf16* __restrict__ dy,
                   const float* __restrict__ lse, const float* __restrict__ delta, int W,
                   float scale, int L, int D, int nkb, int vec, void* __restrict__ dk,
                   void* __restrict__ dv, int gdt) {
  constexpr int LD = DP + 8, NTD = DP / 8;
  extern __shared__ __align__(128) unsigned char smem[];
  bf16* sK = reinterpret_cast<bf16*>(smem);
  bf16* sV = sK + kB * LD;
  bf16* sQ = sV + kB * LD;     // 2 stages
  bf16* sDy = sQ + 2 * kB * LD;  // 2 stages
  float* sRow = reinterpret_cast<float*>(sDy + 2 * kB * LD);  // 2 stages x (lse, delta)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, cq = lane & 3;
  const int kbk = blockIdx.x % nkb, bh = blockIdx.x / nkb;
  const int k0 = kbk * kB;
  const size_t base = (size_t)bh * L * D;
  const int qlo = k0;  // query blocks start at the key block (causal)
  const int qhi = min(k0 + kB + W - 1, L);
  auto issue = [&](int qb, int st) {
    stage_tile<kB, DP, 128>(sQ + st * kB * LD, LD, q + base, D, qb, L, 0, D, vec);
    stage_tile<kB, DP, 128>(sDy + st * kB * LD, LD, dy + base, D, qb, L, 0, D, vec);
    cp_async_commit();
    if (tid < kB) {
      const int r = qb + tid;
      sRow[st * 2 * kB + tid] = r < L ? lse[(size_t)bh * L + r] : 0.f;
      sRow[st * 2 * kB + kB + tid] = r < L ? delta[(size_t)bh * L + r] : 0.f;
    }
  };
  stage_tile<kB, DP, 128>(sK, LD, k + base, D, k0, L, 0, D, vec);
  stage_tile<kB, DP, 128>(sV, LD, v + base, D, k0, L, 0, D, vec);
  issue(qlo, 0);
  const int t0 = k0 + 16 * warp + gq, t1 = t0 + 8;  // this thread's key rows
  float dka[NTD][4], dva[NTD][4];
#pragma unroll
  for (int c = 0; c < NTD; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) dka[c][e] = dva[c][e] = 0.f;
  uint32_t ka[DP / 16][4], va[DP / 16][4];
  int stage = 0;
  for (int qb = qlo; qb < qhi; qb += kB, stage ^= 1) {
    if (qb + kB < qhi) {
      issue(qb + kB, stage ^ 1);
      asm volatile("cp.async.wait_group 1;\n" ::);
    } else {
      cp_async_wait_all();
    }
    __syncthreads();
    if (qb == qlo) {
#pragma unroll
      for (int kk = 0; kk < DP / 16; ++kk) {
        lda_rm(ka[kk], sK, LD, 16 * warp, 16 * kk);
        lda_rm(va[kk], sV, LD, 16 * warp, 16 * kk);
      }
    }
    const bf16* tQ = sQ + stage * kB * LD;
    const bf16* tDy = sDy + stage * kB * LD;
    const float* rl = sRow + stage * 2 * kB;
    float s[8][4], dp[8][4];
#pragma unroll
    for (int c = 0; c < 8; ++c)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[c][e] = dp[c][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < DP / 16; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bq[4], bg[4];
        ldb_nk(bq, tQ, LD, 16 * np, 16 * kk);
        ldb_nk(bg, tDy, LD, 16 * np, 16 * kk);
        mma16816(s[2 * np], ka[kk], bq[0], bq[1]);
        mma16816(s[2 * np + 1], ka[kk], bq[2], bq[3]);
        mma16816(dp[2 * np], va[kk], bg[0], bg[1]);
        mma16816(dp[2 * np + 1], va[kk], bg[2], bg[3]);
      }
    }
    uint32_t pa[4][4], dsa[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      float p[4], ds[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int il = 8 * nt + 2 * cq + (e & 1);
        const int i = qb + il;
        const int t = (e < 2) ? t0 : t1;
        const bool m = in_window(i, t, L, W) && t < L;
        p[e] = m ? __expf(s[nt][e] * scale - rl[il]) : 0.f;
        ds[e] = p[e] * (dp[nt][e] - rl[kB + il]);
      }
      pa[nt >> 1][(nt & 1) * 2 + 0] = pack_bf16(p[0], p[1]);
      pa[nt >> 1][(nt & 1) * 2 + 1] = pack_bf16(p[2], p[3]);
      dsa[nt >> 1][(nt & 1) * 2 + 0] = pack_bf16(ds[0], ds[1]);
      dsa[nt >> 1][(nt & 1) * 2 + 1] = pack_bf16(ds[2], ds[3]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int np = 0; np < NTD / 2; ++np) {
        uint32_t bg[4], bq[4];
        ldb_kn(bg, tDy, LD, 16 * j, 16 * np);
        ldb_kn(bq, tQ, LD, 16 * j, 16 * np);
        mma16816(dva[2 * np], pa[j], bg[0], bg[1]);
        mma16816(dva[2 * np + 1], pa[j], bg[2], bg[3]);
        mma16816(dka[2 * np], dsa[j], bq[0], bq[1]);
        mma16816(dka[2 * np + 1], dsa[j], bq[2], bq[3]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int nt = 0; nt < NTD; ++nt) {
    const int d = 8 * nt + 2 * cq;
    if (t0 < L) {
      if (d < D) {
        store_grad(dk, base + (size_t)t0 * D + d, dka[nt][0] * scale, gdt);
        store_grad(dv, base + (size_t)t0 * D + d, dva[nt][0], gdt);
      }
      if (d + 1 < D) {
        store_grad(dk, base + (size_t)t0 * D + d + 1, dka[nt][1] * scale, gdt);
        store_grad(dv, base + (size_t)t0 * D + d + 1, dva[nt][1], gdt);
      }
    }
    if (t1 < L) {
      if (d < D) {
        store_grad(dk, base + (size_t)t1 * D + d, dka[nt][2] * scale, gdt);
        store_grad(dv, base + (size_t)t1 * D + d, dva[nt][2], gdt);
      }
      if (d + 1 < D) {
        store_grad(dk, base + (size_t)t1 * D + d + 1, dka[nt][3] * scale, gdt);
        store_grad(dv, base + (size_t)t1 * D + d + 1, dva[nt][3], gdt);
      }
    }
  }
}

template <int DP>
size_t fwd_smem() { return (size_t)5 * kB * (DP + 8) * 2; }
template <int DP>
size_t dq_smem() { return (size_t)6 * kB * (DP + 8) * 2; }
template <int DP>
size_t dkv_smem() { return (size_t)6 * kB * (DP + 8) * 2 + 4 * kB * 4; }

template <int DP>
int launch_swa_fwd(const bf16* q, const bf16* k, const bf16* v, const float* meta, int n_meta,
                   int W, int BH, int L, int D, int vec, bf16* y, float* lse, cudaStream_t st) {
  static bool done[64] = {false};
  int rc = ensure_smem_swa(swa_fwd_kernel<DP>, fwd_smem<DP>(), done);
  if (rc) return rc;
  const int nqb = ceil_div(L, kB);
  const float scale_log2 = kLog2e / sqrtf((float)D);
  swa_fwd_kernel<DP><<<(unsigned)((long long)BH * nqb), 128, fwd_smem<DP>(), st>>>(
      q, k, v, meta, n_meta, W, scale_log2, L, D, nqb, vec, y, lse);
  count_launches(1);
  return check_launch("swa_fwd_kernel");
}

template <int DP>
int launch_swa_bwd(const bf16* q, const bf16* k, const bf16* v, const bf16* dy,
                   const float* lse, const float* delta, int W, int BH, int L, int D, int vec,
                   void* dq, void* dk, void* dv, int gdt, cudaStream_t st) {
  static bool done_q[64] = {false}, done_kv[64] = {false};
  int rc = ensure_smem_swa(swa_bwd_dq_kernel<DP>, dq_smem<DP>(), done_q);
  if (rc) return rc;
  rc = ensure_smem_swa(swa_bwd_dkv_kernel<DP>, dkv_smem<DP>(), done_kv);
  if (rc) return rc;
  const int nb = ceil_div(L, kB);
  const float scale = 1.f / sqrtf((float)D);
  swa_bwd_dq_kernel<DP><<<(unsigned)((long long)BH * nb), 128, dq_smem<DP>(), st>>>(
      q, k, v, dy, lse, delta, W, scale, L, D, nb, vec, dq, gdt);
  count_launches(1);
  rc = check_launch("swa_bwd_dq_kernel");
  if (rc) return rc;
  swa_bwd_dkv_kernel<DP><<<(unsigned)((long long)BH * nb), 128, dkv_smem<DP>(), st>>>(
      q, k, v, dy, lse, delta, W, scale, L, D, nb, vec, dk, dv, gdt);
  count_launches(1);
  return check_launch("swa_bwd_dkv_kernel");
}

}  // namespace

int swa_fwd(const bf16* q, const bf16* k, const bf16* v, const float* meta, int n_meta, int W,
            bf16* y, float* lse, int B, int H, int L, int D, cudaStream_t st) {
  const int BH = B * H;
  const int vec = (D % 8 == 0) && aligned16(q) && aligned16(k) && aligned16(v);
  if (D <= 32) return launch_swa_fwd<32>(q, k, v, meta, n_meta, W, BH, L, D, vec, y, lse, st);
  if (D <= 64) return launch_swa_fwd<64>(q, k, v, meta, n_meta, W, BH, L, D, vec, y, lse, st);
  if (D <= 128) return launch_swa_fwd<128>(q, k, v, meta, n_meta, W, BH, L, D, vec, y, lse, st);
  set_error("swa_fwd: head dim above 128 is not supported");
  return LZ_ERR_UNSUPPORTED;
}

int swa_bwd(const bf16* q, const bf16* k, const bf16* v, const float* meta, int n_meta, int W,
            const bf16* y, const float* lse, const bf16* dy, void* dq, void* dk, void* dv,
            int gdt, float* dmeta, const SwaWork& wk, int B, int H, int L, int D,
            cudaStream_t st) {
  const int BH = B * H;
  const long long rows = (long long)BH * L;
  const int nblocks = (int)((rows + kPrepRows - 1) / kPrepRows);
  swa_bwd_prep_kernel<<<nblocks, 256, 0, st>>>(dy, y, lse, meta, n_meta, rows, D, wk.delta,
                                               wk.partial);
  count_launches(1);
  int rc = check_launch("swa_bwd_prep_kernel");
  if (rc) return rc;
  const int vec = (D % 8 == 0) && aligned16(q) && aligned16(k) && aligned16(v) && aligned16(dy);
  if (D <= 32)
    rc = launch_swa_bwd<32>(q, k, v, dy, lse, wk.delta, W, BH, L, D, vec, dq, dk, dv, gdt, st);
  else if (D <= 64)
    rc = launch_swa_bwd<64>(q, k, v, dy, lse, wk.delta, W, BH, L, D, vec, dq, dk, dv, gdt, st);
  else if (D <= 128)
    rc = launch_swa_bwd<128>(q, k, v, dy, lse, wk.delta, W, BH, L, D, vec, dq, dk, dv, gdt, st);
  else {
    set_error("swa_bwd: head dim above 128 is not supported");
    return LZ_ERR_UNSUPPORTED;
  }
  if (rc) return rc;
  if (n_meta > 0 && dmeta) {
    swa_dmeta_kernel<<<1, kMaxMeta, 0, st>>>(wk.partial, nblocks, n_meta, dmeta);
    count_launches(1);
    rc = check_launch("swa_dmeta_kernel");
  }
  return rc;
}

}  // namespace lz
