// Sliding-window softmax attention with sink logits ("meta tokens").
//
// y_i = sum_{t in [i-W+1, i]} exp(s_it) v_t / (sum_j exp(meta_j) + sum_t exp(s_it)),
// s_it = q_i . k_t / sqrt(D)                 (reference: src/lizard_attention.py:34-44)
//
// Forward: flash-style online softmax whose running max / sum start from the
// sinks (src/kernels/swa.py:34-38), so the sinks add to the denominator only.
// The forward also keeps y in fp32 when the caller trains.
// Backward (src/kernels/swa.py:62-133, 158-179), four launches:
//   delta      : delta_i = dy_i . y32_i in fp32 (the reference uses dy . bf16(y),
//                swa.py:164, which loses the small 1 - P differences the sink
//                gradient is made of), and per-block sink-gradient partials.
//   dq kernel  : per query block, dq over the key blocks in its window.
//   dkv kernel : per key block, dk and dv over the query blocks in its window.
//   dmeta      : dmeta_j = -sum_i exp(meta_j - lse_i) delta_i (swa.py:175-176),
//                reduced over the per-block partials in a fixed order.
// Grouped keys and values (GQA): k and v may carry Hkv heads with H % Hkv == 0;
// query head h reads key/value head h / (H / Hkv), which is what the
// reference's caller builds with repeat_interleave (src/lizard_attention.py:
// 73-76). The dk / dv of a key/value head sum over its group of query heads
// inside one CTA, in a fixed order (the autograd of repeat_interleave).
// Optional bf16 residuals q_lo, k_lo (q = q_hi + q_lo) make the logits
// q_hi.k_hi + q_hi.k_lo + q_lo.k_hi, about 16 mantissa bits, for callers whose
// queries and keys are fp32: softmax turns logit rounding into relative
// weight errors, which the sink gradient accumulates.
#include <mutex>

#include "common.cuh"
#include "rope_math.cuh"
#include "swa_layout.h"
#include "tc.cuh"

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

// Element offset of the key/value head that query row block bh reads.
__device__ __forceinline__ size_t kv_base(int bh, int H, int grp, int L, int D) {
  return (size_t)kv_head(bh, H, grp) * L * D;
}

__device__ __forceinline__ bool in_window(int i, int t, int L, int W) {
  return t <= i && i - t < W && i < L;
}

template <int DP>
struct Tile {
  static constexpr int LD = DP + 8;
  static constexpr size_t bytes = (size_t)kB * LD * 2;
};

// Scores of this warp's 16 query rows against the 64 rows of tK (keys):
// s = qa . k_hi (+ qa . k_lo + qla . k_hi).
template <int DP, bool SPLIT>
__device__ __forceinline__ void scores(float (&s)[8][4], const uint32_t (&qa)[DP / 16][4],
                                       const uint32_t (&qla)[DP / 16][4], const bf16* tK,
                                       const bf16* tKl) {
  constexpr int LD = Tile<DP>::LD;
#pragma unroll
  for (int c = 0; c < 8; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) s[c][e] = 0.f;
#pragma unroll
  for (int kk = 0; kk < DP / 16; ++kk) {
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t bk[4];
      ldb_nk(bk, tK, LD, 16 * np, 16 * kk);
      mma16816(s[2 * np], qa[kk], bk[0], bk[1]);
      mma16816(s[2 * np + 1], qa[kk], bk[2], bk[3]);
      if constexpr (SPLIT) {
        uint32_t bl[4];
        ldb_nk(bl, tKl, LD, 16 * np, 16 * kk);
        mma16816(s[2 * np], qa[kk], bl[0], bl[1]);
        mma16816(s[2 * np + 1], qa[kk], bl[2], bl[3]);
        mma16816(s[2 * np], qla[kk], bk[0], bk[1]);
        mma16816(s[2 * np + 1], qla[kk], bk[2], bk[3]);
      }
    }
  }
}

// ---------------------------------------------------------------- forward
template <int DP, bool SPLIT>
struct FwdSmem {
  static constexpr size_t T = Tile<DP>::bytes;
  static constexpr size_t q = 0, ql = q + T, k = ql + (SPLIT ? T : 0), kl = k + 2 * T,
                          v = kl + (SPLIT ? 2 * T : 0), bytes = v + 2 * T;
};

// P enters the P.V product as bf16 hi + lo parts, so the output (and the fp32
// copy kept for the backward's delta) carries about 16 mantissa bits of P
// instead of 8: the sink gradient is a small difference of such sums. The same
// product runs with and without a saved buffer, so y does not depend on it.
template <int DP, bool SPLIT>
__global__ void __launch_bounds__(128)
swa_fwd_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ v,
               const bf16* __restrict__ ql, const bf16* __restrict__ kl,
               const float* __restrict__ meta, int n_meta, int W, float scale_log2, int H,
               int grp, int L, int D, int nqb, int vec, bf16* __restrict__ y,
               float* __restrict__ lse,
               float* __restrict__ y32) {
  using SM = FwdSmem<DP, SPLIT>;
  constexpr int LD = Tile<DP>::LD, NTD = DP / 8;
  constexpr size_t T = Tile<DP>::bytes;
  extern __shared__ __align__(128) unsigned char smem[];
  bf16* sQ = reinterpret_cast<bf16*>(smem + SM::q);
  bf16* sQl = reinterpret_cast<bf16*>(smem + SM::ql);
  auto sK = [&](int s) { return reinterpret_cast<bf16*>(smem + SM::k + s * T); };
  auto sKl = [&](int s) { return reinterpret_cast<bf16*>(smem + SM::kl + s * T); };
  auto sV = [&](int s) { return reinterpret_cast<bf16*>(smem + SM::v + s * T); };
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, cq = lane & 3;
  const int qb = blockIdx.x % nqb, bh = blockIdx.x / nqb;
  const int q0 = qb * kB;
  const size_t base = (size_t)bh * L * D, kvb = kv_base(bh, H, grp, L, D);

  // sinks seed the running max / sum (log2 domain)
  float ms = -1e30f;
  for (int j = 0; j < n_meta; ++j) ms = fmaxf(ms, meta[j] * kLog2e);
  float ls = 0.f;
  for (int j = 0; j < n_meta; ++j) ls += exp2f(meta[j] * kLog2e - ms);

  const int lo = max(q0 - W + 1, 0) / kB * kB;
  const int hi = min(q0 + kB, L);
  auto issue = [&](int kb, int s) {
    stage_tile<kB, DP, 128>(sK(s), LD, k + kvb, D, kb, L, 0, D, vec);
    if (SPLIT) stage_tile<kB, DP, 128>(sKl(s), LD, kl + kvb, D, kb, L, 0, D, vec);
    stage_tile<kB, DP, 128>(sV(s), LD, v + kvb, D, kb, L, 0, D, vec);
  };
  stage_tile<kB, DP, 128>(sQ, LD, q + base, D, q0, L, 0, D, vec);
  if (SPLIT) stage_tile<kB, DP, 128>(sQl, LD, ql + base, D, q0, L, 0, D, vec);
  issue(lo, 0);
  cp_async_commit();

  const int i0 = q0 + 16 * warp + gq, i1 = i0 + 8;
  float m0 = ms, m1 = ms, l0 = ls, l1 = ls;
  float o[NTD][4];
#pragma unroll
  for (int c = 0; c < NTD; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[c][e] = 0.f;
  uint32_t qa[DP / 16][4], qla[DP / 16][4];

  int stage = 0;
  for (int kb = lo; kb < hi; kb += kB, stage ^= 1) {
    if (kb + kB < hi) {
      issue(kb + kB, stage ^ 1);
      cp_async_commit();
      asm volatile("cp.async.wait_group 1;\n" ::);
    } else {
      cp_async_wait_all();
    }
    __syncthreads();
    if (kb == lo) {
#pragma unroll
      for (int kk = 0; kk < DP / 16; ++kk) {
        lda_rm(qa[kk], sQ, LD, 16 * warp, 16 * kk);
        if (SPLIT) lda_rm(qla[kk], sQl, LD, 16 * warp, 16 * kk);
      }
    }
    float s[8][4];
    scores<DP, SPLIT>(s, qa, qla, sK(stage), sKl(stage));
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
    uint32_t pa[4][4], pl[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = exp2f(s[nt][0] - mn0), p1 = exp2f(s[nt][1] - mn0);
      const float p2 = exp2f(s[nt][2] - mn1), p3 = exp2f(s[nt][3] - mn1);
      rs0 += p0 + p1;
      rs1 += p2 + p3;
      const uint32_t h01 = pack_bf16(p0, p1), h23 = pack_bf16(p2, p3);
      pa[nt >> 1][(nt & 1) * 2 + 0] = h01;
      pa[nt >> 1][(nt & 1) * 2 + 1] = h23;
      {
        pl[nt >> 1][(nt & 1) * 2 + 0] = pack_bf16(p0 - bf16_lo(h01), p1 - bf16_hi(h01));
        pl[nt >> 1][(nt & 1) * 2 + 1] = pack_bf16(p2 - bf16_lo(h23), p3 - bf16_hi(h23));
      }
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
    const bf16* tV = sV(stage);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int np = 0; np < NTD / 2; ++np) {
        uint32_t bb[4];
        ldb_kn(bb, tV, LD, 16 * j, 16 * np);
        mma16816(o[2 * np], pa[j], bb[0], bb[1]);
        mma16816(o[2 * np + 1], pa[j], bb[2], bb[3]);
        mma16816(o[2 * np], pl[j], bb[0], bb[1]);
        mma16816(o[2 * np + 1], pl[j], bb[2], bb[3]);
      }
    }
    __syncthreads();
  }
  const float inv0 = 1.f / l0, inv1 = 1.f / l1;
  const bool pair = (D & 1) == 0;
#pragma unroll
  for (int nt = 0; nt < NTD; ++nt) {
    const int d = 8 * nt + 2 * cq;
    if (d >= D) continue;
    const bool has1 = d + 1 < D;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int i = h ? i1 : i0;
      if (i >= L) continue;
      const float inv = h ? inv1 : inv0;
      const float a = o[nt][2 * h] * inv, b = o[nt][2 * h + 1] * inv;
      const size_t at = base + (size_t)i * D + d;
      if (pair && has1) {
        *reinterpret_cast<__nv_bfloat162*>(y + at) = __floats2bfloat162_rn(a, b);
        if (y32) *reinterpret_cast<float2*>(y32 + at) = make_float2(a, b);
      } else {
        y[at] = __float2bfloat16_rn(a);
        if (has1) y[at + 1] = __float2bfloat16_rn(b);
        if (y32) {
          y32[at] = a;
          if (has1) y32[at + 1] = b;
        }
      }
    }
  }
  if (lse && cq == 0) {
    if (i0 < L) lse[(size_t)bh * L + i0] = m0 * kLn2 + logf(l0);
    if (i1 < L) lse[(size_t)bh * L + i1] = m1 * kLn2 + logf(l1);
  }
}

// ------------------------------------------------------- backward: delta
// delta_i = dy_i . y32_i (the fp32 output saved by the forward; the reference
// uses dy . bf16(y), swa.py:164) and, per 64-row block, the sink-gradient
// partials sum_i exp(meta_j - lse_i) delta_i (swa.py:175-176) in a fixed
// order. 4 warps, 16 rows each.
__global__ void __launch_bounds__(128)
swa_bwd_delta_kernel(const bf16* __restrict__ dy, const float* __restrict__ y32,
                     const float* __restrict__ lse, const float* __restrict__ meta, int n_meta,
                     int L, int D, int nqb, int vec, float* __restrict__ delta,
                     float* __restrict__ partial) {
  __shared__ float sDel[kB], sLse[kB];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qb = blockIdx.x % nqb, bh = blockIdx.x / nqb;
  const int q0 = qb * kB, nrows = min(kB, L - q0);
  const size_t rowb = (size_t)bh * L + q0;
  if (tid < kB) sLse[tid] = tid < nrows ? lse[rowb + tid] : 0.f;
  block_row_dots64(dy + rowb * D, y32 + rowb * D, nrows, D, vec, sDel);
  __syncthreads();
  if (tid < nrows) delta[rowb + tid] = sDel[tid];
  // warp w sums sinks j = w, w+4, ... over the block's rows (2 rows per lane)
  for (int j = warp; j < n_meta; j += 4) {
    float x = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int t = lane + 32 * h;
      if (t < nrows) x += __expf(meta[j] - sLse[t]) * sDel[t];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    if (lane == 0) partial[(size_t)blockIdx.x * n_meta + j] = x;
  }
}

// ------------------------------------------------------- backward: dq
// dq_i = scale * sum_t P_it (dy_i . v_t - delta_i) k_t   (swa.py:62-95)
template <int DP, bool SPLIT>
struct DqSmem {
  static constexpr size_t T = Tile<DP>::bytes;
  static constexpr size_t q = 0, ql = q + T, dy = ql + (SPLIT ? T : 0), k = dy + T,
                          kl = k + 2 * T, v = kl + (SPLIT ? 2 * T : 0), bytes = v + 2 * T;
};

template <int DP, bool SPLIT>
__global__ void __launch_bounds__(128)
swa_bwd_dq_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k,
                  const bf16* __restrict__ v, const bf16* __restrict__ ql,
                  const bf16* __restrict__ kl, const bf16* __restrict__ dy,
                  const float* __restrict__ lse, const float* __restrict__ delta, int W,
                  float scale, int H, int grp, int L, int D, int nqb, int vec,
                  void* __restrict__ dq, int gdt) {
  using SM = DqSmem<DP, SPLIT>;
  constexpr int LD = Tile<DP>::LD, NTD = DP / 8;
  constexpr size_t T = Tile<DP>::bytes;
  extern __shared__ __align__(128) unsigned char smem[];
  bf16* sQ = reinterpret_cast<bf16*>(smem + SM::q);
  bf16* sQl = reinterpret_cast<bf16*>(smem + SM::ql);
  bf16* sDy = reinterpret_cast<bf16*>(smem + SM::dy);
  auto sK = [&](int s) { return reinterpret_cast<bf16*>(smem + SM::k + s * T); };
  auto sKl = [&](int s) { return reinterpret_cast<bf16*>(smem + SM::kl + s * T); };
  auto sV = [&](int s) { return reinterpret_cast<bf16*>(smem + SM::v + s * T); };
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, cq = lane & 3;
  const int qb = blockIdx.x % nqb, bh = blockIdx.x / nqb;
  const int q0 = qb * kB;
  const size_t base = (size_t)bh * L * D, kvb = kv_base(bh, H, grp, L, D);
  const int lo = max(q0 - W + 1, 0) / kB * kB;
  const int hi = min(q0 + kB, L);
  auto issue = [&](int kb, int s) {
    stage_tile<kB, DP, 128>(sK(s), LD, k + kvb, D, kb, L, 0, D, vec);
    if (SPLIT) stage_tile<kB, DP, 128>(sKl(s), LD, kl + kvb, D, kb, L, 0, D, vec);
    stage_tile<kB, DP, 128>(sV(s), LD, v + kvb, D, kb, L, 0, D, vec);
  };
  stage_tile<kB, DP, 128>(sQ, LD, q + base, D, q0, L, 0, D, vec);
  if (SPLIT) stage_tile<kB, DP, 128>(sQl, LD, ql + base, D, q0, L, 0, D, vec);
  stage_tile<kB, DP, 128>(sDy, LD, dy + base, D, q0, L, 0, D, vec);
  issue(lo, 0);
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
  uint32_t qa[DP / 16][4], qla[DP / 16][4], ga[DP / 16][4];

  int stage = 0;
  for (int kb = lo; kb < hi; kb += kB, stage ^= 1) {
    if (kb + kB < hi) {
      issue(kb + kB, stage ^ 1);
      cp_async_commit();
      asm volatile("cp.async.wait_group 1;\n" ::);
    } else {
      cp_async_wait_all();
    }
    __syncthreads();
    if (kb == lo) {
#pragma unroll
      for (int kk = 0; kk < DP / 16; ++kk) {
        lda_rm(qa[kk], sQ, LD, 16 * warp, 16 * kk);
        if (SPLIT) lda_rm(qla[kk], sQl, LD, 16 * warp, 16 * kk);
        lda_rm(ga[kk], sDy, LD, 16 * warp, 16 * kk);
      }
    }
    const bf16* tK = sK(stage);
    const bf16* tV = sV(stage);
    float s[8][4], dp[8][4];
    scores<DP, SPLIT>(s, qa, qla, tK, sKl(stage));
#pragma unroll
    for (int c = 0; c < 8; ++c)
#pragma unroll
      for (int e = 0; e < 4; ++e) dp[c][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < DP / 16; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bv[4];
        ldb_nk(bv, tV, LD, 16 * np, 16 * kk);
        mma16816(dp[2 * np], ga[kk], bv[0], bv[1]);
        mma16816(dp[2 * np + 1], ga[kk], bv[2], bv[3]);
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
        const float p =
            in_window(i, t, L, W) ? __expf(s[nt][e] * scale - ((e < 2) ? lse0 : lse1)) : 0.f;
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
  const bool pair = (D & 1) == 0;
#pragma unroll
  for (int nt = 0; nt < NTD; ++nt) {
    const int d = 8 * nt + 2 * cq;
    if (d >= D) continue;
    const bool has1 = d + 1 < D;
    if (i0 < L)
      store_grad2(dq, base + (size_t)i0 * D + d, acc[nt][0] * scale, acc[nt][1] * scale, has1,
                  pair, gdt);
    if (i1 < L)
      store_grad2(dq, base + (size_t)i1 * D + d, acc[nt][2] * scale, acc[nt][3] * scale, has1,
                  pair, gdt);
  }
}

// dmeta_j = -sum_b partial[b][j]: thread t sums blocks t, t + 1024, ... for up
// to 8 sinks at once (the block's sink partials are contiguous); a butterfly
// over each warp's lanes, then warp 0 adds the 32 warp totals the same way:
// the same order on every run.
constexpr int kDmetaThreads = 1024, kDmetaSinks = 8;
__global__ void __launch_bounds__(kDmetaThreads)
swa_dmeta_kernel(const float* __restrict__ partial, int nblocks, int n_meta,
                 float* __restrict__ dmeta) {
  __shared__ float red[kDmetaSinks][32];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int j0 = 0; j0 < n_meta; j0 += kDmetaSinks) {
    const int nj = min(kDmetaSinks, n_meta - j0);
    float s[kDmetaSinks];
#pragma unroll
    for (int j = 0; j < kDmetaSinks; ++j) s[j] = 0.f;
#pragma unroll 4
    for (int b = tid; b < nblocks; b += kDmetaThreads) {
      const float* p = partial + (size_t)b * n_meta + j0;
#pragma unroll
      for (int j = 0; j < kDmetaSinks; ++j)
        if (j < nj) s[j] += p[j];
    }
#pragma unroll
    for (int j = 0; j < kDmetaSinks; ++j) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s[j] += __shfl_xor_sync(0xffffffffu, s[j], o);
      if (lane == 0) red[j][warp] = s[j];
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
      for (int j = 0; j < kDmetaSinks; ++j) {
        float x = red[j][lane];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
        if (lane == 0 && j < nj) dmeta[j0 + j] = -x;
      }
    }
    __syncthreads();
  }
}

// ------------------------------------------------------- backward: dk, dv
// Works on transposed scores s^T = k q^T so every operand stays row-major.
// One CTA per (key block, key/value head): it walks the query blocks of every
// query head in the head's group, one double-buffered loop over
// (group head, query block), so dk and dv are summed over the group in
// registers.
template <int DP, bool SPLIT>
struct DkvSmem {
  static constexpr size_t T = Tile<DP>::bytes;
  static constexpr size_t k = 0, kl = k + T, v = kl + (SPLIT ? T : 0), q = v + T,
                          ql = q + 2 * T, dy = ql + (SPLIT ? 2 * T : 0), rows = dy + 2 * T,
                          bytes = rows + 4 * kB * 4;
};

template <int DP, bool SPLIT>
__global__ void __launch_bounds__(128)
swa_bwd_dkv_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k,
                   const bf16* __restrict__ v, const bf16* __restrict__ ql,
                   const bf16* __restrict__ kl, const bf16* __restrict__ dy,
                   const float* __restrict__ lse, const float* __restrict__ delta, int W,
                   float scale, int H, int grp, int L, int D, int nkb, int vec,
                   void* __restrict__ dk, void* __restrict__ dv, int gdt) {
  using SM = DkvSmem<DP, SPLIT>;
  constexpr int LD = Tile<DP>::LD, NTD = DP / 8;
  constexpr size_t T = Tile<DP>::bytes;
  extern __shared__ __align__(128) unsigned char smem[];
  bf16* sK = reinterpret_cast<bf16*>(smem + SM::k);
  bf16* sKl = reinterpret_cast<bf16*>(smem + SM::kl);
  bf16* sV = reinterpret_cast<bf16*>(smem + SM::v);
  auto sQ = [&](int s) { return reinterpret_cast<bf16*>(smem + SM::q + s * T); };
  auto sQl = [&](int s) { return reinterpret_cast<bf16*>(smem + SM::ql + s * T); };
  auto sDy = [&](int s) { return reinterpret_cast<bf16*>(smem + SM::dy + s * T); };
  float* sRow = reinterpret_cast<float*>(smem + SM::rows);  // 2 stages x (lse, delta)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, cq = lane & 3;
  const int kbk = blockIdx.x % nkb, bkv = blockIdx.x / nkb;  // bkv = b * Hkv + kv head
  const int Hkv = H / grp, b = bkv / Hkv;
  const int bh0 = b * H + (bkv - b * Hkv) * grp;  // first query head of the group
  const int k0 = kbk * kB;
  const size_t kvb = (size_t)bkv * L * D;
  const int qlo = k0;  // query blocks start at the key block (causal)
  const int qhi = min(k0 + kB + W - 1, L);
  const int nq = (qhi - qlo + kB - 1) / kB;  // query blocks per head, >= 1
  const int nit = grp * nq;
  auto issue = [&](int it, int st) {
    const int bh = bh0 + it / nq, qb = qlo + (it % nq) * kB;
    const size_t base = (size_t)bh * L * D;
    stage_tile<kB, DP, 128>(sQ(st), LD, q + base, D, qb, L, 0, D, vec);
    if (SPLIT) stage_tile<kB, DP, 128>(sQl(st), LD, ql + base, D, qb, L, 0, D, vec);
    stage_tile<kB, DP, 128>(sDy(st), LD, dy + base, D, qb, L, 0, D, vec);
    cp_async_commit();
    if (tid < kB) {
      const int r = qb + tid;
      sRow[st * 2 * kB + tid] = r < L ? lse[(size_t)bh * L + r] : 0.f;
      sRow[st * 2 * kB + kB + tid] = r < L ? delta[(size_t)bh * L + r] : 0.f;
    }
  };
  stage_tile<kB, DP, 128>(sK, LD, k + kvb, D, k0, L, 0, D, vec);
  if (SPLIT) stage_tile<kB, DP, 128>(sKl, LD, kl + kvb, D, k0, L, 0, D, vec);
  stage_tile<kB, DP, 128>(sV, LD, v + kvb, D, k0, L, 0, D, vec);
  issue(0, 0);
  const int t0 = k0 + 16 * warp + gq, t1 = t0 + 8;  // this thread's key rows
  float dka[NTD][4], dva[NTD][4];
#pragma unroll
  for (int c = 0; c < NTD; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) dka[c][e] = dva[c][e] = 0.f;
  uint32_t ka[DP / 16][4], kla[DP / 16][4], va[DP / 16][4];
  int stage = 0;
  for (int it = 0; it < nit; ++it, stage ^= 1) {
    const int qb = qlo + (it % nq) * kB;
    if (it + 1 < nit) {
      issue(it + 1, stage ^ 1);
      asm volatile("cp.async.wait_group 1;\n" ::);
    } else {
      cp_async_wait_all();
    }
    __syncthreads();
    if (it == 0) {
#pragma unroll
      for (int kk = 0; kk < DP / 16; ++kk) {
        lda_rm(ka[kk], sK, LD, 16 * warp, 16 * kk);
        if (SPLIT) lda_rm(kla[kk], sKl, LD, 16 * warp, 16 * kk);
        lda_rm(va[kk], sV, LD, 16 * warp, 16 * kk);
      }
    }
    const bf16* tQ = sQ(stage);
    const bf16* tDy = sDy(stage);
    const float* rl = sRow + stage * 2 * kB;
    float s[8][4], dp[8][4];
    scores<DP, SPLIT>(s, ka, kla, tQ, sQl(stage));
#pragma unroll
    for (int c = 0; c < 8; ++c)
#pragma unroll
      for (int e = 0; e < 4; ++e) dp[c][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < DP / 16; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bg[4];
        ldb_nk(bg, tDy, LD, 16 * np, 16 * kk);
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
        store_grad(dk, kvb + (size_t)t0 * D + d, dka[nt][0] * scale, gdt);
        store_grad(dv, kvb + (size_t)t0 * D + d, dva[nt][0], gdt);
      }
      if (d + 1 < D) {
        store_grad(dk, kvb + (size_t)t0 * D + d + 1, dka[nt][1] * scale, gdt);
        store_grad(dv, kvb + (size_t)t0 * D + d + 1, dva[nt][1], gdt);
      }
    }
    if (t1 < L) {
      if (d < D) {
        store_grad(dk, kvb + (size_t)t1 * D + d, dka[nt][2] * scale, gdt);
        store_grad(dv, kvb + (size_t)t1 * D + d, dva[nt][2], gdt);
      }
      if (d + 1 < D) {
        store_grad(dk, kvb + (size_t)t1 * D + d + 1, dka[nt][3] * scale, gdt);
        store_grad(dv, kvb + (size_t)t1 * D + d + 1, dva[nt][3], gdt);
      }
    }
  }
}

// ------------------------------------------------- forward, RoPE inside
// The SWA forward for unrotated queries and keys: q, k, v tiles come straight
// from the caller's tensors (any batch / head / token strides, fp32 or bf16)
// through TMA, the key / value tiles into a 2-stage ring; the CTA rotates the
// q and k tiles in fp32 (Llama rotate-half with cos / sin of each row's
// position; products and sum rounded once each) and splits them into the
// bf16 value + residual tiles the MMAs read, and converts v to bf16. From
// there the online softmax and P V are the forward kernel's, so the results
// equal rotating first (lz_rope_split) and calling the forward. With
// qh_out.. given (training) the kernel also writes the rotated operands the
// backward reads: q rows by their CTA, each key block by the CTA of the
// group's first query head whose query block starts at it.
template <int DP, typename XT>
struct RopeSmem {
  static constexpr size_t T = Tile<DP>::bytes;               // padded bf16 tile
  static constexpr size_t R = (size_t)kB * DP * sizeof(XT);  // raw TMA tile
  static constexpr size_t q = 0, ql = q + T, k = ql + T, kl = k + T, v = kl + T, rq = v + T,
                          rk = rq + R, rv = rk + 2 * R, bars = rv + 2 * R, bytes = bars + 64;
};


// raw [64][DP] (rows t0 ..) -> rotated hi / lo padded tiles, 8 columns of each
// half per item; rows >= L are zero. Optional copies of the rotated rows to
// global hi / lo [.., DP] from row 0 of the head. cos / sin rows must be
// 16-byte aligned (their token stride and base: checked by the host).
template <int DP, typename XT, typename CT>
__device__ __forceinline__ void rotate_tile(const XT* raw, bf16* hi, bf16* lo, int t0, int L,
                                            const CT* cs, const CT* sn, long long cs_sl,
                                            bf16* ghi, bf16* glo) {
  constexpr int LD = Tile<DP>::LD, HALF = DP / 2, G = HALF / 8;
  for (int e = threadIdx.x; e < kB * G; e += 128) {
    const int r = e / G, c = 8 * (e - r * G), t = t0 + r;
    float o1[8], o2[8];
    if (t < L) {
      float x1[8], x2[8], c1[8], c2[8], s1[8], s2[8];
      load8(raw + (size_t)r * DP + c, x1);
      load8(raw + (size_t)r * DP + c + HALF, x2);
      const CT* cr = cs + (size_t)t * cs_sl;
      const CT* sr = sn + (size_t)t * cs_sl;
      load8(cr + c, c1);
      load8(cr + c + HALF, c2);
      load8(sr + c, s1);
      load8(sr + c + HALF, s2);
      rope8(x1, x2, c1, c2, s1, s2, o1, o2);
    } else {
#pragma unroll
      for (int u = 0; u < 8; ++u) o1[u] = o2[u] = 0.f;
    }
    const uint4 h1 = pack8(o1), h2 = pack8(o2);
    const uint4 l1 = resid8(o1, h1), l2 = resid8(o2, h2);
    *reinterpret_cast<uint4*>(hi + r * LD + c) = h1;
    *reinterpret_cast<uint4*>(hi + r * LD + c + HALF) = h2;
    *reinterpret_cast<uint4*>(lo + r * LD + c) = l1;
    *reinterpret_cast<uint4*>(lo + r * LD + c + HALF) = l2;
    if (ghi && t < L) {
      const size_t g = (size_t)t * DP + c;
      *reinterpret_cast<uint4*>(ghi + g) = h1;
      *reinterpret_cast<uint4*>(ghi + g + HALF) = h2;
      *reinterpret_cast<uint4*>(glo + g) = l1;
      *reinterpret_cast<uint4*>(glo + g + HALF) = l2;
    }
  }
}

template <int DP, typename XT, typename CT>
__global__ void __launch_bounds__(128)
swa_rope_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, const CT* __restrict__ cs,
                    const CT* __restrict__ sn, long long cs_sb, long long cs_sl,
                    const float* __restrict__ meta, int n_meta, int W, float scale_log2, int H,
                    int grp, int L, int nqb, bf16* __restrict__ y, float* __restrict__ lse,
                    float* __restrict__ y32, bf16* __restrict__ qh_out,
                    bf16* __restrict__ ql_out, bf16* __restrict__ kh_out,
                    bf16* __restrict__ kl_out) {
  using SM = RopeSmem<DP, XT>;
  constexpr int LD = Tile<DP>::LD, NTD = DP / 8, D = DP;
  extern __shared__ __align__(128) unsigned char smem[];
  bf16* sQ = reinterpret_cast<bf16*>(smem + SM::q);
  bf16* sQl = reinterpret_cast<bf16*>(smem + SM::ql);
  bf16* sK = reinterpret_cast<bf16*>(smem + SM::k);
  bf16* sKl = reinterpret_cast<bf16*>(smem + SM::kl);
  bf16* sV = reinterpret_cast<bf16*>(smem + SM::v);
  const XT* rQ = reinterpret_cast<const XT*>(smem + SM::rq);
  auto rK = [&](int st) { return reinterpret_cast<XT*>(smem + SM::rk + st * SM::R); };
  auto rV = [&](int st) { return reinterpret_cast<XT*>(smem + SM::rv + st * SM::R); };
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::bars);  // q, stage 0, stage 1
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, cq = lane & 3;
  const int qb = blockIdx.x % nqb, bh = blockIdx.x / nqb;
  const int b = bh / H, h = bh - b * H, hk = h / grp;  // key/value head within the row
  const int q0 = qb * kB;
  const size_t base = (size_t)bh * L * D;
  const int Hkv = H / grp;
  const size_t kbase = ((size_t)b * Hkv + hk) * L * D;
  const CT* csb = cs + (size_t)b * cs_sb;
  const CT* snb = sn + (size_t)b * cs_sb;
  const int lo = max(q0 - W + 1, 0) / kB * kB;
  const int hi = min(q0 + kB, L);
  const int nblk = (hi - lo + kB - 1) / kB;
  if (tid == 0) {
    tc::mbar_init(&bars[0], 1);
    tc::mbar_init(&bars[1], 1);
    tc::mbar_init(&bars[2], 1);
    tc::fence_mbar_init();
  }
  __syncthreads();
  auto issue_kv = [&](int i) {  // key block i (from lo) into stage i & 1
    const int st = i & 1;
    tc::mbar_expect_tx(&bars[1 + st], (uint32_t)(2 * SM::R));
    tc::tma_load_4d(rK(st), &tk, 0, lo + i * kB, hk, b, &bars[1 + st]);
    tc::tma_load_4d(rV(st), &tv, 0, lo + i * kB, hk, b, &bars[1 + st]);
  };
  if (tid == 0) {
    tc::mbar_expect_tx(&bars[0], (uint32_t)SM::R);
    tc::tma_load_4d(const_cast<XT*>(rQ), &tq, 0, q0, h, b, &bars[0]);
    issue_kv(0);
    if (nblk > 1) issue_kv(1);
  }

  // sinks seed the running max / sum (log2 domain)
  float ms = -1e30f;
  for (int j = 0; j < n_meta; ++j) ms = fmaxf(ms, meta[j] * kLog2e);
  float ls = 0.f;
  for (int j = 0; j < n_meta; ++j) ls += exp2f(meta[j] * kLog2e - ms);

  tc::mbar_wait(&bars[0], 0, 40);
  rotate_tile<DP, XT, CT>(rQ, sQ, sQl, q0, L, csb, snb, cs_sl,
                          qh_out ? qh_out + base : nullptr, qh_out ? ql_out + base : nullptr);

  const int i0 = q0 + 16 * warp + gq, i1 = i0 + 8;
  float m0 = ms, m1 = ms, l0 = ls, l1 = ls;
  float o[NTD][4];
#pragma unroll
  for (int c = 0; c < NTD; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[c][e] = 0.f;
  uint32_t qa[DP / 16][4], qla[DP / 16][4];

  for (int it = 0; it < nblk; ++it) {
    const int st = it & 1, kb = lo + it * kB;
    tc::mbar_wait(&bars[1 + st], (it >> 1) & 1, 41);
    const bool writer = kh_out && kb == q0 && h % grp == 0;
    rotate_tile<DP, XT, CT>(rK(st), sK, sKl, kb, L, csb, snb, cs_sl,
                            writer ? kh_out + kbase : nullptr, writer ? kl_out + kbase : nullptr);
    {
      const XT* rv = rV(st);
      for (int e = tid; e < kB * D / 8; e += 128) {
        const int r = e / (D / 8), c = 8 * (e - r * (D / 8));
        float x[8];
        load8(rv + (size_t)r * D + c, x);
        *reinterpret_cast<uint4*>(sV + r * LD + c) = pack8(x);
      }
    }
    __syncthreads();  // tiles ready; the raw stage is free
    if (tid == 0 && it + 2 < nblk) {
      tc::fence_proxy_async_smem();
      issue_kv(it + 2);
    }
    if (it == 0) {
#pragma unroll
      for (int kk = 0; kk < DP / 16; ++kk) {
        lda_rm(qa[kk], sQ, LD, 16 * warp, 16 * kk);
        lda_rm(qla[kk], sQl, LD, 16 * warp, 16 * kk);
      }
    }
    float s[8][4];
    scores<DP, true>(s, qa, qla, sK, sKl);
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
    uint32_t pa[4][4], pl[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = exp2f(s[nt][0] - mn0), p1 = exp2f(s[nt][1] - mn0);
      const float p2 = exp2f(s[nt][2] - mn1), p3 = exp2f(s[nt][3] - mn1);
      rs0 += p0 + p1;
      rs1 += p2 + p3;
      const uint32_t h01 = pack_bf16(p0, p1), h23 = pack_bf16(p2, p3);
      pa[nt >> 1][(nt & 1) * 2 + 0] = h01;
      pa[nt >> 1][(nt & 1) * 2 + 1] = h23;
      pl[nt >> 1][(nt & 1) * 2 + 0] = pack_bf16(p0 - bf16_lo(h01), p1 - bf16_hi(h01));
      pl[nt >> 1][(nt & 1) * 2 + 1] = pack_bf16(p2 - bf16_lo(h23), p3 - bf16_hi(h23));
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
        ldb_kn(bb, sV, LD, 16 * j, 16 * np);
        mma16816(o[2 * np], pa[j], bb[0], bb[1]);
        mma16816(o[2 * np + 1], pa[j], bb[2], bb[3]);
        mma16816(o[2 * np], pl[j], bb[0], bb[1]);
        mma16816(o[2 * np + 1], pl[j], bb[2], bb[3]);
      }
    }
    __syncthreads();  // sK, sKl, sV are rewritten by the next block
  }
  const float inv0 = 1.f / l0, inv1 = 1.f / l1;
#pragma unroll
  for (int nt = 0; nt < NTD; ++nt) {
    const int d = 8 * nt + 2 * cq;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int i = hh ? i1 : i0;
      if (i >= L) continue;
      const float inv = hh ? inv1 : inv0;
      const float a = o[nt][2 * hh] * inv, bq = o[nt][2 * hh + 1] * inv;
      const size_t at = base + (size_t)i * D + d;
      *reinterpret_cast<__nv_bfloat162*>(y + at) = __floats2bfloat162_rn(a, bq);
      if (y32) *reinterpret_cast<float2*>(y32 + at) = make_float2(a, bq);
    }
  }
  if (lse && cq == 0) {
    if (i0 < L) lse[(size_t)bh * L + i0] = m0 * kLn2 + logf(l0);
    if (i1 < L) lse[(size_t)bh * L + i1] = m1 * kLn2 + logf(l1);
  }
}

template <int DP, bool SPLIT>
int launch_swa_fwd(const bf16* q, const bf16* k, const bf16* v, const bf16* ql, const bf16* kl,
                   const float* meta, int n_meta, int W, int BH, int H, int grp, int L, int D,
                   int vec, bf16* y, const SwaSaved& sv, cudaStream_t st) {
  using SM = FwdSmem<DP, SPLIT>;
  static bool done[64] = {false};
  int rc = ensure_smem_swa(swa_fwd_kernel<DP, SPLIT>, SM::bytes, done);
  if (rc) return rc;
  const int nqb = ceil_div(L, kB);
  const float scale_log2 = kLog2e / sqrtf((float)D);
  swa_fwd_kernel<DP, SPLIT><<<(unsigned)((long long)BH * nqb), 128, SM::bytes, st>>>(
      q, k, v, ql, kl, meta, n_meta, W, scale_log2, H, grp, L, D, nqb, vec, y, sv.lse, sv.y32);
  count_launches(1);
  return check_launch("swa_fwd_kernel");
}

template <int DP, bool SPLIT>
int launch_swa_bwd(const bf16* q, const bf16* k, const bf16* v, const bf16* ql, const bf16* kl,
                   const bf16* dy, const float* meta, int n_meta, const SwaSaved& sv,
                   const SwaWork& wk, int W, int BH, int H, int grp, int L, int D, int vec,
                   void* dq, void* dk, void* dv, int gdt, cudaStream_t st) {
  const float* lse = sv.lse;
  using SQ = DqSmem<DP, SPLIT>;
  using SKV = DkvSmem<DP, SPLIT>;
  static bool done_q[64] = {false}, done_kv[64] = {false};
  int rc = ensure_smem_swa(swa_bwd_dq_kernel<DP, SPLIT>, SQ::bytes, done_q);
  if (rc) return rc;
  rc = ensure_smem_swa(swa_bwd_dkv_kernel<DP, SPLIT>, SKV::bytes, done_kv);
  if (rc) return rc;
  const int nb = ceil_div(L, kB);
  const float scale = 1.f / sqrtf((float)D);
  const int vec_dots = (D % 4 == 0) && ((uintptr_t)dy & 7) == 0 && aligned16(sv.y32);
  swa_bwd_delta_kernel<<<(unsigned)((long long)BH * nb), 128, 0, st>>>(
      dy, sv.y32, lse, meta, n_meta, L, D, nb, vec_dots, wk.delta, wk.partial);
  count_launches(1);
  rc = check_launch("swa_bwd_delta_kernel");
  if (rc) return rc;
  // head dim 64, window <= 64: the tensor-core dq and dk / dv unless switched off
  rc = D == 64 ? swa_bwd_dq_tc(q, k, v, ql, kl, dy, lse, wk.delta, W, dq, gdt, BH / H, H,
                               H / grp, L, D, st)
               : LZ_ERR_UNSUPPORTED;
  if (rc == LZ_ERR_UNSUPPORTED) {
    swa_bwd_dq_kernel<DP, SPLIT><<<(unsigned)((long long)BH * nb), 128, SQ::bytes, st>>>(
        q, k, v, ql, kl, dy, lse, wk.delta, W, scale, H, grp, L, D, nb, vec, dq, gdt);
    count_launches(1);
    rc = check_launch("swa_bwd_dq_kernel");
  }
  if (rc) return rc;
  if (D == 64) {
    rc = swa_bwd_dkv_tc(q, k, v, ql, kl, dy, lse, wk.delta, W, dk, dv, gdt, BH / H, H, H / grp,
                        L, D, st);
    if (rc != LZ_ERR_UNSUPPORTED) return rc;
  }
  swa_bwd_dkv_kernel<DP, SPLIT><<<(unsigned)((long long)(BH / grp) * nb), 128, SKV::bytes, st>>>(
      q, k, v, ql, kl, dy, lse, wk.delta, W, scale, H, grp, L, D, nb, vec, dk, dv, gdt);
  count_launches(1);
  return check_launch("swa_bwd_dkv_kernel");
}

// [B, Hx, L, D] at element strides (sb, sh, sl, 1) as a 4-D map {D, L, Hx, B},
// box {D, 64, 1, 1} (one 64-row tile of one head), zero fill past L.
bool make_rope_map(CUtensorMap* m, const void* ptr, int x_dtype, int D, int L, int Hx, int B,
                   long long sb, long long sh, long long sl) {
  tc::EncodeTiledFn fn = tc::encode_tiled_fn();
  if (!fn) return false;
  const long long es = x_dtype == LZ_DTYPE_F32 ? 4 : 2;
  if (Hx == 1) sh = (long long)L * sl;  // strides of size-1 dims are not used; keep them legal
  if (B == 1) sb = (long long)Hx * sh;
  if (!aligned16(ptr) || sl <= 0 || sh <= 0 || sb <= 0 || (sl * es) % 16 || (sh * es) % 16 ||
      (sb * es) % 16 || (D * es) % 16)
    return false;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)L, (cuuint64_t)Hx, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)(sl * es), (cuuint64_t)(sh * es), (cuuint64_t)(sb * es)};
  cuuint32_t box[4] = {(cuuint32_t)D, (cuuint32_t)kB, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(m, x_dtype == LZ_DTYPE_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                       : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
            4, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int DP, typename XT, typename CT>
int launch_swa_rope(const SwaRopeArgs& a, const SwaSaved& sv, cudaStream_t st) {
  using SM = RopeSmem<DP, XT>;
  if (SM::bytes > 227 * 1024) return LZ_ERR_UNSUPPORTED;
  const long long ces = a.cs_dtype == LZ_DTYPE_F32 ? 4 : 2;
  if (!aligned16(a.cos) || !aligned16(a.sin) || (a.cs_sl * ces) % 16 || (a.cs_sb * ces) % 16)
    return LZ_ERR_UNSUPPORTED;  // the rotation reads cos / sin rows with 16-byte loads
  CUtensorMap mq, mk, mv;
  if (!make_rope_map(&mq, a.q, a.x_dtype, DP, a.L, a.H, a.B, a.q_sb, a.q_sh, a.q_sl) ||
      !make_rope_map(&mk, a.k, a.x_dtype, DP, a.L, a.Hkv, a.B, a.k_sb, a.k_sh, a.k_sl) ||
      !make_rope_map(&mv, a.v, a.x_dtype, DP, a.L, a.Hkv, a.B, a.v_sb, a.v_sh, a.v_sl))
    return LZ_ERR_UNSUPPORTED;
  static bool done[64] = {false};
  int rc = ensure_smem_swa(swa_rope_fwd_kernel<DP, XT, CT>, SM::bytes, done);
  if (rc) return rc;
  const int nqb = ceil_div(a.L, kB);
  const float scale_log2 = kLog2e / sqrtf((float)DP);
  swa_rope_fwd_kernel<DP, XT, CT><<<(unsigned)((long long)a.B * a.H * nqb), 128, SM::bytes, st>>>(
      mq, mk, mv, static_cast<const CT*>(a.cos), static_cast<const CT*>(a.sin), a.cs_sb, a.cs_sl,
      a.meta, a.n_meta, a.window, scale_log2, a.H, a.H / a.Hkv, a.L, nqb, a.y, sv.lse, sv.y32,
      a.q_hi, a.q_lo, a.k_hi, a.k_lo);
  count_launches(1);
  return check_launch("swa_rope_fwd_kernel");
}

}  // namespace

int swa_fwd(const bf16* q, const bf16* k, const bf16* v, const bf16* ql, const bf16* kl,
            const float* meta, int n_meta, int W, bf16* y, const SwaSaved& sv, int B, int H,
            int Hkv, int L, int D, cudaStream_t st) {
  {
    const int rc = swa_fwd_tc(q, k, v, ql, kl, meta, n_meta, W, y, sv, B, H, Hkv, L, D, st);
    if (rc != LZ_ERR_UNSUPPORTED) return rc;
  }
  const int BH = B * H, grp = H / Hkv;
  const bool split = ql != nullptr;
  int vec = (D % 8 == 0) && aligned16(q) && aligned16(k) && aligned16(v);
  if (split) vec = vec && aligned16(ql) && aligned16(kl);
#define LZ_SWA_FWD(dp)                                                                       \
  return split ? launch_swa_fwd<dp, true>(q, k, v, ql, kl, meta, n_meta, W, BH, H, grp, L, D,  \
                                          vec, y, sv, st)                                    \
               : launch_swa_fwd<dp, false>(q, k, v, ql, kl, meta, n_meta, W, BH, H, grp, L, D, \
                                           vec, y, sv, st);
  if (D <= 32) { LZ_SWA_FWD(32) }
  if (D <= 64) { LZ_SWA_FWD(64) }
  if (D <= 128) { LZ_SWA_FWD(128) }
#undef LZ_SWA_FWD
  set_error("swa_fwd: head dim above 128 is not supported");
  return LZ_ERR_UNSUPPORTED;
}

int swa_rope_fwd(const SwaRopeArgs& a, const SwaSaved& sv, cudaStream_t st) {
  // At the tensor-core shape the fused forward is the tcgen05 kernel or
  // nothing: a decline (fp32 projections, strides its maps cannot take) sends
  // the caller to rotate first, and lz_swa_fwd_gqa then runs the same kernel.
  if (swa_tc_enabled() && a.D == 64 && a.window >= 1 && a.window <= 128)
    return swa_rope_fwd_tc(a, sv, st);
  const bool f32 = a.x_dtype == LZ_DTYPE_F32, cf32 = a.cs_dtype == LZ_DTYPE_F32;
#define LZ_ROPE(dp)                                                                          \
  if (a.D == dp) {                                                                           \
    if (f32) return cf32 ? launch_swa_rope<dp, float, float>(a, sv, st)                     \
                         : launch_swa_rope<dp, float, bf16>(a, sv, st);                     \
    return cf32 ? launch_swa_rope<dp, bf16, float>(a, sv, st)                               \
                : launch_swa_rope<dp, bf16, bf16>(a, sv, st);                               \
  }
  LZ_ROPE(32) LZ_ROPE(64) LZ_ROPE(128)
#undef LZ_ROPE
  return LZ_ERR_UNSUPPORTED;  // other head dims: rotate first (lz_rope_split) and lz_swa_fwd_gqa
}

int swa_bwd(const bf16* q, const bf16* k, const bf16* v, const bf16* ql, const bf16* kl,
            const float* meta, int n_meta, int W, const SwaSaved& sv, const bf16* dy, void* dq,
            void* dk, void* dv, int gdt, float* dmeta, const SwaWork& wk, int B, int H, int Hkv,
            int L, int D, cudaStream_t st) {
  const int BH = B * H, grp = H / Hkv;
  const bool split = ql != nullptr;
  int vec = (D % 8 == 0) && aligned16(q) && aligned16(k) && aligned16(v) && aligned16(dy);
  if (split) vec = vec && aligned16(ql) && aligned16(kl);
  int rc;
#define LZ_SWA_BWD(dp)                                                                         \
  rc = split ? launch_swa_bwd<dp, true>(q, k, v, ql, kl, dy, meta, n_meta, sv, wk, W, BH, H, grp, \
                                        L, D, vec, dq, dk, dv, gdt, st)                        \
             : launch_swa_bwd<dp, false>(q, k, v, ql, kl, dy, meta, n_meta, sv, wk, W, BH, H,  \
                                         grp, L, D, vec, dq, dk, dv, gdt, st);
  if (D <= 32) {
    LZ_SWA_BWD(32)
  } else if (D <= 64) {
    LZ_SWA_BWD(64)
  } else if (D <= 128) {
    LZ_SWA_BWD(128)
  } else {
    set_error("swa_bwd: head dim above 128 is not supported");
    return LZ_ERR_UNSUPPORTED;
  }
#undef LZ_SWA_BWD
  if (rc) return rc;
  if (n_meta > 0 && dmeta) {
    const int nblocks = BH * ceil_div(L, kB);
    swa_dmeta_kernel<<<1, kDmetaThreads, 0, st>>>(wk.partial, nblocks, n_meta, dmeta);
    count_launches(1);
    rc = check_launch("swa_dmeta_kernel");
  }
  return rc;
}

int swa_timeout_flag(unsigned int* out) { return tc::read_timeout_flag_here(out); }
int swa_timeout_clear() { return tc::clear_timeout_flag_here(); }

}  // namespace lz
