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

// dmeta_j = -sum_b partial[b][j]: 256 threads, each summing a fixed strided
// subset of blocks, then a fixed-order tree in shared memory.
__global__ void __launch_bounds__(256)
swa_dmeta_kernel(const float* __restrict__ partial, int nblocks, int n_meta,
                 float* __restrict__ dmeta) {
  __shared__ float red[256];
  const int tid = threadIdx.x;
  for (int j = 0; j < n_meta; ++j) {
    float s = 0.f;
    for (int b = tid; b < nblocks; b += 256) s += partial[(size_t)b * n_meta + j];
    red[tid] = s;
    __syncthreads();
    for (int w = 128; w > 0; w >>= 1) {
      if (tid < w) red[tid] += red[tid + w];
      __syncthreads();
    }
    if (tid == 0) dmeta[j] = -red[0];
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
  swa_bwd_dq_kernel<DP, SPLIT><<<(unsigned)((long long)BH * nb), 128, SQ::bytes, st>>>(
      q, k, v, ql, kl, dy, lse, wk.delta, W, scale, H, grp, L, D, nb, vec, dq, gdt);
  count_launches(1);
  rc = check_launch("swa_bwd_dq_kernel");
  if (rc) return rc;
  swa_bwd_dkv_kernel<DP, SPLIT><<<(unsigned)((long long)(BH / grp) * nb), 128, SKV::bytes, st>>>(
      q, k, v, ql, kl, dy, lse, wk.delta, W, scale, H, grp, L, D, nb, vec, dk, dv, gdt);
  count_launches(1);
  return check_launch("swa_bwd_dkv_kernel");
}

}  // namespace

int swa_fwd(const bf16* q, const bf16* k, const bf16* v, const bf16* ql, const bf16* kl,
            const float* meta, int n_meta, int W, bf16* y, const SwaSaved& sv, int B, int H,
            int Hkv, int L, int D, cudaStream_t st) {
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
    swa_dmeta_kernel<<<1, 256, 0, st>>>(wk.partial, nblocks, n_meta, dmeta);
    count_launches(1);
    rc = check_launch("swa_dmeta_kernel");
  }
  return rc;
}

}  // namespace lz
