// Recurrent decode: one new token per sequence against a cached state.
//
// The reference has no cache (every forward recomputes the whole sequence).
// Both of its branches have an O(1)-per-token form that gives the same
// outputs as the full-sequence forward at the new position:
//
// GLA (src/lizard_attention.py:13-31 as a recurrence): with lg the new
// token's log gate,
//   S <- exp(lg) S + fk^T v,   z <- exp(lg) z + fk     (fp32 state)
//   y  = fq S / max(fq . z, FLT_MIN)
// which is sum_{t <= i} (fq_i . fk_t) exp(G_i - G_t) v_t over the row sum.
// One state serves every query head that reads the same key/value head and
// gate: with a gate shared by the heads (log_gamma [B, L], the Lizard layer's
// case) and grouped keys / values, the Hkv states of a batch row stand for all
// H query heads, as repeat_interleave makes them identical in the reference.
//
// SWA (src/lizard_attention.py:34-44): the new key is rotated (Llama
// rotate-half RoPE at the token's position) and written with its value into a
// ring of the last W rotated keys / values (fp32); each query head of the group
// attends over the min(pos + 1, W) most recent entries with the sink logits in
// the denominator, scale 1/sqrt(D).
#include <algorithm>

#include "common.cuh"
#include "tc.cuh"

namespace lz {
namespace {

// Test switch of the failure-detection path: when set, the SWA decode kernel
// arms its ring-copy barrier but issues no copy, so its bounded wait runs out,
// records its site in the timeout flag, and every CTA returns without writing
// (no copy is in flight, nothing else waits on it). Off unless a test sets it
// through lz_test_withhold_decode_ring_copy.
static __device__ int g_withhold_ring_copy;

constexpr int kT = 256;

// One CTA per (batch row, state head). CG = D / 4 column groups of 4, RG = 256
// / CG row groups; thread (rg, cg) updates rows rg, rg + RG, ... of its 4
// columns and accumulates fq . S for each of the QS query heads of the state.
template <int QS>
__global__ void __launch_bounds__(kT)
gla_decode_kernel(const bf16* __restrict__ fq, const bf16* __restrict__ fk,
                  const bf16* __restrict__ v, const float* __restrict__ lg, int gph,
                  float* __restrict__ S, float* __restrict__ Z, bf16* __restrict__ y, int H,
                  int Hkv, int Hs, int F, int D) {
  extern __shared__ __align__(16) float sm[];
  float* sK = sm;                 // [F]
  float* sV = sK + F;             // [D]
  float* sQ = sV + D;             // [QS][F]
  float* sRed = sQ + QS * F;      // [QS][RG][D] = QS x 1024
  float* sDen = sRed + QS * 1024;  // [QS][8] warp partials
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int sidx = blockIdx.x, b = sidx / Hs, s = sidx - b * Hs;
  const int h0 = b * H + s * QS;  // first query head (global index)
  const int kvh = (Hs == Hkv) ? sidx : kv_head(b * H + s, H, H / Hkv);
  const float gamma = expf(lg[gph ? (size_t)b * H + s : (size_t)b]);
  for (int i = tid; i < F; i += kT) sK[i] = __bfloat162float(fk[(size_t)kvh * F + i]);
  for (int i = tid; i < D; i += kT) sV[i] = __bfloat162float(v[(size_t)kvh * D + i]);
  for (int i = tid; i < QS * F; i += kT) sQ[i] = __bfloat162float(fq[(size_t)h0 * F + i]);
  __syncthreads();

  // normaliser: z <- gamma z + fk (F <= 256: one element per thread); den_h = fq_h . z
  float zd[QS];
#pragma unroll
  for (int h = 0; h < QS; ++h) zd[h] = 0.f;
  float* Zs = Z + (size_t)sidx * F;
  if (tid < F) {
    const float zn = gamma * Zs[tid] + sK[tid];
    Zs[tid] = zn;
#pragma unroll
    for (int h = 0; h < QS; ++h) zd[h] = sQ[h * F + tid] * zn;
  }
#pragma unroll
  for (int h = 0; h < QS; ++h) {
    float x = zd[h];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    if (lane == 0) sDen[h * 8 + warp] = x;
  }

  // state: S <- gamma S + fk^T v; partial y_h over this thread's rows
  const int CG = D / 4, RG = kT / CG;
  const int cg = tid % CG, rg = tid / CG;
  float4* Sb = reinterpret_cast<float4*>(S + (size_t)sidx * F * D);
  float4 acc[QS];
#pragma unroll
  for (int h = 0; h < QS; ++h) acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (rg < RG) {
    const float4 vv = reinterpret_cast<const float4*>(sV)[cg];
    // 8 rows per pass: their loads are all in flight before the first update
    for (int f0 = rg; f0 < F; f0 += 8 * RG) {
      float4 sv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int f = f0 + u * RG;
        if (f < F) sv[u] = Sb[(size_t)f * CG + cg];
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int f = f0 + u * RG;
        if (f < F) {
          const float kf = sK[f];
          sv[u].x = gamma * sv[u].x + kf * vv.x;
          sv[u].y = gamma * sv[u].y + kf * vv.y;
          sv[u].z = gamma * sv[u].z + kf * vv.z;
          sv[u].w = gamma * sv[u].w + kf * vv.w;
          Sb[(size_t)f * CG + cg] = sv[u];
#pragma unroll
          for (int h = 0; h < QS; ++h) {
            const float qf = sQ[h * F + f];
            acc[h].x += qf * sv[u].x;
            acc[h].y += qf * sv[u].y;
            acc[h].z += qf * sv[u].z;
            acc[h].w += qf * sv[u].w;
          }
        }
      }
    }
    // RG * CG = 256 threads exactly when CG divides 256 (D in {4, 8, ..., 256} of powers
    // of two); other D leave rg == RG for the tail threads, which own no rows
#pragma unroll
    for (int h = 0; h < QS; ++h)
      reinterpret_cast<float4*>(sRed + h * 1024 + rg * D)[cg] = acc[h];
  }
  __syncthreads();
  for (int e = tid; e < QS * D; e += kT) {
    const int h = e / D, d = e - h * D;
    float num = 0.f;
    for (int r = 0; r < RG; ++r) num += sRed[h * 1024 + r * D + d];
    float den = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) den += sDen[h * 8 + w];
    y[(size_t)(h0 + h) * D + d] = __float2bfloat16_rn(num / fmaxf(den, kTiny));
  }
}

template <typename T>
__device__ __forceinline__ float ldf(const T* p, size_t i);
template <>
__device__ __forceinline__ float ldf<float>(const float* p, size_t i) { return p[i]; }
template <>
__device__ __forceinline__ float ldf<bf16>(const bf16* p, size_t i) {
  return __bfloat162float(p[i]);
}

// One CTA per (batch row, key/value head). The whole CTA rotates the new key
// and writes it and v into the ring; then each warp takes query heads of the
// group (warp, warp + nwarps, ...): lanes own keys for the scores (a key row
// per lane) and columns for P V (coalesced rows of the value ring).
// STAGE (both rings fit in shared memory, D % 4 == 0, 16-byte aligned rings):
// one bulk copy brings the whole key and value rings of the (row, kv head)
// into shared memory before the new entry is written there and to HBM, so the
// warps' score and P V loops read shared memory instead of walking the ring
// with dependent global loads. In the score loop lane l visits the 16-byte
// chunks of its key row starting at chunk l, so the 8 lanes of a quarter warp
// hit 8 different bank groups.
constexpr int kMaxDecodeWindow = 1024;

template <typename XT, typename CT, bool STAGE>
__global__ void __launch_bounds__(kT)
swa_decode_kernel(const XT* __restrict__ q, long long q_sb, long long q_sh,
                  const XT* __restrict__ k, long long k_sb, long long k_sh,
                  const XT* __restrict__ v, long long v_sb, long long v_sh,
                  const CT* __restrict__ cs, const CT* __restrict__ sn, long long cs_sb,
                  float* __restrict__ kc, float* __restrict__ vc, const int* __restrict__ pos,
                  const float* __restrict__ meta, int n_meta, bf16* __restrict__ y, int H,
                  int Hkv, int W, int D) {
  extern __shared__ __align__(16) float sm[];
  const int nw = blockDim.x >> 5;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // STAGE layout: [mbarrier, 16 B][key ring W x D][value ring W x D][sQ][sP]
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm);
  float* sKr = sm + 4;
  float* sVr = sKr + (size_t)W * D;
  float* base = STAGE ? sVr + (size_t)W * D : sm;
  const int grp = H / Hkv, half = D / 2;
  float* sQall = base;                          // [grp][D] rotated queries of the group
  float* sP = base + grp * D + warp * W;        // [nw][W] softmax weights per warp
  const int bkv = blockIdx.x, b = bkv / Hkv, j = bkv - b * Hkv;
  const int t = pos[b];
  const int slot = t % W, n = min(t + 1, W);
  const CT* cb = cs + (size_t)b * cs_sb;
  const CT* sb = sn + (size_t)b * cs_sb;
  float* kring = kc + (size_t)bkv * W * D;
  float* vring = vc + (size_t)bkv * W * D;
  const XT* kr = k + b * k_sb + j * k_sh;
  const XT* vr = v + b * v_sb + j * v_sh;
  if constexpr (STAGE) {
    // the old ring first (nothing writes it until the copy has landed)
    if (tid == 0) {
      tc::mbar_init(bar, 1);
      tc::fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
      const uint32_t bytes = (uint32_t)W * D * 4;
      tc::mbar_expect_tx(bar, 2 * bytes);
      if (!g_withhold_ring_copy) {
        tc::bulk_load(sKr, kring, bytes, bar);
        tc::bulk_load(sVr, vring, bytes, bar);
      }
    }
  }
  // the group's rotated queries (while the copy is in flight)
  for (int e = tid; e < grp * half; e += blockDim.x) {
    const int g = e / half, d = e - g * half;
    const XT* qr = q + b * q_sb + (j * grp + g) * q_sh;
    const float x1 = ldf(qr, d), x2 = ldf(qr, d + half);
    const float c1 = ldf(cb, d), s1 = ldf(sb, d), c2 = ldf(cb, d + half), s2 = ldf(sb, d + half);
    sQall[g * D + d] = __fadd_rn(__fmul_rn(x1, c1), -__fmul_rn(x2, s1));
    sQall[g * D + d + half] = __fadd_rn(__fmul_rn(x2, c2), __fmul_rn(x1, s2));
  }
  // the new ring entry, held in registers until the old ring has landed
  // (D <= 256 and blockDim >= 32: at most 4 rotated pairs and 8 values a thread)
  float nk1[4], nk2[4], nv[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = tid + i * blockDim.x;
    if (d < half) {
      const float x1 = ldf(kr, d), x2 = ldf(kr, d + half);
      const float c1 = ldf(cb, d), s1 = ldf(sb, d), c2 = ldf(cb, d + half), s2 = ldf(sb, d + half);
      nk1[i] = __fadd_rn(__fmul_rn(x1, c1), -__fmul_rn(x2, s1));
      nk2[i] = __fadd_rn(__fmul_rn(x2, c2), __fmul_rn(x1, s2));
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int d = tid + i * blockDim.x;
    if (d < D) nv[i] = ldf(vr, d);
  }
  if constexpr (STAGE) {
    // one bounded wait, its outcome shared through the header's spare word so
    // that the whole CTA leaves together on a timeout (flag set, nothing else
    // in flight); then every thread observes the completed phase itself
    int* ok = reinterpret_cast<int*>(sm + 2);
    if (tid == 0) *ok = tc::mbar_wait(bar, 0, 90) ? 1 : 0;
    __syncthreads();
    if (!*ok) return;
    (void)tc::mbar_try_wait(bar, 0);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = tid + i * blockDim.x;
    if (d < half) {
      kring[(size_t)slot * D + d] = nk1[i];
      kring[(size_t)slot * D + d + half] = nk2[i];
      if constexpr (STAGE) sKr[slot * D + d] = nk1[i], sKr[slot * D + d + half] = nk2[i];
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int d = tid + i * blockDim.x;
    if (d < D) {
      vring[(size_t)slot * D + d] = nv[i];
      if constexpr (STAGE) sVr[slot * D + d] = nv[i];
    }
  }
  __syncthreads();
  const float scale = rsqrtf((float)D);
  float ms = -1e30f;
  for (int m = 0; m < n_meta; ++m) ms = fmaxf(ms, meta[m]);
  for (int g = warp; g < grp; g += nw) {
    const int hq = j * grp + g;
    const float* sQ = sQall + g * D;
    // The ring rows holding the last n tokens are exactly rows 0 .. n-1 (before
    // the ring fills token t sits in row t), so the loops run over rows and the
    // softmax weights are indexed by row. Scores: a key row per lane.
    const float* kbase = STAGE ? sKr : kring;
    const float* vbase = STAGE ? sVr : vring;
    float mx = ms;
    for (int r = lane; r < n; r += 32) {
      float x = 0.f;
      if ((D & 3) == 0) {
        const float4* kk = reinterpret_cast<const float4*>(kbase + (size_t)r * D);
        const float4* q4 = reinterpret_cast<const float4*>(sQ);
        const int nc = D >> 2;
        int c = STAGE ? lane % nc : 0;  // staged: a different bank group per lane
        for (int i = 0; i < nc; ++i) {
          const float4 kv = kk[c], qv = q4[c];
          x += qv.x * kv.x + qv.y * kv.y + qv.z * kv.z + qv.w * kv.w;
          c = c + 1 == nc ? 0 : c + 1;
        }
      } else {
        const float* kk = kbase + (size_t)r * D;
        for (int d = 0; d < D; ++d) x += sQ[d] * kk[d];
      }
      x *= scale;
      sP[r] = x;
      mx = fmaxf(mx, x);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
    for (int r = lane; r < n; r += 32) {
      const float p = __expf(sP[r] - mx);
      sP[r] = p;
      sum += p;
    }
    for (int m = lane; m < n_meta; m += 32) sum += __expf(meta[m] - mx);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float inv = 1.f / sum;
    __syncwarp();
    // P V: columns per lane, four rows in flight
    for (int d = lane; d < D; d += 32) {
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      const float* vcol = vbase + d;
      int r = 0;
      for (; r + 4 <= n; r += 4) {
        a0 += sP[r] * vcol[(size_t)r * D];
        a1 += sP[r + 1] * vcol[(size_t)(r + 1) * D];
        a2 += sP[r + 2] * vcol[(size_t)(r + 2) * D];
        a3 += sP[r + 3] * vcol[(size_t)(r + 3) * D];
      }
      for (; r < n; ++r) a0 += sP[r] * vcol[(size_t)r * D];
      const float acc = (a0 + a1) + (a2 + a3);
      y[((size_t)b * H + hq) * D + d] = __float2bfloat16_rn(acc * inv);
    }
    __syncwarp();
  }
}

int dtype_ok(int dt) { return dt == LZ_DTYPE_F32 || dt == LZ_DTYPE_BF16; }

template <typename Kern>
int ensure_decode_smem(Kern k, size_t bytes, bool* done) {
  if (bytes <= 48 * 1024) return LZ_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)bytes);
    if (e != cudaSuccess) {
      set_error(std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
      return LZ_ERR_CUDA;
    }
    done[dev] = true;
  }
  return LZ_OK;
}

template <typename XT>
int launch_swa_decode(const void* q, long long q_sb, long long q_sh, const void* k,
                      long long k_sb, long long k_sh, const void* v, long long v_sb,
                      long long v_sh, const void* cs, const void* sn, int cs_dtype,
                      long long cs_sb, float* kc, float* vc, const int* pos, const float* meta,
                      int n_meta, bf16* y, int B, int H, int Hkv, int W, int D,
                      cudaStream_t st) {
  const int nw = std::min(H / Hkv, kT / 32);  // one warp per query head of the group
  const size_t smem0 = ((size_t)(H / Hkv) * D + (size_t)nw * W) * 4;
  const size_t smem1 = 16 + 2 * (size_t)W * D * 4 + smem0;
  // both rings in shared memory: they fit, rows are whole 16-byte chunks and the
  // rings start on 16-byte boundaries (the bulk copy's rules)
  const bool stage = smem1 <= 160 * 1024 && D % 4 == 0 &&
                     ((reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc)) & 15) == 0;
  const size_t smem = stage ? smem1 : smem0;
  const unsigned grid = (unsigned)(B * Hkv);
#define LZ_SWA_DEC(CT_, S_)                                                                   \
  {                                                                                           \
    static bool done[64] = {false};                                                           \
    int rc = ensure_decode_smem(swa_decode_kernel<XT, CT_, S_>, smem, done);                  \
    if (rc) return rc;                                                                        \
    swa_decode_kernel<XT, CT_, S_><<<grid, 32 * nw, smem, st>>>(                              \
        static_cast<const XT*>(q), q_sb, q_sh, static_cast<const XT*>(k), k_sb, k_sh,         \
        static_cast<const XT*>(v), v_sb, v_sh, static_cast<const CT_*>(cs),                   \
        static_cast<const CT_*>(sn), cs_sb, kc, vc, pos, meta, n_meta, y, H, Hkv, W, D);      \
  }
  if (cs_dtype == LZ_DTYPE_F32) {
    if (stage) LZ_SWA_DEC(float, true) else LZ_SWA_DEC(float, false)
  } else {
    if (stage) LZ_SWA_DEC(bf16, true) else LZ_SWA_DEC(bf16, false)
  }
#undef LZ_SWA_DEC
  count_launches(1);
  return check_launch("swa_decode_kernel");
}

}  // namespace
int decode_timeout_flag(unsigned int* out) { return tc::read_timeout_flag_here(out); }
int decode_timeout_clear() { return tc::clear_timeout_flag_here(); }

}  // namespace lz

extern "C" int lz_test_withhold_decode_ring_copy(int on) {
  lz::clear_error();
  const int v = on ? 1 : 0;
  cudaError_t e = cudaMemcpyToSymbol(lz::g_withhold_ring_copy, &v, sizeof(v));
  if (e != cudaSuccess) {
    lz::set_error(std::string("cudaMemcpyToSymbol: ") + cudaGetErrorString(e));
    return LZ_ERR_CUDA;
  }
  return LZ_OK;
}

extern "C" int lz_gla_decode(const void* fq, const void* fk, const void* v,
                             const float* log_gamma, int gate_per_head, float* state,
                             float* zstate, void* y, int B, int H, int Hkv, int Hs, int F, int D,
                             void* stream) {
  using namespace lz;
  clear_error();
  LZ_REQUIRE(B >= 1 && H >= 1 && Hkv >= 1 && F >= 1 && D >= 1, LZ_ERR_INVALID_ARGUMENT,
             "sizes must be positive");
  LZ_REQUIRE(H % Hkv == 0, LZ_ERR_INVALID_ARGUMENT,
             "the key/value head count must divide the query head count");
  LZ_REQUIRE(Hs == H || (Hs == Hkv && !gate_per_head), LZ_ERR_INVALID_ARGUMENT,
             "state heads must be H, or Hkv when the gate is shared by the heads");
  LZ_REQUIRE(F <= 256 && D % 4 == 0 && D <= 256, LZ_ERR_UNSUPPORTED,
             "decode supports F <= 256 and D a multiple of 4 up to 256");
  LZ_REQUIRE(fq && fk && v && log_gamma && state && zstate && y, LZ_ERR_INVALID_ARGUMENT,
             "null pointer");
  LZ_REQUIRE(aligned16(state), LZ_ERR_INVALID_ARGUMENT, "state must be 16-byte aligned");
  const int qs = H / Hs;
  const size_t smem = (size_t)(F + D + qs * F + qs * 1024 + qs * 8) * 4;
  auto st = static_cast<cudaStream_t>(stream);
  const unsigned grid = (unsigned)(B * Hs);
  const int gph = gate_per_head ? 1 : 0;
  auto fq_ = static_cast<const bf16*>(fq);
  auto fk_ = static_cast<const bf16*>(fk);
  auto v_ = static_cast<const bf16*>(v);
  auto y_ = static_cast<bf16*>(y);
  int rc = LZ_OK;
#define LZ_DEC(QS)                                                                           \
  case QS: {                                                                                 \
    static bool done[64] = {false};                                                          \
    rc = ensure_decode_smem(gla_decode_kernel<QS>, smem, done);                             \
    if (rc) return rc;                                                                       \
    gla_decode_kernel<QS><<<grid, kT, smem, st>>>(fq_, fk_, v_, log_gamma, gph, state, zstate, \
                                                  y_, H, Hkv, Hs, F, D);                     \
    break;                                                                                   \
  }
  switch (qs) {
    LZ_DEC(1) LZ_DEC(2) LZ_DEC(4) LZ_DEC(8) LZ_DEC(16)
    default:
      set_error("lz_gla_decode: query heads per state must be 1, 2, 4, 8 or 16");
      return LZ_ERR_UNSUPPORTED;
  }
#undef LZ_DEC
  count_launches(1);
  return check_launch("gla_decode_kernel");
}

extern "C" int lz_swa_decode(const void* q, const void* k, const void* v, int x_dtype,
                             long long q_sb, long long q_sh, long long k_sb, long long k_sh,
                             long long v_sb, long long v_sh, const void* cos, const void* sin,
                             int cs_dtype, long long cs_sb, float* k_ring, float* v_ring,
                             const int* pos, const float* meta, int n_meta, void* y, int B, int H,
                             int Hkv, int window, int D, void* stream) {
  using namespace lz;
  clear_error();
  LZ_REQUIRE(B >= 1 && H >= 1 && Hkv >= 1 && D >= 2 && window >= 1, LZ_ERR_INVALID_ARGUMENT,
             "sizes must be positive");
  LZ_REQUIRE(H % Hkv == 0, LZ_ERR_INVALID_ARGUMENT,
             "the key/value head count must divide the query head count");
  LZ_REQUIRE(D % 2 == 0, LZ_ERR_INVALID_ARGUMENT, "the rotated head dim must be even");
  LZ_REQUIRE(D <= 256 && window <= kMaxDecodeWindow, LZ_ERR_UNSUPPORTED,
             "decode supports D <= 256 and windows up to 1024");
  LZ_REQUIRE(n_meta >= 0 && n_meta <= 32 && (n_meta == 0 || meta), LZ_ERR_INVALID_ARGUMENT,
             "meta must hold n_meta (<= 32) values");
  LZ_REQUIRE(dtype_ok(x_dtype) && dtype_ok(cs_dtype), LZ_ERR_INVALID_ARGUMENT,
             "dtypes must be LZ_DTYPE_F32 or LZ_DTYPE_BF16");
  LZ_REQUIRE(q && k && v && cos && sin && k_ring && v_ring && pos && y,
             LZ_ERR_INVALID_ARGUMENT, "null pointer");
  auto st = static_cast<cudaStream_t>(stream);
  auto yb = static_cast<bf16*>(y);
  if (x_dtype == LZ_DTYPE_F32)
    return launch_swa_decode<float>(q, q_sb, q_sh, k, k_sb, k_sh, v, v_sb, v_sh, cos, sin,
                                    cs_dtype, cs_sb, k_ring, v_ring, pos, meta, n_meta, yb, B,
                                    H, Hkv, window, D, st);
  return launch_swa_decode<bf16>(q, q_sb, q_sh, k, k_sb, k_sh, v, v_sb, v_sh, cos, sin, cs_dtype,
                                 cs_sb, k_ring, v_ring, pos, meta, n_meta, yb, B, H, Hkv, window,
                                 D, st);
}
