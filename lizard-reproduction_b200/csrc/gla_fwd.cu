// GLA forward: one fused kernel per (batch*head, value slice) that walks the
// 64-token chunks in order, keeping the running state S (F x DV, fp32) in
// registers and its bf16 copy in shared memory, so S never goes to HBM.
//
// Algorithm (chunked GLA of the reference, src/kernels/gla.py:19-101):
//   G      = cumsum(log_gamma)               (computed here, gla.py:260)
//   start  = G[chunk_start-1] (0 for the first chunk), end = G[last row]
//   Q~_i   = bf16(fq_i * exp(G_i - start))    (gla.py:84)
//   K~_t   = bf16(fk_t * exp(end - G_t))      (gla.py:55)
//   a_it   = bf16((fq_i . fk_t) * exp(G_i - G_t)), t <= i in the chunk (gla.py:85-90)
//   num_i  = Q~_i S + sum_t a_it v_t,  den_i = Q~_i . z + sum_t a_it   (gla.py:86-95)
//   y_i    = num_i / max(den_i, FLT_MIN)     (gla.py:96)
//   S     <- S * exp(end - start) + K~^T V,  z <- z * exp(end - start) + sum_t K~_t
//                                             (gla.py:56-57)
// The reference splits this into a state kernel that writes S for every
// chunk to HBM and an output kernel that reads it back; here both live in
// one pass.
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "gla_chunk.cuh"
#include "gla_layout.h"

namespace lz {

constexpr int kChunk = 64;

template <int FP, int DV>
struct GlaFwdSmem {
  static constexpr int LDQ = FP + 8;  // padded row (bf16) -> conflict-free ldmatrix
  static constexpr int LDV = DV + 8;
  static constexpr size_t q = 0;
  static constexpr size_t k = q + (size_t)kChunk * LDQ * 2;
  static constexpr size_t v = k + (size_t)kChunk * LDQ * 2;
  static constexpr size_t s = v + (size_t)kChunk * LDV * 2;
  static constexpr size_t z = s + (size_t)FP * LDV * 2;
  static constexpr size_t g = z + (size_t)FP * 4;
  static constexpr size_t scan = g + kChunk * 4;
  static constexpr size_t bytes = scan + 16;
};

template <int FP, int DV>
__global__ void __launch_bounds__(128, 2)
gla_fwd_kernel(const bf16* __restrict__ fq, const bf16* __restrict__ fk,
               const bf16* __restrict__ v, const float* __restrict__ lg, int gate_per_head,
               int H, int grp, int L, int F, int D, int NT, int nslices, int vec_f, int vec_d,
               bf16* __restrict__ y, float* __restrict__ y32, float* __restrict__ den_out,
               float* __restrict__ g_out, bf16* __restrict__ s_out, float* __restrict__ z_out) {
  using SM = GlaFwdSmem<FP, DV>;
  constexpr int LDQ = SM::LDQ, LDV = SM::LDV;
  constexpr int MT = FP / 16;          // 16-row tiles of the state (rows = features)
  constexpr int MTW = (MT + 3) / 4;    // state tiles per warp
  constexpr int NTV = DV / 8;          // 8-col tiles of the value slice
  extern __shared__ __align__(128) unsigned char smem[];
  bf16* sQ = reinterpret_cast<bf16*>(smem + SM::q);
  bf16* sK = reinterpret_cast<bf16*>(smem + SM::k);
  bf16* sV = reinterpret_cast<bf16*>(smem + SM::v);
  bf16* sS = reinterpret_cast<bf16*>(smem + SM::s);
  float* sZ = reinterpret_cast<float*>(smem + SM::z);
  float* sG = reinterpret_cast<float*>(smem + SM::g);
  float* sScan = reinterpret_cast<float*>(smem + SM::scan);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, cq = lane & 3;
  const int slice = blockIdx.x % nslices;
  const int bh = blockIdx.x / nslices;
  const int b = bh / H;
  const int d0 = slice * DV;
  const bool save = (y32 != nullptr);
  const bool lead = (slice == 0);  // writes per-row / per-feature saves once
  const bf16* Q = fq + (size_t)bh * L * F;
  const size_t kvr = (size_t)kv_head(bh, H, grp) * L;  // key/value rows (GQA)
  const bf16* K = fk + kvr * F;
  const bf16* V = v + kvr * D;
  const float* LG = lg + (size_t)(gate_per_head ? bh : b) * L;

  for (int i = tid; i < FP; i += 128) sZ[i] = 0.f;
  for (int i = tid; i < FP * LDV; i += 128) sS[i] = __float2bfloat16_rn(0.f);
  if (save) {  // S_0 = 0, z_0 = 0
    const size_t sb = (size_t)bh * NT * F * D;
    for (int i = tid; i < F * DV; i += 128) {
      const int f = i / DV, d = d0 + i % DV;
      if (d < D) s_out[sb + (size_t)f * D + d] = __float2bfloat16_rn(0.f);
    }
    if (lead)
      for (int f = tid; f < F; f += 128) z_out[(size_t)bh * NT * F + f] = 0.f;
  }

  float st[MTW][NTV][4];
#pragma unroll
  for (int a = 0; a < MTW; ++a)
#pragma unroll
    for (int c = 0; c < NTV; ++c)
#pragma unroll
      for (int e = 0; e < 4; ++e) st[a][c][e] = 0.f;

  stage_tile<kChunk, FP, 128>(sQ, LDQ, Q, F, 0, L, 0, F, vec_f);
  stage_tile<kChunk, FP, 128>(sK, LDQ, K, F, 0, L, 0, F, vec_f);
  stage_tile<kChunk, DV, 128>(sV, LDV, V, D, 0, L, d0, D, vec_d);
  cp_async_commit();

  float carry = 0.f;
  for (int n = 0; n < NT; ++n) {
    const int r0 = n * kChunk;
    const int nvalid = min(kChunk, L - r0);
    // chunk-local inclusive scan of the log gates (two warps of 32)
    if (tid < kChunk) {
      float x = tid < nvalid ? LG[r0 + tid] : 0.f;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += u;
      }
      sG[tid] = x;
      if (lane == 31) sScan[warp] = x;
    }
    cp_async_wait_all();
    __syncthreads();
    if (tid < kChunk) {
      const float gv = sG[tid] + carry + (tid >= 32 ? sScan[0] : 0.f);
      sG[tid] = gv;
      if (save && lead && tid < nvalid) g_out[(size_t)bh * L + r0 + tid] = gv;
    }
    __syncthreads();
    const float start = carry;
    const float end = sG[nvalid - 1];
    carry = end;

    gla_chunk_output<FP, DV>(sQ, sK, sV, sS, sZ, sG, start, nvalid, n > 0,
                             (size_t)bh * L + r0, D, d0, y, save ? y32 : nullptr,
                             (save && lead) ? den_out + (size_t)bh * L + r0 : nullptr);
    __syncthreads();  // sQ, sS, sZ no longer read in this chunk
    if (n + 1 < NT) {
      stage_tile<kChunk, FP, 128>(sQ, LDQ, Q, F, r0 + kChunk, L, 0, F, vec_f);
      cp_async_commit();
    }
    // (f) K~ in place of fk; padded rows become zero
    for (int i = tid; i < kChunk * FP / 8; i += 128) {
      const int t = i / (FP / 8), c = (i % (FP / 8)) * 8;
      const float ks = t < nvalid ? __expf(end - sG[t]) : 0.f;
      uint4* p = reinterpret_cast<uint4*>(sK + t * LDQ + c);
      uint4 w = *p;
      w.x = pack_bf16(bf16_lo(w.x) * ks, bf16_hi(w.x) * ks);
      w.y = pack_bf16(bf16_lo(w.y) * ks, bf16_hi(w.y) * ks);
      w.z = pack_bf16(bf16_lo(w.z) * ks, bf16_hi(w.z) * ks);
      w.w = pack_bf16(bf16_lo(w.w) * ks, bf16_hi(w.w) * ks);
      *p = w;
    }
    __syncthreads();
    const float decay = __expf(end - start);
    for (int f = tid; f < FP; f += 128) {
      float acc = 0.f;
#pragma unroll 8
      for (int t = 0; t < kChunk; ++t) acc += __bfloat162float(sK[t * LDQ + f]);
      const float zn = sZ[f] * decay + acc;
      sZ[f] = zn;
      if (save && lead && n + 1 < NT && f < F) z_out[((size_t)bh * NT + n + 1) * F + f] = zn;
    }
    // (g) S <- S * decay + K~^T V
#pragma unroll
    for (int a = 0; a < MTW; ++a)
#pragma unroll
      for (int c = 0; c < NTV; ++c)
#pragma unroll
        for (int e = 0; e < 4; ++e) st[a][c][e] *= decay;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t bv[NTV / 2][4];
#pragma unroll
      for (int np = 0; np < NTV / 2; ++np) ldb_kn(bv[np], sV, LDV, 16 * j, 16 * np);
#pragma unroll
      for (int mi = 0; mi < MTW; ++mi) {
        const int mt = warp + 4 * mi;
        if (mt < MT) {
          uint32_t a[4];
          lda_tr(a, sK, LDQ, 16 * mt, 16 * j);
#pragma unroll
          for (int np = 0; np < NTV / 2; ++np) {
            mma16816(st[mi][2 * np], a, bv[np][0], bv[np][1]);
            mma16816(st[mi][2 * np + 1], a, bv[np][2], bv[np][3]);
          }
        }
      }
    }
    __syncthreads();  // sK, sV free
    if (n + 1 < NT) {
      stage_tile<kChunk, FP, 128>(sK, LDQ, K, F, r0 + kChunk, L, 0, F, vec_f);
      stage_tile<kChunk, DV, 128>(sV, LDV, V, D, r0 + kChunk, L, d0, D, vec_d);
      cp_async_commit();
    }
    // (h) publish bf16 S_{n+1}
#pragma unroll
    for (int mi = 0; mi < MTW; ++mi) {
      const int mt = warp + 4 * mi;
      if (mt >= MT) continue;
#pragma unroll
      for (int nt = 0; nt < NTV; ++nt) {
        const int f = 16 * mt + gq, dl = 8 * nt + 2 * cq;
        const uint32_t p0 = pack_bf16(st[mi][nt][0], st[mi][nt][1]);
        const uint32_t p1 = pack_bf16(st[mi][nt][2], st[mi][nt][3]);
        *reinterpret_cast<uint32_t*>(sS + f * LDV + dl) = p0;
        *reinterpret_cast<uint32_t*>(sS + (f + 8) * LDV + dl) = p1;
        if (save && n + 1 < NT) {
          const size_t sb = ((size_t)bh * NT + n + 1) * F * D;
          const int d = d0 + dl;
          const __nv_bfloat162 h0 = *reinterpret_cast<const __nv_bfloat162*>(&p0);
          const __nv_bfloat162 h1 = *reinterpret_cast<const __nv_bfloat162*>(&p1);
          if (f < F) {
            if (d < D) s_out[sb + (size_t)f * D + d] = h0.x;
            if (d + 1 < D) s_out[sb + (size_t)f * D + d + 1] = h0.y;
          }
          if (f + 8 < F) {
            if (d < D) s_out[sb + (size_t)(f + 8) * D + d] = h1.x;
            if (d + 1 < D) s_out[sb + (size_t)(f + 8) * D + d + 1] = h1.y;
          }
        }
      }
    }
  }
}

namespace {

template <int FP, int DV>
int launch_fwd(const bf16* fq, const bf16* fk, const bf16* v, const float* lg, int gph, int B,
               int H, int grp, int L, int F, int D, int vec_f, int vec_d, bf16* y,
               const GlaSaved& sv, cudaStream_t stream) {
  using SM = GlaFwdSmem<FP, DV>;
  static std::mutex mu;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 64 && !attr_done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(gla_fwd_kernel<FP, DV>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)SM::bytes);
      if (e != cudaSuccess) {
        set_error(std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
        return LZ_ERR_CUDA;
      }
      attr_done[dev] = true;
    }
  }
  const int NT = ceil_div(L, kChunk);
  const int nslices = ceil_div(D, DV);
  const long long grid = (long long)B * H * nslices;
  gla_fwd_kernel<FP, DV><<<(unsigned)grid, 128, SM::bytes, stream>>>(
      fq, fk, v, lg, gph, H, grp, L, F, D, NT, nslices, vec_f, vec_d, y, sv.y32, sv.den, sv.g,
      sv.s, sv.z);
  count_launches(1);
  return check_launch("gla_fwd_kernel");
}

}  // namespace

int gla_fwd_tc(const bf16* fq, const bf16* fk, const bf16* v, const float* lg, int gph, bf16* y,
               const GlaSaved& sv, int B, int H, int Hkv, int L, int F, int D,
               cudaStream_t stream);
int gla_fwd_tc64(const bf16* fq, const bf16* fk, const bf16* v, const float* lg, int gph,
                 bf16* y, const GlaSaved& sv, int B, int H, int Hkv, int L, int F, int D,
                 cudaStream_t stream);

namespace {
std::atomic<int> g_fwd_tc64{0};
}  // namespace
int gla_set_fwd_tc64(int on) { return g_fwd_tc64.exchange(on ? 1 : 0); }

int gla_fwd(const bf16* fq, const bf16* fk, const bf16* v, const float* lg, int gph, bf16* y,
            const GlaSaved& sv, const GlaFwdWork& fw, int B, int H, int Hkv, int L, int F, int D,
            cudaStream_t stream) {
  if (fw.inc)
    return gla_fwd_split_run(fq, fk, v, lg, gph, y, sv, fw, B, H, Hkv, L, F, D, stream);
  const int BH = B * H, grp = H / Hkv;
  if (gla_saved_chunk(B, H, L, F, D, fq, fk, v) == 128) {
    // tensor-core kernels (two sequences per SM with 64-token chunks, or one
    // with 128-token chunks); in training they also save the 128-token chunk states
    if (g_fwd_tc64.load(std::memory_order_relaxed)) {
      const int rc = gla_fwd_tc64(fq, fk, v, lg, gph, y, sv, B, H, Hkv, L, F, D, stream);
      if (rc != LZ_ERR_UNSUPPORTED) return rc;
    }
    const int rc = gla_fwd_tc(fq, fk, v, lg, gph, y, sv, B, H, Hkv, L, F, D, stream);
    if (rc != LZ_ERR_UNSUPPORTED) return rc;
    if (sv.y32) {
      set_error("gla_fwd: the tensor-core forward is unavailable (tensor map encoding failed)");
      return LZ_ERR_CUDA;
    }
  }
  const int FP = F <= 32 ? 32 : F <= 64 ? 64 : F <= 128 ? 128 : 256;
  int DV = D <= 16 ? 16 : D <= 32 ? 32 : (FP <= 128 ? 64 : 32);
  while (DV > 16 && (long long)BH * ceil_div(D, DV) < 2 * 148) DV /= 2;
  const int vec_f = (F % 8 == 0) && aligned16(fq) && aligned16(fk);
  const int vec_d = (D % 8 == 0) && aligned16(v);
#define LZ_FWD_CASE(fp, dv) \
  if (FP == fp && DV == dv) \
    return launch_fwd<fp, dv>(fq, fk, v, lg, gph, B, H, grp, L, F, D, vec_f, vec_d, y, sv, \
                              stream);
  LZ_FWD_CASE(32, 16) LZ_FWD_CASE(32, 32) LZ_FWD_CASE(32, 64)
  LZ_FWD_CASE(64, 16) LZ_FWD_CASE(64, 32) LZ_FWD_CASE(64, 64)
  LZ_FWD_CASE(128, 16) LZ_FWD_CASE(128, 32) LZ_FWD_CASE(128, 64)
  LZ_FWD_CASE(256, 16) LZ_FWD_CASE(256, 32)
#undef LZ_FWD_CASE
  set_error("gla_fwd: no kernel for this feature/value size");
  return LZ_ERR_UNSUPPORTED;
}

}  // namespace lz
