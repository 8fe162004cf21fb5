// GLA backward. Four launches:
//   1. delta_i = dy_i . y_i (fp32 y saved by the forward; gla.py:242)
//   2. reverse walk over chunks writing the state gradient leaving each chunk,
//      dS_n (bf16) and dz_n (fp32)                       (gla.py:104-132)
//      (with the chunk-parallel schedule, 1 and 2 are gla_split.cu's
//      increment and scan kernels instead)
//   3. one CTA per (chunk, batch*head): dfq, dfk, dv and dG = sum_f(fq dfq -
//      fk dfk) for its 64 rows                         (gla.py:135-194, 254)
//   4. dlog_gamma = reverse cumsum of dG (summed over heads for a per-token
//      gate), the autograd of gla.py:260-262.
#include <mutex>

#include "common.cuh"
#include "gla_layout.h"

namespace lz {

namespace {
constexpr int kC = 64;

// ------------------------------------------------------------------ 1. delta
__global__ void gla_bwd_delta_kernel(const bf16* __restrict__ dy, const float* __restrict__ y32,
                                     float* __restrict__ delta, long long rows, int D) {
  const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const bf16* a = dy + row * D;
  const float* b = y32 + row * D;
  float acc = 0.f;
  for (int d = lane; d < D; d += 32) acc += __bfloat162float(a[d]) * b[d];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) delta[row] = acc;
}

// ------------------------------------------------------- 2. reverse state walk
struct StateSmem {
  static constexpr int LD = 64 + 8;
  static constexpr size_t tile = (size_t)kC * LD * 2;
  static constexpr size_t q = 0;              // 2 stages
  static constexpr size_t dy = q + 2 * tile;  // 2 stages
  static constexpr size_t g = dy + 2 * tile;  // 2 stages x (g, den, delta) x 64
  static constexpr size_t bytes = g + 2 * 3 * kC * 4;
};

__global__ void __launch_bounds__(128)
gla_bwd_state_kernel(const bf16* __restrict__ fq, const bf16* __restrict__ dy,
                     const float* __restrict__ G, const float* __restrict__ den,
                     const float* __restrict__ delta, bf16* __restrict__ ds,
                     float* __restrict__ dz_out, int L, int F, int D, int NT, int nfb, int ndb,
                     int vec_f, int vec_d) {
  using SM = StateSmem;
  constexpr int LD = SM::LD;
  extern __shared__ __align__(128) unsigned char smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, cq = lane & 3;
  int idx = blockIdx.x;
  const int db = idx % ndb;
  idx /= ndb;
  const int fb = idx % nfb;
  const int bh = idx / nfb;
  const int f0 = fb * 64, d0 = db * 64;
  const bf16* Q = fq + (size_t)bh * L * F;
  const bf16* DY = dy + (size_t)bh * L * D;
  const float* Gr = G + (size_t)bh * L;
  const float* DEN = den + (size_t)bh * L;
  const float* DEL = delta + (size_t)bh * L;

  auto sQ = [&](int s) { return reinterpret_cast<bf16*>(smem + SM::q + s * SM::tile); };
  auto sDy = [&](int s) { return reinterpret_cast<bf16*>(smem + SM::dy + s * SM::tile); };
  auto sRow = [&](int s) { return reinterpret_cast<float*>(smem + SM::g) + s * 3 * kC; };

  auto issue = [&](int n, int s) {
    const int r0 = n * kC;
    stage_tile<kC, 64, 128>(sQ(s), LD, Q, F, r0, L, f0, F, vec_f);
    stage_tile<kC, 64, 128>(sDy(s), LD, DY, D, r0, L, d0, D, vec_d);
    cp_async_commit();
    float* rw = sRow(s);
    if (tid < kC) {
      const int r = r0 + tid;
      rw[tid] = r < L ? Gr[r] : 0.f;
      rw[kC + tid] = r < L ? DEN[r] : 1.f;
      rw[2 * kC + tid] = r < L ? DEL[r] : 0.f;
    }
  };

  float acc[8][4];
#pragma unroll
  for (int c = 0; c < 8; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[c][e] = 0.f;
  float dz = 0.f;  // feature f0 + tid (tid < 64)

  issue(NT - 1, 0);
  for (int it = 0; it < NT; ++it) {
    const int n = NT - 1 - it, s = it & 1;
    // gradient leaving chunk n (used by the chunk kernel)
    {
      const size_t base = ((size_t)bh * NT + n) * F * D;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int f = f0 + 16 * warp + gq, d = d0 + 8 * nt + 2 * cq;
        if (f < F) {
          if (d < D) ds[base + (size_t)f * D + d] = __float2bfloat16_rn(acc[nt][0]);
          if (d + 1 < D) ds[base + (size_t)f * D + d + 1] = __float2bfloat16_rn(acc[nt][1]);
        }
        if (f + 8 < F) {
          if (d < D) ds[base + (size_t)(f + 8) * D + d] = __float2bfloat16_rn(acc[nt][2]);
          if (d + 1 < D) ds[base + (size_t)(f + 8) * D + d + 1] = __float2bfloat16_rn(acc[nt][3]);
        }
      }
      if (db == 0 && tid < 64 && f0 + tid < F) dz_out[((size_t)bh * NT + n) * F + f0 + tid] = dz;
    }
    if (n > 0) {
      issue(n - 1, s ^ 1);
      asm volatile("cp.async.wait_group 1;\n" ::);
    } else {
      cp_async_wait_all();
    }
    __syncthreads();
    const int r0 = n * kC, nvalid = min(kC, L - r0);
    const float* rw = sRow(s);
    const float start = n > 0 ? Gr[r0 - 1] : 0.f;
    const float end = rw[nvalid - 1];
    const float decay = __expf(end - start);
    bf16* q = sQ(s);
    // Q^ = bf16(fq * exp(G - start) / den), padded rows zero
    for (int i = tid; i < kC * 8; i += 128) {
      const int t = i >> 3, c = (i & 7) * 8;
      const float sc = t < nvalid ? __expf(rw[t] - start) / fmaxf(rw[kC + t], kTiny) : 0.f;
      uint4* p = reinterpret_cast<uint4*>(q + t * LD + c);
      uint4 w = *p;
      w.x = pack_bf16(bf16_lo(w.x) * sc, bf16_hi(w.x) * sc);
      w.y = pack_bf16(bf16_lo(w.y) * sc, bf16_hi(w.y) * sc);
      w.z = pack_bf16(bf16_lo(w.z) * sc, bf16_hi(w.z) * sc);
      w.w = pack_bf16(bf16_lo(w.w) * sc, bf16_hi(w.w) * sc);
      *p = w;
    }
    __syncthreads();
    if (tid < 64) {
      float sum = 0.f;
#pragma unroll 8
      for (int t = 0; t < kC; ++t) sum += __bfloat162float(q[t * LD + tid]) * rw[2 * kC + t];
      dz = dz * decay + sum;
    }
#pragma unroll
    for (int c = 0; c < 8; ++c)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[c][e] *= decay;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t a[4];
      lda_tr(a, q, LD, 16 * warp, 16 * j);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bb[4];
        ldb_kn(bb, sDy(s), LD, 16 * j, 16 * np);
        mma16816(acc[2 * np], a, bb[0], bb[1]);
        mma16816(acc[2 * np + 1], a, bb[2], bb[3]);
      }
    }
    __syncthreads();
  }
}

// ------------------------------------------------------ 3. per-chunk gradients
// One CTA of 8 warps per (chunk, batch*head). Warp w owns the 16-row strip
// (w & 3) of the chunk and the column half (w >> 2) of every output, so the
// per-warp accumulators stay small; the chunk's S and dS tiles are fetched
// while the scores are formed. Same algebra as gla.py:135-194:
//   a    = bf16(s * decay), s = fq fk^T, decay_it = exp(G_i - G_t), t <= i
//   da   = (dy v^T - delta) / den, dad = da * decay
//   dv   = (a / den)^T dy + bf16(fk * ks) dS
//   dfq  = qs/den * (dy S^T - delta z) + dad fk
//   dfk  = ks * (v dS^T - dz) + dad^T fq
//   dG_i = fq_i . dfq_i - fk_i . dfk_i                     (gla.py:254)
// with qs = exp(G_i - start), ks = exp(end - G_i). The chunk's sum of dG goes
// to dGt for the log-gate kernel.
template <int FP, int DP>
struct ChunkSmem {
  static constexpr int FB = FP < 64 ? FP : 64;  // feature block of S / dS
  static constexpr int LDF = FP + 8, LDD = DP + 8, LDT = kC + 8;
  static constexpr size_t q = 0;
  static constexpr size_t k = q + (size_t)kC * LDF * 2;
  static constexpr size_t v = k + (size_t)kC * LDF * 2;
  static constexpr size_t dy = v + (size_t)kC * LDD * 2;
  static constexpr size_t s = dy + (size_t)kC * LDD * 2;
  static constexpr size_t dS = s + (size_t)FB * LDD * 2;
  static constexpr size_t dad = dS + (size_t)FB * LDD * 2;
  static constexpr size_t aden = dad + (size_t)kC * LDT * 2;
  static constexpr size_t rows = aden + (size_t)kC * LDT * 2;  // g, 1/den, delta
  static constexpr size_t zz = rows + 3 * kC * 4;               // z, dz
  static constexpr size_t dgp = zz + 2 * FP * 4;                // dG of each column half
  static constexpr size_t red = dgp + 2 * kC * 4;
  static constexpr size_t bytes = red + 16;
};

template <int FP, int DP>
__global__ void __launch_bounds__(256, (FP <= 64 && DP <= 64) ? 2 : 1)
gla_bwd_chunk_kernel(const bf16* __restrict__ fq, const bf16* __restrict__ fk,
                     const bf16* __restrict__ v, const bf16* __restrict__ dy,
                     const float* __restrict__ G, const float* __restrict__ den,
                     const float* __restrict__ delta, const bf16* __restrict__ S,
                     const float* __restrict__ Z, const bf16* __restrict__ dS,
                     const float* __restrict__ dZ, void* __restrict__ dfq,
                     void* __restrict__ dfk, void* __restrict__ dv, int gdt, int gdt_kv,
                     float* __restrict__ dG, float* __restrict__ dGt, int H, int grp, int L, int F,
                     int D, int NT, int vec_f, int vec_d, int s_seeded, int ds_seeded) {
  using SM = ChunkSmem<FP, DP>;
  constexpr int FB = SM::FB, LDF = SM::LDF, LDD = SM::LDD, LDT = SM::LDT;
  constexpr int NDH = DP / 16;  // n8 tiles of one column half of dv
  constexpr int NFH = FB / 16;  // n8 tiles of one column half of a feature block
  extern __shared__ __align__(128) unsigned char smem[];
  bf16* sQ = reinterpret_cast<bf16*>(smem + SM::q);
  bf16* sK = reinterpret_cast<bf16*>(smem + SM::k);
  bf16* sV = reinterpret_cast<bf16*>(smem + SM::v);
  bf16* sDy = reinterpret_cast<bf16*>(smem + SM::dy);
  bf16* sS = reinterpret_cast<bf16*>(smem + SM::s);
  bf16* sDS = reinterpret_cast<bf16*>(smem + SM::dS);
  bf16* sDad = reinterpret_cast<bf16*>(smem + SM::dad);
  bf16* sAden = reinterpret_cast<bf16*>(smem + SM::aden);
  float* sG = reinterpret_cast<float*>(smem + SM::rows);
  float* sRden = sG + kC;
  float* sDel = sG + 2 * kC;
  float* sZ = reinterpret_cast<float*>(smem + SM::zz);
  float* sDZ = sZ + FP;
  float* sDgp = reinterpret_cast<float*>(smem + SM::dgp);
  float* sRed = reinterpret_cast<float*>(smem + SM::red);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, cq = lane & 3;
  const int strip = warp & 3, half = warp >> 2;
  const int n = blockIdx.x % NT, bh = blockIdx.x / NT;
  const int r0 = n * kC, nvalid = min(kC, L - r0);
  const size_t rowF = (size_t)bh * L * F, rowD = (size_t)bh * L * D;
  const size_t kvr = (size_t)kv_head(bh, H, grp) * L;  // rows of fk and v (GQA)
  const size_t chunk = (size_t)bh * NT + n;
  const bool with_s = n > 0 || s_seeded;       // state entering the chunk is not zero
  const bool with_ds = n + 1 < NT || ds_seeded;  // gradient leaving the chunk is not zero

  stage_tile<kC, FP, 256>(sQ, LDF, fq + rowF, F, r0, L, 0, F, vec_f);
  stage_tile<kC, FP, 256>(sK, LDF, fk + kvr * F, F, r0, L, 0, F, vec_f);
  stage_tile<kC, DP, 256>(sV, LDD, v + kvr * D, D, r0, L, 0, D, vec_d);
  stage_tile<kC, DP, 256>(sDy, LDD, dy + rowD, D, r0, L, 0, D, vec_d);
  cp_async_commit();
  auto stage_state = [&](int fo) {
    if (with_s) stage_tile<FB, DP, 256>(sS, LDD, S + chunk * F * D, D, fo, F, 0, D, vec_d);
    if (with_ds) stage_tile<FB, DP, 256>(sDS, LDD, dS + chunk * F * D, D, fo, F, 0, D, vec_d);
    cp_async_commit();
  };
  stage_state(0);
  if (tid < kC) {
    const int r = r0 + tid;
    sG[tid] = r < L ? G[(size_t)bh * L + r] : 0.f;
    sRden[tid] = r < L ? 1.f / fmaxf(den[(size_t)bh * L + r], kTiny) : 1.f;
    sDel[tid] = r < L ? delta[(size_t)bh * L + r] : 0.f;
  }
  for (int f = tid; f < FP; f += 256) {
    sZ[f] = (with_s && f < F) ? Z[chunk * F + f] : 0.f;
    sDZ[f] = (with_ds && f < F) ? dZ[chunk * F + f] : 0.f;
  }
  asm volatile("cp.async.wait_group 1;\n" ::);
  __syncthreads();

  const float start = n > 0 ? G[(size_t)bh * L + r0 - 1] : 0.f;
  const float end = sG[nvalid - 1];
  const int i0 = 16 * strip + gq, i1 = i0 + 8;  // rows of this thread (queries or keys)
  const float gi0 = sG[i0], gi1 = sG[i1];
  const float rd0 = sRden[i0], rd1 = sRden[i1];
  const float del0 = sDel[i0], del1 = sDel[i1];
  const int tc = 32 * half;  // this warp's 32 key columns in the score phase

  // (1) s = fq fk^T and p = dy v^T: 16 rows x 32 columns
  float sacc[4][4], pacc[4][4];
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) sacc[c][e] = pacc[c][e] = 0.f;
#pragma unroll 2
  for (int k0 = 0; k0 < FP; k0 += 16) {
    uint32_t a[4];
    lda_rm(a, sQ, LDF, 16 * strip, k0);
#pragma unroll
    for (int np = 0; np < 2; ++np) {
      uint32_t bb[4];
      ldb_nk(bb, sK, LDF, tc + 16 * np, k0);
      mma16816(sacc[2 * np], a, bb[0], bb[1]);
      mma16816(sacc[2 * np + 1], a, bb[2], bb[3]);
    }
  }
#pragma unroll 2
  for (int k0 = 0; k0 < DP; k0 += 16) {
    uint32_t a[4];
    lda_rm(a, sDy, LDD, 16 * strip, k0);
#pragma unroll
    for (int np = 0; np < 2; ++np) {
      uint32_t bb[4];
      ldb_nk(bb, sV, LDD, tc + 16 * np, k0);
      mma16816(pacc[2 * np], a, bb[0], bb[1]);
      mma16816(pacc[2 * np + 1], a, bb[2], bb[3]);
    }
  }
  // (2) dad = (p - delta)/den * decay and a/den, both bf16, into shared memory
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    const int t = tc + 8 * nt + 2 * cq;
    float dadv[4], adv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = (e < 2) ? i0 : i1;
      const int tt = t + (e & 1);
      const bool m = tt <= i && i < nvalid;
      const float dec = m ? __expf(((e < 2) ? gi0 : gi1) - sG[tt]) : 0.f;
      const float a = round_bf16(sacc[nt][e] * dec);
      const float rd = (e < 2) ? rd0 : rd1;
      const float da = m ? (pacc[nt][e] - ((e < 2) ? del0 : del1)) * rd : 0.f;
      dadv[e] = da * dec;
      adv[e] = a * rd;
    }
    *reinterpret_cast<uint32_t*>(sDad + i0 * LDT + t) = pack_bf16(dadv[0], dadv[1]);
    *reinterpret_cast<uint32_t*>(sDad + i1 * LDT + t) = pack_bf16(dadv[2], dadv[3]);
    *reinterpret_cast<uint32_t*>(sAden + i0 * LDT + t) = pack_bf16(adv[0], adv[1]);
    *reinterpret_cast<uint32_t*>(sAden + i1 * LDT + t) = pack_bf16(adv[2], adv[3]);
  }
  __syncthreads();

  // (3) dv (intra) = (a/den)^T dy: key rows of the strip, value columns of the half
  const int dc = half * (DP / 2);
  float dvacc[NDH][4];
#pragma unroll
  for (int c = 0; c < NDH; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) dvacc[c][e] = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t a[4];
    lda_tr(a, sAden, LDT, 16 * strip, 16 * j);
#pragma unroll
    for (int np = 0; np < NDH / 2; ++np) {
      uint32_t bb[4];
      ldb_kn(bb, sDy, LDD, 16 * j, dc + 16 * np);
      mma16816(dvacc[2 * np], a, bb[0], bb[1]);
      mma16816(dvacc[2 * np + 1], a, bb[2], bb[3]);
    }
  }

  const bool v0 = i0 < nvalid, v1 = i1 < nvalid;
  const float qsd0 = v0 ? __expf(gi0 - start) * rd0 : 0.f;
  const float qsd1 = v1 ? __expf(gi1 - start) * rd1 : 0.f;
  const float ks0 = v0 ? __expf(end - gi0) : 0.f;
  const float ks1 = v1 ? __expf(end - gi1) : 0.f;
  const bool fpair = (F & 1) == 0;
  float dg0 = 0.f, dg1 = 0.f;

  for (int fb = 0; fb < FP / FB; ++fb) {
    const int fo = fb * FB;
    if (fb > 0) stage_state(fo);
    cp_async_wait_all();
    __syncthreads();
    const int fcl = half * (FB / 2);  // this warp's columns inside the feature block
    // (4) dfq = qs/den (dy S^T - delta z) + dad fk
    {
      float acc[NFH][4];
#pragma unroll
      for (int c = 0; c < NFH; ++c)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[c][e] = 0.f;
      if (with_s) {
#pragma unroll 2
        for (int k0 = 0; k0 < DP; k0 += 16) {
          uint32_t a[4];
          lda_rm(a, sDy, LDD, 16 * strip, k0);
#pragma unroll
          for (int np = 0; np < NFH / 2; ++np) {
            uint32_t bb[4];
            ldb_nk(bb, sS, LDD, fcl + 16 * np, k0);
            mma16816(acc[2 * np], a, bb[0], bb[1]);
            mma16816(acc[2 * np + 1], a, bb[2], bb[3]);
          }
        }
      }
#pragma unroll
      for (int nt = 0; nt < NFH; ++nt) {
        const int f = fo + fcl + 8 * nt + 2 * cq;
        acc[nt][0] = qsd0 * (acc[nt][0] - del0 * sZ[f]);
        acc[nt][1] = qsd0 * (acc[nt][1] - del0 * sZ[f + 1]);
        acc[nt][2] = qsd1 * (acc[nt][2] - del1 * sZ[f]);
        acc[nt][3] = qsd1 * (acc[nt][3] - del1 * sZ[f + 1]);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t a[4];
        lda_rm(a, sDad, LDT, 16 * strip, 16 * j);
#pragma unroll
        for (int np = 0; np < NFH / 2; ++np) {
          uint32_t bb[4];
          ldb_kn(bb, sK, LDF, 16 * j, fo + fcl + 16 * np);
          mma16816(acc[2 * np], a, bb[0], bb[1]);
          mma16816(acc[2 * np + 1], a, bb[2], bb[3]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < NFH; ++nt) {
        const int f = fo + fcl + 8 * nt + 2 * cq;
        if (f >= F) continue;
        const bool has1 = f + 1 < F;
        dg0 += __bfloat162float(sQ[i0 * LDF + f]) * acc[nt][0] +
               (has1 ? __bfloat162float(sQ[i0 * LDF + f + 1]) * acc[nt][1] : 0.f);
        dg1 += __bfloat162float(sQ[i1 * LDF + f]) * acc[nt][2] +
               (has1 ? __bfloat162float(sQ[i1 * LDF + f + 1]) * acc[nt][3] : 0.f);
        if (v0) store_grad2(dfq, rowF + (size_t)(r0 + i0) * F + f, acc[nt][0], acc[nt][1], has1, fpair, gdt);
        if (v1) store_grad2(dfq, rowF + (size_t)(r0 + i1) * F + f, acc[nt][2], acc[nt][3], has1, fpair, gdt);
      }
    }
    // (5) dfk = ks (v dS^T - dz) + dad^T fq
    {
      float acc[NFH][4];
#pragma unroll
      for (int c = 0; c < NFH; ++c)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[c][e] = 0.f;
      if (with_ds) {
#pragma unroll 2
        for (int k0 = 0; k0 < DP; k0 += 16) {
          uint32_t a[4];
          lda_rm(a, sV, LDD, 16 * strip, k0);
#pragma unroll
          for (int np = 0; np < NFH / 2; ++np) {
            uint32_t bb[4];
            ldb_nk(bb, sDS, LDD, fcl + 16 * np, k0);
            mma16816(acc[2 * np], a, bb[0], bb[1]);
            mma16816(acc[2 * np + 1], a, bb[2], bb[3]);
          }
        }
      }
#pragma unroll
      for (int nt = 0; nt < NFH; ++nt) {
        const int f = fo + fcl + 8 * nt + 2 * cq;
        acc[nt][0] = ks0 * (acc[nt][0] - sDZ[f]);
        acc[nt][1] = ks0 * (acc[nt][1] - sDZ[f + 1]);
        acc[nt][2] = ks1 * (acc[nt][2] - sDZ[f]);
        acc[nt][3] = ks1 * (acc[nt][3] - sDZ[f + 1]);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t a[4];
        lda_tr(a, sDad, LDT, 16 * strip, 16 * j);
#pragma unroll
        for (int np = 0; np < NFH / 2; ++np) {
          uint32_t bb[4];
          ldb_kn(bb, sQ, LDF, 16 * j, fo + fcl + 16 * np);
          mma16816(acc[2 * np], a, bb[0], bb[1]);
          mma16816(acc[2 * np + 1], a, bb[2], bb[3]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < NFH; ++nt) {
        const int f = fo + fcl + 8 * nt + 2 * cq;
        if (f >= F) continue;
        const bool has1 = f + 1 < F;
        dg0 -= __bfloat162float(sK[i0 * LDF + f]) * acc[nt][0] +
               (has1 ? __bfloat162float(sK[i0 * LDF + f + 1]) * acc[nt][1] : 0.f);
        dg1 -= __bfloat162float(sK[i1 * LDF + f]) * acc[nt][2] +
               (has1 ? __bfloat162float(sK[i1 * LDF + f + 1]) * acc[nt][3] : 0.f);
        if (v0) store_grad2(dfk, rowF + (size_t)(r0 + i0) * F + f, acc[nt][0], acc[nt][1], has1, fpair, gdt_kv);
        if (v1) store_grad2(dfk, rowF + (size_t)(r0 + i1) * F + f, acc[nt][2], acc[nt][3], has1, fpair, gdt_kv);
      }
    }
    // (6) dv (inter) += bf16(fk * ks) dS over this feature block
    if (with_ds) {
#pragma unroll
      for (int k0 = 0; k0 < FB; k0 += 16) {
        uint32_t a[4];
        lda_rm(a, sK, LDF, 16 * strip, fo + k0);
        a[0] = pack_bf16(bf16_lo(a[0]) * ks0, bf16_hi(a[0]) * ks0);
        a[1] = pack_bf16(bf16_lo(a[1]) * ks1, bf16_hi(a[1]) * ks1);
        a[2] = pack_bf16(bf16_lo(a[2]) * ks0, bf16_hi(a[2]) * ks0);
        a[3] = pack_bf16(bf16_lo(a[3]) * ks1, bf16_hi(a[3]) * ks1);
#pragma unroll
        for (int np = 0; np < NDH / 2; ++np) {
          uint32_t bb[4];
          ldb_kn(bb, sDS, LDD, k0, dc + 16 * np);
          mma16816(dvacc[2 * np], a, bb[0], bb[1]);
          mma16816(dvacc[2 * np + 1], a, bb[2], bb[3]);
        }
      }
    }
    __syncthreads();  // sS, sDS are restaged for the next feature block
  }
  // (7) dv, dG and the chunk's sum of dG
  const bool dpair = (D & 1) == 0;
#pragma unroll
  for (int nt = 0; nt < NDH; ++nt) {
    const int d = dc + 8 * nt + 2 * cq;
    if (d >= D) continue;
    const bool has1 = d + 1 < D;
    if (v0) store_grad2(dv, rowD + (size_t)(r0 + i0) * D + d, dvacc[nt][0], dvacc[nt][1], has1, dpair, gdt_kv);
    if (v1) store_grad2(dv, rowD + (size_t)(r0 + i1) * D + d, dvacc[nt][2], dvacc[nt][3], has1, dpair, gdt_kv);
  }
  dg0 = quad_sum(dg0);
  dg1 = quad_sum(dg1);
  if (cq == 0) {
    sDgp[half * kC + i0] = dg0;
    sDgp[half * kC + i1] = dg1;
  }
  __syncthreads();
  if (tid < kC) {
    float x = tid < nvalid ? sDgp[tid] + sDgp[kC + tid] : 0.f;
    if (tid < nvalid) dG[(size_t)bh * L + r0 + tid] = x;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    if (lane == 0) sRed[warp] = x;
  }
  __syncthreads();
  if (tid == 0) dGt[chunk] = sRed[0] + sRed[1];
}

// --------------------------------------------------- 4. log-gate gradient
// out[j] = sum_{i >= j} x[i], x = dG (per-head gate) or the sum over heads of
// dG (gate shared by the heads of a batch row): the autograd of the cumsum and
// expand of gla.py:260-262. One CTA of C threads (C = the chunk length of dGt,
// 64 or 128) per (gate row, chunk): the carry is the sum of the later chunks'
// totals (dGt), added in a fixed order, then a suffix scan over the chunk's
// rows. Deterministic.
__global__ void __launch_bounds__(128)
gla_bwd_gate_kernel(const float* __restrict__ dG, const float* __restrict__ dGt,
                    float* __restrict__ out, int H, int L, int NT, int gate_per_head) {
  __shared__ float red[128];
  __shared__ float wtot[4];
  const int C = blockDim.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = blockIdx.x % NT, row = blockIdx.x / NT;
  const int h0 = gate_per_head ? row : row * H;  // first batch*head row of this gate row
  const int nh = gate_per_head ? 1 : H;
  const int later = NT - 1 - n;
  float c = 0.f;
  for (int i = tid; i < nh * later; i += C) {
    const int h = i / later, m = n + 1 + i % later;
    c += dGt[(size_t)(h0 + h) * NT + m];
  }
  red[tid] = c;
  __syncthreads();
  for (int w = C / 2; w > 0; w >>= 1) {
    if (tid < w) red[tid] += red[tid + w];
    __syncthreads();
  }
  const float carry = red[0];
  const int j = n * C + tid;
  float x = 0.f;
  if (j < L) {
    const float* p = dG + (size_t)h0 * L + j;
    for (int h = 0; h < nh; ++h) x += p[(size_t)h * L];
  }
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float u = __shfl_down_sync(0xffffffffu, x, o);
    if (lane + o < 32) x += u;
  }
  if (lane == 0) wtot[warp] = x;
  __syncthreads();
  float after = 0.f;
  for (int w = warp + 1; w < C / 32; ++w) after += wtot[w];
  if (j < L) out[(size_t)row * L + j] = carry + x + after;
}

int launch_gate(const float* dg, const float* dgt, float* dlg, int B, int H, int L, int NT, int C,
                int gph, cudaStream_t stream) {
  const int gate_rows = gph ? B * H : B;
  gla_bwd_gate_kernel<<<(unsigned)((long long)gate_rows * NT), C, 0, stream>>>(dg, dgt, dlg, H, L,
                                                                               NT, gph);
  count_launches(1);
  return check_launch("gla_bwd_gate_kernel");
}

std::mutex g_attr_mu;

template <typename Kern>
int ensure_smem(Kern k, size_t bytes, bool* done) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(g_attr_mu);
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

// Gradients of grouped keys / values (GQA): out[kvh] = sum_g in[kvh * grp + g]
// over the grp query heads that read key/value head kvh, added in head order
// in fp32 (the autograd of the caller's repeat_interleave,
// src/lizard_attention.py:76). per_head = L * cols elements; 4 per thread
// when per_head % 4 == 0 (the scratch is 256-byte aligned).
template <int V>
__global__ void __launch_bounds__(256)
gla_group_sum_kernel(const float* __restrict__ in, void* __restrict__ out, int gdt, int grp,
                     long long per_head, long long n_items) {
  for (long long e = blockIdx.x * 256ll + threadIdx.x; e < n_items;
       e += (long long)gridDim.x * 256) {
    const long long o = e * V;
    const long long kvh = o / per_head, r = o - kvh * per_head;
    const float* src = in + kvh * grp * per_head + r;
    float acc[V];
    if constexpr (V == 4) {
      float4 a = *reinterpret_cast<const float4*>(src);
      for (int g = 1; g < grp; ++g) {
        const float4 b = *reinterpret_cast<const float4*>(src + g * per_head);
        a.x += b.x;
        a.y += b.y;
        a.z += b.z;
        a.w += b.w;
      }
      acc[0] = a.x;
      acc[1] = a.y;
      acc[2] = a.z;
      acc[3] = a.w;
    } else {
      acc[0] = src[0];
      for (int g = 1; g < grp; ++g) acc[0] += src[g * per_head];
    }
#pragma unroll
    for (int u = 0; u < V; u += 2) {
      if constexpr (V == 1)
        store_grad(out, (size_t)o, acc[0], gdt);
      else
        store_grad2(out, (size_t)(o + u), acc[u], acc[u + 1], true, true, gdt);
    }
  }
}

int launch_group_sum(const float* in, void* out, int gdt, int n_kv, int grp, long long per_head,
                     cudaStream_t st) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const bool v4 = per_head % 4 == 0 && aligned16(in) &&
                  (reinterpret_cast<uintptr_t>(out) & (gdt == LZ_DTYPE_BF16 ? 3 : 7)) == 0;
  const long long n_items = (long long)n_kv * per_head / (v4 ? 4 : 1);
  const long long want = (n_items + 255) / 256, cap = (long long)sms * 8;
  const unsigned grid = (unsigned)(want < cap ? (want > 0 ? want : 1) : cap);
  if (v4)
    gla_group_sum_kernel<4><<<grid, 256, 0, st>>>(in, out, gdt, grp, per_head, n_items);
  else
    gla_group_sum_kernel<1><<<grid, 256, 0, st>>>(in, out, gdt, grp, per_head, n_items);
  count_launches(1);
  return check_launch("gla_group_sum_kernel");
}

template <int FP, int DP>
int launch_chunk(const bf16* fq, const bf16* fk, const bf16* v, const bf16* dy,
                 const GlaSaved& sv, const GlaWork& wk, void* dfq, void* dfk, void* dv, int gdt,
                 int gdt_kv, int BH, int H, int grp, int L, int F, int D, int NT, int vec_f,
                 int vec_d, int s_seeded, int ds_seeded, cudaStream_t st) {
  using SM = ChunkSmem<FP, DP>;
  static bool done[64] = {false};
  int rc = ensure_smem(gla_bwd_chunk_kernel<FP, DP>, SM::bytes, done);
  if (rc) return rc;
  gla_bwd_chunk_kernel<FP, DP><<<(unsigned)((long long)BH * NT), 256, SM::bytes, st>>>(
      fq, fk, v, dy, sv.g, sv.den, wk.delta, sv.s, sv.z, wk.ds, wk.dz, dfq, dfk, dv, gdt, gdt_kv,
      wk.dg, wk.dgt, H, grp, L, F, D, NT, vec_f, vec_d, s_seeded, ds_seeded);
  count_launches(1);
  return check_launch("gla_bwd_chunk_kernel");
}

}  // namespace

int gla_bwd_tail(const bf16* fq, const bf16* fk, const bf16* v, int gph, const GlaSaved& sv,
                 const bf16* dy, void* dfq, void* dfk, void* dv, int gdt, int gdt_kv, float* dlg,
                 const GlaWork& wk, int B, int H, int Hkv, int L, int F, int D, int s_seeded,
                 int ds_seeded, cudaStream_t stream) {
  const int BH = B * H, grp = H / Hkv;
  const int NT = (int)gla_nt(L);
  // F = D = 64: per-chunk gradients on the tensor cores over 128-token chunks,
  // reading the scan's 64-token states at stride two (gla_bwd_tc.cu)
  if (F == 64 && D == 64 && gla_split_out_tc_enabled() && aligned16(fq) && aligned16(fk) &&
      aligned16(v) && aligned16(dy) && aligned16(sv.s) && aligned16(wk.ds) &&
      (gdt != LZ_DTYPE_BF16 || aligned16(dfq)) &&
      (gdt_kv != LZ_DTYPE_BF16 || (aligned16(dfk) && aligned16(dv)))) {
    int rc = gla_bwd_tc_chunks(fq, fk, v, dy, sv, wk, dfq, dfk, dv, gdt, gdt_kv, B, H, Hkv, L,
                               s_seeded, ds_seeded, stream, true);
    if (rc) return rc;
    return launch_gate(wk.dg, wk.dgt, dlg, B, H, L, (L + 127) / 128, 128, gph, stream);
  }
  const int vec_f = (F % 8 == 0) && aligned16(fq) && aligned16(fk);
  const int vec_d = (D % 8 == 0) && aligned16(v) && aligned16(dy) && aligned16(sv.s) &&
                    aligned16(wk.ds);
  const int FP = F <= 32 ? 32 : F <= 64 ? 64 : F <= 128 ? 128 : 256;
  const int DP = D <= 32 ? 32 : D <= 64 ? 64 : 128;
  int rc = LZ_OK;
#define LZ_CHUNK_CASE(fp, dp)                                                                  \
  if (FP == fp && DP == dp)                                                                    \
    rc = launch_chunk<fp, dp>(fq, fk, v, dy, sv, wk, dfq, dfk, dv, gdt, gdt_kv, BH, H, grp, L, \
                              F, D, NT, vec_f, vec_d, s_seeded, ds_seeded, stream);            \
  else
  LZ_CHUNK_CASE(32, 32) LZ_CHUNK_CASE(32, 64) LZ_CHUNK_CASE(32, 128)
  LZ_CHUNK_CASE(64, 32) LZ_CHUNK_CASE(64, 64) LZ_CHUNK_CASE(64, 128)
  LZ_CHUNK_CASE(128, 32) LZ_CHUNK_CASE(128, 64) LZ_CHUNK_CASE(128, 128)
  LZ_CHUNK_CASE(256, 32) LZ_CHUNK_CASE(256, 64) LZ_CHUNK_CASE(256, 128) {
    set_error("gla_bwd: no kernel for this feature/value size");
    return LZ_ERR_UNSUPPORTED;
  }
#undef LZ_CHUNK_CASE
  if (rc) return rc;

  return launch_gate(wk.dg, wk.dgt, dlg, B, H, L, NT, kC, gph, stream);
}

int gla_bwd(const bf16* fq, const bf16* fk, const bf16* v, const float* lg, int gph,
            const GlaSaved& sv, const bf16* dy, void* dfq, void* dfk, void* dv, int gdt,
            float* dlg, const GlaWork& wk, int B, int H, int Hkv, int L, int F, int D,
            cudaStream_t stream) {
  (void)lg;
  const int BH = B * H;
  const int NT = (int)gla_nt(L);
  int rc = LZ_OK;
  // grouped keys / values: per-query-head dfk, dv into fp32 scratch, then summed
  const bool gqa = Hkv != H;
  void* dfk_h = gqa ? static_cast<void*>(wk.gk) : dfk;
  void* dv_h = gqa ? static_cast<void*>(wk.gv) : dv;
  const int gdt_kv = gqa ? LZ_DTYPE_F32 : gdt;
  auto finish = [&]() -> int {
    if (!gqa) return LZ_OK;
    int r = launch_group_sum(wk.gk, dfk, gdt, B * Hkv, H / Hkv, (long long)L * F, stream);
    if (r) return r;
    return launch_group_sum(wk.gv, dv, gdt, B * Hkv, H / Hkv, (long long)L * D, stream);
  };
  if (gla_saved_chunk(B, H, L, F, D, fq, fk, v) == 128) {
    // states on the tensor-core forward's 128-token boundaries
    rc = gla_bwd_tc_states(fq, dy, sv, wk, B, H, L, stream);
    if (rc) return rc;
    rc = gla_bwd_tc_chunks(fq, fk, v, dy, sv, wk, dfq, dfk_h, dv_h, gdt, gdt_kv, B, H, Hkv, L, 0,
                           0, stream);
    if (rc) return rc;
    rc = launch_gate(wk.dg, wk.dgt, dlg, B, H, L, (L + 127) / 128, 128, gph, stream);
    if (rc) return rc;
    return finish();
  }
  if (wk.inc) {
    rc = gla_bwd_split_states(fq, dy, sv, wk, B, H, L, F, D, stream);
    if (rc) return rc;
  } else {
    const int vec_f = (F % 8 == 0) && aligned16(fq);
    const int vec_d = (D % 8 == 0) && aligned16(dy);
    const long long rows = (long long)BH * L;
    gla_bwd_delta_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, stream>>>(dy, sv.y32, wk.delta,
                                                                         rows, D);
    count_launches(1);
    rc = check_launch("gla_bwd_delta_kernel");
    if (rc) return rc;
    static bool done[64] = {false};
    rc = ensure_smem(gla_bwd_state_kernel, StateSmem::bytes, done);
    if (rc) return rc;
    const int nfb = ceil_div(F, 64), ndb = ceil_div(D, 64);
    gla_bwd_state_kernel<<<(unsigned)((long long)BH * nfb * ndb), 128, StateSmem::bytes,
                           stream>>>(fq, dy, sv.g, sv.den, wk.delta, wk.ds, wk.dz, L, F, D, NT,
                                     nfb, ndb, vec_f, vec_d);
    count_launches(1);
    rc = check_launch("gla_bwd_state_kernel");
    if (rc) return rc;
  }
  rc = gla_bwd_tail(fq, fk, v, gph, sv, dy, dfq, dfk_h, dv_h, gdt, gdt_kv, dlg, wk, B, H, Hkv, L,
                    F, D, 0, 0, stream);
  if (rc) return rc;
  return finish();
}

}  // namespace lz
