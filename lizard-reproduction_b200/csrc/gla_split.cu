// Chunk-parallel ("split") schedule of GLA, for calls whose batch*heads are
// too few for one sequential walk per head to fill the GPU (B=1, H=32 is 32
// chains on 148 SMs).
//
// The reference's state pass walks the chunks of a head one after another
// (src/kernels/gla.py:33-57 forward, 104-132 backward). Its recurrence is
// linear, S_{n+1} = e^{lam_n} S_n + K~_n^T V_n with lam_n = G_end - G_start of
// chunk n, so it splits into
//   1. increments: every chunk's K~_n^T V_n and sum_t K~_t at once (fp32),
//      together with lam_n, from a chunk-local scan of the log gates;
//   2. scan: an elementwise walk over the chunks, one thread per 2 state
//      entries, writing the bf16 state entering every chunk (the layout the
//      reference stores, gla.py:48-51) -- in fp32 the same products and sums
//      as the reference's walk;
//   3. output: every chunk's y at once from its state (gla.py:60-101).
// The backward reuses step 2 in reverse order on the increments
// Q^_n^T dY_n and Q^_n^T delta_n (gla.py:120-132), whose kernel also forms
// delta = dy . y32 (gla.py:242).
//
// The scan also takes an optional seed (the state entering the first chunk)
// and can return the state after the last chunk, which is all a
// sequence-parallel caller needs to hand a segment's state to the next one.
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "gla_chunk.cuh"
#include "gla_layout.h"

namespace lz {

namespace {

constexpr int kC = 64;
constexpr int kLD = 64 + 8;  // padded bf16 row of a 64-column tile

std::atomic<int> g_schedule{kScheduleAuto};

std::mutex g_split_mu;
template <typename Kern>
int ensure_smem_split(Kern k, size_t bytes, bool* done) {
  if (bytes <= 48 * 1024) return LZ_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(g_split_mu);
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

// Inclusive scan of one chunk's log gates, chunk-local (0 before the chunk).
// Rows past the end of the sequence add 0. Threads 0..63 take part; the whole
// block must call it (it synchronises).
__device__ __forceinline__ void chunk_gate_scan(const float* __restrict__ LG, int r0, int nvalid,
                                                float* sG, float* sScan) {
  const int tid = threadIdx.x, lane = tid & 31;
  if (tid < kC) {
    float x = tid < nvalid ? LG[r0 + tid] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float u = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += u;
    }
    sG[tid] = x;
    if (tid == 31) sScan[0] = x;
  }
  __syncthreads();
  if (tid >= 32 && tid < kC) sG[tid] += sScan[0];
  __syncthreads();
}

// Scales the rows of a staged 64x64 tile in place: row t times sc(t), bf16.
template <typename Scale>
__device__ __forceinline__ void scale_rows(bf16* tile, Scale sc) {
  for (int i = threadIdx.x; i < kC * 8; i += 128) {
    const int t = i >> 3, c = (i & 7) * 8;
    const float s = sc(t);
    uint4* p = reinterpret_cast<uint4*>(tile + t * kLD + c);
    uint4 w = *p;
    w.x = pack_bf16(bf16_lo(w.x) * s, bf16_hi(w.x) * s);
    w.y = pack_bf16(bf16_lo(w.y) * s, bf16_hi(w.y) * s);
    w.z = pack_bf16(bf16_lo(w.z) * s, bf16_hi(w.z) * s);
    w.w = pack_bf16(bf16_lo(w.w) * s, bf16_hi(w.w) * s);
    *p = w;
  }
}

// acc (this warp's 16 rows of A^T B, 64 columns) for 64x64 tiles A (rows =
// chunk rows, columns = state rows) and B (rows = chunk rows).
__device__ __forceinline__ void tile_atb(float (&acc)[8][4], const bf16* A, const bf16* Bt) {
  const int warp = threadIdx.x >> 5;
#pragma unroll
  for (int c = 0; c < 8; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[c][e] = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t a[4];
    lda_tr(a, A, kLD, 16 * warp, 16 * j);
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t bb[4];
      ldb_kn(bb, Bt, kLD, 16 * j, 16 * np);
      mma16816(acc[2 * np], a, bb[0], bb[1]);
      mma16816(acc[2 * np + 1], a, bb[2], bb[3]);
    }
  }
}

// Stores a warp's 16 x 64 fp32 block into a row-major [F, D] matrix at
// (f0 + 16*warp, d0), masked to F x D.
__device__ __forceinline__ void store_block_f32(float* __restrict__ m, const float (&acc)[8][4],
                                                int f0, int d0, int F, int D) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gq = lane >> 2, cq = lane & 3;
  const bool pair = (D & 1) == 0;
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    const int d = d0 + 8 * nt + 2 * cq;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int f = f0 + 16 * warp + gq + 8 * h;
      if (f >= F || d >= D) continue;
      float* p = m + (size_t)f * D + d;
      if (pair) {
        *reinterpret_cast<float2*>(p) = make_float2(acc[nt][2 * h], acc[nt][2 * h + 1]);
      } else {
        p[0] = acc[nt][2 * h];
        if (d + 1 < D) p[1] = acc[nt][2 * h + 1];
      }
    }
  }
}

// ------------------------------------------------- 1f. forward increments
// One CTA per (chunk, batch*head, 64-feature block, 64-value block):
//   inc_n = K~_n^T V_n, K~_t = bf16(fk_t exp(G_end - G_t))   (gla.py:53-56)
//   incz_n = sum_t K~_t (fp32 sum of the bf16 values, gla.py:57)
//   lam_n = G_end - G_start
__global__ void __launch_bounds__(128)
gla_split_finc_kernel(const bf16* __restrict__ fk, const bf16* __restrict__ v,
                      const float* __restrict__ lg, int gph, int H, int grp, int L, int F, int D,
                      int NT, int nfb, int ndb, int vec_f, int vec_d, float* __restrict__ inc,
                      float* __restrict__ incz, float* __restrict__ lam) {
  __shared__ __align__(16) bf16 sK[kC * kLD];
  __shared__ __align__(16) bf16 sV[kC * kLD];
  __shared__ float sG[kC];
  __shared__ float sScan[1];
  const int tid = threadIdx.x;
  int idx = blockIdx.x;
  const int db = idx % ndb;
  idx /= ndb;
  const int fb = idx % nfb;
  idx /= nfb;
  const int n = idx % NT, bh = idx / NT;
  const int f0 = fb * 64, d0 = db * 64, r0 = n * kC, nvalid = min(kC, L - r0);
  const float* LG = lg + (size_t)(gph ? bh : bh / H) * L;

  const size_t kvr = (size_t)kv_head(bh, H, grp) * L;
  stage_tile<kC, 64, 128>(sK, kLD, fk + kvr * F, F, r0, L, f0, F, vec_f);
  stage_tile<kC, 64, 128>(sV, kLD, v + kvr * D, D, r0, L, d0, D, vec_d);
  cp_async_commit();
  chunk_gate_scan(LG, r0, nvalid, sG, sScan);
  cp_async_wait_all();
  __syncthreads();
  const float total = sG[nvalid - 1];
  scale_rows(sK, [&](int t) { return t < nvalid ? __expf(total - sG[t]) : 0.f; });
  __syncthreads();
  const size_t chunk = (size_t)bh * NT + n;
  if (db == 0 && tid < 64 && f0 + tid < F) {
    float sum = 0.f;
#pragma unroll 8
    for (int t = 0; t < kC; ++t) sum += __bfloat162float(sK[t * kLD + tid]);
    incz[chunk * F + f0 + tid] = sum;
  }
  if (fb == 0 && db == 0 && tid == 0) lam[chunk] = total;
  float acc[8][4];
  tile_atb(acc, sK, sV);
  store_block_f32(inc + chunk * F * D, acc, f0, d0, F, D);
}

// ------------------------------------------------ 1b. backward increments
// One CTA per (chunk, batch*head, feature block, value block):
//   delta_t = dy_t . y32_t                                    (gla.py:242)
//   Q^_t = bf16(fq_t exp(G_t - G_start) / den_t)              (gla.py:129)
//   inc_n = Q^_n^T dY_n, incz_n = sum_t Q^_t delta_t          (gla.py:130-132)
//   lam_n = G_end - G_start
__global__ void __launch_bounds__(128)
gla_split_binc_kernel(const bf16* __restrict__ fq, const bf16* __restrict__ dy,
                      const float* __restrict__ y32, const float* __restrict__ G,
                      const float* __restrict__ den, int L, int F, int D, int NT, int nfb,
                      int ndb, int vec_f, int vec_d, int vec_dots, float* __restrict__ delta_out,
                      float* __restrict__ inc, float* __restrict__ incz,
                      float* __restrict__ lam) {
  __shared__ __align__(16) bf16 sQ[kC * kLD];
  __shared__ __align__(16) bf16 sDy[kC * kLD];
  __shared__ float sGl[kC], sDen[kC], sDel[kC];
  const int tid = threadIdx.x;
  int idx = blockIdx.x;
  const int db = idx % ndb;
  idx /= ndb;
  const int fb = idx % nfb;
  idx /= nfb;
  const int n = idx % NT, bh = idx / NT;
  const int f0 = fb * 64, d0 = db * 64, r0 = n * kC, nvalid = min(kC, L - r0);
  const size_t rowb = (size_t)bh * L;

  stage_tile<kC, 64, 128>(sQ, kLD, fq + rowb * F, F, r0, L, f0, F, vec_f);
  stage_tile<kC, 64, 128>(sDy, kLD, dy + rowb * D, D, r0, L, d0, D, vec_d);
  cp_async_commit();
  const float start = n > 0 ? G[rowb + r0 - 1] : 0.f;
  if (tid < kC) {
    const bool ok = tid < nvalid;
    sGl[tid] = ok ? G[rowb + r0 + tid] - start : 0.f;
    sDen[tid] = ok ? den[rowb + r0 + tid] : 1.f;
  }
  // delta over the full value dim
  block_row_dots64(dy + (rowb + r0) * D, y32 + (rowb + r0) * D, nvalid, D, vec_dots, sDel);
  cp_async_wait_all();
  __syncthreads();
  scale_rows(sQ, [&](int t) {
    return t < nvalid ? __expf(sGl[t]) / fmaxf(sDen[t], kTiny) : 0.f;
  });
  if (fb == 0 && db == 0 && tid < nvalid) delta_out[rowb + r0 + tid] = sDel[tid];
  __syncthreads();
  const size_t chunk = (size_t)bh * NT + n;
  if (db == 0 && tid < 64 && f0 + tid < F) {
    float sum = 0.f;
#pragma unroll 8
    for (int t = 0; t < kC; ++t) sum += __bfloat162float(sQ[t * kLD + tid]) * sDel[t];
    incz[chunk * F + f0 + tid] = sum;
  }
  if (fb == 0 && db == 0 && tid == 0) lam[chunk] = sGl[nvalid - 1];
  float acc[8][4];
  tile_atb(acc, sQ, sDy);
  store_block_f32(inc + chunk * F * D, acc, f0, d0, F, D);
}

// ------------------------------------------------------------- 2. scan
// Walks the chunks of every (batch*head) in order (reverse = 0) or backwards
// (reverse = 1); h starts at the seed (or 0) and at each chunk n
//   out_n = bf16(h)  (z: fp32),  h = h * exp(lam_n) + inc_n.
// Items of one batch*head: F*D/VEC state items, F normaliser items and one
// gate item (gs_n = sum_{m<n} lam_m in the forward; gtot = sum of all lam).
// Loads run kStep chunks ahead of the dependent multiply-adds.
constexpr int kStep = 16;

template <int VEC>
__global__ void __launch_bounds__(256)
gla_split_scan_kernel(const float* __restrict__ inc, const float* __restrict__ incz,
                      const float* __restrict__ lam, int BH, int NT, int F, int D, int reverse,
                      const float* __restrict__ seed, const float* __restrict__ seedz,
                      bf16* __restrict__ s_out, float* __restrict__ z_out,
                      float* __restrict__ fin, float* __restrict__ finz,
                      float* __restrict__ gs, float* __restrict__ gtot) {
  const size_t FD = (size_t)F * D;
  const int nS = (int)(FD / VEC);
  const int per = nS + F + 1;
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= (long long)BH * per) return;
  const int bh = (int)(gid / per), item = (int)(gid % per);
  const float* LAM = lam + (size_t)bh * NT;

  if (item == nS + F) {  // gate offsets (gs: forward only) and the total log decay
    float acc = 0.f;
    for (int n = 0; n < NT; ++n) {
      if (gs && !reverse) gs[(size_t)bh * NT + n] = acc;
      acc += LAM[n];
    }
    if (gtot) gtot[bh] = acc;
    return;
  }
  if (item >= nS) {  // normaliser z, one feature
    const int f = item - nS;
    float h = seedz ? seedz[(size_t)bh * F + f] : 0.f;
    for (int s0 = 0; s0 < NT; s0 += kStep) {
      float u[kStep], e[kStep];
#pragma unroll
      for (int j = 0; j < kStep; ++j) {
        const int st = s0 + j;
        const int n = reverse ? NT - 1 - st : st;
        u[j] = st < NT ? __ldg(incz + ((size_t)bh * NT + n) * F + f) : 0.f;
        e[j] = st < NT ? __expf(__ldg(LAM + n)) : 1.f;
      }
#pragma unroll
      for (int j = 0; j < kStep; ++j) {
        const int st = s0 + j;
        if (st >= NT) break;
        const int n = reverse ? NT - 1 - st : st;
        if (z_out) z_out[((size_t)bh * NT + n) * F + f] = h;
        h = h * e[j] + u[j];
      }
    }
    if (finz) finz[(size_t)bh * F + f] = h;
    return;
  }
  // state entries e0 .. e0+VEC-1
  const size_t e0 = (size_t)item * VEC;
  float h[VEC];
#pragma unroll
  for (int c = 0; c < VEC; ++c) h[c] = seed ? seed[(size_t)bh * FD + e0 + c] : 0.f;
  for (int s0 = 0; s0 < NT; s0 += kStep) {
    float u[kStep][VEC], e[kStep];
#pragma unroll
    for (int j = 0; j < kStep; ++j) {
      const int st = s0 + j;
      const int n = reverse ? NT - 1 - st : st;
      const float* p = inc + ((size_t)bh * NT + n) * FD + e0;
      if (st < NT) {
        if constexpr (VEC == 2) {
          const float2 w = __ldg(reinterpret_cast<const float2*>(p));
          u[j][0] = w.x, u[j][1] = w.y;
        } else {
#pragma unroll
          for (int c = 0; c < VEC; ++c) u[j][c] = __ldg(p + c);
        }
        e[j] = __expf(__ldg(LAM + n));
      } else {
#pragma unroll
        for (int c = 0; c < VEC; ++c) u[j][c] = 0.f;
        e[j] = 1.f;
      }
    }
#pragma unroll
    for (int j = 0; j < kStep; ++j) {
      const int st = s0 + j;
      if (st >= NT) break;
      const int n = reverse ? NT - 1 - st : st;
      if (s_out) {
        bf16* q = s_out + ((size_t)bh * NT + n) * FD + e0;
        if constexpr (VEC == 2) {
          *reinterpret_cast<uint32_t*>(q) = pack_bf16(h[0], h[1]);
        } else {
#pragma unroll
          for (int c = 0; c < VEC; ++c) q[c] = __float2bfloat16_rn(h[c]);
        }
      }
#pragma unroll
      for (int c = 0; c < VEC; ++c) h[c] = h[c] * e[j] + u[j][c];
    }
  }
  if (fin) {
#pragma unroll
    for (int c = 0; c < VEC; ++c) fin[(size_t)bh * FD + e0 + c] = h[c];
  }
}

// ------------------------------------------------------------ 3. output
// One CTA per (chunk, batch*head, value slice): y of the chunk's rows from the
// state entering the chunk (gla.py:60-101). Gates in the chunk-local frame.
template <int FP, int DV>
struct SplitOutSmem {
  static constexpr int LDQ = FP + 8, LDV = DV + 8;
  static constexpr size_t q = 0;
  static constexpr size_t k = q + (size_t)kC * LDQ * 2;
  static constexpr size_t v = k + (size_t)kC * LDQ * 2;
  static constexpr size_t s = v + (size_t)kC * LDV * 2;
  static constexpr size_t z = s + (size_t)FP * LDV * 2;
  static constexpr size_t g = z + (size_t)FP * 4;
  static constexpr size_t scan = g + kC * 4;
  static constexpr size_t bytes = scan + 16;
};

template <int FP, int DV>
__global__ void __launch_bounds__(128)
gla_split_out_kernel(const bf16* __restrict__ fq, const bf16* __restrict__ fk,
                     const bf16* __restrict__ v, const float* __restrict__ lg, int gph, int H,
                     int grp, int sgrp, int L, int F, int D, int NT, int nslices, int vec_f,
                     int vec_d, int vec_s,
                     const bf16* __restrict__ s_in, const float* __restrict__ z_in,
                     const float* __restrict__ gs, int seeded, bf16* __restrict__ y,
                     float* __restrict__ y32, float* __restrict__ den_out,
                     float* __restrict__ g_out) {
  using SM = SplitOutSmem<FP, DV>;
  extern __shared__ __align__(128) unsigned char smem[];
  bf16* sQ = reinterpret_cast<bf16*>(smem + SM::q);
  bf16* sK = reinterpret_cast<bf16*>(smem + SM::k);
  bf16* sV = reinterpret_cast<bf16*>(smem + SM::v);
  bf16* sS = reinterpret_cast<bf16*>(smem + SM::s);
  float* sZ = reinterpret_cast<float*>(smem + SM::z);
  float* sG = reinterpret_cast<float*>(smem + SM::g);
  float* sScan = reinterpret_cast<float*>(smem + SM::scan);
  const int tid = threadIdx.x;
  int idx = blockIdx.x;
  const int slice = idx % nslices;
  idx /= nslices;
  const int n = idx % NT, bh = idx / NT;
  const int r0 = n * kC, nvalid = min(kC, L - r0), d0 = slice * DV;
  const bool lead = slice == 0;
  // states, normalisers and gate offsets: per query head, or per key/value head
  // when the gate is shared by the heads (sgrp query heads per state)
  const size_t chunk = (size_t)(sgrp > 1 ? kv_head(bh, H, sgrp) : bh) * NT + n;
  const size_t rowb = (size_t)bh * L;
  const bool with_state = n > 0 || seeded;

  stage_tile<kC, FP, 128>(sQ, SM::LDQ, fq + rowb * F, F, r0, L, 0, F, vec_f);
  const size_t kvr = (size_t)kv_head(bh, H, grp) * L;
  stage_tile<kC, FP, 128>(sK, SM::LDQ, fk + kvr * F, F, r0, L, 0, F, vec_f);
  stage_tile<kC, DV, 128>(sV, SM::LDV, v + kvr * D, D, r0, L, d0, D, vec_d);
  if (with_state) stage_tile<FP, DV, 128>(sS, SM::LDV, s_in + chunk * F * D, D, 0, F, d0, D, vec_s);
  cp_async_commit();
  for (int f = tid; f < FP; f += 128) sZ[f] = (with_state && f < F) ? z_in[chunk * F + f] : 0.f;
  chunk_gate_scan(lg + (size_t)(gph ? bh : bh / H) * L, r0, nvalid, sG, sScan);
  cp_async_wait_all();
  __syncthreads();
  if (g_out && lead && tid < nvalid) g_out[rowb + r0 + tid] = gs[chunk] + sG[tid];
  gla_chunk_output<FP, DV>(sQ, sK, sV, sS, sZ, sG, 0.f, nvalid, with_state, rowb + r0, D, d0, y,
                           y32, (y32 && lead) ? den_out + rowb + r0 : nullptr);
}

template <int FP, int DV>
int launch_out(const bf16* fq, const bf16* fk, const bf16* v, const float* lg, int gph, int BH,
               int H, int grp, int sgrp, int L, int F, int D, int NT, const bf16* s_in,
               const float* z_in,
               const float* gs, int seeded, bf16* y, float* y32, float* den, float* g_out,
               cudaStream_t st) {
  using SM = SplitOutSmem<FP, DV>;
  static bool done[64] = {false};
  int rc = ensure_smem_split(gla_split_out_kernel<FP, DV>, SM::bytes, done);
  if (rc) return rc;
  const int nslices = ceil_div(D, DV);
  const int vec_f = (F % 8 == 0) && aligned16(fq) && aligned16(fk);
  const int vec_d = (D % 8 == 0) && aligned16(v);
  const int vec_s = (D % 8 == 0) && aligned16(s_in);
  gla_split_out_kernel<FP, DV><<<(unsigned)((long long)BH * NT * nslices), 128, SM::bytes, st>>>(
      fq, fk, v, lg, gph, H, grp, sgrp, L, F, D, NT, nslices, vec_f, vec_d, vec_s, s_in, z_in,
      gs, seeded, y, y32, den, g_out);
  count_launches(1);
  return check_launch("gla_split_out_kernel");
}

int launch_scan(const float* inc, const float* incz, const float* lam, int BH, int NT, int F,
                int D, int reverse, const float* seed, const float* seedz, bf16* s_out,
                float* z_out, float* fin, float* finz, float* gs, float* gtot, cudaStream_t st) {
  const size_t FD = (size_t)F * D;
  auto a8 = [](const void* p) { return ((uintptr_t)p & 7) == 0; };
  const bool v2 = FD % 2 == 0 && a8(inc) && (!seed || a8(seed)) && (!fin || a8(fin)) &&
                  (!s_out || ((uintptr_t)s_out & 3) == 0);
  const long long per = (long long)(v2 ? FD / 2 : FD) + F + 1;
  const long long threads = (long long)BH * per;
  const unsigned grid = (unsigned)((threads + 255) / 256);
  if (v2)
    gla_split_scan_kernel<2><<<grid, 256, 0, st>>>(inc, incz, lam, BH, NT, F, D, reverse, seed,
                                                   seedz, s_out, z_out, fin, finz, gs, gtot);
  else
    gla_split_scan_kernel<1><<<grid, 256, 0, st>>>(inc, incz, lam, BH, NT, F, D, reverse, seed,
                                                   seedz, s_out, z_out, fin, finz, gs, gtot);
  count_launches(1);
  return check_launch("gla_split_scan_kernel");
}

}  // namespace

int gla_schedule_override() { return g_schedule.load(std::memory_order_relaxed); }

// Tensor-core chunk outputs in the chunk-parallel forward (on by default;
// tests switch them off to compare with the warp-MMA output kernel). The
// setting must not change between a forward and its backward.
std::atomic<int> g_out_tc{1};
bool gla_split_out_tc_enabled() { return g_out_tc.load(std::memory_order_relaxed) != 0; }
int gla_set_out_tc(int on) { return g_out_tc.exchange(on ? 1 : 0); }

int gla_set_schedule(int s) { return g_schedule.exchange(s); }

int gla_fwd_split_run(const bf16* fq, const bf16* fk, const bf16* v, const float* lg, int gph,
                      bf16* y, const GlaSaved& sv, const GlaFwdWork& fw, int B, int H, int Hkv,
                      int L, int F, int D, cudaStream_t stream) {
  const int BH = B * H, NT = (int)gla_nt(L), grp = H / Hkv;
  const int nfb = ceil_div(F, 64), ndb = ceil_div(D, 64);
  const int vec_f = (F % 8 == 0) && aligned16(fk);
  const int vec_d = (D % 8 == 0) && aligned16(v);
  const bool save = sv.y32 != nullptr;
  // With a gate shared by the heads, the query heads of a key/value group have
  // identical chunk states: without a backward to feed (which reads states per
  // query head), increments and scan run once per key/value head.
  const bool share = !save && !gph && grp > 1;
  const int Hs = share ? Hkv : H, BHs = B * Hs;
  gla_split_finc_kernel<<<(unsigned)((long long)BHs * NT * nfb * ndb), 128, 0, stream>>>(
      fk, v, lg, gph, Hs, share ? 1 : grp, L, F, D, NT, nfb, ndb, vec_f, vec_d, fw.inc, fw.incz,
      fw.lam);
  count_launches(1);
  int rc = check_launch("gla_split_finc_kernel");
  if (rc) return rc;
  bf16* s = save ? sv.s : fw.s;
  float* z = save ? sv.z : fw.z;
  rc = launch_scan(fw.inc, fw.incz, fw.lam, BHs, NT, F, D, 0, nullptr, nullptr, s, z, nullptr,
                   nullptr, save ? fw.gs : nullptr, nullptr, stream);
  if (rc) return rc;
  if (gla_split_out_tc_enabled()) {  // tensor-core chunk outputs (also in training)
    rc = gla_out_tc(fq, fk, v, lg, gph, B, H, Hkv, share ? grp : 1, L, F, D, s, z, y, sv,
                    save ? fw.gs : nullptr, stream);
    if (rc != LZ_ERR_UNSUPPORTED) return rc;
  }
  const int FP = F <= 32 ? 32 : F <= 64 ? 64 : F <= 128 ? 128 : 256;
  const int DV = D <= 16 ? 16 : D <= 32 ? 32 : 64;
  float* y32 = save ? sv.y32 : nullptr;
#define LZ_OUT_CASE(fp, dv)                                                                   \
  if (FP == fp && DV == dv)                                                                   \
    return launch_out<fp, dv>(fq, fk, v, lg, gph, BH, H, grp, share ? grp : 1, L, F, D, NT, s, \
                              z, fw.gs, 0, y, y32, sv.den, save ? sv.g : nullptr, stream);
  LZ_OUT_CASE(32, 16) LZ_OUT_CASE(32, 32) LZ_OUT_CASE(32, 64)
  LZ_OUT_CASE(64, 16) LZ_OUT_CASE(64, 32) LZ_OUT_CASE(64, 64)
  LZ_OUT_CASE(128, 16) LZ_OUT_CASE(128, 32) LZ_OUT_CASE(128, 64)
  LZ_OUT_CASE(256, 16) LZ_OUT_CASE(256, 32) LZ_OUT_CASE(256, 64)
#undef LZ_OUT_CASE
  set_error("gla_fwd: no chunk-parallel kernel for this feature/value size");
  return LZ_ERR_UNSUPPORTED;
}

int gla_bwd_split_states(const bf16* fq, const bf16* dy, const GlaSaved& sv, const GlaWork& wk,
                         int B, int H, int L, int F, int D, cudaStream_t stream) {
  (void)H;
  const int BH = B * H, NT = (int)gla_nt(L);
  const int nfb = ceil_div(F, 64), ndb = ceil_div(D, 64);
  const int vec_f = (F % 8 == 0) && aligned16(fq);
  const int vec_d = (D % 8 == 0) && aligned16(dy);
  const int vec_dots = (D % 4 == 0) && ((uintptr_t)dy & 7) == 0 && aligned16(sv.y32);
  gla_split_binc_kernel<<<(unsigned)((long long)BH * NT * nfb * ndb), 128, 0, stream>>>(
      fq, dy, sv.y32, sv.g, sv.den, L, F, D, NT, nfb, ndb, vec_f, vec_d, vec_dots, wk.delta,
      wk.inc, wk.incz, wk.lam);
  count_launches(1);
  int rc = check_launch("gla_split_binc_kernel");
  if (rc) return rc;
  return launch_scan(wk.inc, wk.incz, wk.lam, BH, NT, F, D, 1, nullptr, nullptr, wk.ds, wk.dz,
                     nullptr, nullptr, nullptr, nullptr, stream);
}

// ------------------------------------------------ sequence-parallel segments
// A rank that owns a contiguous segment of the sequence runs the schedule
// above on its segment in the segment's own gate frame (G = 0 before its first
// token). The only data that crosses ranks is one summary per rank:
//   state [BH, F, D] | zstate [BH, F] | logdecay [BH]      (fp32)
// forward: the state after the segment from a zero start and its total log
// decay; backward: the gradient w.r.t. the state entering the segment from
// the segment's own outputs, and again the log decay.
namespace {

// seed_r = walk over the ranks before r (forward) or after r (backward):
// h <- h * exp(logdecay_q) + state_q, in rank order (reverse: from the last).
__global__ void __launch_bounds__(256)
gla_seg_combine_kernel(const float* __restrict__ summ, int P, int rank, int reverse, int BH,
                       int F, int D, float* __restrict__ seed) {
  const size_t FD = (size_t)F * D, nS = (size_t)BH * FD, nZ = (size_t)BH * F;
  const size_t per = nS + nZ + BH;
  const size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= nS + nZ) return;
  const int bh = e < nS ? (int)(e / FD) : (int)((e - nS) / F);
  float h = 0.f;
  if (!reverse) {
    for (int q = 0; q < rank; ++q)
      h = h * __expf(summ[q * per + nS + nZ + bh]) + summ[q * per + e];
  } else {
    for (int q = P - 1; q > rank; --q)
      h = h * __expf(summ[q * per + nS + nZ + bh]) + summ[q * per + e];
  }
  seed[e] = h;
}

// dlog_gamma[row, :] += sum over the ranks after `rank` of their totals[row]
// (each rank's total is its own dlog_gamma[row, 0]): the reverse cumsum of the
// log-gate gradient continues across the later segments.
__global__ void __launch_bounds__(256)
gla_seg_gate_offset_kernel(float* __restrict__ dlg, const float* __restrict__ totals, int P,
                           int rank, int rows, int L) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)rows * L) return;
  const int row = (int)(i / L);
  float off = 0.f;
  for (int q = P - 1; q > rank; --q) off += totals[(size_t)q * rows + row];
  dlg[i] += off;
}

}  // namespace

size_t gla_seg_summary_floats(int BH, int F, int D) {
  return (size_t)BH * F * D + (size_t)BH * F + BH;
}

int gla_seg_fwd_begin(const bf16* fk, const bf16* v, const float* lg, int gph, float* summary,
                      const GlaFwdWork& fw, int B, int H, int L, int F, int D,
                      cudaStream_t stream) {
  const int BH = B * H, NT = (int)gla_nt(L);
  const int nfb = ceil_div(F, 64), ndb = ceil_div(D, 64);
  const int vec_f = (F % 8 == 0) && aligned16(fk);
  const int vec_d = (D % 8 == 0) && aligned16(v);
  gla_split_finc_kernel<<<(unsigned)((long long)BH * NT * nfb * ndb), 128, 0, stream>>>(
      fk, v, lg, gph, H, 1, L, F, D, NT, nfb, ndb, vec_f, vec_d, fw.inc, fw.incz, fw.lam);
  count_launches(1);
  int rc = check_launch("gla_split_finc_kernel");
  if (rc) return rc;
  const size_t nS = (size_t)BH * F * D, nZ = (size_t)BH * F;
  return launch_scan(fw.inc, fw.incz, fw.lam, BH, NT, F, D, 0, nullptr, nullptr, nullptr,
                     nullptr, summary, summary + nS, nullptr, summary + nS + nZ, stream);
}

int gla_seg_fwd_end(const bf16* fq, const bf16* fk, const bf16* v, const float* lg, int gph,
                    const float* seed, bf16* y, const GlaSaved& sv, const GlaFwdWork& fw, int B,
                    int H, int L, int F, int D, cudaStream_t stream) {
  const int BH = B * H, NT = (int)gla_nt(L);
  const bool save = sv.y32 != nullptr;
  bf16* s = save ? sv.s : fw.s;
  float* z = save ? sv.z : fw.z;
  const size_t nS = (size_t)BH * F * D;
  int rc = launch_scan(fw.inc, fw.incz, fw.lam, BH, NT, F, D, 0, seed, seed ? seed + nS : nullptr,
                       s, z, nullptr, nullptr, save ? fw.gs : nullptr, nullptr, stream);
  if (rc) return rc;
  const int FP = F <= 32 ? 32 : F <= 64 ? 64 : F <= 128 ? 128 : 256;
  const int DV = D <= 16 ? 16 : D <= 32 ? 32 : 64;
  float* y32 = save ? sv.y32 : nullptr;
  const int seeded = seed != nullptr;
#define LZ_OUT_CASE(fp, dv)                                                                   \
  if (FP == fp && DV == dv)                                                                   \
    return launch_out<fp, dv>(fq, fk, v, lg, gph, BH, H, 1, 1, L, F, D, NT, s, z, fw.gs,      \
                              seeded, y, y32, sv.den, save ? sv.g : nullptr, stream);
  LZ_OUT_CASE(32, 16) LZ_OUT_CASE(32, 32) LZ_OUT_CASE(32, 64)
  LZ_OUT_CASE(64, 16) LZ_OUT_CASE(64, 32) LZ_OUT_CASE(64, 64)
  LZ_OUT_CASE(128, 16) LZ_OUT_CASE(128, 32) LZ_OUT_CASE(128, 64)
  LZ_OUT_CASE(256, 16) LZ_OUT_CASE(256, 32) LZ_OUT_CASE(256, 64)
#undef LZ_OUT_CASE
  set_error("gla segment forward: no kernel for this feature/value size");
  return LZ_ERR_UNSUPPORTED;
}

int gla_seg_bwd_begin(const bf16* fq, const bf16* dy, const GlaSaved& sv, float* summary,
                      const GlaWork& wk, int B, int H, int L, int F, int D, cudaStream_t stream) {
  const int BH = B * H, NT = (int)gla_nt(L);
  const int nfb = ceil_div(F, 64), ndb = ceil_div(D, 64);
  const int vec_f = (F % 8 == 0) && aligned16(fq);
  const int vec_d = (D % 8 == 0) && aligned16(dy);
  const int vec_dots = (D % 4 == 0) && ((uintptr_t)dy & 7) == 0 && aligned16(sv.y32);
  gla_split_binc_kernel<<<(unsigned)((long long)BH * NT * nfb * ndb), 128, 0, stream>>>(
      fq, dy, sv.y32, sv.g, sv.den, L, F, D, NT, nfb, ndb, vec_f, vec_d, vec_dots, wk.delta,
      wk.inc, wk.incz, wk.lam);
  count_launches(1);
  int rc = check_launch("gla_split_binc_kernel");
  if (rc) return rc;
  const size_t nS = (size_t)BH * F * D, nZ = (size_t)BH * F;
  return launch_scan(wk.inc, wk.incz, wk.lam, BH, NT, F, D, 1, nullptr, nullptr, nullptr,
                     nullptr, summary, summary + nS, nullptr, summary + nS + nZ, stream);
}

int gla_seg_bwd_end(const bf16* fq, const bf16* fk, const bf16* v, int gph, const GlaSaved& sv,
                    const bf16* dy, const float* dseed, int s_seeded, void* dfq, void* dfk,
                    void* dv, int gdt, float* dlg, const GlaWork& wk, int B, int H, int L, int F,
                    int D, cudaStream_t stream) {
  const int BH = B * H, NT = (int)gla_nt(L);
  const size_t nS = (size_t)BH * F * D;
  int rc = launch_scan(wk.inc, wk.incz, wk.lam, BH, NT, F, D, 1, dseed,
                       dseed ? dseed + nS : nullptr, wk.ds, wk.dz, nullptr, nullptr, nullptr,
                       nullptr, stream);
  if (rc) return rc;
  return gla_bwd_tail(fq, fk, v, gph, sv, dy, dfq, dfk, dv, gdt, gdt, dlg, wk, B, H, H, L, F, D,
                      s_seeded, dseed != nullptr, stream);
}

int gla_seg_combine(const float* summaries, int P, int rank, int reverse, float* seed, int BH,
                    int F, int D, cudaStream_t stream) {
  const size_t n = (size_t)BH * F * D + (size_t)BH * F;
  gla_seg_combine_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(summaries, P, rank,
                                                                          reverse, BH, F, D, seed);
  count_launches(1);
  return check_launch("gla_seg_combine_kernel");
}

int gla_seg_gate_offset(float* dlg, const float* totals, int P, int rank, int rows, int L,
                        cudaStream_t stream) {
  const size_t n = (size_t)rows * L;
  gla_seg_gate_offset_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(dlg, totals, P,
                                                                              rank, rows, L);
  count_launches(1);
  return check_launch("gla_seg_gate_offset_kernel");
}

}  // namespace lz
