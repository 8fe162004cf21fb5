// GLA backward on the 5th-generation tensor cores, F = D = 128, 128-token
// chunks (the chunking of the tensor-core forward, which saved the bf16 state
// S_n and the normaliser z_n entering every chunk).
//
// Kernel 1, reverse state walk (one CTA per batch*head), the reference's
// _gla_bwd_dh (src/kernels/gla.py:104-132) with delta = dy . y32 (gla.py:242):
//   Q^_t = bf16(fq_t exp(G_t - G_start) / den_t)
//   dS_n = state gradient leaving chunk n;  dS <- e^{lam_n} dS + Q^_n^T dY_n
//   dz_n likewise with Q^_n^T delta_n (delta as bf16 hi + lo columns)
// The running dS lives in TMEM; the MMA is the forward's K~^T V pattern.
//
// Kernel 2, per-chunk gradients (one CTA per (chunk, batch*head)), the
// reference's _gla_bwd_dqkv (gla.py:135-194) plus dG (gla.py:254):
//   s = fq fk^T, p = dy v^T                              (TMEM)
//   a = bf16(s decay), dad = bf16((p - delta)/den decay), aden = bf16(a/den)
//   dv  = aden^T dy + ks (fk dS)
//   dfq = dad fk + qs/den (dy S^T - delta z)
//   dfk = dad^T fq + ks (v dS^T - dz)
//   dG_i = fq_i . dfq_i - fk_i . dfk_i, and the chunk's sum of dG
// with decay_it = exp(G_i - G_t) (t <= i), qs = exp(G_i - G_start),
// ks = exp(G_end - G_i). Eight 128 x 128 x 128 MMAs in three phases share the
// 512 TMEM columns; the chunk's tiles, S and then dS, and the bf16 dad / aden
// operands fill 224 KB of shared memory, and the output tiles are staged in
// buffers freed by the phase before them.
//
// Warp roles in both kernels: warp 0 TMA, warp 1 MMA (one thread), warps 2-5
// and 6-9 two groups of 128 threads, thread = TMEM lane = chunk row. Every
// wait is an mbarrier wait bounded at 2 s (tc.cuh). The row groups synchronise
// with bar.sync and never leave their code path early: a wait that gives up
// sets the device flag, every later wait returns at once, and the groups run
// on (writing in-bounds garbage) through every barrier to the end.
#include <atomic>
#include <mutex>
#include <string>

#include "common.cuh"
#include "gla_layout.h"
#include "tc.cuh"

namespace lz {

namespace {

constexpr int kC = 128;
constexpr int kTile = 32768;  // 128 x 128 bf16, two 64-column 128-byte-swizzled boxes
constexpr int kThreads = 320;

__device__ __forceinline__ uint32_t ko_kmajor(int j) { return (j >> 2) * 16384 + (j & 3) * 32; }

// byte offset of element (row, col) of a 128 x 128 bf16 tile in the box layout
__device__ __forceinline__ uint32_t tile_off(int row, int col) {
  return (col >> 6) * 16384 + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) + (col & 7) * 2;
}

// row `row` of a tile as 128 bf16 -> 16 uint4 (8 values each, in column order)
__device__ __forceinline__ void tile_row_load(const unsigned char* tile, int row, uint4 (&w)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i)
    w[i] = *reinterpret_cast<const uint4*>(tile + (i >> 3) * 16384 + row * 128 +
                                           (((i & 7) ^ (row & 7)) << 4));
}
__device__ __forceinline__ void tile_row_store(unsigned char* tile, int row, const uint4 (&w)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i)
    *reinterpret_cast<uint4*>(tile + (i >> 3) * 16384 + row * 128 + (((i & 7) ^ (row & 7)) << 4)) =
        w[i];
}
// 64 fp32 values -> bf16 into row `row`, columns [64 hb, 64 hb + 64)
__device__ __forceinline__ void tile_row_store64(unsigned char* tile, int row, int hb,
                                                 const float (&v)[64]) {
  unsigned char* p = tile + hb * 16384 + row * 128;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint4 w;
    w.x = pack_bf16(v[8 * c + 0], v[8 * c + 1]);
    w.y = pack_bf16(v[8 * c + 2], v[8 * c + 3]);
    w.z = pack_bf16(v[8 * c + 4], v[8 * c + 5]);
    w.w = pack_bf16(v[8 * c + 6], v[8 * c + 7]);
    *reinterpret_cast<uint4*>(p + ((c ^ (row & 7)) << 4)) = w;
  }
}

__device__ __forceinline__ uint4 scale8(uint4 w, float sc) {
  w.x = pack_bf16(bf16_lo(w.x) * sc, bf16_hi(w.x) * sc);
  w.y = pack_bf16(bf16_lo(w.y) * sc, bf16_hi(w.y) * sc);
  w.z = pack_bf16(bf16_lo(w.z) * sc, bf16_hi(w.z) * sc);
  w.w = pack_bf16(bf16_lo(w.w) * sc, bf16_hi(w.w) * sc);
  return w;
}

// sum over 64 columns of bf16(tile[row][64 hb + c]) * v[c]
__device__ __forceinline__ float row_dot64(const unsigned char* tile, int row, int hb,
                                           const float (&v)[64]) {
  const unsigned char* p = tile + hb * 16384 + row * 128;
  float acc = 0.f;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint4 w = *reinterpret_cast<const uint4*>(p + ((c ^ (row & 7)) << 4));
    acc += bf16_lo(w.x) * v[8 * c] + bf16_hi(w.x) * v[8 * c + 1] + bf16_lo(w.y) * v[8 * c + 2] +
           bf16_hi(w.y) * v[8 * c + 3] + bf16_lo(w.z) * v[8 * c + 4] +
           bf16_hi(w.z) * v[8 * c + 5] + bf16_lo(w.w) * v[8 * c + 6] + bf16_hi(w.w) * v[8 * c + 7];
  }
  return acc;
}

// ============================================================ kernel 1
constexpr int kS1Stage = 2 * kTile;         // fq, dy
constexpr int kS1OffStg = 2 * kS1Stage;     // dS staging tile
constexpr int kS1OffDel = kS1OffStg + kTile;  // 2 stages x delta operand block (4 KB)
constexpr int kS1OffMisc = kS1OffDel + 2 * 4096;
constexpr int kS1Smem = kS1OffMisc + 1024;
constexpr uint32_t kT1H = 0, kT1Z = 128, kT1Cols = 256;

enum { B1_FULL0 = 0, B1_FULL1, B1_EMPTY0, B1_EMPTY1, B1_QREADY, B1_HREADY, B1_HDONE, B1_COUNT };

__global__ void __launch_bounds__(kThreads, 1)
gla_bwd_state_tc_kernel(const __grid_constant__ CUtensorMap tq,
                        const __grid_constant__ CUtensorMap tdy,
                        const __grid_constant__ CUtensorMap tds, const float* __restrict__ G,
                        const float* __restrict__ den, const float* __restrict__ y32,
                        const bf16* __restrict__ dy, int L, int NT, float* __restrict__ delta,
                        float* __restrict__ dz_out) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  if (smem_u32(smem_raw) & 1023) {
    if (threadIdx.x == 0) atomicExch(&tc::g_timeout_flag, 0x80000000u | 98u);
    return;
  }
  unsigned char* base = smem_raw;
  unsigned char* misc = base + kS1OffMisc;
  uint64_t* bars = reinterpret_cast<uint64_t*>(misc);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + 256);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.x;
  const size_t rowb = (size_t)bh * L;

  if (tid == 0) {
    tc::mbar_init(&bars[B1_FULL0], 1);
    tc::mbar_init(&bars[B1_FULL1], 1);
    tc::mbar_init(&bars[B1_EMPTY0], 1);
    tc::mbar_init(&bars[B1_EMPTY1], 1);
    tc::mbar_init(&bars[B1_QREADY], 128);
    tc::mbar_init(&bars[B1_HREADY], 128);
    tc::mbar_init(&bars[B1_HDONE], 1);
    tc::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&tq);
    tc::prefetch_tmap(&tdy);
    tc::prefetch_tmap(&tds);
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, kT1Cols);
    tc::tmem_relinquish();
  }
  // delta operand blocks: rows 2..15 stay zero
  for (int i = tid; i < 2 * 4096 / 16; i += kThreads)
    reinterpret_cast<uint4*>(base + kS1OffDel)[i] = make_uint4(0u, 0u, 0u, 0u);
  tc::fence_proxy_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int issued[2] = {0, 0};
      for (int it = 0; it < NT; ++it) {
        const int n = NT - 1 - it, st = it & 1;
        if (it >= 2 && !tc::mbar_wait(&bars[B1_EMPTY0 + st], ((it - 2) >> 1) & 1, 21)) break;
        unsigned char* stage = base + st * kS1Stage;
        uint64_t* full = &bars[B1_FULL0 + st];
        tc::mbar_expect_tx(full, kS1Stage);
        tc::tma_load_3d(stage, &tq, 0, n * kC, bh, full);
        tc::tma_load_3d(stage + 16384, &tq, 64, n * kC, bh, full);
        tc::tma_load_3d(stage + kTile, &tdy, 0, n * kC, bh, full);
        tc::tma_load_3d(stage + kTile + 16384, &tdy, 64, n * kC, bh, full);
        ++issued[st];
      }
      for (int st = 0; st < 2; ++st)
        if (issued[st]) tc::mbar_wait(&bars[B1_FULL0 + st], (issued[st] - 1) & 1, 22);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_h = tc::idesc_bf16(128, 128, 1, 1);  // Q^ (MN) x dY (MN)
      constexpr uint32_t id_z = tc::idesc_bf16(128, 16, 1, 0);   // Q^ (MN) x delta (K)
      for (int it = 0; it < NT; ++it) {
        const int st = it & 1;
        if (!tc::mbar_wait(&bars[B1_QREADY], it & 1, 23)) break;
        if (!tc::mbar_wait(&bars[B1_HREADY], it & 1, 24)) break;
        tc::tc_fence_after();
        const uint32_t qa = smem_u32(base + st * kS1Stage), ya = qa + kTile;
        const uint32_t da = smem_u32(base + kS1OffDel + st * 4096);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          tc::mma_ss(tmem + kT1H, tc::sdesc(qa + 2048 * j, 16384, 1024),
                     tc::sdesc(ya + 2048 * j, 16384, 1024), id_h, (it > 0 || j > 0) ? 1u : 0u);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          tc::mma_ss(tmem + kT1Z, tc::sdesc(qa + 2048 * j, 16384, 1024),
                     tc::sdesc(da + (j >> 2) * 2048 + (j & 3) * 32, 16, 1024), id_z,
                     (it > 0 || j > 0) ? 1u : 0u);
        tc::mma_commit(&bars[B1_HDONE]);
        tc::mma_commit(&bars[B1_EMPTY0 + st]);
        if (it == NT - 1) tc::mbar_wait(&bars[B1_HDONE], it & 1, 29);  // none in flight at exit
      }
    }
  } else if (warp < 6) {
    // ------------------ prep: Q^ in place, delta (global and operand block)
    const int quad = warp & 3, t = quad * 32 + lane;
    for (int it = 0; it < NT; ++it) {
      const int n = NT - 1 - it, st = it & 1, r0 = n * kC;
      const bool valid = r0 + t < L;
      const float start = n > 0 ? G[rowb + r0 - 1] : 0.f;
      float qs = 0.f;
      if (valid) qs = __expf(G[rowb + r0 + t] - start) / fmaxf(den[rowb + r0 + t], kTiny);
      if (warp == 2 && lane == 0 && n > 0)  // the next chunk's fp32 y rows into L2 (64 KB)
        tc::bulk_prefetch_l2(y32 + (rowb + r0 - kC) * 128, (uint32_t)kC * 128 * 4);
      tc::mbar_wait(&bars[B1_FULL0 + st], (it >> 1) & 1, 25);
      unsigned char* stage = base + st * kS1Stage;
      // delta_t = dy_t . y32_t
      float dl = 0.f;
      if (valid) {
        const float4* yr = reinterpret_cast<const float4*>(y32 + (rowb + r0 + t) * 128);
        uint4 w[16];
        tile_row_load(stage + kTile, t, w);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float4 a = yr[2 * i], b = yr[2 * i + 1];
          dl += bf16_lo(w[i].x) * a.x + bf16_hi(w[i].x) * a.y + bf16_lo(w[i].y) * a.z +
                bf16_hi(w[i].y) * a.w + bf16_lo(w[i].z) * b.x + bf16_hi(w[i].z) * b.y +
                bf16_lo(w[i].w) * b.z + bf16_hi(w[i].w) * b.w;
        }
        delta[rowb + r0 + t] = dl;
      }
      {
        const bf16 hi = __float2bfloat16_rn(dl);
        const bf16 lo = __float2bfloat16_rn(dl - __bfloat162float(hi));
        unsigned char* blk = base + kS1OffDel + st * 4096 + (t >> 6) * 2048;
        const int c = t & 63;
        *reinterpret_cast<bf16*>(blk + 0 * 128 + ((((c >> 3) ^ 0) << 4)) + (c & 7) * 2) = hi;
        *reinterpret_cast<bf16*>(blk + 1 * 128 + ((((c >> 3) ^ 1) << 4)) + (c & 7) * 2) = lo;
      }
      {
        uint4 w[16];
        tile_row_load(stage, t, w);
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = scale8(w[i], qs);
        tile_row_store(stage, t, w);
      }
      tc::fence_proxy_async_smem();
      // Every prep thread arrives for this chunk before any arrives for the
      // next: the next chunk's tiles are often loaded already, and one warp's
      // arrival for it would otherwise complete this chunk's phase while
      // another warp's rows of Q^ and delta were still being written.
      tc::named_bar_sync(2, 128);
      tc::mbar_arrive(&bars[B1_QREADY]);
    }
  } else {
    // ------------------ state gradient out, then pre-scale by the chunk decay
    const int quad = warp & 3, f = quad * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
    unsigned char* stg = base + kS1OffStg;
    for (int it = 0; it < NT; ++it) {
      const int n = NT - 1 - it, r0 = n * kC;
      const size_t chunk = (size_t)bh * NT + n;
      const int last = min(r0 + kC, L) - 1;
      const float lam = G[rowb + last] - (n > 0 ? G[rowb + r0 - 1] : 0.f);
      if (f == 0) tc::bulk_wait_read0();  // the previous store has read the staging tile
      tc::named_bar_sync(1, 128);
      if (it == 0) {
        uint4 z[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) z[i] = make_uint4(0u, 0u, 0u, 0u);
        tile_row_store(stg, f, z);
        dz_out[chunk * 128 + f] = 0.f;
      } else {
        tc::mbar_wait(&bars[B1_HDONE], (it - 1) & 1, 27);
        tc::tc_fence_after();
        const float e = __expf(lam);
        float zz[32];
        tc::tmem_ld32(trow + kT1Z, zz);
        tc::tmem_wait_ld();
        dz_out[chunk * 128 + f] = zz[0] + zz[1];
        tc::tmem_st1(trow + kT1Z, __float_as_uint(zz[0] * e));
        tc::tmem_st1(trow + kT1Z + 1, __float_as_uint(zz[1] * e));
#pragma unroll 1
        for (int hb = 0; hb < 2; ++hb) {
          float hv[64];
          tc::tmem_ld64(trow + kT1H + 64 * hb, hv);
          tc::tmem_wait_ld();
          tile_row_store64(stg, f, hb, hv);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t sc[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) sc[j] = __float_as_uint(hv[16 * q + j] * e);
            tc::tmem_st16(trow + kT1H + 64 * hb + 16 * q, sc);
          }
        }
      }
      tc::fence_proxy_async_smem();
      tc::tmem_wait_st();
      tc::tc_fence_before();
      tc::named_bar_sync(1, 128);
      if (f == 0) {
        tc::tma_store_3d(&tds, stg, 0, n * kC, bh);
        tc::tma_store_3d(&tds, stg + 16384, 64, n * kC, bh);
        tc::bulk_commit();
      }
      tc::mbar_arrive(&bars[B1_HREADY]);
    }
    if (f == 0) tc::bulk_wait0();
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kT1Cols);
  }
}

// ============================================================ kernel 2
constexpr int kOQ = 0, kOK = kTile, kOV = 2 * kTile, kODY = 3 * kTile, kOX = 4 * kTile,
              kODAD = 5 * kTile, kOADEN = 6 * kTile, kOMisc = 7 * kTile;
constexpr int kMiscBytes2 = 3072;
constexpr int kSmem2 = kOMisc + kMiscBytes2;  // 232448
// misc: bars [0, 128), tmem slot 128, dGt partials 192 (4 floats), sG2 256, sZ 768,
// sDZ 1280, sDGa 1792
constexpr int kMB = 0, kMTmem = 128, kMRed = 192, kMG = 256, kMZ = 768, kMDZ = 1280, kMDGa = 1792;
constexpr uint32_t kTS = 0, kTP = 128, kTDV = 256, kT5 = 384, kT2Cols = 512;

enum { B2_FULL = 0, B2_SPFULL, B2_EWDONE, B2_P3DONE, B2_T12FREE, B2_DSFULL, B2_P4DONE, B2_DGA,
       B2_COUNT };

// NARROW: F = D = 64 on the chunk-parallel schedule's 64-token states. The
// 64-column tiles are read as the first box of a 128-wide tile whose second box
// TMA fills with zeros (coordinates past the tensor's width), and the state and
// its gradient as 64 x 64 boxes into the first box of a tile whose other rows
// and columns the row threads zero: every product then runs on zero-padded
// 128-wide operands, the padded features and values add nothing, and only the
// first 64 columns of each gradient are written. The state entering 128-token
// chunk n is the scan's state 2n, the gradient leaving it the scan's gradient
// 2n + 1 (the last one for an odd tail), and the K-loops over F or D stop at 64.
template <bool NARROW>
__global__ void __launch_bounds__(kThreads, 1)
gla_bwd_chunk_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv,
                        const __grid_constant__ CUtensorMap tdy,
                        const __grid_constant__ CUtensorMap ts,
                        const __grid_constant__ CUtensorMap tds,
                        const __grid_constant__ CUtensorMap tdfq,
                        const __grid_constant__ CUtensorMap tdfk,
                        const __grid_constant__ CUtensorMap tdv, const float* __restrict__ G,
                        const float* __restrict__ den, const float* __restrict__ delta,
                        const float* __restrict__ Z, const float* __restrict__ dZ, int H, int grp,
                        int L, int NT, int gdt, int gdt_kv, void* __restrict__ dfq,
                        void* __restrict__ dfk,
                        void* __restrict__ dv, float* __restrict__ dG, float* __restrict__ dGt,
                        int s_seeded, int ds_seeded, int pf_ahead) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  if (smem_u32(smem_raw) & 1023) {
    if (threadIdx.x == 0) atomicExch(&tc::g_timeout_flag, 0x80000000u | 97u);
    return;
  }
  unsigned char* base = smem_raw;
  unsigned char* misc = base + kOMisc;
  uint64_t* bars = reinterpret_cast<uint64_t*>(misc + kMB);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + kMTmem);
  float* sRed = reinterpret_cast<float*>(misc + kMRed);
  float* sG2 = reinterpret_cast<float*>(misc + kMG);
  float* sZ = reinterpret_cast<float*>(misc + kMZ);
  float* sDZ = reinterpret_cast<float*>(misc + kMDZ);
  float* sDGa = reinterpret_cast<float*>(misc + kMDGa);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n = blockIdx.x % NT, bh = blockIdx.x / NT;
  const int kvh = kv_head(bh, H, grp);  // head of fk and v (GQA)
  const int r0 = n * kC, nvalid = min(kC, L - r0);
  const size_t rowb = (size_t)bh * L, chunk = (size_t)bh * NT + n;
  constexpr int kW = NARROW ? 64 : 128;   // columns of fq, fk, v, dy and the gradients
  constexpr int kKs = NARROW ? 4 : 8;     // 16-wide K-steps over F or D
  constexpr int kHB = NARROW ? 1 : 2;     // 64-column blocks holding data
  // rows of the 64-token scan states (NARROW): entering = 2n, leaving = 2n + 1
  const int NTs = (L + 63) / 64;
  const int s_row = NARROW ? 2 * n * 64 : r0;
  const int ds_row = NARROW ? min(2 * n + 1, NTs - 1) * 64 : r0;
  const size_t zchunk = NARROW ? (size_t)bh * NTs + 2 * n : chunk;
  const size_t dzchunk = NARROW ? (size_t)bh * NTs + min(2 * n + 1, NTs - 1) : chunk;
  const bool with_s = n > 0 || s_seeded;
  const bool with_ds = n + 1 < NT || ds_seeded;
  const bool bf16_out = gdt == LZ_DTYPE_BF16;    // dfq
  const bool bf16_kv = gdt_kv == LZ_DTYPE_BF16;  // dfk, dv (per query head)

  if (tid == 0) {
    tc::mbar_init(&bars[B2_FULL], 1);
    tc::mbar_init(&bars[B2_SPFULL], 1);
    tc::mbar_init(&bars[B2_EWDONE], 256);
    tc::mbar_init(&bars[B2_P3DONE], 1);
    tc::mbar_init(&bars[B2_T12FREE], 128);
    tc::mbar_init(&bars[B2_DSFULL], 1);
    tc::mbar_init(&bars[B2_P4DONE], 1);
    tc::mbar_init(&bars[B2_DGA], 128);
    tc::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&tq);
    tc::prefetch_tmap(&tk);
    tc::prefetch_tmap(&tv);
    tc::prefetch_tmap(&tdy);
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, kT2Cols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      uint64_t* full = &bars[B2_FULL];
      tc::mbar_expect_tx(full, 4 * kTile + (with_s ? (NARROW ? 8192 : kTile) : 0));
      tc::tma_load_3d(base + kOQ, &tq, 0, r0, bh, full);
      tc::tma_load_3d(base + kOQ + 16384, &tq, 64, r0, bh, full);
      tc::tma_load_3d(base + kOK, &tk, 0, r0, kvh, full);
      tc::tma_load_3d(base + kOK + 16384, &tk, 64, r0, kvh, full);
      tc::tma_load_3d(base + kOV, &tv, 0, r0, kvh, full);
      tc::tma_load_3d(base + kOV + 16384, &tv, 64, r0, kvh, full);
      tc::tma_load_3d(base + kODY, &tdy, 0, r0, bh, full);
      tc::tma_load_3d(base + kODY + 16384, &tdy, 64, r0, bh, full);
      if (with_s) {
        tc::tma_load_3d(base + kOX, &ts, 0, s_row, bh, full);
        if (!NARROW) tc::tma_load_3d(base + kOX + 16384, &ts, 64, r0, bh, full);
      }
      // One CTA per SM: the CTA that starts on an SM when this one ends is about
      // pf_ahead blocks further on. Its tiles and row scalars go to L2 now, so
      // their HBM reads overlap this CTA's MMA phases instead of following them.
      if (pf_ahead > 0 && blockIdx.x + pf_ahead < gridDim.x) {
        const int nb = blockIdx.x + pf_ahead;
        const int pn = nb % NT, pbh = nb / NT, pkvh = kv_head(pbh, H, grp), pr0 = pn * kC;
#pragma unroll
        for (int hb = 0; hb < kHB; ++hb) {
          tc::tma_prefetch_l2_3d(&tq, 64 * hb, pr0, pbh);
          tc::tma_prefetch_l2_3d(&tk, 64 * hb, pr0, pkvh);
          tc::tma_prefetch_l2_3d(&tv, 64 * hb, pr0, pkvh);
          tc::tma_prefetch_l2_3d(&tdy, 64 * hb, pr0, pbh);
        }
        const int ps_row = NARROW ? 2 * pn * 64 : pr0;
        const int pds_row = NARROW ? min(2 * pn + 1, NTs - 1) * 64 : pr0;
        if (pn > 0 || s_seeded)
          for (int hb = 0; hb < kHB; ++hb) tc::tma_prefetch_l2_3d(&ts, 64 * hb, ps_row, pbh);
        if (pn + 1 < NT || ds_seeded)
          for (int hb = 0; hb < kHB; ++hb) tc::tma_prefetch_l2_3d(&tds, 64 * hb, pds_row, pbh);
        // G, den and delta rows of the chunk: whole 16-byte groups inside it
        const size_t prow = (size_t)pbh * L + pr0;
        const uint32_t pbytes = (uint32_t)(min(kC, L - pr0) / 4) * 16;
        if ((prow & 3) == 0 && pbytes > 0) {
          tc::bulk_prefetch_l2(G + prow, pbytes);
          tc::bulk_prefetch_l2(den + prow, pbytes);
          tc::bulk_prefetch_l2(delta + prow, pbytes);
        }
      }
      bool ok = tc::mbar_wait(full, 0, 31);
      if (with_ds && ok) {
        // dS replaces S once the phase-3 MMAs (the last readers of S) are done
        ok = tc::mbar_wait(&bars[B2_P3DONE], 0, 32);
        if (ok) {
          uint64_t* dsf = &bars[B2_DSFULL];
          tc::mbar_expect_tx(dsf, NARROW ? 8192 : kTile);
          tc::tma_load_3d(base + kOX, &tds, 0, ds_row, bh, dsf);
          if (!NARROW) tc::tma_load_3d(base + kOX + 16384, &tds, 64, r0, bh, dsf);
          tc::mbar_wait(dsf, 0, 33);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t id_kk = tc::idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t id_km = tc::idesc_bf16(128, 128, 0, 1);
      constexpr uint32_t id_mm = tc::idesc_bf16(128, 128, 1, 1);
      const uint32_t q = smem_u32(base + kOQ), k = smem_u32(base + kOK),
                     v = smem_u32(base + kOV), y = smem_u32(base + kODY),
                     x = smem_u32(base + kOX), dad = smem_u32(base + kODAD),
                     aden = smem_u32(base + kOADEN);
      bool ok = tc::mbar_wait(&bars[B2_FULL], 0, 34);
      if (ok) {
        tc::tc_fence_after();
        // phase 1: s = fq fk^T, p = dy v^T (K = F, D)
#pragma unroll
        for (int j = 0; j < kKs; ++j)
          tc::mma_ss(tmem + kTS, tc::sdesc(q + ko_kmajor(j), 16, 1024),
                     tc::sdesc(k + ko_kmajor(j), 16, 1024), id_kk, j > 0);
#pragma unroll
        for (int j = 0; j < kKs; ++j)
          tc::mma_ss(tmem + kTP, tc::sdesc(y + ko_kmajor(j), 16, 1024),
                     tc::sdesc(v + ko_kmajor(j), 16, 1024), id_kk, j > 0);
        tc::mma_commit(&bars[B2_SPFULL]);
        ok = tc::mbar_wait(&bars[B2_EWDONE], 0, 35);
      }
      if (ok) {
        tc::tc_fence_after();
        // phase 3: dv_intra = aden^T dy, T1 = dad fk, T2 = dy S^T
#pragma unroll
        for (int j = 0; j < 8; ++j)
          tc::mma_ss(tmem + kTDV, tc::sdesc(aden + 2048 * j, 16384, 1024),
                     tc::sdesc(y + 2048 * j, 16384, 1024), id_mm, j > 0);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          tc::mma_ss(tmem + kTS, tc::sdesc(dad + ko_kmajor(j), 16, 1024),
                     tc::sdesc(k + 2048 * j, 16384, 1024), id_km, j > 0);
        if (with_s) {  // K = D
#pragma unroll
          for (int j = 0; j < kKs; ++j)
            tc::mma_ss(tmem + kTP, tc::sdesc(y + ko_kmajor(j), 16, 1024),
                       tc::sdesc(x + ko_kmajor(j), 16, 1024), id_kk, j > 0);
        }
        tc::mma_commit(&bars[B2_P3DONE]);
        ok = tc::mbar_wait(&bars[B2_T12FREE], 0, 36);
        if (ok && with_ds) ok = tc::mbar_wait(&bars[B2_DSFULL], 0, 37);
      }
      if (ok) {
        tc::tc_fence_after();
        // phase 4: T3 = dad^T fq, T4 = v dS^T, T5 = fk dS
#pragma unroll
        for (int j = 0; j < 8; ++j)
          tc::mma_ss(tmem + kTS, tc::sdesc(dad + 2048 * j, 16384, 1024),
                     tc::sdesc(q + 2048 * j, 16384, 1024), id_mm, j > 0);
        if (with_ds) {  // K = D, then K = F
#pragma unroll
          for (int j = 0; j < kKs; ++j)
            tc::mma_ss(tmem + kTP, tc::sdesc(v + ko_kmajor(j), 16, 1024),
                       tc::sdesc(x + ko_kmajor(j), 16, 1024), id_kk, j > 0);
#pragma unroll
          for (int j = 0; j < kKs; ++j)
            tc::mma_ss(tmem + kT5, tc::sdesc(k + ko_kmajor(j), 16, 1024),
                       tc::sdesc(x + 2048 * j, 16384, 1024), id_km, j > 0);
        }
        tc::mma_commit(&bars[B2_P4DONE]);
        tc::mbar_wait(&bars[B2_P4DONE], 0, 38);  // no MMA in flight at exit
      }
    }
  } else {
    // -------------------------------------------- row threads (two groups)
    const bool grpA = warp < 6;
    const int quad = warp & 3, i = quad * 32 + lane;  // chunk row == TMEM lane
    const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
    const bool valid = i < nvalid;
    const float start = n > 0 ? G[rowb + r0 - 1] : 0.f;
    const float gi = valid ? G[rowb + r0 + i] - start : 0.f;
    const float g2i = gi * kLog2e;
    const float rden = valid ? 1.f / fmaxf(den[rowb + r0 + i], kTiny) : 0.f;
    const float dl = valid ? delta[rowb + r0 + i] : 0.f;
    if (grpA) {
      sG2[i] = g2i;
      sZ[i] = (with_s && i < kW) ? Z[zchunk * kW + i] : 0.f;
      sDZ[i] = (with_ds && i < kW) ? dZ[dzchunk * kW + i] : 0.f;
    }
    if constexpr (NARROW) {
      // the state / gradient tile holds a 64 x 64 box: zero its other rows
      // (bytes [8192, 16384)) and its second box (bytes [16384, 32768))
      const int e = (grpA ? 0 : 128) + i;  // 0..255
      uint4* zt = reinterpret_cast<uint4*>(base + kOX + 8192);
#pragma unroll
      for (int u = 0; u < 6; ++u) zt[e + 256 * u] = make_uint4(0u, 0u, 0u, 0u);
    }
    tc::named_bar_sync(1, 256);
    const float g2end = sG2[nvalid - 1];
    // --- phase 2: dad, aden for columns [64 h, 64 h + 64)
    tc::mbar_wait(&bars[B2_SPFULL], 0, 41);
    tc::tc_fence_after();
    {
      const int h = grpA ? 0 : 1;
#pragma unroll 1
      for (int cb = 0; cb < 2; ++cb) {
        const int c0 = 64 * h + 32 * cb;
        float sv[32], pv[32];
        tc::tmem_ld32(trow + kTS + c0, sv);
        tc::tmem_ld32(trow + kTP + c0, pv);
        tc::tmem_wait_ld();
        uint32_t dadp[16], adenp[16];
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          float dd[2], aa[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int t = c0 + c + e;
            const bool m = valid && t <= i;
            const float dec = m ? tc::ex2(g2i - sG2[t]) : 0.f;
            const float a = round_bf16(sv[c + e] * dec);
            dd[e] = m ? (pv[c + e] - dl) * rden * dec : 0.f;
            aa[e] = a * rden;
          }
          dadp[c >> 1] = pack_bf16(dd[0], dd[1]);
          adenp[c >> 1] = pack_bf16(aa[0], aa[1]);
        }
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          const uint32_t off = tile_off(i, c0 + 8 * c8);
          *reinterpret_cast<uint4*>(base + kODAD + off) =
              make_uint4(dadp[4 * c8], dadp[4 * c8 + 1], dadp[4 * c8 + 2], dadp[4 * c8 + 3]);
          *reinterpret_cast<uint4*>(base + kOADEN + off) =
              make_uint4(adenp[4 * c8], adenp[4 * c8 + 1], adenp[4 * c8 + 2], adenp[4 * c8 + 3]);
        }
      }
    }
    tc::fence_proxy_async_smem();
    tc::tc_fence_before();
    tc::mbar_arrive(&bars[B2_EWDONE]);
    const float qsd = valid ? tc::ex2(g2i) * rden : 0.f;  // exp(G_i - start) / den_i
    const float ks = valid ? tc::ex2(g2end - g2i) : 0.f;  // exp(G_end - G_i)
    if (grpA) {
      // --- dfq = T1 + qs/den (T2 - delta z); staged in the freed aden tile
      float dgq = 0.f;
      tc::mbar_wait(&bars[B2_P3DONE], 0, 42);
      tc::tc_fence_after();
#pragma unroll 1
      for (int hb = 0; hb < kHB; ++hb) {
        float t1[64], t2[64];
        tc::tmem_ld64(trow + kTS + 64 * hb, t1);
        if (with_s) tc::tmem_ld64(trow + kTP + 64 * hb, t2);
        tc::tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const float t2v = with_s ? t2[c] : 0.f;
          t1[c] = t1[c] + qsd * (t2v - dl * sZ[64 * hb + c]);
        }
        dgq += row_dot64(base + kOQ, i, hb, t1);
        if (bf16_out) {
          tile_row_store64(base + kOADEN, i, hb, t1);
        } else if (valid) {
          float4* o = reinterpret_cast<float4*>(static_cast<float*>(dfq) + (rowb + r0 + i) * kW +
                                                64 * hb);
#pragma unroll
          for (int c = 0; c < 16; ++c)
            o[c] = make_float4(t1[4 * c], t1[4 * c + 1], t1[4 * c + 2], t1[4 * c + 3]);
        }
      }
      tc::tc_fence_before();
      tc::mbar_arrive(&bars[B2_T12FREE]);
      sDGa[i] = dgq;
      tc::mbar_arrive(&bars[B2_DGA]);
      if (bf16_out) {
        tc::fence_proxy_async_smem();
        tc::named_bar_sync(2, 128);
        if (i == 0) {
          tc::tma_store_3d(&tdfq, base + kOADEN, 0, r0, bh);
          if (!NARROW) tc::tma_store_3d(&tdfq, base + kOADEN + 16384, 64, r0, bh);
          tc::bulk_commit();
        }
      }
      // --- dv = dv_intra + ks T5; staged in the freed S / dS tile
      tc::mbar_wait(&bars[B2_P4DONE], 0, 44);
      tc::tc_fence_after();
#pragma unroll 1
      for (int hb = 0; hb < kHB; ++hb) {
        float dvv[64], t5[64];
        tc::tmem_ld64(trow + kTDV + 64 * hb, dvv);
        if (with_ds) tc::tmem_ld64(trow + kT5 + 64 * hb, t5);
        tc::tmem_wait_ld();
        if (with_ds) {
#pragma unroll
          for (int c = 0; c < 64; ++c) dvv[c] += ks * t5[c];
        }
        if (bf16_kv) {
          tile_row_store64(base + kOX, i, hb, dvv);
        } else if (valid) {
          float4* o = reinterpret_cast<float4*>(static_cast<float*>(dv) + (rowb + r0 + i) * kW +
                                                64 * hb);
#pragma unroll
          for (int c = 0; c < 16; ++c)
            o[c] = make_float4(dvv[4 * c], dvv[4 * c + 1], dvv[4 * c + 2], dvv[4 * c + 3]);
        }
      }
      if (bf16_kv) {
        tc::fence_proxy_async_smem();
        tc::named_bar_sync(2, 128);
        if (i == 0) {
          tc::tma_store_3d(&tdv, base + kOX, 0, r0, bh);
          if (!NARROW) tc::tma_store_3d(&tdv, base + kOX + 16384, 64, r0, bh);
          tc::bulk_commit();
        }
      }
      if (i == 0) tc::bulk_wait0();
    } else {
      // --- dfk = T3 + ks (T4 - dz); staged in the freed dad tile; dG
      float dgk = 0.f;
      tc::mbar_wait(&bars[B2_P4DONE], 0, 46);
      tc::tc_fence_after();
#pragma unroll 1
      for (int hb = 0; hb < kHB; ++hb) {
        float t3[64], t4[64];
        tc::tmem_ld64(trow + kTS + 64 * hb, t3);
        if (with_ds) tc::tmem_ld64(trow + kTP + 64 * hb, t4);
        tc::tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const float t4v = with_ds ? t4[c] : 0.f;
          t3[c] = t3[c] + ks * (t4v - sDZ[64 * hb + c]);
        }
        dgk += row_dot64(base + kOK, i, hb, t3);
        if (bf16_kv) {
          tile_row_store64(base + kODAD, i, hb, t3);
        } else if (valid) {
          float4* o = reinterpret_cast<float4*>(static_cast<float*>(dfk) + (rowb + r0 + i) * kW +
                                                64 * hb);
#pragma unroll
          for (int c = 0; c < 16; ++c)
            o[c] = make_float4(t3[4 * c], t3[4 * c + 1], t3[4 * c + 2], t3[4 * c + 3]);
        }
      }
      if (bf16_kv) {
        tc::fence_proxy_async_smem();
        tc::named_bar_sync(3, 128);
        if (i == 0) {
          tc::tma_store_3d(&tdfk, base + kODAD, 0, r0, bh);
          if (!NARROW) tc::tma_store_3d(&tdfk, base + kODAD + 16384, 64, r0, bh);
          tc::bulk_commit();
        }
      }
      tc::mbar_wait(&bars[B2_DGA], 0, 48);
      float x = 0.f;
      if (valid) {
        x = sDGa[i] - dgk;
        dG[rowb + r0 + i] = x;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
      if (lane == 0) sRed[quad] = x;
      tc::named_bar_sync(3, 128);
      if (i == 0) {
        dGt[chunk] = sRed[0] + sRed[1] + sRed[2] + sRed[3];
        tc::bulk_wait0();
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kT2Cols);
  }
}

// ------------------------------------------------------------ host helpers

// [BH, rows, cols] bf16 as 3-D {cols, rows, BH}, box {64, box_rows, 1}, 128-byte
// swizzle, zero fill outside (cols 64: a box at column 64 reads zeros)
// The last encode failure of this thread (for the error message).
thread_local int g_map_err = 0;

bool make_map(CUtensorMap* m, const void* ptr, int BH, int rows, int cols = 128,
              int box_rows = 128) {
  tc::EncodeTiledFn fn = tc::encode_tiled_fn();
  g_map_err = -1;
  if (!fn) return false;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)BH};
  cuuint64_t strides[2] = {(cuuint64_t)cols * 2, (cuuint64_t)rows * cols * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r =
      fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  g_map_err = (int)r;
  return r == CUDA_SUCCESS;
}

// "gla_bwd: tensor map encoding failed" with which map and the driver's code.
void map_error(const char* which) {
  set_error(std::string("gla_bwd: tensor map encoding failed (") + which + ", CUresult " +
            std::to_string(g_map_err) + ")");
}

std::mutex g_tc_mu;
// L2 prefetch of the next CTA's operands in the per-chunk gradient kernel (on by
// default; lz_gla_set_bwd_prefetch(0) turns it off to measure it)
std::atomic<int> g_chunk_prefetch{1};

int sm_count() {
  static int n[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && n[dev] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    n[dev] = v > 0 ? v : 148;
  }
  return dev < 64 ? n[dev] : 148;
}

int ensure_attr(const void* fn, int bytes, bool* done) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(g_tc_mu);
  if (dev < 64 && !done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) {
      set_error(std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
      return LZ_ERR_CUDA;
    }
    done[dev] = true;
  }
  return LZ_OK;
}

}  // namespace

// State gradients (dS_n, dz_n) and delta for the 128-token chunk layout.
int gla_bwd_tc_states(const bf16* fq, const bf16* dy, const GlaSaved& sv, const GlaWork& wk,
                      int B, int H, int L, cudaStream_t stream) {
  const int BH = B * H, NT = (L + kC - 1) / kC;
  CUtensorMap mq, mdy, mds;
  if (!make_map(&mq, fq, BH, L)) return map_error("fq"), LZ_ERR_CUDA;
  if (!make_map(&mdy, dy, BH, L)) return map_error("dy"), LZ_ERR_CUDA;
  if (!make_map(&mds, wk.ds, BH, NT * kC)) return map_error("state gradients"), LZ_ERR_CUDA;
  static bool done[64] = {false};
  int rc = ensure_attr(reinterpret_cast<const void*>(gla_bwd_state_tc_kernel), kS1Smem, done);
  if (rc) return rc;
  gla_bwd_state_tc_kernel<<<BH, kThreads, kS1Smem, stream>>>(mq, mdy, mds, sv.g, sv.den, sv.y32,
                                                          dy, L, NT, wk.delta, wk.dz);
  count_launches(1);
  return check_launch("gla_bwd_state_tc_kernel");
}

int gla_bwd_tc_chunks(const bf16* fq, const bf16* fk, const bf16* v, const bf16* dy,
                      const GlaSaved& sv, const GlaWork& wk, void* dfq, void* dfk, void* dv,
                      int gdt, int gdt_kv, int B, int H, int Hkv, int L, int s_seeded,
                      int ds_seeded, cudaStream_t stream, bool narrow) {
  const int BH = B * H, NT = (L + kC - 1) / kC;
  // narrow (F = D = 64): 64-column tensors, and the 64-token scan's states and
  // state gradients [BH, NT64, 64, 64] read as 64 x 64 boxes
  const int W = narrow ? 64 : 128;
  const int srows = narrow ? ((L + 63) / 64) * 64 : NT * kC;
  const int sbox = narrow ? 64 : 128;
  CUtensorMap mq, mk, mv, mdy, ms, mds, mdfq, mdfk, mdv;
  if (!make_map(&mq, fq, BH, L, W)) return map_error("fq"), LZ_ERR_CUDA;
  if (!make_map(&mk, fk, B * Hkv, L, W)) return map_error("fk"), LZ_ERR_CUDA;
  if (!make_map(&mv, v, B * Hkv, L, W)) return map_error("v"), LZ_ERR_CUDA;
  if (!make_map(&mdy, dy, BH, L, W)) return map_error("dy"), LZ_ERR_CUDA;
  if (!make_map(&ms, sv.s, BH, srows, W, sbox)) return map_error("saved states"), LZ_ERR_CUDA;
  if (!make_map(&mds, wk.ds, BH, srows, W, sbox)) return map_error("state gradients"), LZ_ERR_CUDA;
  // fp32 gradients are stored directly; their maps are unused
  mdfq = mdfk = mdv = mq;
  if (gdt == LZ_DTYPE_BF16 && !make_map(&mdfq, dfq, BH, L, W))
    return map_error("dfq"), LZ_ERR_CUDA;
  if (gdt_kv == LZ_DTYPE_BF16 &&
      (!make_map(&mdfk, dfk, BH, L, W) || !make_map(&mdv, dv, BH, L, W)))
    return map_error("dfk / dv"), LZ_ERR_CUDA;
  const unsigned grid = (unsigned)((long long)BH * NT);
  const int pf = g_chunk_prefetch.load() ? sm_count() : 0;
  if (narrow) {
    static bool done[64] = {false};
    int rc = ensure_attr(reinterpret_cast<const void*>(gla_bwd_chunk_tc_kernel<true>), kSmem2,
                         done);
    if (rc) return rc;
    gla_bwd_chunk_tc_kernel<true><<<grid, kThreads, kSmem2, stream>>>(
        mq, mk, mv, mdy, ms, mds, mdfq, mdfk, mdv, sv.g, sv.den, wk.delta, sv.z, wk.dz, H,
        H / Hkv, L, NT, gdt, gdt_kv, dfq, dfk, dv, wk.dg, wk.dgt, s_seeded, ds_seeded, pf);
  } else {
    static bool done[64] = {false};
    int rc = ensure_attr(reinterpret_cast<const void*>(gla_bwd_chunk_tc_kernel<false>), kSmem2,
                         done);
    if (rc) return rc;
    gla_bwd_chunk_tc_kernel<false><<<grid, kThreads, kSmem2, stream>>>(
        mq, mk, mv, mdy, ms, mds, mdfq, mdfk, mdv, sv.g, sv.den, wk.delta, sv.z, wk.dz, H,
        H / Hkv, L, NT, gdt, gdt_kv, dfq, dfk, dv, wk.dg, wk.dgt, s_seeded, ds_seeded, pf);
  }
  count_launches(1);
  return check_launch("gla_bwd_chunk_tc_kernel");
}

int gla_set_bwd_prefetch(int on) { return g_chunk_prefetch.exchange(on ? 1 : 0); }

int gla_bwd_tc_timeout_flag(unsigned int* out) { return tc::read_timeout_flag_here(out); }
int gla_bwd_tc_timeout_clear() { return tc::clear_timeout_flag_here(); }

}  // namespace lz
