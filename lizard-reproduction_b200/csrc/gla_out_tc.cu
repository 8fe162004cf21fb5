// Chunk outputs of the chunk-parallel GLA schedule on the 5th-generation
// tensor cores (tcgen05 + TMEM + TMA), for F in {128, 256} with D = 64,
// F = D = 128 and F = D = 64 (config 3's shape). In training it also writes
// what the backward reads: y in fp32, the row sums and the running log gate G.
//
// After the increments and the scan (gla_split.cu) every chunk's entering state
// S_n (bf16) and normaliser z_n (fp32) are in HBM, so the chunks are
// independent: one CTA of 4 warps takes one 128-token chunk (two 64-token scan
// chunks; the state entering it is the scan's state 2c) and
//   TMA      : fq, fk, v tiles and the bf16 state [F x D] (128-byte swizzle)
//   thread 0 : s = fq fk^T                               -> TMEM [128 x 128]
//   4 warps  : a = bf16(s 2^(g_i - g_t)), t <= i          -> TMEM (A operand),
//              row i per thread (TMEM lane i): the in-chunk gate scan,
//              Q~ = fq 2^(g_i) in place, den_i = sum_t a_it + Q~_i . z_n
//   thread 0 : o = Q~ S_n + a V                          -> TMEM [128 x D]
//   4 warps  : y_i = o_i / max(den_i, FLT_MIN)
// The chunk math is that of the reference (src/kernels/gla.py:60-101) with
// 128-token chunks; the causal decay uses per-32-column reference rows so no
// factor exceeds 1 (as in gla_fwd_tc.cu).
#include "common.cuh"
#include "gla_layout.h"
#include "tc.cuh"

namespace lz {
namespace {

constexpr int kC = 128;       // tokens per CTA
constexpr int kThreads = 128;  // row i of the chunk = thread i = TMEM lane i

template <int F, int D>
struct OutTcSmem {
  static constexpr int FB = F / 64, DB = D / 64;
  static constexpr size_t q = 0;                                   // fq: FB boxes 128 x 64
  static constexpr size_t k = q + (size_t)FB * 16384;              // fk
  static constexpr size_t v = k + (size_t)FB * 16384;              // v: DB boxes 128 x 64
  static constexpr size_t s = v + (size_t)DB * 16384;              // S: DB boxes F x 64
  static constexpr size_t z = s + (size_t)DB * F * 128;            // z_n [F] fp32
  static constexpr size_t g = z + (size_t)F * 4;                   // g2 [128]
  static constexpr size_t bf = g + 512;                            // block factors [128]
  static constexpr size_t scan = bf + 512;                         // 4 warp totals
  static constexpr size_t bars = scan + 32;                        // 3 mbarriers
  static constexpr size_t slot = bars + 32;                        // TMEM base address
  static constexpr size_t bytes = slot + 16;
};

// TMEM columns: s [128 x 128] fp32, o [128 x D] fp32, a [128 x 128] bf16 (64 columns)
template <int D>
struct OutTcTmem {
  static constexpr uint32_t s = 0, o = 128, a = 128 + D, cols = (D == 64) ? 256 : 512;
};
enum { OB_FULL = 0, OB_SDONE, OB_ODONE };

template <int F, int D>
__global__ void __launch_bounds__(kThreads, 1)
gla_out_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                  const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap ts,
                  const float* __restrict__ lg, int gph, const float* __restrict__ z_in, int H,
                  int grp, int sgrp, int L, int NT64, int NC, bf16* __restrict__ y,
                  float* __restrict__ y32, float* __restrict__ den_out, float* __restrict__ g_out,
                  const float* __restrict__ gs) {
  using SM = OutTcSmem<F, D>;
  using TM = OutTcTmem<D>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  if (smem_u32(smem_raw) & 1023) {  // the 128-byte swizzle needs a 1024-byte aligned window
    if (threadIdx.x == 0) atomicExch(&tc::g_timeout_flag, 0x80000000u | 95u);
    return;
  }
  unsigned char* base = smem_raw;
  float* sZ = reinterpret_cast<float*>(base + SM::z);
  float* sG = reinterpret_cast<float*>(base + SM::g);
  float* sB = reinterpret_cast<float*>(base + SM::bf);
  float* sScan = reinterpret_cast<float*>(base + SM::scan);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + SM::bars);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(base + SM::slot);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x % NC, bh = blockIdx.x / NC;
  const int b = bh / H;
  const int kvh = kv_head(bh, H, grp);                        // head of fk and v
  const int shd = sgrp > 1 ? kv_head(bh, H, sgrp) : bh;       // head of the states
  const int r0 = c * kC, nvalid = min(kC, L - r0);
  const size_t schunk = (size_t)shd * NT64 + 2 * c;           // scan chunk entering this one
  const bool with_state = c > 0;

  if (tid == 0) {
    tc::mbar_init(&bars[OB_FULL], 1);
    tc::mbar_init(&bars[OB_SDONE], 1);
    tc::mbar_init(&bars[OB_ODONE], 1);
    tc::fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(tslot, TM::cols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tslot;
  if (tid == 0) {
    const uint32_t bytes = (uint32_t)(SM::FB * 2 * 16384 + SM::DB * 16384) +
                           (with_state ? (uint32_t)(SM::DB * F * 128) : 0u);
    tc::mbar_expect_tx(&bars[OB_FULL], bytes);
#pragma unroll
    for (int j = 0; j < SM::FB; ++j) {
      tc::tma_load_3d(base + SM::q + j * 16384, &tq, 64 * j, r0, bh, &bars[OB_FULL]);
      tc::tma_load_3d(base + SM::k + j * 16384, &tk, 64 * j, r0, kvh, &bars[OB_FULL]);
    }
#pragma unroll
    for (int j = 0; j < SM::DB; ++j) {
      tc::tma_load_3d(base + SM::v + j * 16384, &tv, 64 * j, r0, kvh, &bars[OB_FULL]);
      if (with_state)
        tc::tma_load_3d(base + SM::s + (size_t)j * F * 128, &ts, 64 * j, 0, (int)schunk,
                        &bars[OB_FULL]);
    }
  }

  // in-chunk running log2 gate (the chunk's start is the frame: G_start = 0)
  const int r = tid;
  const bool valid = r < nvalid;
  const float* LG = lg + (size_t)(gph ? bh : b) * L;
  float x = valid ? LG[r0 + r] * kLog2e : 0.f;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float u = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += u;
  }
  if (lane == 31) sScan[warp] = x;
  for (int f = tid; f < F; f += kThreads) sZ[f] = with_state ? z_in[schunk * F + f] : 0.f;
  __syncthreads();
  float pre = 0.f;
#pragma unroll
  for (int qq = 0; qq < 4; ++qq)
    if (qq < warp) pre += sScan[qq];
  const float g2 = pre + x;
  sG[r] = g2;
  sB[r] = tc::ex2(__shfl_sync(0xffffffffu, g2, 31) - g2);  // relative to the block's last row
  __syncthreads();

  if (tid == 0) {
    // s = fq fk^T, K = F in steps of 16 through the 64-column swizzled blocks
    tc::mbar_wait(&bars[OB_FULL], 0, 60);
    tc::tc_fence_after();
    constexpr uint32_t id_s = tc::idesc_bf16(128, 128, 0, 0);
    const uint32_t qa = smem_u32(base + SM::q), ka = smem_u32(base + SM::k);
#pragma unroll
    for (int j = 0; j < F / 16; ++j) {
      const uint32_t ko = (j >> 2) * 16384 + (j & 3) * 32;
      tc::mma_ss(tmem + TM::s, tc::sdesc(qa + ko, 16, 1024), tc::sdesc(ka + ko, 16, 1024), id_s,
                 j > 0);
    }
    tc::mma_commit(&bars[OB_SDONE]);
  }
  tc::mbar_wait(&bars[OB_FULL], 0, 61);
  tc::mbar_wait(&bars[OB_SDONE], 0, 62);
  tc::tc_fence_after();

  // a = bf16(s 2^(g2_r - g2_t)) for t <= r (blocks left of the diagonal as
  // 2^(g2_r - g2_ref) 2^(g2_ref - g2_t), both <= 1), and its row sum
  const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
  float den = 0.f;
#pragma unroll 1
  for (int cb = 0; cb < 4; ++cb) {
    uint32_t pk[16];
    if (cb < warp) {
      float s[32];
      tc::tmem_ld32(trow + TM::s + 32 * cb, s);
      const float ar = valid ? tc::ex2(g2 - sG[32 * cb + 31]) : 0.f;
      const float4* bt = reinterpret_cast<const float4*>(sB + 32 * cb);
      tc::tmem_wait_ld();
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) {
        const float4 f = bt[j4];
        pk[2 * j4] = pack_bf16(s[4 * j4] * f.x * ar, s[4 * j4 + 1] * f.y * ar);
        pk[2 * j4 + 1] = pack_bf16(s[4 * j4 + 2] * f.z * ar, s[4 * j4 + 3] * f.w * ar);
      }
    } else if (cb == warp) {
      float s[32];
      tc::tmem_ld32(trow + TM::s + 32 * cb, s);
      const float4* gt = reinterpret_cast<const float4*>(sG + 32 * cb);
      tc::tmem_wait_ld();
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) {
        const float4 f = gt[j4];
        const int t = 32 * cb + 4 * j4;
        float w0 = s[4 * j4] * tc::ex2(g2 - f.x);
        float w1 = s[4 * j4 + 1] * tc::ex2(g2 - f.y);
        float w2 = s[4 * j4 + 2] * tc::ex2(g2 - f.z);
        float w3 = s[4 * j4 + 3] * tc::ex2(g2 - f.w);
        w0 = (t <= r && valid) ? w0 : 0.f;
        w1 = (t + 1 <= r && valid) ? w1 : 0.f;
        w2 = (t + 2 <= r && valid) ? w2 : 0.f;
        w3 = (t + 3 <= r && valid) ? w3 : 0.f;
        pk[2 * j4] = pack_bf16(w0, w1);
        pk[2 * j4 + 1] = pack_bf16(w2, w3);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) pk[j] = 0u;
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) den += bf16_lo(pk[j]) + bf16_hi(pk[j]);
    tc::tmem_st16(trow + TM::a + 16 * cb, pk);
  }
  // Q~ = fq 2^(g2_r) in place (row r, swizzled blocks) and its product with z_n
  {
    const float qs = valid ? tc::ex2(g2) : 0.f;
#pragma unroll 1
    for (int jb = 0; jb < SM::FB; ++jb) {
      unsigned char* rowp = base + SM::q + jb * 16384 + r * 128;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        uint4* p = reinterpret_cast<uint4*>(rowp + ((i ^ (r & 7)) * 16));
        uint4 w = *p;
        const uint32_t u[4] = {w.x, w.y, w.z, w.w};
        uint32_t o4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          o4[e] = pack_bf16(bf16_lo(u[e]) * qs, bf16_hi(u[e]) * qs);
          const int f = 64 * jb + 8 * i + 2 * e;
          den += bf16_lo(o4[e]) * sZ[f] + bf16_hi(o4[e]) * sZ[f + 1];
        }
        *p = make_uint4(o4[0], o4[1], o4[2], o4[3]);
      }
    }
  }
  tc::fence_proxy_async_smem();
  tc::tmem_wait_st();
  tc::tc_fence_before();
  __syncthreads();

  if (tid == 0) {
    // o = Q~ S_n + a V
    tc::tc_fence_after();
    constexpr uint32_t id_o = tc::idesc_bf16(128, D, 0, 1);  // Q~|a (K-major) x S|V (MN-major)
    const uint32_t qa = smem_u32(base + SM::q), sa = smem_u32(base + SM::s),
                   va = smem_u32(base + SM::v);
    if (with_state) {
#pragma unroll
      for (int j = 0; j < F / 16; ++j) {
        const uint32_t ko = (j >> 2) * 16384 + (j & 3) * 32;
        tc::mma_ss(tmem + TM::o, tc::sdesc(qa + ko, 16, 1024),
                   tc::sdesc(sa + 2048 * j, F * 128, 1024), id_o, j > 0);
      }
    }
#pragma unroll
    for (int j = 0; j < kC / 16; ++j)
      tc::mma_ts(tmem + TM::o, tmem + TM::a + 8 * j, tc::sdesc(va + 2048 * j, 16384, 1024), id_o,
                 (with_state || j > 0) ? 1u : 0u);
    tc::mma_commit(&bars[OB_ODONE]);
  }
  tc::mbar_wait(&bars[OB_ODONE], 0, 63);
  tc::tc_fence_after();
  const float inv = 1.f / fmaxf(den, kTiny);
  const size_t row = (size_t)bh * L + r0 + r;
  bf16* yrow = y + row * D;
  if (y32 && valid) {
    den_out[row] = den;
    g_out[row] = gs[schunk] + g2 * 0.6931471805599453f;  // natural-log G of the row
  }
#pragma unroll 1
  for (int db = 0; db < D / 32; ++db) {
    float o[32];
    tc::tmem_ld32(trow + TM::o + 32 * db, o);
    tc::tmem_wait_ld();
    if (valid) {
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint4 w;
        w.x = pack_bf16(o[8 * q4] * inv, o[8 * q4 + 1] * inv);
        w.y = pack_bf16(o[8 * q4 + 2] * inv, o[8 * q4 + 3] * inv);
        w.z = pack_bf16(o[8 * q4 + 4] * inv, o[8 * q4 + 5] * inv);
        w.w = pack_bf16(o[8 * q4 + 6] * inv, o[8 * q4 + 7] * inv);
        *reinterpret_cast<uint4*>(yrow + 32 * db + 8 * q4) = w;
      }
      if (y32) {
        float4* d32 = reinterpret_cast<float4*>(y32 + row * D + 32 * db);
#pragma unroll
        for (int q4 = 0; q4 < 8; ++q4)
          d32[q4] = make_float4(o[4 * q4] * inv, o[4 * q4 + 1] * inv, o[4 * q4 + 2] * inv,
                                o[4 * q4 + 3] * inv);
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, TM::cols);
  }
}

// ------------------------------------------- one CTA per key/value head and chunk
// Inference with one state per key/value head (a gate shared by the heads,
// grouped keys / values): the query heads of a group differ only in fq, so
// one CTA per (batch row, key/value head, 128-token chunk) loads fk, v, the
// state and z once, scans the gate once, and walks the group's query heads:
//   warp 8   : (one thread) TMA of fk, v, S and each head's fq; per head
//              s = fq fk^T and o_inter = fq S_n (unscaled) into TMEM buffers
//              that alternate between heads, then o_intra = a V
//   warps 0-7: row i = TMEM lane i, two warps per lane quadrant, each with
//              half of the row's work: fq_i . z_n from shared memory (after which
//              the next head's fq may load), the weights a from s as in the
//              kernel above, and y_i = (2^(g_i) o_inter + o_intra) / max(den,
//              FLT_MIN) with den = sum_t a_it + 2^(g_i) fq_i . z_n
// Scaling the inter-chunk product after the MMA (instead of writing
// Q~ = fq 2^(g_i) over fq) keeps fq unchanged, so the next head's fq loads
// while this head's weights and output are formed, and the next head's scores
// run while this head's output is written. All waits are on mbarriers.
constexpr int kGroupRows = 256;                   // 8 row warps, two per TMEM lane quadrant
constexpr int kGroupThreads = kGroupRows + 32;     // + the TMA / MMA warp (warp 8)
enum { GB_KV = 0, GB_FQ, GB_S0, GB_S1, GB_O, GB_FQZ, GB_A, GB_OF0, GB_OF1, GB_N };
// TMEM: s [2 buffers x 128], o_inter [2 x 64], o_intra 64, a (bf16) 64
constexpr uint32_t kTgS = 0, kTgOi = 256, kTgOa = 384, kTgA = 448, kTgCols = 512;

template <int F>
struct OutGroupSmem {
  static constexpr int FB = F / 64;
  static constexpr size_t q = 0;                          // fq: FB boxes 128 x 64
  static constexpr size_t k = q + (size_t)FB * 16384;     // fk
  static constexpr size_t v = k + (size_t)FB * 16384;     // v: 128 x 64
  static constexpr size_t s = v + 16384;                  // S: F x 64
  static constexpr size_t z = s + (size_t)F * 128;        // z_n [F] fp32
  static constexpr size_t g = z + (size_t)F * 4;          // g2 [128]
  static constexpr size_t bf = g + 512;                   // block factors [128]
  static constexpr size_t scan = bf + 512;                // 4 warp totals
  static constexpr size_t red = scan + 32;                // row-sum halves [2 heads][2][128]
  static constexpr size_t bars = red + 2048;              // GB_N mbarriers
  static constexpr size_t slot = bars + 8 * GB_N;         // TMEM base address
  static constexpr size_t bytes = slot + 16;
};

template <int F>
__global__ void __launch_bounds__(kGroupThreads, 1)
gla_out_group_tc_kernel(const __grid_constant__ CUtensorMap tq,
                        const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv,
                        const __grid_constant__ CUtensorMap ts, const float* __restrict__ lg,
                        const float* __restrict__ z_in, int H, int grp, int L, int NT64, int NC,
                        bf16* __restrict__ y) {
  constexpr int D = 64;
  using SM = OutGroupSmem<F>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  if (smem_u32(smem_raw) & 1023) {
    if (threadIdx.x == 0) atomicExch(&tc::g_timeout_flag, 0x80000000u | 93u);
    return;
  }
  unsigned char* base = smem_raw;
  float* sZ = reinterpret_cast<float*>(base + SM::z);
  float* sG = reinterpret_cast<float*>(base + SM::g);
  float* sB = reinterpret_cast<float*>(base + SM::bf);
  float* sScan = reinterpret_cast<float*>(base + SM::scan);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + SM::bars);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(base + SM::slot);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x % NC, bk = blockIdx.x / NC;  // bk = b * Hkv + key/value head
  const int Hkv = H / grp, b = bk / Hkv, j = bk - b * Hkv;
  const int r0 = c * kC, nvalid = min(kC, L - r0);
  const size_t schunk = (size_t)bk * NT64 + 2 * c;  // scan chunk entering this one
  const bool with_state = c > 0;

  if (tid == 0) {
#pragma unroll
    for (int i = 0; i < GB_N; ++i)
      tc::mbar_init(&bars[i],
                    (i == GB_FQZ || i == GB_A || i == GB_OF0 || i == GB_OF1) ? kGroupRows : 1);
    tc::fence_mbar_init();
  }
  if (warp == 8) {
    tc::tmem_alloc(tslot, kTgCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 8) {
    if (lane == 0) {
      const uint32_t kv_bytes = (uint32_t)(SM::FB * 16384 + 16384) +
                                (with_state ? (uint32_t)(F * 128) : 0u);
      tc::mbar_expect_tx(&bars[GB_KV], kv_bytes);
#pragma unroll
      for (int jb = 0; jb < SM::FB; ++jb)
        tc::tma_load_3d(base + SM::k + jb * 16384, &tk, 64 * jb, r0, bk, &bars[GB_KV]);
      tc::tma_load_3d(base + SM::v, &tv, 0, r0, bk, &bars[GB_KV]);
      if (with_state) tc::tma_load_3d(base + SM::s, &ts, 0, 0, (int)schunk, &bars[GB_KV]);
      auto load_fq = [&](int g) {
        tc::mbar_expect_tx(&bars[GB_FQ], (uint32_t)(SM::FB * 16384));
#pragma unroll
        for (int jb = 0; jb < SM::FB; ++jb)
          tc::tma_load_3d(base + SM::q + jb * 16384, &tq, 64 * jb, r0, b * H + j * grp + g,
                          &bars[GB_FQ]);
      };
      load_fq(0);
      tc::mbar_wait(&bars[GB_KV], 0, 50);
      constexpr uint32_t id_s = tc::idesc_bf16(128, 128, 0, 0);  // fq (K) x fk (K)
      constexpr uint32_t id_o = tc::idesc_bf16(128, D, 0, 1);    // fq | a (K) x S | V (MN)
      const uint32_t qa = smem_u32(base + SM::q), ka = smem_u32(base + SM::k),
                     sa = smem_u32(base + SM::s), va = smem_u32(base + SM::v);
      for (int g = 0; g < grp; ++g) {
        const int sb = g & 1;
        const uint32_t ph = (uint32_t)g & 1u, use = (uint32_t)(g >> 1) & 1u;
        tc::mbar_wait(&bars[GB_FQ], ph, 51);
        if (g >= 2) tc::mbar_wait(&bars[GB_OF0 + sb], use ^ 1u, 52);  // o_inter buffer read
        tc::tc_fence_after();
#pragma unroll
        for (int jj = 0; jj < F / 16; ++jj) {
          const uint32_t ko = (jj >> 2) * 16384 + (jj & 3) * 32;
          tc::mma_ss(tmem + kTgS + 128 * sb, tc::sdesc(qa + ko, 16, 1024),
                     tc::sdesc(ka + ko, 16, 1024), id_s, jj > 0);
        }
        if (with_state) {
#pragma unroll
          for (int jj = 0; jj < F / 16; ++jj) {
            const uint32_t ko = (jj >> 2) * 16384 + (jj & 3) * 32;
            tc::mma_ss(tmem + kTgOi + 64 * sb, tc::sdesc(qa + ko, 16, 1024),
                       tc::sdesc(sa + 2048 * jj, F * 128, 1024), id_o, jj > 0);
          }
        }
        tc::mma_commit(&bars[GB_S0 + sb]);
        if (g + 1 < grp) {
          // fq is free once both products have read it and the rows have their fq . z
          tc::mbar_wait(&bars[GB_S0 + sb], use, 53);
          tc::mbar_wait(&bars[GB_FQZ], ph, 54);
          load_fq(g + 1);
        }
        tc::mbar_wait(&bars[GB_A], ph, 55);  // a in TMEM; the last o_intra read
        tc::tc_fence_after();
#pragma unroll
        for (int jj = 0; jj < kC / 16; ++jj)
          tc::mma_ts(tmem + kTgOa, tmem + kTgA + 8 * jj, tc::sdesc(va + 2048 * jj, 16384, 1024),
                     id_o, jj > 0);
        tc::mma_commit(&bars[GB_O]);
      }
    }
    __syncwarp();
  } else {
    // row r = TMEM lane r; the two warps of a lane quadrant split the work of the
    // row: fq . z over features [F/2 hf, F/2 (hf + 1)), the weight blocks 2 hf and
    // 2 hf + 1, and output columns [32 hf, 32 hf + 32)
    const int qd = warp & 3, hf = warp >> 2;
    const int r = 32 * qd + lane;
    float* red = reinterpret_cast<float*>(base + SM::red);
    // in-chunk running log2 gate (the chunk's start is the frame: G_start = 0), shared
    // by the group's heads; both halves of a quadrant form it, half 0 publishes it
    const bool valid = r < nvalid;
    const float* LG = lg + (size_t)b * L;
    float x = valid ? LG[r0 + r] * kLog2e : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float u = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += u;
    }
    if (hf == 0 && lane == 31) sScan[qd] = x;
    for (int f = tid; f < F; f += kGroupRows) sZ[f] = with_state ? z_in[schunk * F + f] : 0.f;
    tc::named_bar_sync(1, kGroupRows);
    float pre = 0.f;
#pragma unroll
    for (int qq = 0; qq < 4; ++qq)
      if (qq < qd) pre += sScan[qq];
    const float g2 = pre + x;
    if (hf == 0) {
      sG[r] = g2;
      sB[r] = tc::ex2(__shfl_sync(0xffffffffu, g2, 31) - g2);  // relative to the block's last row
    }
    tc::named_bar_sync(1, kGroupRows);
    const float qs = valid ? tc::ex2(g2) : 0.f;  // the row scale of fq: Q~_i = fq_i 2^(g2_i)
    const uint32_t trow = tmem + ((uint32_t)(qd * 32) << 16);

    for (int g = 0; g < grp; ++g) {
      const int sb = g & 1;
      const uint32_t ph = (uint32_t)g & 1u, use = (uint32_t)(g >> 1) & 1u;
      // fq_r . z_n from the swizzled fq tile, before the next head's fq may land
      tc::mbar_wait(&bars[GB_FQ], ph, 56);
      float fqz = 0.f;
      if (with_state) {
#pragma unroll 1
        for (int jb = hf * (F / 128); jb < (hf + 1) * (F / 128); ++jb) {
          const unsigned char* rowp = base + SM::q + jb * 16384 + r * 128;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint4 w = *reinterpret_cast<const uint4*>(rowp + ((i ^ (r & 7)) * 16));
            const uint32_t u[4] = {w.x, w.y, w.z, w.w};
            const float* zz = sZ + 64 * jb + 8 * i;
#pragma unroll
            for (int e = 0; e < 4; ++e) fqz += bf16_lo(u[e]) * zz[2 * e] + bf16_hi(u[e]) * zz[2 * e + 1];
          }
        }
      }
      tc::mbar_arrive(&bars[GB_FQZ]);

      // a = bf16(s 2^(g2_r - g2_t)) for t <= r, as gla_out_tc_kernel, and its row sum
      tc::mbar_wait(&bars[GB_S0 + sb], use, 57);
      tc::tc_fence_after();
      float den = 0.f;
#pragma unroll 1
      for (int cb = 2 * hf; cb < 2 * hf + 2; ++cb) {
        uint32_t pk[16];
        if (cb < qd) {
          float sv[32];
          tc::tmem_ld32(trow + kTgS + 128 * sb + 32 * cb, sv);
          const float ar = valid ? tc::ex2(g2 - sG[32 * cb + 31]) : 0.f;
          const float4* bt = reinterpret_cast<const float4*>(sB + 32 * cb);
          tc::tmem_wait_ld();
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4) {
            const float4 f = bt[j4];
            pk[2 * j4] = pack_bf16(sv[4 * j4] * f.x * ar, sv[4 * j4 + 1] * f.y * ar);
            pk[2 * j4 + 1] = pack_bf16(sv[4 * j4 + 2] * f.z * ar, sv[4 * j4 + 3] * f.w * ar);
          }
        } else if (cb == qd) {
          float sv[32];
          tc::tmem_ld32(trow + kTgS + 128 * sb + 32 * cb, sv);
          const float4* gt = reinterpret_cast<const float4*>(sG + 32 * cb);
          tc::tmem_wait_ld();
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4) {
            const float4 f = gt[j4];
            const int t = 32 * cb + 4 * j4;
            float w0 = sv[4 * j4] * tc::ex2(g2 - f.x);
            float w1 = sv[4 * j4 + 1] * tc::ex2(g2 - f.y);
            float w2 = sv[4 * j4 + 2] * tc::ex2(g2 - f.z);
            float w3 = sv[4 * j4 + 3] * tc::ex2(g2 - f.w);
            w0 = (t <= r && valid) ? w0 : 0.f;
            w1 = (t + 1 <= r && valid) ? w1 : 0.f;
            w2 = (t + 2 <= r && valid) ? w2 : 0.f;
            w3 = (t + 3 <= r && valid) ? w3 : 0.f;
            pk[2 * j4] = pack_bf16(w0, w1);
            pk[2 * j4 + 1] = pack_bf16(w2, w3);
          }
        } else {
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) pk[jj] = 0u;
        }
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) den += bf16_lo(pk[jj]) + bf16_hi(pk[jj]);
        tc::tmem_st16(trow + kTgA + 16 * cb, pk);
      }
      den += qs * fqz;  // this half's part of the row sum
      red[(sb * 2 + hf) * 128 + r] = den;
      tc::tmem_wait_st();
      tc::tc_fence_before();
      tc::mbar_arrive(&bars[GB_A]);
      tc::named_bar_sync(2, kGroupRows);  // both halves' row sums written

      tc::mbar_wait(&bars[GB_O], ph, 58);
      tc::tc_fence_after();
      const float inv = 1.f / fmaxf(red[(sb * 2) * 128 + r] + red[(sb * 2 + 1) * 128 + r], kTiny);
      const size_t row = ((size_t)b * H + j * grp + g) * L + r0 + r;
      bf16* yrow = y + row * D;
      {
        const int db = hf;
        float oa[32], oi[32];
        tc::tmem_ld32(trow + kTgOa + 32 * db, oa);
        if (with_state) tc::tmem_ld32(trow + kTgOi + 64 * sb + 32 * db, oi);
        tc::tmem_wait_ld();
        if (!with_state) {
#pragma unroll
          for (int e = 0; e < 32; ++e) oi[e] = 0.f;
        }
        if (valid) {
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            float o8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) o8[e] = (qs * oi[8 * q4 + e] + oa[8 * q4 + e]) * inv;
            uint4 w;
            w.x = pack_bf16(o8[0], o8[1]);
            w.y = pack_bf16(o8[2], o8[3]);
            w.z = pack_bf16(o8[4], o8[5]);
            w.w = pack_bf16(o8[6], o8[7]);
            *reinterpret_cast<uint4*>(yrow + 32 * db + 8 * q4) = w;
          }
        }
      }
      tc::tc_fence_before();
      tc::mbar_arrive(&bars[GB_OF0 + sb]);  // o_inter buffer sb read
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTgCols);
  }
}

// [rows, cols] bf16 viewed as 3-D {cols, inner, outer}, box {64, box_rows, 1},
// 128-byte swizzle, zero fill outside.
bool make_out_map(CUtensorMap* m, const void* ptr, int outer, int inner, int cols, int box_rows) {
  tc::EncodeTiledFn fn = tc::encode_tiled_fn();
  if (!fn || !aligned16(ptr)) return false;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[2] = {(cuuint64_t)cols * 2, (cuuint64_t)inner * cols * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int F, int D>
int launch_out_tc(const bf16* fq, const bf16* fk, const bf16* v, const float* lg, int gph, int B,
                  int H, int Hkv, int sgrp, int L, int NT64, const bf16* s_in, const float* z_in,
                  bf16* y, const GlaSaved& sv, const float* gs, cudaStream_t st) {
  using SM = OutTcSmem<F, D>;
  const int Hs = sgrp > 1 ? H / sgrp : H;
  CUtensorMap mq, mk, mv, ms;
  if (!make_out_map(&mq, fq, B * H, L, F, kC) || !make_out_map(&mk, fk, B * Hkv, L, F, kC) ||
      !make_out_map(&mv, v, B * Hkv, L, D, kC) || !make_out_map(&ms, s_in, B * Hs * NT64, F, D, F))
    return LZ_ERR_UNSUPPORTED;
  const size_t smem = SM::bytes + 1024;  // room to align the window to 1024 bytes
  static bool done[64] = {false};
  {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(gla_out_tc_kernel<F, D>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) {
        set_error(std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
        return LZ_ERR_CUDA;
      }
      done[dev] = true;
    }
  }
  const int NC = (L + kC - 1) / kC;
  gla_out_tc_kernel<F, D><<<(unsigned)((long long)B * H * NC), kThreads, smem, st>>>(
      mq, mk, mv, ms, lg, gph, z_in, H, H / Hkv, sgrp, L, NT64, NC, y, sv.y32, sv.den, sv.g, gs);
  count_launches(1);
  return check_launch("gla_out_tc_kernel");
}

template <int F>
int launch_out_group_tc(const bf16* fq, const bf16* fk, const bf16* v, const float* lg, int B,
                        int H, int Hkv, int L, int NT64, const bf16* s_in, const float* z_in,
                        bf16* y, cudaStream_t st) {
  using SM = OutGroupSmem<F>;
  CUtensorMap mq, mk, mv, ms;
  if (!make_out_map(&mq, fq, B * H, L, F, kC) || !make_out_map(&mk, fk, B * Hkv, L, F, kC) ||
      !make_out_map(&mv, v, B * Hkv, L, 64, kC) ||
      !make_out_map(&ms, s_in, B * Hkv * NT64, F, 64, F))
    return LZ_ERR_UNSUPPORTED;
  static bool done[64] = {false};
  {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(gla_out_group_tc_kernel<F>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)SM::bytes);
      if (e != cudaSuccess) {
        set_error(std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
        return LZ_ERR_CUDA;
      }
      done[dev] = true;
    }
  }
  const int NC = (L + kC - 1) / kC;
  gla_out_group_tc_kernel<F><<<(unsigned)((long long)B * Hkv * NC), kGroupThreads, SM::bytes,
                               st>>>(mq, mk, mv, ms, lg, z_in, H, H / Hkv, L, NT64, NC, y);
  count_launches(1);
  return check_launch("gla_out_group_tc_kernel");
}

}  // namespace

int gla_out_tc(const bf16* fq, const bf16* fk, const bf16* v, const float* lg, int gph, int B,
               int H, int Hkv, int sgrp, int L, int F, int D, const bf16* s_in,
               const float* z_in, bf16* y, const GlaSaved& sv, const float* gs,
               cudaStream_t st) {
  const int NT64 = (L + 63) / 64;
  if (!aligned16(fq) || !aligned16(fk) || !aligned16(v) || !aligned16(s_in) || !aligned16(y) ||
      (sv.y32 && !aligned16(sv.y32)))
    return LZ_ERR_UNSUPPORTED;
  // inference with one state per key/value head (shared gate): one CTA per group
  if (D == 64 && !gph && sgrp > 1 && sgrp == H / Hkv && !sv.y32 && !gs) {
    if (F == 256)
      return launch_out_group_tc<256>(fq, fk, v, lg, B, H, Hkv, L, NT64, s_in, z_in, y, st);
    if (F == 128)
      return launch_out_group_tc<128>(fq, fk, v, lg, B, H, Hkv, L, NT64, s_in, z_in, y, st);
  }
  if (F == 256 && D == 64)
    return launch_out_tc<256, 64>(fq, fk, v, lg, gph, B, H, Hkv, sgrp, L, NT64, s_in, z_in, y, sv, gs,
                                   st);
  if (F == 128 && D == 64)
    return launch_out_tc<128, 64>(fq, fk, v, lg, gph, B, H, Hkv, sgrp, L, NT64, s_in, z_in, y, sv, gs,
                                   st);
  if (F == 128 && D == 128)
    return launch_out_tc<128, 128>(fq, fk, v, lg, gph, B, H, Hkv, sgrp, L, NT64, s_in, z_in, y,
                                   sv, gs, st);
  if (F == 64 && D == 64)
    return launch_out_tc<64, 64>(fq, fk, v, lg, gph, B, H, Hkv, sgrp, L, NT64, s_in, z_in, y, sv,
                                 gs, st);
  return LZ_ERR_UNSUPPORTED;
}

int gla_out_tc_timeout_flag(unsigned int* out) { return tc::read_timeout_flag_here(out); }
int gla_out_tc_timeout_clear() { return tc::clear_timeout_flag_here(); }

}  // namespace lz
