// GLA forward on the 5th-generation tensor cores, F = D = 128, two sequences
// per SM.
//
// One CTA per (batch*head) sequence walks 64-token chunks in order (the
// reference's chunk length, src/kernels/gla.py:19-101). A CTA takes 109 KB of
// shared memory and 256 TMEM columns, so two run on every SM: the 256
// sequences of B = 8, H = 32 are all resident at once (one wave on 148 SMs) and
// each CTA's serial per-chunk chain overlaps the other's.
//
// The running state is kept transposed, S^T [D x F], so that every MMA whose
// rows are value columns has M = 128:
//
//   TMA warp      : fq, fk, v chunk tiles -> 2-stage ring (128-byte swizzle,
//                   48 KB per stage); y of each chunk out of its stage's fq
//                   block (TMA store)
//   MMA thread    : s    = fq fk^T          (M = 64 tokens, N = 64 keys)
//                   o^T  = V^T a^T + S^T Q~^T (M = 128 values, N = 64 tokens;
//                                          S^T bf16 read from TMEM)
//                   S^T += V^T K~          (M = 128, N = 128, K = 64 tokens)
//   row warps (4) : gates (running log2 sum of the chunk), a = bf16(s 2^(g_t -
//                   g_u)) for u <= t and its row sums, K~ = fk 2^(end - g_u) in
//                   place and the normaliser z <- 2^(end - start) z + sum_u K~_u
//   state/output  : Q~ = fq 2^(g_t - start) in place and Q~ . z; S^T (fp32,
//   warps (4)       TMEM) -> bf16 copy (TMEM, the A operand of the inter-chunk
//                   MMA) and 2^(end - start) S^T back in place; y = o /
//                   max(den, FLT_MIN) into the stage's fq block
// (the two groups carry about the same instruction count per chunk, which
// sets the chunk period)
//
// TMEM: S^T fp32 in columns [0, 128), its bf16 copy in [128, 192), and the
// scores s (an M = 64 accumulator: rows in lanes 0-15 of each quadrant)
// sharing [192, 256) with o^T, which the MMA writes once the row warps have
// read s; the next chunk's scores wait until the output warps have read o^T.
//
// In training mode the kernel also stores y in fp32, the row sums, G, and the
// bf16 state and fp32 normaliser entering every 128-token chunk (every other
// 64-token chunk), the layout the backward kernels read (gla_bwd_tc.cu).
#include <mutex>

#include "common.cuh"
#include "gla_layout.h"
#include "tc.cuh"

namespace lz {

namespace {

constexpr int kC = 64;                  // tokens per chunk
constexpr int kBox = 8192;              // one 64 x 64 bf16 box
constexpr int kOffQ = 0, kOffK = 2 * kBox, kOffV = 4 * kBox;
constexpr int kStageBytes = 6 * kBox;   // fq, fk, v: two 64-column boxes each
constexpr int kOffA = 2 * kStageBytes;  // bf16 weights a [64 tokens x 64 keys], K-major
constexpr int kOffMisc = kOffA + kBox;
constexpr int kMiscBytes = 5376;
constexpr int kUsedBytes = kOffMisc + kMiscBytes;  // 111872
constexpr int kSmemBytes = kUsedBytes + 1024;      // room to align the window to 1024 B
// misc block
constexpr int kMiscBars = 0;      // up to 16 mbarriers
constexpr int kMiscTmem = 128;    // TMEM base address
constexpr int kMiscScan = 144;    // 2 warp totals of the gate scan
constexpr int kMiscGS = 160;      // (start2, end2) per chunk parity
constexpr int kMiscG = 256;       // g2 per chunk parity, 2 x 64 floats
constexpr int kMiscDen = 768;     // intra row sums per chunk parity, 2 x 64 floats
constexpr int kMiscQz = 1280;     // Q~ . z, 64 floats
constexpr int kMiscInv = 1536;    // 1 / max(den, FLT_MIN) per chunk parity, 2 x 64 floats
constexpr int kMiscZ = 2048;      // fp32 normaliser z entering the chunk per parity, 2 x 128
constexpr int kMiscZp = 3072;     // column sums of K~ over four 16-token groups, 4 x 128
constexpr int kMiscKs = 5120;     // K~ row factors 2^(end2 - g2_u), 64 floats
// TMEM columns
constexpr uint32_t kTSF = 0, kTSB = 128, kTX = 192, kTCols = 256;

// A wait on the phase of chunk n is correct only while the barrier has not yet
// completed the phase of chunk n + 1. The row warps need nothing from the
// state / output warps to reach the next chunk's gates, nor the MMA thread to
// reach the next chunk's K~, so GATE and KREADY have one barrier per chunk
// parity; for every other barrier the next phase depends on the waiter.
enum { BAR_FULL0 = 0, BAR_FULL1, BAR_EMPTY0, BAR_EMPTY1, BAR_SFULL, BAR_AREADY, BAR_KREADY0,
       BAR_KREADY1, BAR_OFULL, BAR_OFREE, BAR_SREADY, BAR_STDONE, BAR_GATE0, BAR_GATE1,
       BAR_YREADY0, BAR_YREADY1, BAR_COUNT };
static_assert(BAR_COUNT * 8 <= 128, "mbarriers overflow their block");

// warp 0 TMA, warp 1 MMA, warps 2-5 row warps, warps 6-9 state / output warps
constexpr int kThreads = 320;
constexpr int kGroup = 128;

// Timeouts: as in gla_fwd_tc.cu, the two warp groups never leave their chunk
// loops early (they meet at named barriers); after a failed wait every later
// wait returns at once, the groups run through (in-bounds garbage) and the
// kernel ends. The TMA and MMA warps stop at their first failed wait.

// Eight bf16 values times one factor with packed bf16 multiplies: the product
// of two bf16 values is exact in fp32, so each result is the bf16 rounding of
// value * bf16(sc); the factor itself carries the bf16 rounding (2^-9 relative).
__device__ __forceinline__ uint4 scale8(uint4 w, float sc) {
  const __nv_bfloat162 s2 = __float2bfloat162_rn(sc);
  uint32_t* p = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 x = *reinterpret_cast<__nv_bfloat162*>(&p[i]);
    x = __hmul2(x, s2);
    p[i] = *reinterpret_cast<uint32_t*>(&x);
  }
  return w;
}

__global__ void __launch_bounds__(kThreads, 2)
gla_fwd_tc64_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap ty,
                    const float* __restrict__ lg, int gate_per_head, int H, int grp, int L,
                    int NT, int NT128, float* __restrict__ y32, float* __restrict__ den_out,
                    float* __restrict__ g_out, bf16* __restrict__ s_out,
                    float* __restrict__ z_out) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  unsigned char* misc = base + kOffMisc;
  uint64_t* bars = reinterpret_cast<uint64_t*>(misc + kMiscBars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + kMiscTmem);
  float* sScan = reinterpret_cast<float*>(misc + kMiscScan);
  float* sGS = reinterpret_cast<float*>(misc + kMiscGS);
  float* sG = reinterpret_cast<float*>(misc + kMiscG);
  float* sDen = reinterpret_cast<float*>(misc + kMiscDen);
  float* sQz = reinterpret_cast<float*>(misc + kMiscQz);
  float* sInv = reinterpret_cast<float*>(misc + kMiscInv);
  float* sZ = reinterpret_cast<float*>(misc + kMiscZ);
  float* sZp = reinterpret_cast<float*>(misc + kMiscZp);
  float* sKs = reinterpret_cast<float*>(misc + kMiscKs);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.x, b = bh / H;
  const int kvh = kv_head(bh, H, grp);  // head of fk and v (GQA)
  const bool save = (y32 != nullptr);

  if (tid == 0) {
    tc::mbar_init(&bars[BAR_FULL0], 1);
    tc::mbar_init(&bars[BAR_FULL1], 1);
    tc::mbar_init(&bars[BAR_EMPTY0], 1);  // a stage's MMAs are done
    tc::mbar_init(&bars[BAR_EMPTY1], 1);
    tc::mbar_init(&bars[BAR_SFULL], 1);
    tc::mbar_init(&bars[BAR_AREADY], 2 * kGroup);  // a (row warps) and Q~ (state warps)
    tc::mbar_init(&bars[BAR_KREADY0], kGroup);
    tc::mbar_init(&bars[BAR_KREADY1], kGroup);
    tc::mbar_init(&bars[BAR_OFULL], 1);
    tc::mbar_init(&bars[BAR_OFREE], kGroup);
    tc::mbar_init(&bars[BAR_SREADY], kGroup);
    tc::mbar_init(&bars[BAR_STDONE], 1);
    tc::mbar_init(&bars[BAR_GATE0], kGroup);
    tc::mbar_init(&bars[BAR_GATE1], kGroup);
    // y of a chunk is staged (one barrier per stage, so a wait is never two
    // phases behind)
    tc::mbar_init(&bars[BAR_YREADY0], kGroup);
    tc::mbar_init(&bars[BAR_YREADY1], kGroup);
    tc::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&tq);
    tc::prefetch_tmap(&tk);
    tc::prefetch_tmap(&tv);
    tc::prefetch_tmap(&ty);
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, kTCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------- TMA loads and y stores
    if (lane == 0) {
      int issued[2] = {0, 0};
      int stored = 0;  // y tiles of chunks [0, stored) are stored
      auto store_y = [&](int m) -> bool {
        if (!tc::mbar_wait(&bars[BAR_YREADY0 + (m & 1)], (m >> 1) & 1, 14)) return false;
        unsigned char* ystage = base + (m & 1) * kStageBytes + kOffQ;
        tc::tma_store_3d(&ty, ystage, 0, m * kC, bh);
        tc::tma_store_3d(&ty, ystage + kBox, 64, m * kC, bh);
        tc::bulk_commit();
        ++stored;
        return true;
      };
      for (int n = 0; n < NT; ++n) {
        const int st = n & 1;
        unsigned char* stage = base + st * kStageBytes;
        uint64_t* full = &bars[BAR_FULL0 + st];
        // every MMA of chunk n - 2 (same stage) is done
        if (n >= 2 && !tc::mbar_wait(&bars[BAR_EMPTY0 + st], ((n - 2) >> 1) & 1, 1)) break;
        tc::mbar_expect_tx(full, kStageBytes);
        tc::tma_load_3d(stage + kOffK, &tk, 0, n * kC, kvh, full);
        tc::tma_load_3d(stage + kOffK + kBox, &tk, 64, n * kC, kvh, full);
        tc::tma_load_3d(stage + kOffV, &tv, 0, n * kC, kvh, full);
        tc::tma_load_3d(stage + kOffV + kBox, &tv, 64, n * kC, kvh, full);
        ++issued[st];
        // the fq block holds y of chunk n - 2 until its store has read it
        if (n >= 2) {
          if (!store_y(n - 2)) break;
          tc::bulk_wait_read0();
        }
        tc::tma_load_3d(stage + kOffQ, &tq, 0, n * kC, bh, full);
        tc::tma_load_3d(stage + kOffQ + kBox, &tq, 64, n * kC, bh, full);
      }
      while (stored < NT && !*(volatile unsigned int*)&tc::g_timeout_flag && store_y(stored)) {
      }
      tc::bulk_wait0();  // every y store is complete before the CTA exits
      for (int st = 0; st < 2; ++st)  // every issued copy lands before exit
        if (issued[st]) tc::mbar_wait(&bars[BAR_FULL0 + st], (issued[st] - 1) & 1, 9);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t id_s = tc::idesc_bf16(64, 64, 0, 0);     // fq (K) x fk (K)
      constexpr uint32_t id_av = tc::idesc_bf16(128, 64, 1, 0);   // V^T (MN) x a^T (K)
      constexpr uint32_t id_sq = tc::idesc_bf16(128, 64, 0, 0);   // S^T (TMEM) x Q~^T (K)
      constexpr uint32_t id_st = tc::idesc_bf16(128, 128, 1, 1);  // V^T (MN) x K~ (MN)
      const uint32_t a_addr = smem_u32(base + kOffA);
      // s = fq fk^T of chunk m, once its tiles are in and o^T of chunk m - 1
      // (same TMEM columns) has been read
      auto issue_scores = [&](int m) -> bool {
        const int st = m & 1;
        if (!tc::mbar_wait(&bars[BAR_FULL0 + st], (m >> 1) & 1, 2)) return false;
        if (m > 0 && !tc::mbar_wait(&bars[BAR_OFREE], (m - 1) & 1, 12)) return false;
        tc::tc_fence_after();
        const uint32_t stage = smem_u32(base + st * kStageBytes);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t ko = (j >> 2) * kBox + (j & 3) * 32;
          tc::mma_ss(tmem + kTX, tc::sdesc(stage + kOffQ + ko, 16, 1024),
                     tc::sdesc(stage + kOffK + ko, 16, 1024), id_s, j > 0);
        }
        tc::mma_commit(&bars[BAR_SFULL]);
        return true;
      };
      if (issue_scores(0)) {
        for (int n = 0; n < NT; ++n) {
          const int st = n & 1;
          const uint32_t stage = smem_u32(base + st * kStageBytes);
          const uint32_t qa = stage + kOffQ, ka = stage + kOffK, va = stage + kOffV;
          // o^T = V^T a^T + S^T Q~^T: the weights, Q~ and the bf16 state are in place
          if (!tc::mbar_wait(&bars[BAR_AREADY], n & 1, 3)) break;
          if (!tc::mbar_wait(&bars[BAR_SREADY], n & 1, 4)) break;
          tc::tc_fence_after();
#pragma unroll
          for (int j = 0; j < 4; ++j)
            tc::mma_ss(tmem + kTX, tc::sdesc(va + 2048 * j, kBox, 1024),
                       tc::sdesc(a_addr + 32 * j, 16, 1024), id_av, j > 0);
          if (n > 0) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
              tc::mma_ts(tmem + kTX, tmem + kTSB + 8 * j,
                         tc::sdesc(qa + (j >> 2) * kBox + (j & 3) * 32, 16, 1024), id_sq, 1u);
          }
          tc::mma_commit(&bars[BAR_OFULL]);
          // the next chunk's scores go ahead of this chunk's state update, so
          // the row warps can start on them as soon as they are done with K~
          if (n + 1 < NT && !issue_scores(n + 1)) break;
          // S^T += V^T K~ (the state warps pre-scaled S^T by this chunk's decay)
          if (!tc::mbar_wait(&bars[BAR_KREADY0 + st], (n >> 1) & 1, 13)) break;
          tc::tc_fence_after();
#pragma unroll
          for (int j = 0; j < 4; ++j)
            tc::mma_ss(tmem + kTSF, tc::sdesc(va + 2048 * j, kBox, 1024),
                       tc::sdesc(ka + 2048 * j, kBox, 1024), id_st, (n > 0 || j > 0) ? 1u : 0u);
          tc::mma_commit(&bars[BAR_STDONE]);
          tc::mma_commit(&bars[BAR_EMPTY0 + st]);
          if (n + 1 == NT) tc::mbar_wait(&bars[BAR_STDONE], n & 1, 17);  // none in flight at exit
        }
      }
    }
  } else if (warp < 6) {
    // -------- row warps: gates, s -> a and its row sums, Q~ and K~ in place, z
    const int rw = warp - 2;             // 0..3
    const int quad = warp & 3;           // TMEM lane quadrant
    const int e = tid - 64;              // 0..127 within the group
    const uint32_t tq16 = tmem + ((uint32_t)(quad * 32) << 16);
    const float* LG = lg + (size_t)(gate_per_head ? bh : b) * L;
    float carry = 0.f;
    float lg_next = (e < kC && e < L) ? LG[e] : 0.f;
    sZ[e] = 0.f;  // no state enters chunk 0 (parity 0)
    if (save) z_out[(size_t)bh * NT128 * 128 + e] = 0.f;
    tc::named_bar_sync(1, kGroup);
    for (int n = 0; n < NT; ++n) {
      const int r0 = n * kC;
      const int nvalid = min(kC, L - r0);
      const int par = n & 1;
      float* g2c = sG + par * kC;
      // running log2 gate of the chunk: inclusive scan over its 64 rows (warps 2, 3)
      float x = 0.f;
      if (e < kC) {
        x = e < nvalid ? lg_next * kLog2e : 0.f;
        if (r0 + kC + e < L) lg_next = LG[r0 + kC + e];  // the next chunk's gate
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float u = __shfl_up_sync(0xffffffffu, x, o);
          if (lane >= o) x += u;
        }
        if (lane == 31) sScan[rw] = x;
      }
      tc::named_bar_sync(1, kGroup);
      if (e < kC) {
        const float g2 = carry + (rw == 1 ? sScan[0] : 0.f) + x;
        g2c[e] = g2;
        if (e == nvalid - 1) sGS[par * 2 + 1] = g2;
        if (e == 0) sGS[par * 2] = carry;
        if (save && e < nvalid) g_out[(size_t)bh * L + r0 + e] = g2 * 0.6931471805599453f;
      }
      tc::named_bar_sync(1, kGroup);
      const float start2 = carry;
      const float end2 = sGS[par * 2 + 1];
      carry = end2;
      if (e < kC) sKs[e] = e < nvalid ? tc::ex2(end2 - g2c[e]) : 0.f;
      tc::mbar_arrive(&bars[BAR_GATE0 + par]);  // the state warps read this chunk's gates
      tc::mbar_wait(&bars[BAR_SFULL], n & 1, 5);
      tc::tc_fence_after();
      // a = bf16(s 2^(g2_t - g2_u)) for u <= t: row t = 16 quad + (lane & 15),
      // lanes 0-15 take keys [0, 32), lanes 16-31 keys [32, 64)
      {
        const int t = quad * 16 + (lane & 15);
        const int hh = lane >> 4;
        float sc[32];
        tc::tmem_ld16x2_32(tq16 + kTX, sc);
        const float gt = g2c[t];
        const bool tvalid = t < nvalid;
        tc::tmem_wait_ld();
        uint32_t pk[16];
        float den = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int u = 32 * hh + 2 * j;
          float w0 = (u <= t && tvalid) ? sc[2 * j] * tc::ex2(gt - g2c[u]) : 0.f;
          float w1 = (u + 1 <= t && tvalid) ? sc[2 * j + 1] * tc::ex2(gt - g2c[u + 1]) : 0.f;
          pk[j] = pack_bf16(w0, w1);
          den += bf16_lo(pk[j]) + bf16_hi(pk[j]);
        }
        unsigned char* arow = base + kOffA + t * 128;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int cc = 4 * hh + c;  // 16-byte chunk of the row (keys 8 cc .. 8 cc + 7)
          *reinterpret_cast<uint4*>(arow + ((cc ^ (t & 7)) << 4)) =
              make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        }
        den += __shfl_xor_sync(0xffffffffu, den, 16);
        if (hh == 0) sDen[par * kC + t] = den;
      }
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      tc::mbar_arrive(&bars[BAR_AREADY]);
      // K~ = fk 2^(end2 - g2_u) in place, with the column sums of K~: thread e
      // takes four columns (4 p .. 4 p + 3) of the 16-token group tg (the
      // barrier makes every row factor in sKs visible)
      tc::named_bar_sync(1, kGroup);
      {
        unsigned char* stage = base + par * kStageBytes;
        const int p = e & 31, tg = e >> 5;
        unsigned char* col = stage + kOffK + (p >> 4) * kBox + (p & 1) * 8;
        const int chunk = (p & 15) >> 1;
        // every load ahead of its store (the compiler cannot tell the tile and
        // sKs apart, so interleaving would serialise on each store)
        uint2 w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int u = 16 * tg + i;
          w[i] = *reinterpret_cast<const uint2*>(col + u * 128 + ((chunk ^ (u & 7)) << 4));
        }
        float zs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
          const float4 k4 = *reinterpret_cast<const float4*>(sKs + 16 * tg + i);
          const float ks[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint2& x = w[i + j];
            const __nv_bfloat162 k2 = __float2bfloat162_rn(ks[j]);  // as in scale8
            __nv_bfloat162* xh = reinterpret_cast<__nv_bfloat162*>(&x);
            xh[0] = __hmul2(xh[0], k2);
            xh[1] = __hmul2(xh[1], k2);
            zs[0] += bf16_lo(x.x), zs[1] += bf16_hi(x.x), zs[2] += bf16_lo(x.y),
                zs[3] += bf16_hi(x.y);
          }
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int u = 16 * tg + i;
          *reinterpret_cast<uint2*>(col + u * 128 + ((chunk ^ (u & 7)) << 4)) = w[i];
        }
        *reinterpret_cast<float4*>(sZp + tg * 128 + 4 * p) = make_float4(zs[0], zs[1], zs[2], zs[3]);
      }
      tc::fence_proxy_async_smem();
      tc::mbar_arrive(&bars[BAR_KREADY0 + par]);
      tc::named_bar_sync(1, kGroup);
      {
        // z entering the next chunk (the other parity: the state warps may
        // still be reading this chunk's z for Q~ . z)
        const float zn = tc::ex2(end2 - start2) * sZ[par * 128 + e] + sZp[e] + sZp[128 + e] +
                         sZp[256 + e] + sZp[384 + e];
        sZ[(par ^ 1) * 128 + e] = zn;
        if (save && ((n + 1) & 1) == 0 && n + 1 < NT)
          z_out[((size_t)bh * NT128 + (n + 1) / 2) * 128 + e] = zn;
      }
    }
  } else {
    // ------------- state / output warps: S^T for the next chunk; y
    const int quad = warp & 3;
    const int d = quad * 32 + lane;      // value column: TMEM lane of S^T and o^T
    const int e = tid - 192;             // 0..127 within the group
    const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
    if (save) {  // the state entering chunk 0 is zero
      uint4* p = reinterpret_cast<uint4*>(s_out + ((size_t)bh * NT128 * 128 + e) * 128);
#pragma unroll
      for (int i = 0; i < 16; ++i) p[i] = make_uint4(0u, 0u, 0u, 0u);
    }
    for (int n = 0; n < NT; ++n) {
      const int r0 = n * kC;
      const int nvalid = min(kC, L - r0);
      const int par = n & 1;
      tc::mbar_wait(&bars[BAR_GATE0 + par], (n >> 1) & 1, 10);
      // Q~ = fq 2^(g2_t - start2) in place and Q~ . z once the scores (which
      // read fq) are done: thread e scales one 64-column half of row e / 2
      tc::mbar_wait(&bars[BAR_SFULL], n & 1, 8);
      {
        const float start2 = sGS[par * 2];
        const int t = e >> 1, h = e & 1;
        const float qs = t < nvalid ? tc::ex2(sG[par * kC + t] - start2) : 0.f;
        unsigned char* row = base + par * kStageBytes + kOffQ + h * kBox + t * 128;
        const float4* z4 = reinterpret_cast<const float4*>(sZ + par * 128 + 64 * h);
        // every load ahead of the first store (the compiler cannot tell the
        // tile and sZ apart, so interleaving would serialise on each store)
        uint4 w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = *reinterpret_cast<const uint4*>(row + ((i ^ (t & 7)) << 4));
        float dq = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          w[i] = scale8(w[i], qs);
          const float4 za = z4[2 * i], zb = z4[2 * i + 1];
          dq += bf16_lo(w[i].x) * za.x + bf16_hi(w[i].x) * za.y + bf16_lo(w[i].y) * za.z +
                bf16_hi(w[i].y) * za.w + bf16_lo(w[i].z) * zb.x + bf16_hi(w[i].z) * zb.y +
                bf16_lo(w[i].w) * zb.z + bf16_hi(w[i].w) * zb.w;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) *reinterpret_cast<uint4*>(row + ((i ^ (t & 7)) << 4)) = w[i];
        dq += __shfl_xor_sync(0xffffffffu, dq, 1);
        if (h == 0) sQz[t] = dq;
      }
      tc::fence_proxy_async_smem();
      tc::mbar_arrive(&bars[BAR_AREADY]);
      if (n > 0) {
        // S_n^T (complete once chunk n-1's MMAs are done): its bf16 copy for
        // Q~ S_n, and 2^(end - start) S_n^T for the state update of chunk n
        tc::mbar_wait(&bars[BAR_STDONE], (n - 1) & 1, 11);
        tc::tc_fence_after();
        const float decay = tc::ex2(sGS[par * 2 + 1] - sGS[par * 2]);
        const bool keep = save && (n & 1) == 0;  // the state entering 128-token chunk n / 2
        bf16* srow = s_out + ((size_t)bh * NT128 + n / 2) * 128 * 128 + d;
#pragma unroll 1
        for (int hf = 0; hf < 2; ++hf) {
          float sv[64];
          tc::tmem_ld64(trow + kTSF + 64 * hf, sv);
          tc::tmem_wait_ld();
#pragma unroll
          for (int qq = 0; qq < 2; ++qq) {
            const int c0 = 32 * (2 * hf + qq);  // first state column of this quarter
            uint32_t pk[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) pk[j] = pack_bf16(sv[32 * qq + 2 * j], sv[32 * qq + 2 * j + 1]);
            tc::tmem_st16(trow + kTSB + c0 / 2, pk);
            if (keep) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                srow[(size_t)(c0 + 2 * j) * 128] = __ushort_as_bfloat16((unsigned short)(pk[j] & 0xffffu));
                srow[(size_t)(c0 + 2 * j + 1) * 128] = __ushort_as_bfloat16((unsigned short)(pk[j] >> 16));
              }
            }
            uint32_t scl[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) scl[j] = __float_as_uint(sv[32 * qq + j] * decay);
            tc::tmem_st32(trow + kTSF + c0, scl);
          }
        }
        tc::tmem_wait_st();
      }
      tc::tc_fence_before();
      tc::mbar_arrive(&bars[BAR_SREADY]);
      // y of chunk n: o^T row d holds column d of the chunk's 64 outputs
      tc::mbar_wait(&bars[BAR_OFULL], n & 1, 6);
      tc::mbar_wait(&bars[BAR_AREADY], n & 1, 7);  // the row sums are in sDen
      tc::tc_fence_after();
      float o[64];
      tc::tmem_ld64(trow + kTX, o);
      tc::tmem_wait_ld();
      tc::tc_fence_before();
      tc::mbar_arrive(&bars[BAR_OFREE]);
      if (e < kC) {
        const float dtot = sDen[par * kC + e] + sQz[e];
        sInv[par * kC + e] = 1.f / fmaxf(dtot, kTiny);
        if (save && e < nvalid) den_out[(size_t)bh * L + r0 + e] = dtot;
      }
      tc::named_bar_sync(2, kGroup);
      {
        unsigned char* yb = base + par * kStageBytes + kOffQ + (d >> 6) * kBox;
        const int dd = d & 63;
        const int cw = (dd & 7) * 2;
        const float4* inv4 = reinterpret_cast<const float4*>(sInv + par * kC);
#pragma unroll
        for (int t = 0; t < kC; t += 4) {  // all of 1 / den before the first store
          const float4 iv = inv4[t >> 2];
          o[t] *= iv.x, o[t + 1] *= iv.y, o[t + 2] *= iv.z, o[t + 3] *= iv.w;
        }
#pragma unroll
        for (int t = 0; t < kC; ++t)
          *reinterpret_cast<bf16*>(yb + t * 128 + ((((dd >> 3) ^ (t & 7)) << 4) | cw)) =
              __float2bfloat16_rn(o[t]);
        if (save) {
          float* yrow = y32 + ((size_t)bh * L + r0) * 128 + d;
#pragma unroll
          for (int t = 0; t < kC; ++t)
            if (t < nvalid) yrow[(size_t)t * 128] = o[t];
        }
      }
      tc::fence_proxy_async_smem();
      tc::mbar_arrive(&bars[BAR_YREADY0 + par]);
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTCols);
  }
}

// ------------------------------------------------------------ host helpers

// [rows = BH x L, cols] bf16 viewed as 3-D {cols, L, BH}, box {64, 64, 1},
// 128-byte swizzle, zero fill outside.
bool make_map64(CUtensorMap* m, const void* ptr, int BH, int L, int cols) {
  tc::EncodeTiledFn fn = tc::encode_tiled_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)L, (cuuint64_t)BH};
  cuuint64_t strides[2] = {(cuuint64_t)cols * 2, (cuuint64_t)L * cols * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)kC, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// Returns LZ_ERR_UNSUPPORTED (without launching) for shapes this kernel does
// not cover; the caller then tries the next kernel.
int gla_fwd_tc64(const bf16* fq, const bf16* fk, const bf16* v, const float* lg, int gph,
                 bf16* y, const GlaSaved& sv, int B, int H, int Hkv, int L, int F, int D,
                 cudaStream_t stream) {
  if (F != 128 || D != 128) return LZ_ERR_UNSUPPORTED;
  if (!aligned16(fq) || !aligned16(fk) || !aligned16(v) || !aligned16(y)) return LZ_ERR_UNSUPPORTED;
  if (sv.y32 && (!aligned16(sv.y32) || !aligned16(sv.s))) return LZ_ERR_UNSUPPORTED;
  const int BH = B * H;
  CUtensorMap mq, mk, mv, my;
  if (!make_map64(&mq, fq, BH, L, F) || !make_map64(&mk, fk, B * Hkv, L, F) ||
      !make_map64(&mv, v, B * Hkv, L, D) || !make_map64(&my, y, BH, L, D))
    return LZ_ERR_UNSUPPORTED;
  static std::mutex mu;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 64 && !attr_done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(gla_fwd_tc64_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           kSmemBytes);
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gla_fwd_tc64_kernel,
                                 cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared);
      if (e != cudaSuccess) {
        set_error(std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
        return LZ_ERR_CUDA;
      }
      attr_done[dev] = true;
    }
  }
  const int NT = (L + kC - 1) / kC;
  const int NT128 = (L + 127) / 128;
  gla_fwd_tc64_kernel<<<BH, kThreads, kSmemBytes, stream>>>(
      mq, mk, mv, my, lg, gph, H, H / Hkv, L, NT, NT128, sv.y32, sv.den, sv.g, sv.s, sv.z);
  count_launches(1);
  return check_launch("gla_fwd_tc64_kernel");
}

int gla_fwd_tc64_timeout_flag(unsigned int* out) { return tc::read_timeout_flag_here(out); }
int gla_fwd_tc64_timeout_clear() { return tc::clear_timeout_flag_here(); }

}  // namespace lz
