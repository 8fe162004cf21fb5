// GLA forward on the 5th-generation tensor cores (tcgen05 + TMEM + TMA),
// F = D = 128.
//
// One CTA per (batch*head) sequence walks 128-token chunks in order:
//
//   TMA warp     : fq, fk, v chunk tiles -> 2-stage shared-memory ring
//                  (128-byte swizzle, 96 KB per stage)
//   MMA thread   : s  = fq fk^T                        -> TMEM [128 x 128] f32
//                  o  = Q~ S_n  +  a V   (a from TMEM)  -> TMEM [128 x 128] f32
//                  dS = K~^T V,  dz = K~^T 1             -> TMEM
//   epilogue WG  : a = bf16(s * 2^(g2_i - g2_t)), t <= i  -> TMEM (A operand)
//   (4 warps,      Q~ = fq 2^(g2_i - start), K~ = fk 2^(end - g2_t) in place
//    row i per     y_i = o_i / max(den_i, FLT_MIN) -> HBM
//    thread)       S <- 2^(end-start) S + dS (fp32, registers) -> bf16 S (smem)
//
// This is the chunked GLA of the reference (src/kernels/gla.py:19-101) with
// 128-token chunks; the running state stays on the SM. In training mode the
// kernel also stores y in fp32, the row sums, G, and the bf16 state and fp32
// normaliser entering every 128-token chunk (TMA store of the operand block)
// for the backward (gla_bwd_tc.cu). G is the running
// sum of the log gates, kept in base-2 units (g2 = G log2 e) so every decay is
// one ex2. The normaliser state z is fp32 in shared memory and den_i = Q~_i.z
// is summed on the CUDA cores; the intra-chunk row sum uses the same
// bf16-rounded weights as the numerator (gla.py:90-95).
#include <mutex>

#include "common.cuh"
#include "gla_layout.h"
#include "tc.cuh"

namespace lz {

namespace {

constexpr int kC = 128;                     // tokens per chunk
constexpr int kStageBytes = 6 * 16384;      // fq, fk, v: two 64-column blocks each
constexpr int kOffQ = 0, kOffK = 32768, kOffV = 65536;
constexpr int kOffS = 2 * kStageBytes;      // bf16 state S [F x D], MN-major
constexpr int kOffMisc = kOffS + 32768;     // ones row + barriers + per-chunk scalars
constexpr int kMiscBytes = 3072;
constexpr int kSmemBytes = kOffMisc + kMiscBytes;  // = 232448, the sm_100 maximum
// misc block layout. It doubles as the 16-row K-major B operand of the
// row-sum MMAs:
//   block A = bytes [0, 2048): row 0 ones, row 1 z_hi[0:64], row 2 z_lo[0:64]
//   block B = bytes [1024, 3072): row 0 ones, row 1 z_hi[64:128], row 2 z_lo[64:128]
// (block B's rows 0-7 are block A's rows 8-15). den_intra = a . (row 0) and
// den_inter = Q~ . (row 1 + row 2) land in TMEM columns; the products of the
// other rows land in columns that are never read, so the remaining bytes hold
// barriers and per-chunk scalars.
constexpr int kMiscBars = 384;    // up to 16 mbarriers (rows 3..)
constexpr int kMiscGS = 512;      // (start2, end2) per chunk parity
constexpr int kMiscScan = 544;    // 4 warp totals
constexpr int kMiscTmem = 560;    // TMEM base address
constexpr int kMiscG = 1408;      // g2 of the current chunk, 128 floats
constexpr int kMiscB = 2048;      // column decay factors 2^(g2_ref - g2_t), 128 floats
// TMEM columns: scores s, output o, running state S (fp32), normaliser z
// (col 0), bf16 intra weights a (the A operand of a V), row sums: a . 1 at
// kTDI, Q~ . z_hi and Q~ . z_lo at kTDQ + 1, + 2
constexpr uint32_t kTSA = 0, kTO = 128, kTSF = 256, kTZ = 384, kTA = 400, kTDI = 464,
                   kTDQ = 480, kTCols = 512;

enum { BAR_FULL0 = 0, BAR_FULL1, BAR_EMPTY0, BAR_EMPTY1, BAR_SFULL, BAR_AREADY, BAR_OFULL,
       BAR_SREADY, BAR_GATE, BAR_SFDONE, BAR_COUNT };

constexpr int kThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2-5 decay, warps 6-9 output

// Timeouts: the decay and output warpgroups synchronise with bar.sync among
// themselves, so they never leave their chunk loop early. A wait that gives up
// sets the device flag; every later wait then returns at once, the groups run
// through their remaining iterations (writing in-bounds garbage) and reach
// every barrier, and the kernel ends. The TMA and MMA warps use no bar.sync and
// stop at their first failed wait.

__device__ __forceinline__ uint4 scale8(uint4 w, float sc) {
  w.x = pack_bf16(bf16_lo(w.x) * sc, bf16_hi(w.x) * sc);
  w.y = pack_bf16(bf16_lo(w.y) * sc, bf16_hi(w.y) * sc);
  w.z = pack_bf16(bf16_lo(w.z) * sc, bf16_hi(w.z) * sc);
  w.w = pack_bf16(bf16_lo(w.w) * sc, bf16_hi(w.w) * sc);
  return w;
}

__global__ void __launch_bounds__(kThreads, 1)
gla_fwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                  const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap ty,
                  const __grid_constant__ CUtensorMap ts, const float* __restrict__ lg,
                  int gate_per_head, int H, int grp, int L, int NT, bf16* __restrict__ y,
                  float* __restrict__ y32, float* __restrict__ den_out,
                  float* __restrict__ g_out, bf16* __restrict__ s_out,
                  float* __restrict__ z_out) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  if (smem_u32(smem_raw) & 1023) {  // the tile swizzle needs a 1024-byte aligned window
    if (threadIdx.x == 0) atomicExch(&tc::g_timeout_flag, 0x80000000u | 99u);
    return;
  }
  unsigned char* base = smem_raw;
  unsigned char* misc = base + kOffMisc;
  uint64_t* bars = reinterpret_cast<uint64_t*>(misc + kMiscBars);
  float* sG = reinterpret_cast<float*>(misc + kMiscG);
  float* sB = reinterpret_cast<float*>(misc + kMiscB);
  float* sGS = reinterpret_cast<float*>(misc + kMiscGS);
  float* sScan = reinterpret_cast<float*>(misc + kMiscScan);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + kMiscTmem);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.x, b = bh / H;
  const int kvh = kv_head(bh, H, grp);  // head of fk and v (GQA)
  const bool save = (y32 != nullptr);

  if (tid == 0) {
    tc::mbar_init(&bars[BAR_FULL0], 1);
    tc::mbar_init(&bars[BAR_FULL1], 1);
    // a stage is free once its MMAs are done and its fq block, reused as the
    // y staging tile, has been read by the output store
    tc::mbar_init(&bars[BAR_EMPTY0], 2);
    tc::mbar_init(&bars[BAR_EMPTY1], 2);
    tc::mbar_init(&bars[BAR_SFULL], 1);
    tc::mbar_init(&bars[BAR_AREADY], 128);
    tc::mbar_init(&bars[BAR_OFULL], 1);
    tc::mbar_init(&bars[BAR_SREADY], 128);
    tc::mbar_init(&bars[BAR_GATE], 128);
    tc::mbar_init(&bars[BAR_SFDONE], 1);
    tc::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&tq);
    tc::prefetch_tmap(&tk);
    tc::prefetch_tmap(&tv);
    tc::prefetch_tmap(&ty);
    if (save) tc::prefetch_tmap(&ts);
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, kTCols);
    tc::tmem_relinquish();
  }
  if (warp >= 2 && warp < 6) {
    const int e = tid - 64;  // 0..127
    // ones in row 0 of both operand blocks, z = 0 in rows 1 and 2
    if (e < 64) {
      reinterpret_cast<bf16*>(misc)[e] = __float2bfloat16_rn(1.f);
      reinterpret_cast<bf16*>(misc + 1024)[e] = __float2bfloat16_rn(1.f);
    } else {
      const int i = e - 64;
      reinterpret_cast<bf16*>(misc + 128)[i] = __float2bfloat16_rn(0.f);
      reinterpret_cast<bf16*>(misc + 256)[i] = __float2bfloat16_rn(0.f);
      reinterpret_cast<bf16*>(misc + 1024 + 128)[i] = __float2bfloat16_rn(0.f);
      reinterpret_cast<bf16*>(misc + 1024 + 256)[i] = __float2bfloat16_rn(0.f);
    }
    tc::fence_proxy_async_smem();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      int issued[2] = {0, 0};
      for (int n = 0; n < NT; ++n) {
        const int st = n & 1;
        if (n >= 2 && !tc::mbar_wait(&bars[BAR_EMPTY0 + st], ((n - 2) >> 1) & 1, 1)) break;
        unsigned char* stage = base + st * kStageBytes;
        uint64_t* full = &bars[BAR_FULL0 + st];
        tc::mbar_expect_tx(full, kStageBytes);
        tc::tma_load_3d(stage + kOffQ, &tq, 0, n * kC, bh, full);
        tc::tma_load_3d(stage + kOffQ + 16384, &tq, 64, n * kC, bh, full);
        tc::tma_load_3d(stage + kOffK, &tk, 0, n * kC, kvh, full);
        tc::tma_load_3d(stage + kOffK + 16384, &tk, 64, n * kC, kvh, full);
        tc::tma_load_3d(stage + kOffV, &tv, 0, n * kC, kvh, full);
        tc::tma_load_3d(stage + kOffV + 16384, &tv, 64, n * kC, kvh, full);
        ++issued[st];
      }
      for (int st = 0; st < 2; ++st)  // every issued copy lands before exit
        if (issued[st]) tc::mbar_wait(&bars[BAR_FULL0 + st], (issued[st] - 1) & 1, 9);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t id_s = tc::idesc_bf16(128, 128, 0, 0);   // fq (K) x fk (K)
      constexpr uint32_t id_o = tc::idesc_bf16(128, 128, 0, 1);   // Q~|a (K) x S|V (MN)
      constexpr uint32_t id_ds = tc::idesc_bf16(128, 128, 1, 1);  // K~ (MN) x V (MN)
      constexpr uint32_t id_dz = tc::idesc_bf16(128, 16, 1, 0);   // K~ (MN) x ones (K)
      constexpr uint32_t id_n16 = tc::idesc_bf16(128, 16, 0, 0);  // Q~|a (K) x ones|z (K)
      const uint32_t s_addr = smem_u32(base + kOffS);
      const uint32_t ones = smem_u32(misc);
      // s = fq fk^T of chunk m into TMEM, signalled on BAR_SFULL
      auto issue_scores = [&](int m) -> bool {
        const int st = m & 1;
        if (!tc::mbar_wait(&bars[BAR_FULL0 + st], (m >> 1) & 1, 2)) return false;
        tc::tc_fence_after();
        const uint32_t stage = smem_u32(base + st * kStageBytes);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t ko = (j >> 2) * 16384 + (j & 3) * 32;
          tc::mma_ss(tmem + kTSA, tc::sdesc(stage + kOffQ + ko, 16, 1024),
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
          if (!tc::mbar_wait(&bars[BAR_AREADY], n & 1, 3)) break;
          if (n > 0 && !tc::mbar_wait(&bars[BAR_SREADY], (n - 1) & 1, 4)) break;
          tc::tc_fence_after();
          // o = Q~ S_n + a V; row sums Q~ . z_n and a . 1
          if (n > 0) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint32_t ko = (j >> 2) * 16384 + (j & 3) * 32;
              tc::mma_ss(tmem + kTO, tc::sdesc(qa + ko, 16, 1024),
                         tc::sdesc(s_addr + 2048 * j, 16384, 1024), id_o, j > 0);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint32_t ko = (j >> 2) * 16384 + (j & 3) * 32;
              tc::mma_ss(tmem + kTDQ, tc::sdesc(qa + ko, 16, 1024),
                         tc::sdesc(ones + (j >> 2) * 1024 + (j & 3) * 32, 16, 1024), id_n16,
                         j > 0);
            }
          }
#pragma unroll
          for (int j = 0; j < 8; ++j)
            tc::mma_ts(tmem + kTO, tmem + kTA + 8 * j, tc::sdesc(va + 2048 * j, 16384, 1024),
                       id_o, (n > 0 || j > 0) ? 1u : 0u);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            tc::mma_ts(tmem + kTDI, tmem + kTA + 8 * j, tc::sdesc(ones + 32 * (j & 3), 16, 1024),
                       id_n16, j > 0);
          tc::mma_commit(&bars[BAR_OFULL]);
          // next chunk's scores go ahead of this chunk's state update, so the
          // decay warps can start on them while the state MMAs run
          if (n + 1 < NT && !issue_scores(n + 1)) break;
          // running state: the output warps pre-scaled S and z by this chunk's decay
#pragma unroll
          for (int j = 0; j < 8; ++j)
            tc::mma_ss(tmem + kTSF, tc::sdesc(ka + 2048 * j, 16384, 1024),
                       tc::sdesc(va + 2048 * j, 16384, 1024), id_ds, (n > 0 || j > 0) ? 1u : 0u);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            tc::mma_ss(tmem + kTZ, tc::sdesc(ka + 2048 * j, 16384, 1024),
                       tc::sdesc(ones + 32 * (j & 3), 16, 1024), id_dz,
                       (n > 0 || j > 0) ? 1u : 0u);
          tc::mma_commit(&bars[BAR_SFDONE]);
          tc::mma_commit(&bars[BAR_EMPTY0 + st]);
          if (n == NT - 1) tc::mbar_wait(&bars[BAR_SFDONE], n & 1, 17);  // none in flight at exit
        }
      }
    }
  } else if (warp < 6) {
    // ------------------------------- decay warps: gates, s -> a, K~ in place
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // chunk row == TMEM lane
    const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
    const float* LG = lg + (size_t)(gate_per_head ? bh : b) * L;
    float carry = 0.f;
    float lg_next = (r < L) ? LG[r] : 0.f;
    for (int n = 0; n < NT; ++n) {
      const int r0 = n * kC;
      const int nvalid = min(kC, L - r0);
      const bool valid = r < nvalid;
      float x = valid ? lg_next * kLog2e : 0.f;
      if (r0 + kC + r < L) lg_next = LG[r0 + kC + r];  // prefetch the next chunk's gate
      tc::mbar_wait(&bars[BAR_SFULL], n & 1, 5);
      tc::tc_fence_after();
      // running log2 gate: inclusive scan over the chunk's 128 rows
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += u;
      }
      if (lane == 31) sScan[quad] = x;
      tc::named_bar_sync(1, 128);
      float pre = 0.f;
#pragma unroll
      for (int qq = 0; qq < 4; ++qq)
        if (qq < quad) pre += sScan[qq];
      const float g2 = carry + pre + x;
      sG[r] = g2;
      // column factor relative to the last row of this row's 32-block (= lane 31)
      sB[r] = tc::ex2(__shfl_sync(0xffffffffu, g2, 31) - g2);
      const float start2 = carry;
      if (r == 0) sGS[(n & 1) * 2] = start2;
      if (r == nvalid - 1) sGS[(n & 1) * 2 + 1] = g2;
      tc::named_bar_sync(1, 128);
      const float end2 = sGS[(n & 1) * 2 + 1];
      carry = end2;
      tc::mbar_arrive(&bars[BAR_GATE]);
      if (save && valid) g_out[(size_t)bh * L + r0 + r] = g2 * 0.6931471805599453f;
      // a = bf16(s 2^(g2_r - g2_t)) for t <= r. Blocks left of the diagonal use
      // 2^(g2_r - g2_ref) 2^(g2_ref - g2_t) with ref the block's last row (both
      // factors <= 1); the diagonal block takes one ex2 per element; blocks to
      // its right are zero. The row sums come from the MMA (a . 1).
#pragma unroll 1
      for (int cb = 0; cb < 4; ++cb) {
        uint32_t pk[16];
        if (cb < quad) {
          float s[32];
          tc::tmem_ld32(trow + kTSA + 32 * cb, s);
          const float ar = valid ? tc::ex2(g2 - sG[32 * cb + 31]) : 0.f;
          const float4* bt = reinterpret_cast<const float4*>(sB + 32 * cb);
          tc::tmem_wait_ld();
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4) {
            const float4 f = bt[j4];
            const uint32_t p0 = pack_bf16(s[4 * j4] * f.x * ar, s[4 * j4 + 1] * f.y * ar);
            const uint32_t p1 = pack_bf16(s[4 * j4 + 2] * f.z * ar, s[4 * j4 + 3] * f.w * ar);
            pk[2 * j4] = p0;
            pk[2 * j4 + 1] = p1;
          }
        } else if (cb == quad) {
          float s[32];
          tc::tmem_ld32(trow + kTSA + 32 * cb, s);
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
            const uint32_t p0 = pack_bf16(w0, w1), p1 = pack_bf16(w2, w3);
            pk[2 * j4] = p0;
            pk[2 * j4 + 1] = p1;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) pk[j] = 0u;
        }
        tc::tmem_st16(trow + kTA + 16 * cb, pk);
      }
      // K~ = fk 2^(end - g2) in place. The causal mask gives the warp of rows
      // 32q..32q+31 q+1 score blocks, so the K~ rows go to the lighter warps:
      // quad 0 scales rows 0..63, quad 1 rows 64..95, quad 2 rows 96..127.
      {
        unsigned char* stage = base + (n & 1) * kStageBytes;
        const int npass = quad == 0 ? 2 : (quad == 3 ? 0 : 1);
        const int row0 = quad == 0 ? 0 : 32 + 32 * quad;
#pragma unroll 1
        for (int ps = 0; ps < npass; ++ps) {
          const int t = row0 + 32 * ps + lane;
          const float ks = t < nvalid ? tc::ex2(end2 - sG[t]) : 0.f;
          uint4 w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            w[i] = *reinterpret_cast<const uint4*>(stage + kOffK + (i >> 3) * 16384 + t * 128 +
                                                   (((i & 7) ^ (t & 7)) * 16));
#pragma unroll
          for (int i = 0; i < 16; ++i)
            *reinterpret_cast<uint4*>(stage + kOffK + (i >> 3) * 16384 + t * 128 +
                                      (((i & 7) ^ (t & 7)) * 16)) = scale8(w[i], ks);
        }
      }
      tc::fence_proxy_async_smem();
      tc::tmem_wait_st();
      tc::tc_fence_before();
      tc::mbar_arrive(&bars[BAR_AREADY]);
    }
  } else {
    // ------------- output warps: y; S, z for the next chunk; Q~ in place
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // chunk row for o; state row f for S, z
    const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
    unsigned char* srow_base = base + kOffS + r * 128;
    // z_hi / z_lo of state row r: row 1 / row 2 of operand block r / 64, column
    // r % 64, in the 128-byte swizzled layout
    unsigned char* zblk = misc + (r >> 6) * 1024;
    const int zcol = ((((r & 63) >> 3) ^ 1) << 4) + (r & 7) * 2;
    const int zcol2 = ((((r & 63) >> 3) ^ 2) << 4) + (r & 7) * 2;
    if (save) {  // the state entering chunk 0 is zero
      uint4* p = reinterpret_cast<uint4*>(s_out + ((size_t)bh * NT * 128 + r) * 128);
#pragma unroll
      for (int i = 0; i < 16; ++i) p[i] = make_uint4(0u, 0u, 0u, 0u);
      z_out[(size_t)bh * NT * 128 + r] = 0.f;
    }
    for (int n = 0; n < NT; ++n) {
      const int r0 = n * kC;
      const int nvalid = min(kC, L - r0);
      const bool valid = r < nvalid;
      tc::mbar_wait(&bars[BAR_OFULL], n & 1, 6);
      tc::tc_fence_after();
      // y = o / max(den, FLT_MIN), den = a . 1 + Q~ . z_hi + Q~ . z_lo
      float dv[32];
      tc::tmem_ld32(trow + kTDI, dv);
      tc::tmem_wait_ld();
      const float dtot = dv[0] + (n > 0 ? dv[17] + dv[18] : 0.f);
      const float inv = 1.f / fmaxf(dtot, kTiny);
      const size_t row = (size_t)bh * L + r0 + r;
      // y rows go to the stage's fq block (free now: every MMA of this chunk is
      // done) in the 128-byte swizzled box layout, then out with one TMA store
      unsigned char* ystage = base + (n & 1) * kStageBytes + kOffQ;
#pragma unroll 1
      for (int hb = 0; hb < 2; ++hb) {
        float o[64];
        tc::tmem_ld64(trow + kTO + 64 * hb, o);
        tc::tmem_wait_ld();
        unsigned char* yrow = ystage + hb * 16384 + r * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint4 w;
          w.x = pack_bf16(o[8 * c + 0] * inv, o[8 * c + 1] * inv);
          w.y = pack_bf16(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
          w.z = pack_bf16(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
          w.w = pack_bf16(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
          *reinterpret_cast<uint4*>(yrow + ((c ^ (r & 7)) * 16)) = w;
        }
        if (save && valid) {
          float4* d32 = reinterpret_cast<float4*>(y32 + row * 128 + 64 * hb);
#pragma unroll
          for (int q4 = 0; q4 < 16; ++q4)
            d32[q4] = make_float4(o[4 * q4] * inv, o[4 * q4 + 1] * inv, o[4 * q4 + 2] * inv,
                                  o[4 * q4 + 3] * inv);
        }
      }
      tc::fence_proxy_async_smem();
      tc::named_bar_sync(2, 128);
      if (r == 0) {
        tc::tma_store_3d(&ty, ystage, 0, r0, bh);
        tc::tma_store_3d(&ty, ystage + 16384, 64, r0, bh);
        tc::bulk_commit();
      }
      if (save && valid) den_out[row] = dtot;
      if (n + 1 < NT) {
        // prepare chunk n+1: bf16 S_{n+1}; S and z pre-scaled by its decay;
        // Q~_{n+1} in place and its row sums against z_{n+1}
        tc::mbar_wait(&bars[BAR_GATE], (n + 1) & 1, 10);
        tc::mbar_wait(&bars[BAR_SFDONE], n & 1, 11);
        tc::tc_fence_after();
        const float start2 = sGS[((n + 1) & 1) * 2], end2 = sGS[((n + 1) & 1) * 2 + 1];
        const float decay = tc::ex2(end2 - start2);
        const float g2r = sG[r];
        const float zn = tc::tmem_ld1(trow + kTZ);
        tc::tmem_wait_ld();
        if (save) {
          z_out[((size_t)bh * NT + n + 1) * 128 + r] = zn;
          // the previous S store must have read the staging block
          if (r == 0) tc::bulk_wait_read0();
          tc::named_bar_sync(3, 128);
        }
        {
          const bf16 zh = __float2bfloat16_rn(zn);
          *reinterpret_cast<bf16*>(zblk + 128 + zcol) = zh;
          *reinterpret_cast<bf16*>(zblk + 256 + zcol2) =
              __float2bfloat16_rn(zn - __bfloat162float(zh));
        }
        tc::tmem_st1(trow + kTZ, __float_as_uint(zn * decay));
#pragma unroll 1
        for (int hb = 0; hb < 2; ++hb) {
          float sv[64];
          tc::tmem_ld64(trow + kTSF + 64 * hb, sv);
          tc::tmem_wait_ld();
          unsigned char* srow = srow_base + hb * 16384;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float* v8 = &sv[8 * c];
            uint4 w;
            w.x = pack_bf16(v8[0], v8[1]);
            w.y = pack_bf16(v8[2], v8[3]);
            w.z = pack_bf16(v8[4], v8[5]);
            w.w = pack_bf16(v8[6], v8[7]);
            *reinterpret_cast<uint4*>(srow + ((c ^ (r & 7)) * 16)) = w;
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t sc[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) sc[j] = __float_as_uint(sv[16 * q + j] * decay);
            tc::tmem_st16(trow + kTSF + 64 * hb + 16 * q, sc);
          }
        }
        if (save) {  // bf16 S_{n+1} to HBM for the backward, from the operand block
          tc::fence_proxy_async_smem();
          tc::named_bar_sync(3, 128);
          if (r == 0) {
            tc::tma_store_3d(&ts, base + kOffS, 0, (n + 1) * kC, bh);
            tc::tma_store_3d(&ts, base + kOffS + 16384, 64, (n + 1) * kC, bh);
            tc::bulk_commit();
          }
        }
        {
          const bool nvld = r < min(kC, L - r0 - kC);
          const float qs = nvld ? tc::ex2(g2r - start2) : 0.f;
          unsigned char* stage = base + ((n + 1) & 1) * kStageBytes;
          uint4 w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            w[i] = *reinterpret_cast<const uint4*>(stage + kOffQ + (i >> 3) * 16384 + r * 128 +
                                                   (((i & 7) ^ (r & 7)) * 16));
#pragma unroll
          for (int i = 0; i < 16; ++i)
            *reinterpret_cast<uint4*>(stage + kOffQ + (i >> 3) * 16384 + r * 128 +
                                      (((i & 7) ^ (r & 7)) * 16)) = scale8(w[i], qs);
        }
      }
      tc::fence_proxy_async_smem();
      tc::tmem_wait_st();
      tc::tc_fence_before();
      tc::mbar_arrive(&bars[BAR_SREADY]);
      if (r == 0) {  // the y staging block is read: hand the stage back to TMA
        tc::bulk_wait_read0();
        tc::mbar_arrive(&bars[BAR_EMPTY0 + (n & 1)]);
      }
      __syncwarp();
    }
    if (r == 0) tc::bulk_wait0();  // output stores complete before the CTA exits
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTCols);
  }
}

// ------------------------------------------------------------ host helpers

// [rows = BH x L, cols] bf16 viewed as 3-D {cols, L, BH}, box {64, 128, 1},
// 128-byte swizzle, zero fill outside.
bool make_map(CUtensorMap* m, const void* ptr, int BH, int L, int cols) {
  tc::EncodeTiledFn fn = tc::encode_tiled_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)L, (cuuint64_t)BH};
  cuuint64_t strides[2] = {(cuuint64_t)cols * 2, (cuuint64_t)L * cols * 2};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// Returns LZ_ERR_UNSUPPORTED (without launching) for shapes this kernel does
// not cover; the caller then uses the general kernel.
int gla_fwd_tc(const bf16* fq, const bf16* fk, const bf16* v, const float* lg, int gph, bf16* y,
               const GlaSaved& sv, int B, int H, int Hkv, int L, int F, int D,
               cudaStream_t stream) {
  if (F != 128 || D != 128) return LZ_ERR_UNSUPPORTED;
  if (!aligned16(fq) || !aligned16(fk) || !aligned16(v)) return LZ_ERR_UNSUPPORTED;
  if (!aligned16(y) || (sv.y32 && (!aligned16(sv.y32) || !aligned16(sv.s)))) {
    // training with these inputs saves 128-token chunk states, which only this
    // kernel writes: the output buffers must suit its TMA stores
    if (sv.y32) {
      set_error("gla_fwd: y and the saved buffer must be 16-byte aligned when F = D = 128");
      return LZ_ERR_INVALID_ARGUMENT;
    }
    return LZ_ERR_UNSUPPORTED;
  }
  const int BH = B * H;
  CUtensorMap mq, mk, mv, my;
  if (!make_map(&mq, fq, BH, L, F) || !make_map(&mk, fk, B * Hkv, L, F) ||
      !make_map(&mv, v, B * Hkv, L, D) || !make_map(&my, y, BH, L, D))
    return LZ_ERR_UNSUPPORTED;
  static std::mutex mu;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 64 && !attr_done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(gla_fwd_tc_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           kSmemBytes);
      if (e != cudaSuccess) {
        set_error(std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
        return LZ_ERR_CUDA;
      }
      attr_done[dev] = true;
    }
  }
  const int NT = (L + kC - 1) / kC;
  CUtensorMap ms = my;  // unused (not prefetched, not stored) in inference
  if (sv.y32 && !make_map(&ms, sv.s, BH, NT * kC, 128)) return LZ_ERR_UNSUPPORTED;
  gla_fwd_tc_kernel<<<BH, kThreads, kSmemBytes, stream>>>(mq, mk, mv, my, ms, lg, gph, H, H / Hkv,
                                                     L, NT, y, sv.y32, sv.den, sv.g, sv.s, sv.z);
  count_launches(1);
  return check_launch("gla_fwd_tc_kernel");
}

int gla_fwd_tc_timeout_flag(unsigned int* out) { return tc::read_timeout_flag_here(out); }

}  // namespace lz
