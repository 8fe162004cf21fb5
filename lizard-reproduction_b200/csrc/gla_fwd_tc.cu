// GLA forward on the 5th-generation tensor cores (tcgen05 + TMEM + TMA),
// F = D = 128.
//
// One CTA per (batch*head) sequence walks 128-token chunks in order:
//
//   TMA warp      : fq, fk, v chunk tiles -> 2-stage shared-memory ring
//                   (128-byte swizzle, 96 KB per stage); the y tile of each
//                   chunk out of its stage's fq block (TMA store)
//   MMA thread    : s  = fq fk^T                        -> TMEM [128 x 128] f32
//                   o  = a V  (a from TMEM), then  o += Q~ S_n
//                   dS = K~^T V,  dz = K~^T 1             -> TMEM
//   decay warps   : a = bf16(s * 2^(g2_i - g2_t)), t <= i  -> TMEM (A operand)
//   (8 warps, two   and its row sums; K~ = fk 2^(end - g2_t) in place
//    per TMEM lane
//    quadrant)
//   output warps  : y_i = o_i / max(den_i, FLT_MIN) -> staged for the TMA store
//   (8 warps)       Q~ = fq 2^(g2_i - start) in place and Q~ . z;
//                   S <- 2^(end-start) S + dS (fp32, TMEM) -> bf16 S (smem)
//
// This is the chunked GLA of the reference (src/kernels/gla.py:19-101) with
// 128-token chunks; the running state stays on the SM. In training mode the
// kernel also stores y in fp32, the row sums, G, and the bf16 state and fp32
// normaliser entering every 128-token chunk (TMA store of the operand block)
// for the backward (gla_bwd_tc.cu). G is the running sum of the log gates,
// kept in base-2 units (g2 = G log2 e) so every decay is one ex2.
//
// Pipeline. The shared-memory port is the busiest resource: every N = 128
// MMA with both operands in shared memory reads about 128 B per cycle, so the
// kernel keeps the CUDA cores' shared-memory traffic to the in-place Q~ / K~
// scaling, the bf16 state and the y tile, and keeps the per-chunk chain short:
//  * a V is issued as soon as the decay warps have written a and the output
//    warps have read the previous o, ahead of Q~ S_n, which waits for the state;
//  * K~ has its own barrier, so only the state MMAs wait for it;
//  * the row sums run on the CUDA cores (an N = 16 MMA costs about as much
//    issue time as an N = 128 one): the decay warps sum the same bf16-rounded
//    weights the numerator uses (gla.py:90-95) and leave them in TMEM, the
//    output warps form Q~ . z from the scaled Q~ values in registers;
//  * Q~_{n+1} is scaled while the state MMAs of chunk n still run;
//  * the fk / v blocks of a stage go back to TMA when the state MMAs are done,
//    its fq block once the y store has read it (the TMA thread stores y and
//    reloads fq in order);
//  * each TMEM lane quadrant has two decay and two output warps, each taking
//    half of the row's columns.
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
// misc block layout. Bytes [0, 2048) double as the 16-row K-major B operand of
// the normaliser MMA dz = K~^T 1: row 0 (bytes [0, 128)) holds ones, so result
// column 0 is the column sum; the other rows only feed result columns that are
// never read, so their bytes hold barriers and per-chunk scalars.
constexpr int kMiscBars = 128;    // up to 16 mbarriers
constexpr int kMiscGS = 256;      // (start2, end2) per chunk parity
constexpr int kMiscScan = 272;    // 4 warp totals
constexpr int kMiscTmem = 288;    // TMEM base address
constexpr int kMiscG = 512;       // g2 of the current chunk, 128 floats
constexpr int kMiscB = 1024;      // column decay factors 2^(g2_ref - g2_t), 128 floats
constexpr int kMiscZ = 1536;      // fp32 normaliser z entering the chunk, 128 floats
constexpr int kMiscDQ = 2048;     // Q~ . z halves of every row, 2 x 128 floats
// TMEM columns: scores s, output o, running state S (fp32), normaliser z
// (col 0 of a 16-column MMA result), bf16 intra weights a (the A operand of
// a V), intra row sums (chunk parity x column half)
constexpr uint32_t kTSA = 0, kTO = 128, kTSF = 256, kTZ = 384, kTA = 400, kTDI = 464,
                   kTCols = 512;

enum { BAR_FULL0 = 0, BAR_FULL1, BAR_EMPTY0, BAR_EMPTY1, BAR_SFULL, BAR_AREADY, BAR_KREADY,
       BAR_OFULL, BAR_OFREE, BAR_SREADY, BAR_GATE, BAR_SFDONE, BAR_YREADY0, BAR_YREADY1,
       BAR_COUNT };

// warp 0 TMA, warp 1 MMA, warps 2-9 decay, warps 10-17 output
constexpr int kThreads = 576;
constexpr int kGroup = 256;  // threads of the decay group and of the output group

// Timeouts: the decay and output warp groups synchronise with bar.sync among
// themselves, so they never leave their chunk loop early. A wait that gives up
// sets the device flag; every later wait then returns at once, the groups run
// through their remaining iterations (writing in-bounds garbage) and reach
// every barrier, and the kernel ends. The TMA and MMA warps use no bar.sync and
// stop at their first failed wait.

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

__device__ __forceinline__ float sum_bf16x2(uint32_t p) { return bf16_lo(p) + bf16_hi(p); }

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
  float* sZ = reinterpret_cast<float*>(misc + kMiscZ);
  float* sDQ = reinterpret_cast<float*>(misc + kMiscDQ);
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
    // a stage's fk and v blocks are free once its state MMAs are done; its fq
    // block, reused as the y staging tile, once the TMA thread's y store has read it
    tc::mbar_init(&bars[BAR_EMPTY0], 1);
    tc::mbar_init(&bars[BAR_EMPTY1], 1);
    // y of a chunk is staged (one barrier per stage: its phases are the
    // stage's chunks, so a wait is never two phases behind)
    tc::mbar_init(&bars[BAR_YREADY0], kGroup);
    tc::mbar_init(&bars[BAR_YREADY1], kGroup);
    tc::mbar_init(&bars[BAR_SFULL], 1);
    tc::mbar_init(&bars[BAR_AREADY], kGroup);
    tc::mbar_init(&bars[BAR_KREADY], kGroup);
    tc::mbar_init(&bars[BAR_OFULL], 1);
    tc::mbar_init(&bars[BAR_OFREE], kGroup);
    tc::mbar_init(&bars[BAR_SREADY], kGroup);
    tc::mbar_init(&bars[BAR_GATE], kGroup);
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
  if (warp >= 2 && warp < 4) {  // the ones row of the normaliser MMA's B operand
    reinterpret_cast<bf16*>(misc)[tid - 64] = __float2bfloat16_rn(1.f);
    tc::fence_proxy_async_smem();
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
      // y of chunk m leaves from its stage's fq block; the block is reusable
      // once the store has read it
      auto store_y = [&](int m) -> bool {
        if (!tc::mbar_wait(&bars[BAR_YREADY0 + (m & 1)], (m >> 1) & 1, 14)) return false;
        unsigned char* ystage = base + (m & 1) * kStageBytes + kOffQ;
        tc::tma_store_3d(&ty, ystage, 0, m * kC, bh);
        tc::tma_store_3d(&ty, ystage + 16384, 64, m * kC, bh);
        tc::bulk_commit();
        ++stored;
        return true;
      };
      for (int n = 0; n < NT; ++n) {
        const int st = n & 1;
        unsigned char* stage = base + st * kStageBytes;
        uint64_t* full = &bars[BAR_FULL0 + st];
        // fk and v of chunk n - 2 are consumed once its state MMAs are done
        if (n >= 2 && !tc::mbar_wait(&bars[BAR_EMPTY0 + st], ((n - 2) >> 1) & 1, 1)) break;
        tc::mbar_expect_tx(full, kStageBytes);
        tc::tma_load_3d(stage + kOffK, &tk, 0, n * kC, kvh, full);
        tc::tma_load_3d(stage + kOffK + 16384, &tk, 64, n * kC, kvh, full);
        tc::tma_load_3d(stage + kOffV, &tv, 0, n * kC, kvh, full);
        tc::tma_load_3d(stage + kOffV + 16384, &tv, 64, n * kC, kvh, full);
        ++issued[st];
        // the fq block holds y of chunk n - 2 until its store has read it
        if (n >= 2) {
          if (!store_y(n - 2)) break;
          tc::bulk_wait_read0();
        }
        tc::tma_load_3d(stage + kOffQ, &tq, 0, n * kC, bh, full);
        tc::tma_load_3d(stage + kOffQ + 16384, &tq, 64, n * kC, bh, full);
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
      constexpr uint32_t id_s = tc::idesc_bf16(128, 128, 0, 0);   // fq (K) x fk (K)
      constexpr uint32_t id_o = tc::idesc_bf16(128, 128, 0, 1);   // Q~|a (K) x S|V (MN)
      constexpr uint32_t id_ds = tc::idesc_bf16(128, 128, 1, 1);  // K~ (MN) x V (MN)
      constexpr uint32_t id_dz = tc::idesc_bf16(128, 16, 1, 0);   // K~ (MN) x ones (K)
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
          // o = a V: the weights are written and the previous o has been read
          if (!tc::mbar_wait(&bars[BAR_AREADY], n & 1, 3)) break;
          if (n > 0 && !tc::mbar_wait(&bars[BAR_OFREE], (n - 1) & 1, 12)) break;
          tc::tc_fence_after();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            tc::mma_ts(tmem + kTO, tmem + kTA + 8 * j, tc::sdesc(va + 2048 * j, 16384, 1024),
                       id_o, j > 0);
          // o += Q~ S_n once the state and Q~ are in shared memory
          if (n > 0) {
            if (!tc::mbar_wait(&bars[BAR_SREADY], (n - 1) & 1, 4)) break;
            tc::tc_fence_after();
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint32_t ko = (j >> 2) * 16384 + (j & 3) * 32;
              tc::mma_ss(tmem + kTO, tc::sdesc(qa + ko, 16, 1024),
                         tc::sdesc(s_addr + 2048 * j, 16384, 1024), id_o, 1u);
            }
          }
          tc::mma_commit(&bars[BAR_OFULL]);
          // K~ of this chunk is scaled; the next chunk's scores go ahead of this
          // chunk's state update so the decay warps can start on them while the
          // state MMAs run
          if (!tc::mbar_wait(&bars[BAR_KREADY], n & 1, 13)) break;
          tc::tc_fence_after();
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
  } else if (warp < 10) {
    // ------------------- decay warps: gates, s -> a and its row sums, K~ in place
    const int dw = warp - 2;             // 0..7
    const int h = dw >> 2;               // column half of every 32-column score block
    const int quad = warp & 3;
    const int r = quad * 32 + lane;      // chunk row == TMEM lane
    const int et = (dw << 5) | lane;     // 0..255 within the group
    const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
    const float* LG = lg + (size_t)(gate_per_head ? bh : b) * L;
    float carry = 0.f;
    float lg_next = (h == 0 && r < L) ? LG[r] : 0.f;
    for (int n = 0; n < NT; ++n) {
      const int r0 = n * kC;
      const int nvalid = min(kC, L - r0);
      const bool valid = r < nvalid;
      float x = (h == 0 && valid) ? lg_next * kLog2e : 0.f;
      if (h == 0 && r0 + kC + r < L) lg_next = LG[r0 + kC + r];  // the next chunk's gate
      tc::mbar_wait(&bars[BAR_SFULL], n & 1, 5);
      tc::tc_fence_after();
      // running log2 gate: inclusive scan over the chunk's 128 rows (first half)
      if (h == 0) {
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float u = __shfl_up_sync(0xffffffffu, x, o);
          if (lane >= o) x += u;
        }
        if (lane == 31) sScan[quad] = x;
      }
      tc::named_bar_sync(1, kGroup);
      if (h == 0) {
        float pre = 0.f;
#pragma unroll
        for (int qq = 0; qq < 4; ++qq)
          if (qq < quad) pre += sScan[qq];
        const float g2 = carry + pre + x;
        sG[r] = g2;
        // column factor relative to the last row of this row's 32-block (= lane 31)
        sB[r] = tc::ex2(__shfl_sync(0xffffffffu, g2, 31) - g2);
        if (r == 0) sGS[(n & 1) * 2] = carry;
        if (r == nvalid - 1) sGS[(n & 1) * 2 + 1] = g2;
      }
      tc::named_bar_sync(1, kGroup);
      const float g2 = sG[r];
      const float end2 = sGS[(n & 1) * 2 + 1];
      carry = end2;
      tc::mbar_arrive(&bars[BAR_GATE]);
      if (save && valid && h == 0) g_out[(size_t)bh * L + r0 + r] = g2 * 0.6931471805599453f;
      // a = bf16(s 2^(g2_r - g2_t)) for t <= r, this warp's 16 columns of every
      // 32-column block. Blocks left of the diagonal use 2^(g2_r - g2_ref)
      // 2^(g2_ref - g2_t) with ref the block's last row (both factors <= 1); the
      // diagonal block takes one ex2 per element; blocks to its right are zero.
      float den = 0.f;
#pragma unroll 1
      for (int cb = 0; cb < 4; ++cb) {
        uint32_t pk[8];
        const int c0 = 32 * cb + 16 * h;
        if (cb < quad) {
          float sc[16];
          tc::tmem_ld16(trow + kTSA + c0, sc);
          const float ar = valid ? tc::ex2(g2 - sG[32 * cb + 31]) : 0.f;
          const float4* bt = reinterpret_cast<const float4*>(sB + c0);
          tc::tmem_wait_ld();
          const float2 ar2 = make_float2(ar, ar);
#pragma unroll
          for (int j4 = 0; j4 < 4; ++j4) {  // (s * f) * ar, two columns per packed multiply
            const float4 f = bt[j4];
            const float2 p0 = __fmul2_rn(__fmul2_rn(make_float2(sc[4 * j4], sc[4 * j4 + 1]),
                                                    make_float2(f.x, f.y)), ar2);
            const float2 p1 = __fmul2_rn(__fmul2_rn(make_float2(sc[4 * j4 + 2], sc[4 * j4 + 3]),
                                                    make_float2(f.z, f.w)), ar2);
            pk[2 * j4] = pack_bf16(p0.x, p0.y);
            pk[2 * j4 + 1] = pack_bf16(p1.x, p1.y);
          }
        } else if (cb == quad) {
          float sc[16];
          tc::tmem_ld16(trow + kTSA + c0, sc);
          const float4* gt = reinterpret_cast<const float4*>(sG + c0);
          tc::tmem_wait_ld();
#pragma unroll
          for (int j4 = 0; j4 < 4; ++j4) {
            const float4 f = gt[j4];
            const int t = c0 + 4 * j4;
            float w0 = sc[4 * j4] * tc::ex2(g2 - f.x);
            float w1 = sc[4 * j4 + 1] * tc::ex2(g2 - f.y);
            float w2 = sc[4 * j4 + 2] * tc::ex2(g2 - f.z);
            float w3 = sc[4 * j4 + 3] * tc::ex2(g2 - f.w);
            w0 = (t <= r && valid) ? w0 : 0.f;
            w1 = (t + 1 <= r && valid) ? w1 : 0.f;
            w2 = (t + 2 <= r && valid) ? w2 : 0.f;
            w3 = (t + 3 <= r && valid) ? w3 : 0.f;
            pk[2 * j4] = pack_bf16(w0, w1);
            pk[2 * j4 + 1] = pack_bf16(w2, w3);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) pk[j] = 0u;
        }
        if (cb <= quad) {
#pragma unroll
          for (int j = 0; j < 8; ++j) den += sum_bf16x2(pk[j]);
        }
        tc::tmem_st8(trow + kTA + 16 * cb + 8 * h, pk);
      }
      // this half's row sum of the bf16 weights, one column per (parity, half)
      tc::tmem_st1(trow + kTDI + 2 * (n & 1) + h, __float_as_uint(den));
      tc::tmem_wait_st();
      tc::tc_fence_before();
      tc::mbar_arrive(&bars[BAR_AREADY]);
      // K~ = fk 2^(end - g2) in place: thread et scales one 64-column half of row et / 2
      {
        unsigned char* stage = base + (n & 1) * kStageBytes;
        const int t = et >> 1, hb = et & 1;
        const float ks = t < nvalid ? tc::ex2(end2 - sG[t]) : 0.f;
        unsigned char* row = stage + kOffK + hb * 16384 + t * 128;
        uint4 w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          w[i] = *reinterpret_cast<const uint4*>(row + ((i ^ (t & 7)) * 16));
#pragma unroll
        for (int i = 0; i < 8; ++i)
          *reinterpret_cast<uint4*>(row + ((i ^ (t & 7)) * 16)) = scale8(w[i], ks);
      }
      tc::fence_proxy_async_smem();
      tc::mbar_arrive(&bars[BAR_KREADY]);
    }
  } else {
    // ------------- output warps: y; S, z for the next chunk; Q~ in place
    const int ow = warp - 10;            // 0..7
    const int h = ow >> 2;               // column half
    const int quad = warp & 3;
    const int r = quad * 32 + lane;      // chunk row for o; state row f for S, z
    const int et = (ow << 5) | lane;     // 0..255 within the group
    const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
    unsigned char* srow = base + kOffS + h * 16384 + r * 128;  // this half of state row r
    sDQ[h * 128 + r] = 0.f;              // no state enters chunk 0
    if (save) {  // the state entering chunk 0 is zero
      uint4* p = reinterpret_cast<uint4*>(s_out + ((size_t)bh * NT * 128 + r) * 128 + 64 * h);
#pragma unroll
      for (int i = 0; i < 8; ++i) p[i] = make_uint4(0u, 0u, 0u, 0u);
      if (h == 0) z_out[(size_t)bh * NT * 128 + r] = 0.f;
    }
    tc::named_bar_sync(4, kGroup);
    for (int n = 0; n < NT; ++n) {
      const int r0 = n * kC;
      const int nvalid = min(kC, L - r0);
      const bool valid = r < nvalid;
      tc::mbar_wait(&bars[BAR_OFULL], n & 1, 6);
      tc::tc_fence_after();
      // intra row sums (both halves) and this half of o; then o is free for the next a V
      const float di0 = tc::tmem_ld1(trow + kTDI + 2 * (n & 1));
      const float di1 = tc::tmem_ld1(trow + kTDI + 2 * (n & 1) + 1);
      float o[64];
      tc::tmem_ld64(trow + kTO + 64 * h, o);
      // den = a . 1 + Q~ . z (the Q~ . z halves were formed with Q~)
      const float dq = sDQ[r] + sDQ[128 + r];
      tc::tmem_wait_ld();
      tc::tc_fence_before();
      tc::mbar_arrive(&bars[BAR_OFREE]);
      // y = o / max(den, FLT_MIN): this half of row r into the stage's fq block
      // (every MMA reading it is done) in the 128-byte swizzled box layout; the
      // TMA thread stores the tile
      const float dtot = di0 + di1 + dq;
      const float inv = 1.f / fmaxf(dtot, kTiny);
      const size_t row = (size_t)bh * L + r0 + r;
      {
        unsigned char* yrow = base + (n & 1) * kStageBytes + kOffQ + h * 16384 + r * 128;
        const float2 inv2 = make_float2(inv, inv);
#pragma unroll
        for (int i = 0; i < 64; i += 2) {  // o * inv, two columns per packed multiply
          const float2 q = __fmul2_rn(make_float2(o[i], o[i + 1]), inv2);
          o[i] = q.x, o[i + 1] = q.y;
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint4 w;
          w.x = pack_bf16(o[8 * c + 0], o[8 * c + 1]);
          w.y = pack_bf16(o[8 * c + 2], o[8 * c + 3]);
          w.z = pack_bf16(o[8 * c + 4], o[8 * c + 5]);
          w.w = pack_bf16(o[8 * c + 6], o[8 * c + 7]);
          *reinterpret_cast<uint4*>(yrow + ((c ^ (r & 7)) * 16)) = w;
        }
        tc::fence_proxy_async_smem();
        tc::mbar_arrive(&bars[BAR_YREADY0 + (n & 1)]);
      }
      if (valid) {
        if (save) {
          float4* d32 = reinterpret_cast<float4*>(y32 + row * 128 + 64 * h);
#pragma unroll
          for (int q4 = 0; q4 < 16; ++q4)  // o already holds o * inv
            d32[q4] = make_float4(o[4 * q4], o[4 * q4 + 1], o[4 * q4 + 2], o[4 * q4 + 3]);
          if (h == 0) den_out[row] = dtot;
        }
      }
      if (n + 1 < NT) {
        // prepare chunk n+1. Q~_{n+1} in place first: it needs only the gates
        // and the finished scores of chunk n+1, so it overlaps this chunk's
        // state MMAs; the scaled values stay in registers for Q~ . z.
        tc::mbar_wait(&bars[BAR_GATE], (n + 1) & 1, 10);
        tc::mbar_wait(&bars[BAR_SFULL], (n + 1) & 1, 15);
        const float start2 = sGS[((n + 1) & 1) * 2], end2 = sGS[((n + 1) & 1) * 2 + 1];
        const float decay = tc::ex2(end2 - start2);
        uint4 qv[8];
        {
          const bool nvld = r < min(kC, L - r0 - kC);
          const float qs = nvld ? tc::ex2(sG[r] - start2) : 0.f;
          unsigned char* nrow = base + ((n + 1) & 1) * kStageBytes + kOffQ + h * 16384 + r * 128;
#pragma unroll
          for (int i = 0; i < 8; ++i)
            qv[i] = scale8(*reinterpret_cast<const uint4*>(nrow + ((i ^ (r & 7)) * 16)), qs);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            *reinterpret_cast<uint4*>(nrow + ((i ^ (r & 7)) * 16)) = qv[i];
        }
        // then the state: the fp32 z entering chunk n+1, bf16 S_{n+1}; S and z
        // pre-scaled by its decay
        tc::mbar_wait(&bars[BAR_SFDONE], n & 1, 11);
        tc::tc_fence_after();
        if (h == 0) {
          const float zn = tc::tmem_ld1(trow + kTZ);
          tc::tmem_wait_ld();
          if (save) z_out[((size_t)bh * NT + n + 1) * 128 + r] = zn;
          sZ[r] = zn;
          tc::tmem_st1(trow + kTZ, __float_as_uint(zn * decay));
        }
        // the previous S store must have read the staging block (training);
        // every z is in sZ, and every reader of the last Q~ . z halves is done
        if (save && et == 0) tc::bulk_wait_read0();
        tc::named_bar_sync(3, kGroup);
        {
          float sv[64];
          tc::tmem_ld64(trow + kTSF + 64 * h, sv);
          // Q~ . z over this half of row r while the state loads
          const float4* z4 = reinterpret_cast<const float4*>(sZ + 64 * h);
          float2 dq2 = make_float2(0.f, 0.f);
#pragma unroll
          for (int i = 0; i < 8; ++i) {  // two columns per packed FMA
            const uint4 w = qv[i];
            const float4 za = z4[2 * i], zb = z4[2 * i + 1];
            dq2 = __ffma2_rn(make_float2(bf16_lo(w.x), bf16_hi(w.x)), make_float2(za.x, za.y), dq2);
            dq2 = __ffma2_rn(make_float2(bf16_lo(w.y), bf16_hi(w.y)), make_float2(za.z, za.w), dq2);
            dq2 = __ffma2_rn(make_float2(bf16_lo(w.z), bf16_hi(w.z)), make_float2(zb.x, zb.y), dq2);
            dq2 = __ffma2_rn(make_float2(bf16_lo(w.w), bf16_hi(w.w)), make_float2(zb.z, zb.w), dq2);
          }
          const float dqh = dq2.x + dq2.y;
          sDQ[h * 128 + r] = dqh;
          tc::tmem_wait_ld();
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
            uint32_t scl[16];
#pragma unroll
            for (int j = 0; j < 16; j += 2) {  // two columns per packed multiply
              const float2 p = __fmul2_rn(make_float2(sv[16 * q + j], sv[16 * q + j + 1]),
                                          make_float2(decay, decay));
              scl[j] = __float_as_uint(p.x);
              scl[j + 1] = __float_as_uint(p.y);
            }
            tc::tmem_st16(trow + kTSF + 64 * h + 16 * q, scl);
          }
        }
        if (save) {  // bf16 S_{n+1} to HBM for the backward, from the operand block
          tc::fence_proxy_async_smem();
          tc::named_bar_sync(5, kGroup);
          if (et == 0) {
            tc::tma_store_3d(&ts, base + kOffS, 0, (n + 1) * kC, bh);
            tc::tma_store_3d(&ts, base + kOffS + 16384, 64, (n + 1) * kC, bh);
            tc::bulk_commit();
          }
        }
      }
      tc::fence_proxy_async_smem();
      tc::tmem_wait_st();
      tc::tc_fence_before();
      tc::named_bar_sync(4, kGroup);  // the Q~ . z halves of the next chunk are in sDQ
      tc::mbar_arrive(&bars[BAR_SREADY]);
    }
    if (save && et == 0) tc::bulk_wait0();  // state stores complete before the CTA exits
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
int gla_fwd_tc_timeout_clear() { return tc::clear_timeout_flag_here(); }

}  // namespace lz
