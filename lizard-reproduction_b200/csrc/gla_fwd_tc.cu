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
// 128-token chunks; the per-chunk state never leaves the SM. G is the running
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
constexpr int kOffMisc = kOffS + 32768;     // ones row + barriers + gates (2 KB)
constexpr int kSmemBytes = kOffMisc + 2048 + 1024;  // + alignment slack
// misc block (the first 128 B are the "ones" B-operand row of dz = K~^T 1;
// the MMA also reads rows 1..15 of this 2 KB block, whose products land in
// accumulator columns that are never read)
constexpr int kMiscBars = 128, kMiscG = 256, kMiscZ = 768, kMiscScan = 1280, kMiscTmem = 1296;
// TMEM columns
constexpr uint32_t kTS = 0, kTA = 128, kTO = 192, kTDS = 320, kTDZ = 448, kTCols = 512;

enum { BAR_FULL0 = 0, BAR_FULL1, BAR_EMPTY0, BAR_EMPTY1, BAR_SFULL, BAR_AREADY, BAR_OFULL,
       BAR_SREADY, BAR_COUNT };

__global__ void __launch_bounds__(192, 1)
gla_fwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                  const __grid_constant__ CUtensorMap tv, const float* __restrict__ lg,
                  int gate_per_head, int H, int L, int NT, bf16* __restrict__ y,
                  float* __restrict__ y32, float* __restrict__ den_out,
                  float* __restrict__ g_out) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* misc = base + kOffMisc;
  uint64_t* bars = reinterpret_cast<uint64_t*>(misc + kMiscBars);
  float* sG = reinterpret_cast<float*>(misc + kMiscG);
  float* sZ = reinterpret_cast<float*>(misc + kMiscZ);
  float* sScan = reinterpret_cast<float*>(misc + kMiscScan);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + kMiscTmem);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.x, b = bh / H;
  const bool save = (y32 != nullptr);

  if (tid == 0) {
    tc::mbar_init(&bars[BAR_FULL0], 1);
    tc::mbar_init(&bars[BAR_FULL1], 1);
    tc::mbar_init(&bars[BAR_EMPTY0], 1);
    tc::mbar_init(&bars[BAR_EMPTY1], 1);
    tc::mbar_init(&bars[BAR_SFULL], 1);
    tc::mbar_init(&bars[BAR_AREADY], 128);
    tc::mbar_init(&bars[BAR_OFULL], 1);
    tc::mbar_init(&bars[BAR_SREADY], 128);
    tc::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&tq);
    tc::prefetch_tmap(&tk);
    tc::prefetch_tmap(&tv);
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, kTCols);
    tc::tmem_relinquish();
  }
  if (warp >= 2) {
    const int e = tid - 64;  // 0..127
    if (e < 64) reinterpret_cast<bf16*>(misc)[e] = __float2bfloat16_rn(1.f);
    sZ[e] = 0.f;
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
        tc::tma_load_3d(stage + kOffK, &tk, 0, n * kC, bh, full);
        tc::tma_load_3d(stage + kOffK + 16384, &tk, 64, n * kC, bh, full);
        tc::tma_load_3d(stage + kOffV, &tv, 0, n * kC, bh, full);
        tc::tma_load_3d(stage + kOffV + 16384, &tv, 64, n * kC, bh, full);
        ++issued[st];
      }
      // let every issued copy land before the CTA can exit
      for (int st = 0; st < 2; ++st)
        if (issued[st]) tc::mbar_wait(&bars[BAR_FULL0 + st], (issued[st] - 1) & 1, 9);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t id_s = tc::idesc_bf16(128, 128, 0, 0);   // fq (K) x fk (K)
      constexpr uint32_t id_o = tc::idesc_bf16(128, 128, 0, 1);   // Q~ (K) x S (MN)
      constexpr uint32_t id_ds = tc::idesc_bf16(128, 128, 1, 1);  // K~ (MN) x V (MN)
      constexpr uint32_t id_dz = tc::idesc_bf16(128, 16, 1, 0);   // K~ (MN) x ones (K)
      const uint32_t s_addr = smem_u32(base + kOffS);
      const uint32_t ones = smem_u32(misc);
      for (int n = 0; n < NT; ++n) {
        const int st = n & 1;
        if (!tc::mbar_wait(&bars[BAR_FULL0 + st], (n >> 1) & 1, 2)) break;
        tc::tc_fence_after();
        const uint32_t stage = smem_u32(base + st * kStageBytes);
        const uint32_t qa = stage + kOffQ, ka = stage + kOffK, va = stage + kOffV;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t ko = (j >> 2) * 16384 + (j & 3) * 32;
          tc::mma_ss(tmem + kTS, tc::sdesc(qa + ko, 16, 1024), tc::sdesc(ka + ko, 16, 1024), id_s,
                     j > 0);
        }
        tc::mma_commit(&bars[BAR_SFULL]);
        if (!tc::mbar_wait(&bars[BAR_AREADY], n & 1, 3)) break;
        if (n > 0 && !tc::mbar_wait(&bars[BAR_SREADY], (n - 1) & 1, 4)) break;
        tc::tc_fence_after();
        if (n > 0) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t ko = (j >> 2) * 16384 + (j & 3) * 32;
            tc::mma_ss(tmem + kTO, tc::sdesc(qa + ko, 16, 1024),
                       tc::sdesc(s_addr + 2048 * j, 16384, 1024), id_o, j > 0);
          }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j)
          tc::mma_ts(tmem + kTO, tmem + kTA + 8 * j, tc::sdesc(va + 2048 * j, 16384, 1024), id_o,
                     (n > 0 || j > 0) ? 1u : 0u);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          tc::mma_ss(tmem + kTDS, tc::sdesc(ka + 2048 * j, 16384, 1024),
                     tc::sdesc(va + 2048 * j, 16384, 1024), id_ds, j > 0);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          tc::mma_ss(tmem + kTDZ, tc::sdesc(ka + 2048 * j, 16384, 1024),
                     tc::sdesc(ones + 32 * (j & 3), 16, 1024), id_dz, j > 0);
        tc::mma_commit(&bars[BAR_OFULL]);
        tc::mma_commit(&bars[BAR_EMPTY0 + st]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // chunk row == TMEM lane == state row f
    const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
    const float* LG = lg + (size_t)(gate_per_head ? bh : b) * L;
    float S[128];
#pragma unroll
    for (int i = 0; i < 128; ++i) S[i] = 0.f;
    float z = 0.f, carry = 0.f;
    unsigned char* srow_base = base + kOffS + r * 128;
    for (int n = 0; n < NT; ++n) {
      const int r0 = n * kC;
      const int nvalid = min(kC, L - r0);
      const bool valid = r < nvalid;
      // running log2 gate: inclusive scan over the chunk's 128 rows
      float x = valid ? LG[r0 + r] * kLog2e : 0.f;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += u;
      }
      if (lane == 31) sScan[quad] = x;
      tc::named_bar_sync(1, 128);  // also orders last chunk's sZ writes
      float pre = 0.f;
#pragma unroll
      for (int qq = 0; qq < 4; ++qq)
        if (qq < quad) pre += sScan[qq];
      const float g2 = carry + pre + x;
      sG[r] = g2;
      tc::named_bar_sync(1, 128);
      const float start2 = carry, end2 = sG[nvalid - 1];
      carry = end2;
      if (save && valid) g_out[(size_t)bh * L + r0 + r] = g2 * 0.6931471805599453f;

      if (!__all_sync(0xffffffffu, tc::mbar_wait(&bars[BAR_SFULL], n & 1, 5))) break;
      tc::tc_fence_after();
      // a = bf16(s * decay) for t <= r, row sum of the rounded weights
      float den = 0.f;
#pragma unroll
      for (int cb = 0; cb < 4; ++cb) {
        float s[32];
        tc::tmem_ld32(trow + kTS + 32 * cb, s);
        tc::tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int t0 = 32 * cb + 2 * j;
          const float w0 = (t0 <= r && valid) ? s[2 * j] * exp2f(g2 - sG[t0]) : 0.f;
          const float w1 = (t0 + 1 <= r && valid) ? s[2 * j + 1] * exp2f(g2 - sG[t0 + 1]) : 0.f;
          pk[j] = pack_bf16(w0, w1);
          den += bf16_lo(pk[j]) + bf16_hi(pk[j]);
        }
        tc::tmem_st16(trow + kTA + 16 * cb, pk);
      }
      // Q~ and K~ rows in place (row r of each swizzled 64-column block);
      // den += Q~_r . z
      {
        unsigned char* stage = base + (n & 1) * kStageBytes;
        const float qs = valid ? exp2f(g2 - start2) : 0.f;
        const float ks = valid ? exp2f(end2 - g2) : 0.f;
        float dz = 0.f;
#pragma unroll
        for (int blk = 0; blk < 2; ++blk) {
          unsigned char* rq = stage + kOffQ + blk * 16384 + r * 128;
          unsigned char* rk = stage + kOffK + blk * 16384 + r * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const int p = (c ^ (r & 7)) * 16;
            uint4 w = *reinterpret_cast<uint4*>(rq + p);
            w.x = pack_bf16(bf16_lo(w.x) * qs, bf16_hi(w.x) * qs);
            w.y = pack_bf16(bf16_lo(w.y) * qs, bf16_hi(w.y) * qs);
            w.z = pack_bf16(bf16_lo(w.z) * qs, bf16_hi(w.z) * qs);
            w.w = pack_bf16(bf16_lo(w.w) * qs, bf16_hi(w.w) * qs);
            *reinterpret_cast<uint4*>(rq + p) = w;
            const float* zz = sZ + blk * 64 + c * 8;
            dz += bf16_lo(w.x) * zz[0] + bf16_hi(w.x) * zz[1] + bf16_lo(w.y) * zz[2] +
                  bf16_hi(w.y) * zz[3] + bf16_lo(w.z) * zz[4] + bf16_hi(w.z) * zz[5] +
                  bf16_lo(w.w) * zz[6] + bf16_hi(w.w) * zz[7];
            uint4 u = *reinterpret_cast<uint4*>(rk + p);
            u.x = pack_bf16(bf16_lo(u.x) * ks, bf16_hi(u.x) * ks);
            u.y = pack_bf16(bf16_lo(u.y) * ks, bf16_hi(u.y) * ks);
            u.z = pack_bf16(bf16_lo(u.z) * ks, bf16_hi(u.z) * ks);
            u.w = pack_bf16(bf16_lo(u.w) * ks, bf16_hi(u.w) * ks);
            *reinterpret_cast<uint4*>(rk + p) = u;
          }
        }
        den += dz;
      }
      tc::fence_proxy_async_smem();
      tc::tmem_wait_st();
      tc::tc_fence_before();
      tc::mbar_arrive(&bars[BAR_AREADY]);

      if (!__all_sync(0xffffffffu, tc::mbar_wait(&bars[BAR_OFULL], n & 1, 6))) break;
      tc::tc_fence_after();
      const float inv = 1.f / fmaxf(den, kTiny);
      const size_t row = (size_t)bh * L + r0 + r;
#pragma unroll
      for (int cb = 0; cb < 4; ++cb) {
        float o[32];
        tc::tmem_ld32(trow + kTO + 32 * cb, o);
        tc::tmem_wait_ld();
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(y + row * 128 + 32 * cb);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint4 w;
            w.x = pack_bf16(o[8 * q4 + 0] * inv, o[8 * q4 + 1] * inv);
            w.y = pack_bf16(o[8 * q4 + 2] * inv, o[8 * q4 + 3] * inv);
            w.z = pack_bf16(o[8 * q4 + 4] * inv, o[8 * q4 + 5] * inv);
            w.w = pack_bf16(o[8 * q4 + 6] * inv, o[8 * q4 + 7] * inv);
            dst[q4] = w;
          }
          if (save) {
            float4* d32 = reinterpret_cast<float4*>(y32 + row * 128 + 32 * cb);
#pragma unroll
            for (int q4 = 0; q4 < 8; ++q4)
              d32[q4] = make_float4(o[4 * q4] * inv, o[4 * q4 + 1] * inv, o[4 * q4 + 2] * inv,
                                    o[4 * q4 + 3] * inv);
          }
        }
      }
      if (save && valid) den_out[row] = den;
      // S <- 2^(end-start) S + dS ; publish bf16 S for the next chunk
      const float decay = exp2f(end2 - start2);
#pragma unroll
      for (int cb = 0; cb < 4; ++cb) {
        float d[32];
        tc::tmem_ld32(trow + kTDS + 32 * cb, d);
        tc::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) S[32 * cb + j] = S[32 * cb + j] * decay + d[j];
        unsigned char* srow = srow_base + (cb >> 1) * 16384;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int c = (cb & 1) * 4 + cc;
          const float* v8 = &S[32 * cb + 8 * cc];
          uint4 w;
          w.x = pack_bf16(v8[0], v8[1]);
          w.y = pack_bf16(v8[2], v8[3]);
          w.z = pack_bf16(v8[4], v8[5]);
          w.w = pack_bf16(v8[6], v8[7]);
          *reinterpret_cast<uint4*>(srow + ((c ^ (r & 7)) * 16)) = w;
        }
      }
      const float dzn = tc::tmem_ld1(trow + kTDZ);
      tc::tmem_wait_ld();
      z = z * decay + dzn;
      sZ[r] = z;
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      tc::mbar_arrive(&bars[BAR_SREADY]);
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
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// [rows = BH x L, cols] bf16 viewed as 3-D {cols, L, BH}, box {64, 128, 1},
// 128-byte swizzle, zero fill outside.
bool make_map(CUtensorMap* m, const void* ptr, int BH, int L, int cols) {
  EncodeTiledFn fn = encode_fn();
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
               const GlaSaved& sv, int B, int H, int L, int F, int D, cudaStream_t stream) {
  if (F != 128 || D != 128) return LZ_ERR_UNSUPPORTED;
  if (!aligned16(fq) || !aligned16(fk) || !aligned16(v) || !aligned16(y)) return LZ_ERR_UNSUPPORTED;
  if (sv.y32 && !aligned16(sv.y32)) return LZ_ERR_UNSUPPORTED;
  const int BH = B * H;
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, fq, BH, L, F) || !make_map(&mk, fk, BH, L, F) || !make_map(&mv, v, BH, L, D))
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
  gla_fwd_tc_kernel<<<BH, 192, kSmemBytes, stream>>>(mq, mk, mv, lg, gph, H, L, NT, y, sv.y32,
                                                     sv.den, sv.g);
  count_launches(1);
  return check_launch("gla_fwd_tc_kernel");
}

int gla_tc_timeout_flag(unsigned int* out) {
  cudaError_t e = cudaMemcpyFromSymbol(out, tc::g_timeout_flag, sizeof(unsigned int));
  if (e != cudaSuccess) {
    set_error(std::string("cudaMemcpyFromSymbol: ") + cudaGetErrorString(e));
    return LZ_ERR_CUDA;
  }
  return LZ_OK;
}

}  // namespace lz
