// Sliding-window attention forward on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA) for head dim 64 and windows of at most 64 keys, the
// Lizard layer's shape (reference: src/lizard_attention.py:34-44 and the
// Triton forward src/kernels/swa.py:19-59).
//
// One CTA of 8 warps takes 128 query rows [q0, q0 + 128) of one batch row and
// one key/value head, and every query head of that head's group in turn:
//   TMA      : keys and values of rows [q0 - 64, q0 + 128) (192 rows; rows
//              outside the sequence arrive as zeros) once, and each head's 128
//              query rows, all in the 128-byte swizzled operand layout
//   all      : RoPE variant: rotate the keys once and each head's queries in
//              fp32, in place, and split them into bf16 hi + lo operand tiles
//              (the same arithmetic as the 64-row kernels and lz_rope_split)
//   thread 0 : s = q_hi k_hi^T (+ q_hi k_lo^T + q_lo k_hi^T) -> TMEM [128 x 192]
//   8 warps  : row i = TMEM lane i, its window's 96 columns split between the
//              two warps of the lane quadrant: the max (seeded by the sinks,
//              exchanged through shared memory), p = 2^(x - max) split into
//              bf16 hi + lo written over s as the A operand of P V, row sums
//   thread 0 : o = p_hi V + p_lo V                             -> TMEM [128 x 64]
//   8 warps  : y_i = o_i / l_i, 32 columns per warp (training: also lse_i and
//              y_i in fp32)
// The heads overlap: P V of head g runs while the warps rotate the queries of
// head g + 1 (their TMA load was issued when the scores of head g had read the
// query tiles), and the scores of head g + 1 run while the warps write the
// output of head g. One softmax pass over the whole window replaces the online
// rescaling of the 64-key-block kernels; the products carry the same precision
// (about 16 mantissa bits in the logits and in P). 109 KB of shared memory and
// 256 TMEM columns per CTA: two CTAs per SM.
#include <atomic>

#include "common.cuh"
#include "rope_math.cuh"
#include "swa_layout.h"
#include "tc.cuh"

namespace lz {
namespace {

constexpr int kQ = 128;   // query rows per CTA (= TMEM lanes)
constexpr int kThreads = 256;
constexpr int kNK = 192;  // key rows per CTA: [q0 - 64, q0 + 128)
constexpr int kDh = 64;   // head dim (one 128-byte swizzle row)
constexpr float kLn2f = 0.6931471805599453f;

struct SwaTcSmem {
  static constexpr size_t kh = 0, kl = kh + kNK * 128, v = kl + kNK * 128, qh = v + kNK * 128,
                          ql = qh + kQ * 128, red = ql + kQ * 128,  // [2][2][128] fp32
                          bars = red + 2048, slot = bars + 32, bytes = slot + 16;
};
// TMEM columns: s [128 x 192] fp32; p hi / lo (bf16 pairs, 96 columns each)
// written over s; o [128 x 64] fp32
constexpr uint32_t kTmS = 0, kTmPh = 0, kTmPl = kNK / 2, kTmO = kNK, kTmCols = 256;
enum { SB_KV = 0, SB_Q, SB_S, SB_O };

// byte offset of 16-byte chunk c of row r in a 128-byte swizzled tile
__device__ __forceinline__ uint32_t sw128(int r, int c) {
  return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4));
}

// Rotate rows [ROW0, ROW0 + NROWS) of a raw bf16 tile that sits in `lo` (row r
// holds token t0 + r) in place: hi / lo parts of the rotated row into `hi` /
// `lo`, zero for tokens outside [0, L). Rows r >= row_out with a token in the
// sequence are also copied to ghi / glo ([L, 64] of the head) when given.
// Items (row, 8-column pair) are spread over the CTA; a thread's loads are all
// issued before the first rotation.
template <int ROW0, int NROWS, typename CT>
__device__ __forceinline__ void rotate_rows(unsigned char* hi, unsigned char* lo, int t0, int L,
                                            const CT* cs, const CT* sn, long long cs_sl,
                                            int row_out, bf16* ghi, bf16* glo) {
  static_assert(NROWS * 4 % kThreads == 0, "whole items per thread");
  constexpr int kItems = NROWS * 4 / kThreads;
  Raw8<bf16> x1[kItems], x2[kItems];
  Raw8<CT> c1[kItems], c2[kItems], s1[kItems], s2[kItems];
#pragma unroll
  for (int it = 0; it < kItems; ++it) {
    const int e = threadIdx.x + it * kThreads, r = ROW0 + (e >> 2), c8 = e & 3, t = t0 + r;
    if (t >= 0 && t < L) {
      x1[it].load(reinterpret_cast<const bf16*>(lo + sw128(r, c8)));
      x2[it].load(reinterpret_cast<const bf16*>(lo + sw128(r, c8 + 4)));
      const CT* cr = cs + (size_t)t * cs_sl;
      const CT* sr = sn + (size_t)t * cs_sl;
      c1[it].load(cr + 8 * c8);
      c2[it].load(cr + 8 * c8 + kDh / 2);
      s1[it].load(sr + 8 * c8);
      s2[it].load(sr + 8 * c8 + kDh / 2);
    }
  }
#pragma unroll
  for (int it = 0; it < kItems; ++it) {
    const int e = threadIdx.x + it * kThreads, r = ROW0 + (e >> 2), c8 = e & 3, t = t0 + r;
    const uint32_t o1 = sw128(r, c8), o2 = sw128(r, c8 + 4);
    float a1[8], a2[8];
    if (t >= 0 && t < L) {
      float fx1[8], fx2[8], fc1[8], fc2[8], fs1[8], fs2[8];
      x1[it].get(fx1);
      x2[it].get(fx2);
      c1[it].get(fc1);
      c2[it].get(fc2);
      s1[it].get(fs1);
      s2[it].get(fs2);
      rope8(fx1, fx2, fc1, fc2, fs1, fs2, a1, a2);
    } else {
#pragma unroll
      for (int u = 0; u < 8; ++u) a1[u] = a2[u] = 0.f;
    }
    const uint4 h1 = pack8(a1), h2 = pack8(a2);
    const uint4 l1 = resid8(a1, h1), l2 = resid8(a2, h2);
    *reinterpret_cast<uint4*>(hi + o1) = h1;
    *reinterpret_cast<uint4*>(hi + o2) = h2;
    *reinterpret_cast<uint4*>(lo + o1) = l1;
    *reinterpret_cast<uint4*>(lo + o2) = l2;
    if (ghi && r >= row_out && t >= 0 && t < L) {
      const size_t g = (size_t)t * kDh + 8 * c8;
      *reinterpret_cast<uint4*>(ghi + g) = h1;
      *reinterpret_cast<uint4*>(ghi + g + kDh / 2) = h2;
      *reinterpret_cast<uint4*>(glo + g) = l1;
      *reinterpret_cast<uint4*>(glo + g + kDh / 2) = l2;
    }
  }
}

// ROPE: q, k are the unrotated bf16 projections (maps tq, tk), rotated here.
// Otherwise q, k are the rotated operands; SPLIT adds their bf16 residuals
// (maps tql, tkl). v is bf16 in both.
template <bool ROPE, bool SPLIT, typename CT>
__global__ void __launch_bounds__(kThreads, 2)
swa_fwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                  const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tql,
                  const __grid_constant__ CUtensorMap tkl, const CT* __restrict__ cs,
                  const CT* __restrict__ sn, long long cs_sb, long long cs_sl,
                  const float* __restrict__ meta, int n_meta, int W, float scale_log2, int H,
                  int grp, int L, int nqb, bf16* __restrict__ y, float* __restrict__ lse,
                  float* __restrict__ y32, bf16* __restrict__ qh_out, bf16* __restrict__ ql_out,
                  bf16* __restrict__ kh_out, bf16* __restrict__ kl_out) {
  using SM = SwaTcSmem;
  extern __shared__ __align__(1024) unsigned char smem[];
  if (smem_u32(smem) & 1023) {  // the 128-byte swizzle needs a 1024-byte aligned window
    if (threadIdx.x == 0) atomicExch(&tc::g_timeout_flag, 0x80000000u | 89u);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::bars);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + SM::slot);
  float* red = reinterpret_cast<float*>(smem + SM::red);  // [max | sum][half][row]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = warp & 3, hf = warp >> 2;  // TMEM lane quadrant, column half
  const int qb = blockIdx.x % nqb, bk = blockIdx.x / nqb;
  const int Hkv = H / grp, b = bk / Hkv, hk = bk - b * Hkv;
  const int q0 = qb * kQ, k0 = q0 - (kNK - kQ);
  constexpr uint32_t kTileK = kNK * 128, kTileQ = kQ * 128;

  if (tid == 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) tc::mbar_init(&bars[j], 1);
    tc::fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(tslot, kTmCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tslot;

  auto issue_q = [&](int g) {  // query rows of head hk * grp + g
    const int h = hk * grp + g;
    tc::mbar_expect_tx(&bars[SB_Q], (!ROPE && SPLIT) ? 2 * kTileQ : kTileQ);
    if (ROPE) {
      tc::tma_load_4d(smem + SM::ql, &tq, 0, q0, h, b, &bars[SB_Q]);  // raw rows land in lo
    } else {
      tc::tma_load_4d(smem + SM::qh, &tq, 0, q0, h, b, &bars[SB_Q]);
      if (SPLIT) tc::tma_load_4d(smem + SM::ql, &tql, 0, q0, h, b, &bars[SB_Q]);
    }
  };
  auto issue_s = [&]() {  // s = q k^T into TMEM columns [0, 192)
    tc::tc_fence_after();
    constexpr uint32_t id_s = tc::idesc_bf16(kQ, kNK, 0, 0);  // q (K-major) x k (K-major)
    const uint32_t qh = smem_u32(smem + SM::qh), ql = smem_u32(smem + SM::ql),
                   kh = smem_u32(smem + SM::kh), kl = smem_u32(smem + SM::kl);
#pragma unroll
    for (int j = 0; j < kDh / 16; ++j)
      tc::mma_ss(tmem + kTmS, tc::sdesc(qh + 32 * j, 16, 1024), tc::sdesc(kh + 32 * j, 16, 1024),
                 id_s, j > 0);
    if (SPLIT || ROPE) {
#pragma unroll
      for (int j = 0; j < kDh / 16; ++j)
        tc::mma_ss(tmem + kTmS, tc::sdesc(qh + 32 * j, 16, 1024),
                   tc::sdesc(kl + 32 * j, 16, 1024), id_s, 1u);
#pragma unroll
      for (int j = 0; j < kDh / 16; ++j)
        tc::mma_ss(tmem + kTmS, tc::sdesc(ql + 32 * j, 16, 1024),
                   tc::sdesc(kh + 32 * j, 16, 1024), id_s, 1u);
    }
    tc::mma_commit(&bars[SB_S]);
  };
  if (tid == 0) {
    tc::mbar_expect_tx(&bars[SB_KV], (!ROPE && SPLIT) ? 3 * kTileK : 2 * kTileK);
    if (ROPE) {
      tc::tma_load_4d(smem + SM::kl, &tk, 0, k0, hk, b, &bars[SB_KV]);
    } else {
      tc::tma_load_4d(smem + SM::kh, &tk, 0, k0, hk, b, &bars[SB_KV]);
      if (SPLIT) tc::tma_load_4d(smem + SM::kl, &tkl, 0, k0, hk, b, &bars[SB_KV]);
    }
    tc::tma_load_4d(smem + SM::v, &tv, 0, k0, hk, b, &bars[SB_KV]);
    issue_q(0);
  }

  // sinks seed the max and the row sum (log2 domain)
  float ms = -1e30f;
  for (int j = 0; j < n_meta; ++j) ms = fmaxf(ms, meta[j] * kLog2e);
  float ls = 0.f;
  for (int j = 0; j < n_meta; ++j) ls += exp2f(meta[j] * kLog2e - ms);

  const CT* csb = ROPE ? cs + (size_t)b * cs_sb : nullptr;
  const CT* snb = ROPE ? sn + (size_t)b * cs_sb : nullptr;
  auto rotate_q = [&](int g) {
    const size_t hrow = ((size_t)b * H + hk * grp + g) * L;
    rotate_rows<0, kQ, CT>(smem + SM::qh, smem + SM::ql, q0, L, csb, snb, cs_sl, 0,
                           qh_out ? qh_out + hrow * kDh : nullptr,
                           qh_out ? ql_out + hrow * kDh : nullptr);
  };
  tc::mbar_wait(&bars[SB_KV], 0, 80);
  if (ROPE) {
    const size_t kvb = ((size_t)b * Hkv + hk) * L * kDh;
    bf16* gh = kh_out ? kh_out + kvb : nullptr;
    bf16* gl = kh_out ? kl_out + kvb : nullptr;
    rotate_rows<0, 128, CT>(smem + SM::kh, smem + SM::kl, k0, L, csb, snb, cs_sl, kNK - kQ, gh,
                            gl);
    rotate_rows<128, kNK - 128, CT>(smem + SM::kh, smem + SM::kl, k0, L, csb, snb, cs_sl,
                                    kNK - kQ, gh, gl);
  }
  tc::mbar_wait(&bars[SB_Q], 0, 81);
  if (ROPE) rotate_q(0);
  tc::fence_proxy_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  if (tid == 0) issue_s();

  const int r = 32 * qd + lane, i = q0 + r;
  const uint32_t trow = tmem + ((uint32_t)(32 * qd) << 16);
  const int cw = 32 * qd + 48 * hf;  // first score column of this thread's half window
  for (int g = 0; g < grp; ++g) {
    const uint32_t ph = (uint32_t)g & 1u;
    const bool next = g + 1 < grp;
    tc::mbar_wait(&bars[SB_S], ph, 82);
    tc::tc_fence_after();
    if (tid == 0 && next) issue_q(g + 1);  // the scores have read the query tiles

    // the window of row i is keys t in (i - W, i], t >= 0: columns t - k0 in
    // [32 qd + 1, 32 qd + 95]; this thread takes 48 of them
    float s[3][16];
#pragma unroll
    for (int k = 0; k < 3; ++k) tc::tmem_ld16(trow + kTmS + cw + 16 * k, s[k]);
    tc::tmem_wait_ld();
    float mx = ms;
#pragma unroll
    for (int k = 0; k < 3; ++k)
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int t = k0 + cw + 16 * k + u;
        const bool ok = t <= i && t > i - W && t >= 0;
        const float x = ok ? s[k][u] * scale_log2 : -INFINITY;
        s[k][u] = x;
        mx = fmaxf(mx, x);
      }
    red[hf * kQ + r] = mx;
    __syncthreads();
    mx = fmaxf(mx, red[(1 - hf) * kQ + r]);
    float l = 0.f;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      uint32_t phi[8], plo[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float p0 = exp2f(s[k][2 * j] - mx), p1 = exp2f(s[k][2 * j + 1] - mx);
        l += p0 + p1;
        const uint32_t hpk = pack_bf16(p0, p1);
        phi[j] = hpk;
        plo[j] = pack_bf16(p0 - bf16_lo(hpk), p1 - bf16_hi(hpk));
      }
      tc::tmem_st8(trow + kTmPh + cw / 2 + 8 * k, phi);
      tc::tmem_st8(trow + kTmPl + cw / 2 + 8 * k, plo);
    }
    {  // p is zero outside the window: packed columns [0, 16 qd) and [16 qd + 48, 96)
      uint32_t zero[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) zero[j] = 0u;
      const int z0 = hf ? 16 * qd + 48 : 0, z1 = hf ? kNK / 2 : 16 * qd;
#pragma unroll 1
      for (int c = z0; c < z1; c += 8) {
        tc::tmem_st8(trow + kTmPh + c, zero);
        tc::tmem_st8(trow + kTmPl + c, zero);
      }
    }
    red[2 * kQ + hf * kQ + r] = l;  // row sums, read after the P V sync
    tc::tmem_wait_st();
    tc::tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc::tc_fence_after();
      constexpr uint32_t id_o = tc::idesc_bf16(kQ, kDh, 0, 1);  // p (TMEM) x V (MN-major)
      const uint32_t va = smem_u32(smem + SM::v);
#pragma unroll
      for (int j = 0; j < kNK / 16; ++j)
        tc::mma_ts(tmem + kTmO, tmem + kTmPh + 8 * j, tc::sdesc(va + 2048 * j, kTileK, 1024), id_o,
                   j > 0);
#pragma unroll
      for (int j = 0; j < kNK / 16; ++j)
        tc::mma_ts(tmem + kTmO, tmem + kTmPl + 8 * j, tc::sdesc(va + 2048 * j, kTileK, 1024), id_o,
                   1u);
      tc::mma_commit(&bars[SB_O]);
    }
    const float lrow = ls * exp2f(ms - mx) + red[2 * kQ + r] + red[3 * kQ + r];
    // while P V runs: the next head's query tiles
    if (next) {
      tc::mbar_wait(&bars[SB_Q], ph ^ 1u, 81);
      if (ROPE) rotate_q(g + 1);
      tc::fence_proxy_async_smem();
    }
    tc::mbar_wait(&bars[SB_O], ph, 83);
    tc::tc_fence_after();
    tc::tc_fence_before();
    __syncthreads();  // P V done (s / p columns free), the next query tiles written
    if (tid == 0 && next) issue_s();  // runs while the warps write this head's output

    const float inv = 1.f / lrow;
    const size_t row = ((size_t)b * H + hk * grp + g) * L + i;
    float o[32];
    tc::tmem_ld32(trow + kTmO + 32 * hf, o);
    tc::tmem_wait_ld();
    if (i < L) {
      bf16* yr = y + row * kDh + 32 * hf;
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint4 w;
        w.x = pack_bf16(o[8 * q4] * inv, o[8 * q4 + 1] * inv);
        w.y = pack_bf16(o[8 * q4 + 2] * inv, o[8 * q4 + 3] * inv);
        w.z = pack_bf16(o[8 * q4 + 4] * inv, o[8 * q4 + 5] * inv);
        w.w = pack_bf16(o[8 * q4 + 6] * inv, o[8 * q4 + 7] * inv);
        reinterpret_cast<uint4*>(yr)[q4] = w;
      }
      if (y32) {
        float4* d32 = reinterpret_cast<float4*>(y32 + row * kDh + 32 * hf);
#pragma unroll
        for (int q4 = 0; q4 < 8; ++q4)
          d32[q4] = make_float4(o[4 * q4] * inv, o[4 * q4 + 1] * inv, o[4 * q4 + 2] * inv,
                                o[4 * q4 + 3] * inv);
      }
      if (lse && hf == 0) lse[row] = mx * kLn2f + logf(lrow);
    }
    tc::tc_fence_before();
    __syncthreads();  // o and the row-sum slots are free for the next head
  }
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTmCols);
  }
}

// bf16 [B, Hx, L, 64] at element strides (sb, sh, sl, 1) as a 4-D map
// {64, L, Hx, B}, box {64, box_rows, 1, 1}, 128-byte swizzle, zero fill
// outside the tensor.
bool make_tc_map(CUtensorMap* m, const void* ptr, int L, int Hx, int B, long long sb,
                 long long sh, long long sl, int box_rows) {
  tc::EncodeTiledFn fn = tc::encode_tiled_fn();
  if (!fn || !ptr) return false;
  if (Hx == 1) sh = (long long)L * sl;  // strides of size-1 dims are not used; keep them legal
  if (B == 1) sb = (long long)Hx * sh;
  if (!aligned16(ptr) || sl <= 0 || sh <= 0 || sb <= 0 || (sl * 2) % 16 || (sh * 2) % 16 ||
      (sb * 2) % 16)
    return false;
  cuuint64_t dims[4] = {(cuuint64_t)kDh, (cuuint64_t)L, (cuuint64_t)Hx, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)(sl * 2), (cuuint64_t)(sh * 2), (cuuint64_t)(sb * 2)};
  cuuint32_t box[4] = {(cuuint32_t)kDh, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

std::atomic<int> g_swa_tc{1};

template <bool ROPE, bool SPLIT, typename CT>
int launch_swa_tc(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                  const CUtensorMap& mql, const CUtensorMap& mkl, const void* cs, const void* sn,
                  long long cs_sb, long long cs_sl, const float* meta, int n_meta, int W, int B,
                  int H, int Hkv, int L, bf16* y, const SwaSaved& sv, bf16* qh_out,
                  bf16* ql_out, bf16* kh_out, bf16* kl_out, cudaStream_t st) {
  static bool done[64] = {false};
  {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !done[dev]) {
      cudaError_t e = cudaFuncSetAttribute(swa_fwd_tc_kernel<ROPE, SPLIT, CT>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)SwaTcSmem::bytes);
      if (e != cudaSuccess) {
        set_error(std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
        return LZ_ERR_CUDA;
      }
      done[dev] = true;
    }
  }
  const int nqb = ceil_div(L, kQ);
  const float scale_log2 = kLog2e / sqrtf((float)kDh);
  swa_fwd_tc_kernel<ROPE, SPLIT, CT>
      <<<(unsigned)((long long)B * Hkv * nqb), kThreads, SwaTcSmem::bytes, st>>>(
          mq, mk, mv, mql, mkl, static_cast<const CT*>(cs), static_cast<const CT*>(sn), cs_sb,
          cs_sl, meta, n_meta, W, scale_log2, H, H / Hkv, L, nqb, y, sv.lse, sv.y32, qh_out,
          ql_out, kh_out, kl_out);
  count_launches(1);
  return check_launch("swa_fwd_tc_kernel");
}

}  // namespace

bool swa_tc_enabled() { return g_swa_tc.load(std::memory_order_relaxed) != 0; }
int swa_set_tc(int on) { return g_swa_tc.exchange(on ? 1 : 0); }

int swa_rope_fwd_tc(const SwaRopeArgs& a, const SwaSaved& sv, cudaStream_t st) {
  if (!swa_tc_enabled() || a.D != kDh || a.x_dtype != LZ_DTYPE_BF16 || a.window < 1 ||
      a.window > kNK - kQ)
    return LZ_ERR_UNSUPPORTED;
  const long long ces = a.cs_dtype == LZ_DTYPE_F32 ? 4 : 2;
  if (!aligned16(a.cos) || !aligned16(a.sin) || (a.cs_sl * ces) % 16 || (a.cs_sb * ces) % 16)
    return LZ_ERR_UNSUPPORTED;  // the rotation reads cos / sin rows with 16-byte loads
  if (a.q_hi && (!aligned16(a.q_hi) || !aligned16(a.q_lo) || !aligned16(a.k_hi) ||
                 !aligned16(a.k_lo)))
    return LZ_ERR_UNSUPPORTED;
  if (!aligned16(a.y) || (sv.y32 && !aligned16(sv.y32))) return LZ_ERR_UNSUPPORTED;
  CUtensorMap mq, mk, mv;
  if (!make_tc_map(&mq, a.q, a.L, a.H, a.B, a.q_sb, a.q_sh, a.q_sl, kQ) ||
      !make_tc_map(&mk, a.k, a.L, a.Hkv, a.B, a.k_sb, a.k_sh, a.k_sl, kNK) ||
      !make_tc_map(&mv, a.v, a.L, a.Hkv, a.B, a.v_sb, a.v_sh, a.v_sl, kNK))
    return LZ_ERR_UNSUPPORTED;
  if (a.cs_dtype == LZ_DTYPE_F32)
    return launch_swa_tc<true, true, float>(mq, mk, mv, mq, mk, a.cos, a.sin, a.cs_sb, a.cs_sl,
                                            a.meta, a.n_meta, a.window, a.B, a.H, a.Hkv, a.L,
                                            a.y, sv, a.q_hi, a.q_lo, a.k_hi, a.k_lo, st);
  return launch_swa_tc<true, true, bf16>(mq, mk, mv, mq, mk, a.cos, a.sin, a.cs_sb, a.cs_sl,
                                         a.meta, a.n_meta, a.window, a.B, a.H, a.Hkv, a.L, a.y,
                                         sv, a.q_hi, a.q_lo, a.k_hi, a.k_lo, st);
}

int swa_fwd_tc(const bf16* q, const bf16* k, const bf16* v, const bf16* ql, const bf16* kl,
               const float* meta, int n_meta, int W, bf16* y, const SwaSaved& sv, int B, int H,
               int Hkv, int L, int D, cudaStream_t st) {
  if (!swa_tc_enabled() || D != kDh || W < 1 || W > kNK - kQ) return LZ_ERR_UNSUPPORTED;
  if (!aligned16(y) || (sv.y32 && !aligned16(sv.y32))) return LZ_ERR_UNSUPPORTED;
  const long long sl = kDh, sh = (long long)L * kDh;
  CUtensorMap mq, mk, mv, mql, mkl;
  if (!make_tc_map(&mq, q, L, H, B, H * sh, sh, sl, kQ) ||
      !make_tc_map(&mk, k, L, Hkv, B, Hkv * sh, sh, sl, kNK) ||
      !make_tc_map(&mv, v, L, Hkv, B, Hkv * sh, sh, sl, kNK))
    return LZ_ERR_UNSUPPORTED;
  if (ql) {
    if (!make_tc_map(&mql, ql, L, H, B, H * sh, sh, sl, kQ) ||
        !make_tc_map(&mkl, kl, L, Hkv, B, Hkv * sh, sh, sl, kNK))
      return LZ_ERR_UNSUPPORTED;
    return launch_swa_tc<false, true, float>(mq, mk, mv, mql, mkl, nullptr, nullptr, 0, 0, meta,
                                             n_meta, W, B, H, Hkv, L, y, sv, nullptr, nullptr,
                                             nullptr, nullptr, st);
  }
  return launch_swa_tc<false, false, float>(mq, mk, mv, mq, mk, nullptr, nullptr, 0, 0, meta,
                                            n_meta, W, B, H, Hkv, L, y, sv, nullptr, nullptr,
                                            nullptr, nullptr, st);
}

int swa_tc_timeout_flag(unsigned int* out) { return tc::read_timeout_flag_here(out); }

}  // namespace lz

extern "C" int lz_swa_set_tc(int on) { return lz::swa_set_tc(on); }
