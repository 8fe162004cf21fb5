// Sliding-window attention on the 5th-generation tensor cores (tcgen05 + TMEM
// + TMA) for head dim 64 and windows of at most 64 keys, the Lizard layer's
// shape (reference: src/lizard_attention.py:34-44 and the Triton kernels
// src/kernels/swa.py:19-133): the forward (below), and the dq and dk / dv
// kernels of the backward (further down; delta and the sink gradient stay in
// swa.cu). Windows of 65 to 128 keys (the reference's training configs use
// 128) have their own wider forward, dq and dk / dv kernels near the end.
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
#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "rope_math.cuh"
#include "swa_layout.h"
#include "tc.cuh"

namespace lz {
namespace {

constexpr int kQ = 128;   // query rows per CTA (= TMEM lanes)
constexpr int kThreads = 256;  // the row warps (two per TMEM lane quadrant)
constexpr int kCtaThreads = kThreads + 32;  // + the TMA / MMA warp of the backward kernels
// named barriers of the backward: row warps -> MMA warp (operands in TMEM), row warps
enum { NB_PREADY = 2, NB_ROWS = 3 };
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
        // x - mx <= 0 (or -inf outside the window): the hardware 2^x, error ~2^-22
        const float p0 = tc::ex2(s[k][2 * j] - mx), p1 = tc::ex2(s[k][2 * j + 1] - mx);
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

// ------------------------------------------------------------ backward: dk, dv
// One CTA of 9 warps per 128 key rows [k0, k0 + 128) of one (batch row,
// key/value head); it walks the query heads of the group, each through the 192
// query rows [k0, k0 + 192) that can see those keys (W <= 64), with the query /
// dy tiles of the next head in a second shared-memory stage:
//   warp 8   : TMA; s^T = k q^T (hi / lo terms as the forward), dp^T = v dy^T
//              -> TMEM [128 x 192] each; then dv += p^T dy and dk += ds^T q
//              with p^T, ds^T from TMEM -> TMEM [128 x 64] each, summed over
//              the group's heads
//   8 warps  : key row t = TMEM lane t, the 96 query columns that can see it
//              split between the two warps of the lane quadrant:
//              p = exp(s scale - lse_i), ds = p (dp - delta_i), written as bf16
//              over s^T once every score column of the CTA has been read
// The arithmetic is that of swa_bwd_dkv_kernel (bf16 p and ds, q_hi in dk;
// the reference's Triton backward, src/kernels/swa.py:97-133). 195 KB of
// shared memory and all 512 TMEM columns: one CTA per SM.
constexpr int kBK = 128;  // key rows per CTA
constexpr int kBQ = 192;  // query rows per head: [k0, k0 + 192)
struct DkvTcSmem {
  static constexpr size_t kh = 0, kl = kh + kBK * 128, v = kl + kBK * 128, st = v + kBK * 128;
  static constexpr size_t sq = 0, sql = kBQ * 128, sdy = 2 * kBQ * 128, sbytes = 3 * kBQ * 128;
  static constexpr size_t rows = st + 2 * sbytes;  // [2 stages][lse | delta][192] fp32
  static constexpr size_t bars = rows + 2 * 2 * kBQ * 4, slot = bars + 64, bytes = slot + 16;
};
// TMEM: s^T [0, 192) with p^T (bf16 pairs, [0, 96)) and ds^T ([96, 192)) over
// it; dp^T [192, 384); dv [384, 448); dk [448, 512)
constexpr uint32_t kTbS = 0, kTbP = 0, kTbDs = 96, kTbDp = 192, kTbDv = 384, kTbDk = 448,
                   kTbCols = 512;
enum { DB_KV = 0, DB_Q0, DB_Q1, DB_SD, DB_PD };

// 32 gradient values of a row, scaled, to fp32 or bf16 (16-byte stores)
__device__ __forceinline__ void store_grad32(void* out, size_t at, const float (&o)[32], float mul,
                                             int gdt) {
  if (gdt == LZ_DTYPE_BF16) {
    uint4* d16 = reinterpret_cast<uint4*>(static_cast<bf16*>(out) + at);
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4)
      d16[q4] = make_uint4(pack_bf16(o[8 * q4] * mul, o[8 * q4 + 1] * mul),
                           pack_bf16(o[8 * q4 + 2] * mul, o[8 * q4 + 3] * mul),
                           pack_bf16(o[8 * q4 + 4] * mul, o[8 * q4 + 5] * mul),
                           pack_bf16(o[8 * q4 + 6] * mul, o[8 * q4 + 7] * mul));
  } else {
    float4* d32 = reinterpret_cast<float4*>(static_cast<float*>(out) + at);
#pragma unroll
    for (int q4 = 0; q4 < 8; ++q4)
      d32[q4] = make_float4(o[4 * q4] * mul, o[4 * q4 + 1] * mul, o[4 * q4 + 2] * mul,
                            o[4 * q4 + 3] * mul);
  }
}

template <bool SPLIT>
__global__ void __launch_bounds__(kCtaThreads, 1)
swa_bwd_dkv_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tql,
                      const __grid_constant__ CUtensorMap tdy, const __grid_constant__ CUtensorMap tk,
                      const __grid_constant__ CUtensorMap tkl, const __grid_constant__ CUtensorMap tv,
                      const float* __restrict__ lse, const float* __restrict__ delta, int W,
                      float scale, int H, int grp, int L, int nkt, void* __restrict__ dk,
                      void* __restrict__ dv, int gdt) {
  using SM = DkvTcSmem;
  extern __shared__ __align__(1024) unsigned char smem[];
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) atomicExch(&tc::g_timeout_flag, 0x80000000u | 88u);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::bars);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + SM::slot);
  float* rows = reinterpret_cast<float*>(smem + SM::rows);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kt = blockIdx.x % nkt, bk = blockIdx.x / nkt;
  const int Hkv = H / grp, b = bk / Hkv, hk = bk - b * Hkv;
  const int k0 = kt * kBK;
  constexpr uint32_t kTileK = kBK * 128, kTileQ = kBQ * 128;

  if (tid == 0) {
#pragma unroll
    for (int j = 0; j < 5; ++j) tc::mbar_init(&bars[j], 1);
    tc::fence_mbar_init();
  }
  if (warp == 8) {
    tc::tmem_alloc(tslot, kTbCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 8) {
    const bool issuer = lane == 0;
    auto load_stage = [&](int g) {  // query / dy rows of head hk * grp + g into stage g & 1
      const int h = hk * grp + g;
      unsigned char* st = smem + SM::st + (g & 1) * SM::sbytes;
      uint64_t* bar = &bars[DB_Q0 + (g & 1)];
      tc::mbar_expect_tx(bar, (SPLIT ? 3 : 2) * kTileQ);
      tc::tma_load_4d(st + SM::sq, &tq, 0, k0, h, b, bar);
      if (SPLIT) tc::tma_load_4d(st + SM::sql, &tql, 0, k0, h, b, bar);
      tc::tma_load_4d(st + SM::sdy, &tdy, 0, k0, h, b, bar);
    };
    if (issuer) {
      tc::mbar_expect_tx(&bars[DB_KV], (SPLIT ? 3 : 2) * kTileK);
      tc::tma_load_4d(smem + SM::kh, &tk, 0, k0, hk, b, &bars[DB_KV]);
      if (SPLIT) tc::tma_load_4d(smem + SM::kl, &tkl, 0, k0, hk, b, &bars[DB_KV]);
      tc::tma_load_4d(smem + SM::v, &tv, 0, k0, hk, b, &bars[DB_KV]);
      load_stage(0);
      if (grp > 1) load_stage(1);
      tc::mbar_wait(&bars[DB_KV], 0, 70);
    }
    __syncwarp();
    for (int g = 0; g < grp; ++g) {
      const uint32_t ph = (uint32_t)g & 1u;
      unsigned char* st = smem + SM::st + (g & 1) * SM::sbytes;
      if (issuer) {
        tc::mbar_wait(&bars[DB_Q0 + (g & 1)], (uint32_t)(g >> 1) & 1u, 71);
        if (g > 0) tc::mbar_wait(&bars[DB_PD], ph ^ 1u, 72);  // p / ds of head g - 1 read
        tc::tc_fence_after();
        constexpr uint32_t id_s = tc::idesc_bf16(kBK, kBQ, 0, 0);  // K-major x K-major
        const uint32_t kh = smem_u32(smem + SM::kh), kl = smem_u32(smem + SM::kl),
                       va = smem_u32(smem + SM::v), qh = smem_u32(st + SM::sq),
                       ql = smem_u32(st + SM::sql), dya = smem_u32(st + SM::sdy);
#pragma unroll
        for (int j = 0; j < kDh / 16; ++j)
          tc::mma_ss(tmem + kTbS, tc::sdesc(kh + 32 * j, 16, 1024),
                     tc::sdesc(qh + 32 * j, 16, 1024), id_s, j > 0);
        if (SPLIT) {
#pragma unroll
          for (int j = 0; j < kDh / 16; ++j)
            tc::mma_ss(tmem + kTbS, tc::sdesc(kh + 32 * j, 16, 1024),
                       tc::sdesc(ql + 32 * j, 16, 1024), id_s, 1u);
#pragma unroll
          for (int j = 0; j < kDh / 16; ++j)
            tc::mma_ss(tmem + kTbS, tc::sdesc(kl + 32 * j, 16, 1024),
                       tc::sdesc(qh + 32 * j, 16, 1024), id_s, 1u);
        }
#pragma unroll
        for (int j = 0; j < kDh / 16; ++j)
          tc::mma_ss(tmem + kTbDp, tc::sdesc(va + 32 * j, 16, 1024),
                     tc::sdesc(dya + 32 * j, 16, 1024), id_s, j > 0);
        tc::mma_commit(&bars[DB_SD]);
      }
      __syncwarp();
      tc::named_bar_sync(NB_PREADY, kCtaThreads);  // p^T and ds^T in TMEM
      if (issuer) {
        tc::tc_fence_after();
        constexpr uint32_t id_o = tc::idesc_bf16(kBK, kDh, 0, 1);  // TMEM x MN-major
        const uint32_t qh = smem_u32(st + SM::sq), dya = smem_u32(st + SM::sdy);
#pragma unroll
        for (int j = 0; j < kBQ / 16; ++j)
          tc::mma_ts(tmem + kTbDv, tmem + kTbP + 8 * j, tc::sdesc(dya + 2048 * j, kTileQ, 1024),
                     id_o, (g > 0 || j > 0) ? 1u : 0u);
#pragma unroll
        for (int j = 0; j < kBQ / 16; ++j)
          tc::mma_ts(tmem + kTbDk, tmem + kTbDs + 8 * j, tc::sdesc(qh + 2048 * j, kTileQ, 1024),
                     id_o, (g > 0 || j > 0) ? 1u : 0u);
        tc::mma_commit(&bars[DB_PD]);
        if (g + 2 < grp) {
          tc::mbar_wait(&bars[DB_PD], ph, 73);  // stage g & 1 read by every MMA of head g
          load_stage(g + 2);
        }
      }
      __syncwarp();
    }
  } else {
    const int qd = warp & 3, hf = warp >> 2;
    const int r = 32 * qd + lane, t = k0 + r;  // this thread's key row
    const uint32_t trow = tmem + ((uint32_t)(32 * qd) << 16);
    const int cw = 32 * qd + 48 * hf;  // first query column of this thread's half window
    for (int g = 0; g < grp; ++g) {
      const uint32_t ph = (uint32_t)g & 1u;
      const size_t bh = (size_t)b * H + hk * grp + g;
      float* rl = rows + (g & 1) * 2 * kBQ;  // lse, then delta, of query rows k0 + c
      for (int c = tid; c < kBQ; c += kThreads) {
        const int i = k0 + c;
        rl[c] = i < L ? lse[bh * L + i] : 0.f;
        rl[kBQ + c] = i < L ? delta[bh * L + i] : 0.f;
      }
      tc::named_bar_sync(NB_ROWS, kThreads);
      tc::mbar_wait(&bars[DB_SD], ph, 74);
      tc::tc_fence_after();
      // p and ds of the 48 columns in registers (bf16 pairs) before any store:
      // the stores land on score columns that this thread and its partner warp
      // (the other half of the lane quadrant) read
      uint32_t pk[3][8], dk8[3][8];
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        float sv[16], dpv[16];
        tc::tmem_ld16(trow + kTbS + cw + 16 * k, sv);
        tc::tmem_ld16(trow + kTbDp + cw + 16 * k, dpv);
        tc::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float p2[2], d2[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int c = cw + 16 * k + 2 * j + e, i = k0 + c;
            const bool ok = i >= t && i < t + W && i < L && t < L;
            const float p = ok ? __expf(sv[2 * j + e] * scale - rl[c]) : 0.f;
            p2[e] = p;
            d2[e] = p * (dpv[2 * j + e] - rl[kBQ + c]);
          }
          pk[k][j] = pack_bf16(p2[0], p2[1]);
          dk8[k][j] = pack_bf16(d2[0], d2[1]);
        }
      }
      tc::tc_fence_before();
      tc::named_bar_sync(NB_ROWS, kThreads);  // every score column of the CTA read
      tc::tc_fence_after();
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        tc::tmem_st8(trow + kTbP + cw / 2 + 8 * k, pk[k]);
        tc::tmem_st8(trow + kTbDs + cw / 2 + 8 * k, dk8[k]);
      }
      {  // zero outside the window: packed columns [0, 16 qd) and [16 qd + 48, 96)
        uint32_t zero[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) zero[j] = 0u;
        const int z0 = hf ? 16 * qd + 48 : 0, z1 = hf ? kBQ / 2 : 16 * qd;
#pragma unroll 1
        for (int c = z0; c < z1; c += 8) {
          tc::tmem_st8(trow + kTbP + c, zero);
          tc::tmem_st8(trow + kTbDs + c, zero);
        }
      }
      tc::tmem_wait_st();
      tc::tc_fence_before();
      tc::named_bar_arrive(NB_PREADY, kCtaThreads);
    }
    // dv (warps of half 0) and dk (half 1) of this key row, summed over the group
    tc::mbar_wait(&bars[DB_PD], (uint32_t)(grp - 1) & 1u, 75);
    tc::tc_fence_after();
    const size_t orow = ((size_t)bk * L + t) * kDh;
#pragma unroll 1
    for (int db = 0; db < 2; ++db) {
      float o[32];
      tc::tmem_ld32(trow + (hf ? kTbDk : kTbDv) + 32 * db, o);
      tc::tmem_wait_ld();
      if (t < L) store_grad32(hf ? dk : dv, orow + 32 * db, o, hf ? scale : 1.f, gdt);
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTbCols);
  }
}

// The same dk / dv for bf16 operands (no residual tiles), persistent: one CTA
// per SM walks its tiles (b, key/value head, key tile) and, in each, the
// group's query heads as a flat sequence of items. Two key / value buffers
// and two query / dy stages let the next tile's and the next items' tiles
// load while this one computes, and the next tile's scores run while the row
// warps write this tile's dk / dv (the accumulators are overwritten only
// after that write-out). 167 KB of shared memory, 512 TMEM columns.
struct DkvPersistSmem {
  static constexpr size_t KVB = 2 * kBK * 128, QB = 2 * kBQ * 128;  // k + v; q + dy
  static constexpr size_t kv = 0, qs = 2 * KVB, rows = qs + 2 * QB;
  static constexpr size_t bars = rows + 2 * 2 * kBQ * 4, slot = bars + 64, bytes = slot + 16;
};
enum { PB_KV0 = 0, PB_KV1, PB_Q0, PB_Q1, PB_SD, PB_PD, PB_EPI, PB_N };

__global__ void __launch_bounds__(kCtaThreads, 1)
swa_bwd_dkv_tc_persist_kernel(const __grid_constant__ CUtensorMap tq,
                              const __grid_constant__ CUtensorMap tdy,
                              const __grid_constant__ CUtensorMap tk,
                              const __grid_constant__ CUtensorMap tv,
                              const float* __restrict__ lse, const float* __restrict__ delta,
                              int W, float scale, int H, int grp, int L, int nkt, int ntiles,
                              void* __restrict__ dk, void* __restrict__ dv, int gdt) {
  using SM = DkvPersistSmem;
  extern __shared__ __align__(1024) unsigned char smem[];
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) atomicExch(&tc::g_timeout_flag, 0x80000000u | 86u);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::bars);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + SM::slot);
  float* rows = reinterpret_cast<float*>(smem + SM::rows);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int Hkv = H / grp;
  constexpr uint32_t kTileK = kBK * 128, kTileQ = kBQ * 128;
  // this CTA's tiles: blockIdx.x + kl gridDim.x, kl < nloc; items (kl, g), w = kl grp + g
  const int nloc = (int)((ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x);
  const int nitems = nloc * grp;
  auto tile = [&](int kl, int& b, int& hk, int& k0) {
    const int tt = (int)blockIdx.x + kl * (int)gridDim.x;
    const int kt = tt % nkt, bk = tt / nkt;
    b = bk / Hkv, hk = bk - b * Hkv, k0 = kt * kBK;
  };

  if (tid == 0) {
#pragma unroll
    for (int j = 0; j < PB_N; ++j) tc::mbar_init(&bars[j], j == PB_EPI ? kThreads : 1);
    tc::fence_mbar_init();
  }
  if (warp == 8) {
    tc::tmem_alloc(tslot, kTbCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 8) {
    const bool issuer = lane == 0;
    auto load_kv = [&](int kl) {
      int b, hk, k0;
      tile(kl, b, hk, k0);
      unsigned char* buf = smem + SM::kv + (kl & 1) * SM::KVB;
      uint64_t* bar = &bars[PB_KV0 + (kl & 1)];
      tc::mbar_expect_tx(bar, 2 * kTileK);
      tc::tma_load_4d(buf, &tk, 0, k0, hk, b, bar);
      tc::tma_load_4d(buf + kTileK, &tv, 0, k0, hk, b, bar);
    };
    auto load_q = [&](int w) {
      int b, hk, k0;
      tile(w / grp, b, hk, k0);
      const int h = hk * grp + w % grp;
      unsigned char* st = smem + SM::qs + (w & 1) * SM::QB;
      uint64_t* bar = &bars[PB_Q0 + (w & 1)];
      tc::mbar_expect_tx(bar, 2 * kTileQ);
      tc::tma_load_4d(st, &tq, 0, k0, h, b, bar);
      tc::tma_load_4d(st + kTileQ, &tdy, 0, k0, h, b, bar);
    };
    if (issuer) {
      if (nloc > 0) load_kv(0);
      if (nloc > 1) load_kv(1);
      if (nitems > 0) load_q(0);
      if (nitems > 1) load_q(1);
    }
    __syncwarp();
    for (int w = 0; w < nitems; ++w) {
      const int kl = w / grp, g = w - kl * grp;
      const unsigned char* kvb = smem + SM::kv + (kl & 1) * SM::KVB;
      const unsigned char* st = smem + SM::qs + (w & 1) * SM::QB;
      if (issuer) {
        if (g == 0) tc::mbar_wait(&bars[PB_KV0 + (kl & 1)], (uint32_t)(kl >> 1) & 1u, 77);
        tc::mbar_wait(&bars[PB_Q0 + (w & 1)], (uint32_t)(w >> 1) & 1u, 78);
        if (w > 0) tc::mbar_wait(&bars[PB_PD], (uint32_t)(w - 1) & 1u, 79);  // p / ds read
        tc::tc_fence_after();
        constexpr uint32_t id_s = tc::idesc_bf16(kBK, kBQ, 0, 0);  // K-major x K-major
        const uint32_t kh = smem_u32(kvb), va = kh + kTileK, qh = smem_u32(st),
                       dya = qh + kTileQ;
#pragma unroll
        for (int j = 0; j < kDh / 16; ++j)
          tc::mma_ss(tmem + kTbS, tc::sdesc(kh + 32 * j, 16, 1024),
                     tc::sdesc(qh + 32 * j, 16, 1024), id_s, j > 0);
#pragma unroll
        for (int j = 0; j < kDh / 16; ++j)
          tc::mma_ss(tmem + kTbDp, tc::sdesc(va + 32 * j, 16, 1024),
                     tc::sdesc(dya + 32 * j, 16, 1024), id_s, j > 0);
        tc::mma_commit(&bars[PB_SD]);
      }
      __syncwarp();
      tc::named_bar_sync(NB_PREADY, kCtaThreads);  // p^T and ds^T in TMEM
      if (issuer) {
        // a tile's first head overwrites the accumulators: the last tile's dk / dv
        // must have been written out
        if (g == 0 && kl > 0) tc::mbar_wait(&bars[PB_EPI], (uint32_t)(kl - 1) & 1u, 80);
        tc::tc_fence_after();
        constexpr uint32_t id_o = tc::idesc_bf16(kBK, kDh, 0, 1);  // TMEM x MN-major
        const uint32_t qh = smem_u32(st), dya = qh + kTileQ;
#pragma unroll
        for (int j = 0; j < kBQ / 16; ++j)
          tc::mma_ts(tmem + kTbDv, tmem + kTbP + 8 * j, tc::sdesc(dya + 2048 * j, kTileQ, 1024),
                     id_o, (g > 0 || j > 0) ? 1u : 0u);
#pragma unroll
        for (int j = 0; j < kBQ / 16; ++j)
          tc::mma_ts(tmem + kTbDk, tmem + kTbDs + 8 * j, tc::sdesc(qh + 2048 * j, kTileQ, 1024),
                     id_o, (g > 0 || j > 0) ? 1u : 0u);
        tc::mma_commit(&bars[PB_PD]);
        const bool refill_q = w + 2 < nitems, refill_kv = g == grp - 1 && kl + 2 < nloc;
        if (refill_q || refill_kv) {
          tc::mbar_wait(&bars[PB_PD], (uint32_t)w & 1u, 81);  // item w's tiles read
          if (refill_q) load_q(w + 2);
          if (refill_kv) load_kv(kl + 2);
        }
      }
      __syncwarp();
    }
  } else {
    const int qd = warp & 3, hf = warp >> 2;
    const int r = 32 * qd + lane;
    const uint32_t trow = tmem + ((uint32_t)(32 * qd) << 16);
    const int cw = 32 * qd + 48 * hf;  // first query column of this thread's half window
    const float scale_log2 = scale * kLog2e;
    static_assert(kBQ <= kThreads, "one query row's lse / delta per row thread");
    // thread tid < kBQ loads lse and delta of query row k0 + tid of item w2,
    // one item ahead
    auto row_stats = [&](int w2, float& a, float& d) {
      const int kl2 = w2 / grp, g2 = w2 - kl2 * grp;
      int b2, hk2, k02;
      tile(kl2, b2, hk2, k02);
      const size_t bh2 = (size_t)b2 * H + hk2 * grp + g2;
      const int i = k02 + tid;
      a = tid < kBQ && i < L ? lse[bh2 * L + i] : 0.f;
      d = tid < kBQ && i < L ? delta[bh2 * L + i] : 0.f;
    };
    float nl = 0.f, nd = 0.f;
    if (nitems > 0) row_stats(0, nl, nd);
    for (int w = 0; w < nitems; ++w) {
      const int kl = w / grp, g = w - kl * grp;
      int b, hk, k0;
      tile(kl, b, hk, k0);
      const int t = k0 + r;  // this thread's key row
      float* rl = rows + (w & 1) * 2 * kBQ;  // lse, then delta, of query rows k0 + c
      if (tid < kBQ) {
        rl[tid] = nl * kLog2e;  // lse in base 2
        rl[kBQ + tid] = nd;
      }
      tc::named_bar_sync(NB_ROWS, kThreads);
      if (w + 1 < nitems) row_stats(w + 1, nl, nd);
      tc::mbar_wait(&bars[PB_SD], (uint32_t)w & 1u, 82);
      tc::tc_fence_after();
      uint32_t pk[3][8], dk8[3][8];
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        float sv[16], dpv[16];
        tc::tmem_ld16(trow + kTbS + cw + 16 * k, sv);
        tc::tmem_ld16(trow + kTbDp + cw + 16 * k, dpv);
        tc::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float p2[2], d2[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int c = cw + 16 * k + 2 * j + e, i = k0 + c;
            const bool ok = i >= t && i < t + W && i < L && t < L;
            const float p = ok ? tc::ex2(sv[2 * j + e] * scale_log2 - rl[c]) : 0.f;
            p2[e] = p;
            d2[e] = p * (dpv[2 * j + e] - rl[kBQ + c]);
          }
          pk[k][j] = pack_bf16(p2[0], p2[1]);
          dk8[k][j] = pack_bf16(d2[0], d2[1]);
        }
      }
      tc::tc_fence_before();
      tc::named_bar_sync(NB_ROWS, kThreads);  // every score column of the CTA read
      tc::tc_fence_after();
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        tc::tmem_st8(trow + kTbP + cw / 2 + 8 * k, pk[k]);
        tc::tmem_st8(trow + kTbDs + cw / 2 + 8 * k, dk8[k]);
      }
      {  // zero outside the window: packed columns [0, 16 qd) and [16 qd + 48, 96)
        uint32_t zero[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) zero[j] = 0u;
        const int z0 = hf ? 16 * qd + 48 : 0, z1 = hf ? kBQ / 2 : 16 * qd;
#pragma unroll 1
        for (int c = z0; c < z1; c += 8) {
          tc::tmem_st8(trow + kTbP + c, zero);
          tc::tmem_st8(trow + kTbDs + c, zero);
        }
      }
      tc::tmem_wait_st();
      tc::tc_fence_before();
      tc::named_bar_arrive(NB_PREADY, kCtaThreads);
      if (g == grp - 1) {  // the tile's dv (half 0) and dk (half 1), summed over the group
        tc::mbar_wait(&bars[PB_PD], (uint32_t)w & 1u, 83);
        tc::tc_fence_after();
        const size_t orow = (((size_t)b * Hkv + hk) * L + t) * kDh;
#pragma unroll 1
        for (int db = 0; db < 2; ++db) {
          float o[32];
          tc::tmem_ld32(trow + (hf ? kTbDk : kTbDv) + 32 * db, o);
          tc::tmem_wait_ld();
          if (t < L) store_grad32(hf ? dk : dv, orow + 32 * db, o, hf ? scale : 1.f, gdt);
        }
        tc::tc_fence_before();
        tc::mbar_arrive(&bars[PB_EPI]);
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTbCols);
  }
}

// ------------------------------------------------------------ backward: dq
// One CTA of 9 warps per 128 query rows [q0, q0 + 128) of one (batch row,
// key/value head) and each query head of the group in turn; keys / values
// [q0 - 64, q0 + 128) as in the forward, taken in two halves of 96 keys:
//   warp 8   : TMA; per half, s = q k^T (hi / lo terms) and dp = dy v^T
//              -> TMEM [128 x 96] each; then dq += ds k_hi with ds from TMEM
//              -> TMEM [128 x 64]
//   8 warps  : query row i = TMEM lane i, the key columns of its window in
//              this half split between the two warps of the lane quadrant:
//              ds = exp(s scale - lse_i) (dp - delta_i) written as bf16 over s
//              once every score column has been read; then dq_i = scale
//              (ds k)_i to HBM
// The arithmetic is that of swa_bwd_dq_kernel (bf16 ds, k_hi; the reference's
// Triton backward, src/kernels/swa.py:62-95). The query / dy tiles of the next
// head load into a second stage. 256 TMEM columns; with bf16 operands (no
// residual tiles) 112 KB of shared memory, so two CTAs share an SM.
constexpr int kHalf = kNK / 2;  // keys per half
template <bool SPLIT>
struct DqTcSmem {
  static constexpr size_t KT = kNK * 128, QT = kQ * 128;
  static constexpr size_t kh = 0, kl = kh + KT, v = kl + (SPLIT ? KT : 0), st = v + KT;
  static constexpr size_t sq = 0, sql = QT, sdy = sql + (SPLIT ? QT : 0), sbytes = sdy + QT;
  static constexpr size_t bars = st + 2 * sbytes, slot = bars + 64, bytes = slot + 16;
};
// TMEM: s of a half [0, 96) with ds (bf16 pairs, [0, 48)) over it; dp [96, 192); dq [192, 256)
constexpr uint32_t kTqS = 0, kTqDs = 0, kTqDp = kHalf, kTqDq = 2 * kHalf, kTqCols = 256;
enum { QB_KV = 0, QB_Q0, QB_Q1, QB_SD, QB_HALF, QB_DQ };

template <bool SPLIT>
__global__ void __launch_bounds__(kCtaThreads, SPLIT ? 1 : 2)
swa_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tql,
                     const __grid_constant__ CUtensorMap tdy, const __grid_constant__ CUtensorMap tk,
                     const __grid_constant__ CUtensorMap tkl, const __grid_constant__ CUtensorMap tv,
                     const float* __restrict__ lse, const float* __restrict__ delta, int W,
                     float scale, int H, int grp, int L, int nqb, void* __restrict__ dq, int gdt) {
  using SM = DqTcSmem<SPLIT>;
  extern __shared__ __align__(1024) unsigned char smem[];
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) atomicExch(&tc::g_timeout_flag, 0x80000000u | 87u);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::bars);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + SM::slot);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qb = blockIdx.x % nqb, bk = blockIdx.x / nqb;
  const int Hkv = H / grp, b = bk / Hkv, hk = bk - b * Hkv;
  const int q0 = qb * kQ, k0 = q0 - (kNK - kQ);
  constexpr uint32_t kTileK = kNK * 128, kTileQ = kQ * 128;

  if (tid == 0) {
#pragma unroll
    for (int j = 0; j < 6; ++j) tc::mbar_init(&bars[j], 1);
    tc::fence_mbar_init();
  }
  if (warp == 8) {
    tc::tmem_alloc(tslot, kTqCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 8) {
    const bool issuer = lane == 0;
    auto load_stage = [&](int g) {  // query / dy rows of head hk * grp + g into stage g & 1
      const int h = hk * grp + g;
      unsigned char* st = smem + SM::st + (g & 1) * SM::sbytes;
      uint64_t* bar = &bars[QB_Q0 + (g & 1)];
      tc::mbar_expect_tx(bar, (SPLIT ? 3 : 2) * kTileQ);
      tc::tma_load_4d(st + SM::sq, &tq, 0, q0, h, b, bar);
      if (SPLIT) tc::tma_load_4d(st + SM::sql, &tql, 0, q0, h, b, bar);
      tc::tma_load_4d(st + SM::sdy, &tdy, 0, q0, h, b, bar);
    };
    if (issuer) {
      tc::mbar_expect_tx(&bars[QB_KV], (SPLIT ? 3 : 2) * kTileK);
      tc::tma_load_4d(smem + SM::kh, &tk, 0, k0, hk, b, &bars[QB_KV]);
      if (SPLIT) tc::tma_load_4d(smem + SM::kl, &tkl, 0, k0, hk, b, &bars[QB_KV]);
      tc::tma_load_4d(smem + SM::v, &tv, 0, k0, hk, b, &bars[QB_KV]);
      load_stage(0);
      if (grp > 1) load_stage(1);
      tc::mbar_wait(&bars[QB_KV], 0, 60);
    }
    __syncwarp();
    for (int g = 0; g < grp; ++g) {
      const uint32_t ph = (uint32_t)g & 1u;
      unsigned char* st = smem + SM::st + (g & 1) * SM::sbytes;
      const uint32_t kh = smem_u32(smem + SM::kh), kl = smem_u32(smem + SM::kl),
                     va = smem_u32(smem + SM::v), qh = smem_u32(st + SM::sq),
                     ql = smem_u32(st + SM::sql), dya = smem_u32(st + SM::sdy);
      for (int hv = 0; hv < 2; ++hv) {
        const uint32_t ko = (uint32_t)(hv * kHalf * 128);  // the half's first key row
        if (issuer) {
          if (hv == 0) {
            tc::mbar_wait(&bars[QB_Q0 + (g & 1)], (uint32_t)(g >> 1) & 1u, 61);
            if (g > 0) tc::mbar_wait(&bars[QB_DQ], ph ^ 1u, 62);  // head g - 1's MMAs done
          } else {
            tc::mbar_wait(&bars[QB_HALF], ph, 66);  // the first half's ds has been read
          }
          tc::tc_fence_after();
          constexpr uint32_t id_s = tc::idesc_bf16(kQ, kHalf, 0, 0);  // K-major x K-major
#pragma unroll
          for (int j = 0; j < kDh / 16; ++j)
            tc::mma_ss(tmem + kTqS, tc::sdesc(qh + 32 * j, 16, 1024),
                       tc::sdesc(kh + ko + 32 * j, 16, 1024), id_s, j > 0);
          if (SPLIT) {
#pragma unroll
            for (int j = 0; j < kDh / 16; ++j)
              tc::mma_ss(tmem + kTqS, tc::sdesc(qh + 32 * j, 16, 1024),
                         tc::sdesc(kl + ko + 32 * j, 16, 1024), id_s, 1u);
#pragma unroll
            for (int j = 0; j < kDh / 16; ++j)
              tc::mma_ss(tmem + kTqS, tc::sdesc(ql + 32 * j, 16, 1024),
                         tc::sdesc(kh + ko + 32 * j, 16, 1024), id_s, 1u);
          }
#pragma unroll
          for (int j = 0; j < kDh / 16; ++j)
            tc::mma_ss(tmem + kTqDp, tc::sdesc(dya + 32 * j, 16, 1024),
                       tc::sdesc(va + ko + 32 * j, 16, 1024), id_s, j > 0);
          tc::mma_commit(&bars[QB_SD]);
        }
        __syncwarp();
        tc::named_bar_sync(NB_PREADY, kCtaThreads);  // this half's ds in TMEM
        if (issuer) {
          tc::tc_fence_after();
          constexpr uint32_t id_o = tc::idesc_bf16(kQ, kDh, 0, 1);  // TMEM x MN-major
#pragma unroll
          for (int j = 0; j < kHalf / 16; ++j)
            tc::mma_ts(tmem + kTqDq, tmem + kTqDs + 8 * j,
                       tc::sdesc(kh + ko + 2048 * j, kTileK, 1024), id_o,
                       (hv > 0 || j > 0) ? 1u : 0u);
          tc::mma_commit(&bars[hv == 0 ? QB_HALF : QB_DQ]);
          if (hv == 1 && g + 2 < grp) {
            tc::mbar_wait(&bars[QB_DQ], ph, 63);  // stage g & 1 read by every MMA of head g
            load_stage(g + 2);
          }
        }
        __syncwarp();
      }
    }
  } else {
    const int qd = warp & 3, hf = warp >> 2;
    const int r = 32 * qd + lane, i = q0 + r;  // this thread's query row
    const uint32_t trow = tmem + ((uint32_t)(32 * qd) << 16);
    const int cw = 32 * qd + 48 * hf;  // first key column of this thread's half window
    for (int g = 0; g < grp; ++g) {
      const uint32_t ph = (uint32_t)g & 1u;
      const size_t row = ((size_t)b * H + hk * grp + g) * L + i;
      const float lse_i = i < L ? lse[row] : 0.f, dl_i = i < L ? delta[row] : 0.f;
      for (int hv = 0; hv < 2; ++hv) {
        tc::mbar_wait(&bars[QB_SD], (uint32_t)hv, 64);  // two phases per head: parity = half
        tc::tc_fence_after();
        // 16-column chunks k of this thread's window that fall in this half
        uint32_t dk8[3][8];
#pragma unroll
        for (int k = 0; k < 3; ++k) {
          const int c0 = cw + 16 * k;  // key column in [0, 192)
          if (c0 >= hv * kHalf && c0 < (hv + 1) * kHalf) {
            float sv[16], dpv[16];
            tc::tmem_ld16(trow + kTqS + (c0 - hv * kHalf), sv);
            tc::tmem_ld16(trow + kTqDp + (c0 - hv * kHalf), dpv);
            tc::tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              float d2[2];
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int t = k0 + c0 + 2 * j + e;
                const bool ok = t <= i && t > i - W && t >= 0 && i < L;
                const float p = ok ? __expf(sv[2 * j + e] * scale - lse_i) : 0.f;
                d2[e] = p * (dpv[2 * j + e] - dl_i);
              }
              dk8[k][j] = pack_bf16(d2[0], d2[1]);
            }
          }
        }
        tc::tc_fence_before();
        tc::named_bar_sync(NB_ROWS, kThreads);  // every score column of the half read
        tc::tc_fence_after();
        // the half's 6 packed 8-column chunks (16 keys each): this quadrant's window
        // covers 16-key chunks [2 qd, 2 qd + 6) of the 12; half 0 of the quadrant owns
        // its first 3 and the zeros below, half 1 its last 3 and the zeros above
        uint32_t zero[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) zero[j] = 0u;
#pragma unroll
        for (int pc = 0; pc < kHalf / 16; ++pc) {
          const int rel = hv * (kHalf / 16) + pc - 2 * qd;  // chunk index in the window
          const uint32_t dst = trow + kTqDs + 8 * pc;
          if (rel >= 0 && rel < 6) {
            if (rel / 3 == hf) {
              if (rel % 3 == 0) tc::tmem_st8(dst, dk8[0]);
              else if (rel % 3 == 1) tc::tmem_st8(dst, dk8[1]);
              else tc::tmem_st8(dst, dk8[2]);
            }
          } else if ((rel < 0) == (hf == 0)) {
            tc::tmem_st8(dst, zero);
          }
        }
        tc::tmem_wait_st();
        tc::tc_fence_before();
        tc::named_bar_arrive(NB_PREADY, kCtaThreads);
      }
      tc::mbar_wait(&bars[QB_DQ], ph, 65);
      tc::tc_fence_after();
      float o[32];
      tc::tmem_ld32(trow + kTqDq + 32 * hf, o);  // this warp's 32 columns of dq
      tc::tmem_wait_ld();
      if (i < L) store_grad32(dq, row * kDh + 32 * hf, o, scale, gdt);
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTqCols);
  }
}

// dq for bf16 operands as a persistent kernel: one CTA per SM walks its tiles
// (b, key/value head, 128 query rows) and the group's query heads in each as
// a flat sequence of items, with two key / value buffers and two query / dy
// stages loading ahead, all 192 key columns in one pass (s [0, 192) with ds
// over it, dp [192, 384)) and dq in two TMEM buffers that alternate between
// items, so an item's dq is written out while the next item computes.
// 161 KB of shared memory, 512 TMEM columns.
struct DqPersistSmem {
  static constexpr size_t KVB = 2 * kNK * 128, QB = 2 * kQ * 128;  // k + v; q + dy
  static constexpr size_t kv = 0, qs = 2 * KVB, bars = qs + 2 * QB, slot = bars + 128,
                          bytes = slot + 16;
};
enum { QP_KV0 = 0, QP_KV1, QP_Q0, QP_Q1, QP_SD, QP_DQ, QP_EPI0, QP_EPI1, QP_N };
constexpr uint32_t kTpS = 0, kTpDs = 0, kTpDp = kNK, kTpDq = 2 * kNK, kTpCols = 512;

__global__ void __launch_bounds__(kCtaThreads, 1)
swa_bwd_dq_tc_persist_kernel(const __grid_constant__ CUtensorMap tq,
                             const __grid_constant__ CUtensorMap tdy,
                             const __grid_constant__ CUtensorMap tk,
                             const __grid_constant__ CUtensorMap tv,
                             const float* __restrict__ lse, const float* __restrict__ delta,
                             int W, float scale, int H, int grp, int L, int nqb, int ntiles,
                             void* __restrict__ dq, int gdt) {
  using SM = DqPersistSmem;
  extern __shared__ __align__(1024) unsigned char smem[];
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) atomicExch(&tc::g_timeout_flag, 0x80000000u | 85u);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::bars);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + SM::slot);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int Hkv = H / grp;
  constexpr uint32_t kTileK = kNK * 128, kTileQ = kQ * 128;
  const int nloc = (int)((ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x);
  const int nitems = nloc * grp;
  auto tile = [&](int kl, int& b, int& hk, int& q0) {
    const int tt = (int)blockIdx.x + kl * (int)gridDim.x;
    const int qb = tt % nqb, bk = tt / nqb;
    b = bk / Hkv, hk = bk - b * Hkv, q0 = qb * kQ;
  };

  if (tid == 0) {
#pragma unroll
    for (int j = 0; j < QP_N; ++j)
      tc::mbar_init(&bars[j], (j == QP_EPI0 || j == QP_EPI1) ? kThreads : 1);
    tc::fence_mbar_init();
  }
  if (warp == 8) {
    tc::tmem_alloc(tslot, kTpCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 8) {
    const bool issuer = lane == 0;
    auto load_kv = [&](int kl) {
      int b, hk, q0;
      tile(kl, b, hk, q0);
      unsigned char* buf = smem + SM::kv + (kl & 1) * SM::KVB;
      uint64_t* bar = &bars[QP_KV0 + (kl & 1)];
      tc::mbar_expect_tx(bar, 2 * kTileK);
      tc::tma_load_4d(buf, &tk, 0, q0 - (kNK - kQ), hk, b, bar);
      tc::tma_load_4d(buf + kTileK, &tv, 0, q0 - (kNK - kQ), hk, b, bar);
    };
    auto load_q = [&](int w) {
      int b, hk, q0;
      tile(w / grp, b, hk, q0);
      const int h = hk * grp + w % grp;
      unsigned char* st = smem + SM::qs + (w & 1) * SM::QB;
      uint64_t* bar = &bars[QP_Q0 + (w & 1)];
      tc::mbar_expect_tx(bar, 2 * kTileQ);
      tc::tma_load_4d(st, &tq, 0, q0, h, b, bar);
      tc::tma_load_4d(st + kTileQ, &tdy, 0, q0, h, b, bar);
    };
    if (issuer) {
      if (nloc > 0) load_kv(0);
      if (nloc > 1) load_kv(1);
      if (nitems > 0) load_q(0);
      if (nitems > 1) load_q(1);
    }
    __syncwarp();
    for (int w = 0; w < nitems; ++w) {
      const int kl = w / grp, g = w - kl * grp;
      const unsigned char* kvb = smem + SM::kv + (kl & 1) * SM::KVB;
      const unsigned char* st = smem + SM::qs + (w & 1) * SM::QB;
      if (issuer) {
        if (g == 0) tc::mbar_wait(&bars[QP_KV0 + (kl & 1)], (uint32_t)(kl >> 1) & 1u, 90);
        tc::mbar_wait(&bars[QP_Q0 + (w & 1)], (uint32_t)(w >> 1) & 1u, 91);
        if (w > 0) tc::mbar_wait(&bars[QP_DQ], (uint32_t)(w - 1) & 1u, 92);  // ds read
        tc::tc_fence_after();
        constexpr uint32_t id_s = tc::idesc_bf16(kQ, kNK, 0, 0);  // K-major x K-major
        const uint32_t kh = smem_u32(kvb), va = kh + kTileK, qh = smem_u32(st),
                       dya = qh + kTileQ;
#pragma unroll
        for (int j = 0; j < kDh / 16; ++j)
          tc::mma_ss(tmem + kTpS, tc::sdesc(qh + 32 * j, 16, 1024),
                     tc::sdesc(kh + 32 * j, 16, 1024), id_s, j > 0);
#pragma unroll
        for (int j = 0; j < kDh / 16; ++j)
          tc::mma_ss(tmem + kTpDp, tc::sdesc(dya + 32 * j, 16, 1024),
                     tc::sdesc(va + 32 * j, 16, 1024), id_s, j > 0);
        tc::mma_commit(&bars[QP_SD]);
      }
      __syncwarp();
      tc::named_bar_sync(NB_PREADY, kCtaThreads);  // ds in TMEM
      if (issuer) {
        // dq buffer w & 1 was last read by item w - 2's write-out
        if (w >= 2) tc::mbar_wait(&bars[QP_EPI0 + (w & 1)], (((uint32_t)w >> 1) & 1u) ^ 1u, 93);
        tc::tc_fence_after();
        constexpr uint32_t id_o = tc::idesc_bf16(kQ, kDh, 0, 1);  // TMEM x MN-major
        const uint32_t kh = smem_u32(kvb);
#pragma unroll
        for (int j = 0; j < kNK / 16; ++j)
          tc::mma_ts(tmem + kTpDq + 64 * (w & 1), tmem + kTpDs + 8 * j,
                     tc::sdesc(kh + 2048 * j, kTileK, 1024), id_o, j > 0);
        tc::mma_commit(&bars[QP_DQ]);
        const bool refill_q = w + 2 < nitems, refill_kv = g == grp - 1 && kl + 2 < nloc;
        if (refill_q || refill_kv) {
          tc::mbar_wait(&bars[QP_DQ], (uint32_t)w & 1u, 94);  // item w's tiles read
          if (refill_q) load_q(w + 2);
          if (refill_kv) load_kv(kl + 2);
        }
      }
      __syncwarp();
    }
  } else {
    const int qd = warp & 3, hf = warp >> 2;
    const int r = 32 * qd + lane;
    const uint32_t trow = tmem + ((uint32_t)(32 * qd) << 16);
    const int cw = 32 * qd + 48 * hf;  // first key column of this thread's half window
    const float scale_log2 = scale * kLog2e;
    // lse and delta of this thread's row in item w2, loaded one item ahead
    auto row_stats = [&](int w2, float& a, float& d) {
      const int kl2 = w2 / grp, g2 = w2 - kl2 * grp;
      int b2, hk2, q02;
      tile(kl2, b2, hk2, q02);
      const int i2 = q02 + r;
      const size_t row2 = ((size_t)b2 * H + hk2 * grp + g2) * L + i2;
      a = i2 < L ? lse[row2] : 0.f;
      d = i2 < L ? delta[row2] : 0.f;
    };
    float nl = 0.f, nd = 0.f;
    if (nitems > 0) row_stats(0, nl, nd);
    for (int w = 0; w < nitems; ++w) {
      const int kl = w / grp, g = w - kl * grp;
      int b, hk, q0;
      tile(kl, b, hk, q0);
      const int i = q0 + r, k0 = q0 - (kNK - kQ);  // this thread's query row
      const size_t row = ((size_t)b * H + hk * grp + g) * L + i;
      const float lse_i = nl * kLog2e, dl_i = nd;  // lse in base 2
      if (w + 1 < nitems) row_stats(w + 1, nl, nd);
      tc::mbar_wait(&bars[QP_SD], (uint32_t)w & 1u, 95);
      tc::tc_fence_after();
      uint32_t dk8[3][8];
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        float sv[16], dpv[16];
        tc::tmem_ld16(trow + kTpS + cw + 16 * k, sv);
        tc::tmem_ld16(trow + kTpDp + cw + 16 * k, dpv);
        tc::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float d2[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int t = k0 + cw + 16 * k + 2 * j + e;
            const bool ok = t <= i && t > i - W && t >= 0 && i < L;
            const float p = ok ? tc::ex2(sv[2 * j + e] * scale_log2 - lse_i) : 0.f;
            d2[e] = p * (dpv[2 * j + e] - dl_i);
          }
          dk8[k][j] = pack_bf16(d2[0], d2[1]);
        }
      }
      tc::tc_fence_before();
      tc::named_bar_sync(NB_ROWS, kThreads);  // every score column of the CTA read
      tc::tc_fence_after();
#pragma unroll
      for (int k = 0; k < 3; ++k) tc::tmem_st8(trow + kTpDs + cw / 2 + 8 * k, dk8[k]);
      {  // zero outside the window: packed columns [0, 16 qd) and [16 qd + 48, 96)
        uint32_t zero[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) zero[j] = 0u;
        const int z0 = hf ? 16 * qd + 48 : 0, z1 = hf ? kNK / 2 : 16 * qd;
#pragma unroll 1
        for (int c = z0; c < z1; c += 8) tc::tmem_st8(trow + kTpDs + c, zero);
      }
      tc::tmem_wait_st();
      tc::tc_fence_before();
      tc::named_bar_arrive(NB_PREADY, kCtaThreads);
      tc::mbar_wait(&bars[QP_DQ], (uint32_t)w & 1u, 96);
      tc::tc_fence_after();
      float o[32];
      tc::tmem_ld32(trow + kTpDq + 64 * (w & 1) + 32 * hf, o);  // this warp's 32 columns
      tc::tmem_wait_ld();
      if (i < L) store_grad32(dq, row * kDh + 32 * hf, o, scale, gdt);
      tc::tc_fence_before();
      tc::mbar_arrive(&bars[QP_EPI0 + (w & 1)]);
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTpCols);
  }
}

// The forward for bf16 operands (already rotated, no residual tiles) as a
// persistent kernel, two CTAs per SM: each CTA walks its tiles (b, key/value
// head, 128 query rows) and the group's query heads in each as one sequence of
// items. A TMA / MMA warp (warp 8) keeps the next tile's keys and the next
// items' queries loading ahead (two key buffers, two query stages, one value
// buffer refilled as soon as a tile's last p V is done) and issues s = q k^T
// and o = p_hi V + p_lo V; the next item's scores run while the row warps
// write this item's output. The row warps' softmax is the arithmetic of
// swa_fwd_tc_kernel. 106 KB of shared memory and 256 TMEM columns per CTA.
struct FwdPersistSmem {
  static constexpr size_t KB = kNK * 128, QB = kQ * 128;  // one k or v tile; one q tile
  static constexpr size_t k = 0, v = 2 * KB, qs = v + KB, red = qs + 2 * QB;  // [max | sum][2][128]
  static constexpr size_t bars = red + 2 * 2 * 128 * 4, slot = bars + 128, bytes = slot + 16;
};
enum { FP_K0 = 0, FP_K1, FP_V, FP_Q0, FP_Q1, FP_S, FP_O, FP_N };
constexpr uint32_t kTfS = 0, kTfPh = 0, kTfPl = kNK / 2, kTfO = kNK, kTfCols = 256;

__global__ void __launch_bounds__(kCtaThreads, 2)
swa_fwd_tc_persist_kernel(const __grid_constant__ CUtensorMap tq,
                          const __grid_constant__ CUtensorMap tk,
                          const __grid_constant__ CUtensorMap tv,
                          const float* __restrict__ meta, int n_meta, int W, float scale_log2,
                          int H, int grp, int L, int nqb, int ntiles, bf16* __restrict__ y,
                          float* __restrict__ lse, float* __restrict__ y32) {
  using SM = FwdPersistSmem;
  extern __shared__ __align__(1024) unsigned char smem[];
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) atomicExch(&tc::g_timeout_flag, 0x80000000u | 84u);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::bars);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + SM::slot);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int Hkv = H / grp;
  constexpr uint32_t kTileK = kNK * 128, kTileQ = kQ * 128;
  const int nloc = (int)((ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x);
  const int nitems = nloc * grp;
  auto tile = [&](int kl, int& b, int& hk, int& q0) {
    const int tt = (int)blockIdx.x + kl * (int)gridDim.x;
    const int qb = tt % nqb, bk = tt / nqb;
    b = bk / Hkv, hk = bk - b * Hkv, q0 = qb * kQ;
  };

  if (tid == 0) {
#pragma unroll
    for (int j = 0; j < FP_N; ++j) tc::mbar_init(&bars[j], 1);
    tc::fence_mbar_init();
  }
  if (warp == 8) {
    tc::tmem_alloc(tslot, kTfCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 8) {
    const bool issuer = lane == 0;
    auto load_k = [&](int kl) {
      int b, hk, q0;
      tile(kl, b, hk, q0);
      uint64_t* bar = &bars[FP_K0 + (kl & 1)];
      tc::mbar_expect_tx(bar, kTileK);
      tc::tma_load_4d(smem + SM::k + (kl & 1) * SM::KB, &tk, 0, q0 - (kNK - kQ), hk, b, bar);
    };
    auto load_v = [&](int kl) {
      int b, hk, q0;
      tile(kl, b, hk, q0);
      tc::mbar_expect_tx(&bars[FP_V], kTileK);
      tc::tma_load_4d(smem + SM::v, &tv, 0, q0 - (kNK - kQ), hk, b, &bars[FP_V]);
    };
    auto load_q = [&](int w) {
      int b, hk, q0;
      tile(w / grp, b, hk, q0);
      uint64_t* bar = &bars[FP_Q0 + (w & 1)];
      tc::mbar_expect_tx(bar, kTileQ);
      tc::tma_load_4d(smem + SM::qs + (w & 1) * SM::QB, &tq, 0, q0, hk * grp + w % grp, b, bar);
    };
    if (issuer) {
      if (nloc > 0) load_k(0), load_v(0);
      if (nloc > 1) load_k(1);
      if (nitems > 0) load_q(0);
      if (nitems > 1) load_q(1);
    }
    __syncwarp();
    for (int w = 0; w < nitems; ++w) {
      const int kl = w / grp, g = w - kl * grp;
      if (issuer) {
        if (g == 0) tc::mbar_wait(&bars[FP_K0 + (kl & 1)], (uint32_t)(kl >> 1) & 1u, 100);
        tc::mbar_wait(&bars[FP_Q0 + (w & 1)], (uint32_t)(w >> 1) & 1u, 101);
        if (w > 0) tc::mbar_wait(&bars[FP_O], (uint32_t)(w - 1) & 1u, 102);  // p read
        tc::tc_fence_after();
        constexpr uint32_t id_s = tc::idesc_bf16(kQ, kNK, 0, 0);  // q (K-major) x k (K-major)
        const uint32_t kh = smem_u32(smem + SM::k + (kl & 1) * SM::KB);
        const uint32_t qh = smem_u32(smem + SM::qs + (w & 1) * SM::QB);
#pragma unroll
        for (int j = 0; j < kDh / 16; ++j)
          tc::mma_ss(tmem + kTfS, tc::sdesc(qh + 32 * j, 16, 1024),
                     tc::sdesc(kh + 32 * j, 16, 1024), id_s, j > 0);
        tc::mma_commit(&bars[FP_S]);
      }
      __syncwarp();
      // p in TMEM; the row warps have also read the previous item's o
      tc::named_bar_sync(NB_PREADY, kCtaThreads);
      if (issuer) {
        if (g == 0) tc::mbar_wait(&bars[FP_V], (uint32_t)kl & 1u, 103);
        tc::tc_fence_after();
        constexpr uint32_t id_o = tc::idesc_bf16(kQ, kDh, 0, 1);  // p (TMEM) x V (MN-major)
        const uint32_t va = smem_u32(smem + SM::v);
#pragma unroll
        for (int j = 0; j < kNK / 16; ++j)
          tc::mma_ts(tmem + kTfO, tmem + kTfPh + 8 * j, tc::sdesc(va + 2048 * j, kTileK, 1024),
                     id_o, j > 0);
#pragma unroll
        for (int j = 0; j < kNK / 16; ++j)
          tc::mma_ts(tmem + kTfO, tmem + kTfPl + 8 * j, tc::sdesc(va + 2048 * j, kTileK, 1024),
                     id_o, 1u);
        tc::mma_commit(&bars[FP_O]);
        const bool last = g == grp - 1;
        const bool refill = w + 2 < nitems || (last && kl + 1 < nloc);
        if (refill) {
          tc::mbar_wait(&bars[FP_O], (uint32_t)w & 1u, 104);  // item w's tiles read
          if (w + 2 < nitems) load_q(w + 2);
          if (last && kl + 1 < nloc) load_v(kl + 1);
          if (last && kl + 2 < nloc) load_k(kl + 2);
        }
      }
      __syncwarp();
    }
  } else {
    const int qd = warp & 3, hf = warp >> 2;
    const int r = 32 * qd + lane;
    const uint32_t trow = tmem + ((uint32_t)(32 * qd) << 16);
    const int cw = 32 * qd + 48 * hf;  // first score column of this thread's half window
    float* red = reinterpret_cast<float*>(smem + SM::red);  // [max | sum][half][row]
    // sinks seed the max and the row sum (log2 domain)
    float ms = -1e30f;
    for (int j = 0; j < n_meta; ++j) ms = fmaxf(ms, meta[j] * kLog2e);
    float ls = 0.f;
    for (int j = 0; j < n_meta; ++j) ls += exp2f(meta[j] * kLog2e - ms);
    for (int w = 0; w < nitems; ++w) {
      const int kl = w / grp, g = w - kl * grp;
      int b, hk, q0;
      tile(kl, b, hk, q0);
      const int i = q0 + r, k0 = q0 - (kNK - kQ);
      tc::mbar_wait(&bars[FP_S], (uint32_t)w & 1u, 105);
      tc::tc_fence_after();
      float sv[3][16];
#pragma unroll
      for (int k = 0; k < 3; ++k) tc::tmem_ld16(trow + kTfS + cw + 16 * k, sv[k]);
      tc::tmem_wait_ld();
      float mx = ms;
#pragma unroll
      for (int k = 0; k < 3; ++k)
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const int t = k0 + cw + 16 * k + u;
          const bool ok = t <= i && t > i - W && t >= 0;
          const float x = ok ? sv[k][u] * scale_log2 : -INFINITY;
          sv[k][u] = x;
          mx = fmaxf(mx, x);
        }
      red[hf * kQ + r] = mx;
      tc::tc_fence_before();
      tc::named_bar_sync(NB_ROWS, kThreads);  // the partner's max; every score column read
      tc::tc_fence_after();
      mx = fmaxf(mx, red[(1 - hf) * kQ + r]);
      float l = 0.f;
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        uint32_t phi[8], plo[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float p0 = tc::ex2(sv[k][2 * j] - mx), p1 = tc::ex2(sv[k][2 * j + 1] - mx);
          l += p0 + p1;
          const uint32_t hpk = pack_bf16(p0, p1);
          phi[j] = hpk;
          plo[j] = pack_bf16(p0 - bf16_lo(hpk), p1 - bf16_hi(hpk));
        }
        tc::tmem_st8(trow + kTfPh + cw / 2 + 8 * k, phi);
        tc::tmem_st8(trow + kTfPl + cw / 2 + 8 * k, plo);
      }
      {  // p is zero outside the window: packed columns [0, 16 qd) and [16 qd + 48, 96)
        uint32_t zero[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) zero[j] = 0u;
        const int z0 = hf ? 16 * qd + 48 : 0, z1 = hf ? kNK / 2 : 16 * qd;
#pragma unroll 1
        for (int c = z0; c < z1; c += 8) {
          tc::tmem_st8(trow + kTfPh + c, zero);
          tc::tmem_st8(trow + kTfPl + c, zero);
        }
      }
      red[2 * kQ + hf * kQ + r] = l;
      tc::tmem_wait_st();
      tc::tc_fence_before();
      tc::named_bar_sync(NB_ROWS, kThreads);  // both halves' p stored and row sums written
      tc::named_bar_arrive(NB_PREADY, kCtaThreads);
      const float lrow = ls * exp2f(ms - mx) + red[2 * kQ + r] + red[3 * kQ + r];
      const float inv = 1.f / lrow;
      const size_t row = ((size_t)b * H + hk * grp + g) * L + i;
      tc::mbar_wait(&bars[FP_O], (uint32_t)w & 1u, 106);
      tc::tc_fence_after();
      float o[32];
      tc::tmem_ld32(trow + kTfO + 32 * hf, o);
      tc::tmem_wait_ld();
      tc::tc_fence_before();
      if (i < L) {
        bf16* yr = y + row * kDh + 32 * hf;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          uint4 wv;
          wv.x = pack_bf16(o[8 * q4] * inv, o[8 * q4 + 1] * inv);
          wv.y = pack_bf16(o[8 * q4 + 2] * inv, o[8 * q4 + 3] * inv);
          wv.z = pack_bf16(o[8 * q4 + 4] * inv, o[8 * q4 + 5] * inv);
          wv.w = pack_bf16(o[8 * q4 + 6] * inv, o[8 * q4 + 7] * inv);
          reinterpret_cast<uint4*>(yr)[q4] = wv;
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
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTfCols);
  }
}

// ============================================================ windows 65 ... 128
// The same three products for 64 < W <= 128 (the reference's own training
// configs use window 128). A 128-row tile then sees 128 keys to its left, so
// each kernel splits the wider tile to stay within 256 TMEM columns:
//   forward : 128 query rows against the 256 keys [q0 - 128, q0 + 128) in two
//             halves of 128, each with its own softmax pass and P V
//             accumulator, merged at the end by the two maxima
//   dq      : the 256 keys in four quarters of 64, ds of a quarter over its
//             scores
//   dk / dv : the 256 query rows [k0, k0 + 256) that can see a 128-key tile in
//             items of 64 rows, four per query head, dk and dv summed in TMEM
//             over the items and the group's heads
// With bf16 operands two CTAs share an SM. Each row warp covers a fixed half
// of the columns of a half / quarter / item (masked outside the window), so
// every column of the bf16 operands is written; in the backward kernels a warp
// writes them over score columns it has itself already read, so no barrier
// separates the reads from the writes. Precision as the kernels above: logits
// from the hi / lo terms, p in bf16 hi + lo for P V, bf16 p and ds in the
// gradients.
constexpr int kH2 = 128;            // keys left of a query tile (window <= 128)
constexpr int kNK2 = kQ + kH2;      // 256 key rows per forward / dq tile
template <bool SPLIT>
struct Fwd128Smem {
  static constexpr size_t KT = kNK2 * 128, QT = kQ * 128;
  static constexpr size_t kh = 0, kl = kh + KT, v = kl + (SPLIT ? KT : 0), qh = v + KT,
                          ql = qh + QT, red = ql + (SPLIT ? QT : 0), bars = red + 2048,
                          slot = bars + 32, bytes = slot + 16;
};
// TMEM: s of one key half [0, 128) with p hi / lo (bf16 pairs, 64 columns
// each) over it; o of the left half [128, 192), of the right half [192, 256)
constexpr uint32_t kT2S = 0, kT2Ph = 0, kT2Pl = 64, kT2OA = 128, kT2OB = 192, kT2Cols = 256;

// The forward takes the 256 keys in two halves of 128, [q0 - 128, q0) and
// [q0, q0 + 128), each with its own softmax pass and P V product into its own
// accumulator: the left half's max m_A (seeded by the sinks), then the right
// half's p relative to m = max(m_A, its own max), and at the end
// o = o_A 2^(m_A - m) + o_B. 256 TMEM columns and, for bf16 operands, 82 KB of
// shared memory: two CTAs per SM. Each row warp covers 64 of a half's 128
// columns; 16-column chunks that no row of its lane quadrant can see are
// skipped (no TMEM load, p = 0).
// ROPE: q, k are the unrotated bf16 projections (maps tq, tk, raw rows landing
// in the residual buffers), rotated and split into bf16 hi + lo in the CTA as
// in the window <= 64 forward; the rotated operands go to qh_out ... kl_out
// when given. Otherwise q, k are the rotated operands (SPLIT: with residuals).
template <bool ROPE, bool SPLIT, typename CT>
__global__ void __launch_bounds__(kThreads, (SPLIT || ROPE) ? 1 : 2)
swa_fwd_tc128_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                     const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tql,
                     const __grid_constant__ CUtensorMap tkl, const CT* __restrict__ cs,
                     const CT* __restrict__ sn, long long cs_sb, long long cs_sl,
                     const float* __restrict__ meta, int n_meta, int W, float scale_log2, int H,
                     int grp, int L, int nqb, bf16* __restrict__ y, float* __restrict__ lse,
                     float* __restrict__ y32, bf16* __restrict__ qh_out,
                     bf16* __restrict__ ql_out, bf16* __restrict__ kh_out,
                     bf16* __restrict__ kl_out) {
  static_assert(SPLIT || !ROPE, "the rotation writes bf16 hi + lo operands");
  using SM = Fwd128Smem<SPLIT>;
  extern __shared__ __align__(1024) unsigned char smem[];
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) atomicExch(&tc::g_timeout_flag, 0x80000000u | 85u);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::bars);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + SM::slot);
  float* red = reinterpret_cast<float*>(smem + SM::red);  // [max | sum][half][row]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = warp & 3, hf = warp >> 2;
  const int qb = blockIdx.x % nqb, bk = blockIdx.x / nqb;
  const int Hkv = H / grp, b = bk / Hkv, hk = bk - b * Hkv;
  const int q0 = qb * kQ, k0 = q0 - kH2;
  constexpr uint32_t kTileK = kNK2 * 128, kTileQ = kQ * 128;

  if (tid == 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) tc::mbar_init(&bars[j], 1);
    tc::fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(tslot, kT2Cols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tslot;

  auto issue_q = [&](int g) {
    const int h = hk * grp + g;
    tc::mbar_expect_tx(&bars[SB_Q], (SPLIT && !ROPE) ? 2 * kTileQ : kTileQ);
    if (ROPE) {
      tc::tma_load_4d(smem + SM::ql, &tq, 0, q0, h, b, &bars[SB_Q]);  // raw rows land in lo
    } else {
      tc::tma_load_4d(smem + SM::qh, &tq, 0, q0, h, b, &bars[SB_Q]);
      if (SPLIT) tc::tma_load_4d(smem + SM::ql, &tql, 0, q0, h, b, &bars[SB_Q]);
    }
  };
  auto issue_s = [&](int hv) {  // s = q k^T of key half hv into TMEM columns [0, 128)
    tc::tc_fence_after();
    constexpr uint32_t id_s = tc::idesc_bf16(kQ, 128, 0, 0);
    const uint32_t ko = (uint32_t)(hv * 128 * 128);
    const uint32_t qh = smem_u32(smem + SM::qh), ql = smem_u32(smem + SM::ql),
                   kh = smem_u32(smem + SM::kh) + ko, kl = smem_u32(smem + SM::kl) + ko;
#pragma unroll
    for (int j = 0; j < kDh / 16; ++j)
      tc::mma_ss(tmem + kT2S, tc::sdesc(qh + 32 * j, 16, 1024), tc::sdesc(kh + 32 * j, 16, 1024),
                 id_s, j > 0);
    if (SPLIT) {
#pragma unroll
      for (int j = 0; j < kDh / 16; ++j)
        tc::mma_ss(tmem + kT2S, tc::sdesc(qh + 32 * j, 16, 1024),
                   tc::sdesc(kl + 32 * j, 16, 1024), id_s, 1u);
#pragma unroll
      for (int j = 0; j < kDh / 16; ++j)
        tc::mma_ss(tmem + kT2S, tc::sdesc(ql + 32 * j, 16, 1024),
                   tc::sdesc(kh + 32 * j, 16, 1024), id_s, 1u);
    }
    tc::mma_commit(&bars[SB_S]);
  };
  if (tid == 0) {
    tc::mbar_expect_tx(&bars[SB_KV], (SPLIT && !ROPE) ? 3 * kTileK : 2 * kTileK);
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
  tc::mbar_wait(&bars[SB_KV], 0, 110);
  if (ROPE) {  // the 256 key rows once; this tile's own 128 rows go out for the backward
    const size_t kvb = ((size_t)b * Hkv + hk) * L * kDh;
    bf16* gh = kh_out ? kh_out + kvb : nullptr;
    bf16* gl = kh_out ? kl_out + kvb : nullptr;
    rotate_rows<0, 128, CT>(smem + SM::kh, smem + SM::kl, k0, L, csb, snb, cs_sl, kH2, gh, gl);
    rotate_rows<128, 128, CT>(smem + SM::kh, smem + SM::kl, k0, L, csb, snb, cs_sl, kH2, gh,
                              gl);
  }
  tc::mbar_wait(&bars[SB_Q], 0, 111);
  if (ROPE) rotate_q(0);
  tc::fence_proxy_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  if (tid == 0) issue_s(0);

  const int r = 32 * qd + lane, i = q0 + r;
  const uint32_t trow = tmem + ((uint32_t)(32 * qd) << 16);
  const int imin = q0 + 32 * qd, imax = imin + 31;  // the lane quadrant's query rows
  for (int g = 0; g < grp; ++g) {
    const bool next = g + 1 < grp;
    float mA = ms, lA = 0.f, mrow = ms, lB = 0.f;
#pragma unroll 1
    for (int hv = 0; hv < 2; ++hv) {
      tc::mbar_wait(&bars[SB_S], (uint32_t)hv, 112);  // two score commits per head
      tc::tc_fence_after();
      if (tid == 0 && hv == 1 && next) issue_q(g + 1);  // both halves' scores read q
      // this warp's 64 columns of the half: keys t = k0 + 128 hv + 64 hf + c
      const int tb = k0 + 128 * hv + 64 * hf;
      float s[4][16];
      bool live[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int t0 = tb + 16 * k;
        live[k] = !(t0 > imax || t0 + 15 <= imin - W);  // some row of the quadrant sees it
        if (live[k]) tc::tmem_ld16(trow + kT2S + 64 * hf + 16 * k, s[k]);
      }
      tc::tmem_wait_ld();
      float mx = -INFINITY;
#pragma unroll
      for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const int t = tb + 16 * k + u;
          const bool ok = live[k] && t <= i && t > i - W && t >= 0;
          const float x = ok ? s[k][u] * scale_log2 : -INFINITY;
          s[k][u] = x;
          mx = fmaxf(mx, x);
        }
      red[hf * kQ + r] = mx;
      __syncthreads();  // every score column read; the partner's max in red
      mx = fmaxf(mx, red[(1 - hf) * kQ + r]);
      // reference of this half's p: m_A (with the sinks) on the left, then
      // m = max(m_A, the right half's max)
      const float mref = hv == 0 ? fmaxf(ms, mx) : fmaxf(mA, mx);
      float l = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint32_t phi[8], plo[8];
        if (live[k]) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float p0 = tc::ex2(s[k][2 * j] - mref), p1 = tc::ex2(s[k][2 * j + 1] - mref);
            l += p0 + p1;
            const uint32_t hpk = pack_bf16(p0, p1);
            phi[j] = hpk;
            plo[j] = pack_bf16(p0 - bf16_lo(hpk), p1 - bf16_hi(hpk));
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) phi[j] = plo[j] = 0u;
        }
        tc::tmem_st8(trow + kT2Ph + 32 * hf + 8 * k, phi);
        tc::tmem_st8(trow + kT2Pl + 32 * hf + 8 * k, plo);
      }
      red[2 * kQ + hf * kQ + r] = l;
      tc::tmem_wait_st();
      tc::tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        tc::tc_fence_after();
        constexpr uint32_t id_o = tc::idesc_bf16(kQ, kDh, 0, 1);  // p (TMEM) x V (MN-major)
        const uint32_t va = smem_u32(smem + SM::v) + (uint32_t)(hv * 128 * 128);
        const uint32_t od = tmem + (hv ? kT2OB : kT2OA);
#pragma unroll
        for (int j = 0; j < 128 / 16; ++j)
          tc::mma_ts(od, tmem + kT2Ph + 8 * j, tc::sdesc(va + 2048 * j, kTileK, 1024), id_o,
                     j > 0);
#pragma unroll
        for (int j = 0; j < 128 / 16; ++j)
          tc::mma_ts(od, tmem + kT2Pl + 8 * j, tc::sdesc(va + 2048 * j, kTileK, 1024), id_o, 1u);
        tc::mma_commit(&bars[SB_O]);
      }
      const float lh = red[2 * kQ + r] + red[3 * kQ + r];
      if (hv == 0) {
        mA = mref, lA = lh;
      } else {
        mrow = mref, lB = lh;
      }
      if (hv == 1 && next) {  // the next head's query tiles, rotated while P V runs
        tc::mbar_wait(&bars[SB_Q], (uint32_t)(g + 1) & 1u, 111);
        if (ROPE) rotate_q(g + 1);
        tc::fence_proxy_async_smem();
      }
      tc::mbar_wait(&bars[SB_O], (uint32_t)hv, 113);  // two P V commits per head
      tc::tc_fence_after();
      tc::tc_fence_before();
      __syncthreads();  // P V done (s / p columns and the row slots free)
      if (tid == 0 && (hv == 0 || next)) issue_s(hv ^ 1);  // right half, or the next head's left
    }
    const float fa = tc::ex2(mA - mrow);  // <= 1
    const float lrow = ls * exp2f(ms - mrow) + lA * fa + lB;
    const float inv = 1.f / lrow;
    const size_t row = ((size_t)b * H + hk * grp + g) * L + i;
#pragma unroll 1
    for (int c16 = 0; c16 < 2; ++c16) {  // this warp's 32 output columns, 16 at a time
      const int c0 = 32 * hf + 16 * c16;
      float oa[16], ob[16];
      tc::tmem_ld16(trow + kT2OA + c0, oa);
      tc::tmem_ld16(trow + kT2OB + c0, ob);
      tc::tmem_wait_ld();
#pragma unroll
      for (int u = 0; u < 16; ++u) oa[u] = (oa[u] * fa + ob[u]) * inv;
      if (i < L) {
        uint4* yr = reinterpret_cast<uint4*>(y + row * kDh + c0);
#pragma unroll
        for (int q4 = 0; q4 < 2; ++q4)
          yr[q4] = make_uint4(pack_bf16(oa[8 * q4], oa[8 * q4 + 1]),
                              pack_bf16(oa[8 * q4 + 2], oa[8 * q4 + 3]),
                              pack_bf16(oa[8 * q4 + 4], oa[8 * q4 + 5]),
                              pack_bf16(oa[8 * q4 + 6], oa[8 * q4 + 7]));
        if (y32) {
          float4* d32 = reinterpret_cast<float4*>(y32 + row * kDh + c0);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
            d32[q4] = make_float4(oa[4 * q4], oa[4 * q4 + 1], oa[4 * q4 + 2], oa[4 * q4 + 3]);
        }
      }
    }
    if (i < L && lse && hf == 0) lse[row] = mrow * kLn2f + logf(lrow);
    tc::tc_fence_before();
    __syncthreads();  // both o accumulators read before the next head's P V
  }
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kT2Cols);
  }
}

// dq for 64 < W <= 128: one CTA of 9 warps per 128 query rows and each query
// head of the group; the keys [q0 - 128, q0 + 128) in four quarters of 64, so
// the scores, dp and dq fit 256 TMEM columns and, with bf16 operands (96 KB
// of shared memory, one query / dy stage), two CTAs share an SM.
constexpr int kQK = 64;  // keys per quarter
template <bool SPLIT>
struct Dq128Smem {
  static constexpr size_t KT = kNK2 * 128, QT = kQ * 128;
  static constexpr size_t kh = 0, kl = kh + KT, v = kl + (SPLIT ? KT : 0), st = v + KT;
  static constexpr size_t sq = 0, sql = QT, sdy = sql + (SPLIT ? QT : 0), sbytes = sdy + QT;
  static constexpr size_t bars = st + sbytes, slot = bars + 64, bytes = slot + 16;
};
// TMEM: s of a quarter [0, 64) with ds (bf16 pairs) over it in [0, 16) and
// [32, 48) (the first half of each row warp's 32 score columns); dp [64, 128);
// dq [128, 192)
constexpr uint32_t kU2S = 0, kU2Ds = 0, kU2Dp = 64, kU2Dq = 128, kU2Cols = 256;

template <bool SPLIT>
__global__ void __launch_bounds__(kCtaThreads, SPLIT ? 1 : 2)
swa_bwd_dq_tc128_kernel(const __grid_constant__ CUtensorMap tq,
                        const __grid_constant__ CUtensorMap tql,
                        const __grid_constant__ CUtensorMap tdy,
                        const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tkl,
                        const __grid_constant__ CUtensorMap tv, const float* __restrict__ lse,
                        const float* __restrict__ delta, int W, float scale, int H, int grp, int L,
                        int nqb, void* __restrict__ dq, int gdt) {
  using SM = Dq128Smem<SPLIT>;
  extern __shared__ __align__(1024) unsigned char smem[];
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) atomicExch(&tc::g_timeout_flag, 0x80000000u | 84u);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::bars);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + SM::slot);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qb = blockIdx.x % nqb, bk = blockIdx.x / nqb;
  const int Hkv = H / grp, b = bk / Hkv, hk = bk - b * Hkv;
  const int q0 = qb * kQ, k0 = q0 - kH2;
  constexpr uint32_t kTileK = kNK2 * 128, kTileQ = kQ * 128;

  if (tid == 0) {
#pragma unroll
    for (int j = 0; j < 6; ++j) tc::mbar_init(&bars[j], 1);
    tc::fence_mbar_init();
  }
  if (warp == 8) {
    tc::tmem_alloc(tslot, kU2Cols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 8) {
    const bool issuer = lane == 0;
    auto load_stage = [&](int g) {  // query / dy rows of head hk * grp + g
      const int h = hk * grp + g;
      unsigned char* st = smem + SM::st;
      uint64_t* bar = &bars[QB_Q0];
      tc::mbar_expect_tx(bar, (SPLIT ? 3 : 2) * kTileQ);
      tc::tma_load_4d(st + SM::sq, &tq, 0, q0, h, b, bar);
      if (SPLIT) tc::tma_load_4d(st + SM::sql, &tql, 0, q0, h, b, bar);
      tc::tma_load_4d(st + SM::sdy, &tdy, 0, q0, h, b, bar);
    };
    if (issuer) {
      tc::mbar_expect_tx(&bars[QB_KV], (SPLIT ? 3 : 2) * kTileK);
      tc::tma_load_4d(smem + SM::kh, &tk, 0, k0, hk, b, &bars[QB_KV]);
      if (SPLIT) tc::tma_load_4d(smem + SM::kl, &tkl, 0, k0, hk, b, &bars[QB_KV]);
      tc::tma_load_4d(smem + SM::v, &tv, 0, k0, hk, b, &bars[QB_KV]);
      load_stage(0);
      tc::mbar_wait(&bars[QB_KV], 0, 114);
    }
    __syncwarp();
    const uint32_t kh = smem_u32(smem + SM::kh), kl = smem_u32(smem + SM::kl),
                   va = smem_u32(smem + SM::v), qh = smem_u32(smem + SM::st + SM::sq),
                   ql = smem_u32(smem + SM::st + SM::sql), dya = smem_u32(smem + SM::st + SM::sdy);
    for (int g = 0; g < grp; ++g) {
      for (int qv = 0; qv < 4; ++qv) {
        const uint32_t ko = (uint32_t)(qv * kQK * 128);  // the quarter's first key row
        if (issuer) {
          // the previous quarter's ds has been read (one commit per quarter, four
          // per head, so its parity is that of qv - 1; for qv = 0 the last quarter
          // of head g - 1, waited here too so no later wait sees a stale phase)
          if (qv > 0 || g > 0) tc::mbar_wait(&bars[QB_HALF], (uint32_t)(qv + 3) & 1u, 117);
          // head g's tiles landed (loaded once head g - 1's MMAs were done)
          if (qv == 0) tc::mbar_wait(&bars[QB_Q0], (uint32_t)g & 1u, 115);
          tc::tc_fence_after();
          constexpr uint32_t id_s = tc::idesc_bf16(kQ, kQK, 0, 0);  // K-major x K-major
#pragma unroll
          for (int j = 0; j < kDh / 16; ++j)
            tc::mma_ss(tmem + kU2S, tc::sdesc(qh + 32 * j, 16, 1024),
                       tc::sdesc(kh + ko + 32 * j, 16, 1024), id_s, j > 0);
          if (SPLIT) {
#pragma unroll
            for (int j = 0; j < kDh / 16; ++j)
              tc::mma_ss(tmem + kU2S, tc::sdesc(qh + 32 * j, 16, 1024),
                         tc::sdesc(kl + ko + 32 * j, 16, 1024), id_s, 1u);
#pragma unroll
            for (int j = 0; j < kDh / 16; ++j)
              tc::mma_ss(tmem + kU2S, tc::sdesc(ql + 32 * j, 16, 1024),
                         tc::sdesc(kh + ko + 32 * j, 16, 1024), id_s, 1u);
          }
#pragma unroll
          for (int j = 0; j < kDh / 16; ++j)
            tc::mma_ss(tmem + kU2Dp, tc::sdesc(dya + 32 * j, 16, 1024),
                       tc::sdesc(va + ko + 32 * j, 16, 1024), id_s, j > 0);
          tc::mma_commit(&bars[QB_SD]);
        }
        __syncwarp();
        tc::named_bar_sync(NB_PREADY, kCtaThreads);  // this quarter's ds in TMEM
        if (issuer) {
          tc::tc_fence_after();
          constexpr uint32_t id_o = tc::idesc_bf16(kQ, kDh, 0, 1);  // TMEM x MN-major
          // keys 16 j.. of the quarter: packed columns 32 (j / 2) + 8 (j % 2)
#pragma unroll
          for (int j = 0; j < kQK / 16; ++j)
            tc::mma_ts(tmem + kU2Dq, tmem + kU2Ds + 32 * (j >> 1) + 8 * (j & 1),
                       tc::sdesc(kh + ko + 2048 * j, kTileK, 1024), id_o,
                       (qv > 0 || j > 0) ? 1u : 0u);
          tc::mma_commit(&bars[QB_HALF]);
          if (qv == 3) {
            tc::mma_commit(&bars[QB_DQ]);
            if (g + 1 < grp) {
              tc::mbar_wait(&bars[QB_DQ], (uint32_t)g & 1u, 118);  // the stage's last reader
              load_stage(g + 1);
            }
          }
        }
        __syncwarp();
      }
    }
  } else {
    const int qd = warp & 3, hf = warp >> 2;
    const int r = 32 * qd + lane, i = q0 + r;  // this thread's query row
    const uint32_t trow = tmem + ((uint32_t)(32 * qd) << 16);
    for (int g = 0; g < grp; ++g) {
      const uint32_t ph = (uint32_t)g & 1u;
      const size_t row = ((size_t)b * H + hk * grp + g) * L + i;
      const float lse_i = i < L ? lse[row] : 0.f, dl_i = i < L ? delta[row] : 0.f;
      for (int qv = 0; qv < 4; ++qv) {
        tc::mbar_wait(&bars[QB_SD], (uint32_t)qv & 1u, 119);  // four phases per head
        tc::tc_fence_after();
        // columns [32 hf, 32 hf + 32) of this quarter (keys t = k0 + 64 qv + c).
        // The bf16 ds of 16-column chunk k goes to packed columns 32 hf + 8 k,
        // inside the score columns this thread has already read (chunk 0), so no
        // other warp's columns are touched and no barrier is needed.
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int c0 = 32 * hf + 16 * k;
          uint32_t dk8[8];
          // keys that no row of this lane quadrant can see: ds = 0, no loads
          const int t0 = k0 + kQK * qv + c0, i0 = q0 + 32 * qd;
          if (t0 > i0 + 31 || t0 + 15 <= i0 - W) {
#pragma unroll
            for (int j = 0; j < 8; ++j) dk8[j] = 0u;
            tc::tmem_st8(trow + kU2Ds + 32 * hf + 8 * k, dk8);
            continue;
          }
          float sv[16], dpv[16];
          tc::tmem_ld16(trow + kU2S + c0, sv);
          tc::tmem_ld16(trow + kU2Dp + c0, dpv);
          tc::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float d2[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int t = k0 + kQK * qv + c0 + 2 * j + e;
              const bool ok = t <= i && t > i - W && t >= 0 && i < L;
              const float p = ok ? __expf(sv[2 * j + e] * scale - lse_i) : 0.f;
              d2[e] = p * (dpv[2 * j + e] - dl_i);
            }
            dk8[j] = pack_bf16(d2[0], d2[1]);
          }
          tc::tmem_st8(trow + kU2Ds + 32 * hf + 8 * k, dk8);
        }
        tc::tmem_wait_st();
        tc::tc_fence_before();
        tc::named_bar_arrive(NB_PREADY, kCtaThreads);
      }
      tc::mbar_wait(&bars[QB_DQ], ph, 120);
      tc::tc_fence_after();
      float o[32];
      tc::tmem_ld32(trow + kU2Dq + 32 * hf, o);  // this warp's 32 columns of dq
      tc::tmem_wait_ld();
      if (i < L) store_grad32(dq, row * kDh + 32 * hf, o, scale, gdt);
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kU2Cols);
  }
}

// dk / dv for 64 < W <= 128: one CTA of 9 warps per 128 key rows [k0, k0 + 128)
// of one (batch row, key/value head). The query rows that see them,
// [k0, k0 + 256), come as items of 64 rows, four per query head, each with its
// q (q_lo) and dy tiles in one of two shared-memory stages:
//   warp 8 : s^T = k q^T (hi / lo terms), dp^T = v dy^T -> TMEM [128 x 64]
//            each; then dv += p^T dy and dk += ds^T q_hi with p^T, ds^T from
//            TMEM, summed over the items and the group's heads
//   8 warps: key row t = TMEM lane t, 32 of the item's 64 query columns each
// 256 TMEM columns and at most 98 KB of shared memory: two CTAs per SM.
constexpr int kIQ = 64;  // query rows per item
template <bool SPLIT>
struct Dkv128Smem {
  static constexpr size_t KT = kBK * 128, QT = kIQ * 128;
  static constexpr size_t kh = 0, kl = kh + KT, v = kl + (SPLIT ? KT : 0), st = v + KT;
  static constexpr size_t sq = 0, sql = QT, sdy = sql + (SPLIT ? QT : 0), sbytes = sdy + QT;
  static constexpr size_t rows = st + 2 * sbytes;  // [2 stages][lse | delta][64] fp32
  static constexpr size_t bars = rows + 2 * 2 * kIQ * 4, slot = bars + 64, bytes = slot + 16;
};
// TMEM: s^T [0, 64) with p^T (bf16 pairs) over it in [0, 16) and [32, 48);
// dp^T [64, 128) with ds^T over it in [64, 80) and [96, 112); dv [128, 192);
// dk [192, 256)
constexpr uint32_t kV2S = 0, kV2P = 0, kV2Ds = 64, kV2Dp = 64, kV2Dv = 128, kV2Dk = 192,
                   kV2Cols = 256;

template <bool SPLIT>
__global__ void __launch_bounds__(kCtaThreads, 2)
swa_bwd_dkv_tc128_kernel(const __grid_constant__ CUtensorMap tq,
                         const __grid_constant__ CUtensorMap tql,
                         const __grid_constant__ CUtensorMap tdy,
                         const __grid_constant__ CUtensorMap tk,
                         const __grid_constant__ CUtensorMap tkl,
                         const __grid_constant__ CUtensorMap tv, const float* __restrict__ lse,
                         const float* __restrict__ delta, int W, float scale, int H, int grp,
                         int L, int nkt, void* __restrict__ dk, void* __restrict__ dv, int gdt) {
  using SM = Dkv128Smem<SPLIT>;
  extern __shared__ __align__(1024) unsigned char smem[];
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) atomicExch(&tc::g_timeout_flag, 0x80000000u | 83u);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::bars);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + SM::slot);
  float* rows = reinterpret_cast<float*>(smem + SM::rows);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kt = blockIdx.x % nkt, bk = blockIdx.x / nkt;
  const int Hkv = H / grp, b = bk / Hkv, hk = bk - b * Hkv;
  const int k0 = kt * kBK;
  const int nit = 4 * grp;  // items: (head it / 4, query rows k0 + 64 (it % 4))
  constexpr uint32_t kTileK = kBK * 128, kTileQ = kIQ * 128;

  if (tid == 0) {
#pragma unroll
    for (int j = 0; j < 5; ++j) tc::mbar_init(&bars[j], 1);
    tc::fence_mbar_init();
  }
  if (warp == 8) {
    tc::tmem_alloc(tslot, kV2Cols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 8) {
    const bool issuer = lane == 0;
    auto load_stage = [&](int it) {  // item it's query / dy rows into stage it & 1
      const int h = hk * grp + (it >> 2), qr = k0 + kIQ * (it & 3);
      unsigned char* st = smem + SM::st + (it & 1) * SM::sbytes;
      uint64_t* bar = &bars[DB_Q0 + (it & 1)];
      tc::mbar_expect_tx(bar, (SPLIT ? 3 : 2) * kTileQ);
      tc::tma_load_4d(st + SM::sq, &tq, 0, qr, h, b, bar);
      if (SPLIT) tc::tma_load_4d(st + SM::sql, &tql, 0, qr, h, b, bar);
      tc::tma_load_4d(st + SM::sdy, &tdy, 0, qr, h, b, bar);
    };
    if (issuer) {
      tc::mbar_expect_tx(&bars[DB_KV], (SPLIT ? 3 : 2) * kTileK);
      tc::tma_load_4d(smem + SM::kh, &tk, 0, k0, hk, b, &bars[DB_KV]);
      if (SPLIT) tc::tma_load_4d(smem + SM::kl, &tkl, 0, k0, hk, b, &bars[DB_KV]);
      tc::tma_load_4d(smem + SM::v, &tv, 0, k0, hk, b, &bars[DB_KV]);
      load_stage(0);
      load_stage(1);
      tc::mbar_wait(&bars[DB_KV], 0, 121);
    }
    __syncwarp();
    for (int it = 0; it < nit; ++it) {
      const uint32_t ph = (uint32_t)it & 1u;
      unsigned char* st = smem + SM::st + (it & 1) * SM::sbytes;
      if (issuer) {
        tc::mbar_wait(&bars[DB_Q0 + (it & 1)], (uint32_t)(it >> 1) & 1u, 122);
        if (it > 0) tc::mbar_wait(&bars[DB_PD], ph ^ 1u, 123);  // p / ds of item it - 1 read
        tc::tc_fence_after();
        constexpr uint32_t id_s = tc::idesc_bf16(kBK, kIQ, 0, 0);  // K-major x K-major
        const uint32_t kh = smem_u32(smem + SM::kh), kl = smem_u32(smem + SM::kl),
                       va = smem_u32(smem + SM::v), qh = smem_u32(st + SM::sq),
                       ql = smem_u32(st + SM::sql), dya = smem_u32(st + SM::sdy);
#pragma unroll
        for (int j = 0; j < kDh / 16; ++j)
          tc::mma_ss(tmem + kV2S, tc::sdesc(kh + 32 * j, 16, 1024),
                     tc::sdesc(qh + 32 * j, 16, 1024), id_s, j > 0);
        if (SPLIT) {
#pragma unroll
          for (int j = 0; j < kDh / 16; ++j)
            tc::mma_ss(tmem + kV2S, tc::sdesc(kh + 32 * j, 16, 1024),
                       tc::sdesc(ql + 32 * j, 16, 1024), id_s, 1u);
#pragma unroll
          for (int j = 0; j < kDh / 16; ++j)
            tc::mma_ss(tmem + kV2S, tc::sdesc(kl + 32 * j, 16, 1024),
                       tc::sdesc(qh + 32 * j, 16, 1024), id_s, 1u);
        }
#pragma unroll
        for (int j = 0; j < kDh / 16; ++j)
          tc::mma_ss(tmem + kV2Dp, tc::sdesc(va + 32 * j, 16, 1024),
                     tc::sdesc(dya + 32 * j, 16, 1024), id_s, j > 0);
        tc::mma_commit(&bars[DB_SD]);
      }
      __syncwarp();
      tc::named_bar_sync(NB_PREADY, kCtaThreads);  // p^T and ds^T in TMEM
      if (issuer) {
        tc::tc_fence_after();
        constexpr uint32_t id_o = tc::idesc_bf16(kBK, kDh, 0, 1);  // TMEM x MN-major
        const uint32_t qh = smem_u32(st + SM::sq), dya = smem_u32(st + SM::sdy);
        // query rows 16 j.. of the item: packed columns 32 (j / 2) + 8 (j % 2)
#pragma unroll
        for (int j = 0; j < kIQ / 16; ++j)
          tc::mma_ts(tmem + kV2Dv, tmem + kV2P + 32 * (j >> 1) + 8 * (j & 1),
                     tc::sdesc(dya + 2048 * j, kTileQ, 1024), id_o, (it > 0 || j > 0) ? 1u : 0u);
#pragma unroll
        for (int j = 0; j < kIQ / 16; ++j)
          tc::mma_ts(tmem + kV2Dk, tmem + kV2Ds + 32 * (j >> 1) + 8 * (j & 1),
                     tc::sdesc(qh + 2048 * j, kTileQ, 1024), id_o, (it > 0 || j > 0) ? 1u : 0u);
        tc::mma_commit(&bars[DB_PD]);
        if (it + 2 < nit) {
          tc::mbar_wait(&bars[DB_PD], ph, 124);  // stage it & 1 read by every MMA of item it
          load_stage(it + 2);
        }
      }
      __syncwarp();
    }
  } else {
    const int qd = warp & 3, hf = warp >> 2;
    const int r = 32 * qd + lane, t = k0 + r;  // this thread's key row
    const uint32_t trow = tmem + ((uint32_t)(32 * qd) << 16);
    for (int it = 0; it < nit; ++it) {
      const uint32_t ph = (uint32_t)it & 1u;
      const int g = it >> 2, qr = k0 + kIQ * (it & 3);
      const size_t bh = (size_t)b * H + hk * grp + g;
      float* rl = rows + (it & 1) * 2 * kIQ;  // lse, then delta, of query rows qr + c
      for (int c = tid; c < kIQ; c += kThreads) {
        const int i = qr + c;
        rl[c] = i < L ? lse[bh * L + i] : 0.f;
        rl[kIQ + c] = i < L ? delta[bh * L + i] : 0.f;
      }
      tc::named_bar_sync(NB_ROWS, kThreads);
      tc::mbar_wait(&bars[DB_SD], ph, 125);
      tc::tc_fence_after();
      // p and ds of columns [32 hf, 32 hf + 32). Chunk k's bf16 p goes to packed
      // columns 32 hf + 8 k over s^T and its ds to the same columns over dp^T,
      // inside what this thread has already read (chunk 0): no other warp's
      // columns are touched and no barrier is needed.
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        uint32_t pk[8], dk8[8];
        // query rows that see no key row of this lane quadrant: p = ds = 0, no loads
        const int c0 = 32 * hf + 16 * k, tq0 = k0 + 32 * qd;
        if (qr + c0 + 15 < tq0 || qr + c0 >= tq0 + 31 + W) {
#pragma unroll
          for (int j = 0; j < 8; ++j) pk[j] = dk8[j] = 0u;
          tc::tmem_st8(trow + kV2P + 32 * hf + 8 * k, pk);
          tc::tmem_st8(trow + kV2Ds + 32 * hf + 8 * k, dk8);
          continue;
        }
        float sv[16], dpv[16];
        tc::tmem_ld16(trow + kV2S + 32 * hf + 16 * k, sv);
        tc::tmem_ld16(trow + kV2Dp + 32 * hf + 16 * k, dpv);
        tc::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float p2[2], d2[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int c = 32 * hf + 16 * k + 2 * j + e, i = qr + c;
            const bool ok = i >= t && i < t + W && i < L && t < L;
            const float p = ok ? __expf(sv[2 * j + e] * scale - rl[c]) : 0.f;
            p2[e] = p;
            d2[e] = p * (dpv[2 * j + e] - rl[kIQ + c]);
          }
          pk[j] = pack_bf16(p2[0], p2[1]);
          dk8[j] = pack_bf16(d2[0], d2[1]);
        }
        tc::tmem_st8(trow + kV2P + 32 * hf + 8 * k, pk);
        tc::tmem_st8(trow + kV2Ds + 32 * hf + 8 * k, dk8);
      }
      tc::tmem_wait_st();
      tc::tc_fence_before();
      tc::named_bar_arrive(NB_PREADY, kCtaThreads);
    }
    // dv (warps of half 0) and dk (half 1) of this key row, summed over the items
    tc::mbar_wait(&bars[DB_PD], (uint32_t)(nit - 1) & 1u, 126);
    tc::tc_fence_after();
    const size_t orow = ((size_t)bk * L + t) * kDh;
#pragma unroll 1
    for (int db = 0; db < 2; ++db) {
      float o[32];
      tc::tmem_ld32(trow + (hf ? kV2Dk : kV2Dv) + 32 * db, o);
      tc::tmem_wait_ld();
      if (t < L) store_grad32(hf ? dk : dv, orow + 32 * db, o, hf ? scale : 1.f, gdt);
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kV2Cols);
  }
}

// Tensor maps of the backward operands ([B, H or Hkv, L, 64] contiguous bf16);
// false when one cannot be built.
bool bwd_maps(const bf16* q, const bf16* ql, const bf16* dy, const bf16* k, const bf16* kl,
              const bf16* v, int B, int H, int Hkv, int L, int qrows, int krows, CUtensorMap* m) {
  const long long sl = kDh, sh = (long long)L * kDh;
  if (!make_tc_map(&m[0], q, L, H, B, H * sh, sh, sl, qrows) ||
      !make_tc_map(&m[2], dy, L, H, B, H * sh, sh, sl, qrows) ||
      !make_tc_map(&m[3], k, L, Hkv, B, Hkv * sh, sh, sl, krows) ||
      !make_tc_map(&m[5], v, L, Hkv, B, Hkv * sh, sh, sl, krows))
    return false;
  if (!ql) {
    m[1] = m[0], m[4] = m[3];
    return true;
  }
  return make_tc_map(&m[1], ql, L, H, B, H * sh, sh, sl, qrows) &&
         make_tc_map(&m[4], kl, L, Hkv, B, Hkv * sh, sh, sl, krows);
}

template <typename Kern>
int ensure_tc_smem(Kern kern, size_t bytes, bool* done) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)bytes);
    if (e != cudaSuccess) {
      set_error(std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
      return LZ_ERR_CUDA;
    }
    done[dev] = true;
  }
  return LZ_OK;
}

// Shared memory a 256-TMEM-column kernel asks for at least: more than a third
// of the SM's 227 KB, so at most two of its CTAs share an SM (a third would
// wait inside the TMEM allocation).
constexpr size_t kTwoPerSm = 80 * 1024;

int swa_fwd_tc128(const bf16* q, const bf16* k, const bf16* v, const bf16* ql, const bf16* kl,
                  const float* meta, int n_meta, int W, bf16* y, const SwaSaved& sv, int B,
                  int H, int Hkv, int L, cudaStream_t st) {
  const long long sl = kDh, sh = (long long)L * kDh;
  const bool split = ql != nullptr;
  CUtensorMap mq, mk, mv, mql, mkl;
  if (!make_tc_map(&mq, q, L, H, B, H * sh, sh, sl, kQ) ||
      !make_tc_map(&mk, k, L, Hkv, B, Hkv * sh, sh, sl, kNK2) ||
      !make_tc_map(&mv, v, L, Hkv, B, Hkv * sh, sh, sl, kNK2))
    return LZ_ERR_UNSUPPORTED;
  if (split) {
    if (!make_tc_map(&mql, ql, L, H, B, H * sh, sh, sl, kQ) ||
        !make_tc_map(&mkl, kl, L, Hkv, B, Hkv * sh, sh, sl, kNK2))
      return LZ_ERR_UNSUPPORTED;
  } else {
    mql = mq, mkl = mk;
  }
  auto kern = split ? swa_fwd_tc128_kernel<false, true, float>
                    : swa_fwd_tc128_kernel<false, false, float>;
  const size_t smem = split ? Fwd128Smem<true>::bytes : Fwd128Smem<false>::bytes;
  static bool done[2][64] = {{false}};
  const int rc = ensure_tc_smem(kern, smem, done[split]);
  if (rc) return rc;
  const int nqb = ceil_div(L, kQ);
  kern<<<(unsigned)((long long)B * Hkv * nqb), kThreads, smem, st>>>(
      mq, mk, mv, mql, mkl, nullptr, nullptr, 0, 0, meta, n_meta, W,
      kLog2e / sqrtf((float)kDh), H, H / Hkv, L, nqb, y, sv.lse, sv.y32, nullptr, nullptr,
      nullptr, nullptr);
  count_launches(1);
  return check_launch("swa_fwd_tc128_kernel");
}

// The fused rotation for windows 65 ... 128 (bf16 projections read in place).
template <typename CT>
int swa_rope_fwd_tc128(const SwaRopeArgs& a, const SwaSaved& sv, cudaStream_t st) {
  CUtensorMap mq, mk, mv;
  if (!make_tc_map(&mq, a.q, a.L, a.H, a.B, a.q_sb, a.q_sh, a.q_sl, kQ) ||
      !make_tc_map(&mk, a.k, a.L, a.Hkv, a.B, a.k_sb, a.k_sh, a.k_sl, kNK2) ||
      !make_tc_map(&mv, a.v, a.L, a.Hkv, a.B, a.v_sb, a.v_sh, a.v_sl, kNK2))
    return LZ_ERR_UNSUPPORTED;
  auto kern = swa_fwd_tc128_kernel<true, true, CT>;
  static bool done[64] = {false};
  const int rc = ensure_tc_smem(kern, Fwd128Smem<true>::bytes, done);
  if (rc) return rc;
  const int nqb = ceil_div(a.L, kQ);
  kern<<<(unsigned)((long long)a.B * a.Hkv * nqb), kThreads, Fwd128Smem<true>::bytes, st>>>(
      mq, mk, mv, mq, mk, static_cast<const CT*>(a.cos), static_cast<const CT*>(a.sin), a.cs_sb,
      a.cs_sl, a.meta, a.n_meta, a.window, kLog2e / sqrtf((float)kDh), a.H, a.H / a.Hkv, a.L,
      nqb, a.y, sv.lse, sv.y32, a.q_hi, a.q_lo, a.k_hi, a.k_lo);
  count_launches(1);
  return check_launch("swa_fwd_tc128_kernel");
}

int swa_bwd_dq_tc128(const CUtensorMap* m, bool split, const float* lse, const float* delta,
                     int W, void* dq, int gdt, int B, int H, int Hkv, int L, cudaStream_t st) {
  auto kern = split ? swa_bwd_dq_tc128_kernel<true> : swa_bwd_dq_tc128_kernel<false>;
  const size_t smem = split ? Dq128Smem<true>::bytes : Dq128Smem<false>::bytes;
  static bool done[2][64] = {{false}};
  const int rc = ensure_tc_smem(kern, smem, done[split]);
  if (rc) return rc;
  const int nqb = ceil_div(L, kQ);
  kern<<<(unsigned)((long long)B * Hkv * nqb), kCtaThreads, smem, st>>>(
      m[0], m[1], m[2], m[3], m[4], m[5], lse, delta, W, 1.f / sqrtf((float)kDh), H, H / Hkv, L,
      nqb, dq, gdt);
  count_launches(1);
  return check_launch("swa_bwd_dq_tc128_kernel");
}

int swa_bwd_dkv_tc128(const CUtensorMap* m, bool split, const float* lse, const float* delta,
                      int W, void* dk, void* dv, int gdt, int B, int H, int Hkv, int L,
                      cudaStream_t st) {
  auto kern = split ? swa_bwd_dkv_tc128_kernel<true> : swa_bwd_dkv_tc128_kernel<false>;
  // 256 TMEM columns per CTA: at most two CTAs per SM, or a third would wait
  // inside the TMEM allocation; the bf16 variant's 67 KB alone would let three in
  const size_t smem =
      std::max(split ? Dkv128Smem<true>::bytes : Dkv128Smem<false>::bytes, kTwoPerSm);
  static bool done[2][64] = {{false}};
  const int rc = ensure_tc_smem(kern, smem, done[split]);
  if (rc) return rc;
  const int nkt = ceil_div(L, kBK);
  kern<<<(unsigned)((long long)B * Hkv * nkt), kCtaThreads, smem, st>>>(
      m[0], m[1], m[2], m[3], m[4], m[5], lse, delta, W, 1.f / sqrtf((float)kDh), H, H / Hkv, L,
      nkt, dk, dv, gdt);
  count_launches(1);
  return check_launch("swa_bwd_dkv_tc128_kernel");
}

}  // namespace

bool swa_tc_enabled() { return g_swa_tc.load(std::memory_order_relaxed) != 0; }
int swa_set_tc(int on) { return g_swa_tc.exchange(on ? 1 : 0); }

int swa_rope_fwd_tc(const SwaRopeArgs& a, const SwaSaved& sv, cudaStream_t st) {
  if (!swa_tc_enabled() || a.D != kDh || a.x_dtype != LZ_DTYPE_BF16 || a.window < 1 ||
      a.window > kH2)
    return LZ_ERR_UNSUPPORTED;
  const long long ces = a.cs_dtype == LZ_DTYPE_F32 ? 4 : 2;
  if (!aligned16(a.cos) || !aligned16(a.sin) || (a.cs_sl * ces) % 16 || (a.cs_sb * ces) % 16)
    return LZ_ERR_UNSUPPORTED;  // the rotation reads cos / sin rows with 16-byte loads
  if (a.q_hi && (!aligned16(a.q_hi) || !aligned16(a.q_lo) || !aligned16(a.k_hi) ||
                 !aligned16(a.k_lo)))
    return LZ_ERR_UNSUPPORTED;
  if (!aligned16(a.y) || (sv.y32 && !aligned16(sv.y32))) return LZ_ERR_UNSUPPORTED;
  if (a.window > kNK - kQ)
    return a.cs_dtype == LZ_DTYPE_F32 ? swa_rope_fwd_tc128<float>(a, sv, st)
                                      : swa_rope_fwd_tc128<bf16>(a, sv, st);
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
  if (!swa_tc_enabled() || D != kDh || W < 1 || W > kH2) return LZ_ERR_UNSUPPORTED;
  if (!aligned16(y) || (sv.y32 && !aligned16(sv.y32))) return LZ_ERR_UNSUPPORTED;
  if (W > kNK - kQ)
    return swa_fwd_tc128(q, k, v, ql, kl, meta, n_meta, W, y, sv, B, H, Hkv, L, st);
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
  // bf16 operands: the persistent kernel, two CTAs per SM, once every CTA gets
  // at least 8 tiles (with fewer, whole tiles split unevenly over the CTAs and
  // the one-tile-per-CTA kernel's scheduling does better: B = 4, 8 key / value
  // heads, L = 2048 measured 47 us against 45)
  const int nqb = ceil_div(L, kQ);
  const long long ntiles = (long long)B * Hkv * nqb;
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  if (nsm <= 0) nsm = 148;
  if (ntiles < 16ll * nsm || ntiles >= (1ll << 31))
    return launch_swa_tc<false, false, float>(mq, mk, mv, mq, mk, nullptr, nullptr, 0, 0, meta,
                                              n_meta, W, B, H, Hkv, L, y, sv, nullptr, nullptr,
                                              nullptr, nullptr, st);
  static bool done_p[64] = {false};
  const int rc = ensure_tc_smem(swa_fwd_tc_persist_kernel, FwdPersistSmem::bytes, done_p);
  if (rc) return rc;
  const int grid = (int)std::min<long long>(ntiles, 2ll * nsm);
  swa_fwd_tc_persist_kernel<<<grid, kCtaThreads, FwdPersistSmem::bytes, st>>>(
      mq, mk, mv, meta, n_meta, W, kLog2e / sqrtf((float)kDh), H, H / Hkv, L, nqb, (int)ntiles,
      y, sv.lse, sv.y32);
  count_launches(1);
  return check_launch("swa_fwd_tc_persist_kernel");
}

int swa_bwd_dkv_tc(const bf16* q, const bf16* k, const bf16* v, const bf16* ql, const bf16* kl,
                   const bf16* dy, const float* lse, const float* delta, int W, void* dk,
                   void* dv, int gdt, int B, int H, int Hkv, int L, int D, cudaStream_t st) {
  if (!swa_tc_enabled() || D != kDh || W < 1 || W > kH2) return LZ_ERR_UNSUPPORTED;
  if (!aligned16(dk) || !aligned16(dv)) return LZ_ERR_UNSUPPORTED;
  CUtensorMap m[6];
  if (W > kBQ - kBK) {
    if (!bwd_maps(q, ql, dy, k, kl, v, B, H, Hkv, L, kIQ, kBK, m)) return LZ_ERR_UNSUPPORTED;
    return swa_bwd_dkv_tc128(m, ql != nullptr, lse, delta, W, dk, dv, gdt, B, H, Hkv, L, st);
  }
  if (!bwd_maps(q, ql, dy, k, kl, v, B, H, Hkv, L, kBQ, kBK, m)) return LZ_ERR_UNSUPPORTED;
  const bool split = ql != nullptr;
  const int nkt = ceil_div(L, kBK);
  if (!split) {  // bf16 operands: the persistent kernel, one CTA per SM
    static bool done_p[64] = {false};
    const int rc = ensure_tc_smem(swa_bwd_dkv_tc_persist_kernel, DkvPersistSmem::bytes, done_p);
    if (rc) return rc;
    const long long ntiles = (long long)B * Hkv * nkt;
    if (ntiles >= (1ll << 31)) return LZ_ERR_UNSUPPORTED;
    int dev = 0, nsm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    const int grid = (int)std::min<long long>(ntiles, nsm > 0 ? nsm : 148);
    swa_bwd_dkv_tc_persist_kernel<<<grid, kCtaThreads, DkvPersistSmem::bytes, st>>>(
        m[0], m[2], m[3], m[5], lse, delta, W, 1.f / sqrtf((float)kDh), H, H / Hkv, L, nkt,
        (int)ntiles, dk, dv, gdt);
    count_launches(1);
    return check_launch("swa_bwd_dkv_tc_persist_kernel");
  }
  auto kern = split ? swa_bwd_dkv_tc_kernel<true> : swa_bwd_dkv_tc_kernel<false>;
  static bool done[2][64] = {{false}};
  const int rc = ensure_tc_smem(kern, DkvTcSmem::bytes, done[split]);
  if (rc) return rc;
  kern<<<(unsigned)((long long)B * Hkv * nkt), kCtaThreads, DkvTcSmem::bytes, st>>>(
      m[0], m[1], m[2], m[3], m[4], m[5], lse, delta, W, 1.f / sqrtf((float)kDh), H, H / Hkv, L,
      nkt, dk, dv, gdt);
  count_launches(1);
  return check_launch("swa_bwd_dkv_tc_kernel");
}

int swa_bwd_dq_tc(const bf16* q, const bf16* k, const bf16* v, const bf16* ql, const bf16* kl,
                  const bf16* dy, const float* lse, const float* delta, int W, void* dq, int gdt,
                  int B, int H, int Hkv, int L, int D, cudaStream_t st) {
  if (!swa_tc_enabled() || D != kDh || W < 1 || W > kH2) return LZ_ERR_UNSUPPORTED;
  if (!aligned16(dq)) return LZ_ERR_UNSUPPORTED;
  CUtensorMap m[6];
  if (W > kNK - kQ) {
    if (!bwd_maps(q, ql, dy, k, kl, v, B, H, Hkv, L, kQ, kNK2, m)) return LZ_ERR_UNSUPPORTED;
    return swa_bwd_dq_tc128(m, ql != nullptr, lse, delta, W, dq, gdt, B, H, Hkv, L, st);
  }
  if (!bwd_maps(q, ql, dy, k, kl, v, B, H, Hkv, L, kQ, kNK, m)) return LZ_ERR_UNSUPPORTED;
  const bool split = ql != nullptr;
  if (!split) {  // bf16 operands: the persistent kernel, one CTA per SM
    static bool done_p[64] = {false};
    const int rc = ensure_tc_smem(swa_bwd_dq_tc_persist_kernel, DqPersistSmem::bytes, done_p);
    if (rc) return rc;
    const int nqb = ceil_div(L, kQ);
    const long long ntiles = (long long)B * Hkv * nqb;
    if (ntiles >= (1ll << 31)) return LZ_ERR_UNSUPPORTED;
    int dev = 0, nsm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    const int grid = (int)std::min<long long>(ntiles, nsm > 0 ? nsm : 148);
    swa_bwd_dq_tc_persist_kernel<<<grid, kCtaThreads, DqPersistSmem::bytes, st>>>(
        m[0], m[2], m[3], m[5], lse, delta, W, 1.f / sqrtf((float)kDh), H, H / Hkv, L, nqb,
        (int)ntiles, dq, gdt);
    count_launches(1);
    return check_launch("swa_bwd_dq_tc_persist_kernel");
  }
  auto kern = split ? swa_bwd_dq_tc_kernel<true> : swa_bwd_dq_tc_kernel<false>;
  const size_t smem = split ? DqTcSmem<true>::bytes : DqTcSmem<false>::bytes;
  static bool done[2][64] = {{false}};
  const int rc = ensure_tc_smem(kern, smem, done[split]);
  if (rc) return rc;
  const int nqb = ceil_div(L, kQ);
  kern<<<(unsigned)((long long)B * Hkv * nqb), kCtaThreads, smem, st>>>(
      m[0], m[1], m[2], m[3], m[4], m[5], lse, delta, W, 1.f / sqrtf((float)kDh), H, H / Hkv, L,
      nqb, dq, gdt);
  count_launches(1);
  return check_launch("swa_bwd_dq_tc_kernel");
}

int swa_tc_timeout_flag(unsigned int* out) { return tc::read_timeout_flag_here(out); }
int swa_tc_timeout_clear() { return tc::clear_timeout_flag_here(); }

}  // namespace lz

extern "C" int lz_swa_set_tc(int on) { return lz::swa_set_tc(on); }
