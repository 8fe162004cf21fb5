// Hedgehog feature map, fused: f = [softmax(x W^T), softmax(-x W^T)] in bf16
// (reference: src/lizard_attention.py:9-11), the GLA prologue that turns a
// head's queries / keys x [R, Dh] into features [R, 2 Fd].
//
// Forward, per 64-row tile and 8 warps (warp = 16 rows x half of the feature
// columns): xw = x W^T on the tensor cores (mma.sync bf16 -> fp32; an fp32 x
// or W enters as bf16 hi + lo parts, xw = hi.hi + hi.lo + lo.hi, so the
// logits carry ~16 mantissa bits, as the reference's fp32 matmul does to
// within the bf16 output rounding), both softmaxes in registers (quad shuffles,
// then the two column halves through shared memory), and the bf16 features
// written from the fragments with 16-byte stores after a quad transpose. The
// next tile's x is loaded into registers while this tile computes. The
// reference materialises xw, two fp32 softmaxes and their concatenation, and
// GLA then casts them.
//
// Backward (the autograd of the same three torch ops): per tile, recompute xw
// and both softmaxes, then
//   g = p+ (df+ - sum p+ df+) - p- (df- - sum p- df-)     (d xw, fp32)
//   dx = g W,  dW += g^T x
// with g entering both products as bf16 hi + lo. dW is accumulated per CTA in
// registers over the CTA's tiles (persistent grid) and reduced over CTAs in a
// fixed order by a second kernel: deterministic.
//
// Bandwidth-bound: 2 Dh Fd flop per (Dh + 2 Fd) x 2-4 bytes.
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "rope_math.cuh"
#include "tc.cuh"
#include <atomic>

namespace lz {

namespace {

constexpr int kR = 64;   // rows per tile
constexpr int kT = 256;  // threads: 8 warps = 4 row blocks x 2 column halves

template <int DHP, int FDP>
struct HhSmem {
  static constexpr int LDX = DHP + 8, LDW = DHP + 8, LDG = FDP + 8;
  static constexpr size_t whi = 0;
  static constexpr size_t wlo = whi + (size_t)FDP * LDW * 2;
  static constexpr size_t xhi = wlo + (size_t)FDP * LDW * 2;
  static constexpr size_t xlo = xhi + (size_t)kR * LDX * 2;
  static constexpr size_t red = xlo + (size_t)kR * LDX * 2;  // 4 stats x 2 halves x 64 rows
  static constexpr size_t fwd_bytes = red + 4 * 2 * kR * 4;
  static constexpr size_t ghi = fwd_bytes;                   // backward: g hi / lo
  static constexpr size_t glo = ghi + (size_t)kR * LDG * 2;
  static constexpr size_t bwd_bytes = glo + (size_t)kR * LDG * 2;
};

template <typename T>
__device__ __forceinline__ float ld_f(const T* p, size_t i);
template <>
__device__ __forceinline__ float ld_f<float>(const float* p, size_t i) { return p[i]; }
template <>
__device__ __forceinline__ float ld_f<bf16>(const bf16* p, size_t i) {
  return __bfloat162float(p[i]);
}

// rows x cols of a row-major [*, ld] matrix -> bf16 hi / lo tiles, zero padded
template <typename T, int ROWS, int COLS>
__device__ __forceinline__ void split_tile(bf16* hi, bf16* lo, int lds, const T* g, int ld,
                                           int r0, int nrows, int ncols) {
  for (int i = threadIdx.x; i < ROWS * COLS; i += kT) {
    const int r = i / COLS, c = i % COLS;
    const float x = (r0 + r < nrows && c < ncols) ? ld_f<T>(g, (size_t)(r0 + r) * ld + c) : 0.f;
    const bf16 h = __float2bfloat16_rn(x);
    hi[r * lds + c] = h;
    lo[r * lds + c] = __float2bfloat16_rn(x - __bfloat162float(h));
  }
}

// Row r of x (r over the B*H*L rows in (batch, head, token) order) starts at
// element b*sb + h*sh + t*sl, so a projection output [B, L, H*Dh] is read in
// place as [B, H, L, Dh]; a contiguous [R, Dh] x is H = 1, L = R, sl = Dh.
struct XRows {
  int H, L;
  long long sb, sh, sl;
  __host__ __device__ __forceinline__ size_t off(long long r) const {
    if (H == 1 && r < L) return (size_t)(r * sl);  // one head (a contiguous x): rows are tokens
    const int ri = (int)r, t = ri % L, bh = ri / L;  // rows < 2^31 (checked by the host)
    return (size_t)((long long)(bh / H) * sb + (long long)(bh % H) * sh + (long long)t * sl);
  }
};

// rows x cols of x -> bf16 hi / lo tiles, zero padded
template <typename T, int ROWS, int COLS>
__device__ __forceinline__ void split_rows(bf16* hi, bf16* lo, int lds, const T* g,
                                           const XRows& m, int r0, int nrows, int ncols) {
  for (int i = threadIdx.x; i < ROWS * COLS; i += kT) {
    const int r = i / COLS, c = i % COLS;
    const float x = (r0 + r < nrows && c < ncols) ? ld_f<T>(g, m.off(r0 + r) + c) : 0.f;
    const bf16 h = __float2bfloat16_rn(x);
    hi[r * lds + c] = h;
    lo[r * lds + c] = __float2bfloat16_rn(x - __bfloat162float(h));
  }
}

// Vector loads of one 64-row tile of x (fp32 or bf16) into registers,
// 16 bytes per load, zero beyond R; stored to the hi / lo tiles afterwards.
template <typename XT, int DHP>
struct XTile {
  static constexpr int EPV = 16 / sizeof(XT);
  static constexpr int VPR = DHP / EPV;
  static constexpr int NV = (kR * VPR + kT - 1) / kT;
  uint4 v[NV];
  __device__ __forceinline__ void load(const XT* x, const XRows& m, int r0, int R, int Dh) {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int i = threadIdx.x + kT * k;
      const int r = i / VPR, c = (i % VPR) * EPV;
      v[k] = (i < kR * VPR && r0 + r < R && c < Dh)
                 ? *reinterpret_cast<const uint4*>(x + m.off(r0 + r) + c)
                 : make_uint4(0u, 0u, 0u, 0u);
    }
  }
  __device__ __forceinline__ void store(bf16* hi, bf16* lo, int lds) const {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int i = threadIdx.x + kT * k;
      if (i >= kR * VPR) continue;
      const int r = i / VPR, c = (i % VPR) * EPV;
      if constexpr (sizeof(XT) == 4) {
        const float f[4] = {__uint_as_float(v[k].x), __uint_as_float(v[k].y),
                            __uint_as_float(v[k].z), __uint_as_float(v[k].w)};
        uint32_t h[2], l[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          h[j] = pack_bf16(f[2 * j], f[2 * j + 1]);
          l[j] = pack_bf16(f[2 * j] - bf16_lo(h[j]), f[2 * j + 1] - bf16_hi(h[j]));
        }
        *reinterpret_cast<uint2*>(hi + r * lds + c) = make_uint2(h[0], h[1]);
        *reinterpret_cast<uint2*>(lo + r * lds + c) = make_uint2(l[0], l[1]);
      } else {
        *reinterpret_cast<uint4*>(hi + r * lds + c) = v[k];
      }
    }
  }
};

__device__ __forceinline__ uint32_t sel4(uint32_t a, uint32_t b, uint32_t c, uint32_t d, int i) {
  return i == 0 ? a : i == 1 ? b : i == 2 ? c : d;
}
// Quad transpose of 32-bit words. In: lane cq holds word in[j] of n-tile 4k+j
// (the fragment pair at columns 2 cq, 2 cq + 1 of that tile). Out: lane cq
// holds words 0..3 of n-tile 4k + cq, i.e. its 8 consecutive columns. The
// same exchange turns 8 loaded consecutive columns back into fragment pairs.
__device__ __forceinline__ void quad_xpose(const uint32_t (&in)[4], uint32_t (&out)[4]) {
  const int lane = threadIdx.x & 31, cq = lane & 3;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const uint32_t send = sel4(in[0], in[1], in[2], in[3], (cq + r) & 3);
    const uint32_t recv = __shfl_sync(0xffffffffu, send, (lane & ~3) | ((cq - r) & 3));
    const int slot = (cq - r) & 3;
#pragma unroll
    for (int q = 0; q < 4; ++q) out[q] = (q == slot) ? recv : (r == 0 ? 0u : out[q]);
  }
}

// xw for this warp's 16 rows (row block rb) and FDP / 2 columns from c0;
// XS: x has a lo part (fp32 x). W (fp32) always has one.
template <int DHP, int FDP, bool XS>
__device__ __forceinline__ void logits(float (&acc)[FDP / 16][4], const bf16* xh, const bf16* xl,
                                       const bf16* wh, const bf16* wl, int rb, int c0) {
  using SM = HhSmem<DHP, FDP>;
  constexpr int NTH = FDP / 16;
#pragma unroll
  for (int c = 0; c < NTH; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[c][e] = 0.f;
#pragma unroll
  for (int k0 = 0; k0 < DHP; k0 += 16) {
    uint32_t ah[4], al[4];
    lda_rm(ah, xh, SM::LDX, 16 * rb, k0);
    if constexpr (XS) lda_rm(al, xl, SM::LDX, 16 * rb, k0);
#pragma unroll
    for (int np = 0; np < NTH / 2; ++np) {
      uint32_t bh[4], bl[4];
      ldb_nk(bh, wh, SM::LDW, c0 + 16 * np, k0);
      mma16816(acc[2 * np], ah, bh[0], bh[1]);
      mma16816(acc[2 * np + 1], ah, bh[2], bh[3]);
      ldb_nk(bl, wl, SM::LDW, c0 + 16 * np, k0);
      mma16816(acc[2 * np], ah, bl[0], bl[1]);
      mma16816(acc[2 * np + 1], ah, bl[2], bl[3]);
      if constexpr (XS) {
        mma16816(acc[2 * np], al, bh[0], bh[1]);
        mma16816(acc[2 * np + 1], al, bh[2], bh[3]);
      }
    }
  }
}

__device__ __forceinline__ float quad_max(float x) {
  x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 1));
  return fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 2));
}

// Row statistic over the two column halves: every quad writes its half's
// value for rows `row` and `row + 8`, then all read both (fixed order).
__device__ __forceinline__ void exchange2(float* red, int stat, int half, int row, float (&v)[2],
                                          int op /* 0 max, 1 min, 2 sum */) {
  const int cq = threadIdx.x & 3;
  if (cq == 0) {
    red[(stat * 2 + half) * kR + row] = v[0];
    red[(stat * 2 + half) * kR + row + 8] = v[1];
  }
  __syncthreads();
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const float a = red[(stat * 2 + 0) * kR + row + 8 * h];
    const float b = red[(stat * 2 + 1) * kR + row + 8 * h];
    v[h] = op == 0 ? fmaxf(a, b) : op == 1 ? fminf(a, b) : a + b;
  }
}

// Both softmaxes of this warp's fragments (columns c0 + ..): acc -> p+, pm -> p-.
// FULL: Fd == FDP, no column is masked.
template <int FDP, bool FULL>
__device__ __forceinline__ void softmaxes(float (&acc)[FDP / 16][4], float (&pm)[FDP / 16][4],
                                          int c0, int Fd, float* red, int half, int row) {
  constexpr int NTH = FDP / 16;
  const int cq = threadIdx.x & 3;
  float mx[2] = {-INFINITY, -INFINITY}, mn[2] = {INFINITY, INFINITY};
#pragma unroll
  for (int nt = 0; nt < NTH; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int c = c0 + 8 * nt + 2 * cq + (e & 1);
      if (FULL || c < Fd) {
        mx[e >> 1] = fmaxf(mx[e >> 1], acc[nt][e]);
        mn[e >> 1] = fminf(mn[e >> 1], acc[nt][e]);
      }
    }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    mx[h] = quad_max(mx[h]);
    mn[h] = -quad_max(-mn[h]);
  }
  exchange2(red, 0, half, row, mx, 0);
  exchange2(red, 1, half, row, mn, 1);
  float sp[2] = {0.f, 0.f}, sm[2] = {0.f, 0.f};
#pragma unroll
  for (int nt = 0; nt < NTH; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int c = c0 + 8 * nt + 2 * cq + (e & 1), h = e >> 1;
      const bool ok = FULL || c < Fd;
      const float ep = ok ? __expf(acc[nt][e] - mx[h]) : 0.f;
      const float em = ok ? __expf(mn[h] - acc[nt][e]) : 0.f;
      acc[nt][e] = ep;
      pm[nt][e] = em;
      sp[h] += ep;
      sm[h] += em;
    }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    sp[h] = quad_sum(sp[h]);
    sm[h] = quad_sum(sm[h]);
  }
  exchange2(red, 2, half, row, sp, 2);
  exchange2(red, 3, half, row, sm, 2);
  const float ip[2] = {1.f / sp[0], 1.f / sp[1]}, im[2] = {1.f / sm[0], 1.f / sm[1]};
#pragma unroll
  for (int nt = 0; nt < NTH; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      acc[nt][e] *= ip[e >> 1];
      pm[nt][e] *= im[e >> 1];
    }
}

template <typename XT, int DHP, int FDP, bool FULL>
__global__ void __launch_bounds__(kT)
hedgehog_fwd_kernel(const XT* __restrict__ x, XRows xm, const float* __restrict__ w, int R,
                    int Dh, int Fd, int vec, bf16* __restrict__ f) {
  using SM = HhSmem<DHP, FDP>;
  constexpr int NTH = FDP / 16;
  extern __shared__ __align__(128) unsigned char smem[];
  bf16* wh = reinterpret_cast<bf16*>(smem + SM::whi);
  bf16* wl = reinterpret_cast<bf16*>(smem + SM::wlo);
  bf16* xh = reinterpret_cast<bf16*>(smem + SM::xhi);
  bf16* xl = reinterpret_cast<bf16*>(smem + SM::xlo);
  float* red = reinterpret_cast<float*>(smem + SM::red);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, cq = lane & 3;
  const int rb = warp & 3, half = warp >> 2, c0 = half * (FDP / 2);
  const int lrow = 16 * rb + gq;  // this thread's tile rows: lrow, lrow + 8
  split_tile<float, FDP, DHP>(wh, wl, SM::LDW, w, Dh, 0, Fd, Dh);
  const int ntiles = (R + kR - 1) / kR;
  const int F2 = 2 * Fd;
  XTile<XT, DHP> xt;
  if (vec && (int)blockIdx.x < ntiles) xt.load(x, xm, blockIdx.x * kR, R, Dh);
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int r0 = tile * kR;
    __syncthreads();  // the previous tile's x is consumed; W is staged
    if (vec)
      xt.store(xh, xl, SM::LDX);
    else
      split_rows<XT, kR, DHP>(xh, xl, SM::LDX, x, xm, r0, R, Dh);
    __syncthreads();
    if (vec && tile + (int)gridDim.x < ntiles) xt.load(x, xm, r0 + gridDim.x * kR, R, Dh);
    float acc[NTH][4], pm[NTH][4];
    logits<DHP, FDP, sizeof(XT) == 4>(acc, xh, xl, wh, wl, rb, c0);
    softmaxes<FDP, FULL>(acc, pm, c0, Fd, red, half, lrow);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = r0 + lrow + 8 * h;
      bf16* out = f + (size_t)row * F2;
      bool done = false;
      if constexpr (NTH % 4 == 0) {
        if (vec && (Fd % 8) == 0) {
#pragma unroll
          for (int k = 0; k < NTH / 4; ++k) {
            uint32_t ip[4], im[4], op[4], om[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              ip[j] = pack_bf16(acc[4 * k + j][2 * h], acc[4 * k + j][2 * h + 1]);
              im[j] = pack_bf16(pm[4 * k + j][2 * h], pm[4 * k + j][2 * h + 1]);
            }
            quad_xpose(ip, op);
            quad_xpose(im, om);
            const int c = c0 + 8 * (4 * k + cq);
            if (row < R && (FULL || c < Fd)) {
              *reinterpret_cast<uint4*>(out + c) = make_uint4(op[0], op[1], op[2], op[3]);
              *reinterpret_cast<uint4*>(out + Fd + c) = make_uint4(om[0], om[1], om[2], om[3]);
            }
          }
          done = true;
        }
      }
      if (!done && row < R) {
#pragma unroll
        for (int nt = 0; nt < NTH; ++nt) {
          const int c = c0 + 8 * nt + 2 * cq;
          if (c < Fd) {
            out[c] = __float2bfloat16_rn(acc[nt][2 * h]);
            out[Fd + c] = __float2bfloat16_rn(pm[nt][2 * h]);
          }
          if (c + 1 < Fd) {
            out[c + 1] = __float2bfloat16_rn(acc[nt][2 * h + 1]);
            out[Fd + c + 1] = __float2bfloat16_rn(pm[nt][2 * h + 1]);
          }
        }
      }
    }
  }
}

// The fragment pairs of df for this warp's columns: pr[nt][h] = columns
// c0 + 8 nt + 2 cq, +1 of row `row + 8 h`, read from `src` = the row's first
// column of the half (p+ or p-). With vec, 16-byte loads of 8 consecutive
// columns and a quad transpose; else element loads.
template <typename GT, int NTH>
__device__ __forceinline__ void load_df(float2 (&pr)[NTH][2], const GT* __restrict__ df,
                                        int row, int R, int F2, int cbase, int Fd, int c0,
                                        bool vec) {
  const int cq = threadIdx.x & 3;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = row + 8 * h;
    const GT* src = df + (size_t)r * F2 + cbase;
    bool done = false;
    if constexpr (NTH % 4 == 0) {
      if (vec) {
#pragma unroll
        for (int k = 0; k < NTH / 4; ++k) {
          const int c = c0 + 8 * (4 * k + cq);
          const bool ok = r < R && c < Fd;
          if constexpr (sizeof(GT) == 2) {
            const uint4 w = ok ? *reinterpret_cast<const uint4*>(src + c) : make_uint4(0, 0, 0, 0);
            const uint32_t in[4] = {w.x, w.y, w.z, w.w};
            uint32_t out[4];
            quad_xpose(in, out);
#pragma unroll
            for (int j = 0; j < 4; ++j)
              pr[4 * k + j][h] = make_float2(bf16_lo(out[j]), bf16_hi(out[j]));
          } else {
            const uint4 a = ok ? *reinterpret_cast<const uint4*>(src + c) : make_uint4(0, 0, 0, 0);
            const uint4 b =
                ok ? *reinterpret_cast<const uint4*>(src + c + 4) : make_uint4(0, 0, 0, 0);
            const uint32_t lo_in[4] = {a.x, a.z, b.x, b.z}, hi_in[4] = {a.y, a.w, b.y, b.w};
            uint32_t lo_out[4], hi_out[4];
            quad_xpose(lo_in, lo_out);
            quad_xpose(hi_in, hi_out);
#pragma unroll
            for (int j = 0; j < 4; ++j)
              pr[4 * k + j][h] =
                  make_float2(__uint_as_float(lo_out[j]), __uint_as_float(hi_out[j]));
          }
        }
        done = true;
      }
    }
    if (!done) {
#pragma unroll
      for (int nt = 0; nt < NTH; ++nt) {
        const int c = c0 + 8 * nt + 2 * cq;
        const float a = (r < R && c < Fd) ? ld_f<GT>(src, c) : 0.f;
        const float b = (r < R && c + 1 < Fd) ? ld_f<GT>(src, c + 1) : 0.f;
        pr[nt][h] = make_float2(a, b);
      }
    }
  }
}

template <typename XT, typename GT, int DHP, int FDP, bool FULL>
__global__ void __launch_bounds__(kT)
hedgehog_bwd_kernel(const XT* __restrict__ x, const float* __restrict__ w,
                    const GT* __restrict__ df, XRows xm, int R, int Dh, int Fd, int vec,
                    int vec_df,
                    float* __restrict__ dx, float* __restrict__ dw_part) {
  using SM = HhSmem<DHP, FDP>;
  constexpr int NTH = FDP / 16;
  extern __shared__ __align__(128) unsigned char smem[];
  bf16* wh = reinterpret_cast<bf16*>(smem + SM::whi);
  bf16* wl = reinterpret_cast<bf16*>(smem + SM::wlo);
  bf16* xh = reinterpret_cast<bf16*>(smem + SM::xhi);
  bf16* xl = reinterpret_cast<bf16*>(smem + SM::xlo);
  float* red = reinterpret_cast<float*>(smem + SM::red);
  bf16* gh = reinterpret_cast<bf16*>(smem + SM::ghi);
  bf16* gl = reinterpret_cast<bf16*>(smem + SM::glo);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, cq = lane & 3;
  const int rb = warp & 3, half = warp >> 2, c0 = half * (FDP / 2);
  const int lrow = 16 * rb + gq;
  split_tile<float, FDP, DHP>(wh, wl, SM::LDW, w, Dh, 0, Fd, Dh);
  constexpr int MT = FDP / 16;       // 16-row tiles of dW (rows = features)
  constexpr int MTW = (MT + 7) / 8;  // per warp
  float dwa[MTW][DHP / 8][4];
#pragma unroll
  for (int a = 0; a < MTW; ++a)
#pragma unroll
    for (int c = 0; c < DHP / 8; ++c)
#pragma unroll
      for (int e = 0; e < 4; ++e) dwa[a][c][e] = 0.f;
  const int ntiles = (R + kR - 1) / kR;
  const int F2 = 2 * Fd;
  XTile<XT, DHP> xt;
  if (vec && (int)blockIdx.x < ntiles) xt.load(x, xm, blockIdx.x * kR, R, Dh);
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int r0 = tile * kR;
    __syncthreads();
    if (vec)
      xt.store(xh, xl, SM::LDX);
    else
      split_rows<XT, kR, DHP>(xh, xl, SM::LDX, x, xm, r0, R, Dh);
    __syncthreads();
    if (vec && tile + (int)gridDim.x < ntiles) xt.load(x, xm, r0 + gridDim.x * kR, R, Dh);
    float acc[NTH][4], pm[NTH][4];
    logits<DHP, FDP, sizeof(XT) == 4>(acc, xh, xl, wh, wl, rb, c0);
    softmaxes<FDP, FULL>(acc, pm, c0, Fd, red, half, lrow);
    // g = p+ (df+ - s+) - p- (df- - s-)
    {
      float2 dp[NTH][2], dm[NTH][2];
      load_df<GT, NTH>(dp, df, r0 + lrow, R, F2, 0, Fd, c0, vec_df);
      load_df<GT, NTH>(dm, df, r0 + lrow, R, F2, Fd, Fd, c0, vec_df);
      float sp[2] = {0.f, 0.f}, sm[2] = {0.f, 0.f};
#pragma unroll
      for (int nt = 0; nt < NTH; ++nt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          sp[h] += acc[nt][2 * h] * dp[nt][h].x + acc[nt][2 * h + 1] * dp[nt][h].y;
          sm[h] += pm[nt][2 * h] * dm[nt][h].x + pm[nt][2 * h + 1] * dm[nt][h].y;
        }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        sp[h] = quad_sum(sp[h]);
        sm[h] = quad_sum(sm[h]);
      }
      // the max / min slots of `red` are free again at this point
      exchange2(red, 0, half, lrow, sp, 2);
      exchange2(red, 1, half, lrow, sm, 2);
#pragma unroll
      for (int nt = 0; nt < NTH; ++nt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          acc[nt][2 * h] =
              acc[nt][2 * h] * (dp[nt][h].x - sp[h]) - pm[nt][2 * h] * (dm[nt][h].x - sm[h]);
          acc[nt][2 * h + 1] = acc[nt][2 * h + 1] * (dp[nt][h].y - sp[h]) -
                               pm[nt][2 * h + 1] * (dm[nt][h].y - sm[h]);
        }
    }
    // g (bf16 hi / lo) to shared memory
#pragma unroll
    for (int nt = 0; nt < NTH; ++nt) {
      const int c = c0 + 8 * nt + 2 * cq;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = lrow + 8 * h;
        const uint32_t hi = pack_bf16(acc[nt][2 * h], acc[nt][2 * h + 1]);
        const uint32_t lo =
            pack_bf16(acc[nt][2 * h] - bf16_lo(hi), acc[nt][2 * h + 1] - bf16_hi(hi));
        *reinterpret_cast<uint32_t*>(gh + row * SM::LDG + c) = hi;
        *reinterpret_cast<uint32_t*>(gl + row * SM::LDG + c) = lo;
      }
    }
    __syncthreads();
    // dx = g W: this warp's 16 rows, value columns [half * DHP/2, +DHP/2)
    {
      constexpr int NDH = DHP / 16;
      const int d0 = half * (DHP / 2);
      float dxa[NDH][4];
#pragma unroll
      for (int c = 0; c < NDH; ++c)
#pragma unroll
        for (int e = 0; e < 4; ++e) dxa[c][e] = 0.f;
#pragma unroll
      for (int k0 = 0; k0 < FDP; k0 += 16) {
        uint32_t ah[4], al[4];
        lda_rm(ah, gh, SM::LDG, 16 * rb, k0);
        lda_rm(al, gl, SM::LDG, 16 * rb, k0);
#pragma unroll
        for (int np = 0; np < NDH / 2; ++np) {
          uint32_t bh[4], bl[4];
          ldb_kn(bh, wh, SM::LDW, k0, d0 + 16 * np);
          mma16816(dxa[2 * np], ah, bh[0], bh[1]);
          mma16816(dxa[2 * np + 1], ah, bh[2], bh[3]);
          mma16816(dxa[2 * np], al, bh[0], bh[1]);
          mma16816(dxa[2 * np + 1], al, bh[2], bh[3]);
          ldb_kn(bl, wl, SM::LDW, k0, d0 + 16 * np);
          mma16816(dxa[2 * np], ah, bl[0], bl[1]);
          mma16816(dxa[2 * np + 1], ah, bl[2], bl[3]);
        }
      }
      const bool pair = (Dh & 1) == 0;
#pragma unroll
      for (int nt = 0; nt < NDH; ++nt) {
        const int d = d0 + 8 * nt + 2 * cq;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = r0 + lrow + 8 * h;
          if (row >= R || d >= Dh) continue;
          float* o = dx + (size_t)row * Dh + d;
          if (pair) {
            *reinterpret_cast<float2*>(o) = make_float2(dxa[nt][2 * h], dxa[nt][2 * h + 1]);
          } else {
            o[0] = dxa[nt][2 * h];
            if (d + 1 < Dh) o[1] = dxa[nt][2 * h + 1];
          }
        }
      }
    }
    // dW += g^T x: M = features (this warp's 16-row tiles), K = rows, N = Dh
#pragma unroll
    for (int mi = 0; mi < MTW; ++mi) {
      const int mt = warp + 8 * mi;
      if (mt >= MT) continue;
#pragma unroll
      for (int k0 = 0; k0 < kR; k0 += 16) {
        uint32_t ah[4], al[4];
        lda_tr(ah, gh, SM::LDG, 16 * mt, k0);
        lda_tr(al, gl, SM::LDG, 16 * mt, k0);
#pragma unroll
        for (int np = 0; np < DHP / 16; ++np) {
          uint32_t bh[4], bl[4];
          ldb_kn(bh, xh, SM::LDX, k0, 16 * np);
          mma16816(dwa[mi][2 * np], ah, bh[0], bh[1]);
          mma16816(dwa[mi][2 * np + 1], ah, bh[2], bh[3]);
          mma16816(dwa[mi][2 * np], al, bh[0], bh[1]);
          mma16816(dwa[mi][2 * np + 1], al, bh[2], bh[3]);
          if constexpr (sizeof(XT) == 4) {
            ldb_kn(bl, xl, SM::LDX, k0, 16 * np);
            mma16816(dwa[mi][2 * np], ah, bl[0], bl[1]);
            mma16816(dwa[mi][2 * np + 1], ah, bl[2], bl[3]);
          }
        }
      }
    }
  }
  // this CTA's dW partial [FDP, DHP] (the reduction reads only [Fd, Dh])
  float* part = dw_part + (size_t)blockIdx.x * FDP * DHP;
#pragma unroll
  for (int mi = 0; mi < MTW; ++mi) {
    const int mt = warp + 8 * mi;
    if (mt >= MT) continue;
#pragma unroll
    for (int nt = 0; nt < DHP / 8; ++nt) {
      const int d = 8 * nt + 2 * cq;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c = 16 * mt + gq + 8 * h;
        *reinterpret_cast<float2*>(part + c * DHP + d) =
            make_float2(dwa[mi][nt][2 * h], dwa[mi][nt][2 * h + 1]);
      }
    }
  }
}

// dW[c][d] = sum over CTAs of the partials, in CTA order
__global__ void __launch_bounds__(256)
hedgehog_dw_reduce_kernel(const float* __restrict__ part, int nparts, int FDP, int DHP, int Fd,
                          int Dh, float* __restrict__ dw) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= Fd * Dh) return;
  const int c = i / Dh, d = i % Dh;
  float s = 0.f;
  for (int p = 0; p < nparts; ++p) s += part[((size_t)p * FDP + c) * DHP + d];
  dw[i] = s;
}

std::mutex g_hh_mu;
template <typename Kern>
int hh_attr(Kern k, size_t bytes, bool* done) {
  if (bytes <= 48 * 1024) return LZ_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(g_hh_mu);
  if (dev < 64 && !done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) {
      set_error(std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
      return LZ_ERR_CUDA;
    }
    done[dev] = true;
  }
  return LZ_OK;
}

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

int dims_pad(int Dh, int Fd, int* dhp, int* fdp) {
  *dhp = Dh <= 32 ? 32 : Dh <= 64 ? 64 : Dh <= 128 ? 128 : 0;
  *fdp = Fd <= 32 ? 32 : Fd <= 64 ? 64 : Fd <= 128 ? 128 : 0;
  return (*dhp && *fdp) ? LZ_OK : LZ_ERR_UNSUPPORTED;
}

// ------------------------------------------------- forward for a few rows
// Decode-sized inputs (fewer rows than one 64-row tile per SM, e.g. one token
// of every head of a batch): a warp per row, 8 rows per CTA, so that the grid
// spreads over the SMs instead of a handful of tiles. Each CTA stages W in
// shared memory ([Fd][Dh + 1] fp32: a lane's feature row, one bank apart from
// the next lane's); lane l owns features l, l + 32, l + 64, l + 96 and takes
// the logits as fp32 dot products, then both softmaxes with warp shuffles.
constexpr int kRowWarps = 8;

template <typename XT>
__global__ void __launch_bounds__(kRowWarps * 32)
hedgehog_fwd_rows_kernel(const XT* __restrict__ x, XRows xm, const float* __restrict__ w, int R,
                         int Dh, int Fd, bf16* __restrict__ f) {
  extern __shared__ float hsm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int LW = Dh + 1;
  float* sW = hsm;                                  // [Fd][Dh + 1]
  float* sX = hsm + Fd * LW + warp * Dh;            // [8][Dh]
  const long long r = (long long)blockIdx.x * kRowWarps + warp;
  if (r < R) {
    const XT* xr = x + xm.off(r);
    for (int d = lane; d < Dh; d += 32) sX[d] = ld_f(xr, d);
  }
  if ((Dh & 3) == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0) {
    // 16-byte loads, up to 8 of a thread's in flight at once
    const int n4 = Fd * Dh / 4;
    for (int e0 = tid; e0 < n4; e0 += 8 * kRowWarps * 32) {
      float4 v4[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int e = e0 + u * kRowWarps * 32;
        if (e < n4) v4[u] = reinterpret_cast<const float4*>(w)[e];
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int e = e0 + u * kRowWarps * 32;
        if (e < n4) {
          const int fi = (4 * e) / Dh, d = 4 * e - fi * Dh;
          float* dst = sW + fi * LW + d;
          dst[0] = v4[u].x, dst[1] = v4[u].y, dst[2] = v4[u].z, dst[3] = v4[u].w;
        }
      }
    }
  } else {
    for (int e = tid; e < Fd * Dh; e += kRowWarps * 32) {
      const int fi = e / Dh, d = e - fi * Dh;
      sW[fi * LW + d] = w[e];
    }
  }
  __syncthreads();
  if (r >= R) return;
  float z[4] = {0.f, 0.f, 0.f, 0.f};
  for (int d = 0; d < Dh; ++d) {
    const float xd = sX[d];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (lane + 32 * i < Fd) z[i] = fmaf(xd, sW[(lane + 32 * i) * LW + d], z[i]);
  }
  float mx = -INFINITY, mn = INFINITY;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (lane + 32 * i < Fd) mx = fmaxf(mx, z[i]), mn = fminf(mn, z[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
  }
  float ep[4], em[4], sp = 0.f, sm = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bool ok = lane + 32 * i < Fd;
    ep[i] = ok ? __expf(z[i] - mx) : 0.f;
    em[i] = ok ? __expf(mn - z[i]) : 0.f;
    sp += ep[i], sm += em[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sp += __shfl_xor_sync(0xffffffffu, sp, o);
    sm += __shfl_xor_sync(0xffffffffu, sm, o);
  }
  const float ip = 1.f / sp, im = 1.f / sm;
  bf16* fr = f + (size_t)r * 2 * Fd;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (lane + 32 * i < Fd) {
      fr[lane + 32 * i] = __float2bfloat16_rn(ep[i] * ip);
      fr[Fd + lane + 32 * i] = __float2bfloat16_rn(em[i] * im);
    }
}

// ------------------------------------------------- forward on the tensor cores
// bf16 x with Dh = 64, Fd = 128 (the model's feature map): persistent CTAs of
// 4 warps, two per SM; W is split once into bf16 hi / lo in the 128-byte
// swizzled K-major layout; each 128-row x tile (of one head, from any batch /
// head / token strides) comes by TMA, and the next tile's x loads as soon as
// this tile's product has read it; one thread issues x W_hi^T + x W_lo^T into
// TMEM [128 x 128]; each thread then takes its row (TMEM lane): the max and
// min of the logits, e+ = exp(l - max) and e- = exp(min - l) written back to
// TMEM (one exponential per feature) with their sums, then the normalised
// features as bf16 into a 128-byte swizzled staging tile, which TMA stores
// write out (4 boxes of 128 rows x 64 features; rows past the head's end are
// not written) while the next tile's product and first passes run.
constexpr int kTcDh = 64, kTcFd = 128;
struct HhTcSmem {
  static constexpr size_t whi = 0, wlo = 16384, x = 32768, out = x + 16384;  // out: 4 x 16 KB
  static constexpr size_t bars = out + 4 * 16384, slot = bars + 32, bytes = slot + 16;
};

__global__ void __launch_bounds__(128, 2)
hedgehog_fwd_tc_kernel(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tf,
                       const float* __restrict__ w, int H, int ntl, long long ntiles) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  if (smem_u32(smem_raw) & 1023) {
    if (threadIdx.x == 0) atomicExch(&tc::g_timeout_flag, 0x80000000u | 94u);
    return;
  }
  unsigned char* base = smem_raw;
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + HhTcSmem::bars);  // x full, MMA done
  uint32_t* tslot = reinterpret_cast<uint32_t*>(base + HhTcSmem::slot);
  const int tid = threadIdx.x, warp = tid >> 5;
  if (tid == 0) {
    tc::mbar_init(&bars[0], 1);
    tc::mbar_init(&bars[1], 1);
    tc::fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(tslot, 256);
    tc::tmem_relinquish();
  }
  // W [Fd rows x Dh] fp32 -> bf16 hi / lo, row n at n * 128 bytes, 16-byte chunk c
  // of the row at (c ^ (n & 7)) * 16
  for (int e = tid; e < kTcFd * kTcDh / 8; e += 128) {
    const int n = e >> 3, c = e & 7;
    const float4 a = *reinterpret_cast<const float4*>(w + n * kTcDh + 8 * c);
    const float4 b4 = *reinterpret_cast<const float4*>(w + n * kTcDh + 8 * c + 4);
    const float v8[8] = {a.x, a.y, a.z, a.w, b4.x, b4.y, b4.z, b4.w};
    uint32_t h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      h[j] = pack_bf16(v8[2 * j], v8[2 * j + 1]);
      l[j] = pack_bf16(v8[2 * j] - bf16_lo(h[j]), v8[2 * j + 1] - bf16_hi(h[j]));
    }
    const size_t off = (size_t)n * 128 + ((c ^ (n & 7)) * 16);
    *reinterpret_cast<uint4*>(base + HhTcSmem::whi + off) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(base + HhTcSmem::wlo + off) = make_uint4(l[0], l[1], l[2], l[3]);
  }
  tc::fence_proxy_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
  auto issue = [&](long long t) {
    const int bh = (int)(t / ntl), t0 = (int)(t - (long long)bh * ntl) * 128;
    tc::mbar_expect_tx(&bars[0], 16384);
    tc::tma_load_4d(base + HhTcSmem::x, &tx, 0, t0, bh % H, bh / H, &bars[0]);
  };
  if (tid == 0 && (long long)blockIdx.x < ntiles) issue(blockIdx.x);
  int i = 0;
  for (long long t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
    const uint32_t ph = (uint32_t)i & 1u;
    if (tid == 0) {
      tc::mbar_wait(&bars[0], ph, 70);
      tc::tc_fence_after();
      constexpr uint32_t id = tc::idesc_bf16(128, 128, 0, 0);
      const uint32_t xa = smem_u32(base + HhTcSmem::x);
      const uint32_t wh = smem_u32(base + HhTcSmem::whi), wl = smem_u32(base + HhTcSmem::wlo);
#pragma unroll
      for (int j = 0; j < kTcDh / 16; ++j)
        tc::mma_ss(tmem, tc::sdesc(xa + 32 * j, 16, 1024), tc::sdesc(wh + 32 * j, 16, 1024), id,
                   j > 0);
#pragma unroll
      for (int j = 0; j < kTcDh / 16; ++j)
        tc::mma_ss(tmem, tc::sdesc(xa + 32 * j, 16, 1024), tc::sdesc(wl + 32 * j, 16, 1024), id,
                   1u);
      tc::mma_commit(&bars[1]);
    }
    tc::mbar_wait(&bars[1], ph, 71);
    tc::tc_fence_after();
    if (tid == 0 && t + gridDim.x < ntiles) issue(t + gridDim.x);  // the product has read x
    // pass 1: max and min of the row's logits
    float mx = -INFINITY, mn = INFINITY;
#pragma unroll 1
    for (int q = 0; q < 4; ++q) {
      float l[32];
      tc::tmem_ld32(trow + 32 * q, l);
      tc::tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        mx = fmaxf(mx, l[j]);
        mn = fminf(mn, l[j]);
      }
    }
    // pass 2: e+ = exp(l - max) over the logits' columns and e- = exp(min - l) at
    // 128 + the same (fp32 in TMEM), and their sums: one exponential per feature
    float sp = 0.f, sm = 0.f;
#pragma unroll 1
    for (int q = 0; q < 4; ++q) {
      float l[32];
      tc::tmem_ld32(trow + 32 * q, l);
      tc::tmem_wait_ld();
      uint32_t ep[2][16], em[2][16];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float a = __expf(l[j] - mx), b = __expf(mn - l[j]);
        sp += a;
        sm += b;
        ep[j >> 4][j & 15] = __float_as_uint(a);
        em[j >> 4][j & 15] = __float_as_uint(b);
      }
      tc::tmem_st16(trow + 32 * q, ep[0]);
      tc::tmem_st16(trow + 32 * q + 16, ep[1]);
      tc::tmem_st16(trow + 128 + 32 * q, em[0]);
      tc::tmem_st16(trow + 128 + 32 * q + 16, em[1]);
    }
    tc::tmem_wait_st();
    const float ip = 1.f / sp, im = 1.f / sm;
    if (tid == 0 && i > 0) tc::bulk_wait_read0();  // the last tile's stores have read the staging
    __syncthreads();
    // pass 3: normalised features into the staging tile (box b = features 64b..64b+63)
    const int r = tid;
#pragma unroll 1
    for (int q = 0; q < 8; ++q) {  // feature columns 32q..32q+31 (e+ then e-)
      float a[32];
      tc::tmem_ld32(trow + 32 * q, a);
      tc::tmem_wait_ld();
      const float inv = q < 4 ? ip : im;
      unsigned char* box = base + HhTcSmem::out + (q >> 1) * 16384 + r * 128;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float e8[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) e8[u] = a[8 * k + u] * inv;
        const int c = 4 * (q & 1) + k;  // 16-byte chunk within the box row
        *reinterpret_cast<uint4*>(box + ((c ^ (r & 7)) << 4)) = pack8(e8);
      }
    }
    tc::fence_proxy_async_smem();
    tc::tc_fence_before();
    __syncthreads();  // staging written; TMEM free for the next product
    if (tid == 0) {
      tc::tc_fence_after();
      const int bh = (int)(t / ntl), t0 = (int)(t - (long long)bh * ntl) * 128;
#pragma unroll
      for (int b = 0; b < 4; ++b)
        tc::tma_store_3d(&tf, base + HhTcSmem::out + b * 16384, 64 * b, t0, bh);
      tc::bulk_commit();
    }
  }
  if (tid == 0) tc::bulk_wait0();
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 256);
  }
}

// Tensor-core forward on (default) or off (the warp-MMA kernel), for tests.
std::atomic<int> g_hh_tc{1};
bool hh_tc_enabled() { return g_hh_tc.load(std::memory_order_relaxed) != 0; }
// Inputs with at most this many rows take the warp-per-row forward; -1 (the
// default) means fewer rows than one 64-row tile per SM, 0 never.
std::atomic<long long> g_hh_rows_max{-1};
long long hh_rows_max() {
  const long long v = g_hh_rows_max.load(std::memory_order_relaxed);
  return v < 0 ? (long long)kR * sm_count() - 1 : v;
}

template <typename XT>
int launch_fwd_rows(const void* x, const XRows& xm, const float* w, int R, int Dh, int Fd,
                    bf16* f, cudaStream_t st) {
  const size_t smem = ((size_t)Fd * (Dh + 1) + (size_t)kRowWarps * Dh) * 4;
  static bool done[64] = {false};
  int rc = hh_attr(hedgehog_fwd_rows_kernel<XT>, smem, done);
  if (rc) return rc;
  const int grid = (R + kRowWarps - 1) / kRowWarps;
  hedgehog_fwd_rows_kernel<XT><<<grid, kRowWarps * 32, smem, st>>>(static_cast<const XT*>(x), xm,
                                                                    w, R, Dh, Fd, f);
  count_launches(1);
  return check_launch("hedgehog_fwd_rows_kernel");
}

// persistent grid: two CTAs of 8 warps per SM
int hh_grid(int R) {
  const int ntiles = (R + kR - 1) / kR;
  return std::max(1, std::min(ntiles, sm_count() * 2));
}

// 16-byte x loads need every row start 16-byte aligned
bool rows_vec(const void* x, const XRows& m, int Dh, int es) {
  return Dh % (16 / es) == 0 && aligned16(x) && (m.sl * es) % 16 == 0 &&
         (m.sh * es) % 16 == 0 && (m.sb * es) % 16 == 0;
}

template <typename XT, int DHP, int FDP, bool FULL>
int launch_fwd_t(const void* x, const XRows& xm, const float* w, int R, int Dh, int Fd, bf16* f,
                 cudaStream_t st) {
  using SM = HhSmem<DHP, FDP>;
  static bool done[64] = {false};
  int rc = hh_attr(hedgehog_fwd_kernel<XT, DHP, FDP, FULL>, SM::fwd_bytes, done);
  if (rc) return rc;
  const int vec = rows_vec(x, xm, Dh, (int)sizeof(XT)) && aligned16(f);
  hedgehog_fwd_kernel<XT, DHP, FDP, FULL><<<hh_grid(R), kT, SM::fwd_bytes, st>>>(
      static_cast<const XT*>(x), xm, w, R, Dh, Fd, vec, f);
  count_launches(1);
  return check_launch("hedgehog_fwd_kernel");
}
template <typename XT, int DHP, int FDP>
int launch_fwd(const void* x, const XRows& xm, const float* w, int R, int Dh, int Fd, bf16* f,
               cudaStream_t st) {
  return Fd == FDP ? launch_fwd_t<XT, DHP, FDP, true>(x, xm, w, R, Dh, Fd, f, st)
                   : launch_fwd_t<XT, DHP, FDP, false>(x, xm, w, R, Dh, Fd, f, st);
}

template <typename XT, typename GT, int DHP, int FDP, bool FULL>
int launch_bwd_t(const void* x, const XRows& xm, const float* w, const void* df, int R, int Dh,
                 int Fd, float* dx, float* dw, void* work, cudaStream_t st) {
  using SM = HhSmem<DHP, FDP>;
  static bool done[64] = {false};
  int rc = hh_attr(hedgehog_bwd_kernel<XT, GT, DHP, FDP, FULL>, SM::bwd_bytes, done);
  if (rc) return rc;
  const int grid = hh_grid(R);
  const int vec = rows_vec(x, xm, Dh, (int)sizeof(XT));
  const int vec_df = (Fd % 8 == 0) && aligned16(df);
  float* part = static_cast<float*>(work);
  hedgehog_bwd_kernel<XT, GT, DHP, FDP, FULL><<<grid, kT, SM::bwd_bytes, st>>>(
      static_cast<const XT*>(x), w, static_cast<const GT*>(df), xm, R, Dh, Fd, vec, vec_df, dx,
      part);
  count_launches(1);
  rc = check_launch("hedgehog_bwd_kernel");
  if (rc) return rc;
  hedgehog_dw_reduce_kernel<<<(Fd * Dh + 255) / 256, 256, 0, st>>>(part, grid, FDP, DHP, Fd, Dh,
                                                                   dw);
  count_launches(1);
  return check_launch("hedgehog_dw_reduce_kernel");
}
template <typename XT, typename GT, int DHP, int FDP>
int launch_bwd(const void* x, const XRows& xm, const float* w, const void* df, int R, int Dh,
               int Fd, float* dx, float* dw, void* work, cudaStream_t st) {
  return Fd == FDP
             ? launch_bwd_t<XT, GT, DHP, FDP, true>(x, xm, w, df, R, Dh, Fd, dx, dw, work, st)
             : launch_bwd_t<XT, GT, DHP, FDP, false>(x, xm, w, df, R, Dh, Fd, dx, dw, work, st);
}

}  // namespace

size_t hedgehog_bwd_workspace(int R, int Dh, int Fd) {
  int dhp, fdp;
  if (dims_pad(Dh, Fd, &dhp, &fdp)) return 0;
  return (size_t)hh_grid(R) * fdp * dhp * 4;
}

// The tensor-core forward for bf16 x, Dh = 64, Fd = 128; LZ_ERR_UNSUPPORTED
// (nothing launched) when the rows cannot be tiled by TMA.
int hedgehog_fwd_tc(const void* x, const XRows& xm, const float* w, int R, bf16* f,
                    cudaStream_t st) {
  if (!aligned16(x) || !aligned16(w) || !aligned16(f) || (xm.sl * 2) % 16 ||
      (xm.sh * 2) % 16 || (xm.sb * 2) % 16 || xm.sl <= 0)
    return LZ_ERR_UNSUPPORTED;
  const long long heads = (long long)R / xm.L, B = heads / xm.H;
  if (heads * xm.L != R || B * xm.H != heads) return LZ_ERR_UNSUPPORTED;
  tc::EncodeTiledFn fn = tc::encode_tiled_fn();
  if (!fn) return LZ_ERR_UNSUPPORTED;
  const long long sh = xm.H > 1 ? xm.sh : (long long)xm.L * xm.sl;
  const long long sb = B > 1 ? xm.sb : xm.H * sh;
  CUtensorMap mx;
  cuuint64_t dims[4] = {(cuuint64_t)kTcDh, (cuuint64_t)xm.L, (cuuint64_t)xm.H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)(xm.sl * 2), (cuuint64_t)(sh * 2), (cuuint64_t)(sb * 2)};
  cuuint32_t box[4] = {(cuuint32_t)kTcDh, 128, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  if (fn(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(x), dims, strides, box, estr,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return LZ_ERR_UNSUPPORTED;
  // features [heads, L, 256] as a 3-D map {256, L, heads}, box {64, 128, 1}: stores clip
  // at each head's last row
  CUtensorMap mf;
  cuuint64_t fdims[3] = {(cuuint64_t)(2 * kTcFd), (cuuint64_t)xm.L, (cuuint64_t)heads};
  cuuint64_t fstr[2] = {(cuuint64_t)(2 * kTcFd * 2), (cuuint64_t)xm.L * 2 * kTcFd * 2};
  cuuint32_t fbox[3] = {64, 128, 1};
  cuuint32_t festr[3] = {1, 1, 1};
  if (fn(&mf, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, f, fdims, fstr, fbox, festr,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return LZ_ERR_UNSUPPORTED;
  static bool done[64] = {false};
  int rc = hh_attr(hedgehog_fwd_tc_kernel, HhTcSmem::bytes, done);
  if (rc) return rc;
  const int ntl = (xm.L + 127) / 128;
  const long long ntiles = heads * ntl;
  const int grid = (int)std::min<long long>(ntiles, 2LL * sm_count());
  hedgehog_fwd_tc_kernel<<<grid, 128, HhTcSmem::bytes, st>>>(mx, mf, w, xm.H, ntl, ntiles);
  count_launches(1);
  return check_launch("hedgehog_fwd_tc_kernel");
}

int hedgehog_fwd(const void* x, int x_dtype, const XRows& xm, const float* w, int R, int Dh,
                 int Fd, bf16* f, cudaStream_t st) {
  if (R <= hh_rows_max() && Dh <= 128 && Fd <= 128)
    return x_dtype == LZ_DTYPE_F32 ? launch_fwd_rows<float>(x, xm, w, R, Dh, Fd, f, st)
                                   : launch_fwd_rows<bf16>(x, xm, w, R, Dh, Fd, f, st);
  if (x_dtype == LZ_DTYPE_BF16 && Dh == kTcDh && Fd == kTcFd && hh_tc_enabled()) {
    const int rc = hedgehog_fwd_tc(x, xm, w, R, f, st);
    if (rc != LZ_ERR_UNSUPPORTED) return rc;
  }
  int dhp, fdp;
  if (dims_pad(Dh, Fd, &dhp, &fdp)) {
    set_error("hedgehog: head dim and feature dim must be <= 128");
    return LZ_ERR_UNSUPPORTED;
  }
  const int xs = x_dtype == LZ_DTYPE_F32;
#define LZ_HH_FWD(dh, fd)                                                                 \
  if (dhp == dh && fdp == fd)                                                             \
    return xs ? launch_fwd<float, dh, fd>(x, xm, w, R, Dh, Fd, f, st)                     \
              : launch_fwd<bf16, dh, fd>(x, xm, w, R, Dh, Fd, f, st);
  LZ_HH_FWD(32, 32) LZ_HH_FWD(32, 64) LZ_HH_FWD(32, 128)
  LZ_HH_FWD(64, 32) LZ_HH_FWD(64, 64) LZ_HH_FWD(64, 128)
  LZ_HH_FWD(128, 32) LZ_HH_FWD(128, 64) LZ_HH_FWD(128, 128)
#undef LZ_HH_FWD
  return LZ_ERR_UNSUPPORTED;
}

int hedgehog_bwd(const void* x, int x_dtype, const XRows& xm, const float* w, const void* df,
                 int df_dtype, int R, int Dh, int Fd, float* dx, float* dw, void* work,
                 cudaStream_t st) {
  int dhp, fdp;
  if (dims_pad(Dh, Fd, &dhp, &fdp)) {
    set_error("hedgehog: head dim and feature dim must be <= 128");
    return LZ_ERR_UNSUPPORTED;
  }
  const bool xf = x_dtype == LZ_DTYPE_F32, gf = df_dtype == LZ_DTYPE_F32;
#define LZ_HH_BWD(dh, fd)                                                                        \
  if (dhp == dh && fdp == fd) {                                                                  \
    if (xf && gf)                                                                                \
      return launch_bwd<float, float, dh, fd>(x, xm, w, df, R, Dh, Fd, dx, dw, work, st);        \
    if (xf) return launch_bwd<float, bf16, dh, fd>(x, xm, w, df, R, Dh, Fd, dx, dw, work, st);   \
    if (gf) return launch_bwd<bf16, float, dh, fd>(x, xm, w, df, R, Dh, Fd, dx, dw, work, st);   \
    return launch_bwd<bf16, bf16, dh, fd>(x, xm, w, df, R, Dh, Fd, dx, dw, work, st);            \
  }
  LZ_HH_BWD(32, 32) LZ_HH_BWD(32, 64) LZ_HH_BWD(32, 128)
  LZ_HH_BWD(64, 32) LZ_HH_BWD(64, 64) LZ_HH_BWD(64, 128)
  LZ_HH_BWD(128, 32) LZ_HH_BWD(128, 64) LZ_HH_BWD(128, 128)
#undef LZ_HH_BWD
  return LZ_ERR_UNSUPPORTED;
}

int hedgehog_timeout_flag(unsigned int* out) { return tc::read_timeout_flag_here(out); }
int hedgehog_timeout_clear() { return tc::clear_timeout_flag_here(); }

}  // namespace lz

extern "C" int lz_hedgehog_set_tc(int on) { return lz::g_hh_tc.exchange(on ? 1 : 0); }

extern "C" long long lz_hedgehog_set_rows_max(long long rows) {
  return lz::g_hh_rows_max.exchange(rows < 0 ? -1 : rows);
}

extern "C" size_t lz_hedgehog_bwd_workspace_bytes(int R, int Dh, int Fd) {
  if (R < 1 || Dh < 1 || Fd < 1) return 0;
  return lz::hedgehog_bwd_workspace(R, Dh, Fd);
}

extern "C" int lz_hedgehog_fwd(const void* x, int x_dtype, const float* weight, void* f, int R,
                               int Dh, int Fd, void* stream) {
  lz::clear_error();
  LZ_REQUIRE(x && weight && f, LZ_ERR_INVALID_ARGUMENT, "null pointer");
  LZ_REQUIRE(R >= 1 && Dh >= 1 && Fd >= 1, LZ_ERR_INVALID_ARGUMENT, "sizes must be positive");
  LZ_REQUIRE(x_dtype == LZ_DTYPE_F32 || x_dtype == LZ_DTYPE_BF16, LZ_ERR_INVALID_ARGUMENT,
             "x_dtype must be LZ_DTYPE_F32 or LZ_DTYPE_BF16");
  const lz::XRows xm{1, R, (long long)R * Dh, (long long)R * Dh, Dh};
  return lz::hedgehog_fwd(x, x_dtype, xm, weight, R, Dh, Fd, static_cast<bf16*>(f),
                          static_cast<cudaStream_t>(stream));
}

extern "C" int lz_hedgehog_fwd_strided(const void* x, int x_dtype, long long x_sb,
                                       long long x_sh, long long x_sl, int B, int Hx, int L,
                                       const float* weight, void* f, int Dh, int Fd,
                                       void* stream) {
  lz::clear_error();
  LZ_REQUIRE(x && weight && f, LZ_ERR_INVALID_ARGUMENT, "null pointer");
  LZ_REQUIRE(B >= 1 && Hx >= 1 && L >= 1 && Dh >= 1 && Fd >= 1, LZ_ERR_INVALID_ARGUMENT,
             "sizes must be positive");
  LZ_REQUIRE((long long)B * Hx * L < (1ll << 31), LZ_ERR_INVALID_ARGUMENT, "too many rows");
  LZ_REQUIRE(x_dtype == LZ_DTYPE_F32 || x_dtype == LZ_DTYPE_BF16, LZ_ERR_INVALID_ARGUMENT,
             "x_dtype must be LZ_DTYPE_F32 or LZ_DTYPE_BF16");
  const lz::XRows xm{Hx, L, x_sb, x_sh, x_sl};
  return lz::hedgehog_fwd(x, x_dtype, xm, weight, B * Hx * L, Dh, Fd, static_cast<bf16*>(f),
                          static_cast<cudaStream_t>(stream));
}

extern "C" int lz_hedgehog_bwd(const void* x, int x_dtype, const float* weight, const void* df,
                               int df_dtype, float* dx, float* dweight, void* workspace,
                               size_t workspace_bytes, int R, int Dh, int Fd, void* stream) {
  lz::clear_error();
  LZ_REQUIRE(x && weight && df && dx && dweight && workspace, LZ_ERR_INVALID_ARGUMENT,
             "null pointer");
  LZ_REQUIRE(R >= 1 && Dh >= 1 && Fd >= 1, LZ_ERR_INVALID_ARGUMENT, "sizes must be positive");
  LZ_REQUIRE((x_dtype == LZ_DTYPE_F32 || x_dtype == LZ_DTYPE_BF16) &&
                 (df_dtype == LZ_DTYPE_F32 || df_dtype == LZ_DTYPE_BF16),
             LZ_ERR_INVALID_ARGUMENT, "dtypes must be LZ_DTYPE_F32 or LZ_DTYPE_BF16");
  LZ_REQUIRE(workspace_bytes >= lz::hedgehog_bwd_workspace(R, Dh, Fd), LZ_ERR_WORKSPACE,
             "workspace too small (lz_hedgehog_bwd_workspace_bytes)");
  const lz::XRows xm{1, R, (long long)R * Dh, (long long)R * Dh, Dh};
  return lz::hedgehog_bwd(x, x_dtype, xm, weight, df, df_dtype, R, Dh, Fd, dx, dweight,
                          workspace, static_cast<cudaStream_t>(stream));
}

extern "C" int lz_hedgehog_bwd_strided(const void* x, int x_dtype, long long x_sb,
                                       long long x_sh, long long x_sl, int B, int Hx, int L,
                                       const float* weight, const void* df, int df_dtype,
                                       float* dx, float* dweight, void* workspace,
                                       size_t workspace_bytes, int Dh, int Fd, void* stream) {
  lz::clear_error();
  LZ_REQUIRE(x && weight && df && dx && dweight && workspace, LZ_ERR_INVALID_ARGUMENT,
             "null pointer");
  LZ_REQUIRE(B >= 1 && Hx >= 1 && L >= 1 && Dh >= 1 && Fd >= 1, LZ_ERR_INVALID_ARGUMENT,
             "sizes must be positive");
  LZ_REQUIRE((long long)B * Hx * L < (1ll << 31), LZ_ERR_INVALID_ARGUMENT, "too many rows");
  LZ_REQUIRE((x_dtype == LZ_DTYPE_F32 || x_dtype == LZ_DTYPE_BF16) &&
                 (df_dtype == LZ_DTYPE_F32 || df_dtype == LZ_DTYPE_BF16),
             LZ_ERR_INVALID_ARGUMENT, "dtypes must be LZ_DTYPE_F32 or LZ_DTYPE_BF16");
  const int R = B * Hx * L;
  LZ_REQUIRE(workspace_bytes >= lz::hedgehog_bwd_workspace(R, Dh, Fd), LZ_ERR_WORKSPACE,
             "workspace too small (lz_hedgehog_bwd_workspace_bytes)");
  const lz::XRows xm{Hx, L, x_sb, x_sh, x_sl};
  return lz::hedgehog_bwd(x, x_dtype, xm, weight, df, df_dtype, R, Dh, Fd, dx, dweight,
                          workspace, static_cast<cudaStream_t>(stream));
}
