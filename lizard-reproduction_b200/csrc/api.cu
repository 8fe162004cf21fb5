// extern "C" entry points declared in include/lizard_cuda.h: argument
// validation, carving of caller-owned buffers, dispatch to the kernels.
#include <algorithm>

#include "common.cuh"
#include "gla_layout.h"
#include "swa_layout.h"

namespace {

int check_sizes(int B, int H, int L, int F, int D) {
  LZ_REQUIRE(B >= 1 && H >= 1 && L >= 1, LZ_ERR_INVALID_ARGUMENT,
             "B, H and L must be positive");
  LZ_REQUIRE(F >= 1 && D >= 1, LZ_ERR_INVALID_ARGUMENT, "feature and value dims must be positive");
  LZ_REQUIRE((long long)B * H * L < (1ll << 31), LZ_ERR_UNSUPPORTED, "B*H*L must fit in int32");
  return LZ_OK;
}

}  // namespace

namespace lz {
// Each unit whose kernels hold bounded waits has its own copy of the flag.
int gla_fwd_tc_timeout_flag(unsigned int* out);
int gla_fwd_tc64_timeout_flag(unsigned int* out);
int gla_bwd_tc_timeout_flag(unsigned int* out);
int gla_out_tc_timeout_flag(unsigned int* out);
int hedgehog_timeout_flag(unsigned int* out);
int swa_timeout_flag(unsigned int* out);
int swa_tc_timeout_flag(unsigned int* out);
int decode_timeout_flag(unsigned int* out);
int gla_fwd_tc_timeout_clear();
int gla_fwd_tc64_timeout_clear();
int gla_bwd_tc_timeout_clear();
int gla_out_tc_timeout_clear();
int hedgehog_timeout_clear();
int swa_timeout_clear();
int swa_tc_timeout_clear();
int decode_timeout_clear();
}  // namespace lz

extern "C" int lz_device_timeout_flag(unsigned int* site) {
  lz::clear_error();
  LZ_REQUIRE(site, LZ_ERR_INVALID_ARGUMENT, "null pointer");
  int (*const readers[])(unsigned int*) = {
      lz::gla_fwd_tc_timeout_flag, lz::gla_fwd_tc64_timeout_flag, lz::gla_bwd_tc_timeout_flag,
      lz::gla_out_tc_timeout_flag, lz::hedgehog_timeout_flag,     lz::swa_timeout_flag,
      lz::swa_tc_timeout_flag,     lz::decode_timeout_flag};
  *site = 0;
  for (auto rd : readers) {
    unsigned int v = 0;
    const int rc = rd(&v);
    if (rc) return rc;
    if (v) {
      *site = v;
      break;
    }
  }
  return LZ_OK;
}

extern "C" int lz_device_timeout_clear(void) {
  lz::clear_error();
  int (*const clearers[])() = {
      lz::gla_fwd_tc_timeout_clear, lz::gla_fwd_tc64_timeout_clear, lz::gla_bwd_tc_timeout_clear,
      lz::gla_out_tc_timeout_clear, lz::hedgehog_timeout_clear,     lz::swa_timeout_clear,
      lz::swa_tc_timeout_clear,     lz::decode_timeout_clear};
  for (auto cl : clearers) {
    const int rc = cl();
    if (rc) return rc;
  }
  return LZ_OK;
}

extern "C" size_t lz_gla_saved_bytes(int B, int H, int L, int F, int D, int chunk) {
  (void)chunk;
  if (B < 1 || H < 1 || L < 1 || F < 1 || D < 1) return 0;
  return lz::gla_saved_layout(B, H, L, F, D, nullptr, nullptr);
}

extern "C" size_t lz_gla_bwd_workspace_bytes(int B, int H, int L, int F, int D, int chunk) {
  (void)chunk;
  if (B < 1 || H < 1 || L < 1 || F < 1 || D < 1) return 0;
  return lz::gla_work_layout(B, H, L, F, D, lz::gla_bwd_split(B, H, L, F, D), nullptr, nullptr);
}

extern "C" size_t lz_gla_bwd_gqa_workspace_bytes(int B, int H, int Hkv, int L, int F, int D,
                                                 int chunk) {
  (void)chunk;
  if (B < 1 || H < 1 || L < 1 || F < 1 || D < 1 || Hkv < 1 || H % Hkv) return 0;
  return lz::gla_work_layout(B, H, L, F, D, lz::gla_bwd_split(B, H, L, F, D), nullptr, nullptr,
                             Hkv != H);
}

extern "C" size_t lz_gla_fwd_gqa_workspace_bytes(int B, int H, int Hkv, int L, int F, int D,
                                                 int chunk, int gate_per_head, int training) {
  (void)chunk;
  if (B < 1 || H < 1 || L < 1 || F < 1 || D < 1 || Hkv < 1 || H % Hkv) return 0;
  if (!lz::gla_fwd_split(B, H, L, F, D)) return 0;
  const int Hs = (!training && !gate_per_head && Hkv < H) ? Hkv : H;
  return lz::gla_fwd_work_layout(B, H, L, F, D, nullptr, nullptr, Hs);
}

extern "C" size_t lz_gla_fwd_workspace_bytes(int B, int H, int L, int F, int D, int chunk) {
  (void)chunk;
  if (B < 1 || H < 1 || L < 1 || F < 1 || D < 1) return 0;
  if (!lz::gla_fwd_split(B, H, L, F, D)) return 0;
  return lz::gla_fwd_work_layout(B, H, L, F, D, nullptr, nullptr);
}

namespace lz {
int gla_set_schedule(int s);
}

extern "C" int lz_gla_set_schedule(int schedule) {
  lz::clear_error();
  if (schedule < 0 || schedule > 2) {
    lz::set_error("schedule must be 0 (auto), 1 (walk) or 2 (chunk-parallel)");
    return -LZ_ERR_INVALID_ARGUMENT;
  }
  return lz::gla_set_schedule(schedule);
}

namespace lz {
int gla_set_out_tc(int on);
}

extern "C" int lz_gla_set_split_out_tc(int on) { return lz::gla_set_out_tc(on); }

namespace lz {
int gla_set_fwd_tc64(int on);
}

extern "C" int lz_gla_set_fwd_tc64(int on) { return lz::gla_set_fwd_tc64(on); }

namespace lz {
int gla_set_bwd_prefetch(int on);
}

extern "C" int lz_gla_set_bwd_prefetch(int on) { return lz::gla_set_bwd_prefetch(on); }

extern "C" int lz_gla_fwd_gqa(const void* fq, const void* fk, const void* v,
                              const float* log_gamma, int gate_per_head, void* y, void* saved,
                              size_t saved_bytes, void* workspace, size_t workspace_bytes, int B,
                              int H, int Hkv, int L, int F, int D, int chunk, void* stream) {
  lz::clear_error();
  int rc = check_sizes(B, H, L, F, D);
  if (rc) return rc;
  LZ_REQUIRE(Hkv >= 1 && H % Hkv == 0, LZ_ERR_INVALID_ARGUMENT,
             "the key/value head count must divide the query head count");
  LZ_REQUIRE(fq && fk && v && log_gamma && y, LZ_ERR_INVALID_ARGUMENT, "null tensor pointer");
  LZ_REQUIRE(chunk >= 1, LZ_ERR_INVALID_ARGUMENT, "chunk must be >= 1");
  LZ_REQUIRE(F <= 256, LZ_ERR_UNSUPPORTED, "feature dim above 256 is not supported");
  LZ_REQUIRE(D <= 256, LZ_ERR_UNSUPPORTED, "value dim above 256 is not supported");
  lz::GlaSaved sv;
  if (saved) {
    const size_t need = lz::gla_saved_layout(B, H, L, F, D, nullptr, nullptr);
    LZ_REQUIRE(saved_bytes >= need, LZ_ERR_WORKSPACE, "saved buffer too small");
    LZ_REQUIRE(lz::aligned16(saved), LZ_ERR_INVALID_ARGUMENT, "saved buffer must be 16-byte aligned");
    lz::gla_saved_layout(B, H, L, F, D, static_cast<unsigned char*>(saved), &sv);
  }
  lz::GlaFwdWork fw;
  if (lz::gla_fwd_split(B, H, L, F, D)) {
    // one state per key/value head when nothing is saved and the gate is shared
    const int Hs = (!saved && !gate_per_head && Hkv < H) ? Hkv : H;
    const size_t need = lz::gla_fwd_work_layout(B, H, L, F, D, nullptr, nullptr, Hs);
    LZ_REQUIRE(workspace && workspace_bytes >= need, LZ_ERR_WORKSPACE,
               "workspace too small (lz_gla_fwd_gqa_workspace_bytes)");
    LZ_REQUIRE(lz::aligned16(workspace), LZ_ERR_INVALID_ARGUMENT,
               "workspace must be 16-byte aligned");
    lz::gla_fwd_work_layout(B, H, L, F, D, static_cast<unsigned char*>(workspace), &fw, Hs);
  }
  return lz::gla_fwd(static_cast<const bf16*>(fq), static_cast<const bf16*>(fk),
                     static_cast<const bf16*>(v), log_gamma, gate_per_head ? 1 : 0,
                     static_cast<bf16*>(y), sv, fw, B, H, Hkv, L, F, D,
                     static_cast<cudaStream_t>(stream));
}

extern "C" int lz_gla_fwd(const void* fq, const void* fk, const void* v, const float* log_gamma,
                          int gate_per_head, void* y, void* saved, size_t saved_bytes,
                          void* workspace, size_t workspace_bytes, int B, int H, int L, int F,
                          int D, int chunk, void* stream) {
  return lz_gla_fwd_gqa(fq, fk, v, log_gamma, gate_per_head, y, saved, saved_bytes, workspace,
                        workspace_bytes, B, H, H, L, F, D, chunk, stream);
}

extern "C" int lz_gla_bwd_gqa(const void* fq, const void* fk, const void* v,
                              const float* log_gamma, int gate_per_head, const void* saved,
                              size_t saved_bytes, const void* dy, void* dfq, void* dfk, void* dv,
                              int grad_dtype, float* dlog_gamma, void* workspace,
                              size_t workspace_bytes, int B, int H, int Hkv, int L, int F, int D,
                              int chunk, void* stream) {
  lz::clear_error();
  int rc = check_sizes(B, H, L, F, D);
  if (rc) return rc;
  LZ_REQUIRE(Hkv >= 1 && H % Hkv == 0, LZ_ERR_INVALID_ARGUMENT,
             "the key/value head count must divide the query head count");
  LZ_REQUIRE(fq && fk && v && log_gamma && saved && dy && dfq && dfk && dv && dlog_gamma &&
                 workspace,
             LZ_ERR_INVALID_ARGUMENT, "null pointer");
  LZ_REQUIRE(chunk >= 1, LZ_ERR_INVALID_ARGUMENT, "chunk must be >= 1");
  LZ_REQUIRE(grad_dtype == LZ_DTYPE_F32 || grad_dtype == LZ_DTYPE_BF16, LZ_ERR_INVALID_ARGUMENT,
             "grad_dtype must be LZ_DTYPE_F32 or LZ_DTYPE_BF16");
  LZ_REQUIRE(F <= 256, LZ_ERR_UNSUPPORTED, "feature dim above 256 is not supported");
  LZ_REQUIRE(D <= 128, LZ_ERR_UNSUPPORTED, "value dim above 128 is not supported in the backward");
  const size_t need_s = lz::gla_saved_layout(B, H, L, F, D, nullptr, nullptr);
  const bool split = lz::gla_bwd_split(B, H, L, F, D);
  const size_t need_w = lz::gla_work_layout(B, H, L, F, D, split, nullptr, nullptr, Hkv != H);
  LZ_REQUIRE(saved_bytes >= need_s, LZ_ERR_WORKSPACE, "saved buffer too small");
  LZ_REQUIRE(workspace_bytes >= need_w, LZ_ERR_WORKSPACE, "workspace too small");
  LZ_REQUIRE(lz::aligned16(saved) && lz::aligned16(workspace), LZ_ERR_INVALID_ARGUMENT,
             "saved buffer and workspace must be 16-byte aligned");
  lz::GlaSaved sv;
  lz::GlaWork wk;
  lz::gla_saved_layout(B, H, L, F, D, (unsigned char*)const_cast<void*>(saved), &sv);
  lz::gla_work_layout(B, H, L, F, D, split, static_cast<unsigned char*>(workspace), &wk,
                      Hkv != H);
  return lz::gla_bwd(static_cast<const bf16*>(fq), static_cast<const bf16*>(fk),
                     static_cast<const bf16*>(v), log_gamma, gate_per_head ? 1 : 0, sv,
                     static_cast<const bf16*>(dy), dfq, dfk, dv, grad_dtype, dlog_gamma, wk, B,
                     H, Hkv, L, F, D, static_cast<cudaStream_t>(stream));
}

extern "C" int lz_gla_bwd(const void* fq, const void* fk, const void* v, const float* log_gamma,
                          int gate_per_head, const void* saved, size_t saved_bytes,
                          const void* dy, void* dfq, void* dfk, void* dv, int grad_dtype,
                          float* dlog_gamma, void* workspace, size_t workspace_bytes, int B,
                          int H, int L, int F, int D, int chunk, void* stream) {
  return lz_gla_bwd_gqa(fq, fk, v, log_gamma, gate_per_head, saved, saved_bytes, dy, dfq, dfk, dv,
                        grad_dtype, dlog_gamma, workspace, workspace_bytes, B, H, H, L, F, D,
                        chunk, stream);
}

extern "C" size_t lz_swa_saved_bytes(int B, int H, int L, int D) {
  if (B < 1 || H < 1 || L < 1 || D < 1) return 0;
  return lz::swa_saved_layout(B, H, L, D, nullptr, nullptr);
}

extern "C" size_t lz_swa_bwd_workspace_bytes(int B, int H, int L, int D, int n_meta) {
  (void)D;
  if (B < 1 || H < 1 || L < 1 || n_meta < 0) return 0;
  return lz::swa_work_layout(B, H, L, n_meta, nullptr, nullptr);
}

extern "C" int lz_swa_fwd_gqa(const void* q, const void* k, const void* v, const void* q_lo,
                              const void* k_lo, const float* meta, int n_meta, int window,
                              void* y, void* saved, size_t saved_bytes, int B, int H, int Hkv,
                              int L, int D, void* stream) {
  lz::clear_error();
  int rc = check_sizes(B, H, L, 1, D);
  if (rc) return rc;
  LZ_REQUIRE(Hkv >= 1 && H % Hkv == 0, LZ_ERR_INVALID_ARGUMENT,
             "the key/value head count must divide the query head count");
  LZ_REQUIRE(q && k && v && y, LZ_ERR_INVALID_ARGUMENT, "null tensor pointer");
  LZ_REQUIRE((q_lo == nullptr) == (k_lo == nullptr), LZ_ERR_INVALID_ARGUMENT,
             "q_lo and k_lo must be both null or both set");
  LZ_REQUIRE(n_meta >= 0 && (n_meta == 0 || meta), LZ_ERR_INVALID_ARGUMENT,
             "meta must be non-null when n_meta > 0");
  LZ_REQUIRE(n_meta <= lz::kMaxMeta, LZ_ERR_UNSUPPORTED, "more than 32 sink logits");
  LZ_REQUIRE(window >= 1, LZ_ERR_INVALID_ARGUMENT, "window must be >= 1");
  LZ_REQUIRE(D <= 128, LZ_ERR_UNSUPPORTED, "head dim above 128 is not supported");
  lz::SwaSaved sv;
  if (saved) {
    LZ_REQUIRE(saved_bytes >= lz::swa_saved_layout(B, H, L, D, nullptr, nullptr),
               LZ_ERR_WORKSPACE, "saved buffer too small");
    LZ_REQUIRE(lz::aligned16(saved), LZ_ERR_INVALID_ARGUMENT,
               "saved buffer must be 16-byte aligned");
    lz::swa_saved_layout(B, H, L, D, static_cast<unsigned char*>(saved), &sv);
  }
  return lz::swa_fwd(static_cast<const bf16*>(q), static_cast<const bf16*>(k),
                     static_cast<const bf16*>(v), static_cast<const bf16*>(q_lo),
                     static_cast<const bf16*>(k_lo), meta, n_meta, window,
                     static_cast<bf16*>(y), sv, B, H, Hkv, L, D,
                     static_cast<cudaStream_t>(stream));
}

extern "C" int lz_swa_rope_fwd(const void* q, const void* k, const void* v, int x_dtype,
                               long long q_sb, long long q_sh, long long q_sl, long long k_sb,
                               long long k_sh, long long k_sl, long long v_sb, long long v_sh,
                               long long v_sl, const void* cos, const void* sin, int cs_dtype,
                               long long cs_sb, long long cs_sl, const float* meta, int n_meta,
                               int window, void* y, void* saved, size_t saved_bytes, void* q_hi,
                               void* q_lo, void* k_hi, void* k_lo, int B, int H, int Hkv, int L,
                               int D, void* stream) {
  lz::clear_error();
  int rc = check_sizes(B, H, L, 1, D);
  if (rc) return rc;
  LZ_REQUIRE(Hkv >= 1 && H % Hkv == 0, LZ_ERR_INVALID_ARGUMENT,
             "the key/value head count must divide the query head count");
  LZ_REQUIRE(q && k && v && cos && sin && y, LZ_ERR_INVALID_ARGUMENT, "null tensor pointer");
  LZ_REQUIRE((x_dtype == LZ_DTYPE_F32 || x_dtype == LZ_DTYPE_BF16) &&
                 (cs_dtype == LZ_DTYPE_F32 || cs_dtype == LZ_DTYPE_BF16),
             LZ_ERR_INVALID_ARGUMENT, "dtypes must be LZ_DTYPE_F32 or LZ_DTYPE_BF16");
  LZ_REQUIRE(n_meta >= 0 && (n_meta == 0 || meta), LZ_ERR_INVALID_ARGUMENT,
             "meta must be non-null when n_meta > 0");
  LZ_REQUIRE(n_meta <= lz::kMaxMeta, LZ_ERR_UNSUPPORTED, "more than 32 sink logits");
  LZ_REQUIRE(window >= 1, LZ_ERR_INVALID_ARGUMENT, "window must be >= 1");
  LZ_REQUIRE(D % 2 == 0, LZ_ERR_INVALID_ARGUMENT, "the rotated head dim must be even");
  LZ_REQUIRE((q_hi == nullptr) == (q_lo == nullptr) && (q_hi == nullptr) == (k_hi == nullptr) &&
                 (k_hi == nullptr) == (k_lo == nullptr),
             LZ_ERR_INVALID_ARGUMENT, "the rotated operand outputs must be all null or all set");
  LZ_REQUIRE(!q_hi || (lz::aligned16(q_hi) && lz::aligned16(q_lo) && lz::aligned16(k_hi) &&
                       lz::aligned16(k_lo)),
             LZ_ERR_INVALID_ARGUMENT, "rotated operand outputs must be 16-byte aligned");
  LZ_REQUIRE(lz::aligned16(y), LZ_ERR_INVALID_ARGUMENT, "y must be 16-byte aligned");
  lz::SwaSaved sv;
  if (saved) {
    LZ_REQUIRE(saved_bytes >= lz::swa_saved_layout(B, H, L, D, nullptr, nullptr),
               LZ_ERR_WORKSPACE, "saved buffer too small");
    LZ_REQUIRE(lz::aligned16(saved), LZ_ERR_INVALID_ARGUMENT,
               "saved buffer must be 16-byte aligned");
    lz::swa_saved_layout(B, H, L, D, static_cast<unsigned char*>(saved), &sv);
  }
  lz::SwaRopeArgs a{q, k, v, x_dtype, q_sb, q_sh, q_sl, k_sb, k_sh, k_sl, v_sb, v_sh, v_sl,
                    cos, sin, cs_dtype, cs_sb, cs_sl, meta, n_meta, window,
                    static_cast<bf16*>(y), static_cast<bf16*>(q_hi), static_cast<bf16*>(q_lo),
                    static_cast<bf16*>(k_hi), static_cast<bf16*>(k_lo), B, H, Hkv, L, D};
  rc = lz::swa_rope_fwd(a, sv, static_cast<cudaStream_t>(stream));
  if (rc == LZ_ERR_UNSUPPORTED)
    lz::set_error("lz_swa_rope_fwd: head dim or strides outside the TMA path (rotate with "
                  "lz_rope_split and call lz_swa_fwd_gqa)");
  return rc;
}

extern "C" int lz_swa_fwd(const void* q, const void* k, const void* v, const void* q_lo,
                          const void* k_lo, const float* meta, int n_meta, int window, void* y,
                          void* saved, size_t saved_bytes, int B, int H, int L, int D,
                          void* stream) {
  return lz_swa_fwd_gqa(q, k, v, q_lo, k_lo, meta, n_meta, window, y, saved, saved_bytes, B, H,
                        H, L, D, stream);
}

extern "C" int lz_swa_bwd_gqa(const void* q, const void* k, const void* v, const void* q_lo,
                              const void* k_lo, const float* meta, int n_meta, int window,
                              const void* saved, size_t saved_bytes, const void* dy, void* dq,
                              void* dk, void* dv, int grad_dtype, float* dmeta,
                              void* workspace, size_t workspace_bytes, int B, int H, int Hkv,
                              int L, int D, void* stream) {
  lz::clear_error();
  int rc = check_sizes(B, H, L, 1, D);
  if (rc) return rc;
  LZ_REQUIRE(Hkv >= 1 && H % Hkv == 0, LZ_ERR_INVALID_ARGUMENT,
             "the key/value head count must divide the query head count");
  LZ_REQUIRE(q && k && v && saved && dy && dq && dk && dv && workspace,
             LZ_ERR_INVALID_ARGUMENT, "null pointer");
  LZ_REQUIRE((q_lo == nullptr) == (k_lo == nullptr), LZ_ERR_INVALID_ARGUMENT,
             "q_lo and k_lo must be both null or both set");
  LZ_REQUIRE(n_meta >= 0 && (n_meta == 0 || (meta && dmeta)), LZ_ERR_INVALID_ARGUMENT,
             "meta and dmeta must be non-null when n_meta > 0");
  LZ_REQUIRE(n_meta <= lz::kMaxMeta, LZ_ERR_UNSUPPORTED, "more than 32 sink logits");
  LZ_REQUIRE(window >= 1, LZ_ERR_INVALID_ARGUMENT, "window must be >= 1");
  LZ_REQUIRE(grad_dtype == LZ_DTYPE_F32 || grad_dtype == LZ_DTYPE_BF16, LZ_ERR_INVALID_ARGUMENT,
             "grad_dtype must be LZ_DTYPE_F32 or LZ_DTYPE_BF16");
  LZ_REQUIRE(D <= 128, LZ_ERR_UNSUPPORTED, "head dim above 128 is not supported");
  LZ_REQUIRE(saved_bytes >= lz::swa_saved_layout(B, H, L, D, nullptr, nullptr),
             LZ_ERR_WORKSPACE, "saved buffer too small");
  LZ_REQUIRE(workspace_bytes >= lz::swa_work_layout(B, H, L, n_meta, nullptr, nullptr),
             LZ_ERR_WORKSPACE, "workspace too small");
  LZ_REQUIRE(lz::aligned16(saved), LZ_ERR_INVALID_ARGUMENT,
             "saved buffer must be 16-byte aligned");
  lz::SwaSaved sv;
  lz::swa_saved_layout(B, H, L, D, (unsigned char*)const_cast<void*>(saved), &sv);
  lz::SwaWork wk;
  lz::swa_work_layout(B, H, L, n_meta, static_cast<unsigned char*>(workspace), &wk);
  return lz::swa_bwd(static_cast<const bf16*>(q), static_cast<const bf16*>(k),
                     static_cast<const bf16*>(v), static_cast<const bf16*>(q_lo),
                     static_cast<const bf16*>(k_lo), meta, n_meta, window,
                     sv, static_cast<const bf16*>(dy), dq, dk, dv,
                     grad_dtype, dmeta, wk, B, H, Hkv, L, D, static_cast<cudaStream_t>(stream));
}

extern "C" int lz_swa_bwd(const void* q, const void* k, const void* v, const void* q_lo,
                          const void* k_lo, const float* meta, int n_meta, int window,
                          const void* saved, size_t saved_bytes, const void* dy, void* dq,
                          void* dk, void* dv, int grad_dtype, float* dmeta, void* workspace,
                          size_t workspace_bytes, int B, int H, int L, int D, void* stream) {
  return lz_swa_bwd_gqa(q, k, v, q_lo, k_lo, meta, n_meta, window, saved, saved_bytes, dy, dq,
                        dk, dv, grad_dtype, dmeta, workspace, workspace_bytes, B, H, H, L, D,
                        stream);
}

// ------------------------------------------------ sequence-parallel segments
namespace {

int seg_common(int B, int H, int L, int F, int D, void* workspace, size_t workspace_bytes) {
  int rc = check_sizes(B, H, L, F, D);
  if (rc) return rc;
  LZ_REQUIRE(F <= 256, LZ_ERR_UNSUPPORTED, "feature dim above 256 is not supported");
  LZ_REQUIRE(D <= 128, LZ_ERR_UNSUPPORTED, "value dim above 128 is not supported");
  LZ_REQUIRE(workspace, LZ_ERR_INVALID_ARGUMENT, "null workspace");
  LZ_REQUIRE(lz::aligned16(workspace), LZ_ERR_INVALID_ARGUMENT,
             "workspace must be 16-byte aligned");
  const size_t need = std::max(lz::gla_fwd_work_layout(B, H, L, F, D, nullptr, nullptr),
                               lz::gla_work_layout(B, H, L, F, D, true, nullptr, nullptr));
  LZ_REQUIRE(workspace_bytes >= need, LZ_ERR_WORKSPACE,
             "workspace too small (lz_gla_seg_workspace_bytes)");
  return LZ_OK;
}

int seg_saved(int B, int H, int L, int F, int D, const void* saved, size_t saved_bytes,
              lz::GlaSaved* sv) {
  LZ_REQUIRE(saved_bytes >= lz::gla_saved_layout(B, H, L, F, D, nullptr, nullptr),
             LZ_ERR_WORKSPACE, "saved buffer too small");
  LZ_REQUIRE(lz::aligned16(saved), LZ_ERR_INVALID_ARGUMENT, "saved buffer must be 16-byte aligned");
  lz::gla_saved_layout(B, H, L, F, D, (unsigned char*)const_cast<void*>(saved), sv);
  return LZ_OK;
}

}  // namespace

extern "C" size_t lz_gla_seg_workspace_bytes(int B, int H, int L, int F, int D) {
  if (B < 1 || H < 1 || L < 1 || F < 1 || D < 1) return 0;
  return std::max(lz::gla_fwd_work_layout(B, H, L, F, D, nullptr, nullptr),
                  lz::gla_work_layout(B, H, L, F, D, true, nullptr, nullptr));
}

extern "C" size_t lz_gla_seg_summary_floats(int B, int H, int F, int D) {
  if (B < 1 || H < 1 || F < 1 || D < 1) return 0;
  return lz::gla_seg_summary_floats(B * H, F, D);
}

extern "C" int lz_gla_seg_fwd_begin(const void* fk, const void* v, const float* log_gamma,
                                    int gate_per_head, float* summary, void* workspace,
                                    size_t workspace_bytes, int B, int H, int L, int F, int D,
                                    void* stream) {
  lz::clear_error();
  int rc = seg_common(B, H, L, F, D, workspace, workspace_bytes);
  if (rc) return rc;
  LZ_REQUIRE(fk && v && log_gamma && summary, LZ_ERR_INVALID_ARGUMENT, "null pointer");
  lz::GlaFwdWork fw;
  lz::gla_fwd_work_layout(B, H, L, F, D, static_cast<unsigned char*>(workspace), &fw);
  return lz::gla_seg_fwd_begin(static_cast<const bf16*>(fk), static_cast<const bf16*>(v),
                               log_gamma, gate_per_head ? 1 : 0, summary, fw, B, H, L, F, D,
                               static_cast<cudaStream_t>(stream));
}

extern "C" int lz_gla_seg_fwd_end(const void* fq, const void* fk, const void* v,
                                  const float* log_gamma, int gate_per_head, const float* seed,
                                  void* y, void* saved, size_t saved_bytes, void* workspace,
                                  size_t workspace_bytes, int B, int H, int L, int F, int D,
                                  void* stream) {
  lz::clear_error();
  int rc = seg_common(B, H, L, F, D, workspace, workspace_bytes);
  if (rc) return rc;
  LZ_REQUIRE(fq && fk && v && log_gamma && y, LZ_ERR_INVALID_ARGUMENT, "null pointer");
  lz::GlaSaved sv;
  if (saved) {
    rc = seg_saved(B, H, L, F, D, saved, saved_bytes, &sv);
    if (rc) return rc;
  }
  lz::GlaFwdWork fw;
  lz::gla_fwd_work_layout(B, H, L, F, D, static_cast<unsigned char*>(workspace), &fw);
  return lz::gla_seg_fwd_end(static_cast<const bf16*>(fq), static_cast<const bf16*>(fk),
                             static_cast<const bf16*>(v), log_gamma, gate_per_head ? 1 : 0, seed,
                             static_cast<bf16*>(y), sv, fw, B, H, L, F, D,
                             static_cast<cudaStream_t>(stream));
}

extern "C" int lz_gla_seg_bwd_begin(const void* fq, const void* saved, size_t saved_bytes,
                                    const void* dy, float* summary, void* workspace,
                                    size_t workspace_bytes, int B, int H, int L, int F, int D,
                                    void* stream) {
  lz::clear_error();
  int rc = seg_common(B, H, L, F, D, workspace, workspace_bytes);
  if (rc) return rc;
  LZ_REQUIRE(fq && saved && dy && summary, LZ_ERR_INVALID_ARGUMENT, "null pointer");
  lz::GlaSaved sv;
  rc = seg_saved(B, H, L, F, D, saved, saved_bytes, &sv);
  if (rc) return rc;
  lz::GlaWork wk;
  lz::gla_work_layout(B, H, L, F, D, true, static_cast<unsigned char*>(workspace), &wk);
  return lz::gla_seg_bwd_begin(static_cast<const bf16*>(fq), static_cast<const bf16*>(dy), sv,
                               summary, wk, B, H, L, F, D, static_cast<cudaStream_t>(stream));
}

extern "C" int lz_gla_seg_bwd_end(const void* fq, const void* fk, const void* v,
                                  int gate_per_head, const void* saved, size_t saved_bytes,
                                  const void* dy, const float* dseed, int seeded_forward,
                                  void* dfq, void* dfk, void* dv, int grad_dtype,
                                  float* dlog_gamma, void* workspace, size_t workspace_bytes,
                                  int B, int H, int L, int F, int D, void* stream) {
  lz::clear_error();
  int rc = seg_common(B, H, L, F, D, workspace, workspace_bytes);
  if (rc) return rc;
  LZ_REQUIRE(fq && fk && v && saved && dy && dfq && dfk && dv && dlog_gamma,
             LZ_ERR_INVALID_ARGUMENT, "null pointer");
  LZ_REQUIRE(grad_dtype == LZ_DTYPE_F32 || grad_dtype == LZ_DTYPE_BF16, LZ_ERR_INVALID_ARGUMENT,
             "grad_dtype must be LZ_DTYPE_F32 or LZ_DTYPE_BF16");
  lz::GlaSaved sv;
  rc = seg_saved(B, H, L, F, D, saved, saved_bytes, &sv);
  if (rc) return rc;
  lz::GlaWork wk;
  lz::gla_work_layout(B, H, L, F, D, true, static_cast<unsigned char*>(workspace), &wk);
  return lz::gla_seg_bwd_end(static_cast<const bf16*>(fq), static_cast<const bf16*>(fk),
                             static_cast<const bf16*>(v), gate_per_head ? 1 : 0, sv,
                             static_cast<const bf16*>(dy), dseed, seeded_forward ? 1 : 0, dfq,
                             dfk, dv, grad_dtype, dlog_gamma, wk, B, H, L, F, D,
                             static_cast<cudaStream_t>(stream));
}

extern "C" int lz_gla_seg_combine(const float* summaries, int P, int rank, int reverse,
                                  float* seed, int B, int H, int F, int D, void* stream) {
  lz::clear_error();
  LZ_REQUIRE(summaries && seed, LZ_ERR_INVALID_ARGUMENT, "null pointer");
  LZ_REQUIRE(P >= 1 && rank >= 0 && rank < P, LZ_ERR_INVALID_ARGUMENT, "rank must be in [0, P)");
  LZ_REQUIRE(B >= 1 && H >= 1 && F >= 1 && D >= 1, LZ_ERR_INVALID_ARGUMENT,
             "sizes must be positive");
  return lz::gla_seg_combine(summaries, P, rank, reverse ? 1 : 0, seed, B * H, F, D,
                             static_cast<cudaStream_t>(stream));
}

extern "C" int lz_gla_seg_gate_offset(float* dlog_gamma, const float* totals, int P, int rank,
                                      int rows, int L, void* stream) {
  lz::clear_error();
  LZ_REQUIRE(dlog_gamma && totals, LZ_ERR_INVALID_ARGUMENT, "null pointer");
  LZ_REQUIRE(P >= 1 && rank >= 0 && rank < P, LZ_ERR_INVALID_ARGUMENT, "rank must be in [0, P)");
  LZ_REQUIRE(rows >= 1 && L >= 1, LZ_ERR_INVALID_ARGUMENT, "sizes must be positive");
  return lz::gla_seg_gate_offset(dlog_gamma, totals, P, rank, rows, L,
                                 static_cast<cudaStream_t>(stream));
}
