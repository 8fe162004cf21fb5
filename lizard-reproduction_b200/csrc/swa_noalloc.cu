// lz_swa_bwd_noalloc: the SWA backward for callers that cannot allocate.
//
// Some hosts hand a plugin nothing but its input and output buffers: a
// serving runtime's custom-op hook with no workspace request, or an
// embedding framework whose allocator the plugin cannot reach. Such a caller
// has no way to provide the workspace lz_swa_bwd asks for. This entry point
// uses instead a fixed scratch array that lives in the library image on
// every GPU that loads it, and calls no allocator at all.
//
// Limits and sharing:
//  * The scratch holds kNoAllocScratchBytes (4 MiB): the per-row delta
//    (4 B x B*H*L) and the per-block sink partials (4 B x B*H*ceil(L/64) x
//    n_meta), each 256-byte aligned. Larger problems are rejected with
//    LZ_ERR_UNSUPPORTED; use lz_swa_bwd with a caller-owned workspace.
//  * Every call on a device shares the one array and finds the previous
//    call's contents there. Nothing in it needs to start at zero: the dq
//    kernel writes every delta and partial before they are read. Calls whose
//    work overlaps on the GPU (different streams, no ordering between them)
//    race on the array; serialise them.
//  * The first call on each device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current and caches it; make that
//    first call before any stream capture. The cached address belongs to the
//    device's primary context: after cudaDeviceReset (or anything else that
//    destroys that context) it is stale, so a process that resets a device
//    must not call this entry point on it again.
#include <mutex>

#include "common.cuh"
#include "swa_layout.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;

// Host code must not use this name as a pointer: on the host it is only a
// stand-in for the symbol. Its device address comes from scratch_address().
static __device__ __align__(256) unsigned char g_swa_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_addr[64] = {nullptr};

int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    lz::set_error(std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    return LZ_ERR_CUDA;
  }
  if (dev < 0 || dev >= 64) {
    lz::set_error("lz_swa_bwd_noalloc: device ordinal above 63");
    return LZ_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_swa_scratch);
    if (e != cudaSuccess || p == nullptr) {
      lz::set_error(std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
      return LZ_ERR_CUDA;
    }
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return LZ_OK;
}

}  // namespace

extern "C" int lz_swa_bwd(const void* q, const void* k, const void* v, const void* q_lo,
                          const void* k_lo, const float* meta, int n_meta, int window,
                          const void* saved, size_t saved_bytes, const void* dy, void* dq,
                          void* dk, void* dv, int grad_dtype, float* dmeta, void* workspace,
                          size_t workspace_bytes, int B, int H, int L, int D, void* stream);

extern "C" int lz_swa_bwd_noalloc(const void* q, const void* k, const void* v, const void* q_lo,
                                  const void* k_lo, const float* meta, int n_meta, int window,
                                  const void* saved, size_t saved_bytes, const void* dy,
                                  void* dq, void* dk, void* dv, int grad_dtype, float* dmeta,
                                  int B, int H, int L, int D, void* stream) {
  lz::clear_error();
  LZ_REQUIRE(B >= 1 && H >= 1 && L >= 1 && n_meta >= 0, LZ_ERR_INVALID_ARGUMENT,
             "B, H, L must be positive and n_meta non-negative");
  const size_t need = lz::swa_work_layout(B, H, L, n_meta, nullptr, nullptr);
  LZ_REQUIRE(need <= kNoAllocScratchBytes, LZ_ERR_UNSUPPORTED,
             "problem needs " + std::to_string(need) +
                 " bytes of scratch, above the fixed 4 MiB of lz_swa_bwd_noalloc; "
                 "call lz_swa_bwd with a workspace");
  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc) return rc;
  return lz_swa_bwd(q, k, v, q_lo, k_lo, meta, n_meta, window, saved, saved_bytes, dy, dq, dk,
                    dv, grad_dtype, dmeta, scratch, kNoAllocScratchBytes, B, H, L, D, stream);
}
