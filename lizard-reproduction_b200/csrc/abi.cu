// Error reporting, version and launch accounting of the C ABI.
#include <atomic>
#include <string>

#include "common.cuh"

namespace lz {

static thread_local std::string g_last_error;
static std::atomic<uint64_t> g_launches{0};

void set_error(const std::string& msg) { g_last_error = msg; }
void clear_error() { g_last_error.clear(); }
void count_launches(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return LZ_ERR_CUDA;
  }
  return LZ_OK;
}

}  // namespace lz

extern "C" int lz_abi_version(void) { return LZ_ABI_VERSION; }

extern "C" const char* lz_last_error_string(void) { return lz::g_last_error.c_str(); }

extern "C" uint64_t lz_launch_count(void) {
  return lz::g_launches.load(std::memory_order_relaxed);
}
