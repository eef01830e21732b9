// Error plumbing and device queries shared by every entry point.
#include <stdarg.h>
#include <stdio.h>

#include <atomic>

#include "common.cuh"
#include "tmap.cuh"

namespace gdn {

EncodeTiledFn encode_tiled() {
  // looked up once (a function-local static is initialised once, thread-safe)
  static const EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFn>(p);
    return nullptr;
  }();
  return fn;
}

static thread_local char g_last_error[1024] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

void clear_error() { g_last_error[0] = 0; }

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: CUDA launch failed: %s", what, cudaGetErrorString(e));
    return GDN_ERR_CUDA;
  }
  return GDN_OK;
}

int sm_count() {
  // per device; concurrent first calls store the same value
  static std::atomic<int> cached[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cached[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

static std::atomic<int64_t> g_wait_limit{-1};

uint32_t wait_limit(uint32_t dflt) {
  const int64_t v = g_wait_limit.load(std::memory_order_relaxed);
  return v < 0 ? dflt : (uint32_t)(v > 0xFFFFFFFFll ? 0xFFFFFFFFll : v);
}

}  // namespace gdn

extern "C" int gdn_abi_version(void) { return GDN_ABI_VERSION; }

extern "C" void gdn_set_wait_limit(int64_t polls) {
  gdn::g_wait_limit.store(polls < 0 ? -1 : polls, std::memory_order_relaxed);
}

extern "C" const char* gdn_last_error(void) { return gdn::g_last_error; }
