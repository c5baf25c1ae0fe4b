// Error state, ABI version and launch count of the C entry points.
#include <atomic>

#include "common.cuh"

namespace lsb {

static thread_local char g_last_error[1024] = "";
static std::atomic<int64_t> g_launches{0};

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

}  // namespace lsb

extern "C" const char* lsb_last_error(void) { return lsb::g_last_error; }

extern "C" int lsb_abi_version(void) { return 1; }

extern "C" int64_t lsb_kernel_launch_count(void) {
  return lsb::g_launches.load(std::memory_order_relaxed);
}

// ---------------------------------------------------------------------------
// Sticky device error word: kernels OR LSB_DEVERR_* bits into it instead of
// faulting on a bad index. One word per device, addressed through the runtime.
// ---------------------------------------------------------------------------
__device__ int g_lsb_device_error;

int* lsb_device_error_flag() {
  static int* cached[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!cached[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_lsb_device_error) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    cached[dev] = static_cast<int*>(p);
  }
  return cached[dev];
}

extern "C" int lsb_device_error_word(int32_t* out, int32_t reset, void* stream) {
  int* flag = lsb_device_error_flag();
  if (!flag) return lsb::fail(LSB_ERR_CUDA, "device error word unavailable");
  int value = 0;
  LSB_CUDA(cudaMemcpyAsync(&value, flag, sizeof(int), cudaMemcpyDeviceToHost,
                           lsb::as_stream(stream)));
  if (reset) LSB_CUDA(cudaMemsetAsync(flag, 0, sizeof(int), lsb::as_stream(stream)));
  LSB_CUDA(cudaStreamSynchronize(lsb::as_stream(stream)));
  if (out) *out = value;
  return LSB_OK;
}
