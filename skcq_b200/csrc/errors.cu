// Error reporting across the C ABI and small host-side helpers.
#include <stdarg.h>
#include <string.h>

#include "common.cuh"

namespace skcq {

static thread_local char g_last_error[1024] = "";

// Device-side error word: set by bounded waits and device checks, read (and
// cleared) by skcq_poll_device_error().
__device__ int g_device_error = 0;

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof g_last_error, fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(SKCQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return SKCQ_OK;
}

int* device_error_word() {
  static thread_local int* ptr = nullptr;
  static thread_local int dev = -1;
  int cur = 0;
  cudaGetDevice(&cur);
  if (ptr == nullptr || dev != cur) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    ptr = static_cast<int*>(p);
    dev = cur;
  }
  return ptr;
}

}  // namespace skcq

extern "C" int skcq_last_error(char* buf, size_t len) {
  if (buf == nullptr || len == 0) return SKCQ_ERR_INVALID;
  strncpy(buf, skcq::g_last_error, len - 1);
  buf[len - 1] = '\0';
  return SKCQ_OK;
}

extern "C" int skcq_abi_version(void) { return 10; }

extern "C" int skcq_packed_width(int metric, int bs) {
  if (bs <= 0) return skcq::set_error(SKCQ_ERR_INVALID, "block size must be positive (got %d)", bs);
  int k = 3 * bs + (metric == SKCQ_METRIC_L2 ? 2 : 0);
  return (k + 7) / 8 * 8;
}

extern "C" int skcq_poll_device_error(void* stream) {
  int* word = skcq::device_error_word();
  if (word == nullptr) return skcq::set_error(SKCQ_ERR_CUDA, "cannot resolve the device error word");
  int host = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(&host, word, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return skcq::set_error(SKCQ_ERR_CUDA, "device error poll: %s", cudaGetErrorString(e));
  if (host != 0) {
    int zero = 0;
    cudaMemcpyAsync(word, &zero, sizeof(int), cudaMemcpyHostToDevice, s);
    cudaStreamSynchronize(s);
    return skcq::set_error(SKCQ_ERR_DEVICE, "device-side check failed (code %d)", host);
  }
  return SKCQ_OK;
}

// Self-test of the bounded device waits: one thread waits on a shared-memory
// mbarrier that nothing arrives on, with the given clock limit, through the
// same wait the kernels use. The wait runs out, records SKCQ_DEVICE_CODE_SELFTEST
// in the device error word and the kernel returns; nothing faults or hangs.
__global__ void selftest_wait_kernel(long long limit_clocks, int* err) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  skcq::mbar_init(&bar, 1);
  skcq::fence_barrier_init();
  skcq::mbar_wait_limit(&bar, 0, err, SKCQ_DEVICE_CODE_SELFTEST, limit_clocks);
}

extern "C" int skcq_selftest_wait_timeout(long long limit_clocks, void* stream) {
  SKCQ_REQUIRE(limit_clocks > 0 && limit_clocks <= 4000000000ll, SKCQ_ERR_INVALID,
               "selftest_wait_timeout: limit %lld clocks outside (0, 4e9]", limit_clocks);
  int* err = skcq::device_error_word();
  if (err == nullptr) return skcq::set_error(SKCQ_ERR_CUDA, "selftest_wait_timeout: no device error word");
  selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_clocks, err);
  return skcq::check_launch("selftest_wait_timeout");
}
