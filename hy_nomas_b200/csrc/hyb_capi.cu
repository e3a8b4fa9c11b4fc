// Library identity, per-thread error messages and device checks for the C ABI.
#include <stdarg.h>
#include <string.h>

#include "hyb_common.cuh"

namespace hyb {

static thread_local char g_last_error[1024] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int device_cc_major() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return -1;
  return major;
}

}  // namespace hyb

extern "C" int hyb_version(void) { return HYB_ABI_VERSION; }

extern "C" int hyb_last_error(char* buf, size_t len) {
  size_t n = strlen(hyb::g_last_error);
  if (buf != nullptr && len > 0) {
    size_t c = n < len - 1 ? n : len - 1;
    memcpy(buf, hyb::g_last_error, c);
    buf[c] = 0;
  }
  return static_cast<int>(n);
}

extern "C" int hyb_device_supported(void) { return hyb::device_cc_major() == 10 ? 1 : 0; }

namespace hyb {
namespace {
__global__ void exp2_poly_kernel(const float* x, float* y, long long n) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; 2 * i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const bool two = 2 * i + 1 < n;
    const float2 e = exp2_poly2(make_float2(x[2 * i], two ? x[2 * i + 1] : 0.f));
    y[2 * i] = e.x;
    if (two) y[2 * i + 1] = e.y;
  }
}
}  // namespace
}  // namespace hyb

extern "C" int hyb_exp2_poly_eval(const float* x, float* y, int64_t n, void* stream) {
  if (n < 0 || (n > 0 && (x == nullptr || y == nullptr)))
    return hyb::fail(HYB_ERR_INVALID_ARG, "exp2_poly_eval: bad arguments");
  if (n == 0) return HYB_OK;
  long long blocks = ((n + 1) / 2 + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  hyb::exp2_poly_kernel<<<static_cast<int>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n);
  HYB_CHECK_LAUNCH();
  return HYB_OK;
}
