// Library-wide C-ABI plumbing: version, thread-local error message, device
// architecture gate, SM count cache.
#include "jo_common.cuh"

#include <string.h>

namespace jo {

static thread_local char g_err[1024] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

static constexpr int kMaxDev = 64;
static int g_arch[kMaxDev] = {0};   // 0 = unknown
static int g_sms[kMaxDev] = {0};

static int query(int dev) {
  if (dev < 0 || dev >= kMaxDev) return -1;
  if (g_arch[dev] == 0) {
    int mj = 0, mn = 0, sms = 0;
    if (cudaDeviceGetAttribute(&mj, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&mn, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      cudaGetLastError();
      return -1;
    }
    g_sms[dev] = sms;
    g_arch[dev] = mj * 10 + mn;
  }
  return g_arch[dev];
}

int require_sm100() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    set_error("joyomni_b200: no CUDA device available");
    return JO_ERR_CUDA;
  }
  int arch = query(dev);
  if (arch < 0) {
    set_error("joyomni_b200: cannot query device %d", dev);
    return JO_ERR_CUDA;
  }
  if (arch != 100) {
    set_error("joyomni_b200 kernels are built for sm_100a only; current device has compute capability %d",
              arch);
    return JO_ERR_ARCH;
  }
  return JO_OK;
}

int sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  query(dev);
  return (dev >= 0 && dev < kMaxDev && g_sms[dev] > 0) ? g_sms[dev] : 148;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: CUDA launch failed: %s", what, cudaGetErrorString(e));
    return JO_ERR_CUDA;
  }
  return JO_OK;
}

}  // namespace jo

extern "C" {

int jo_version(void) { return 100; }

const char* jo_last_error(void) { return jo::g_err; }

int jo_device_arch(int device) {
  int a = jo::query(device);
  if (a < 0) {
    jo::set_error("jo_device_arch: cannot query device %d", device);
    return JO_ERR_CUDA;
  }
  return a;
}

}  // extern "C"
