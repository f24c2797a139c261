// Library-wide status entry points: version, thread-local error messages, device error words.
#include "common.cuh"

#include <mutex>
#include <vector>

namespace xsake {

static thread_local std::string t_last_error;

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error.assign(buf);
  return code;
}

void clear_error() { t_last_error.clear(); }

static std::vector<DeviceErrorReader>& readers() {
  static std::vector<DeviceErrorReader> r;
  return r;
}
static std::mutex& readers_mu() {
  static std::mutex m;
  return m;
}

void register_device_error_reader(DeviceErrorReader fn) {
  std::lock_guard<std::mutex> g(readers_mu());
  readers().push_back(fn);
}

static constexpr int kMaxDevices = 64;
static DeviceInfo g_info[kMaxDevices];
static std::once_flag g_info_once[kMaxDevices];

int device_info(DeviceInfo* out) {
  int dev = 0;
  XSAKE_CUDA_TRY(cudaGetDevice(&dev));
  XSAKE_REQUIRE(dev >= 0 && dev < kMaxDevices, XSAKE_EUNSUPPORTED, "device ordinal %d", dev);
  cudaError_t err = cudaSuccess;
  std::call_once(g_info_once[dev], [&] {
    DeviceInfo d;
    int v = 0;
    err = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (err == cudaSuccess) err = cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev);
    if (err == cudaSuccess) err = cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (err == cudaSuccess) err = cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    d.smem_optin = (size_t)v;
    g_info[dev] = d;
  });
  XSAKE_REQUIRE(err == cudaSuccess, XSAKE_ECUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(err));
  XSAKE_REQUIRE(g_info[dev].sm_count > 0, XSAKE_ECUDA, "device attributes unavailable");
  *out = g_info[dev];
  return XSAKE_OK;
}

}  // namespace xsake

extern "C" {

int xsake_abi_version(void) { return XSAKE_ABI_VERSION; }

const char* xsake_last_error(void) { return xsake::t_last_error.c_str(); }

int xsake_device_error(void* stream, int32_t* code) {
  XSAKE_REQUIRE(code != nullptr, XSAKE_EINVAL, "code is NULL");
  *code = 0;
  std::vector<xsake::DeviceErrorReader> rs;
  {
    std::lock_guard<std::mutex> g(xsake::readers_mu());
    rs = xsake::readers();
  }
  for (auto fn : rs) {
    int32_t c = 0;
    if (fn(xsake::as_stream(stream), &c) != 0)
      return xsake::set_error(XSAKE_ECUDA, "reading a device error word failed: %s",
                              cudaGetErrorString(cudaGetLastError()));
    if (c != 0 && *code == 0) *code = c;
  }
  return XSAKE_OK;
}

}  // extern "C"
