// Error reporting, device error word and small host utilities of the C ABI.
#include <mutex>
#include <string>

#include "common.cuh"
#include "grid_sync.cuh"

namespace aoakv {

// Device-side error word (one per device that loads the library). Kernels
// receive its address as a parameter and set it with raise_dev_error().
__device__ int g_dev_error;

namespace {
thread_local std::string t_last_error;
constexpr int kMaxDevices = 64;
std::mutex g_mu;
int* g_err_ptr[kMaxDevices] = {nullptr};
int g_sms[kMaxDevices] = {0};
}  // namespace

int set_error(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

int cuda_status(cudaError_t st, const char* what) {
  if (st == cudaSuccess) return AOAKV_OK;
  return set_error(AOAKV_ERR_CUDA, std::string(what) + ": " +
                                       cudaGetErrorName(st) + " (" +
                                       cudaGetErrorString(st) + ")");
}

int* dev_error_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_err_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_dev_error) != cudaSuccess) return nullptr;
    g_err_ptr[dev] = static_cast<int*>(p);
  }
  return g_err_ptr[dev];
}

int num_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return 148;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_sms[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) !=
            cudaSuccess ||
        n <= 0)
      n = 148;
    g_sms[dev] = n;
  }
  return g_sms[dev];
}

}  // namespace aoakv

extern "C" {

const char* aoakv_last_error(void) { return aoakv::t_last_error.c_str(); }

int aoakv_version(void) { return 1 * 10000 + 0 * 100 + 0; }

int aoakv_get_device_error(int32_t* code_out, int32_t clear) {
  AOAKV_CHECK_ARG(code_out != nullptr, "code_out is NULL");
  int* p = aoakv::dev_error_ptr();
  if (!p)
    return aoakv::set_error(AOAKV_ERR_CUDA,
                            "cannot resolve the device error word");
  AOAKV_CUDA_TRY(cudaDeviceSynchronize(), "aoakv_get_device_error sync");
  int v = 0;
  AOAKV_CUDA_TRY(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost),
                 "aoakv_get_device_error read");
  *code_out = v;
  if (clear) {
    AOAKV_CUDA_TRY(cudaMemset(p, 0, sizeof(int)), "aoakv_get_device_error clear");
    AOAKV_CUDA_TRY(cudaDeviceSynchronize(), "aoakv_get_device_error sync");
  }
  return AOAKV_OK;
}

// One CTA waits, bounded by limit_us, until *flag >= target: the wait the
// fused step kernels use between their phases, with a caller-chosen limit.
namespace {
__global__ void debug_wait_kernel(const uint32_t* flag, uint32_t target, uint64_t limit_ns,
                                  int* err) {
  __shared__ int ok_s;
  aoakv::cta_wait_geq(flag, target, &ok_s, err, limit_ns);
}
}  // namespace

int aoakv_debug_wait_flag(const uint32_t* flag, uint32_t target, int32_t limit_us,
                          void* stream) {
  AOAKV_CHECK_ARG(flag != nullptr, "debug_wait_flag: flag is NULL");
  AOAKV_CHECK_ARG(limit_us >= 1 && limit_us <= 1000000,
                  "debug_wait_flag: limit_us must be in [1, 1000000]");
  int* err = aoakv::dev_error_ptr();
  if (!err) return aoakv::set_error(AOAKV_ERR_CUDA, "cannot resolve the device error word");
  debug_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      flag, target, static_cast<uint64_t>(limit_us) * 1000ull, err);
  AOAKV_CUDA_TRY(cudaGetLastError(), "debug_wait_flag launch");
  return AOAKV_OK;
}

}  // extern "C"
