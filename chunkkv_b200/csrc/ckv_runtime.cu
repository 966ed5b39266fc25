// Library plumbing of the C ABI: error message, device error word, SM count.
#include <mutex>

#include "ckv_common.cuh"

namespace ckv {

static thread_local std::string g_last_error;

void set_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

constexpr int kMaxDevices = 64;

int num_sms() {
  static int cache[kMaxDevices] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

int set_smem_limit(const void* kernel, int bytes) {
  // One attribute call per (kernel, device) and size: the cap is raised when a launch needs
  // more than the largest size set so far (kernels whose shared memory depends on the
  // shape); the table is small and append-only.
  struct Entry {
    const void* k;
    int dev;
    int bytes;
  };
  static Entry done[256];
  static int n_done = 0;
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  Entry* hit = nullptr;
  for (int i = 0; i < n_done; ++i)
    if (done[i].k == kernel && done[i].dev == dev) hit = &done[i];
  if (hit && hit->bytes >= bytes) return 0;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) {
    set_error("cudaFuncSetAttribute(%d bytes): %s", bytes, cudaGetErrorString(e));
    return CKV_ERR_CUDA;
  }
  if (hit)
    hit->bytes = bytes;
  else if (n_done < 256)
    done[n_done++] = {kernel, dev, bytes};
  return 0;
}

// Per-translation-unit device error words (each .cu owns one).
uint32_t read_clear_err_rope();
uint32_t read_clear_err_select();
uint32_t read_clear_err_gemm();
uint32_t read_clear_err_attention_tc();
uint32_t read_clear_err_elementwise();
uint32_t read_clear_err_tp_reduce();
uint32_t read_clear_err_gemv_fused();

}  // namespace ckv

extern "C" {

const char* ckv_version(void) { return "chunkkv_b200 0.1 (sm_100a)"; }

const char* ckv_last_error(void) { return ckv::g_last_error.c_str(); }

int ckv_get_device_error(uint32_t* code) {
  if (code == nullptr) {
    ckv::set_error("ckv_get_device_error: null output");
    return CKV_ERR_ARG;
  }
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    ckv::set_error("ckv_get_device_error: device sync failed: %s", cudaGetErrorString(e));
    return CKV_ERR_CUDA;
  }
  *code = ckv::read_clear_err_rope() | ckv::read_clear_err_select() | ckv::read_clear_err_gemm() |
          ckv::read_clear_err_attention_tc() |
          ckv::read_clear_err_elementwise() | ckv::read_clear_err_tp_reduce() |
          ckv::read_clear_err_gemv_fused();
  return CKV_OK;
}

}  // extern "C"
