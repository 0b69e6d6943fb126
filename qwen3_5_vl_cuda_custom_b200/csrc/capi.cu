// Library-wide C ABI pieces: status strings, last-error detail, the per-device
// error word, SM count and tensor-map encoding through the driver entry point.
#include <cudaTypedefs.h>
#include <stdarg.h>
#include <stdio.h>

#include <atomic>
#include <map>
#include <mutex>
#include <utility>

#include "sm100.cuh"

namespace q35 {

namespace {
thread_local char g_last_msg[512] = "";
constexpr int kMaxDevices = 64;
int *g_err_word[kMaxDevices] = {};
int g_num_sms[kMaxDevices] = {};
std::mutex g_mu;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int current_device(int *dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (*dev < 0 || *dev >= kMaxDevices)
    return fail(Q35_ERR_NO_DEVICE, "device ordinal %d out of range", *dev);
  return Q35_OK;
}
}  // namespace

int fail(int status, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_msg, sizeof(g_last_msg), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_fail(cudaError_t e, const char *what) {
  return fail(Q35_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int *device_error_word() {
  int dev = 0;
  if (current_device(&dev) != Q35_OK) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_err_word[dev] == nullptr) {
    int *p = nullptr;
    if (cudaMalloc(&p, 4 * sizeof(int)) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, 4 * sizeof(int)) != cudaSuccess) return nullptr;
    g_err_word[dev] = p;
  }
  return g_err_word[dev];
}

thread_local int g_sm_limit = 0;  // 0: all SMs

int num_sms() {
  int dev = 0;
  if (current_device(&dev) != Q35_OK) return 1;
  if (g_num_sms[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_num_sms[dev] = n > 0 ? n : 1;
  }
  const int hw = g_num_sms[dev];
  return (g_sm_limit > 0 && g_sm_limit < hw) ? g_sm_limit : hw;
}

int ensure_smem_attr(const void *kernel, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<int, const void *>, int> done;
  int dev = 0;
  int st = current_device(&dev);
  if (st) return st;
  std::lock_guard<std::mutex> lk(mu);
  auto key = std::make_pair(dev, kernel);
  auto it = done.find(key);
  if (it != done.end() && it->second >= bytes) return Q35_OK;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic smem)");
  done[key] = bytes;
  return Q35_OK;
}

int make_tmap_bf16_2d(CUtensorMap *map, const void *base, uint64_t inner,
                      uint64_t outer, uint64_t row_pitch_bytes,
                      uint32_t box_inner, uint32_t box_outer) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_encode == nullptr) {
      cudaDriverEntryPointQueryResult q;
      void *fn = nullptr;
      cudaError_t e = cudaGetDriverEntryPointByVersion(
          "cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
      if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
        return fail(Q35_ERR_CUDA, "cuTensorMapEncodeTiled entry point missing");
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  }
  if (!aligned16(base) || (row_pitch_bytes & 15u) != 0)
    return fail(Q35_ERR_ALIGN, "TMA operand %p pitch %llu not 16-byte aligned",
                base, (unsigned long long)row_pitch_bytes);
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_pitch_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                        const_cast<void *>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(Q35_ERR_CUDA,
                "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu box %u x %u",
                (int)r, (unsigned long long)inner, (unsigned long long)outer,
                box_inner, box_outer);
  return Q35_OK;
}

std::atomic<long long> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

}  // namespace q35

extern "C" {

int64_t q35_launch_count(void) { return q35::g_launches.load(); }

const char *q35_status_string(int status) {
  switch (status) {
    case Q35_OK: return "ok";
    case Q35_ERR_INVALID: return "invalid argument";
    case Q35_ERR_SHAPE: return "unsupported shape";
    case Q35_ERR_ALIGN: return "pointer or pitch not 16-byte aligned";
    case Q35_ERR_UNSUPPORTED: return "unsupported configuration";
    case Q35_ERR_CUDA: return "CUDA error";
    case Q35_ERR_DEVICE: return "device-side error recorded";
    case Q35_ERR_NO_DEVICE: return "no usable CUDA device";
    default: return "unknown status";
  }
}

const char *q35_last_error_message(void) { return q35::g_last_msg; }

const char *q35_version(void) { return "q35b200 sm_100a"; }

int q35_set_sm_limit(int n) {
  if (n < 0) return q35::fail(Q35_ERR_INVALID, "sm limit %d < 0", n);
  q35::g_sm_limit = n;
  return Q35_OK;
}

int q35_device_error_check(int32_t *info4) {
  int *w = q35::device_error_word();
  if (w == nullptr) return q35::fail(Q35_ERR_CUDA, "no device error word");
  Q35_CHECK_CUDA(cudaDeviceSynchronize());
  int host[4] = {0, 0, 0, 0};
  Q35_CHECK_CUDA(cudaMemcpy(host, w, sizeof(host), cudaMemcpyDeviceToHost));
  if (info4)
    for (int i = 0; i < 4; ++i) info4[i] = host[i];
  if (host[0] != 0) {
    Q35_CHECK_CUDA(cudaMemset(w, 0, sizeof(host)));
    return q35::fail(Q35_ERR_DEVICE, "device error code %d at site %d (%d, %d)",
                     host[0], host[1], host[2], host[3]);
  }
  return Q35_OK;
}

}  // extern "C"
