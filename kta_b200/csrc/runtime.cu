// Per-device library state and the small entries of the C ABI: version, status text,
// device status block, SM count, tensor-map encoding.
#include <mutex>
#include <set>
#include <utility>

#include <cudaTypedefs.h>

#include "kta_common.cuh"
#include "kta_host.h"

namespace {

constexpr int kMaxDevices = 64;

// The device status block the kernels' watchdogs write (kta_common.cuh record_status).
__device__ unsigned int g_kta_device_status[4];

struct DeviceState {
  std::once_flag once;
  unsigned int* status = nullptr;
  int sm_count = 0;
  int cc_major = -1;
};

DeviceState g_devices[kMaxDevices];

PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;
std::once_flag g_encode_once;

DeviceState* state_of_current() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  DeviceState* s = &g_devices[dev];
  std::call_once(s->once, [s, dev]() {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_kta_device_status) == cudaSuccess) {
      s->status = static_cast<unsigned int*>(p);
    } else {
      (void)cudaGetLastError();
    }
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess) {
      s->sm_count = v;
    }
    if (cudaDeviceGetAttribute(&v, cudaDevAttrComputeCapabilityMajor, dev) == cudaSuccess) {
      s->cc_major = v;
    }
  });
  return s;
}

thread_local int t_last_error = KTA_OK;

}  // namespace

namespace kta {

unsigned int* device_status_ptr() {
  DeviceState* s = state_of_current();
  return s ? s->status : nullptr;
}

int current_sm_count() {
  DeviceState* s = state_of_current();
  return s ? s->sm_count : 0;
}

int current_cc_major() {
  DeviceState* s = state_of_current();
  return s ? s->cc_major : -1;
}

int require_sm100() {
  int major = current_cc_major();
  if (major < 0) return KTA_ERR_NO_DEVICE;
  if (major != 10) return KTA_ERR_NO_DEVICE;
  return KTA_OK;
}

int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, []() {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    } else {
      (void)cudaGetLastError();
    }
  });
  if (g_encode_tiled == nullptr) return KTA_ERR_CUDA;
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) {
    if (strides_bytes[i] % 16 != 0) return KTA_ERR_ALIGN;
    gstride[i] = strides_bytes[i];
  }
  CUresult r = g_encode_tiled(map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base),
                              gdim, gstride, bdim, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? KTA_OK : KTA_ERR_INVALID_ARG;
}

int launch_status() {
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return KTA_OK;
  return KTA_ERR_LAUNCH;
}

void set_last_error(int s) { t_last_error = s; }

int set_kernel_smem(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return KTA_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({kernel, dev})) return KTA_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
      cudaSuccess) {
    (void)cudaGetLastError();
    return KTA_ERR_LAUNCH;
  }
  done.insert({kernel, dev});
  return KTA_OK;
}

}  // namespace kta

namespace {

// Site recorded by the watchdog self-test.
constexpr unsigned int kSelftestSite = 0x7F01;

// One thread waits, through the kernels' own bounded wait, for a phase of a barrier that no
// thread ever completes: the wait expires after `timeout_ns`, records KTA_ERR_DEVICE_TIMEOUT
// and the site, and the kernel returns. Nothing faults and nothing is left waiting.
__global__ void watchdog_selftest_kernel(unsigned int* status, unsigned long long timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    kta::mbar_init(&bar, 1);
    abort_flag = 0;
    kta::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    (void)kta::mbar_wait(&bar, 0u, &abort_flag, status, kSelftestSite, timeout_ns);
  }
}

}  // namespace

extern "C" {

int kta_abi_version(void) { return KTA_ABI_VERSION; }

int kta_watchdog_selftest(uint64_t timeout_ns, void* stream) {
  if (timeout_ns < 1000ull || timeout_ns > 10000000000ull) return KTA_ERR_INVALID_ARG;
  int s = kta::require_sm100();
  if (s != KTA_OK) return s;
  unsigned int* status = kta::device_status_ptr();
  if (status == nullptr) return KTA_ERR_NO_DEVICE;
  watchdog_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      status, static_cast<unsigned long long>(timeout_ns));
  return kta::launch_status();
}

const char* kta_status_string(int status) {
  switch (status) {
    case KTA_OK:
      return "ok";
    case KTA_ERR_INVALID_ARG:
      return "invalid argument";
    case KTA_ERR_UNSUPPORTED:
      return "unsupported shape or parameter";
    case KTA_ERR_ALIGN:
      return "pointer or stride not 16-byte aligned";
    case KTA_ERR_LAUNCH:
      return "kernel launch failed";
    case KTA_ERR_DEVICE_TIMEOUT:
      return "device-side bounded wait expired";
    case KTA_ERR_NO_DEVICE:
      return "no sm_100 CUDA device";
    case KTA_ERR_WORKSPACE:
      return "workspace missing or too small";
    case KTA_ERR_CUDA:
      return "CUDA runtime or driver error";
    case KTA_ERR_DEVICE_BOUNDS:
      return "device-side bounds check failed";
    default:
      return "unknown status";
  }
}

int kta_device_status(uint32_t* words, int clear) {
  if (words == nullptr) return KTA_ERR_INVALID_ARG;
  unsigned int* p = kta::device_status_ptr();
  if (p == nullptr) return KTA_ERR_NO_DEVICE;
  if (cudaDeviceSynchronize() != cudaSuccess) return KTA_ERR_CUDA;
  if (cudaMemcpy(words, p, 4 * sizeof(unsigned int), cudaMemcpyDeviceToHost) != cudaSuccess) {
    return KTA_ERR_CUDA;
  }
  if (clear) {
    if (cudaMemset(p, 0, 4 * sizeof(unsigned int)) != cudaSuccess) return KTA_ERR_CUDA;
    if (cudaDeviceSynchronize() != cudaSuccess) return KTA_ERR_CUDA;
  }
  return KTA_OK;
}

int kta_sm_count(void) { return kta::current_sm_count(); }

int kta_last_error(void) { return t_last_error; }

}  // extern "C"
