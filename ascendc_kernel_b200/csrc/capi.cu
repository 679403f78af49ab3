// Status strings, the per-device error word, device-info cache and the TMA
// tensor-map encoder used by all entry points.
#include <mutex>

#include "common.cuh"
#include "host_util.h"

namespace dsa {

// Per-device error word. Kernels receive its device address (see
// device_error_word) and OR DSA_DEVERR_* codes into it.
__device__ unsigned int g_dsa_device_error = 0;

int device_error_word(unsigned int** ptr) {
  static std::mutex mu;
  static unsigned int* cache[64] = {nullptr};
  int dev = 0;
  int st = cuda_status(cudaGetDevice(&dev));
  if (st != DSA_OK) return st;
  if (dev < 0 || dev >= 64) return DSA_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    st = cuda_status(cudaGetSymbolAddress(&p, g_dsa_device_error));
    if (st != DSA_OK) return st;
    cache[dev] = static_cast<unsigned int*>(p);
  }
  *ptr = cache[dev];
  return DSA_OK;
}

static thread_local int t_last_cuda_error = 0;

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return DSA_OK;
  t_last_cuda_error = static_cast<int>(e);
  return DSA_ERR_CUDA;
}

int current_device_info(DeviceInfo* info) {
  static std::mutex mu;
  static DeviceInfo cache[64];
  int dev = 0;
  int st = cuda_status(cudaGetDevice(&dev));
  if (st != DSA_OK) return st;
  if (dev < 0 || dev >= 64) return DSA_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev].device != dev) {
    DeviceInfo d;
    d.device = dev;
    st = cuda_status(cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev));
    if (st != DSA_OK) return st;
    st = cuda_status(
        cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    if (st != DSA_OK) return st;
    st = cuda_status(cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev));
    if (st != DSA_OK) return st;
    st = cuda_status(cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev));
    if (st != DSA_OK) return st;
    cache[dev] = d;
  }
  *info = cache[dev];
  if (info->major != 10) return DSA_ERR_NO_DEVICE;
  return DSA_OK;
}

typedef CUresult (*PFN_EncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_EncodeTiled get_encode_fn() {
  static PFN_EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_EncodeTiled>(p);
    }
  });
  return fn;
}

int encode_tensor_map(CUtensorMap* tm, CUtensorMapDataType dtype, int rank, const void* base,
                      const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                      CUtensorMapSwizzle swizzle) {
  PFN_EncodeTiled fn = get_encode_fn();
  if (fn == nullptr) return DSA_ERR_CUDA;
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  CUresult r = fn(tm, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, s, b, e,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    t_last_cuda_error = static_cast<int>(r);
    return DSA_ERR_MISALIGNED;
  }
  return DSA_OK;
}

}  // namespace dsa

extern "C" {

const char* dsa_status_string(int status) {
  switch (status) {
    case DSA_OK: return "DSA_OK";
    case DSA_ERR_INVALID_ARGUMENT: return "DSA_ERR_INVALID_ARGUMENT";
    case DSA_ERR_UNSUPPORTED: return "DSA_ERR_UNSUPPORTED";
    case DSA_ERR_MISALIGNED: return "DSA_ERR_MISALIGNED";
    case DSA_ERR_CUDA: return "DSA_ERR_CUDA";
    case DSA_ERR_WORKSPACE: return "DSA_ERR_WORKSPACE";
    case DSA_ERR_NO_DEVICE: return "DSA_ERR_NO_DEVICE";
    default: return "DSA_ERR_UNKNOWN";
  }
}

int dsa_last_cuda_error(void) { return dsa::t_last_cuda_error; }

int dsa_device_error_read(int device, unsigned int* code_out, int clear) {
  if (code_out == nullptr) return DSA_ERR_INVALID_ARGUMENT;
  int prev = 0;
  int st = dsa::cuda_status(cudaGetDevice(&prev));
  if (st != DSA_OK) return st;
  st = dsa::cuda_status(cudaSetDevice(device));
  if (st != DSA_OK) return st;
  st = dsa::cuda_status(cudaDeviceSynchronize());
  if (st == DSA_OK) {
    unsigned int v = 0;
    st = dsa::cuda_status(cudaMemcpyFromSymbol(&v, dsa::g_dsa_device_error, sizeof(v)));
    if (st == DSA_OK) {
      *code_out = v;
      if (clear) {
        const unsigned int zero = 0;
        st = dsa::cuda_status(cudaMemcpyToSymbol(dsa::g_dsa_device_error, &zero, sizeof(zero)));
      }
    }
  }
  cudaSetDevice(prev);
  return st;
}

int dsa_version(void) { return 100; }

}  // extern "C"
