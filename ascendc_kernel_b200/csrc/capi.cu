// Status strings, the per-device error word, device-info cache and the TMA
// tensor-map encoder used by all entry points.
#include <mutex>
#include <utility>
#include <vector>

#include "common.cuh"
#include "host_util.h"

namespace dsa {

// Error word of each context that loads this module. Kernels receive its
// device address (see device_error_word) and OR DSA_DEVERR_* codes into it.
__device__ unsigned int g_dsa_device_error = 0;

static thread_local int t_last_cuda_error = 0;

namespace {

typedef CUresult (*PFN_CtxGetCurrent)(CUcontext*);
typedef CUresult (*PFN_CtxGetId)(CUcontext, unsigned long long*);

struct CtxFns {
  PFN_CtxGetCurrent get_current = nullptr;
  PFN_CtxGetId get_id = nullptr;
};

const CtxFns& ctx_fns() {
  static CtxFns f;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      f.get_current = reinterpret_cast<PFN_CtxGetCurrent>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      f.get_id = reinterpret_cast<PFN_CtxGetId>(p);
  });
  return f;
}

// (context id, key, tag) -> value; a handful of entries per context. The key
// is a symbol (tag -1) or a kernel (tag = the attribute set on it).
struct CtxEntry {
  unsigned long long ctx;
  const void* key;
  int tag;
  void* value;
};
std::mutex g_ctx_mu;
std::vector<CtxEntry> g_ctx_cache;

bool ctx_lookup(unsigned long long ctx, const void* key, int tag, void** value) {
  std::lock_guard<std::mutex> lock(g_ctx_mu);
  for (const CtxEntry& e : g_ctx_cache)
    if (e.ctx == ctx && e.key == key && e.tag == tag) {
      *value = e.value;
      return true;
    }
  return false;
}

void ctx_store(unsigned long long ctx, const void* key, int tag, void* value) {
  std::lock_guard<std::mutex> lock(g_ctx_mu);
  for (const CtxEntry& e : g_ctx_cache)
    if (e.ctx == ctx && e.key == key && e.tag == tag) return;
  g_ctx_cache.push_back(CtxEntry{ctx, key, tag, value});
}

}  // namespace

int current_context_id(unsigned long long* id) {
  *id = 0;
  const CtxFns& f = ctx_fns();
  if (f.get_current == nullptr || f.get_id == nullptr) return DSA_ERR_CUDA;
  CUcontext c = nullptr;
  CUresult r = f.get_current(&c);
  if (r == CUDA_SUCCESS && c != nullptr) r = f.get_id(c, id);
  if (r != CUDA_SUCCESS) {
    t_last_cuda_error = static_cast<int>(r);
    return DSA_ERR_CUDA;
  }
  return DSA_OK;
}

int context_symbol_address(const void* symbol, void** out) {
  unsigned long long id = 0;
  int st = current_context_id(&id);
  if (st != DSA_OK) return st;
  if (id != 0 && ctx_lookup(id, symbol, -1, out)) return DSA_OK;
  void* p = nullptr;
  st = cuda_status(cudaGetSymbolAddress(&p, symbol));
  if (st != DSA_OK) return st;
  // with no context current before, the lookup has made the device's primary one current
  if (id == 0 && (st = current_context_id(&id)) != DSA_OK) return st;
  if (id != 0) ctx_store(id, symbol, -1, p);
  *out = p;
  return DSA_OK;
}

int set_func_attribute_once(const void* func, cudaFuncAttribute attr, int value) {
  unsigned long long id = 0;
  int st = current_context_id(&id);
  if (st != DSA_OK) return st;
  void* seen = nullptr;
  const int tag = static_cast<int>(attr);
  if (id != 0 && ctx_lookup(id, func, tag, &seen)) return DSA_OK;
  st = cuda_status(cudaFuncSetAttribute(func, attr, value));
  if (st != DSA_OK) return st;
  if (id == 0 && (st = current_context_id(&id)) != DSA_OK) return st;
  if (id != 0) ctx_store(id, func, tag, const_cast<void*>(func));
  return DSA_OK;
}

namespace {
thread_local std::vector<std::pair<unsigned long long, SideStream>> t_side_streams;
}  // namespace

int thread_side_stream(SideStream* out, bool may_create) {
  unsigned long long id = 0;
  int st = current_context_id(&id);
  if (st != DSA_OK) return st;
  if (id != 0)
    for (const auto& e : t_side_streams)
      if (e.first == id) {
        *out = e.second;
        return DSA_OK;
      }
  if (!may_create) return DSA_ERR_UNSUPPORTED;
  SideStream s;
  st = cuda_status(cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking));
  if (st == DSA_OK) st = cuda_status(cudaEventCreateWithFlags(&s.fork, cudaEventDisableTiming));
  if (st == DSA_OK) st = cuda_status(cudaEventCreateWithFlags(&s.join, cudaEventDisableTiming));
  if (st == DSA_OK && id == 0) st = current_context_id(&id);
  if (st != DSA_OK || id == 0) {
    if (s.join) cudaEventDestroy(s.join);
    if (s.fork) cudaEventDestroy(s.fork);
    if (s.stream) cudaStreamDestroy(s.stream);
    return st != DSA_OK ? st : DSA_ERR_CUDA;
  }
  t_side_streams.emplace_back(id, s);
  *out = s;
  return DSA_OK;
}

int device_error_word(unsigned int** ptr) {
  void* p = nullptr;
  const int st = context_symbol_address(&g_dsa_device_error, &p);
  if (st == DSA_OK) *ptr = static_cast<unsigned int*>(p);
  return st;
}

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
  // the current context stays (it may be one the caller created) when it is on `device`
  if (device != prev && (st = dsa::cuda_status(cudaSetDevice(device))) != DSA_OK) return st;
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
  if (device != prev) cudaSetDevice(prev);
  return st;
}

int dsa_version(void) { return 100; }

}  // extern "C"
