// Host-side helpers shared by the entry points: CUDA error capture, device
// properties cache, and TMA tensor-map encoding through the driver entry point
// (so the library needs no link-time dependency on libcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "dsa_b200.h"

namespace dsa {

// Records `e` as this thread's last CUDA error and returns DSA_ERR_CUDA, or
// DSA_OK when e == cudaSuccess.
int cuda_status(cudaError_t e);

// Number of SMs and the max opt-in shared memory per block of the current device.
struct DeviceInfo {
  int device = -1;
  int num_sms = 0;
  int max_smem_optin = 0;
  int major = 0;
  int minor = 0;
};
int current_device_info(DeviceInfo* info);

// Encodes a tiled tensor map. dims/strides follow the driver API: dims[0] is
// the innermost extent; strides[i] (bytes) is the stride of dim i+1.
int encode_tensor_map(CUtensorMap* tm, CUtensorMapDataType dtype, int rank, const void* base,
                      const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                      CUtensorMapSwizzle swizzle);

// Device address of the error word in the calling thread's current context.
int device_error_word(unsigned int** ptr);

// Id of the calling thread's current CUDA context (cuCtxGetId), 0 when no
// context is current yet. A module-scope __device__ variable has its own
// address in every context, and a kernel attribute is set per context, so the
// caches below are keyed by this id, not by the device ordinal.
int current_context_id(unsigned long long* id);

// Device address of the module-scope __device__ variable whose host-side
// stand-in is `symbol`, in the current context (looked up once per context).
int context_symbol_address(const void* symbol, void** out);

// cudaFuncSetAttribute(func, attr, value), once per context, kernel and attribute.
int set_func_attribute_once(const void* func, cudaFuncAttribute attr, int value);
inline int set_max_dynamic_smem(const void* func, int bytes) {
  return set_func_attribute_once(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

// A stream and a fork / join event pair of the calling thread in its current
// context, created on first use and kept until the process exits (one set per
// host thread, so concurrent callers never share a side stream). Entry points
// use it to run two independent launch chains of one call concurrently: record
// `fork` on the caller's stream, make `stream` wait on it, launch one chain on
// `stream`, record `join` there and make the caller's stream wait on `join`.
// With may_create false (the caller's stream is being captured into a CUDA
// graph) a missing set is reported as DSA_ERR_UNSUPPORTED instead of created.
struct SideStream {
  cudaStream_t stream = nullptr;
  cudaEvent_t fork = nullptr;
  cudaEvent_t join = nullptr;
};
int thread_side_stream(SideStream* out, bool may_create);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace dsa
