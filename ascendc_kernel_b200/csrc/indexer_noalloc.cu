// Lightning Indexer entry point that allocates nothing.
//
// Some callers cannot hand this library a workspace: plug-ins whose host
// framework owns all device memory and forbids allocating inside an operator,
// and latency-critical paths where a cudaMalloc/cudaFree (which can
// synchronize the device) is not acceptable. For them the operand slices and
// the q and w intermediates of the indexer live in a fixed array compiled into this
// library, of kNoAllocScratchBytes per device; every device that loads the
// library keeps it until the process exits.
//
// The first call in a CUDA context (the device's primary context, or one the
// caller created and made current) looks up the device address of that array
// (cudaGetSymbolAddress) and caches it for that context; make that first call
// before any stream capture. All calls on a device share the array, so calls whose
// kernels overlap on the GPU (e.g. on two streams) race on it; every byte a
// call reads from the array is written earlier by the same call, so nothing
// has to be cleared between calls.
#include "common.cuh"
#include "host_util.h"

namespace dsa {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t{128} << 20;  // 128 MiB

static __device__ __align__(256) unsigned char g_indexer_scratch[kNoAllocScratchBytes];

// The array's device address in the calling thread's current context: looked
// up with cudaGetSymbolAddress the first time a context calls, then cached
// under the context's id (each context that loads the library has its own copy
// of the array at its own address).
int scratch_address(void** out) { return context_symbol_address(g_indexer_scratch, out); }

}  // namespace
}  // namespace dsa

extern "C" int dsa_indexer_fwd_noalloc(const void* x, const void* qr, const void* wq_b,
                                       const void* w_proj, const float* cos_tab,
                                       const float* sin_tab, const void* kv_cache,
                                       int64_t kv_batch_stride, int64_t* out, int64_t batch,
                                       int64_t seqlen, int dim, int q_lora_rank, int n_heads,
                                       int head_dim, int rope_dim, int index_topk,
                                       int64_t start_pos, int ratio, int64_t offset,
                                       float w_scale, void* stream) {
  if (batch < 0 || seqlen < 0 || ratio <= 0 || start_pos < 0) return DSA_ERR_INVALID_ARGUMENT;
  if (batch == 0 || seqlen == 0) return DSA_OK;
  const int64_t n_cand = (start_pos + seqlen) / ratio;
  const int topk = static_cast<int>(index_topk < n_cand ? index_topk : n_cand);
  const size_t need = dsa_indexer_workspace_bytes(batch, seqlen, n_heads, head_dim, n_cand, topk);
  if (need == 0) return DSA_ERR_INVALID_ARGUMENT;
  if (need > dsa::kNoAllocScratchBytes) return DSA_ERR_WORKSPACE;
  void* ws = nullptr;
  const int st = dsa::scratch_address(&ws);
  if (st != DSA_OK) return st;
  return dsa_indexer_fwd(x, qr, wq_b, w_proj, cos_tab, sin_tab, kv_cache, kv_batch_stride, out,
                         ws, dsa::kNoAllocScratchBytes, batch, seqlen, dim, q_lora_rank, n_heads,
                         head_dim, rope_dim, index_topk, start_pos, ratio, offset, w_scale,
                         stream);
}
