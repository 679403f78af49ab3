// Lightning Indexer entry points (kernels added in the next step).
#include "common.cuh"
#include "host_util.h"

extern "C" int dsa_indexer_qproj_rope(const void*, const void*, const float*, const float*, void*,
                                      int64_t, int, int, int, int, int64_t, void*) {
  return DSA_ERR_UNSUPPORTED;
}
extern "C" int dsa_indexer_wproj(const void*, const void*, void*, int64_t, int, int, float, void*) {
  return DSA_ERR_UNSUPPORTED;
}
extern "C" int dsa_indexer_score_topk(const void*, const void*, const void*, int64_t, int64_t*,
                                      int64_t, int64_t, int, int, int64_t, int, int64_t, int,
                                      int64_t, void*) {
  return DSA_ERR_UNSUPPORTED;
}
extern "C" size_t dsa_indexer_workspace_bytes(int64_t batch, int64_t seqlen, int n_heads,
                                              int head_dim) {
  return 0;
}
extern "C" int dsa_indexer_fwd(const void*, const void*, const void*, const void*, const float*,
                               const float*, const void*, int64_t, int64_t*, void*, size_t, int64_t,
                               int64_t, int, int, int, int, int, int, int64_t, int, int64_t, float,
                               void*) {
  return DSA_ERR_UNSUPPORTED;
}
