// Index score, tensor-core path (tcgen05 + TMA). Not built yet: the entry point
// reports MSA_ERR_UNSUPPORTED and the host dispatcher never selects it.
#include "common.cuh"

extern "C" int msa_index_score_fwd_tc(const void*, const void*, int, const int32_t*, int32_t, int64_t, int32_t,
                                      int32_t, int32_t, int32_t, float, float*, void*) {
  return msa::set_error(MSA_ERR_UNSUPPORTED, "msa_index_score_fwd_tc: tensor-core score kernel not built");
}
