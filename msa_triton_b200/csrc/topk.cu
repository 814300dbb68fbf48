// Top-k block selection: one warp per (token, group) row.
//
// Semantics of triton/topk.py:11-47 / eager/ops.py:94-129: future blocks rank
// -inf, the local_blocks most recent causal blocks rank +inf, the top
// min(K, NB) are kept in descending rank, -inf picks become -1, tail -1.
// Equal ranks are ordered by ascending block id (torch.topk leaves this open).
//
// Each candidate is a 64-bit key: order-preserving float bits of its rank in
// the high word and the complemented block id in the low word, so one unsigned
// max both ranks and breaks ties. Rows of up to 32 * kMaxPerLane blocks keep
// their keys in registers; each of the K rounds is a lane-local max plus a
// 5-step warp max, and the winning lane retires its key. No temporaries touch
// memory: the only traffic is reading the scores row and writing K ids.
#include "common.cuh"

namespace msa {
namespace {

__device__ __forceinline__ uint32_t ordered_bits(float x) {
  uint32_t u = __float_as_uint(x);
  if (u == 0x80000000u) u = 0u;  // -0.0 ties with +0.0
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr uint64_t kRetired = 0ull;  // below every live key (ordered(-inf) > 0)

template <int kPerLane>
__global__ void topk_kernel(const float* __restrict__ scores, const int32_t* __restrict__ cu, int nseq,
                            int64_t rows, int groups, int nb, int block, int k, int local,
                            int32_t* __restrict__ out) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int64_t t = row / groups;
  const int s = find_sequence(cu, nseq, t);
  const int64_t qb = (t - cu[s]) / block;
  const float* src = scores + row * nb;
  uint64_t key[kPerLane];
  const uint32_t neg_inf = ordered_bits(-INFINITY), pos_inf = ordered_bits(INFINITY);
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) {
    const int b = lane + 32 * i;
    key[i] = kRetired;
    if (b < nb) {
      uint32_t r;
      if (b > qb) r = neg_inf;
      else if (local > 0 && b > qb - local) r = pos_inf;
      else r = ordered_bits(__ldg(src + b));
      key[i] = ((uint64_t)r << 32) | (uint32_t)(~(uint32_t)b);
    }
  }
  const int count = min(k, nb);
  int32_t* dst = out + row * k;
  for (int r = 0; r < count; ++r) {
    uint64_t best = kRetired;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) best = key[i] > best ? key[i] : best;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    const uint32_t b = ~(uint32_t)(best & 0xffffffffu);
    const bool is_neg_inf = (uint32_t)(best >> 32) == neg_inf;
    if (lane == 0) dst[r] = is_neg_inf ? -1 : (int32_t)b;
    if (is_neg_inf) {  // everything left ranks -inf as well
      for (int rr = r + 1 + lane; rr < k; rr += 32) dst[rr] = -1;
      return;
    }
#pragma unroll
    for (int i = 0; i < kPerLane; ++i)
      if (key[i] == best) key[i] = kRetired;
  }
  for (int rr = count + lane; rr < k; rr += 32) dst[rr] = -1;
}

}  // namespace
}  // namespace msa

using namespace msa;

extern "C" int msa_topk(const float* scores, const int32_t* cu_seqlens, int32_t nseq, int64_t total_tokens,
                        int32_t groups, int32_t num_blocks, int32_t block_size, int32_t topk_blocks,
                        int32_t local_blocks, int32_t* indices, void* stream) {
  MSA_CHECK_ARG(nseq >= 1 && groups >= 1 && num_blocks >= 1 && block_size >= 1, "msa_topk: bad sizes");
  MSA_CHECK_ARG(topk_blocks >= 0 && local_blocks >= 0 && local_blocks <= topk_blocks, "msa_topk: bad K/local");
  MSA_CHECK_ARG(num_blocks <= 32 * 64, "msa_topk: more than 2048 blocks per row unsupported");
  const int64_t rows = total_tokens * groups;
  if (rows == 0 || topk_blocks == 0) return MSA_OK;
  constexpr int kWarps = 8;
  const unsigned grid = ceil_div(rows, kWarps);
  cudaStream_t st = as_stream(stream);
#define MSA_TOPK_LAUNCH(P)                                                                     \
  topk_kernel<P><<<grid, kWarps * 32, 0, st>>>(scores, cu_seqlens, nseq, rows, groups, num_blocks, \
                                               block_size, topk_blocks, local_blocks, indices)
  if (num_blocks <= 32) MSA_TOPK_LAUNCH(1);
  else if (num_blocks <= 64) MSA_TOPK_LAUNCH(2);
  else if (num_blocks <= 128) MSA_TOPK_LAUNCH(4);
  else if (num_blocks <= 256) MSA_TOPK_LAUNCH(8);
  else if (num_blocks <= 512) MSA_TOPK_LAUNCH(16);
  else if (num_blocks <= 1024) MSA_TOPK_LAUNCH(32);
  else MSA_TOPK_LAUNCH(64);
#undef MSA_TOPK_LAUNCH
  count_launches(1);
  return launch_status("topk");
}
