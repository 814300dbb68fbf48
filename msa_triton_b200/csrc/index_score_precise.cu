// Index score, precise path: float64 dot products and exact block-max winners.
//
// Forward follows triton/index_score.py:93-136 (per (token, group, block):
// causal dots then max; -inf for future blocks; optional winner state), the
// backward follows :139-232 (ties split equally as torch.amax does). Dots are
// computed in float64 from the exact input values, so winners and ties are
// those of the float64 oracle (tests/reference_fp64.py:16-45) rather than of a
// two-float32 compensated sum.
#include "common.cuh"

namespace msa {
namespace {

constexpr int kScoreThreads = 128;

// One CTA per (token, group) row; loops over the row's causal blocks.
__global__ void __launch_bounds__(kScoreThreads)
score_fwd_precise_kernel(const void* __restrict__ iq, const void* __restrict__ ik, int dtype,
                         const int32_t* __restrict__ cu, int nseq, int groups, int dim, int nb,
                         int block, double scale, float* __restrict__ scores,
                         double* __restrict__ max_val, int32_t* __restrict__ tie_info) {
  extern __shared__ double smem[];
  double* q = smem;  // [dim]
  __shared__ double red_best[kScoreThreads / 32];
  __shared__ int red_cnt[kScoreThreads / 32];
  __shared__ int red_first[kScoreThreads / 32];

  const int64_t row = blockIdx.x;
  const int64_t t = row / groups;
  const int g = (int)(row % groups);
  const int s = find_sequence(cu, nseq, t);
  const int64_t start = cu[s];
  const int64_t pos = t - start;
  const int64_t qb = pos / block;
  for (int d = threadIdx.x; d < dim; d += blockDim.x) q[d] = load_f64(iq, (t * groups + g) * dim + d, dtype);
  const int64_t out_base = row * nb;
  for (int64_t b = qb + 1 + threadIdx.x; b < nb; b += blockDim.x) {
    if (scores) scores[out_base + b] = -INFINITY;
    if (max_val) { max_val[out_base + b] = -INFINITY; tie_info[out_base + b] = 0; }
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t b = 0; b <= qb && b < nb; ++b) {
    double best = -INFINITY;
    int cnt = 0, first = INT32_MAX;
    for (int o = threadIdx.x; o < block; o += blockDim.x) {
      const int64_t j = start + b * block + o;
      if (j > t) break;
      const double v = __dmul_rn(scale, dot_f64(q, ik, j * dim, dtype, dim));
      if (v > best) { best = v; cnt = 1; first = o; }
      else if (v == best) { ++cnt; first = min(first, o); }
    }
    // warp then CTA reduction of (best, count of best, first offset of best)
    double wbest = warp_max(best);
    int wcnt = (best == wbest) ? cnt : 0;
    int wfirst = (best == wbest) ? first : INT32_MAX;
    wcnt = warp_sum(wcnt);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) wfirst = min(wfirst, __shfl_xor_sync(0xffffffffu, wfirst, o));
    if (lane == 0) { red_best[warp] = wbest; red_cnt[warp] = wcnt; red_first[warp] = wfirst; }
    __syncthreads();
    if (threadIdx.x == 0) {
      double m = red_best[0];
      for (int w = 1; w < kScoreThreads / 32; ++w) m = fmax(m, red_best[w]);
      int c = 0, f = INT32_MAX;
      for (int w = 0; w < kScoreThreads / 32; ++w)
        if (red_best[w] == m) { c += red_cnt[w]; f = min(f, red_first[w]); }
      if (scores) scores[out_base + b] = __double2float_rn(m);
      if (max_val) {
        max_val[out_base + b] = m;
        tie_info[out_base + b] = (c == 1) ? f + 1 : -c;
      }
    }
    __syncthreads();
  }
}

// dQ: one warp per (token, group); lanes own dimensions.
__global__ void score_bwd_q_precise_kernel(const void* __restrict__ iq, const void* __restrict__ ik, int dtype,
                                           const int32_t* __restrict__ cu, int nseq, int64_t rows, int groups,
                                           int dim, int nb, int block, double scale,
                                           const double* __restrict__ max_val,
                                           const int32_t* __restrict__ tie_info,
                                           const float* __restrict__ ds, void* __restrict__ dq) {
  extern __shared__ double smem[];
  const int warps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * warps + warp;
  if (row >= rows) return;
  double* q = smem + (size_t)warp * dim;
  const int64_t t = row / groups;
  const int g = (int)(row % groups);
  const int s = find_sequence(cu, nseq, t);
  const int64_t start = cu[s];
  const int64_t qb = (t - start) / block;
  for (int d = lane; d < dim; d += 32) q[d] = load_f64(iq, (t * groups + g) * dim + d, dtype);
  __syncwarp();
  constexpr int kMaxPerLane = 16;  // dim <= 512
  double acc[kMaxPerLane];
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) acc[i] = 0.0;
  for (int64_t b = 0; b <= qb && b < nb; ++b) {
    const int64_t idx = row * nb + b;
    const int info = tie_info[idx];
    const double w0 = __dmul_rn((double)ds[idx], scale);
    if (info > 0) {
      const int64_t j = start + b * block + info - 1;
#pragma unroll
      for (int i = 0; i < kMaxPerLane; ++i) {
        const int d = lane + 32 * i;
        if (d < dim) acc[i] += w0 * load_f64(ik, j * dim + d, dtype);
      }
    } else if (info < 0) {
      const double w = w0 / (double)(-info);
      const double m = max_val[idx];
      for (int o0 = 0; o0 < block; o0 += 32) {
        const int o = o0 + lane;
        const int64_t j = start + b * block + o;
        bool win = false;
        if (o < block && j <= t) win = __dmul_rn(scale, dot_f64(q, ik, j * dim, dtype, dim)) == m;
        unsigned mask = __ballot_sync(0xffffffffu, win);
        while (mask) {
          const int src = __ffs(mask) - 1;
          mask &= mask - 1;
          const int64_t jw = start + b * block + o0 + src;
#pragma unroll
          for (int i = 0; i < kMaxPerLane; ++i) {
            const int d = lane + 32 * i;
            if (d < dim) acc[i] += w * load_f64(ik, jw * dim + d, dtype);
          }
        }
        if (start + b * block + o0 + 32 > t) break;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int d = lane + 32 * i;
    if (d < dim) store_from_f64(dq, (t * groups + g) * dim + d, dtype, acc[i]);
  }
}

// dK: one warp per key token; sums over later queries of the sequence and all
// groups in a fixed order (query chunk, group, query).
__global__ void score_bwd_k_precise_kernel(const void* __restrict__ iq, const void* __restrict__ ik, int dtype,
                                           const int32_t* __restrict__ cu, int nseq, int64_t total, int groups,
                                           int dim, int nb, int block, double scale,
                                           const double* __restrict__ max_val,
                                           const int32_t* __restrict__ tie_info,
                                           const float* __restrict__ ds, void* __restrict__ dk) {
  extern __shared__ double smem[];
  const int warps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t j = (int64_t)blockIdx.x * warps + warp;
  if (j >= total) return;
  double* kv = smem + (size_t)warp * dim;
  const int s = find_sequence(cu, nseq, j);
  const int64_t start = cu[s], end = cu[s + 1];
  const int64_t bj = (j - start) / block;
  const int oj = (int)((j - start) % block);
  for (int d = lane; d < dim; d += 32) kv[d] = load_f64(ik, j * dim + d, dtype);
  __syncwarp();
  constexpr int kMaxPerLane = 16;
  double acc[kMaxPerLane];
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) acc[i] = 0.0;
  for (int64_t t0 = j; t0 < end; t0 += 32) {
    const int64_t t = t0 + lane;
    for (int g = 0; g < groups; ++g) {
      bool win = false;
      double w = 0.0;
      if (t < end) {
        const int64_t idx = (t * groups + g) * nb + bj;
        const int info = tie_info[idx];
        if (info > 0) {
          win = (oj == info - 1);
          w = __dmul_rn((double)ds[idx], scale);
        } else if (info < 0) {
          // same float64 value as the forward: dot(q_row, k_j) in the q-operand order
          double qrow_dot = 0.0;
          for (int d = 0; d < dim; ++d)
            qrow_dot = __dadd_rn(qrow_dot, __dmul_rn(load_f64(iq, (t * groups + g) * dim + d, dtype), kv[d]));
          win = __dmul_rn(scale, qrow_dot) == max_val[idx];
          w = __dmul_rn((double)ds[idx], scale) / (double)(-info);
        }
      }
      unsigned mask = __ballot_sync(0xffffffffu, win);
      while (mask) {
        const int src = __ffs(mask) - 1;
        mask &= mask - 1;
        const double ws = __shfl_sync(0xffffffffu, w, src);
        const int64_t tw = t0 + src;
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) {
          const int d = lane + 32 * i;
          if (d < dim) acc[i] += ws * load_f64(iq, (tw * groups + g) * dim + d, dtype);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int d = lane + 32 * i;
    if (d < dim) store_from_f64(dk, j * dim + d, dtype, acc[i]);
  }
}

}  // namespace
}  // namespace msa

using namespace msa;

extern "C" int msa_index_score_fwd(const void* index_q, const void* index_k, int dtype,
                                   const int32_t* cu_seqlens, int32_t nseq, int64_t total_tokens,
                                   int32_t groups, int32_t index_dim, int32_t num_blocks,
                                   int32_t block_size, double scale, float* scores, double* max_val,
                                   int32_t* tie_info, void* stream) {
  MSA_CHECK_ARG(valid_dtype(dtype), "msa_index_score_fwd: bad dtype %d", dtype);
  MSA_CHECK_ARG(nseq >= 1 && groups >= 1 && index_dim >= 1 && block_size >= 1 && num_blocks >= 1,
                "msa_index_score_fwd: bad sizes");
  MSA_CHECK_ARG(index_dim <= 4096, "msa_index_score_fwd: index_dim > 4096 unsupported");
  MSA_CHECK_ARG((max_val == nullptr) == (tie_info == nullptr), "msa_index_score_fwd: state pointers must be both set or both NULL");
  MSA_CHECK_ARG(scores || max_val, "msa_index_score_fwd: nothing to write");
  if (total_tokens == 0) return MSA_OK;
  const int64_t rows = total_tokens * groups;
  MSA_CHECK_ARG(rows <= 0x7fffffffLL, "msa_index_score_fwd: T*G exceeds grid capacity");
  score_fwd_precise_kernel<<<(unsigned)rows, kScoreThreads, sizeof(double) * index_dim, as_stream(stream)>>>(
      index_q, index_k, dtype, cu_seqlens, nseq, groups, index_dim, num_blocks, block_size, scale, scores,
      max_val, tie_info); count_launches(1);
  return launch_status("score_fwd_precise");
}

extern "C" int msa_index_score_bwd(const void* index_q, const void* index_k, int dtype,
                                   const int32_t* cu_seqlens, int32_t nseq, int64_t total_tokens,
                                   int32_t groups, int32_t index_dim, int32_t num_blocks,
                                   int32_t block_size, double scale, const double* max_val,
                                   const int32_t* tie_info, const float* dscores, void* d_index_q,
                                   void* d_index_k, void* stream) {
  MSA_CHECK_ARG(valid_dtype(dtype), "msa_index_score_bwd: bad dtype %d", dtype);
  MSA_CHECK_ARG(index_dim >= 1 && index_dim <= 512, "msa_index_score_bwd: index_dim must be in [1, 512]");
  MSA_CHECK_ARG(max_val && tie_info && dscores, "msa_index_score_bwd: missing state");
  if (total_tokens == 0) return MSA_OK;
  constexpr int kWarps = 4;
  const size_t smem = sizeof(double) * index_dim * kWarps;
  if (d_index_q) {
    const int64_t rows = total_tokens * groups;
    score_bwd_q_precise_kernel<<<ceil_div(rows, kWarps), kWarps * 32, smem, as_stream(stream)>>>(
        index_q, index_k, dtype, cu_seqlens, nseq, rows, groups, index_dim, num_blocks, block_size, scale,
        max_val, tie_info, dscores, d_index_q); count_launches(1);
    if (int st = launch_status("score_bwd_q_precise")) return st;
  }
  if (d_index_k) {
    score_bwd_k_precise_kernel<<<ceil_div(total_tokens, kWarps), kWarps * 32, smem, as_stream(stream)>>>(
        index_q, index_k, dtype, cu_seqlens, nseq, total_tokens, groups, index_dim, num_blocks, block_size,
        scale, max_val, tie_info, dscores, d_index_k); count_launches(1);
    if (int st = launch_status("score_bwd_k_precise")) return st;
  }
  return MSA_OK;
}
