// Index score backward for the tensor-core forward's winner state.
//
// The gradient of a block maximum goes to the block's winning key (ties share
// it equally, torch.amax; triton/index_score.py:139-232):
//   dIQ[t][g] = scale * sum_b ds[t][g][b] * (mean of the winners' index_k rows)
//   dIK[j]    = scale * sum over (t, g, b) that j wins of ds[t][g][b] * index_q[t][g] / ties
// tie_info (from msa_index_score_fwd_tc_state) holds the winner offset + 1 or
// -(number of tied keys), whose float64 maximum is in max_val; tied keys are
// found again by recomputing the float64 scores (same dot order as the fixup).
//
// dIQ: one warp per (token, group) row walks the row's causal blocks.
// dIK: the winner table is transposed without atomics. A CTA takes one key
// block and one chunk of CT query tokens, loads the chunk's (tie_info, ds)
// pairs into shared memory, and warp w sums the contributions to keys
// 8w .. 8w + 7 of the block in (token, group) order; a second kernel adds the
// chunks' partial sums in chunk order. Everything accumulates in float64 and is
// rounded once (float64 -> float32 -> dtype), as the precise kernels do.
#include "attn_common.cuh"

namespace msa {
namespace {

using attn::block_sequence;

constexpr int kBwdKWarps = 16;
constexpr int kChunkEntries = 8192;  // (token, group) pairs per dIK chunk (at least 128 tokens)
constexpr int kBatch = 8;            // dIQ: winners whose key rows are loaded together
template <int kPer>
constexpr int kBatchK = kPer == 2 ? 16 : 8;  // dIK: entries whose query rows are loaded together
constexpr int kLoadBatch = 8;        // dIK: (tie_info, ds) entries in flight per thread while loading a chunk

inline int chunk_tokens(int groups) { return std::max(128, kChunkEntries / groups); }

// The kPer consecutive 16-bit elements at element i (a multiple of kPer, so the
// vector load is aligned) as float: one 4- or 8-byte load per lane, a whole
// 64- or 128-element row per warp in one request. bf16 -> float is a shift, so
// the only conversion left per element is the one float -> double of the sum.
template <int kPer>
__device__ __forceinline__ void load_run_f32(const void* p, int64_t i, int dtype, float (&out)[kPer]) {
  static_assert(kPer == 2 || kPer == 4, "64 or 128 elements per row");
  const uint16_t* src = static_cast<const uint16_t*>(p) + i;
  uint32_t w[kPer / 2];
  if constexpr (kPer == 2) {
    w[0] = *reinterpret_cast<const uint32_t*>(src);
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(src);
    w[0] = u.x;
    w[1] = u.y;
  }
#pragma unroll
  for (int h = 0; h < kPer / 2; ++h) {
    if (dtype == MSA_BF16) {
      out[2 * h] = __uint_as_float(w[h] << 16);
      out[2 * h + 1] = __uint_as_float(w[h] & 0xffff0000u);
    } else {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[h]));
      out[2 * h] = f.x;
      out[2 * h + 1] = f.y;
    }
  }
}

// float64 scores scale * q . k_j of the 4 keys o = lane + 32 i of block start_b
// (keys past t are not candidates) equal to m: bit i set.
__device__ __forceinline__ unsigned tied_keys(const double* q, const void* ik, int dtype, int dim, int64_t start_b,
                                              int64_t t, double scale, double m, int lane) {
  unsigned bits = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t j = start_b + lane + 32 * i;
    if (j <= t && __dmul_rn(scale, dot_f64(q, ik, j * dim, dtype, dim)) == m) bits |= 1u << i;
  }
  return bits;
}

template <int kPer>  // head dims per lane: Di / 32
__global__ void score_bwd_q_tc_kernel(const void* __restrict__ iq, const void* __restrict__ ik, int dtype,
                                      const int32_t* __restrict__ cu, int nseq, int64_t rows, int groups, int dim,
                                      int nb, double scale, const int32_t* __restrict__ tie_info,
                                      const double* __restrict__ max_val, const float* __restrict__ ds,
                                      void* __restrict__ dq) {
  extern __shared__ double qsm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  double* q = qsm + (size_t)warp * dim;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < rows; row += warps) {
    const int64_t t = row / groups;
    const int64_t start = cu[find_sequence(cu, nseq, t)];
    const int qb = (int)((t - start) >> 7);
    double acc[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) acc[i] = 0.0;
    bool q_loaded = false;
    // (tie_info, ds) of the row's next 32 blocks are loaded while this chunk's gathers run
    auto chunk_info = [&](int b0, int& info, float& w) {
      const int b = b0 + lane;
      const bool in = b <= qb && b < nb;
      info = in ? tie_info[row * nb + b] : 0;
      w = in ? ds[row * nb + b] : 0.f;
    };
    int info_next;
    float w_next;
    chunk_info(0, info_next, w_next);
    for (int b0 = 0; b0 <= qb && b0 < nb; b0 += 32) {
      const int info = info_next;
      const float w = w_next;
      chunk_info(b0 + 32, info_next, w_next);
      // unique winners, eight at a time so their key-row loads are in flight together
      unsigned mask = __ballot_sync(0xffffffffu, info > 0 && w != 0.f);
      while (mask) {
        float kv[kBatch][kPer];
        double wv[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const int src = mask ? __ffs(mask) - 1 : 0;
          const bool on = mask != 0u;
          mask &= mask - 1;
          const int bi = __shfl_sync(0xffffffffu, info, src);
          wv[u] = on ? __dmul_rn((double)__shfl_sync(0xffffffffu, w, src), scale) : 0.0;
          const int64_t j = start + (int64_t)(b0 + src) * 128 + (on ? bi - 1 : 0);
          load_run_f32<kPer>(ik, j * dim + lane * kPer, dtype, kv[u]);
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u)
#pragma unroll
          for (int i = 0; i < kPer; ++i) acc[i] += wv[u] * (double)kv[u][i];
      }
      // ties
      mask = __ballot_sync(0xffffffffu, info < 0 && w != 0.f);
      while (mask) {
        const int src = __ffs(mask) - 1;
        mask &= mask - 1;
        const int bi = __shfl_sync(0xffffffffu, info, src);
        const double wi = __dmul_rn((double)__shfl_sync(0xffffffffu, w, src), scale);
        const int64_t start_b = start + (int64_t)(b0 + src) * 128;
        {
          if (!q_loaded) {
            for (int d = lane; d < dim; d += 32) q[d] = load_f64(iq, row * dim + d, dtype);
            __syncwarp();
            q_loaded = true;
          }
          const double m = max_val[row * nb + b0 + src];
          const double wt = wi / (double)(-bi);
          const unsigned mine = tied_keys(q, ik, dtype, dim, start_b, t, scale, m, lane);
          for (int i = 0; i < 4; ++i) {
            unsigned wm = __ballot_sync(0xffffffffu, (mine >> i) & 1u);
            while (wm) {
              const int l = __ffs(wm) - 1;
              wm &= wm - 1;
              const int64_t j = start_b + l + 32 * i;
#pragma unroll
              for (int e = 0; e < kPer; ++e) acc[e] += wt * load_f64(ik, j * dim + lane * kPer + e, dtype);
            }
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) store_from_f64(dq, row * dim + lane * kPer + i, dtype, acc[i]);
  }
}

// One CTA per (global key block gb, query chunk c): float64 partial sums of the
// block's 128 keys x dim into part[(gb * n_chunks + c)]. Chunks before the block
// or past the sequence have no entries and write nothing (the reduction skips them).
// The chunk's unique-winner entries are first sorted by winning key offset with
// a stable counting sort (warp w ranks its 1/16 of the entries with match.any),
// so warp w then walks the contiguous runs of its offsets 8w .. 8w + 7 in entry
// order, eight query-row gathers in flight at a time.
template <int kPer>
__global__ void __launch_bounds__(kBwdKWarps * 32, 1)
score_bwd_k_part_kernel(const void* __restrict__ iq, const void* __restrict__ ik, int dtype,
                        const int32_t* __restrict__ cu, const int32_t* __restrict__ cbl, int nseq, int groups,
                        int dim, int nb, int ct, int n_chunks, double scale, const int32_t* __restrict__ tie_info,
                        const double* __restrict__ max_val, const float* __restrict__ ds,
                        double* __restrict__ part) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int gb = blockIdx.x / n_chunks, c = blockIdx.x - gb * n_chunks;
  if (gb >= cbl[nseq]) return;
  const int s = block_sequence(cbl, nseq, gb);
  const int64_t start = cu[s], len = cu[s + 1] - start;
  const int b = gb - cbl[s];
  const int64_t t_lo = start + max((int64_t)c * ct, (int64_t)b * 128), t_hi = start + min((int64_t)(c + 1) * ct, len);
  if (t_lo >= t_hi) return;
  const int n = (int)((t_hi - t_lo) * groups);
  constexpr int kMaxEntries = 2 * kChunkEntries;
  int2* ent = reinterpret_cast<int2*>(sm);                              // (tie_info, ds bits) per entry
  int32_t* order = reinterpret_cast<int32_t*>(ent + kMaxEntries);      // entries sorted by winning offset
  int32_t* cnt = order + kMaxEntries;                                  // [warp][offset] counts, then cursors
  int32_t* run = cnt + kBwdKWarps * 128;                               // [offset] run start, [128 + offset] length
  double* qbuf = reinterpret_cast<double*>(run + 256);
  __shared__ int any_tie;
  if (threadIdx.x == 0) any_tie = 0;
  __syncthreads();
  // the chunk's entries sit nb words apart: kLoadBatch of each thread's loads in flight at once
  bool tie = false;
  for (int e0 = threadIdx.x; e0 < n; e0 += kLoadBatch * blockDim.x) {
    int2 v[kLoadBatch];
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int e = e0 + u * blockDim.x;
      const int64_t idx = ((t_lo * groups) + min(e, n - 1)) * nb + b;  // row (t_lo + e / G, e % G) of block b
      v[u] = make_int2(tie_info[idx], __float_as_int(ds[idx]));
    }
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int e = e0 + u * blockDim.x;
      if (e < n) {
        ent[e] = v[u];
        tie |= v[u].x < 0 && __int_as_float(v[u].y) != 0.f;
      }
    }
  }
  if (tie) any_tie = 1;  // benign race: every writer stores 1
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  for (int o = lane; o < 128; o += 32) cnt[warp * 128 + o] = 0;
  __syncthreads();
  // counting sort, pass 1: per-warp counts of each offset over the warp's segment
  const int seg = ((n + kBwdKWarps - 1) / kBwdKWarps + 31) & ~31;
  const int e_beg = warp * seg, e_end = min(n, e_beg + seg);
  auto key_of = [&](int e) -> int {
    if (e >= e_end) return -1 - lane;
    const int2 v = ent[e];
    return (v.x > 0 && __int_as_float(v.y) != 0.f) ? v.x - 1 : -1 - lane;
  };
  for (int e0 = e_beg; e0 < e_end; e0 += 32) {
    const int key = key_of(e0 + lane);
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    if (key >= 0 && (peers & lt) == 0) cnt[warp * 128 + key] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  // per offset: run lengths, and each warp's first position inside its offset's run
  if (threadIdx.x < 128) {
    const int o = threadIdx.x;
    int acc = 0;
    for (int w = 0; w < kBwdKWarps; ++w) {
      const int x = cnt[w * 128 + o];
      cnt[w * 128 + o] = acc;
      acc += x;
    }
    run[128 + o] = acc;
  }
  __syncthreads();
  if (warp == 0) {  // exclusive scan of the run lengths (4 offsets per lane)
    int v[4], sum = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[i] = run[128 + lane * 4 + i];
      sum += v[i];
    }
    int x = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    int base = x - sum;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      run[lane * 4 + i] = base;
      base += v[i];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kBwdKWarps * 128; i += blockDim.x) cnt[i] += run[i & 127];
  __syncthreads();
  // pass 2: stable scatter of the entry indices
  for (int e0 = e_beg; e0 < e_end; e0 += 32) {
    const int key = key_of(e0 + lane);
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    if (key >= 0) order[cnt[warp * 128 + key] + __popc(peers & lt)] = e0 + lane;
    __syncwarp();
    if (key >= 0 && (peers & lt) == 0) cnt[warp * 128 + key] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();

  double* q = qbuf + (size_t)warp * dim;
  const int64_t start_b = start + (int64_t)b * 128;
  double acc[8][kPer];
#pragma unroll
  for (int k = 0; k < 8; ++k)
#pragma unroll
    for (int i = 0; i < kPer; ++i) acc[k][i] = 0.0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int o = warp * 8 + k, r0 = run[o], r1 = r0 + run[128 + o];
    for (int r = r0; r < r1; r += kBatchK<kPer>) {
      float qv[kBatchK<kPer>][kPer];
      double wv[kBatchK<kPer>];
#pragma unroll
      for (int u = 0; u < kBatchK<kPer>; ++u) {
        const bool on = r + u < r1;
        const int e = order[on ? r + u : r0];
        wv[u] = on ? __dmul_rn((double)__int_as_float(ent[e].y), scale) : 0.0;
        const int64_t row = t_lo * groups + e;
        load_run_f32<kPer>(iq, row * dim + lane * kPer, dtype, qv[u]);
      }
#pragma unroll
      for (int u = 0; u < kBatchK<kPer>; ++u)
#pragma unroll
        for (int i = 0; i < kPer; ++i) acc[k][i] += wv[u] * (double)qv[u][i];
    }
  }
  // ties (when the chunk has any): every warp checks its own 8 keys
  for (int e0 = 0; any_tie && e0 < n; e0 += 32) {
    const int e = e0 + lane;
    const int2 v = e < n ? ent[e] : make_int2(0, 0);
    unsigned mask = __ballot_sync(0xffffffffu, v.x < 0 && __int_as_float(v.y) != 0.f);
    while (mask) {
      const int src = __ffs(mask) - 1;
      mask &= mask - 1;
      const int info = __shfl_sync(0xffffffffu, v.x, src);
      const double w = __dmul_rn((double)__int_as_float(__shfl_sync(0xffffffffu, v.y, src)), scale);
      const int64_t row = t_lo * groups + e0 + src, t = row / groups;
      for (int d = lane; d < dim; d += 32) q[d] = load_f64(iq, row * dim + d, dtype);
      __syncwarp();
      const int64_t j = start_b + warp * 8 + (lane & 7);
      const bool win = lane < 8 && j <= t &&
                       __dmul_rn(scale, dot_f64(q, ik, j * dim, dtype, dim)) == max_val[row * nb + b];
      const unsigned wins = __ballot_sync(0xffffffffu, win);
      const double wt = w / (double)(-info);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        if ((wins >> kk) & 1u)
#pragma unroll
          for (int i = 0; i < kPer; ++i) acc[kk][i] += wt * q[lane * kPer + i];
      __syncwarp();
    }
  }
  double* out = part + ((int64_t)blockIdx.x * 128 + warp * 8) * dim;
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
#pragma unroll
    for (int i = 0; i < kPer; ++i) out[kk * dim + lane * kPer + i] = acc[kk][i];
}

// dIK[key][d] = sum over the key block's chunks (in chunk order) of the partial sums.
__global__ void score_bwd_k_reduce_kernel(const int32_t* __restrict__ cu, const int32_t* __restrict__ cbl, int nseq,
                                          int dim, int ct, int n_chunks, const double* __restrict__ part,
                                          int dtype, void* __restrict__ dk) {
  const int64_t total_blocks = cbl[nseq];
  const int64_t n = total_blocks * 128 * dim;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int d = (int)(idx % dim);
    const int64_t ko = idx / dim;
    const int gb = (int)(ko >> 7), o = (int)(ko & 127);
    const int s = block_sequence(cbl, nseq, gb);
    const int64_t start = cu[s], len = cu[s + 1] - start;
    const int b = gb - cbl[s];
    if ((int64_t)b * 128 + o >= len) continue;
    double acc = 0.0;
    const int c_lo = (int)(((int64_t)b * 128) / ct), c_hi = (int)((len + ct - 1) / ct);
    for (int c = c_lo; c < c_hi; ++c) acc += part[(((int64_t)gb * n_chunks + c) * 128 + o) * dim + d];
    store_from_f64(dk, (start + (int64_t)b * 128 + o) * dim + d, dtype, acc);
  }
}

struct ScoreBwdWorkspace {
  int32_t* cbl;
  double* part;
  size_t bytes;
};

ScoreBwdWorkspace carve_score_bwd(void* base, int64_t total_tokens, int32_t nseq, int32_t groups, int32_t dim,
                                  int32_t num_blocks) {
  ScoreBwdWorkspace w{};
  char* b = static_cast<char*>(base);
  const int64_t max_blocks = (total_tokens + 127) / 128 + nseq;
  const int ct = chunk_tokens(groups);
  const int64_t n_chunks = ((int64_t)num_blocks * 128 + ct - 1) / ct;
  w.cbl = reinterpret_cast<int32_t*>(b);
  size_t off = ((sizeof(int32_t) * (nseq + 1)) + 255) & ~size_t(255);
  w.part = reinterpret_cast<double*>(b + off);
  off += sizeof(double) * (size_t)max_blocks * n_chunks * 128 * dim;
  w.bytes = off;
  return w;
}

}  // namespace
}  // namespace msa

using namespace msa;

extern "C" size_t msa_index_score_bwd_tc_workspace_size(int64_t total_tokens, int32_t nseq, int32_t groups,
                                                        int32_t index_dim, int32_t num_blocks) {
  if (total_tokens < 0 || nseq < 1 || groups < 1 || index_dim < 1 || num_blocks < 1) return 0;
  return carve_score_bwd(nullptr, total_tokens, nseq, groups, index_dim, num_blocks).bytes;
}

extern "C" int msa_index_score_bwd_tc(const void* index_q, const void* index_k, int dtype, const int32_t* cu_seqlens,
                                      int32_t nseq, int64_t total_tokens, int32_t groups, int32_t index_dim,
                                      int32_t num_blocks, int32_t block_size, double scale, const double* max_val,
                                      const int32_t* tie_info, const float* dscores, void* dq, void* dk,
                                      void* workspace, size_t workspace_bytes, void* stream) {
  MSA_CHECK_ARG(dtype == MSA_BF16 || dtype == MSA_F16, "msa_index_score_bwd_tc: bf16/f16 only");
  MSA_CHECK_ARG(index_dim == 64 || index_dim == 128, "msa_index_score_bwd_tc: index_dim must be 64 or 128");
  MSA_CHECK_ARG((reinterpret_cast<uintptr_t>(index_q) | reinterpret_cast<uintptr_t>(index_k)) % 16 == 0,
                "msa_index_score_bwd_tc: index_q and index_k must be 16-byte aligned");
  MSA_CHECK_ARG(block_size == 128 && nseq >= 1 && num_blocks >= 1 && groups >= 1,
                "msa_index_score_bwd_tc: bad sizes");
  MSA_CHECK_ARG(total_tokens * groups * (int64_t)num_blocks < ((int64_t)1 << 40), "msa_index_score_bwd_tc: too large");
  if (total_tokens == 0 || (!dq && !dk)) return MSA_OK;
  const ScoreBwdWorkspace w = carve_score_bwd(workspace, total_tokens, nseq, groups, index_dim, num_blocks);
  MSA_CHECK_ARG(workspace && workspace_bytes >= w.bytes, "msa_index_score_bwd_tc: workspace too small");
  cudaStream_t st = as_stream(stream);
  int dev = 0, sms = 148;
  MSA_CUDA_RETURN(cudaGetDevice(&dev));
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t rows = total_tokens * groups;
  if (dq) {
    auto kq = index_dim == 64 ? score_bwd_q_tc_kernel<2> : score_bwd_q_tc_kernel<4>;
    kq<<<sms * 8, 256, 8 * index_dim * sizeof(double), st>>>(index_q, index_k, dtype, cu_seqlens, nseq, rows, groups,
                                                            index_dim, num_blocks, scale, tie_info, max_val, dscores,
                                                            dq);
    count_launches(1);
  }
  if (dk) {
    const int ct = chunk_tokens(groups);
    const int n_chunks = (int)(((int64_t)num_blocks * 128 + ct - 1) / ct);
    const int64_t max_blocks = (total_tokens + 127) / 128 + nseq;
    MSA_CHECK_ARG(max_blocks * n_chunks < ((int64_t)1 << 31), "msa_index_score_bwd_tc: too many chunks");
    if (int e = msa_block_prefix(cu_seqlens, nseq, block_size, w.cbl, stream)) return e;
    const size_t smem = (size_t)2 * kChunkEntries * (sizeof(int2) + sizeof(int32_t)) +
                        sizeof(int32_t) * (kBwdKWarps * 128 + 256) + (size_t)kBwdKWarps * index_dim * sizeof(double);
    auto kk = index_dim == 64 ? score_bwd_k_part_kernel<2> : score_bwd_k_part_kernel<4>;
    MSA_CUDA_RETURN(cudaFuncSetAttribute(kk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kk<<<(unsigned)(max_blocks * n_chunks), kBwdKWarps * 32, smem, st>>>(
        index_q, index_k, dtype, cu_seqlens, w.cbl, nseq, groups, index_dim, num_blocks, ct, n_chunks, scale,
        tie_info, max_val, dscores, w.part);
    score_bwd_k_reduce_kernel<<<sms * 8, 256, 0, st>>>(cu_seqlens, w.cbl, nseq, index_dim, ct, n_chunks, w.part,
                                                       dtype, dk);
    count_launches(2);
  }
  return launch_status("index_score_bwd_tc");
}
