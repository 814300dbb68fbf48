// Sparse attention, precise path: float64 arithmetic with a single rounding of
// each public output. Used for shapes off the tensor-core path (any head dim,
// block size, dtype) and as the reference-accuracy implementation.
//
//   forward  : triton/sparse_attention.py:35-84 (per (token, head) online
//              softmax over the selected blocks; empty rows -> 0 / -inf)
//   backward : query-owned dQ + softmax centre (:87-198, without atomics) and
//              key-owned dK/dV walking the k2q CSR (:223-295), fixed order.
//   private  : query-owned dK/dV with atomics (:398-426), regression only.
//
// Keys are visited block by block in slot order, 32 at a time: one warp-wide
// float64 dot per key (lanes own head dimensions), then one exponential per
// lane for the whole chunk. A block id repeated in a row counts once, which is
// the float64 oracle's semantics (tests/reference_fp64.py:74).
#include <algorithm>

#include "common.cuh"

namespace msa {
namespace {

constexpr int kWarps = 4;
constexpr int kMaxPerLane = 8;  // head_dim <= 256

struct RowGeom {
  int64_t t, start, qb;
  int h, g;
};

__device__ __forceinline__ RowGeom row_geom(const int32_t* cu, int nseq, int64_t row, int hq, int ratio, int block) {
  RowGeom r;
  r.t = row / hq;
  r.h = (int)(row % hq);
  r.g = r.h / ratio;
  const int s = find_sequence(cu, nseq, r.t);
  r.start = cu[s];
  r.qb = (r.t - r.start) / block;
  return r;
}

// True if block b at `slot` is a valid, first occurrence in the row.
__device__ __forceinline__ bool first_valid_block(const int32_t* __restrict__ ids, int slot, int b, int64_t qb) {
  if (b < 0 || b > qb) return false;
  for (int s = 0; s < slot; ++s)
    if (__ldg(ids + s) == b) return false;
  return true;
}

__device__ __forceinline__ void load_row(double* acc, const void* p, int64_t off, int dtype, int dim, int lane) {
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int d = lane + 32 * i;
    acc[i] = d < dim ? load_f64(p, off + d, dtype) : 0.0;
  }
}

// The one dot product of every attention kernel: explicit fused multiply-adds in
// a fixed order, then a fixed butterfly, so forward and backward recompute
// bit-identical logits. Logit scaling and the subtraction of the row maximum /
// LSE are also explicit (__dmul_rn / __dsub_rn): a contracted fma(scale, dot,
// -lse) would leave a residual where the forward saw exactly zero. With this a
// key seen by a single query gets P == 1 exactly, and outputs that land on a
// bf16 rounding midpoint round like the float64 oracle.
__device__ __forceinline__ double warp_dot(const double* a, const void* p, int64_t off, int dtype, int dim, int lane) {
  double s = 0.0;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int d = lane + 32 * i;
    if (d < dim) s = __fma_rn(a[i], load_f64(p, off + d, dtype), s);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s = __dadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
  return s;
}

// One (token, head) row of the precise forward, executed by one warp.
__device__ void precise_fwd_row(const void* __restrict__ q, const void* __restrict__ k, const void* __restrict__ v,
                                int dtype, const int32_t* __restrict__ ids, const int32_t* __restrict__ cu, int nseq,
                                int64_t row, int hq, int groups, int dim, int topk, int block, double scale,
                                void* __restrict__ out, float* __restrict__ lse, double* __restrict__ lse64) {
  const int lane = threadIdx.x & 31;
  const RowGeom r = row_geom(cu, nseq, row, hq, hq / groups, block);
  double qv[kMaxPerLane], acc[kMaxPerLane];
  load_row(qv, q, row * dim, dtype, dim, lane);
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) acc[i] = 0.0;
  double m = -INFINITY, l = 0.0;
  const int32_t* my_ids = ids + (r.t * groups + r.g) * (int64_t)topk;
  for (int slot = 0; slot < topk; ++slot) {
    const int b = __ldg(my_ids + slot);
    if (!first_valid_block(my_ids, slot, b, r.qb)) continue;
    const int64_t k0 = r.start + (int64_t)b * block;
    const int64_t k1 = min(k0 + block, r.t + 1);
    for (int64_t c0 = k0; c0 < k1; c0 += 32) {
      const int n = (int)(k1 - c0 < 32 ? k1 - c0 : 32);
      double s_mine = -INFINITY;
      for (int i = 0; i < n; ++i) {
        const double s = __dmul_rn(scale, warp_dot(qv, k, ((c0 + i) * groups + r.g) * dim, dtype, dim, lane));
        if (lane == i) s_mine = s;
      }
      const double m_new = fmax(m, warp_max(s_mine));
      const double alpha = (m == -INFINITY) ? 0.0 : exp(__dsub_rn(m, m_new));
      const double p_mine = (lane < n) ? exp(__dsub_rn(s_mine, m_new)) : 0.0;
      l = l * alpha + warp_sum(p_mine);
#pragma unroll
      for (int d = 0; d < kMaxPerLane; ++d) acc[d] *= alpha;
      for (int i = 0; i < n; ++i) {
        const double p = __shfl_sync(0xffffffffu, p_mine, i);
        const int64_t voff = ((c0 + i) * groups + r.g) * dim;
#pragma unroll
        for (int d = 0; d < kMaxPerLane; ++d) {
          const int dd = lane + 32 * d;
          if (dd < dim) acc[d] += p * load_f64(v, voff + dd, dtype);
        }
      }
      m = m_new;
    }
  }
  const double inv = l > 0.0 ? 1.0 / l : 0.0;
#pragma unroll
  for (int d = 0; d < kMaxPerLane; ++d) {
    const int dd = lane + 32 * d;
    if (dd < dim) store_from_f64(out, row * dim + dd, dtype, acc[d] * inv);
  }
  if (lane == 0) {
    const double ls = l > 0.0 ? __dadd_rn(m, log(l)) : -INFINITY;
    lse[row] = __double2float_rn(ls);
    if (lse64) lse64[row] = ls;
  }
}

__global__ void __launch_bounds__(kWarps * 32)
attn_fwd_precise_kernel(const void* __restrict__ q, const void* __restrict__ k, const void* __restrict__ v, int dtype,
                        const int32_t* __restrict__ ids, const int32_t* __restrict__ cu, int nseq, int64_t rows,
                        int hq, int groups, int dim, int topk, int block, double scale, void* __restrict__ out,
                        float* __restrict__ lse, double* __restrict__ lse64) {
  const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  precise_fwd_row(q, k, v, dtype, ids, cu, nseq, row, hq, groups, dim, topk, block, scale, out, lse, lse64);
}

// Recompute listed rows with the precise forward (rows the tensor-core path
// cannot bound safely). list[0] = count, list[1..] = row ids.
__global__ void __launch_bounds__(kWarps * 32)
attn_fwd_fixup_kernel(const void* __restrict__ q, const void* __restrict__ k, const void* __restrict__ v, int dtype,
                      const int32_t* __restrict__ ids, const int32_t* __restrict__ cu, int nseq, int hq, int groups,
                      int dim, int topk, int block, double scale, const int32_t* __restrict__ list,
                      void* __restrict__ out, float* __restrict__ lse) {
  const int n = list[0];
  for (int64_t i = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); i < n; i += (int64_t)gridDim.x * kWarps)
    precise_fwd_row(q, k, v, dtype, ids, cu, nseq, list[1 + i], hq, groups, dim, topk, block, scale, out, lse,
                    nullptr);
}

// Query-owned backward. With P_j = exp(s_j - lse) and dP_j = dO . v_j:
//   delta = sum_j P_j dP_j,  dQ = scale * (sum_j P_j dP_j k_j - delta * sum_j P_j k_j).
// In atomic mode the same pass also adds dK_j += scale * P_j (dP_j - delta) q and
// dV_j += P_j dO into float64 accumulators, which needs delta first: the pass
// runs twice (the first only accumulates delta).
template <bool kAtomic>
__global__ void __launch_bounds__(kWarps * 32)
attn_bwd_q_precise_kernel(const void* __restrict__ q, const void* __restrict__ k, const void* __restrict__ v,
                          const void* __restrict__ dout, int dtype, const int32_t* __restrict__ ids,
                          const int32_t* __restrict__ cu, int nseq, int64_t rows, int hq, int groups, int dim,
                          int topk, int block, double scale, const double* __restrict__ lse64,
                          void* __restrict__ dq, double* __restrict__ delta_out, double* __restrict__ dk_acc,
                          double* __restrict__ dv_acc) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const RowGeom r = row_geom(cu, nseq, row, hq, hq / groups, block);
  double qv[kMaxPerLane], go[kMaxPerLane], a[kMaxPerLane], bsum[kMaxPerLane];
  load_row(qv, q, row * dim, dtype, dim, lane);
  load_row(go, dout, row * dim, dtype, dim, lane);
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) a[i] = bsum[i] = 0.0;
  const double ls = lse64[row];
  double delta = 0.0;
  const int32_t* my_ids = ids + (r.t * groups + r.g) * (int64_t)topk;
  const int passes = kAtomic ? 2 : 1;
  if (ls != -INFINITY) {
    for (int pass = 0; pass < passes; ++pass) {
      const bool accumulate_kv = kAtomic && pass == 1;
      for (int slot = 0; slot < topk; ++slot) {
        const int b = __ldg(my_ids + slot);
        if (!first_valid_block(my_ids, slot, b, r.qb)) continue;
        const int64_t k0 = r.start + (int64_t)b * block;
        const int64_t k1 = min(k0 + block, r.t + 1);
        for (int64_t c0 = k0; c0 < k1; c0 += 32) {
          const int n = (int)(k1 - c0 < 32 ? k1 - c0 : 32);
          double p_mine = 0.0, dp_mine = 0.0;
          for (int i = 0; i < n; ++i) {
            const int64_t off = ((c0 + i) * groups + r.g) * dim;
            const double s = __dmul_rn(scale, warp_dot(qv, k, off, dtype, dim, lane));
            const double dp = warp_dot(go, v, off, dtype, dim, lane);
            if (lane == i) { p_mine = exp(__dsub_rn(s, ls)); dp_mine = dp; }
          }
          if (!accumulate_kv) {
            const double w_mine = p_mine * dp_mine;
            if (pass == 0) delta += warp_sum(w_mine);
            if (!kAtomic) {
              for (int i = 0; i < n; ++i) {
                const double p = __shfl_sync(0xffffffffu, p_mine, i);
                const double w = __shfl_sync(0xffffffffu, w_mine, i);
                const int64_t off = ((c0 + i) * groups + r.g) * dim;
#pragma unroll
                for (int d = 0; d < kMaxPerLane; ++d) {
                  const int dd = lane + 32 * d;
                  if (dd < dim) {
                    const double kk = load_f64(k, off + dd, dtype);
                    a[d] += w * kk;
                    bsum[d] += p * kk;
                  }
                }
              }
            }
          } else {
            for (int i = 0; i < n; ++i) {
              const double p = __shfl_sync(0xffffffffu, p_mine, i);
              const double ds = p * (__shfl_sync(0xffffffffu, dp_mine, i) - delta) * scale;
              const int64_t off = ((c0 + i) * groups + r.g) * dim;
#pragma unroll
              for (int d = 0; d < kMaxPerLane; ++d) {
                const int dd = lane + 32 * d;
                if (dd < dim) {
                  a[d] += ds * load_f64(k, off + dd, dtype);
                  if (dk_acc) atomicAdd(dk_acc + off + dd, ds * qv[d]);
                  if (dv_acc) atomicAdd(dv_acc + off + dd, p * go[d]);
                }
              }
            }
          }
        }
      }
    }
  }
  if (dq) {
#pragma unroll
    for (int d = 0; d < kMaxPerLane; ++d) {
      const int dd = lane + 32 * d;
      if (dd < dim) store_from_f64(dq, row * dim + dd, dtype, kAtomic ? a[d] : scale * (a[d] - delta * bsum[d]));
    }
  }
  if (delta_out && lane == 0) delta_out[row] = delta;
}

// Key-owned dK/dV: one warp per (key token, group) walks the CSR row of its
// block; edges in (query, slot) order, heads of the group in order.
__global__ void __launch_bounds__(kWarps * 32)
attn_bwd_kv_precise_kernel(const void* __restrict__ q, const void* __restrict__ k, const void* __restrict__ v,
                           const void* __restrict__ dout, int dtype, const int32_t* __restrict__ ids,
                           const int32_t* __restrict__ cu, const int32_t* __restrict__ cu_block_lens,
                           const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ queries,
                           const int32_t* __restrict__ slots, int nseq, int64_t rows, int hq, int groups,
                           int dim, int topk, int block, double scale, const double* __restrict__ lse64,
                           const double* __restrict__ delta64, void* __restrict__ dk, void* __restrict__ dv) {
  const int lane = threadIdx.x & 31;
  const int64_t item = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (item >= rows) return;
  const int64_t j = item / groups;
  const int g = (int)(item % groups);
  const int s = find_sequence(cu, nseq, j);
  const int64_t start = cu[s];
  const int b = (int)((j - start) / block);
  const int64_t csr_row = ((int64_t)cu_block_lens[s] + b) * groups + g;
  const int ratio = hq / groups;
  double gk[kMaxPerLane], gv[kMaxPerLane];
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) gk[i] = gv[i] = 0.0;
  const int e1 = row_ptr[csr_row + 1];
  for (int e = row_ptr[csr_row]; e < e1; ++e) {
    const int64_t t = queries[e];
    if (t < j) continue;  // key j is in the query's future
    const int slot = slots[e];
    const int32_t* my_ids = ids + (t * groups + g) * (int64_t)topk;
    if (!first_valid_block(my_ids, slot, b, b)) continue;  // a repeated slot counts once
    for (int hh = 0; hh < ratio; ++hh) {
      const int64_t qrow = t * hq + (int64_t)g * ratio + hh;
      const double ls = lse64[qrow];
      if (ls == -INFINITY) continue;
      double qd[kMaxPerLane], god[kMaxPerLane];
      load_row(qd, q, qrow * dim, dtype, dim, lane);
      load_row(god, dout, qrow * dim, dtype, dim, lane);
      const double sdot = warp_dot(qd, k, item * dim, dtype, dim, lane);
      const double pdot = warp_dot(god, v, item * dim, dtype, dim, lane);
      const double p = exp(__dsub_rn(__dmul_rn(scale, sdot), ls));
      const double ds = p * (pdot - (delta64 ? delta64[qrow] : 0.0)) * scale;
#pragma unroll
      for (int d = 0; d < kMaxPerLane; ++d) { gk[d] += ds * qd[d]; gv[d] += p * god[d]; }
    }
  }
#pragma unroll
  for (int d = 0; d < kMaxPerLane; ++d) {
    const int dd = lane + 32 * d;
    if (dd < dim) {
      if (dk) store_from_f64(dk, item * dim + dd, dtype, gk[d]);
      if (dv) store_from_f64(dv, item * dim + dd, dtype, gv[d]);
    }
  }
}

__global__ void f64_to_dtype_kernel(const double* __restrict__ src, void* __restrict__ dst, int dtype, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    store_from_f64(dst, i, dtype, src[i]);
}

}  // namespace

// Launch the precise fixup of listed rows (used by the tensor-core forward).
int launch_fwd_fixup(const void* q, const void* k, const void* v, int dtype, const int32_t* ids, const int32_t* cu,
                     int nseq, int hq, int groups, int dim, int topk, int block, double scale, const int32_t* list,
                     void* out, float* lse, cudaStream_t st) {
  attn_fwd_fixup_kernel<<<148, kWarps * 32, 0, st>>>(q, k, v, dtype, ids, cu, nseq, hq, groups, dim, topk, block,
                                                     scale, list, out, lse);
  count_launches(1);
  return launch_status("attn_fwd_fixup");
}

namespace {

int check_common(const char* fn, int dtype, int32_t nseq, int32_t q_heads, int32_t groups, int32_t head_dim,
                 int32_t topk, int32_t block) {
  MSA_CHECK_ARG(valid_dtype(dtype), "%s: bad dtype %d", fn, dtype);
  MSA_CHECK_ARG(nseq >= 1 && groups >= 1 && q_heads >= groups && q_heads % groups == 0, "%s: bad head counts", fn);
  MSA_CHECK_ARG(head_dim >= 1 && head_dim <= 32 * kMaxPerLane, "%s: head_dim must be in [1, %d]", fn,
                32 * kMaxPerLane);
  MSA_CHECK_ARG(topk >= 0 && block >= 1, "%s: bad topk / block size", fn);
  return MSA_OK;
}

}  // namespace
}  // namespace msa

using namespace msa;

extern "C" int msa_attn_fwd(const void* q, const void* k, const void* v, int dtype, const int32_t* indices,
                            const int32_t* cu_seqlens, int32_t nseq, int64_t total_tokens, int32_t q_heads,
                            int32_t groups, int32_t head_dim, int32_t topk_blocks, int32_t block_size,
                            double scale, void* out, float* lse, double* lse64, void* stream) {
  if (int st = check_common("msa_attn_fwd", dtype, nseq, q_heads, groups, head_dim, topk_blocks, block_size)) return st;
  const int64_t rows = total_tokens * q_heads;
  if (rows == 0) return MSA_OK;
  attn_fwd_precise_kernel<<<ceil_div(rows, kWarps), kWarps * 32, 0, as_stream(stream)>>>(
      q, k, v, dtype, indices, cu_seqlens, nseq, rows, q_heads, groups, head_dim, topk_blocks, block_size, scale,
      out, lse, lse64); count_launches(1);
  return launch_status("attn_fwd_precise");
}

extern "C" int msa_attn_bwd_q(const void* q, const void* k, const void* v, const void* dout, int dtype,
                              const int32_t* indices, const int32_t* cu_seqlens, int32_t nseq, int64_t total_tokens,
                              int32_t q_heads, int32_t groups, int32_t head_dim, int32_t topk_blocks,
                              int32_t block_size, double scale, const double* lse64, void* dq, double* delta64,
                              void* stream) {
  if (int st = check_common("msa_attn_bwd_q", dtype, nseq, q_heads, groups, head_dim, topk_blocks, block_size)) return st;
  const int64_t rows = total_tokens * q_heads;
  if (rows == 0 || (!dq && !delta64)) return MSA_OK;
  attn_bwd_q_precise_kernel<false><<<ceil_div(rows, kWarps), kWarps * 32, 0, as_stream(stream)>>>(
      q, k, v, dout, dtype, indices, cu_seqlens, nseq, rows, q_heads, groups, head_dim, topk_blocks, block_size,
      scale, lse64, dq, delta64, nullptr, nullptr); count_launches(1);
  return launch_status("attn_bwd_q_precise");
}

extern "C" int msa_attn_bwd_kv(const void* q, const void* k, const void* v, const void* dout, int dtype,
                               const int32_t* indices, const int32_t* cu_seqlens, const int32_t* cu_block_lens,
                               const int32_t* row_ptr, const int32_t* query_indices, const int32_t* slot_indices,
                               int32_t nseq, int64_t total_tokens, int32_t q_heads, int32_t groups, int32_t head_dim,
                               int32_t topk_blocks, int32_t block_size, double scale, const double* lse64,
                               const double* delta64, void* dk, void* dv, void* stream) {
  if (int st = check_common("msa_attn_bwd_kv", dtype, nseq, q_heads, groups, head_dim, topk_blocks, block_size)) return st;
  MSA_CHECK_ARG(!dk || delta64, "msa_attn_bwd_kv: dK needs delta64");
  const int64_t rows = total_tokens * groups;
  if (rows == 0 || (!dk && !dv)) return MSA_OK;
  attn_bwd_kv_precise_kernel<<<ceil_div(rows, kWarps), kWarps * 32, 0, as_stream(stream)>>>(
      q, k, v, dout, dtype, indices, cu_seqlens, cu_block_lens, row_ptr, query_indices, slot_indices, nseq, rows,
      q_heads, groups, head_dim, topk_blocks, block_size, scale, lse64, delta64, dk, dv); count_launches(1);
  return launch_status("attn_bwd_kv_precise");
}

extern "C" int msa_attn_bwd_atomic(const void* q, const void* k, const void* v, const void* dout, int dtype,
                                   const int32_t* indices, const int32_t* cu_seqlens, int32_t nseq,
                                   int64_t total_tokens, int32_t q_heads, int32_t groups, int32_t head_dim,
                                   int32_t topk_blocks, int32_t block_size, double scale, const double* lse64,
                                   void* dq, double* dk_acc, double* dv_acc, void* dk, void* dv, void* stream) {
  if (int st = check_common("msa_attn_bwd_atomic", dtype, nseq, q_heads, groups, head_dim, topk_blocks, block_size))
    return st;
  MSA_CHECK_ARG((dk == nullptr) == (dk_acc == nullptr) && (dv == nullptr) == (dv_acc == nullptr),
                "msa_attn_bwd_atomic: each of dk/dv needs its float64 accumulator");
  cudaStream_t st = as_stream(stream);
  const int64_t kv_elems = total_tokens * groups * (int64_t)head_dim;
  if (dk_acc) MSA_CUDA_RETURN(cudaMemsetAsync(dk_acc, 0, sizeof(double) * kv_elems, st));
  if (dv_acc) MSA_CUDA_RETURN(cudaMemsetAsync(dv_acc, 0, sizeof(double) * kv_elems, st));
  const int64_t rows = total_tokens * q_heads;
  if (rows > 0) {
    attn_bwd_q_precise_kernel<true><<<ceil_div(rows, kWarps), kWarps * 32, 0, st>>>(
        q, k, v, dout, dtype, indices, cu_seqlens, nseq, rows, q_heads, groups, head_dim, topk_blocks, block_size,
        scale, lse64, dq, nullptr, dk_acc, dv_acc); count_launches(1);
    if (int s2 = launch_status("attn_bwd_atomic")) return s2;
  }
  if (kv_elems > 0) {
    const unsigned grid = (unsigned)std::min<int64_t>(4096, ceil_div(kv_elems, 256));
    if (dk) f64_to_dtype_kernel<<<grid, 256, 0, st>>>(dk_acc, dk, dtype, kv_elems); count_launches(1);
    if (dv) f64_to_dtype_kernel<<<grid, 256, 0, st>>>(dv_acc, dv, dtype, kv_elems); count_launches(1);
  }
  return launch_status("attn_bwd_atomic_convert");
}
