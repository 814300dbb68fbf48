// Index KL loss (indexer training, sparse stage). The reference specifies the
// loss but has no kernel for it (docs/msa_training_flow.md:92-138,
// docs/implementation_plan.md:66-69). On the selected causal tokens J(t, g) of
// each (query token, group):
//   student  p_s = softmax_J(index_scale * iq[t,g] . ik[j])
//   teacher  p_T = mean over the group's heads of softmax_J(scale * q[t,h] . k[j,g])
//   loss     = sum_{t,g} KL(p_T || p_s) / (T * G),  dL/ds_j = (p_s(j) - p_T(j)) / (T * G)
//
// Three steps:
//   1. teacher: p_T per (pair, selection slot, key) into pt[T*G][K][B]. The
//      tensor-core family runs the attention forward kernel in its teacher mode
//      (attention_tc.cu, S = Q K^T on tcgen05, P = exp(S - lse) with the main
//      attention's LSE, head mean in registers); the precise family computes it
//      here in float64 (kl_teacher_kernel).
//   2. student (kl_student_kernel, one warp per pair): the student logits, their
//      log-sum-exp, the pair's KL, dIQ directly, and g_j = index_scale * dL/ds_j
//      written over p_T in place (0 for keys past the query).
//   3. dIK (kl_dik_kernel): key-owned, walking the k2q CSR of every group in
//      fixed order (no atomics), dik[j] = sum over selecting pairs of g_j iq[t,g].
// The loss is summed per pair and reduced in a fixed order (deterministic).
#include <algorithm>
#include <cmath>
#include <mutex>

#include "common.cuh"
#include "tc_common.cuh"

namespace msa {
namespace {

// Slot j of a pair selects a block for the first time and causally (the
// attention's key set, tests/reference_fp64.py:74-75).
__device__ __forceinline__ bool first_valid_slot(const int32_t* __restrict__ ids, int j, int b, int cur) {
  if (b < 0 || b > cur) return false;
  for (int i = 0; i < j; ++i)
    if (ids[i] == b) return false;
  return true;
}

template <typename T>
__device__ __forceinline__ T load_as(const void* p, int64_t i, int dtype) {
  return (T)load_f64(p, i, dtype);
}

template <>
__device__ __forceinline__ float load_as<float>(const void* p, int64_t i, int dtype) {
  if (dtype == MSA_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dtype == MSA_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ float exp_t(float x) { return __expf(x); }
__device__ __forceinline__ double exp_t(double x) { return exp(x); }
__device__ __forceinline__ float log_t(float x) { return __logf(x); }
__device__ __forceinline__ double log_t(double x) { return log(x); }
__device__ __forceinline__ float max_t(float a, float b) { return fmaxf(a, b); }
__device__ __forceinline__ double max_t(double a, double b) { return fmax(a, b); }

constexpr int kMaxIndexDim = 256;  // index_dim <= 256: 8 dims per lane

// --------------------------------------------------------------------------- student
// Dot product of a shared-memory float row with index_k row `key` (16-byte loads
// for 16-bit inputs whose rows are whole 16-byte units).
template <typename T>
__device__ __forceinline__ T dot_key(const T* __restrict__ qs, const void* __restrict__ ik, int64_t key, int dim,
                                     int dtype) {
  T acc = T(0);
  if (dtype != MSA_F32 && (dim & 7) == 0) {
    const uint4* row = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(ik) + key * dim * 2);
    for (int d8 = 0; d8 < dim / 8; ++d8) {
      const uint4 u = row[d8];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = dtype == MSA_F16 ? __half22float2(*reinterpret_cast<const __half2*>(&w[e]))
                                          : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[e]));
        acc += qs[d8 * 8 + 2 * e] * (T)f.x;
        acc += qs[d8 * 8 + 2 * e + 1] * (T)f.y;
      }
    }
    return acc;
  }
  for (int d = 0; d < dim; ++d) acc += qs[d] * load_as<T>(ik, key * dim + d, dtype);
  return acc;
}

// One warp per (token, group) pair, 8 warps per CTA. Lanes take keys for the
// logits (the pair's iq row in shared memory); for dIQ each lane owns index
// dims lane, lane + 32, ... and each 32-key chunk's g_j are broadcast.
constexpr int kStudentWarps = 8;

template <typename T>
__global__ void __launch_bounds__(kStudentWarps * 32, 2)
kl_student_kernel(const void* __restrict__ iq, const void* __restrict__ ik, int dtype,
                  const int32_t* __restrict__ ids, const int32_t* __restrict__ cu, int nseq, int64_t pairs,
                  int groups, int index_dim, int topk, int block, T index_scale, T inv_n, int need_grad,
                  T* __restrict__ pt, double* __restrict__ loss_pair, T* __restrict__ diq) {
  __shared__ T sq[kStudentWarps][kMaxIndexDim];
  const int lane = threadIdx.x & 31;
  T* qs = sq[threadIdx.x >> 5];
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t p = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; p < pairs; p += warps) {
    const int64_t t = p / groups;
    const int s = find_sequence(cu, nseq, t);
    const int64_t seq0 = cu[s];
    const int pos = (int)(t - seq0), cur = pos / block;
    const int32_t* row_ids = ids + p * topk;
    __syncwarp();
    for (int d = lane; d < index_dim; d += 32) qs[d] = load_as<T>(iq, p * index_dim + d, dtype);
    __syncwarp();
    // pass 1: running maximum and sum of exp per lane, then combined across the warp
    T m = T(-INFINITY), l = T(0);
    for (int j = 0; j < topk; ++j) {
      const int b = row_ids[j];
      if (!first_valid_slot(row_ids, j, b, cur)) continue;
      const int nk = b < cur ? block : pos - b * block + 1;
      for (int c = lane; c < nk; c += 32) {
        const T x = dot_key(qs, ik, seq0 + (int64_t)b * block + c, index_dim, dtype) * index_scale;
        const T m2 = max_t(m, x);
        l = l * exp_t(m - m2) + exp_t(x - m2);
        m = m2;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const T m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const T l2 = __shfl_xor_sync(0xffffffffu, l, o);
      const T mm = max_t(m, m2);
      l = (m == T(-INFINITY) ? T(0) : l * exp_t(m - mm)) + (m2 == T(-INFINITY) ? T(0) : l2 * exp_t(m2 - mm));
      m = mm;
    }
    T dacc[kMaxIndexDim / 32];
#pragma unroll
    for (int i = 0; i < kMaxIndexDim / 32; ++i) dacc[i] = T(0);
    double kl = 0.0;
    if (l > T(0)) {
      const T lse = m + log_t(l);
      for (int j = 0; j < topk; ++j) {
        const int b = row_ids[j];
        if (!first_valid_slot(row_ids, j, b, cur)) continue;
        const int nk = b < cur ? block : pos - b * block + 1;
        const int64_t key0 = seq0 + (int64_t)b * block;
        T* slot_pt = pt + (p * topk + j) * block;
        for (int c0 = 0; c0 < block; c0 += 32) {
          const int c = c0 + lane;
          T g = T(0);
          if (c < nk) {
            const T ls = dot_key(qs, ik, key0 + c, index_dim, dtype) * index_scale - lse;  // log p_s
            const T ptv = slot_pt[c];
            if (ptv > T(0)) kl += (double)(ptv * (log_t(ptv) - ls));
            g = (exp_t(ls) - ptv) * inv_n * index_scale;
          }
          if (need_grad) {
            if (c < block) slot_pt[c] = g;  // 0 past the query: the dIK pass sums rows blindly
            const int ncc = min(32, nk - c0);
            for (int cc = 0; cc < ncc; ++cc) {
              const T gc = __shfl_sync(0xffffffffu, g, cc);
#pragma unroll
              for (int i = 0; i < kMaxIndexDim / 32; ++i) {
                const int d = lane + 32 * i;
                if (d < index_dim) dacc[i] += gc * load_as<T>(ik, (key0 + c0 + cc) * index_dim + d, dtype);
              }
            }
          }
        }
      }
    }
    kl = warp_sum(kl);
    if (lane == 0) loss_pair[p] = kl;
    if (need_grad) {
#pragma unroll
      for (int i = 0; i < kMaxIndexDim / 32; ++i) {
        const int d = lane + 32 * i;
        if (d < index_dim) diq[p * index_dim + d] = dacc[i];
      }
    }
  }
}

// Fast form for 16-bit inputs with index_dim 64 and 128-token blocks (float32):
// the pair's scaled iq row lives in every lane's registers (no shared-memory
// operand per product), lanes take keys, each dot product runs as 8 independent
// partial sums over 16-byte loads; pass 2 adds each key's dIQ contribution into
// per-lane accumulators (its index_k row reloaded, an L1 hit), one warp
// reduction per pair at the end.
constexpr int kFastDim = 64;

__device__ __forceinline__ void unpack8(const uint4 u, int f16, float* x) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = f16 ? __half22float2(*reinterpret_cast<const __half2*>(&w[e]))
                         : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[e]));
    x[2 * e] = f.x;
    x[2 * e + 1] = f.y;
  }
}

__device__ __forceinline__ float dot64(const float* __restrict__ qv, const void* __restrict__ ik, int64_t row,
                                       int f16) {
  const uint4* r = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(ik) + row * kFastDim * 2);
  uint4 u[kFastDim / 8];
#pragma unroll
  for (int d8 = 0; d8 < kFastDim / 8; ++d8) u[d8] = r[d8];  // all loads in flight first
  float part[8];
#pragma unroll
  for (int d8 = 0; d8 < kFastDim / 8; ++d8) {
    float x[8];
    unpack8(u[d8], f16, x);
    float a = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) a = fmaf(qv[d8 * 8 + e], x[e], a);
    part[d8] = a;
  }
  return ((part[0] + part[1]) + (part[2] + part[3])) + ((part[4] + part[5]) + (part[6] + part[7]));
}

__global__ void __launch_bounds__(128)
kl_student_fast_kernel(const void* __restrict__ iq, const void* __restrict__ ik, int f16,
                       const int32_t* __restrict__ ids, const int32_t* __restrict__ cu, int nseq, int64_t pairs,
                       int groups, int topk, float index_scale, float inv_n, int need_grad, float* __restrict__ pt,
                       double* __restrict__ loss_pair, float* __restrict__ diq) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  constexpr int kBlock = 128;
  for (int64_t p = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; p < pairs; p += warps) {
    const int64_t t = p / groups;
    const int s = find_sequence(cu, nseq, t);
    const int64_t seq0 = cu[s];
    const int pos = (int)(t - seq0), cur = pos / kBlock;
    const int32_t* row_ids = ids + p * topk;
    float qv[kFastDim];
    {
      const uint4* r = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(iq) + p * kFastDim * 2);
#pragma unroll
      for (int d8 = 0; d8 < kFastDim / 8; ++d8) unpack8(r[d8], f16, qv + d8 * 8);
#pragma unroll
      for (int d = 0; d < kFastDim; ++d) qv[d] *= index_scale;
    }
    float m = -INFINITY, l = 0.f;
    for (int j = 0; j < topk; ++j) {
      const int b = row_ids[j];
      if (!first_valid_slot(row_ids, j, b, cur)) continue;
      const int nk = b < cur ? kBlock : pos - b * kBlock + 1;
      for (int c = lane; c < nk; c += 32) {
        const float x = dot64(qv, ik, seq0 + (int64_t)b * kBlock + c, f16);
        const float m2 = fmaxf(m, x);
        l = l * __expf(m - m2) + __expf(x - m2);
        m = m2;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float l2 = __shfl_xor_sync(0xffffffffu, l, o);
      const float mm = fmaxf(m, m2);
      l = (m == -INFINITY ? 0.f : l * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : l2 * __expf(m2 - mm));
      m = mm;
    }
    float dacc[kFastDim];
#pragma unroll
    for (int d = 0; d < kFastDim; ++d) dacc[d] = 0.f;
    double kl = 0.0;
    if (l > 0.f) {
      const float lse = m + __logf(l);
      for (int j = 0; j < topk; ++j) {
        const int b = row_ids[j];
        if (!first_valid_slot(row_ids, j, b, cur)) continue;
        const int nk = b < cur ? kBlock : pos - b * kBlock + 1;
        float* slot_pt = pt + (p * topk + j) * kBlock;
        for (int c = lane; c < kBlock; c += 32) {
          float g = 0.f;
          if (c < nk) {
            const int64_t row = seq0 + (int64_t)b * kBlock + c;
            const float ls = dot64(qv, ik, row, f16) - lse;  // log p_s
            const float ptv = slot_pt[c];
            if (ptv > 0.f) kl += (double)(ptv * (__logf(ptv) - ls));
            g = (__expf(ls) - ptv) * inv_n * index_scale;
            if (need_grad) {
              const uint4* r = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(ik) + row * kFastDim * 2);
#pragma unroll
              for (int d8 = 0; d8 < kFastDim / 8; ++d8) {
                float x[8];
                unpack8(r[d8], f16, x);
#pragma unroll
                for (int e = 0; e < 8; ++e) dacc[d8 * 8 + e] = fmaf(g, x[e], dacc[d8 * 8 + e]);
              }
            }
          }
          if (need_grad) slot_pt[c] = g;  // 0 past the query: the dIK pass sums rows blindly
        }
      }
    }
    kl = warp_sum(kl);
    if (lane == 0) loss_pair[p] = kl;
    if (need_grad) {
#pragma unroll
      for (int d = 0; d < kFastDim; ++d) {
        const float v = warp_sum(dacc[d]);
        if (lane == (d & 31)) diq[p * kFastDim + d] = v;
      }
    }
  }
}

// --------------------------------------------------------------------------- dIK
// One CTA of 128 threads per (global key block, group, 128-key slice): thread c
// owns key c of the block and walks the group's CSR row of the block in edge
// order (a repeated (query, slot) of one query -- a duplicated block id -- counts
// once), 32 index dims at a time, the selecting pairs' iq rows staged in shared
// memory; the per-group sums go to part[key][group][Di] and kl_dik_reduce_kernel
// adds the groups in order (no atomics; one CTA per (block, group) spreads the
// hot early blocks' long rows over G CTAs).
constexpr int kDikThreads = 128;
constexpr int kDikEdges = 32;

template <typename T>
__global__ void __launch_bounds__(kDikThreads)
kl_dik_kernel(const void* __restrict__ iq, int dtype, const int32_t* __restrict__ cu,
              const int32_t* __restrict__ cbl, const int32_t* __restrict__ row_ptr,
              const int32_t* __restrict__ queries, const int32_t* __restrict__ slots, int nseq, int groups,
              int index_dim, int topk, int block, const T* __restrict__ g_pt, T* __restrict__ part) {
  constexpr int kDims = 64;  // index dims per pass over the row
  __shared__ T sq[kDikEdges][kDims];
  __shared__ int64_t soff[kDikEdges];
  const int gb = blockIdx.x, g = blockIdx.y;
  const int c = blockIdx.z * kDikThreads + threadIdx.x;
  int lo = 0, hi = nseq - 1;  // sequence of global block gb
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cbl[mid] <= gb) lo = mid; else hi = mid - 1;
  }
  const int64_t key0 = cu[lo] + (int64_t)(gb - cbl[lo]) * block;
  const int nk = (int)min((int64_t)block, (int64_t)cu[lo + 1] - key0);
  const int row = gb * groups + g;
  const int e0 = row_ptr[row], e1 = row_ptr[row + 1];
  for (int d0 = 0; d0 < index_dim; d0 += kDims) {
    T acc[kDims];
#pragma unroll
    for (int i = 0; i < kDims; ++i) acc[i] = T(0);
    for (int eb = e0; eb < e1; eb += kDikEdges) {
      const int ne = min(kDikEdges, e1 - eb);
      __syncthreads();
      // rows past the batch's end are zeroed: the product loop below runs in steps of 8 edges
      for (int x = threadIdx.x; x < kDikEdges * kDims; x += kDikThreads) {
        const int e = x / kDims, d = d0 + (x % kDims);
        if (e >= ne) {
          sq[e][x % kDims] = T(0);
          if (x % kDims == 0) soff[e] = -1;
          continue;
        }
        const int tq = queries[eb + e];
        const bool dup = eb + e > e0 && queries[eb + e - 1] == tq;
        const int64_t pair = (int64_t)tq * groups + g;
        sq[e][x % kDims] = (!dup && d < index_dim) ? load_as<T>(iq, pair * index_dim + d, dtype) : T(0);
        if (x % kDims == 0) soff[e] = dup ? -1 : (pair * topk + slots[eb + e]) * block;
      }
      __syncthreads();
      if (c < nk) {
        for (int e0 = 0; e0 < ne; e0 += 8) {
          T gv[8];  // eight loads in flight before their products
#pragma unroll
          for (int e = 0; e < 8; ++e) gv[e] = soff[e0 + e] >= 0 ? g_pt[soff[e0 + e] + c] : T(0);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
#pragma unroll
            for (int i = 0; i < kDims; ++i) acc[i] += gv[e] * sq[e0 + e][i];
          }
        }
      }
    }
    if (c < nk) {
#pragma unroll
      for (int i = 0; i < kDims; ++i)
        if (d0 + i < index_dim) part[((key0 + c) * groups + g) * index_dim + d0 + i] = acc[i];
    }
  }
}

// dik[j][d] = sum over groups g (in order) of part[j][g][d]; keys of blocks no
// query selected get 0.
template <typename T>
__global__ void kl_dik_reduce_kernel(const T* __restrict__ part, int64_t total, int groups, int index_dim,
                                     T* __restrict__ dik) {
  const int64_t n = total * index_dim;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = i / index_dim;
    const int d = (int)(i - j * index_dim);
    T s = T(0);
    for (int g = 0; g < groups; ++g) s += part[(j * groups + g) * index_dim + d];
    dik[i] = s;
  }
}

// --------------------------------------------------------------------------- teacher (precise)
// One warp per pair, float64: for each head of the group, the log-sum-exp of its
// logits over the pair's keys (lanes take keys), then p_h / h added into pt.
__global__ void kl_teacher_kernel(const void* __restrict__ q, const void* __restrict__ k, int dtype,
                                  const int32_t* __restrict__ ids, const int32_t* __restrict__ cu, int nseq,
                                  int64_t pairs, int q_heads, int groups, int dim, int topk, int block, double scale,
                                  double* __restrict__ pt) {
  const int lane = threadIdx.x & 31;
  const int h = q_heads / groups;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t p = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; p < pairs; p += warps) {
    const int64_t t = p / groups;
    const int g = (int)(p - t * groups);
    const int s = find_sequence(cu, nseq, t);
    const int64_t seq0 = cu[s];
    const int pos = (int)(t - seq0), cur = pos / block;
    const int32_t* row_ids = ids + p * topk;
    for (int j = 0; j < topk; ++j) {  // zero the pair's valid slots
      if (!first_valid_slot(row_ids, j, row_ids[j], cur)) continue;
      for (int c = lane; c < block; c += 32) pt[(p * topk + j) * block + c] = 0.0;
    }
    __syncwarp();
    for (int hh = 0; hh < h; ++hh) {
      const int64_t qoff = (t * q_heads + (int64_t)g * h + hh) * dim;
      auto logit = [&](int64_t key) -> double {
        double acc = 0.0;
        for (int d = 0; d < dim; ++d) acc += load_f64(q, qoff + d, dtype) * load_f64(k, (key * groups + g) * dim + d, dtype);
        return acc * scale;
      };
      double m = -INFINITY, l = 0.0;
      for (int j = 0; j < topk; ++j) {
        const int b = row_ids[j];
        if (!first_valid_slot(row_ids, j, b, cur)) continue;
        const int nk = b < cur ? block : pos - b * block + 1;
        for (int c = lane; c < nk; c += 32) {
          const double x = logit(seq0 + (int64_t)b * block + c);
          const double m2 = fmax(m, x);
          l = l * exp(m - m2) + exp(x - m2);
          m = m2;
        }
      }
      // combine the lanes' (m, l)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const double m2 = __shfl_xor_sync(0xffffffffu, m, o);
        const double l2 = __shfl_xor_sync(0xffffffffu, l, o);
        const double mm = fmax(m, m2);
        l = (m == -INFINITY ? 0.0 : l * exp(m - mm)) + (m2 == -INFINITY ? 0.0 : l2 * exp(m2 - mm));
        m = mm;
      }
      if (!(l > 0.0)) continue;
      const double lse = m + log(l);
      for (int j = 0; j < topk; ++j) {
        const int b = row_ids[j];
        if (!first_valid_slot(row_ids, j, b, cur)) continue;
        const int nk = b < cur ? block : pos - b * block + 1;
        for (int c = lane; c < nk; c += 32)
          pt[(p * topk + j) * block + c] += exp(logit(seq0 + (int64_t)b * block + c) - lse) / h;
      }
    }
  }
}

// Fixed-order sum of the per-pair losses times 1 / n (one CTA).
__global__ void __launch_bounds__(1024) kl_loss_reduce_kernel(const double* __restrict__ loss_pair, int64_t pairs,
                                                               double inv_n, double* __restrict__ loss) {
  __shared__ double part[1024];
  const int64_t per = (pairs + 1023) / 1024;
  double s = 0.0;
  for (int64_t i = threadIdx.x * per, e = min(pairs, (int64_t)(threadIdx.x + 1) * per); i < e; ++i) s += loss_pair[i];
  part[threadIdx.x] = s;
  __syncthreads();
  for (int w = 512; w > 0; w >>= 1) {
    if ((int)threadIdx.x < w) part[threadIdx.x] += part[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) *loss = part[0] * inv_n;
}

// --------------------------------------------------------------------------- tensor-core family, after the teacher
// Streaming student: the teacher pass wrote p_T (pt) and the student logits (sbuf)
// for every (pair, slot, key); one warp per pair reads both rows of each valid slot
// (lane = 4 keys), forms the pair's log-sum-exp, its KL and g = index_scale * dL/ds
// (written over pt). No index_k reads.
__global__ void __launch_bounds__(256)
kl_student_stream_kernel(const float* __restrict__ sbuf, float* __restrict__ pt, const int32_t* __restrict__ ids,
                         const int32_t* __restrict__ cu, int nseq, int64_t pairs, int groups, int topk,
                         float index_scale, float inv_n, int need_grad, double* __restrict__ loss_pair) {
  constexpr int kBlock = 128;
  const int lane = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t p = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; p < pairs; p += warps) {
    const int64_t t = p / groups;
    const int s = find_sequence(cu, nseq, t);
    const int pos = (int)(t - cu[s]), cur = pos / kBlock;
    const int32_t* row_ids = ids + p * topk;
    // slots that count (block in range, first occurrence of its id): lane j decides slot j
    // with one match.any when K <= 32, else every lane walks the list
    unsigned valid = 0u;
    int bl = -1;
    if (topk <= 32) {
      bl = lane < topk ? row_ids[lane] : -1;
      const unsigned peers = __match_any_sync(0xffffffffu, bl);
      valid = __ballot_sync(0xffffffffu, lane < topk && bl >= 0 && bl <= cur && (peers & ((1u << lane) - 1u)) == 0u);
    }
    auto slot_ok = [&](int j, int& b) -> bool {
      if (topk <= 32) {
        b = __shfl_sync(0xffffffffu, bl, j);
        return (valid >> j) & 1u;
      }
      b = row_ids[j];
      return first_valid_slot(row_ids, j, b, cur);
    };
    // pass 1: log-sum-exp; per row each lane folds its 4 keys into (m, l) with one rescale
    float m = -INFINITY, l = 0.f;
    for (int j = 0; j < topk; ++j) {
      int b;
      if (!slot_ok(j, b)) continue;  // warp-uniform
      const int nk = b < cur ? kBlock : pos - b * kBlock + 1;
      const float4 x = reinterpret_cast<const float4*>(sbuf + (p * topk + j) * kBlock)[lane];
      const float x0 = lane * 4 + 0 < nk ? x.x : -INFINITY, x1 = lane * 4 + 1 < nk ? x.y : -INFINITY;
      const float x2 = lane * 4 + 2 < nk ? x.z : -INFINITY, x3 = lane * 4 + 3 < nk ? x.w : -INFINITY;
      const float m2 = fmaxf(m, fmaxf(fmaxf(x0, x1), fmaxf(x2, x3)));
      if (m2 != -INFINITY) {
        l = l * __expf(m - m2) + ((__expf(x0 - m2) + __expf(x1 - m2)) + (__expf(x2 - m2) + __expf(x3 - m2)));
        m = m2;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float l2 = __shfl_xor_sync(0xffffffffu, l, o);
      const float mm = fmaxf(m, m2);
      l = (m == -INFINITY ? 0.f : l * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : l2 * __expf(m2 - mm));
      m = mm;
    }
    double kl = 0.0;
    if (l > 0.f) {
      const float lse = m + __logf(l);
      const float gscale = inv_n * index_scale;
      for (int j = 0; j < topk; ++j) {
        int b;
        if (!slot_ok(j, b)) continue;
        const int nk = b < cur ? kBlock : pos - b * kBlock + 1;
        const float4 x = reinterpret_cast<const float4*>(sbuf + (p * topk + j) * kBlock)[lane];
        float4* prow = reinterpret_cast<float4*>(pt + (p * topk + j) * kBlock);
        const float4 pv = prow[lane];
        const float xs[4] = {x.x, x.y, x.z, x.w}, ps[4] = {pv.x, pv.y, pv.z, pv.w};
        float gs[4], klr = 0.f;  // the row's 4 KL terms summed in float, added to the pair's float64 sum
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          gs[u] = 0.f;
          if (lane * 4 + u < nk) {
            const float ls = xs[u] - lse;  // log p_s
            if (ps[u] > 0.f) klr += ps[u] * (__logf(ps[u]) - ls);
            gs[u] = (__expf(ls) - ps[u]) * gscale;
          }
        }
        kl += (double)klr;
        if (need_grad) prow[lane] = make_float4(gs[0], gs[1], gs[2], gs[3]);  // 0 past the query
      }
    }
    kl = warp_sum(kl);
    if (lane == 0) loss_pair[p] = kl;
  }
}

// ---------------------------------------------------------------------------
// Tensor-core student logits and gradients (16-bit index tensors, Di = 64).
//
// One CTA (128 threads) per (key block, group) walks the group's k2q CSR row of
// the block in batches of 128 edges (an edge = one (query, selection slot) of
// the group that selected the block). Shared memory holds, in 128-byte-swizzled
// 128-byte rows (16-byte chunk j of row r at j ^ (r & 7)):
//   IK [128 keys][64 dims]     the block's index_k rows (zero past the sequence),
//   IQ [128 edges][64 dims]    the batch's index_q rows (zero for skipped edges),
//   G  [2][128 edges][64 keys] the batch's logit gradients (keys 0-63, 64-127).
// One layout serves both operand majors: IK is the K-major B of S = IQ.IK^T and
// the MN-major B of dIQ = G.IK; IQ the K-major A of S and the MN-major B of
// dIK = G^T.IQ; G the K-major A of dIQ and the MN-major A of dIK. One thread
// issues the MMAs (accumulators in TMEM, thread = TMEM lane = edge or key for the
// epilogue). Repeated (query, slot) edges of one query (duplicated block ids)
// count once.
constexpr int kKlEdges = 128;
constexpr int kKlSmemLogits = 2 * 16384 + 1024;            // IK, IQ (+ alignment)
constexpr int kKlSmemGrad = 2 * 16384 + 2 * 16384 + 1024;  // IK, IQ, G (+ alignment)

__device__ __forceinline__ uint8_t* kl_align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Byte offset of 16-byte chunk j of 128-byte row r in a 128-byte-swizzled tile.
__device__ __forceinline__ uint32_t sw128_off(int r, int j) { return (uint32_t)(r * 128 + ((j ^ (r & 7)) << 4)); }

// Sequence, first key and key count of global key block gb.
__device__ __forceinline__ void kl_block_keys(const int32_t* __restrict__ cu, const int32_t* __restrict__ cbl,
                                              int nseq, int gb, int64_t& key0, int& nk) {
  int lo = 0, hi = nseq - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cbl[mid] <= gb) lo = mid; else hi = mid - 1;
  }
  key0 = cu[lo] + (int64_t)(gb - cbl[lo]) * 128;
  nk = (int)min((int64_t)128, (int64_t)cu[lo + 1] - key0);
}

// The block's index_k rows into the swizzled IK tile (16 B per thread-step).
__device__ __forceinline__ void kl_stage_ik(uint8_t* sik, const void* __restrict__ ik, int64_t key0, int nk, int tid) {
  uint4 v[8];  // all eight loads in flight before the first store
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int x = tid + 128 * i, c = x >> 3, j = x & 7;
    v[i] = c < nk ? reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(ik) + (key0 + c) * 128)[j]
                  : make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int x = tid + 128 * i;
    *reinterpret_cast<uint4*>(sik + sw128_off(x >> 3, x & 7)) = v[i];
  }
}

// Edge e of the batch starting at CSR position eb (e < ne): its query, the
// previous edge's query (a repeat means a duplicated block id, counted once) and
// its selection slot. Loaded a batch ahead so the loads overlap the MMAs.
struct KlEdgeRaw {
  int q, prev, slot;
};
__device__ __forceinline__ KlEdgeRaw kl_edge_load(const int32_t* __restrict__ queries,
                                                  const int32_t* __restrict__ slots, int e0, int eb, int ne, int e) {
  KlEdgeRaw r{-1, -1, 0};
  if (e < ne) {
    r.q = queries[eb + e];
    r.prev = eb + e > e0 ? queries[eb + e - 1] : -1;
    r.slot = slots[eb + e];
  }
  return r;
}
// pair * topk + slot, or -1 (past the row end or a repeated edge)
__device__ __forceinline__ int64_t kl_edge_off(const KlEdgeRaw& r, int groups, int g, int topk) {
  return (r.q >= 0 && r.q != r.prev) ? ((int64_t)r.q * groups + g) * topk + r.slot : -1;
}

// The batch's index_q rows (soff: the edges' offsets), eight 16-byte loads per
// thread in flight, then into the swizzled IQ tile.
__device__ __forceinline__ void kl_load_iq(uint4 (&v)[8], const int64_t* soff, const void* __restrict__ iq, int topk,
                                           int tid) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int x = tid + 128 * i, e = x >> 3, j = x & 7;
    const int64_t o = soff[e];
    v[i] = o >= 0 ? reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(iq) + (o / topk) * 128)[j]
                  : make_uint4(0u, 0u, 0u, 0u);
  }
}
__device__ __forceinline__ void kl_store_iq(uint8_t* siq, const uint4 (&v)[8], int tid) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int x = tid + 128 * i;
    *reinterpret_cast<uint4*>(siq + sw128_off(x >> 3, x & 7)) = v[i];
  }
}

// S = IQ . IK^T for every edge of the row: sbuf[(pair, slot)][key] = index_scale *
// S (keys past the sequence come out 0 and are never read).
__global__ void __launch_bounds__(128)
kl_logits_mma_kernel(const void* __restrict__ iq, const void* __restrict__ ik, int f16,
                     const int32_t* __restrict__ cu, const int32_t* __restrict__ cbl,
                     const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ queries,
                     const int32_t* __restrict__ slots, int nseq, int groups, int topk, float index_scale,
                     int* __restrict__ err, float* __restrict__ sbuf) {
  extern __shared__ __align__(1024) uint8_t kl_smem_raw[];
  __shared__ int64_t soff[2][kKlEdges];  // per batch parity
  __shared__ uint64_t done;
  __shared__ uint32_t tmem_base;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int gb = blockIdx.x, g = blockIdx.y;
  const int row = gb * groups + g;
  const int e0 = row_ptr[row], e1 = row_ptr[row + 1];
  if (e0 == e1) return;
  uint8_t* smem = kl_align1024(kl_smem_raw);
  uint8_t* sik = smem;
  uint8_t* siq = smem + 16384;  // rewritten for the next batch once this batch's MMA is complete
  int64_t key0;
  int nk;
  kl_block_keys(cu, cbl, nseq, gb, key0, nk);
  if (tid == 0) {
    tc::mbar_init(&done, 1);
    tc::fence_barrier_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(&tmem_base, 128);
    tc::tmem_relinquish();
  }
  const int nbat = (e1 - e0 + kKlEdges - 1) / kKlEdges;
  {  // batch 0's edges and index_q rows
    soff[0][tid] = kl_edge_off(kl_edge_load(queries, slots, e0, e0, min(kKlEdges, e1 - e0), tid), groups, g, topk);
    kl_stage_ik(sik, ik, key0, nk, tid);
    __syncthreads();
    uint4 v[8];
    kl_load_iq(v, soff[0], iq, topk, tid);
    kl_store_iq(siq, v, tid);
  }
  tc::fence_proxy_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = tmem_base;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
  const uint32_t idesc = tc::idesc_f16(!f16, 128, 128, false, false);
  bool ok = true;
  for (int i = 0; i < nbat && ok; ++i) {
    const int buf = i & 1;
    const bool more = i + 1 < nbat;
    const int eb_next = e0 + (i + 1) * kKlEdges;
    const KlEdgeRaw nxt = kl_edge_load(queries, slots, e0, eb_next, more ? min(kKlEdges, e1 - eb_next) : 0, tid);
    if (tid == 0) {
      tc::tc_fence_after();
      const uint32_t a0 = tc::smem_u32(siq), b0 = tc::smem_u32(sik);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        tc::umma_ss(tmem, tc::desc_kmajor_sw128(a0 + ks * 32), tc::desc_kmajor_sw128(b0 + ks * 32), idesc, ks > 0);
      tc::umma_commit(&done);
    }
    // the next batch: edge offsets, then its index_q rows in flight during this batch's epilogue
    uint4 v[8];
    if (more) {
      soff[buf ^ 1][tid] = kl_edge_off(nxt, groups, g, topk);
      __syncthreads();
      kl_load_iq(v, soff[buf ^ 1], iq, topk, tid);
    }
    ok = tc::mbar_wait(&done, i & 1, err, 1);
    tc::tc_fence_after();
    const int64_t o = soff[buf][tid];  // thread = edge = TMEM lane
#pragma unroll 1
    for (int q = 0; q < 4; ++q) {
      uint32_t r[32];
      tc::tmem_ld32(tmem + lane_base + q * 32, r);
      tc::tmem_wait_ld();
      if (ok && o >= 0) {
        float4* dst = reinterpret_cast<float4*>(sbuf + o * 128 + q * 32);
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4)
          dst[c4] = make_float4(__uint_as_float(r[4 * c4]) * index_scale, __uint_as_float(r[4 * c4 + 1]) * index_scale,
                                __uint_as_float(r[4 * c4 + 2]) * index_scale, __uint_as_float(r[4 * c4 + 3]) * index_scale);
      }
    }
    if (more) {
      kl_store_iq(siq, v, tid);
      tc::fence_proxy_async_smem();
    }
    tc::tc_fence_before();
    ok = __syncthreads_and(ok);  // TMEM is rewritten by the next batch's MMA
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 128);
  }
}

// Gradients: per batch dIK += G^T . IQ (M = 128 keys, N = 64 dims, K = the
// batch's edges; accumulated in TMEM over the whole row) and dIQ = G . IK (M = 128
// edges, N = 64 dims, K = 128 keys) into diq_part[(pair, slot)]. The logit
// gradients g (float32, tiny: a 1/(T*G) factor) are staged as 16-bit values
// scaled by gscale, a power of two that brings them near 1 (exact; the
// epilogues multiply by 1/gscale).
__global__ void __launch_bounds__(128)
kl_grad_mma_kernel(const void* __restrict__ iq, const void* __restrict__ ik, int f16,
                   const int32_t* __restrict__ cu, const int32_t* __restrict__ cbl,
                   const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ queries,
                   const int32_t* __restrict__ slots, int nseq, int groups, int topk, const float* __restrict__ g_pt,
                   float gscale, int* __restrict__ err, float* __restrict__ dik_part, float* __restrict__ diq_part) {
  extern __shared__ __align__(1024) uint8_t kl_smem_raw[];
  __shared__ int64_t soff[2][kKlEdges];  // per batch parity
  __shared__ uint64_t done;
  __shared__ uint32_t tmem_base;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int gb = blockIdx.x, g = blockIdx.y;
  const int row = gb * groups + g;
  const int e0 = row_ptr[row], e1 = row_ptr[row + 1];
  if (e0 == e1) return;
  uint8_t* smem = kl_align1024(kl_smem_raw);
  uint8_t* sik = smem;
  uint8_t* siq = smem + 16384;
  uint8_t* sg = smem + 32768;  // two 16 KB halves: keys 0-63, 64-127
  int64_t key0;
  int nk;
  kl_block_keys(cu, cbl, nseq, gb, key0, nk);
  if (tid == 0) {
    tc::mbar_init(&done, 1);
    tc::fence_barrier_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(&tmem_base, 128);  // dIK at column 0, the batch's dIQ at 64
    tc::tmem_relinquish();
  }
  const int nbat = (e1 - e0 + kKlEdges - 1) / kKlEdges;
  {  // batch 0's edges and index_q rows
    soff[0][tid] = kl_edge_off(kl_edge_load(queries, slots, e0, e0, min(kKlEdges, e1 - e0), tid), groups, g, topk);
    kl_stage_ik(sik, ik, key0, nk, tid);
    __syncthreads();
    uint4 v[8];
    kl_load_iq(v, soff[0], iq, topk, tid);
    kl_store_iq(siq, v, tid);
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = tmem_base;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
  const uint32_t id_dk = tc::idesc_f16(!f16, 128, 64, true, true);   // M keys, N dims, K edges
  const uint32_t id_dq = tc::idesc_f16(!f16, 128, 64, false, true);  // M edges, N dims, K keys
  const float inv = 1.f / gscale;
  bool ok = true;
  for (int batch = 0; batch < nbat && ok; ++batch) {
    const int buf = batch & 1;
    const bool more = batch + 1 < nbat;
    const int eb_next = e0 + (batch + 1) * kKlEdges;
    const KlEdgeRaw nxt = kl_edge_load(queries, slots, e0, eb_next, more ? min(kKlEdges, e1 - eb_next) : 0, tid);
    const int64_t* so = soff[buf];
    // G: thread -> (edge e, keys 8j .. 8j + 7); 16 threads read one edge's 512-byte
    // row; eight rows' loads in flight at a time
    const int j16 = tid & 15, c0 = j16 * 8;
#pragma unroll 1
    for (int x0 = 0; x0 < kKlEdges * 16; x0 += 8 * 128) {
      float4 a[8], b[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int64_t o = so[(x0 + tid + 128 * i) >> 4];
        a[i] = o >= 0 ? *reinterpret_cast<const float4*>(g_pt + o * 128 + c0) : make_float4(0.f, 0.f, 0.f, 0.f);
        b[i] = o >= 0 ? *reinterpret_cast<const float4*>(g_pt + o * 128 + c0 + 4) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int e = (x0 + tid + 128 * i) >> 4;
        const float v[8] = {a[i].x, a[i].y, a[i].z, a[i].w, b[i].x, b[i].y, b[i].z, b[i].w};
        uint32_t w[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float lo = c0 + 2 * u < nk ? v[2 * u] * gscale : 0.f;  // keys past the sequence: 0
          const float hi = c0 + 2 * u + 1 < nk ? v[2 * u + 1] * gscale : 0.f;
          if (f16) {
            const __half2 h = __floats2half2_rn(lo, hi);
            w[u] = *reinterpret_cast<const uint32_t*>(&h);
          } else {
            const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
            w[u] = *reinterpret_cast<const uint32_t*>(&h);
          }
        }
        *reinterpret_cast<uint4*>(sg + (c0 >> 6) * 16384 + sw128_off(e, (c0 & 63) >> 3)) =
            make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    tc::fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
      tc::tc_fence_after();
      const uint32_t a_g = tc::smem_u32(sg), b_q = tc::smem_u32(siq), b_k = tc::smem_u32(sik);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)  // dIK: K = 16 edges per step (2048 B of each operand)
        tc::umma_ss(tmem, tc::desc_mnmajor_sw128(a_g + ks * 2048, 16384), tc::desc_mnmajor_sw128(b_q + ks * 2048, 16384),
                    id_dk, (batch > 0 || ks > 0) ? 1u : 0u);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)  // dIQ: K = 16 keys per step
        tc::umma_ss(tmem + 64, tc::desc_kmajor_sw128(a_g + (ks >> 2) * 16384 + (ks & 3) * 32),
                    tc::desc_mnmajor_sw128(b_k + ks * 2048, 16384), id_dq, ks > 0 ? 1u : 0u);
      tc::umma_commit(&done);
    }
    // the next batch: edge offsets, then its index_q rows in flight during this batch's epilogue
    uint4 vq[8];
    if (more) {
      soff[buf ^ 1][tid] = kl_edge_off(nxt, groups, g, topk);
      __syncthreads();
      kl_load_iq(vq, soff[buf ^ 1], iq, topk, tid);
    }
    ok = tc::mbar_wait(&done, batch & 1, err, 2);
    tc::tc_fence_after();
    const int64_t o = so[tid];  // thread = edge = TMEM lane
#pragma unroll 1
    for (int q = 0; q < 2; ++q) {
      uint32_t r[32];
      tc::tmem_ld32(tmem + 64 + lane_base + q * 32, r);
      tc::tmem_wait_ld();
      if (ok && o >= 0) {
        float4* dst = reinterpret_cast<float4*>(diq_part + o * 64 + q * 32);
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4)
          dst[c4] = make_float4(__uint_as_float(r[4 * c4]) * inv, __uint_as_float(r[4 * c4 + 1]) * inv,
                                __uint_as_float(r[4 * c4 + 2]) * inv, __uint_as_float(r[4 * c4 + 3]) * inv);
      }
    }
    if (more) kl_store_iq(siq, vq, tid);  // this batch's MMAs, the tile's readers, are complete
    tc::tc_fence_before();
    ok = __syncthreads_and(ok);  // TMEM's dIQ columns and the staged tiles are reused by the next batch
  }
  if (ok) {  // dIK of key tid = TMEM lane tid
    tc::tc_fence_after();
#pragma unroll 1
    for (int q = 0; q < 2; ++q) {
      uint32_t v[32];
      tc::tmem_ld32(tmem + lane_base + q * 32, v);
      tc::tmem_wait_ld();
      if (tid < nk) {
        float4* dst = reinterpret_cast<float4*>(dik_part + ((key0 + tid) * groups + g) * 64 + q * 32);
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4)
          dst[c4] = make_float4(__uint_as_float(v[4 * c4]) * inv, __uint_as_float(v[4 * c4 + 1]) * inv,
                                __uint_as_float(v[4 * c4 + 2]) * inv, __uint_as_float(v[4 * c4 + 3]) * inv);
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 128);
  }
}

// dIQ[pair] = sum over the pair's valid distinct slots (in slot order) of diq_part; one warp per pair.
__global__ void kl_diq_reduce_kernel(const float* __restrict__ diq_part, const int32_t* __restrict__ ids,
                                     const int32_t* __restrict__ cu, int nseq, int64_t pairs, int groups, int topk,
                                     float* __restrict__ diq) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t p = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; p < pairs; p += warps) {
    const int64_t t = p / groups;
    const int s = find_sequence(cu, nseq, t);
    const int cur = (int)(t - cu[s]) / 128;
    const int32_t* row_ids = ids + p * topk;
    float2 acc = make_float2(0.f, 0.f);
    for (int j = 0; j < topk; ++j) {
      if (!first_valid_slot(row_ids, j, row_ids[j], cur)) continue;
      const float2 v = reinterpret_cast<const float2*>(diq_part + (p * topk + j) * 64)[lane];
      acc.x += v.x;
      acc.y += v.y;
    }
    reinterpret_cast<float2*>(diq + p * 64)[lane] = acc;
  }
}

// A kernel error word poisons n floats with NaN (no-op otherwise).
__global__ void kl_poison_kernel(const int* __restrict__ err, int64_t n, float* __restrict__ p) {
  if (*err == 0) return;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    p[i] = __int_as_float(0x7fc00000);
}

constexpr int kKlMaxDevices = 64;
__device__ int g_kl_err;  // error word of the logits kernel (each device's copy of the module has its own)

}  // namespace
}  // namespace msa

using namespace msa;

// Device address of this device's logits error word (looked up once per device).
static int kl_err_word(int** out) {
  static std::mutex mu;
  static int* addr[kKlMaxDevices] = {};
  int dev = 0;
  MSA_CUDA_RETURN(cudaGetDevice(&dev));
  MSA_CHECK_ARG(dev >= 0 && dev < kKlMaxDevices, "index KL: device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* base = nullptr;
    MSA_CUDA_RETURN(cudaGetSymbolAddress(&base, g_kl_err));
    addr[dev] = static_cast<int*>(base);
  }
  *out = addr[dev];
  return MSA_OK;
}

extern "C" int msa_index_kl_teacher(const void* q, const void* k, int dtype, const int32_t* indices,
                                    const int32_t* cu_seqlens, int32_t nseq, int64_t total_tokens, int32_t q_heads,
                                    int32_t groups, int32_t head_dim, int32_t topk_blocks, int32_t block_size,
                                    double scale, double* pt, void* stream) {
  MSA_CHECK_ARG(valid_dtype(dtype), "msa_index_kl_teacher: bad dtype");
  MSA_CHECK_ARG(nseq >= 1 && groups >= 1 && q_heads % groups == 0 && head_dim >= 1 && topk_blocks >= 0 &&
                    block_size >= 1,
                "msa_index_kl_teacher: bad sizes");
  const int64_t pairs = total_tokens * groups;
  if (pairs == 0 || topk_blocks == 0) return MSA_OK;
  kl_teacher_kernel<<<ceil_div(pairs, 8), 256, 0, as_stream(stream)>>>(q, k, dtype, indices, cu_seqlens, nseq, pairs,
                                                                       q_heads, groups, head_dim, topk_blocks,
                                                                       block_size, scale, pt);
  count_launches(1);
  return launch_status("index_kl_teacher");
}

extern "C" size_t msa_index_kl_student_workspace_size(int64_t total_tokens, int32_t groups) {
  return sizeof(double) * (size_t)(total_tokens * groups + 1);
}

extern "C" int msa_index_kl_student(const void* index_q, const void* index_k, int dtype, const int32_t* indices,
                                    const int32_t* cu_seqlens, int32_t nseq, int64_t total_tokens, int32_t groups,
                                    int32_t index_dim, int32_t topk_blocks, int32_t block_size, double index_scale,
                                    void* pt, int pt_f64, int need_grad, double* loss, void* d_index_q_acc,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  MSA_CHECK_ARG(valid_dtype(dtype), "msa_index_kl_student: bad dtype");
  MSA_CHECK_ARG(index_dim >= 1 && index_dim <= kMaxIndexDim, "msa_index_kl_student: index_dim must be in [1, %d]",
                kMaxIndexDim);
  MSA_CHECK_ARG(nseq >= 1 && groups >= 1 && topk_blocks >= 0 && block_size >= 1, "msa_index_kl_student: bad sizes");
  const int64_t pairs = total_tokens * groups;
  MSA_CHECK_ARG(workspace && workspace_bytes >= msa_index_kl_student_workspace_size(total_tokens, groups),
                "msa_index_kl_student: workspace too small");
  cudaStream_t st = as_stream(stream);
  double* loss_pair = static_cast<double*>(workspace);
  if (pairs == 0) {
    MSA_CUDA_RETURN(cudaMemsetAsync(loss, 0, sizeof(double), st));
    return MSA_OK;
  }
  const double inv_n = 1.0 / (double)pairs;
  const unsigned grid = (unsigned)std::min<int64_t>(ceil_div(pairs, kStudentWarps), 148 * 64);
  if (pt_f64)
    kl_student_kernel<double><<<grid, kStudentWarps * 32, 0, st>>>(index_q, index_k, dtype, indices, cu_seqlens, nseq, pairs, groups,
                                                    index_dim, topk_blocks, block_size, index_scale, inv_n, need_grad,
                                                    static_cast<double*>(pt), loss_pair,
                                                    static_cast<double*>(d_index_q_acc));
  else if (dtype != MSA_F32 && block_size == 128 && index_dim == kFastDim) {
    const unsigned fgrid = (unsigned)std::min<int64_t>(ceil_div(pairs, 4), 148 * 64);
    kl_student_fast_kernel<<<fgrid, 128, 0, st>>>(index_q, index_k, dtype == MSA_F16 ? 1 : 0, indices, cu_seqlens, nseq, pairs, groups,
                                topk_blocks, (float)index_scale, (float)inv_n, need_grad, static_cast<float*>(pt),
                                loss_pair, static_cast<float*>(d_index_q_acc));
  } else
    kl_student_kernel<float><<<grid, kStudentWarps * 32, 0, st>>>(index_q, index_k, dtype, indices, cu_seqlens, nseq, pairs, groups,
                                                   index_dim, topk_blocks, block_size, (float)index_scale,
                                                   (float)inv_n, need_grad, static_cast<float*>(pt), loss_pair,
                                                   static_cast<float*>(d_index_q_acc));
  kl_loss_reduce_kernel<<<1, 1024, 0, st>>>(loss_pair, pairs, inv_n, loss);
  count_launches(2);
  return launch_status("index_kl_student");
}

extern "C" size_t msa_index_kl_dik_workspace_size(int64_t total_tokens, int32_t groups, int32_t index_dim,
                                                  int pt_f64) {
  return (size_t)total_tokens * groups * index_dim * (pt_f64 ? 8 : 4) + 256;
}

extern "C" int msa_index_kl_dik(const void* index_q, int dtype, const int32_t* cu_seqlens, const int32_t* cu_block_lens,
                                const int32_t* row_ptr, const int32_t* query_indices, const int32_t* slot_indices,
                                int32_t nseq, int64_t total_tokens, int32_t groups, int32_t index_dim,
                                int32_t topk_blocks, int32_t block_size, int32_t total_blocks, const void* g_pt,
                                int pt_f64, void* d_index_k_acc, void* workspace, size_t workspace_bytes,
                                void* stream) {
  MSA_CHECK_ARG(valid_dtype(dtype), "msa_index_kl_dik: bad dtype");
  MSA_CHECK_ARG(nseq >= 1 && groups >= 1 && index_dim >= 1 && block_size >= 1 && total_blocks >= 0,
                "msa_index_kl_dik: bad sizes");
  MSA_CHECK_ARG(workspace && workspace_bytes >= msa_index_kl_dik_workspace_size(total_tokens, groups, index_dim, pt_f64),
                "msa_index_kl_dik: workspace too small");
  if (total_tokens == 0) return MSA_OK;
  cudaStream_t st = as_stream(stream);
  // keys of blocks that no query selected keep a zero gradient
  MSA_CUDA_RETURN(cudaMemsetAsync(workspace, 0, (size_t)total_tokens * groups * index_dim * (pt_f64 ? 8 : 4), st));
  const unsigned red_grid = (unsigned)std::min<int64_t>(ceil_div(total_tokens * index_dim, 256), 148 * 32);
  if (total_blocks > 0) {
    const dim3 grid((unsigned)total_blocks, (unsigned)groups, (unsigned)ceil_div(block_size, kDikThreads));
    if (pt_f64)
      kl_dik_kernel<double><<<grid, kDikThreads, 0, st>>>(index_q, dtype, cu_seqlens, cu_block_lens, row_ptr,
                                                          query_indices, slot_indices, nseq, groups, index_dim,
                                                          topk_blocks, block_size, static_cast<const double*>(g_pt),
                                                          static_cast<double*>(workspace));
    else
      kl_dik_kernel<float><<<grid, kDikThreads, 0, st>>>(index_q, dtype, cu_seqlens, cu_block_lens, row_ptr,
                                                         query_indices, slot_indices, nseq, groups, index_dim,
                                                         topk_blocks, block_size, static_cast<const float*>(g_pt),
                                                         static_cast<float*>(workspace));
    count_launches(1);
  }
  if (pt_f64)
    kl_dik_reduce_kernel<double><<<red_grid, 256, 0, st>>>(static_cast<const double*>(workspace), total_tokens, groups,
                                                           index_dim, static_cast<double*>(d_index_k_acc));
  else
    kl_dik_reduce_kernel<float><<<red_grid, 256, 0, st>>>(static_cast<const float*>(workspace), total_tokens, groups,
                                                          index_dim, static_cast<float*>(d_index_k_acc));
  count_launches(1);
  return launch_status("index_kl_dik");
}

extern "C" int msa_index_kl_student_tc(const float* sbuf, float* pt, const int32_t* indices, const int32_t* cu_seqlens,
                                       int32_t nseq, int64_t total_tokens, int32_t groups, int32_t topk_blocks,
                                       double index_scale, int need_grad, double* loss, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  MSA_CHECK_ARG(nseq >= 1 && groups >= 1 && topk_blocks >= 0, "msa_index_kl_student_tc: bad sizes");
  MSA_CHECK_ARG(workspace && workspace_bytes >= msa_index_kl_student_workspace_size(total_tokens, groups),
                "msa_index_kl_student_tc: workspace too small");
  cudaStream_t st = as_stream(stream);
  const int64_t pairs = total_tokens * groups;
  if (pairs == 0) {
    MSA_CUDA_RETURN(cudaMemsetAsync(loss, 0, sizeof(double), st));
    return MSA_OK;
  }
  double* loss_pair = static_cast<double*>(workspace);
  const double inv_n = 1.0 / (double)pairs;
  kl_student_stream_kernel<<<(unsigned)std::min<int64_t>(ceil_div(pairs, 8), 148 * 64), 256, 0, st>>>(
      sbuf, pt, indices, cu_seqlens, nseq, pairs, groups, topk_blocks, (float)index_scale, (float)inv_n, need_grad,
      loss_pair);
  kl_loss_reduce_kernel<<<1, 1024, 0, st>>>(loss_pair, pairs, inv_n, loss);
  count_launches(2);
  return launch_status("index_kl_student_tc");
}

extern "C" size_t msa_index_kl_grad_tc_workspace_size(int64_t total_tokens, int32_t groups, int32_t topk_blocks) {
  // per-(pair, slot) dIQ rows, then per-(key, group) dIK rows, float32 x 64 dims
  return sizeof(float) * 64 * (size_t)(total_tokens * groups) * (size_t)(topk_blocks + 1) + 256;
}

extern "C" int msa_index_kl_grad_tc(const void* index_q, const void* index_k, int dtype, const int32_t* indices,
                                    const int32_t* cu_seqlens, const int32_t* cu_block_lens, const int32_t* row_ptr,
                                    const int32_t* query_indices, const int32_t* slot_indices, int32_t nseq,
                                    int64_t total_tokens, int32_t groups, int32_t topk_blocks, int32_t total_blocks,
                                    double index_scale, const float* g_pt, float* d_index_q, float* d_index_k,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  MSA_CHECK_ARG(dtype == MSA_BF16 || dtype == MSA_F16, "msa_index_kl_grad_tc: bf16/f16 only");
  MSA_CHECK_ARG(nseq >= 1 && groups >= 1 && topk_blocks >= 0 && total_blocks >= 0, "msa_index_kl_grad_tc: bad sizes");
  MSA_CHECK_ARG(workspace && workspace_bytes >= msa_index_kl_grad_tc_workspace_size(total_tokens, groups, topk_blocks),
                "msa_index_kl_grad_tc: workspace too small");
  if (total_tokens == 0) return MSA_OK;
  cudaStream_t st = as_stream(stream);
  const int64_t pairs = total_tokens * groups;
  float* diq_part = static_cast<float*>(workspace);
  float* dik_part = diq_part + (size_t)pairs * topk_blocks * 64;
  int* err = reinterpret_cast<int*>(dik_part + (size_t)pairs * 64);  // the workspace's last 256 bytes
  // |g| <= |index_scale| / (T * G): stage g * 2^k with 2^k near (T * G) / |index_scale|
  const double mag = (double)pairs / (index_scale != 0.0 ? fabs(index_scale) : 1.0);
  const int k = std::max(-100, std::min(100, (int)std::lround(std::log2(mag))));
  const float gscale = std::ldexp(1.0f, k);
  // keys of blocks that no query selected keep a zero gradient
  MSA_CUDA_RETURN(cudaMemsetAsync(dik_part, 0, sizeof(float) * 64 * (size_t)pairs + sizeof(int), st));
  if (total_blocks > 0) {
    MSA_CUDA_RETURN(cudaFuncSetAttribute(kl_grad_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kKlSmemGrad));
    kl_grad_mma_kernel<<<dim3((unsigned)total_blocks, (unsigned)groups), 128, kKlSmemGrad, st>>>(
        index_q, index_k, dtype == MSA_F16 ? 1 : 0, cu_seqlens, cu_block_lens, row_ptr, query_indices, slot_indices,
        nseq, groups, topk_blocks, g_pt, gscale, err, dik_part, diq_part);
    count_launches(1);
  }
  kl_diq_reduce_kernel<<<(unsigned)std::min<int64_t>(ceil_div(pairs, 8), 148 * 64), 256, 0, st>>>(
      diq_part, indices, cu_seqlens, nseq, pairs, groups, topk_blocks, d_index_q);
  kl_dik_reduce_kernel<float><<<(unsigned)std::min<int64_t>(ceil_div(total_tokens * 64, 256), 148 * 32), 256, 0, st>>>(
      dik_part, total_tokens, groups, 64, d_index_k);
  // a kernel that gave up on a wait poisons both gradients with NaN
  kl_poison_kernel<<<148 * 4, 256, 0, st>>>(err, pairs * 64, d_index_q);
  kl_poison_kernel<<<148 * 4, 256, 0, st>>>(err, total_tokens * 64, d_index_k);
  count_launches(4);
  return launch_status("index_kl_grad_tc");
}

extern "C" int msa_index_kl_logits_tc(const void* index_q, const void* index_k, int dtype, const int32_t* cu_seqlens,
                                      const int32_t* cu_block_lens, const int32_t* row_ptr,
                                      const int32_t* query_indices, const int32_t* slot_indices, int32_t nseq,
                                      int64_t total_tokens, int32_t groups, int32_t topk_blocks, int32_t total_blocks,
                                      double index_scale, float* sbuf, void* stream) {
  MSA_CHECK_ARG(dtype == MSA_BF16 || dtype == MSA_F16, "msa_index_kl_logits_tc: bf16/f16 only");
  MSA_CHECK_ARG(nseq >= 1 && groups >= 1 && topk_blocks >= 0 && total_blocks >= 0, "msa_index_kl_logits_tc: bad sizes");
  if (total_tokens == 0 || total_blocks == 0) return MSA_OK;
  int* err = nullptr;
  if (int e = kl_err_word(&err)) return e;
  cudaStream_t st = as_stream(stream);
  MSA_CUDA_RETURN(cudaMemsetAsync(err, 0, sizeof(int), st));
  // at most four CTAs per SM: four 128-column TMEM allocations fill the SM's 512
  constexpr int smem_bytes = kKlSmemLogits > 52 * 1024 ? kKlSmemLogits : 52 * 1024;
  MSA_CUDA_RETURN(cudaFuncSetAttribute(kl_logits_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes));
  kl_logits_mma_kernel<<<dim3((unsigned)total_blocks, (unsigned)groups), 128, smem_bytes, st>>>(
      index_q, index_k, dtype == MSA_F16 ? 1 : 0, cu_seqlens, cu_block_lens, row_ptr, query_indices, slot_indices,
      nseq, groups, topk_blocks, (float)index_scale, err, sbuf);
  kl_poison_kernel<<<148 * 4, 256, 0, st>>>(err, total_tokens * groups * (int64_t)topk_blocks * 128, sbuf);
  count_launches(2);
  return launch_status("index_kl_logits_tc");
}
