// Decode over a paged KV cache: one new query token per request attends to its
// selected blocks of keys stored in fixed-size pages (the serving-side layout of
// the reference's notes on vLLM-Ascend, docs/vllm_ascend_k2q.md:22-40: a block
// table maps each request's logical pages to physical pages). The reference
// implements no decode path; these kernels follow the same selection semantics
// as the prefill path: a query at position p = seq_len - 1 sees key j of a
// selected block b iff b <= p / block_size and j <= p; a repeated block id counts
// once; -1 pads.
//
// Decode is HBM-bound (each (request, group) reads its K selected blocks of K and
// V once for its h query heads), so the kernels are CUDA-core kernels with
// 16-byte loads:
//   * index score: one CTA per (request, logical block), thread = key, all groups;
//   * attention: split over the selected blocks, one CTA per (request, group,
//     slot) computing the block's partial softmax (max, sum, unnormalised P V) for
//     the group's heads; a combine kernel merges the partials per (request, head)
//     (out = sum O_j e^(m_j - M) / L, lse = M + log L).
#include <algorithm>

#include "common.cuh"

namespace msa {
namespace {

constexpr int kThreads = 128;
constexpr int kMaxHeads = 16;   // query heads per group
constexpr int kMaxDim = 256;    // head / index dim

template <typename F>
__device__ __forceinline__ void for_row(const void* base, int64_t row, int dim, int dtype, F&& f) {
  // calls f(d, value) for the `dim` elements of row `row` (16-byte loads for 16-bit rows of whole units)
  if (dtype != MSA_F32 && (dim & 7) == 0) {
    const uint4* r = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(base) + row * dim * 2);
    for (int d8 = 0; d8 < dim / 8; ++d8) {
      const uint4 u = r[d8];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 x = dtype == MSA_F16 ? __half22float2(*reinterpret_cast<const __half2*>(&w[e]))
                                          : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[e]));
        f(d8 * 8 + 2 * e, x.x);
        f(d8 * 8 + 2 * e + 1, x.y);
      }
    }
    return;
  }
  for (int d = 0; d < dim; ++d) f(d, (float)load_f64(base, row * dim + d, dtype));
}

__device__ __forceinline__ float to_f32(const void* p, int64_t i, int dtype) {
  if (dtype == MSA_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dtype == MSA_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_f32(void* p, int64_t i, int dtype, float x) {
  if (dtype == MSA_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(x);
  else if (dtype == MSA_F16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(x);
  else reinterpret_cast<float*>(p)[i] = x;
}

// Physical cache row of request b's logical key j (rows of `heads` x dim each page slot).
__device__ __forceinline__ int64_t cache_slot(const int32_t* __restrict__ block_table, int max_pages, int page_size,
                                              int b, int64_t j) {
  const int page = block_table[(int64_t)b * max_pages + j / page_size];
  return (int64_t)page * page_size + j % page_size;
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float m = red[0];
  for (int w = 1; w < kThreads / 32; ++w) m = fmaxf(m, red[w]);
  __syncthreads();
  return m;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
  for (int w = 0; w < kThreads / 32; ++w) s += red[w];
  __syncthreads();
  return s;
}

// ------------------------------------------------------------------ index score
// scores[b][g][blk] = max over the block's keys j <= p of scale * iq[b][g] . ik[j]; -inf past p.
__global__ void __launch_bounds__(kThreads)
decode_score_kernel(const void* __restrict__ iq, const void* __restrict__ ik_cache, int dtype,
                    const int32_t* __restrict__ block_table, const int32_t* __restrict__ seq_lens, int groups,
                    int dim, int page_size, int max_pages, int num_blocks, int block, float scale,
                    float* __restrict__ scores) {
  __shared__ float qs[kMaxHeads * kMaxDim];
  __shared__ float red[kThreads / 32];
  const int b = blockIdx.x, blk = blockIdx.y;
  const int pos = seq_lens[b] - 1;
  float* dst = scores + ((int64_t)b * groups) * num_blocks + blk;
  if (pos < 0 || blk > pos / block) {
    for (int g = threadIdx.x; g < groups; g += kThreads) dst[(int64_t)g * num_blocks] = -INFINITY;
    return;
  }
  for (int i = threadIdx.x; i < groups * dim; i += kThreads) qs[i] = to_f32(iq, (int64_t)b * groups * dim + i, dtype);
  __syncthreads();
  const int n = min(block, pos - blk * block + 1);
  for (int g = 0; g < groups; ++g) {
    float best = -INFINITY;
    for (int c = threadIdx.x; c < n; c += kThreads) {
      const int64_t row = cache_slot(block_table, max_pages, page_size, b, (int64_t)blk * block + c);
      float acc = 0.f;
      for_row(ik_cache, row, dim, dtype, [&](int d, float x) { acc = fmaf(qs[g * dim + d], x, acc); });
      best = fmaxf(best, acc * scale);
    }
    best = block_max(best, red);
    if (threadIdx.x == 0) dst[(int64_t)g * num_blocks] = best;
  }
}

// ------------------------------------------------------------------ attention partials
// One CTA per (request, group, slot). Keys go in passes of 128 (thread c takes
// key c0 + c and holds its logits for the group's h heads); each pass's P sits
// in shared memory for the P V product, where thread d accumulates output dim d,
// and passes merge online. Statistics are in base-2 units (logits times
// scale * log2 e).
__global__ void __launch_bounds__(kThreads)
decode_partial_kernel(const void* __restrict__ q, const void* __restrict__ k_cache, const void* __restrict__ v_cache,
                      int dtype, const int32_t* __restrict__ block_table, const int32_t* __restrict__ seq_lens,
                      const int32_t* __restrict__ ids, int q_heads, int groups, int dim, int page_size,
                      int max_pages, int topk, int block, float scale_log2, float* __restrict__ part_m,
                      float* __restrict__ part_l, float* __restrict__ part_o) {
  __shared__ float qs[kMaxHeads * kMaxDim];
  __shared__ float ps[kThreads][kMaxHeads + 1];
  __shared__ float red[kThreads / 32];
  __shared__ float run_m[kMaxHeads], run_l[kMaxHeads], alpha[kMaxHeads];
  const int tid = threadIdx.x;
  const int bg = blockIdx.x, j = blockIdx.y;
  const int b = bg / groups, g = bg - b * groups;
  const int h = q_heads / groups;
  const int pos = seq_lens[b] - 1;
  const int32_t* row_ids = ids + (int64_t)bg * topk;
  const int blk = row_ids[j];
  bool valid = pos >= 0 && blk >= 0 && blk <= pos / block;
  for (int i = 0; i < j && valid; ++i) valid = row_ids[i] != blk;  // a repeated block counts once
  const int64_t part = (int64_t)bg * topk + j;
  if (!valid) {
    if (tid < h) {
      part_m[part * h + tid] = -INFINITY;
      part_l[part * h + tid] = 0.f;
    }
    return;
  }
  const int64_t q0 = ((int64_t)b * q_heads + (int64_t)g * h) * dim;
  for (int i = tid; i < h * dim; i += kThreads) qs[i] = to_f32(q, q0 + i, dtype);
  __syncthreads();
  const int n = min(block, pos - blk * block + 1);  // causal: the query's own block up to the query
  for (int c0 = 0; c0 < n; c0 += kThreads) {
    const int c = c0 + tid;
    float s[kMaxHeads];
#pragma unroll
    for (int hh = 0; hh < kMaxHeads; ++hh) s[hh] = 0.f;
    if (c < n) {
      const int64_t row = cache_slot(block_table, max_pages, page_size, b, (int64_t)blk * block + c) * groups + g;
      for_row(k_cache, row, dim, dtype, [&](int d, float x) {
#pragma unroll
        for (int hh = 0; hh < kMaxHeads; ++hh)
          if (hh < h) s[hh] = fmaf(qs[hh * dim + d], x, s[hh]);
      });
    }
    for (int hh = 0; hh < h; ++hh) {
      float x = -INFINITY;
#pragma unroll
      for (int u = 0; u < kMaxHeads; ++u)
        if (u == hh) x = s[u];  // static register indexing
      x = c < n ? x * scale_log2 : -INFINITY;
      const float mm_pass = block_max(x, red);
      const float mm = c0 == 0 ? mm_pass : fmaxf(run_m[hh], mm_pass);
      const float p = c < n ? exp2f(x - mm) : 0.f;
      ps[tid][hh] = p;
      const float l = block_sum(p, red);
      if (tid == 0) {
        const float a = c0 == 0 ? 0.f : exp2f(run_m[hh] - mm);
        alpha[hh] = a;
        run_l[hh] = (c0 == 0 ? 0.f : run_l[hh] * a) + l;
        run_m[hh] = mm;
      }
    }
    __syncthreads();
    const int kn = min(kThreads, n - c0);
    for (int d = tid; d < dim; d += kThreads) {
      float acc[kMaxHeads];
#pragma unroll
      for (int hh = 0; hh < kMaxHeads; ++hh) acc[hh] = 0.f;
      for (int cc = 0; cc < kn; ++cc) {
        const int64_t row =
            cache_slot(block_table, max_pages, page_size, b, (int64_t)blk * block + c0 + cc) * groups + g;
        const float x = to_f32(v_cache, row * dim + d, dtype);
#pragma unroll
        for (int hh = 0; hh < kMaxHeads; ++hh)
          if (hh < h) acc[hh] = fmaf(ps[cc][hh], x, acc[hh]);
      }
#pragma unroll
      for (int hh = 0; hh < kMaxHeads; ++hh) {
        if (hh < h) {
          float* o = part_o + (part * h + hh) * dim + d;
          *o = (c0 == 0 ? 0.f : *o * alpha[hh]) + acc[hh];
        }
      }
    }
    __syncthreads();
  }
  if (tid < h) {
    part_m[part * h + tid] = run_m[tid];
    part_l[part * h + tid] = run_l[tid];
  }
}

// One warp per (request, query head): merge the slots' partials.
__global__ void decode_combine_kernel(const float* __restrict__ part_m, const float* __restrict__ part_l,
                                      const float* __restrict__ part_o, int batch, int q_heads, int groups, int dim,
                                      int topk, int dtype, void* __restrict__ out, float* __restrict__ lse) {
  const int lane = threadIdx.x & 31;
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (row >= (int64_t)batch * q_heads) return;
  const int b = (int)(row / q_heads), hd = (int)(row - (int64_t)b * q_heads);
  const int h = q_heads / groups, bg = b * groups + hd / h, hh = hd % h;
  float m = -INFINITY;
  for (int j = 0; j < topk; ++j) m = fmaxf(m, part_m[((int64_t)bg * topk + j) * h + hh]);
  float l = 0.f;
  if (m > -INFINITY)
    for (int j = 0; j < topk; ++j) {
      const float mj = part_m[((int64_t)bg * topk + j) * h + hh];
      if (mj > -INFINITY) l += part_l[((int64_t)bg * topk + j) * h + hh] * exp2f(mj - m);
    }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  for (int d = lane; d < dim; d += 32) {
    float acc = 0.f;
    if (l > 0.f)
      for (int j = 0; j < topk; ++j) {
        const float mj = part_m[((int64_t)bg * topk + j) * h + hh];
        if (mj > -INFINITY) acc += part_o[(((int64_t)bg * topk + j) * h + hh) * dim + d] * exp2f(mj - m);
      }
    store_f32(out, row * dim + d, dtype, acc * inv);
  }
  if (lane == 0) lse[row] = l > 0.f ? (m + log2f(l)) * 0.6931471805599453f : -INFINITY;
}

}  // namespace
}  // namespace msa

using namespace msa;

extern "C" int msa_decode_index_score(const void* index_q, const void* index_k_cache, int dtype,
                                      const int32_t* block_table, const int32_t* seq_lens, int32_t batch,
                                      int32_t groups, int32_t index_dim, int32_t page_size, int32_t max_pages,
                                      int32_t num_blocks, int32_t block_size, double scale, float* scores,
                                      void* stream) {
  MSA_CHECK_ARG(valid_dtype(dtype), "msa_decode_index_score: bad dtype");
  MSA_CHECK_ARG(groups >= 1 && groups <= kMaxHeads && index_dim >= 1 && groups * index_dim <= kMaxHeads * kMaxDim,
                "msa_decode_index_score: groups * index_dim must be at most %d", kMaxHeads * kMaxDim);
  MSA_CHECK_ARG(page_size >= 1 && max_pages >= 1 && num_blocks >= 1 && block_size >= 1 && batch >= 0,
                "msa_decode_index_score: bad sizes");
  if (batch == 0) return MSA_OK;
  decode_score_kernel<<<dim3((unsigned)batch, (unsigned)num_blocks), kThreads, 0, as_stream(stream)>>>(
      index_q, index_k_cache, dtype, block_table, seq_lens, groups, index_dim, page_size, max_pages, num_blocks,
      block_size, (float)scale, scores);
  count_launches(1);
  return launch_status("decode_index_score");
}

extern "C" size_t msa_decode_attn_workspace_size(int32_t batch, int32_t q_heads, int32_t head_dim,
                                                 int32_t topk_blocks) {
  return sizeof(float) * (size_t)batch * q_heads * topk_blocks * (head_dim + 2) + 256;
}

extern "C" int msa_decode_attn(const void* q, const void* k_cache, const void* v_cache, int dtype,
                               const int32_t* block_table, const int32_t* seq_lens, const int32_t* indices,
                               int32_t batch, int32_t q_heads, int32_t groups, int32_t head_dim, int32_t page_size,
                               int32_t max_pages, int32_t topk_blocks, int32_t block_size, double scale, void* out,
                               float* lse, void* workspace, size_t workspace_bytes, void* stream) {
  MSA_CHECK_ARG(valid_dtype(dtype), "msa_decode_attn: bad dtype");
  MSA_CHECK_ARG(groups >= 1 && q_heads % groups == 0 && q_heads / groups <= kMaxHeads,
                "msa_decode_attn: at most %d query heads per group", kMaxHeads);
  MSA_CHECK_ARG(head_dim >= 1 && head_dim <= kMaxDim, "msa_decode_attn: head_dim must be in [1, %d]", kMaxDim);
  MSA_CHECK_ARG(page_size >= 1 && max_pages >= 1 && block_size >= 1 && topk_blocks >= 0 && batch >= 0,
                "msa_decode_attn: bad sizes");
  MSA_CHECK_ARG(workspace_bytes >= msa_decode_attn_workspace_size(batch, q_heads, head_dim, topk_blocks),
                "msa_decode_attn: workspace too small");
  if (batch == 0) return MSA_OK;
  cudaStream_t st = as_stream(stream);
  const size_t parts = (size_t)batch * q_heads * topk_blocks;  // (request, group, slot, head)
  float* part_m = static_cast<float*>(workspace);
  float* part_l = part_m + parts;
  float* part_o = part_l + parts;
  if (topk_blocks > 0) {
    decode_partial_kernel<<<dim3((unsigned)(batch * groups), (unsigned)topk_blocks), kThreads, 0, st>>>(
        q, k_cache, v_cache, dtype, block_table, seq_lens, indices, q_heads, groups, head_dim, page_size, max_pages,
        topk_blocks, block_size, (float)(scale * 1.4426950408889634), part_m, part_l, part_o);
    count_launches(1);
  }
  decode_combine_kernel<<<ceil_div((int64_t)batch * q_heads * 32, 256), 256, 0, st>>>(
      part_m, part_l, part_o, batch, q_heads, groups, head_dim, topk_blocks, dtype, out, lse);
  count_launches(1);
  return launch_status("decode_attn");
}
