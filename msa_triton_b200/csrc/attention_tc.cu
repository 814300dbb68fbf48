// Sparse attention forward, tensor-core path (sm_100a: TMA + tcgen05 + TMEM).
//
// Organisation: key-block stationary. The work list is the k2q CSR (one row per
// (128-key block, group); triton/k2q.py:39-128), cut into chunks of 128/h
// selector tokens (h = query heads per group). A chunk is one M = 128 tile whose
// rows are (token, head) pairs: TMA gathers each selector token's h query rows
// (contiguous in q[T][Hq][D]) into the tile, so the block's K/V, loaded once per
// row, serve every head of every selecting token.
//
//   S   = Q_tile . K_b^T                      tcgen05, SMEM x SMEM -> TMEM (f32)
//   P   = exp(scale*S - bound_row), causal    softmax warps, P -> TMEM as bf16/f16
//   O_e = P . V_b                             tcgen05, TMEM x SMEM -> TMEM (f32)
//   O_acc[t, heads] += O_e ; l_acc += rowsum(P)   TMA bulk tensor reductions
//
// A query's softmax spans up to K chunks on different CTAs, so the exponent is
// taken against a per-row static upper bound, bound = |scale| |q_row| max_j|k_j|
// (Cauchy-Schwarz), instead of a running maximum; contributions then add with
// no rescaling. Rows whose bound exceeds kBoundLimit (where exp(S - bound)
// could underflow for every key) are recomputed by the float64 row kernel.
// finalize: out = O_acc / l, lse = bound + log(l).
//
// Roles (384 threads): warp 0 = TMA producer, warp 1 = MMA issuer, warps 4-7
// and 8-11 = two softmax/epilogue warpgroups taking alternate chunks, each with
// its own TMEM stage (S/P 128 columns + O 128 columns).
#include <algorithm>

#include "tc_common.cuh"

namespace msa {
int launch_fwd_fixup(const void* q, const void* k, const void* v, int dtype, const int32_t* ids, const int32_t* cu,
                     int nseq, int hq, int groups, int dim, int topk, int block, double scale, const int32_t* list,
                     void* out, float* lse, cudaStream_t st);

namespace {

using namespace tc;

constexpr int kD = 128;
constexpr int kFwdThreads = 384;
constexpr float kLog2e = 1.4426950408889634f;
// exp(S - bound) >= exp(-2 bound) must stay a normal float for the row maximum.
constexpr float kBoundLimit = 43.0f;
constexpr int kSmemFwd = 6 * 32768 + 1024;

struct FwdArgs {
  const int32_t* row_ptr;
  const int32_t* queries;
  const int32_t* chunk_ptr;
  const int32_t* cu;
  const int32_t* cbl;  // cu_block_lens
  const float* bound;  // [T*Hq]
  float* l_acc;        // [T*Hq]
  int* err;
  int nseq, num_rows, groups, hq, h, tpc;
  float scale_log2;
  int f16;  // 1: fp16 operands, 0: bf16
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Largest row r with chunk_ptr[r] <= w (rows without chunks are skipped).
__device__ __forceinline__ int first_row_of(const int32_t* chunk_ptr, int num_rows, int w) {
  int lo = 0, hi = num_rows - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (chunk_ptr[mid] <= w) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ int advance_row(const int32_t* chunk_ptr, int row, int w) {
  while (chunk_ptr[row + 1] <= w) ++row;
  return row;
}

struct RowInfo {
  int g, e_begin, e_end;
  int kb0;  // packed token id of the block's first key
};

__device__ __forceinline__ RowInfo row_info(const FwdArgs& a, int row) {
  RowInfo ri;
  const int gb = row / a.groups;
  ri.g = row - gb * a.groups;
  int lo = 0, hi = a.nseq - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (a.cbl[mid] <= gb) lo = mid; else hi = mid - 1;
  }
  ri.kb0 = a.cu[lo] + (gb - a.cbl[lo]) * 128;
  ri.e_begin = a.row_ptr[row];
  ri.e_end = a.row_ptr[row + 1];
  return ri;
}

// A repeated slot of the same query sits right after its first occurrence in the
// row (edges are ordered by query, then slot); it selects the block only once.
__device__ __forceinline__ bool is_dup(const int32_t* queries, int e, int e_begin, int t) {
  return e > e_begin && __ldg(queries + e - 1) == t;
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi, int f16) {
  if (f16) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__global__ void __launch_bounds__(kFwdThreads, 1)
attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap, const __grid_constant__ CUtensorMap omap, FwdArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sQ0 = smem;                 // Q tiles: 2 stages x (2 d-chunks x 128 rows x 128 B)
  uint8_t* sK = smem + 2 * 32768;      // K block (2 d-chunks x 128 keys x 128 B)
  uint8_t* sV = smem + 3 * 32768;      // V block
  uint8_t* sStage0 = smem + 4 * 32768; // O staging: 2 warpgroups x (2 d-chunks x 128 rows x 128 B)
  __shared__ uint64_t q_full[2], q_empty[2], s_full[2], p_full[2], o_full[2], o_free[2];
  __shared__ uint64_t kv_full, kv_empty;
  __shared__ uint32_t tmem_base;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int j = 0; j < 2; ++j) {
      mbar_init(&q_full[j], 1);
      mbar_init(&q_empty[j], 1);
      mbar_init(&s_full[j], 1);
      mbar_init(&p_full[j], 4);
      mbar_init(&o_full[j], 1);
      mbar_init(&o_free[j], 4);
    }
    mbar_init(&kv_full, 1);
    mbar_init(&kv_empty, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  const int total_chunks = a.chunk_ptr[a.num_rows];
  const int w_begin = (int)((int64_t)blockIdx.x * total_chunks / gridDim.x);
  const int w_end = (int)((int64_t)(blockIdx.x + 1) * total_chunks / gridDim.x);
  const int n_items = w_end - w_begin;
  const int h = a.h, tpc = a.tpc;

  if (n_items > 0 && warp == 0 && lane == 0) {
    // ---------------------------------------------------------------- producer
    tma_prefetch_desc(&qmap);
    tma_prefetch_desc(&kmap);
    tma_prefetch_desc(&vmap);
    int row = -1, rows_started = 0;
    RowInfo ri{};
    for (int i = 0; i < n_items; ++i) {
      const int w = w_begin + i;
      const int r = row < 0 ? first_row_of(a.chunk_ptr, a.num_rows, w) : advance_row(a.chunk_ptr, row, w);
      if (r != row) {
        if (rows_started > 0 && !mbar_wait(&kv_empty, (rows_started - 1) & 1, a.err, 11)) break;
        row = r;
        ri = row_info(a, row);
        ++rows_started;
        mbar_arrive_expect_tx(&kv_full, 4 * 16384);
        for (int dc = 0; dc < 2; ++dc) {
          tma_load_3d(sK + dc * 16384, &kmap, &kv_full, dc * 64, ri.g, ri.kb0);
          tma_load_3d(sV + dc * 16384, &vmap, &kv_full, dc * 64, ri.g, ri.kb0);
        }
      }
      const int j = i & 1;
      if (i >= 2 && !mbar_wait(&q_empty[j], ((i >> 1) - 1) & 1, a.err, 12)) break;
      const int e0 = ri.e_begin + (w - a.chunk_ptr[row]) * tpc;
      const int e1 = min(e0 + tpc, ri.e_end);
      uint32_t nv = 0;
      for (int e = e0; e < e1; ++e) nv += is_dup(a.queries, e, ri.e_begin, __ldg(a.queries + e)) ? 0u : 1u;
      mbar_arrive_expect_tx(&q_full[j], nv * (uint32_t)h * 256u);
      uint8_t* sQ = sQ0 + j * 32768;
      for (int e = e0; e < e1; ++e) {
        const int t = __ldg(a.queries + e);
        if (is_dup(a.queries, e, ri.e_begin, t)) continue;
        for (int dc = 0; dc < 2; ++dc)
          tma_load_3d(sQ + dc * 16384 + (e - e0) * h * 128, &qmap, &q_full[j], dc * 64, ri.g * h, t);
      }
    }
  } else if (n_items > 0 && warp == 1 && lane == 0) {
    // ---------------------------------------------------------------- MMA issuer
    const uint32_t id_s = idesc_f16(!a.f16, 128, 128, false, false);
    const uint32_t id_pv = idesc_f16(!a.f16, 128, 128, false, true);
    auto issue_s = [&](int i) -> bool {
      const int j = i & 1;
      if (!mbar_wait(&q_full[j], (i >> 1) & 1, a.err, 21)) return false;
      if (i >= 2 && !mbar_wait(&o_full[j], ((i >> 1) - 1) & 1, a.err, 22)) return false;
      tc_fence_after();
      const uint32_t sq = smem_u32(sQ0 + j * 32768), sk = smem_u32(sK);
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
        umma_ss(tmem + j * 256, desc_kmajor_sw128(sq + off), desc_kmajor_sw128(sk + off), id_s, ks > 0);
      }
      umma_commit(&s_full[j]);
      umma_commit(&q_empty[j]);
      return true;
    };
    auto issue_pv = [&](int i) -> bool {
      const int j = i & 1;
      if (!mbar_wait(&p_full[j], (i >> 1) & 1, a.err, 23)) return false;
      if (i >= 2 && !mbar_wait(&o_free[j], ((i >> 1) - 1) & 1, a.err, 24)) return false;
      tc_fence_after();
      const uint32_t sv = smem_u32(sV);
      for (int ks = 0; ks < 8; ++ks)
        umma_ts(tmem + j * 256 + 128, tmem + j * 256 + ks * 8, desc_mnmajor_sw128(sv + ks * 2048, 16384), id_pv,
                ks > 0);
      umma_commit(&o_full[j]);
      return true;
    };
    int row = -1, rows_seen = 0;
    bool ok = true;
    for (int i = 0; i < n_items && ok; ++i) {
      const int w = w_begin + i;
      const int r = row < 0 ? first_row_of(a.chunk_ptr, a.num_rows, w) : advance_row(a.chunk_ptr, row, w);
      const bool new_row = r != row;
      if (new_row && i > 0) {  // the previous chunk's P.V must be done with V before K/V are replaced
        ok = issue_pv(i - 1);
        if (!ok) break;
        umma_commit(&kv_empty);
      }
      if (new_row) {
        row = r;
        ok = mbar_wait(&kv_full, rows_seen & 1, a.err, 25);
        ++rows_seen;
        if (!ok) break;
      }
      ok = issue_s(i);
      if (ok && !new_row && i > 0) ok = issue_pv(i - 1);
    }
    if (ok) {
      issue_pv(n_items - 1);
      umma_commit(&kv_empty);
    }
  } else if (n_items > 0 && warp >= 4) {
    // ---------------------------------------------------------------- softmax + epilogue
    const int wg = (warp - 4) >> 2;
    const int qd = warp & 3;
    const int r = qd * 32 + lane;  // tile row == TMEM lane
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const uint32_t t_s = tmem + wg * 256 + lane_base, t_o = t_s + 128;
    uint8_t* stage = sStage0 + wg * 32768;
    int row = -1;
    RowInfo ri{};
    bool pending = false;
    for (int i = wg; i < n_items; i += 2) {
      const int w = w_begin + i;
      const int rr = row < 0 ? first_row_of(a.chunk_ptr, a.num_rows, w) : advance_row(a.chunk_ptr, row, w);
      if (rr != row) {
        row = rr;
        ri = row_info(a, row);
      }
      const int e0 = ri.e_begin + (w - a.chunk_ptr[row]) * tpc;
      const int e1 = min(e0 + tpc, ri.e_end);
      const int pos = r / h, hh = r - (r / h) * h;
      const int e = e0 + pos;
      bool valid = e < e1;
      int t = 0;
      if (valid) {
        t = __ldg(a.queries + e);
        valid = !is_dup(a.queries, e, ri.e_begin, t);
      }
      const int64_t rowid = (int64_t)t * a.hq + ri.g * h + hh;
      const float nbound = valid ? -__ldg(a.bound + rowid) * kLog2e : 0.f;
      const int qoff = t - ri.kb0;  // key c of the block is visible iff c <= qoff
      if (!mbar_wait_warp(&s_full[wg], (i >> 1) & 1, a.err, 31)) break;
      tc_fence_after();
      float l = 0.f;
      for (int half = 0; half < 2; ++half) {
        uint32_t packed[32];
#pragma unroll
        for (int sub = 0; sub < 2; ++sub) {
          const int c = half * 2 + sub;
          uint32_t sr[32];
          tmem_ld32(t_s + c * 32, sr);
          tmem_wait_ld();
#pragma unroll
          for (int kk = 0; kk < 32; kk += 2) {
            const int key = c * 32 + kk;
            const float p0 = (valid && key <= qoff) ? exp2f(fmaf(__uint_as_float(sr[kk]), a.scale_log2, nbound)) : 0.f;
            const float p1 =
                (valid && key + 1 <= qoff) ? exp2f(fmaf(__uint_as_float(sr[kk + 1]), a.scale_log2, nbound)) : 0.f;
            l += p0 + p1;
            packed[sub * 16 + (kk >> 1)] = pack2(p0, p1, a.f16);
          }
        }
        tmem_st32(t_s + half * 32, packed);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[wg]);
      if (valid) atomicAdd(a.l_acc + rowid, l);
      if (!mbar_wait_warp(&o_full[wg], (i >> 1) & 1, a.err, 32)) break;
      tc_fence_after();
      for (int half = 0; half < 2; ++half) {
        if (pending) {
          if (lane == 0) bulk_wait_read0();
          __syncwarp();
          pending = false;
        }
#pragma unroll
        for (int dcl = 0; dcl < 2; ++dcl) {
          uint32_t orr[32];
          tmem_ld32(t_o + (half * 2 + dcl) * 32, orr);
          tmem_wait_ld();
          uint8_t* rowp = stage + dcl * 16384 + r * 128;
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<uint4*>(rowp + ((u ^ (r & 7)) << 4)) =
                make_uint4(orr[4 * u], orr[4 * u + 1], orr[4 * u + 2], orr[4 * u + 3]);
        }
        if (half == 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&o_free[wg]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          for (int p2 = qd * 32 / h; p2 < (qd + 1) * 32 / h; ++p2) {
            const int e2 = e0 + p2;
            if (e2 >= e1) break;
            const int t2 = __ldg(a.queries + e2);
            if (is_dup(a.queries, e2, ri.e_begin, t2)) continue;
            for (int dcl = 0; dcl < 2; ++dcl)
              tma_reduce_add_3d(&omap, stage + dcl * 16384 + p2 * h * 128, (half * 2 + dcl) * 32, ri.g * h, t2);
          }
          bulk_commit();
        }
        pending = true;
      }
    }
    if (lane == 0) bulk_wait0();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------- helpers
// Largest |k| over all key rows (float bits are ordered for non-negative values).
__global__ void key_norm_max_kernel(const void* __restrict__ k, int dtype, int64_t rows, unsigned* __restrict__ kmax) {
  const int lane = threadIdx.x & 31;
  float best = 0.f;
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < rows;
       row += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    float s = 0.f;
    for (int d = lane; d < kD; d += 32) {
      const float x = (float)load_f64(k, row * kD + d, dtype);
      s = fmaf(x, x, s);
    }
    best = fmaxf(best, sqrtf(warp_sum(s)));
  }
  if (lane == 0) atomicMax(kmax, __float_as_uint(best));
}

// Per query row: bound = |scale| |q| max|k| (slightly inflated so float
// rounding cannot put a logit above it); rows beyond the limit are listed.
__global__ void row_bound_kernel(const void* __restrict__ q, int dtype, int64_t rows, const unsigned* __restrict__ kmax,
                                 float abs_scale, float* __restrict__ bound, int32_t* __restrict__ fix_list) {
  const int lane = threadIdx.x & 31;
  const float km = __uint_as_float(*kmax);
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < rows;
       row += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    float s = 0.f;
    for (int d = lane; d < kD; d += 32) {
      const float x = (float)load_f64(q, row * kD + d, dtype);
      s = fmaf(x, x, s);
    }
    s = warp_sum(s);
    if (lane == 0) {
      const float b = abs_scale * sqrtf(s) * km * 1.0001f + 1e-6f;
      bound[row] = b;
      if (b > kBoundLimit) {
        const int slot = atomicAdd(fix_list, 1);
        fix_list[1 + slot] = (int32_t)row;
      }
    }
  }
}

// chunk_ptr[r] = sum over rows < r of ceil(len / tpc); one CTA of 1024 threads.
__global__ void __launch_bounds__(1024) chunk_ptr_kernel(const int32_t* __restrict__ row_ptr, int num_rows, int tpc,
                                                         int32_t* __restrict__ chunk_ptr) {
  __shared__ int32_t warp_tot[32];
  __shared__ int32_t carry;
  if (threadIdx.x == 0) {
    carry = 0;
    chunk_ptr[0] = 0;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int base = 0; base < num_rows; base += 1024) {
    const int r = base + threadIdx.x;
    const int c = r < num_rows ? (row_ptr[r + 1] - row_ptr[r] + tpc - 1) / tpc : 0;
    int x = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int wsum = warp_tot[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, wsum, o);
        if (lane >= o) wsum += y;
      }
      warp_tot[lane] = wsum;
    }
    __syncthreads();
    const int incl = x + (warp > 0 ? warp_tot[warp - 1] : 0);
    if (r < num_rows) chunk_ptr[r + 1] = carry + incl;
    __syncthreads();
    if (threadIdx.x == 1023) carry += incl;
    __syncthreads();
  }
}

// out = O_acc / l (16 threads per row, 8 columns each); lse = bound + log(l).
// A kernel error word poisons the outputs with NaN instead of leaving stale data.
__global__ void fwd_finalize_kernel(const float* __restrict__ o_acc, const float* __restrict__ l_acc,
                                    const float* __restrict__ bound, int64_t rows, int f16, const int* __restrict__ err,
                                    void* __restrict__ out, float* __restrict__ lse) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t row = idx >> 4;
  const int c = (int)(idx & 15);
  if (row >= rows) return;
  const bool bad = *err != 0;
  const float l = l_acc[row];
  const float inv = bad ? __int_as_float(0x7fc00000) : (l > 0.f ? 1.f / l : 0.f);
  const float4 a = *reinterpret_cast<const float4*>(o_acc + row * kD + c * 8);
  const float4 b = *reinterpret_cast<const float4*>(o_acc + row * kD + c * 8 + 4);
  uint4 packed;
  packed.x = pack2(a.x * inv, a.y * inv, f16);
  packed.y = pack2(a.z * inv, a.w * inv, f16);
  packed.z = pack2(b.x * inv, b.y * inv, f16);
  packed.w = pack2(b.z * inv, b.w * inv, f16);
  *reinterpret_cast<uint4*>(static_cast<uint8_t*>(out) + (row * kD + c * 8) * 2) = packed;
  if (c == 0) lse[row] = bad ? __int_as_float(0x7fc00000) : (l > 0.f ? bound[row] + logf(l) : -INFINITY);
}

struct FwdWorkspace {
  float* o_acc;
  float* l_acc;
  float* bound;
  int32_t* chunk_ptr;
  int32_t* fix_list;
  unsigned* kmax;
  int* err;
  size_t bytes;
};

inline size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

FwdWorkspace carve_fwd(void* base, int64_t rows, int64_t num_rows) {
  FwdWorkspace w{};
  char* b = static_cast<char*>(base);
  size_t off = 0;
  w.o_acc = reinterpret_cast<float*>(b + off);
  off = a256(off + sizeof(float) * rows * kD);
  w.l_acc = reinterpret_cast<float*>(b + off);
  off = a256(off + sizeof(float) * rows);
  const size_t zero_end = off;  // o_acc and l_acc are zeroed together
  w.bound = reinterpret_cast<float*>(b + off);
  off = a256(off + sizeof(float) * rows);
  w.chunk_ptr = reinterpret_cast<int32_t*>(b + off);
  off = a256(off + sizeof(int32_t) * (num_rows + 1));
  w.kmax = reinterpret_cast<unsigned*>(b + off);
  w.err = reinterpret_cast<int*>(b + off + 4);
  w.fix_list = reinterpret_cast<int32_t*>(b + off + 8);
  off = a256(off + 8 + sizeof(int32_t) * (rows + 1));
  w.bytes = off;
  (void)zero_end;
  return w;
}

}  // namespace
}  // namespace msa

using namespace msa;

extern "C" size_t msa_attn_fwd_tc_workspace_size(int64_t total_tokens, int32_t q_heads, int32_t num_rows) {
  return carve_fwd(nullptr, total_tokens * q_heads, num_rows).bytes;
}

extern "C" int msa_attn_fwd_tc(const void* q, const void* k, const void* v, int dtype, const int32_t* indices,
                               const int32_t* cu_seqlens, const int32_t* cu_block_lens, const int32_t* row_ptr,
                               const int32_t* query_indices, int32_t nseq, int64_t total_tokens, int32_t q_heads,
                               int32_t groups, int32_t head_dim, int32_t topk_blocks, int32_t block_size, double scale,
                               int32_t num_rows, void* out, float* lse, void* workspace, size_t workspace_bytes,
                               void* stream) {
  MSA_CHECK_ARG(dtype == MSA_BF16 || dtype == MSA_F16, "msa_attn_fwd_tc: bf16/f16 only");
  MSA_CHECK_ARG(head_dim == kD && block_size == 128, "msa_attn_fwd_tc: head_dim and block_size must be 128");
  MSA_CHECK_ARG(groups >= 1 && q_heads % groups == 0, "msa_attn_fwd_tc: bad head counts");
  const int h = q_heads / groups;
  MSA_CHECK_ARG(h == 4 || h == 8 || h == 16, "msa_attn_fwd_tc: query heads per group must be 4, 8 or 16");
  MSA_CHECK_ARG(total_tokens < (int64_t)1 << 31 && num_rows >= 0, "msa_attn_fwd_tc: size out of range");
  const int64_t rows = total_tokens * q_heads;
  if (rows == 0) return MSA_OK;
  const FwdWorkspace w = carve_fwd(workspace, rows, num_rows);
  MSA_CHECK_ARG(workspace && workspace_bytes >= w.bytes, "msa_attn_fwd_tc: workspace too small");
  cudaStream_t st = as_stream(stream);
  const int cd = tc::tma_dtype(dtype) == CU_TENSOR_MAP_DATA_TYPE_FLOAT16 ? 1 : 0;

  CUtensorMap qmap, kmap, vmap, omap;
  {
    const uint64_t dq[3] = {(uint64_t)kD, (uint64_t)q_heads, (uint64_t)total_tokens};
    const uint64_t sq[2] = {(uint64_t)kD * 2, (uint64_t)q_heads * kD * 2};
    const uint32_t bq[3] = {64, (uint32_t)h, 1};
    if (int e = tc::encode_tensor_map(&qmap, tc::tma_dtype(dtype), 3, q, dq, sq, bq, CU_TENSOR_MAP_SWIZZLE_128B)) return e;
    const uint64_t dk[3] = {(uint64_t)kD, (uint64_t)groups, (uint64_t)total_tokens};
    const uint64_t sk[2] = {(uint64_t)kD * 2, (uint64_t)groups * kD * 2};
    const uint32_t bk[3] = {64, 1, 128};
    if (int e = tc::encode_tensor_map(&kmap, tc::tma_dtype(dtype), 3, k, dk, sk, bk, CU_TENSOR_MAP_SWIZZLE_128B)) return e;
    if (int e = tc::encode_tensor_map(&vmap, tc::tma_dtype(dtype), 3, v, dk, sk, bk, CU_TENSOR_MAP_SWIZZLE_128B)) return e;
    const uint64_t so[2] = {(uint64_t)kD * 4, (uint64_t)q_heads * kD * 4};
    const uint32_t bo[3] = {32, (uint32_t)h, 1};
    if (int e = tc::encode_tensor_map(&omap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, w.o_acc, dq, so, bo,
                                      CU_TENSOR_MAP_SWIZZLE_128B))
      return e;
  }
  // zero O_acc and l_acc (contiguous) and the small counters
  MSA_CUDA_RETURN(cudaMemsetAsync(w.o_acc, 0, reinterpret_cast<char*>(w.bound) - reinterpret_cast<char*>(w.o_acc), st));
  MSA_CUDA_RETURN(cudaMemsetAsync(w.kmax, 0, 12, st));
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  key_norm_max_kernel<<<sms * 4, 256, 0, st>>>(k, dtype, total_tokens * groups, w.kmax);
  row_bound_kernel<<<sms * 8, 256, 0, st>>>(q, dtype, rows, w.kmax, (float)fabs(scale), w.bound, w.fix_list);
  count_launches(2);
  if (num_rows > 0) {
    chunk_ptr_kernel<<<1, 1024, 0, st>>>(row_ptr, num_rows, 128 / h, w.chunk_ptr);
    FwdArgs fa{row_ptr, query_indices, w.chunk_ptr, cu_seqlens, cu_block_lens, w.bound, w.l_acc, w.err,
               nseq, num_rows, groups, q_heads, h, 128 / h, (float)(scale * 1.4426950408889634), cd};
    MSA_CUDA_RETURN(cudaFuncSetAttribute(attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemFwd));
    attn_fwd_tc_kernel<<<sms, kFwdThreads, kSmemFwd, st>>>(qmap, kmap, vmap, omap, fa);
    count_launches(2);
  }
  fwd_finalize_kernel<<<ceil_div(rows * 16, 256), 256, 0, st>>>(w.o_acc, w.l_acc, w.bound, rows, cd, w.err, out, lse);
  count_launches(1);
  if (int e = launch_status("attn_fwd_tc")) return e;
  return launch_fwd_fixup(q, k, v, dtype, indices, cu_seqlens, nseq, q_heads, groups, head_dim, topk_blocks,
                          block_size, scale, w.fix_list, out, lse, st);
}

extern "C" int msa_attn_fwd_tc_error(const void* workspace, int64_t total_tokens, int32_t q_heads, int32_t num_rows,
                                     int32_t* host_err) {
  const FwdWorkspace w = carve_fwd(const_cast<void*>(workspace), total_tokens * q_heads, num_rows);
  MSA_CUDA_RETURN(cudaMemcpy(host_err, w.err, sizeof(int32_t), cudaMemcpyDeviceToHost));
  return MSA_OK;
}
