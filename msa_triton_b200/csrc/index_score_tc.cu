// Index score, tensor-core path (sm_100a: TMA + tcgen05 + TMEM).
//
//   scores[t][g][b] = scale * max_{j in block b, j <= t} index_q[t][g] . index_k[j]
// (the _index_score_forward contract, triton/index_score.py:93-136), with
// future and out-of-sequence blocks -inf. The T x T logits never reach memory.
//
// A work item is one tile of 128 rows: 128/G consecutive tokens of one sequence
// times the G groups, i.e. 128 consecutive rows of index_q viewed as [T*G][Di]
// (one TMA box per 64 columns). The tile walks the causal key blocks
// b = 0 .. qb of its sequence (all its tokens share qb because 128/G divides
// 128): TMA loads the 128 x Di block of index_k, one thread issues
// S = IQ . IK_b^T (M = N = 128) into one of four TMEM stages, and an epilogue
// warpgroup (thread = tile row) reads S back with tcgen05.ld and takes the row
// maximum (diagonal block: keys up to the token only). Maxima of four blocks go
// out as one 16-byte store. Items are dealt to CTAs round-robin, each
// sequence's tiles last-first (the longest causal rows first).
#include <mutex>

#include "attn_common.cuh"

namespace msa {
namespace {

using namespace tc;
using namespace attn;

constexpr int kScoreThreads = 256;  // warp 0 producer, warp 1 MMA issuer, warps 4-7 epilogue
constexpr int kIkStages = 4;
constexpr int kTmStages = 4;
constexpr int kMetaSlots = 4;
constexpr int kSmemScore = 2 * 32768 + kIkStages * 32768 + 1024;

struct ItemMeta {
  int32_t seq_start, n_tokens, t0, qb;  // sequence start, tokens in the tile, first token, diagonal block
  int32_t done, pad0, pad1, pad2;
};

struct ScoreArgs {
  const int32_t* cu;
  float* scores;
  int* err;
  int nseq, groups, nb, tq, kchunks;  // tq = 128 / G tokens per tile, kchunks = Di / 64
  int q_lo, q_hi;                     // query tokens scored: [q_lo, q_hi)
  float abs_scale;
  int neg;  // 1: negative scale (the maximum of scale * dot is scale * the minimum dot)
  int f16;
};

// Item order: sequences in order, each sequence's tiles last-first; CTA c takes
// items c, c + grid, ... fn(seq_start, seq_len, tile) runs for each of its items.
// Only tiles that hold a token of [q_lo, q_hi) are items (their other tokens are
// not written).
template <typename F>
__device__ __forceinline__ bool for_my_items(const ScoreArgs& a, F&& fn) {
  int64_t base = 0;
  for (int s = 0; s < a.nseq; ++s) {
    const int start = a.cu[s], len = a.cu[s + 1] - start;
    const int lo = max(a.q_lo, start), hi = min(a.q_hi, start + len);
    if (lo >= hi) continue;
    const int t_first = (lo - start) / a.tq, t_last = (hi - 1 - start) / a.tq;
    const int nt = t_last - t_first + 1;
    const int64_t first = base + (((int64_t)blockIdx.x - base) % gridDim.x + gridDim.x) % gridDim.x;
    for (int64_t i = first; i < base + nt; i += gridDim.x)
      if (!fn(start, len, t_last - (int)(i - base))) return false;
    base += nt;
  }
  return true;
}

__device__ __forceinline__ void store_maxima(float* row, int cb, int nb, const float (&v)[4]) {
  if ((nb & 3) == 0) {
    *reinterpret_cast<float4*>(row + cb) = make_float4(v[0], v[1], v[2], v[3]);
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (cb + k < nb) row[cb + k] = v[k];
  }
}

__global__ void __launch_bounds__(kScoreThreads, 1)
score_tc_kernel(const __grid_constant__ CUtensorMap iqmap, const __grid_constant__ CUtensorMap ikmap, ScoreArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sIQ = smem;              // 2 tiles x (Di/64 chunks x 128 rows x 128 B)
  uint8_t* sIK = smem + 2 * 32768;  // kIkStages key blocks, same layout
  __shared__ ItemMeta meta[kMetaSlots];
  __shared__ uint64_t meta_full[kMetaSlots], meta_empty[kMetaSlots], iq_full[2], iq_empty[2];
  __shared__ uint64_t ik_full[kIkStages], ik_empty[kIkStages], s_full[kTmStages], s_free[kTmStages];
  __shared__ uint32_t tmem_base;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int j = 0; j < kMetaSlots; ++j) {
      mbar_init(&meta_full[j], 1);
      mbar_init(&meta_empty[j], 5);  // MMA issuer + 4 epilogue warps
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&iq_full[j], 1);
      mbar_init(&iq_empty[j], 1);
    }
    for (int j = 0; j < kIkStages; ++j) {
      mbar_init(&ik_full[j], 1);
      mbar_init(&ik_empty[j], 1);
    }
    for (int j = 0; j < kTmStages; ++j) {
      mbar_init(&s_full[j], 1);
      mbar_init(&s_free[j], 4);
    }
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
  const uint32_t tile_bytes = 16384u * a.kchunks;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      tma_prefetch_desc(&iqmap);
      tma_prefetch_desc(&ikmap);
      int item = 0, blk = 0;
      const bool ok = for_my_items(a, [&](int start, int len, int tile) -> bool {
        const int ms = item % kMetaSlots, ib = item & 1;
        if (item >= kMetaSlots && !mbar_wait(&meta_empty[ms], ((item / kMetaSlots) - 1) & 1, a.err, 1)) return false;
        const int t0 = start + tile * a.tq;
        const int qb = (tile * a.tq) >> 7;
        meta[ms] = ItemMeta{start, min(a.tq, len - tile * a.tq), t0, qb, 0, 0, 0, 0};
        mbar_arrive(&meta_full[ms]);
        if (item >= 2 && !mbar_wait(&iq_empty[ib], ((item >> 1) - 1) & 1, a.err, 2)) return false;
        mbar_arrive_expect_tx(&iq_full[ib], tile_bytes);
        for (int c = 0; c < a.kchunks; ++c)
          tma_load_2d(sIQ + ib * 32768 + c * 16384, &iqmap, &iq_full[ib], c * 64, t0 * a.groups);
        for (int b = 0; b <= qb; ++b, ++blk) {
          const int st = blk % kIkStages;
          if (blk >= kIkStages && !mbar_wait(&ik_empty[st], ((blk / kIkStages) - 1) & 1, a.err, 3)) return false;
          mbar_arrive_expect_tx(&ik_full[st], tile_bytes);
          for (int c = 0; c < a.kchunks; ++c)
            tma_load_2d(sIK + st * 32768 + c * 16384, &ikmap, &ik_full[st], c * 64, start + b * 128);
        }
        ++item;
        return true;
      });
      if (ok) {  // end marker for the consumers
        const int ms = item % kMetaSlots;
        if (item < kMetaSlots || mbar_wait(&meta_empty[ms], ((item / kMetaSlots) - 1) & 1, a.err, 4)) {
          meta[ms].done = 1;
          mbar_arrive(&meta_full[ms]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      const uint32_t idesc = idesc_f16(!a.f16, 128, 128, false, false);
      int blk = 0;
      bool ok = true;
      for (int item = 0; ok; ++item) {
        const int ms = item % kMetaSlots, ib = item & 1;
        if (!mbar_wait(&meta_full[ms], (item / kMetaSlots) & 1, a.err, 11)) break;
        const int done = meta[ms].done, qb = meta[ms].qb;
        if (done) break;
        mbar_arrive(&meta_empty[ms]);
        if (!mbar_wait(&iq_full[ib], (item >> 1) & 1, a.err, 12)) break;
        const uint32_t sq = smem_u32(sIQ + ib * 32768);
        for (int b = 0; b <= qb; ++b, ++blk) {
          const int st = blk % kIkStages, ts = blk % kTmStages;
          if (!mbar_wait(&ik_full[st], (blk / kIkStages) & 1, a.err, 13)) { ok = false; break; }
          if (blk >= kTmStages && !mbar_wait(&s_free[ts], ((blk / kTmStages) - 1) & 1, a.err, 14)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sk = smem_u32(sIK + st * 32768);
          for (int ks = 0; ks < 4 * a.kchunks; ++ks) {
            const uint32_t off = (ks >> 2) * 16384 + (ks & 3) * 32;
            umma_ss(tmem + ts * 128, desc_kmajor_sw128(sq + off), desc_kmajor_sw128(sk + off), idesc, ks > 0);
          }
          umma_commit(&s_full[ts]);
          umma_commit(&ik_empty[st]);
        }
        if (ok) umma_commit(&iq_empty[ib]);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue: row maxima
    const int qd = warp & 3;
    const int r = qd * 32 + lane;  // tile row == TMEM lane
    const int tok_local = r / a.groups, g = r - tok_local * a.groups;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const float none = a.neg ? INFINITY : -INFINITY;  // identity of the reduction
    int blk = 0;
    for (int item = 0;; ++item) {
      const int ms = item % kMetaSlots;
      if (!mbar_wait_warp(&meta_full[ms], (item / kMetaSlots) & 1, a.err, 21)) break;
      const ItemMeta m = meta[ms];
      if (m.done) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&meta_empty[ms]);
      const int token = m.t0 + tok_local;
      const bool valid = tok_local < m.n_tokens && token >= a.q_lo && token < a.q_hi;
      const int lim = ((m.t0 - m.seq_start) & 127) + tok_local;  // diagonal block: key c visible iff c <= lim
      float* row = a.scores + ((int64_t)token * a.groups + g) * a.nb;
      float acc[4];
      bool ok = true;
      for (int b = 0; b <= m.qb; ++b, ++blk) {
        const int ts = blk % kTmStages;
        if (!mbar_wait_warp(&s_full[ts], (blk / kTmStages) & 1, a.err, 22)) { ok = false; break; }
        tc_fence_after();
        float red = none;
        const bool diag = b == m.qb;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t v0[32], v1[32];
          tmem_ld32(tmem + ts * 128 + lane_base + half * 64, v0);
          tmem_ld32(tmem + ts * 128 + lane_base + half * 64 + 32, v1);
          tmem_wait_ld();
          if (half == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_free[ts]);
          }
          if (!diag) {
            if (a.neg) {
#pragma unroll
              for (int c = 0; c < 32; ++c) red = fminf(red, fminf(__uint_as_float(v0[c]), __uint_as_float(v1[c])));
            } else {
#pragma unroll
              for (int c = 0; c < 32; ++c) red = fmaxf(red, fmaxf(__uint_as_float(v0[c]), __uint_as_float(v1[c])));
            }
          } else {
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              const float x0 = half * 64 + c <= lim ? __uint_as_float(v0[c]) : none;
              const float x1 = half * 64 + 32 + c <= lim ? __uint_as_float(v1[c]) : none;
              red = a.neg ? fminf(red, fminf(x0, x1)) : fmaxf(red, fmaxf(x0, x1));
            }
          }
        }
        acc[b & 3] = red * (a.neg ? -a.abs_scale : a.abs_scale);
        if ((b & 3) == 3 || diag) {
          for (int k = (b & 3) + 1; k < 4; ++k) acc[k] = -INFINITY;
          if (valid) store_maxima(row, b & ~3, a.nb, acc);
        }
      }
      if (!ok) break;
      if (valid) {  // future / out-of-sequence blocks
        const float ninf[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        for (int cb = (m.qb | 3) + 1; cb < a.nb; cb += 4) store_maxima(row, cb, a.nb, ninf);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// A kernel error word poisons every score with NaN (no-op otherwise).
__global__ void score_poison_kernel(const int* __restrict__ err, int64_t n, float* __restrict__ scores) {
  if (*err == 0) return;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    scores[i] = __int_as_float(0x7fc00000);
}

// Error word of the kernel, one per device (calls on one device that overlap share it).
static __device__ int g_score_err;
constexpr int kMaxDevices = 64;
std::mutex g_err_mu;
int* g_err_addr[kMaxDevices] = {};

}  // namespace
}  // namespace msa

using namespace msa;

extern "C" int msa_index_score_fwd_tc(const void* index_q, const void* index_k, int dtype, const int32_t* cu_seqlens,
                                      int32_t nseq, int64_t total_tokens, int32_t groups, int32_t index_dim,
                                      int32_t num_blocks, int32_t block_size, float scale, int64_t q_lo,
                                      int64_t q_hi, float* scores, void* stream) {
  MSA_CHECK_ARG(dtype == MSA_BF16 || dtype == MSA_F16, "msa_index_score_fwd_tc: bf16/f16 only");
  MSA_CHECK_ARG(index_dim == 64 || index_dim == 128, "msa_index_score_fwd_tc: index_dim must be 64 or 128");
  MSA_CHECK_ARG(block_size == 128, "msa_index_score_fwd_tc: block_size must be 128");
  MSA_CHECK_ARG(groups >= 1 && groups <= 128 && (groups & (groups - 1)) == 0,
                "msa_index_score_fwd_tc: groups must be a power of two <= 128");
  MSA_CHECK_ARG(nseq >= 1 && num_blocks >= 1, "msa_index_score_fwd_tc: bad sizes");
  MSA_CHECK_ARG(total_tokens * groups < ((int64_t)1 << 31), "msa_index_score_fwd_tc: T * G exceeds int32 rows");
  MSA_CHECK_ARG(0 <= q_lo && q_lo <= q_hi && q_hi <= total_tokens, "msa_index_score_fwd_tc: bad query range");
  if (total_tokens == 0 || q_lo == q_hi) return MSA_OK;
  int dev = 0;
  MSA_CUDA_RETURN(cudaGetDevice(&dev));
  MSA_CHECK_ARG(dev >= 0 && dev < kMaxDevices, "msa_index_score_fwd_tc: device ordinal %d out of range", dev);
  int* err = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_err_mu);
    if (!g_err_addr[dev]) {
      void* addr = nullptr;
      MSA_CUDA_RETURN(cudaGetSymbolAddress(&addr, g_score_err));
      g_err_addr[dev] = static_cast<int*>(addr);
    }
    err = g_err_addr[dev];
  }
  CUtensorMap iqmap, ikmap;
  const CUtensorMapDataType dt = tma_dtype(dtype);
  {
    const uint64_t dq[2] = {(uint64_t)index_dim, (uint64_t)(total_tokens * groups)};
    const uint64_t sq[1] = {(uint64_t)index_dim * 2};
    const uint32_t box[2] = {64, 128};
    if (int e = encode_tensor_map(&iqmap, dt, 2, index_q, dq, sq, box, CU_TENSOR_MAP_SWIZZLE_128B)) return e;
    const uint64_t dk[2] = {(uint64_t)index_dim, (uint64_t)total_tokens};
    if (int e = encode_tensor_map(&ikmap, dt, 2, index_k, dk, sq, box, CU_TENSOR_MAP_SWIZZLE_128B)) return e;
  }
  cudaStream_t st = as_stream(stream);
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  MSA_CUDA_RETURN(cudaMemsetAsync(err, 0, sizeof(int), st));
  ScoreArgs sa{cu_seqlens, scores, err, nseq, groups, num_blocks, 128 / groups, index_dim / 64, (int)q_lo, (int)q_hi,
               fabsf(scale), scale < 0.f ? 1 : 0, dtype == MSA_F16 ? 1 : 0};
  MSA_CUDA_RETURN(cudaFuncSetAttribute(score_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemScore));
  score_tc_kernel<<<sms, kScoreThreads, kSmemScore, st>>>(iqmap, ikmap, sa);
  score_poison_kernel<<<sms * 4, 256, 0, st>>>(err, (q_hi - q_lo) * groups * (int64_t)num_blocks,
                                               scores + q_lo * groups * (int64_t)num_blocks);
  count_launches(2);
  return launch_status("index_score_fwd_tc");
}
