// Top-k block selection: one warp per (token, group) row.
//
// Semantics of triton/topk.py:11-47 / eager/ops.py:94-129: future blocks rank
// -inf, the local_blocks most recent causal blocks rank +inf, the top
// min(K, NB) are kept in descending rank, -inf picks become -1, tail -1.
// Equal ranks are ordered by ascending block id (torch.topk leaves this open).
//
// Each candidate is a 64-bit key: order-preserving float bits of its rank in
// the high word (the "rank word") and the complemented block id in the low
// word, so one unsigned max both ranks and breaks ties. A lane holds the rank
// words of blocks lane, lane + 32, ... in registers (the block id is the
// register's position); no temporaries touch global memory: the only traffic is
// reading the causal part of the scores row and writing K ids.
//
// Threshold path (K <= 48): bisect the rank-word range with warp-wide counts
// (redux.sync) until between K and kCap (32 or 64) keys lie at or above the
// threshold, gather those keys through 512 bytes of shared memory into one or
// two per lane and bitonic-sort them across the warp; the first K are the
// answer. A row whose K-th key shares its rank word with so many others that no
// threshold leaves at most kCap keys (long runs of equal scores), a row that
// must pad with keys ranked below -inf, and every row of a larger K take the
// round path: K rounds of a lane-local max plus a warp max, retiring the
// winner. Both paths emit the same K keys in the same order.
#include <type_traits>

#include "common.cuh"

namespace msa {
namespace {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ uint32_t ordered_bits(float x) {
  uint32_t u = __float_as_uint(x);
  if (u == 0x80000000u) u = 0u;  // -0.0 ties with +0.0
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ uint64_t make_key(uint32_t rank, int b) {
  return ((uint64_t)rank << 32) | (uint32_t)(~(uint32_t)b);
}

constexpr uint64_t kRetired = 0ull;  // below every real key (its low word ~b is never 0)

// Round path: K rounds of max + retire over all of the row's keys. Keys are
// rebuilt from the rank words each round; a bit per register marks retired ones
// (the winner's block id names its lane and register directly).
template <int kPerLane>
__device__ __forceinline__ void select_rounds(const uint32_t (&rank)[kPerLane], int nb, int lane, int k, int count,
                                              uint32_t neg_inf, int32_t* __restrict__ dst) {
  using Mask = typename std::conditional<(kPerLane > 32), uint64_t, uint32_t>::type;
  Mask live = 0;
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) live |= (Mask)(lane + 32 * i < nb) << i;
  for (int r = 0; r < count; ++r) {
    uint64_t best = kRetired;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
      const uint64_t key = (live >> i) & 1 ? make_key(rank[i], lane + 32 * i) : kRetired;
      best = key > best ? key : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t other = __shfl_xor_sync(kFull, best, o);
      best = other > best ? other : best;
    }
    const uint32_t b = ~(uint32_t)(best & 0xffffffffu);
    const bool is_neg_inf = (uint32_t)(best >> 32) == neg_inf;
    if (lane == 0) dst[r] = is_neg_inf ? -1 : (int32_t)b;
    if (is_neg_inf) {  // everything left ranks -inf as well
      for (int rr = r + 1 + lane; rr < k; rr += 32) dst[rr] = -1;
      return;
    }
    if ((int)(b & 31) == lane) live &= ~((Mask)1 << (b >> 5));
  }
  for (int rr = count + lane; rr < k; rr += 32) dst[rr] = -1;
}

// The float whose order-preserving bits are u (inverse of ordered_bits).
__device__ __forceinline__ float from_ordered(uint32_t u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

// One compare-exchange step of a descending bitonic sort over kCap keys laid out
// as element e = 32 * r + lane (r = register): partner e ^ j, j < 32.
template <typename Key>
__device__ __forceinline__ Key bitonic_step(Key x, int e, int j, int k) {
  const Key y = __shfl_xor_sync(kFull, x, j);
  const bool take_max = ((e & j) == 0) == ((e & k) == 0);
  return take_max ? (x > y ? x : y) : (x < y ? x : y);
}

// Descending bitonic sort of kCap (32 or 64) keys: element lane in x0, lane + 32 in x1.
template <int kCap, typename Key>
__device__ __forceinline__ void bitonic_sort(Key& x0, Key& x1, int lane) {
#pragma unroll
  for (int kk = 2; kk <= kCap; kk <<= 1) {
#pragma unroll
    for (int j = kk >> 1; j > 0; j >>= 1) {
      if (j == 32) {  // kk = 64: partners sit in the two registers of one lane
        const Key a = x0 > x1 ? x0 : x1, b = x0 > x1 ? x1 : x0;
        x0 = a;
        x1 = b;
      } else {
        x0 = bitonic_step(x0, lane, j, kk);
        if constexpr (kCap == 64) x1 = bitonic_step(x1, lane + 32, j, kk);
      }
    }
  }
}

// Output position p: local block p (p < n_l), the (p - n_l)-th sorted free key
// (p - n_l < need), or -1.
template <int kCap, typename Key, typename Decode>
__device__ __forceinline__ void emit_sorted(Key x0, Key x1, int lane, int n_l, int need, int count, int qb,
                                            int32_t* __restrict__ dst, Decode decode) {
#pragma unroll
  for (int half = 0; half < (kCap == 64 ? 2 : 1); ++half) {
    const int p = lane + 32 * half;
    const int j = p - n_l;  // rank among the free keys
    const Key a = __shfl_sync(kFull, x0, j & 31);
    Key key = a;
    if constexpr (kCap == 64) {
      const Key b = __shfl_sync(kFull, x1, j & 31);
      key = j >= 32 ? b : a;
    }
    const int32_t id = p < n_l ? qb - n_l + 1 + p : j < need ? decode(key) : -1;
    if (p < count) dst[p] = id;
  }
}

// Rank words of the whole row with the reference's ranking (future -inf,
// forced local +inf, 0 past the row). All loads are issued before any is used,
// from addresses clamped into the causal part of the row (future positions
// re-read the row's last causal score, a line already being fetched): no branch
// separates them.
template <int kPerLane>
__device__ __forceinline__ void load_ranks(uint32_t (&rank)[kPerLane], const float* __restrict__ src, int lane,
                                           int nb, int qb, int local, uint32_t neg_inf, uint32_t pos_inf) {
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) rank[i] = __float_as_uint(__ldg(src + min(lane + 32 * i, qb)));
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) {
    const int b = lane + 32 * i;
    const uint32_t r = ordered_bits(__uint_as_float(rank[i]));
    rank[i] = b >= nb ? 0u : b > qb ? neg_inf : (local > 0 && b > qb - local) ? pos_inf : r;
  }
}

// The round path for one row from scratch, out of line: the threshold path
// calls it only for rows it cannot take, and its registers stay out of the
// threshold path's allocation.
template <int kPerLane>
__device__ __noinline__ void rounds_row(const float* __restrict__ src, int lane, int nb, int qb, int local, int k,
                                        int count, uint32_t neg_inf, uint32_t pos_inf, int32_t* __restrict__ dst) {
  uint32_t rank[kPerLane];
  load_ranks(rank, src, lane, nb, qb, local, neg_inf, pos_inf);
  select_rounds(rank, nb, lane, k, count, neg_inf, dst);
}

// kCap = 0: round path only (K > 48). kCap = 32 (K <= 16) or 64 (K <= 48):
// threshold path with the round path as the per-row fallback. Threshold
// variants of up to 1024 blocks fit 64 registers without spills: four CTAs
// (32 warps) per SM.
//
// The threshold path splits the row the way the ranking does: the n_l forced
// local blocks rank +inf and come first (equal ranks: ascending id), future
// blocks rank -inf and only ever become -1, so when every remaining causal
// score ("free" blocks, b <= qb - local) is finite the answer is the local
// blocks, then the best `need` free blocks in descending order, then -1. Only
// the free blocks are searched and sorted.
template <int kPerLane, int kCap>
__global__ void __launch_bounds__(256, (kPerLane <= 16 && kCap > 0) ? 4 : (kPerLane <= 32 && kCap > 0) ? 3 : 1)
    topk_kernel(const float* __restrict__ scores, const int32_t* __restrict__ cu, const int32_t* __restrict__ positions,
                int nseq, int64_t rows, int groups, int nb, int block, int k, int local, int32_t* __restrict__ out) {
  constexpr int kWarps = 8;
  __shared__ float stage_val[kWarps][kCap > 0 ? kCap : 1];
  __shared__ int32_t stage_blk[kWarps][kCap > 0 ? kCap : 1];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarps + warp;
  if (row >= rows) return;
  const int64_t t = rows <= INT32_MAX ? (int64_t)((uint32_t)row / (uint32_t)groups) : row / groups;
  // the query's block: from its position in its sequence (cu_seqlens), or given directly (decode)
  const int qb = positions != nullptr ? (int)((uint32_t)positions[t] / (uint32_t)block)
                                      : (int)((uint32_t)(t - cu[find_sequence(cu, nseq, t)]) / (uint32_t)block);
  const float* src = scores + row * nb;
  const uint32_t neg_inf = ordered_bits(-INFINITY), pos_inf = ordered_bits(INFINITY);
  const int count = min(k, nb);
  int32_t* dst = out + row * k;
  if constexpr (kCap == 0) {
    uint32_t rank[kPerLane];
    load_ranks(rank, src, lane, nb, qb, local, neg_inf, pos_inf);
    select_rounds(rank, nb, lane, k, count, neg_inf, dst);
  } else {
    const int free_end = qb - local;  // free blocks: [0, free_end]
    const int n_free = max(free_end + 1, 0);
    const int n_l = min(local, qb + 1);  // local blocks: [qb - n_l + 1, qb]
    const int need = min(max(count - n_l, 0), n_free);
    // Free scores (-inf elsewhere: below every finite score), their range, and
    // whether any free score is infinite or NaN. The threshold search runs on
    // rank words but counts with float compares: for finite scores both orders
    // agree (-0.0 and +0.0 tie in both), so only the range ends and the
    // candidates are ever converted.
    float f[kPerLane];
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) f[i] = __ldg(src + min(lane + 32 * i, qb));
    float f_lo = INFINITY, f_hi = -INFINITY;
    bool bad = false;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
      const bool is_free = lane + 32 * i <= free_end;
      bad |= is_free && !(fabsf(f[i]) < INFINITY);
      f[i] = is_free ? f[i] : -INFINITY;
      f_hi = fmaxf(f_hi, f[i]);
      f_lo = is_free ? fminf(f_lo, f[i]) : f_lo;
    }
    if (__any_sync(kFull, bad)) {  // non-finite free scores: the reference ranking, round path
      rounds_row<kPerLane>(src, lane, nb, qb, local, k, count, neg_inf, pos_inf, dst);
      return;
    }
    if (need == 0) {  // local blocks only (n_l <= count <= k), then -1
      for (int rr = lane; rr < k; rr += 32) dst[rr] = rr < n_l ? qb - n_l + 1 + rr : -1;
      return;
    }
    auto count_ge = [&](float x) {  // this lane's free scores >= x
      uint32_t c0 = 0, c1 = 0, c2 = 0, c3 = 0;  // four partial counts: short add chains
#pragma unroll
      for (int i = 0; i < kPerLane; i += 4) {
        c0 += f[i] >= x;
        if (i + 1 < kPerLane) c1 += f[i + 1] >= x;
        if (i + 2 < kPerLane) c2 += f[i + 2] >= x;
        if (i + 3 < kPerLane) c3 += f[i + 3] >= x;
      }
      return (c0 + c1) + (c2 + c3);
    };
    // Invariant: c(lo) >= need > c(hi), c(x) = #free keys with rank word >= x.
    // lo and hi stay inside the finite rank words, so every probe decodes to a
    // finite float.
    uint32_t lo = __reduce_min_sync(kFull, ordered_bits(f_lo));
    const uint32_t top = __reduce_max_sync(kFull, ordered_bits(f_hi));
    uint32_t hi = top + 1;
    uint32_t c_lo = n_free;
    uint32_t mine = count_ge(from_ordered(lo));  // this lane's share of c(lo)
    while (c_lo > (uint32_t)kCap) {
      if (hi - lo <= 1) {  // the need-th rank word is shared by more than kCap - need others
        rounds_row<kPerLane>(src, lane, nb, qb, local, k, count, neg_inf, pos_inf, dst);
        return;
      }
      const uint32_t mid = lo + ((hi - lo) >> 1);
      const uint32_t m = count_ge(from_ordered(mid));
      const uint32_t c = __reduce_add_sync(kFull, m);
      if ((int)c >= need) {
        lo = mid;
        c_lo = c;
        mine = m;
      } else {
        hi = mid;
      }
    }
    const float thr = from_ordered(lo);
    // Gather the candidates (score, block id): exclusive prefix of the per-lane
    // counts gives each lane its first slot in the warp's shared-memory stage.
    uint32_t incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += y;
    }
    float* sval = stage_val[warp];
    int32_t* sblk = stage_blk[warp];
    uint32_t pos = incl - mine;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
      if (f[i] >= thr) {
        sval[pos] = f[i];
        sblk[pos] = lane + 32 * i;
        ++pos;
      }
    }
    __syncwarp();
    // Sort keys. When the candidates' rank words span fewer than 2^(32 - bbits)
    // values (bbits = bits of a block id), a 32-bit key (rank word - thr + 1,
    // complemented block id) orders them as the 64-bit key does; padding is 0,
    // below every real key.
    const int bbits = nb > 1 ? 32 - __clz(nb - 1) : 0;
    const uint32_t bmask = (uint32_t)((1ull << bbits) - 1);
    const bool packed = (uint64_t)(top - lo) + 1 < (1ull << (32 - bbits));
    const int n_c = (int)c_lo;
    if (packed) {
      auto key_of = [&](int e) -> uint32_t {
        if (e >= n_c) return 0u;
        return ((ordered_bits(sval[e]) - lo + 1) << bbits) | (~(uint32_t)sblk[e] & bmask);
      };
      uint32_t x0 = key_of(lane), x1 = kCap == 64 ? key_of(lane + 32) : 0u;
      bitonic_sort<kCap>(x0, x1, lane);
      emit_sorted<kCap>(x0, x1, lane, n_l, need, count, qb, dst,
                        [&](uint32_t key) { return (int32_t)(~key & bmask); });
    } else {
      auto key_of = [&](int e) -> uint64_t {
        if (e >= n_c) return kRetired;
        return make_key(ordered_bits(sval[e]), sblk[e]);
      };
      uint64_t x0 = key_of(lane), x1 = kCap == 64 ? key_of(lane + 32) : kRetired;
      bitonic_sort<kCap>(x0, x1, lane);
      emit_sorted<kCap>(x0, x1, lane, n_l, need, count, qb, dst,
                        [&](uint64_t key) { return (int32_t)~(uint32_t)(key & 0xffffffffu); });
    }
    for (int rr = count + lane; rr < k; rr += 32) dst[rr] = -1;
  }
}

}  // namespace
}  // namespace msa

using namespace msa;

static int topk_launch(const float* scores, const int32_t* cu_seqlens, const int32_t* positions, int32_t nseq,
                       int64_t total_tokens, int32_t groups, int32_t num_blocks, int32_t block_size,
                       int32_t topk_blocks, int32_t local_blocks, int32_t* indices, void* stream) {
  MSA_CHECK_ARG(nseq >= 1 && groups >= 1 && num_blocks >= 1 && block_size >= 1, "msa_topk: bad sizes");
  MSA_CHECK_ARG(topk_blocks >= 0 && local_blocks >= 0 && local_blocks <= topk_blocks, "msa_topk: bad K/local");
  MSA_CHECK_ARG(num_blocks <= 32 * 64, "msa_topk: more than 2048 blocks per row unsupported");
  const int64_t rows = total_tokens * groups;
  if (rows == 0 || topk_blocks == 0) return MSA_OK;
  constexpr int kWarps = 8;
  const unsigned grid = ceil_div(rows, kWarps);
  cudaStream_t st = as_stream(stream);
  const int count = topk_blocks < num_blocks ? topk_blocks : num_blocks;
#define MSA_TOPK_LAUNCH(P, C)                                                                      \
  topk_kernel<P, C><<<grid, kWarps * 32, 0, st>>>(scores, cu_seqlens, positions, nseq, rows, groups, \
                                                  num_blocks, block_size, topk_blocks, local_blocks, indices)
#define MSA_TOPK_CAP(P)                               \
  do {                                                \
    if (count <= 16) MSA_TOPK_LAUNCH(P, 32);          \
    else if (count <= 48) MSA_TOPK_LAUNCH(P, 64);     \
    else MSA_TOPK_LAUNCH(P, 0);                       \
  } while (0)
  if (num_blocks <= 32) MSA_TOPK_CAP(1);
  else if (num_blocks <= 64) MSA_TOPK_CAP(2);
  else if (num_blocks <= 128) MSA_TOPK_CAP(4);
  else if (num_blocks <= 256) MSA_TOPK_CAP(8);
  else if (num_blocks <= 512) MSA_TOPK_CAP(16);
  else if (num_blocks <= 1024) MSA_TOPK_CAP(32);
  else MSA_TOPK_CAP(64);
#undef MSA_TOPK_CAP
#undef MSA_TOPK_LAUNCH
  count_launches(1);
  return launch_status("topk");
}

extern "C" int msa_topk(const float* scores, const int32_t* cu_seqlens, int32_t nseq, int64_t total_tokens,
                        int32_t groups, int32_t num_blocks, int32_t block_size, int32_t topk_blocks,
                        int32_t local_blocks, int32_t* indices, void* stream) {
  return topk_launch(scores, cu_seqlens, nullptr, nseq, total_tokens, groups, num_blocks, block_size, topk_blocks,
                     local_blocks, indices, stream);
}

extern "C" int msa_topk_positions(const float* scores, const int32_t* positions, int64_t total_tokens, int32_t groups,
                                  int32_t num_blocks, int32_t block_size, int32_t topk_blocks, int32_t local_blocks,
                                  int32_t* indices, void* stream) {
  return topk_launch(scores, nullptr, positions, 1, total_tokens, groups, num_blocks, block_size, topk_blocks,
                     local_blocks, indices, stream);
}
