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
// 128) two blocks at a time: TMA loads the 256 x Di rows of index_k of blocks
// 2p and 2p + 1, a thread issues S = IQ . IK^T (M = 128, N = 256) into one of
// two 256-column TMEM stages, and two epilogue warpgroups (thread = tile row;
// warpgroup e owns stage e) read S back with tcgen05.ld and take each block's
// row maximum (diagonal block: keys up to the token only). A thread issuing
// MMAs and barrier waits is latency-bound (each barrier poll, MMA and commit
// costs on the order of 100 cycles), so the pairs halve that cost per block and
// two issuing threads (even / odd pairs, one per TMEM stage) run two such
// chains at once. Items are dealt to CTAs round-robin, each sequence's tiles
// last-first (the longest causal rows first).
#include <mutex>

#include "attn_common.cuh"

namespace msa {
namespace {

using namespace tc;
using namespace attn;

constexpr int kScoreThreads = 384;  // warp 0 producer, warps 1-2 MMA issuers, warps 4-11 epilogue (two warpgroups)
constexpr int kIkStagesMax = 6;  // index_k ring of key-block pairs: 6 at Di = 64, 2 at 128
constexpr int kTmStages = 2;     // TMEM: two stages of 256 columns (one per epilogue warpgroup)
constexpr int kMetaSlots = 4;
constexpr int kSmemScoreMax = 232448 - 2048;  // the opt-in maximum less static shared memory and its slack

// Dynamic shared memory of a ring of `stages` index_k block pairs (+ 2 index_q tiles, + alignment).
constexpr int score_smem(int tile_bytes, int stages) { return (2 + 2 * stages) * tile_bytes + 1024; }

struct ItemMeta {
  int32_t seq_start, n_tokens, t0, qb;  // sequence start, tokens in the tile, first token, diagonal block
  int32_t done, pad0, pad1, pad2;
};

struct ScoreArgs {
  const int32_t* cu;
  float* scores;
  int* err;
  // winner state (the kState kernel): per (token, group, block) the winning key's
  // offset + 1, or kFixup where another key comes within the float32 error margin
  int32_t* tie_info;
  const float* qnorm;     // [T*G] |index_q row|
  const unsigned* kmax;   // max |index_k row| (float bits)
  int nseq, groups, nb, tq, kchunks;  // tq = 128 / G tokens per tile, kchunks = Di / 64
  int q_lo, q_hi;                     // query tokens scored: [q_lo, q_hi)
  float abs_scale;
  int neg;  // 1: negative scale (the maximum of scale * dot is scale * the minimum dot)
  int f16;
  int nst;  // index_k ring stages, each a pair of key blocks (<= kIkStagesMax)
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

constexpr int32_t kFixup = INT32_MIN;  // winner state to be decided in float64

__device__ __forceinline__ void store_info(int32_t* row, int cb, int nb, const int32_t (&v)[4]) {
  if ((nb & 3) == 0) {
    *reinterpret_cast<int4*>(row + cb) = make_int4(v[0], v[1], v[2], v[3]);
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (cb + k < nb) row[cb + k] = v[k];
  }
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

// Three-input maximum / minimum (one sm_100 instruction; like fmaxf / fminf, a
// NaN input is ignored unless all are NaN).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float min3f(float a, float b, float c) {
  float r;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// One level of a three-way reduction tree: N values to ceil(N / 3).
template <bool kNeg, int N>
__device__ __forceinline__ void reduce3_level(float* t) {
#pragma unroll
  for (int i = 0; i < N / 3; ++i)
    t[i] = kNeg ? min3f(t[3 * i], t[3 * i + 1], t[3 * i + 2]) : max3f(t[3 * i], t[3 * i + 1], t[3 * i + 2]);
  if constexpr (N % 3 == 2)
    t[N / 3] = kNeg ? fminf(t[N - 2], t[N - 1]) : fmaxf(t[N - 2], t[N - 1]);
  else if constexpr (N % 3 == 1)
    t[N / 3] = t[N - 1];
}

// Row reductions over one 128-column tile row held in registers (v[q][c] =
// column 32q + c). kDiag: only columns <= lim are visible. kNeg: the scale is
// negative, so the public maximum is scale * the minimum dot.
//
// Maximum (minimum) as a tree of three-input operations (128 -> 43 -> 15 -> 5
// -> 2 -> 1, 65 instructions), each level independent of itself.
template <bool kNeg, bool kDiag>
__device__ __forceinline__ float row_extreme(const uint32_t (&v)[4][32], int lim) {
  const float none = kNeg ? INFINITY : -INFINITY;
  float t[128];
#pragma unroll
  for (int col = 0; col < 128; ++col)
    t[col] = (!kDiag || col <= lim) ? __uint_as_float(v[col >> 5][col & 31]) : none;
  reduce3_level<kNeg, 128>(t);
  reduce3_level<kNeg, 43>(t);
  reduce3_level<kNeg, 15>(t);
  reduce3_level<kNeg, 5>(t);
  return kNeg ? fminf(t[0], t[1]) : fmaxf(t[0], t[1]);
}

struct WinnerState {
  float best, second;  // largest signed dot and the largest of the others
  int arg;             // column of `best` (meaningful when it is unique)
};

// Best signed dot, runner-up and argmax over the visible columns, as eight
// independent streams of 16 columns merged at the end (the same best and
// runner-up as one pass in any order; NaN dots are skipped as in one pass).
template <bool kNeg, bool kDiag>
__device__ __forceinline__ WinnerState row_winner(const uint32_t (&v)[4][32], int lim) {
  float best[8], second[8];
  int arg[8];
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    best[s] = -INFINITY;
    second[s] = -INFINITY;
    arg[s] = 0;
  }
#pragma unroll
  for (int c = 0; c < 16; ++c) {
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      const int col = s * 16 + c;
      const float x = __uint_as_float(v[col >> 5][col & 31]);
      const float sd = (!kDiag || col <= lim) ? (kNeg ? -x : x) : -INFINITY;
      const bool gt = sd > best[s];
      second[s] = gt ? best[s] : fmaxf(second[s], sd);
      arg[s] = gt ? col : arg[s];
      best[s] = gt ? sd : best[s];
    }
  }
  WinnerState w{best[0], second[0], arg[0]};
#pragma unroll
  for (int s = 1; s < 8; ++s) {
    const bool gt = best[s] > w.best;
    w.second = gt ? fmaxf(w.best, second[s]) : fmaxf(w.second, best[s]);
    w.arg = gt ? arg[s] : w.arg;
    w.best = gt ? best[s] : w.best;
  }
  return w;
}

// kState: also the winner state of every causal block (tie_info), for the
// backward. The winner of a block is the key with the largest signed dot; it is
// taken from the float32 values when no other visible key comes within
// `margin` of it (twice a bound on the float32 accumulation error of one dot,
// Di * 2^-22 * |q| * max|k|, four times the bound the tests check), so it is
// the float64 winner too; otherwise the entry is left to the float64 fixup.
template <bool kState>
__global__ void __launch_bounds__(kScoreThreads, 1)
score_tc_kernel(const __grid_constant__ CUtensorMap iqmap, const __grid_constant__ CUtensorMap ikmap, ScoreArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const uint32_t tile_bytes = 16384u * a.kchunks;
  uint8_t* sIQ = smem;                   // 2 tiles x (Di/64 chunks x 128 rows x 128 B)
  uint8_t* sIK = smem + 2 * tile_bytes;  // a.nst stages x (Di/64 chunks x 256 rows (2 blocks) x 128 B)
  const uint32_t pair_bytes = 2 * tile_bytes;
  __shared__ ItemMeta meta[kMetaSlots];
  __shared__ uint64_t meta_full[kMetaSlots], meta_empty[kMetaSlots], iq_full[2], iq_empty[2];
  __shared__ uint64_t ik_full[kIkStagesMax], ik_empty[kIkStagesMax], s_full[kTmStages], s_free[kTmStages];
  __shared__ uint32_t tmem_base;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int j = 0; j < kMetaSlots; ++j) {
      mbar_init(&meta_full[j], 1);
      mbar_init(&meta_empty[j], 10);  // 2 MMA issuers + 8 epilogue warps
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&iq_full[j], 1);
      mbar_init(&iq_empty[j], 2);  // both MMA issuers
    }
    for (int j = 0; j < a.nst; ++j) {
      mbar_init(&ik_full[j], 1);
      mbar_init(&ik_empty[j], 1);
    }
    for (int j = 0; j < kTmStages; ++j) {
      mbar_init(&s_full[j], 1);
      mbar_init(&s_free[j], 4);  // the 4 warps of the stage's warpgroup
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
  const int nst = a.nst;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      tma_prefetch_desc(&iqmap);
      tma_prefetch_desc(&ikmap);
      int item = 0, pc = 0;  // pc: key-block pairs so far
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
          tma_load_2d(sIQ + ib * tile_bytes + c * 16384, &iqmap, &iq_full[ib], c * 64, t0 * a.groups);
        // key blocks in pairs (2p, 2p + 1); an odd count repeats block qb as the
        // second of the last pair (its scores are never read)
        for (int b = 0; b <= qb; b += 2, ++pc) {
          const int st = pc % nst;
          if (pc >= nst && !mbar_wait(&ik_empty[st], ((pc / nst) - 1) & 1, a.err, 3)) return false;
          mbar_arrive_expect_tx(&ik_full[st], pair_bytes);
          for (int j = 0; j < 2; ++j)
            for (int c = 0; c < a.kchunks; ++c)
              tma_load_2d(sIK + st * pair_bytes + c * 32768 + j * 16384, &ikmap, &ik_full[st], c * 64,
                          start + min(b + j, qb) * 128);
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
  } else if (warp == 1 || warp == 2) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuers
      // Issuer u (warp 1 + u) takes the pairs pc with pc % 2 == u: its own ring
      // stages (nst is even) and TMEM stage u, so the two latency chains of
      // barrier polls, MMA issue and commits run side by side. Both wait for every
      // item's index_q tile and both release it (iq_empty counts two).
      const int u = warp - 1;
      const uint32_t idesc = idesc_f16(!a.f16, 128, 256, false, false);  // N = 256: two key blocks
      int pc = 0;
      bool ok = true;
      for (int item = 0; ok; ++item) {
        const int ms = item % kMetaSlots, ib = item & 1;
        if (!mbar_wait(&meta_full[ms], (item / kMetaSlots) & 1, a.err, 11)) break;
        const int done = meta[ms].done, qb = meta[ms].qb;
        if (done) break;
        mbar_arrive(&meta_empty[ms]);
        if (!mbar_wait(&iq_full[ib], (item >> 1) & 1, a.err, 12)) break;
        const uint32_t sq = smem_u32(sIQ + ib * tile_bytes);
        for (int b = 0; b <= qb; b += 2, ++pc) {
          const int st = pc % nst, ts = pc & 1;
          if (ts != u) continue;
          if (!mbar_wait(&ik_full[st], (pc / nst) & 1, a.err, 13)) { ok = false; break; }
          if (pc >= kTmStages && !mbar_wait(&s_free[ts], ((pc >> 1) - 1) & 1, a.err, 14)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sk = smem_u32(sIK + st * pair_bytes);
          for (int ks = 0; ks < 4 * a.kchunks; ++ks) {
            const uint32_t col = (ks & 3) * 32;
            umma_ss(tmem + ts * 256, desc_kmajor_sw128(sq + (ks >> 2) * 16384 + col),
                    desc_kmajor_sw128(sk + (ks >> 2) * 32768 + col), idesc, ks > 0);
          }
          umma_commit(&s_full[ts]);
          umma_commit(&ik_empty[st]);
        }
        if (ok) umma_commit(&iq_empty[ib]);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue: row maxima
    // Two warpgroups: warpgroup e (warps 4-7: e = 0, warps 8-11: e = 1) owns TMEM
    // stage e, i.e. every other key-block pair, so each stage is read in order by
    // one warpgroup while the other reduces; each block's maximum goes out as one
    // 4-byte store.
    const int qd = warp & 3;
    const int e = (warp - 4) >> 2;
    const int r = qd * 32 + lane;  // tile row == TMEM lane
    const int tok_local = r / a.groups, g = r - tok_local * a.groups;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    int pc = 0;
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
      int32_t* row_info = kState ? a.tie_info + ((int64_t)token * a.groups + g) * a.nb : nullptr;
      float margin = 0.f;
      if (kState && valid)
        margin = 2.f * (float)(a.kchunks * 64) * 2.384185791015625e-07f *  // Di * 2^-22
                 a.qnorm[(int64_t)token * a.groups + g] * __uint_as_float(*a.kmax);
      // block b's row maximum (and winner state) from its 128 columns v
      auto reduce_block = [&](int b, const uint32_t (&v)[4][32]) {
        const bool diag = b == m.qb;
        float red;
        if (kState) {
          WinnerState w;
          if (diag) w = a.neg ? row_winner<true, true>(v, lim) : row_winner<false, true>(v, lim);
          else w = a.neg ? row_winner<true, false>(v, lim) : row_winner<false, false>(v, lim);
          red = a.neg ? -w.best : w.best;
          if (valid) row_info[b] = w.best - w.second > margin ? w.arg + 1 : kFixup;
        } else {
          if (diag) red = a.neg ? row_extreme<true, true>(v, lim) : row_extreme<false, true>(v, lim);
          else red = a.neg ? row_extreme<true, false>(v, lim) : row_extreme<false, false>(v, lim);
        }
        if (valid) row[b] = red * (a.neg ? -a.abs_scale : a.abs_scale);
      };
      bool ok = true;
      for (int bb = 0; bb <= m.qb; bb += 2, ++pc) {
        const int ts = pc & 1;
        if (ts != e) continue;  // the other warpgroup's pair
        if (!mbar_wait_warp(&s_full[ts], (pc >> 1) & 1, a.err, 22)) { ok = false; break; }
        tc_fence_after();
        const bool two = bb + 1 <= m.qb;  // else the pair's second block repeats the diagonal
        uint32_t v[4][32];
#pragma unroll
        for (int q = 0; q < 4; ++q) tmem_ld32(tmem + ts * 256 + lane_base + q * 32, v[q]);
        tmem_wait_ld();
        if (!two) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s_free[ts]);
        }
        reduce_block(bb, v);
        if (two) {
#pragma unroll
          for (int q = 0; q < 4; ++q) tmem_ld32(tmem + ts * 256 + 128 + lane_base + q * 32, v[q]);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s_free[ts]);
          reduce_block(bb + 1, v);
        }
      }
      if (!ok) break;
      if (valid) {  // future / out-of-sequence blocks: the rest of the diagonal's group of four
        // by warpgroup 0, then groups of four split between the warpgroups
        const float ninf[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        const int32_t zero4[4] = {0, 0, 0, 0};
        if (e == 0) {
          for (int cb = m.qb + 1; cb <= (m.qb | 3) && cb < a.nb; ++cb) {
            row[cb] = -INFINITY;
            if (kState) row_info[cb] = 0;
          }
        }
        for (int cb = (m.qb | 3) + 1 + 4 * e; cb < a.nb; cb += 8) {
          store_maxima(row, cb, a.nb, ninf);
          if (kState) store_info(row_info, cb, a.nb, zero4);
        }
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

// |index_q row| for every (token, group) row and max |index_k row| (float bits,
// atomicMax); float64 sums rounded up so the margins built on them are bounds.
__global__ void score_norms_kernel(const void* __restrict__ iq, const void* __restrict__ ik, int dtype,
                                   int64_t qrows, int64_t krows, int dim, float* __restrict__ qnorm,
                                   unsigned* __restrict__ kmax) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < qrows + krows; r += warps) {
    const bool is_q = r < qrows;
    const void* base = is_q ? iq : ik;
    const int64_t row = is_q ? r : r - qrows;
    double sq = 0.0;
    for (int d = lane; d < dim; d += 32) {
      const double x = load_f64(base, row * dim + d, dtype);
      sq += x * x;
    }
    sq = warp_sum(sq);
    if (lane == 0) {
      const float n = (float)(sqrt(sq) * 1.0000001) * 1.0001f;
      if (is_q) qnorm[row] = n; else atomicMax(kmax, __float_as_uint(n));
    }
  }
}

// float64 dot products q . k_j of the 4 keys j = j0 + 32 i (-inf past token t), each
// summed in order d = 0 .. dim-1 with separately rounded products and sums: the same
// bits as dot_f64 (the backward's tie test compares them for equality). The key rows
// are read 32 elements at a time, four 16-byte loads per key issued together, instead
// of one dependent 2-byte load per element.
__device__ __forceinline__ void fixup_dots(const double* __restrict__ q, const void* __restrict__ ik, int dtype,
                                           int dim, int64_t j0, int64_t t, double (&v)[4]) {
  double acc[4] = {0.0, 0.0, 0.0, 0.0};
  const uint16_t* base = static_cast<const uint16_t*>(ik);
  for (int c0 = 0; c0 < dim; c0 += 32) {
    uint4 raw[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t j = j0 + 32 * i;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc)
        raw[i][cc] = j <= t ? *reinterpret_cast<const uint4*>(base + j * dim + c0 + cc * 8) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const double qd = q[c0 + cc * 8 + e];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t w = (&raw[i][cc].x)[e >> 1];
          const uint16_t hbits = (e & 1) ? (uint16_t)(w >> 16) : (uint16_t)(w & 0xffffu);
          const float f = dtype == MSA_BF16 ? __uint_as_float((uint32_t)hbits << 16)
                                            : __half2float(__ushort_as_half(hbits));
          acc[i] = __dadd_rn(acc[i], __dmul_rn(qd, (double)f));
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = j0 + 32 * i <= t ? acc[i] : -INFINITY;
}

// Entries the tensor-core epilogue left undecided (kFixup): the block's float64
// scores scale * q . k_j (the precise kernel's dot order), their maximum into
// max_val and the winner state into tie_info: winner offset + 1 when one key
// attains it, else -(number of tied keys). One warp per (token, group) row.
__global__ void score_fixup_kernel(const void* __restrict__ iq, const void* __restrict__ ik, int dtype,
                                   const int32_t* __restrict__ cu, int nseq, int64_t rows, int groups, int dim,
                                   int nb, double scale, int32_t* __restrict__ tie_info,
                                   double* __restrict__ max_val) {
  extern __shared__ double qsm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  double* q = qsm + (size_t)warp * dim;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < rows; row += warps) {
    const int64_t t = row / groups;
    bool loaded = false;
    int64_t start = 0;
    for (int b00 = 0; b00 < nb; b00 += 256) {
      // the row's winner state, 8 chunks of 32 blocks loaded together, then its marked entries
      unsigned marks[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int b = b00 + 32 * c + lane;
        marks[c] = b < nb && tie_info[row * nb + b] == kFixup;
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) marks[c] = __ballot_sync(0xffffffffu, marks[c] != 0u);
      for (int c = 0; c < 8; ++c) {
        unsigned mask = marks[c];
        if (mask && !loaded) {
          start = cu[find_sequence(cu, nseq, t)];
          for (int d = lane; d < dim; d += 32) q[d] = load_f64(iq, row * dim + d, dtype);
          __syncwarp();
          loaded = true;
        }
        while (mask) {
          const int bb = b00 + 32 * c + __ffs(mask) - 1;
          mask &= mask - 1;
          double v[4];
          double m = -INFINITY;
          fixup_dots(q, ik, dtype, dim, start + (int64_t)bb * 128 + lane, t, v);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            v[i] = v[i] == -INFINITY ? v[i] : __dmul_rn(scale, v[i]);
            m = fmax(m, v[i]);
          }
          m = warp_max(m);
          int cnt = 0, off = 0;
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (v[i] == m) {
              ++cnt;
              off = lane + 32 * i;
            }
          const int total = warp_sum(cnt);
          const unsigned who = __ballot_sync(0xffffffffu, cnt > 0);
          const int winner = __shfl_sync(0xffffffffu, off, __ffs(who) - 1);
          if (lane == 0) {
            max_val[row * nb + bb] = m;
            tie_info[row * nb + bb] = total == 1 ? winner + 1 : -total;
          }
        }
      }
    }
  }
}

// Error word of the kernel, one per device (calls on one device that overlap share it).
static __device__ int g_score_err;
constexpr int kMaxDevices = 64;
std::mutex g_err_mu;
int* g_err_addr[kMaxDevices] = {};

}  // namespace
}  // namespace msa

using namespace msa;

// Shared launcher: scores for the query range [q_lo, q_hi), and with tie_info the
// winner state (qnorm / kmax: the margin's norms, computed here).
static int launch_score(const void* index_q, const void* index_k, int dtype, const int32_t* cu_seqlens, int32_t nseq,
                        int64_t total_tokens, int32_t groups, int32_t index_dim, int32_t num_blocks,
                        int32_t block_size, float scale, int64_t q_lo, int64_t q_hi, float* scores,
                        int32_t* tie_info, double* max_val, float* qnorm, unsigned* kmax, void* stream) {
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
  const int tile_bytes = 16384 * (index_dim / 64);
  int nst = ((kSmemScoreMax - 1024) / tile_bytes - 2) / 2;  // key-block pairs that fit beside 2 index_q tiles
  nst = (nst < kIkStagesMax ? nst : kIkStagesMax) & ~1;  // even: each MMA issuer owns every other stage
  const int smem_bytes = score_smem(tile_bytes, nst);
  ScoreArgs sa{cu_seqlens, scores, err, tie_info, qnorm, kmax, nseq, groups, num_blocks, 128 / groups,
               index_dim / 64, (int)q_lo, (int)q_hi, fabsf(scale), scale < 0.f ? 1 : 0, dtype == MSA_F16 ? 1 : 0,
               nst};
  if (tie_info) {
    MSA_CUDA_RETURN(cudaMemsetAsync(kmax, 0, sizeof(unsigned), st));
    score_norms_kernel<<<sms * 8, 256, 0, st>>>(index_q, index_k, dtype, total_tokens * groups, total_tokens,
                                                index_dim, qnorm, kmax);
    MSA_CUDA_RETURN(cudaFuncSetAttribute(score_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         smem_bytes));
    score_tc_kernel<true><<<sms, kScoreThreads, smem_bytes, st>>>(iqmap, ikmap, sa);
    score_fixup_kernel<<<sms * 16, 256, 8 * index_dim * sizeof(double), st>>>(
        index_q, index_k, dtype, cu_seqlens, nseq, total_tokens * groups, groups, index_dim, num_blocks,
        (double)scale, tie_info, max_val);
    count_launches(3);
  } else {
    MSA_CUDA_RETURN(cudaFuncSetAttribute(score_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         smem_bytes));
    score_tc_kernel<false><<<sms, kScoreThreads, smem_bytes, st>>>(iqmap, ikmap, sa);
    count_launches(1);
  }
  score_poison_kernel<<<sms * 4, 256, 0, st>>>(err, (q_hi - q_lo) * groups * (int64_t)num_blocks,
                                               scores + q_lo * groups * (int64_t)num_blocks);
  count_launches(1);
  return launch_status("index_score_fwd_tc");
}

extern "C" int msa_index_score_fwd_tc(const void* index_q, const void* index_k, int dtype, const int32_t* cu_seqlens,
                                      int32_t nseq, int64_t total_tokens, int32_t groups, int32_t index_dim,
                                      int32_t num_blocks, int32_t block_size, float scale, int64_t q_lo,
                                      int64_t q_hi, float* scores, void* stream) {
  return launch_score(index_q, index_k, dtype, cu_seqlens, nseq, total_tokens, groups, index_dim, num_blocks,
                      block_size, scale, q_lo, q_hi, scores, nullptr, nullptr, nullptr, nullptr, stream);
}

extern "C" size_t msa_index_score_state_workspace_size(int64_t total_tokens, int32_t groups) {
  return 256 + ((sizeof(float) * (size_t)total_tokens * groups + 255) & ~size_t(255));
}

extern "C" int msa_index_score_fwd_tc_state(const void* index_q, const void* index_k, int dtype,
                                            const int32_t* cu_seqlens, int32_t nseq, int64_t total_tokens,
                                            int32_t groups, int32_t index_dim, int32_t num_blocks,
                                            int32_t block_size, float scale, float* scores, int32_t* tie_info,
                                            double* max_val, void* workspace, size_t workspace_bytes, void* stream) {
  MSA_CHECK_ARG(tie_info && max_val, "msa_index_score_fwd_tc_state: tie_info and max_val are required");
  MSA_CHECK_ARG(workspace && workspace_bytes >= msa_index_score_state_workspace_size(total_tokens, groups),
                "msa_index_score_fwd_tc_state: workspace too small");
  unsigned* kmax = static_cast<unsigned*>(workspace);
  float* qnorm = reinterpret_cast<float*>(static_cast<char*>(workspace) + 256);
  return launch_score(index_q, index_k, dtype, cu_seqlens, nseq, total_tokens, groups, index_dim, num_blocks,
                      block_size, scale, 0, total_tokens, scores, tie_info, max_val, qnorm, kmax, stream);
}
