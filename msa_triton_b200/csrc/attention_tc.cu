// Sparse attention forward, tensor-core path (sm_100a: TMA + tcgen05 + TMEM).
//
// Organisation: key-block stationary. The work list is the k2q CSR (one row per
// (128-key block, group); triton/k2q.py:39-128), cut into chunks of 128/h
// selector tokens (h = query heads per group). A chunk is one M = 128 tile whose
// rows are (token, head) pairs: TMA gathers each selector token's h query rows
// (contiguous in q[T][Hq][D]) into the tile, so the block's K/V, loaded once per
// row, serve every head of every selecting token. With h = 4 the chunk holds 32
// tokens, whose 4-row groups are copied with cp.async (a TMA box of 4 rows
// would not fill a 1024-byte swizzle atom).
//
//   S   = Q_tile . K_b^T                      tcgen05, SMEM x SMEM -> TMEM (f32)
//   P   = exp(scale*S - bound_row), causal    softmax warps, P -> TMEM as bf16/f16
//   O_e = P . V_b                             tcgen05, TMEM x SMEM -> TMEM (f32)
//   O_acc[t, heads] += O_e ; l_acc += rowsum(P)   red.global.add (f32)
//
// A query's softmax spans up to K chunks on different CTAs, so the exponent is
// taken against a per-row static upper bound instead of a running maximum;
// contributions then add with no rescaling. The bound is Cauchy-Schwarz over the
// row's own selected blocks: bound = |scale| |q_row| max_{b selected} max_{j in b}|k_j|
// (per (key block, group) key-norm maxima), so exp(S - bound) <= 1 never overflows.
// finalize: out = O_acc / l, lse = bound + log(l). A row whose bound sits so far
// above its logits that l < 2^-88 (keys below 2^-126 flush to zero and would no
// longer be negligible) is re-run: its (token, group) pair goes through the same
// kernel once more over a filtered CSR, centred on the row's exact logit maximum
// (a float32 pass over the pair's selected keys). Rows still short after that
// (none are expected: the maximum term is exp(0) = 1) take the float64 row kernel.
//
// Roles (384 threads): warp 0 = TMA producer, warp 1 = MMA issuer, warps 4-7
// and 8-11 = two softmax/epilogue warpgroups taking alternate chunks, each with
// its own TMEM stage (S/P 128 columns + O 128 columns).
#include <algorithm>

#include "attn_common.cuh"

namespace msa {
int launch_fwd_fixup(const void* q, const void* k, const void* v, int dtype, const int32_t* ids, const int32_t* cu,
                     int nseq, int hq, int groups, int dim, int topk, int block, double scale, const int32_t* list,
                     void* out, float* lse, cudaStream_t st);

namespace {

using namespace tc;
using namespace attn;

constexpr int kD = 128;
constexpr int kFwdThreads = 384;
// A row is accurate when l = sum_j exp(S_j - bound) >= 2^-88: keys whose term
// flushes to zero (< 2^-126) then weigh < #keys * 2^-38 of the row's mass.
constexpr float kMinRowMass = 3.2311742677852644e-27f;  // 2^-88
constexpr int kSmemFwd = 3 * 32768 + 2 * 32768 + 8 * 32 * 36 * 4 + 1024;

// Per-chunk metadata, precomputed for every work item by item_meta_kernel and
// brought into a shared ring with one bulk copy per item.
struct __align__(16) TileMeta {
  int32_t tok[32];     // token id per chunk position, -1: past the chunk end or a repeated slot
  int32_t kb0, g;      // first key token of the block, group
  int32_t flags;       // bit 0: first chunk of its key block in this CTA, bit 1: last
  int32_t pad;
};
static_assert(sizeof(TileMeta) % 16 == 0, "bulk copies move multiples of 16 bytes");

struct FwdArgs {
  const void* q;  // [T][Hq][128], read directly by the 4-heads-per-group gather
  const int32_t* row_ptr;
  const int32_t* queries;
  const int32_t* work_ptr;  // [n_waves * num_rows + 1] exclusive prefix of chunks, wave-major
  const int32_t* wave_off;  // [(n_waves + 1) * num_rows] first edge of each (wave, row)
  const TileMeta* gmeta;    // [total items] per-item metadata (see item_meta_kernel)
  const int32_t* cu;
  const int32_t* cbl;  // cu_block_lens
  const float* bound;  // [T*Hq]
  float* l_acc;        // [T*Hq]
  float* o_acc;        // [T*Hq*128]
  int* err;
  int nseq, num_rows, groups, hq, h, tpc, n_waves;
  float scale_log2;
  int f16;  // 1: fp16 operands, 0: bf16
  // teacher mode (index KL loss) only: the selection slot of every item position
  // and the output p_T [T*G][K][128] (head-mean probabilities)
  const int32_t* gslot;
  float* pt;
  int topk;
};

// Sum-scatter across the h lanes of one token (lanes differing in the bits of
// `mask` and below): n values per lane in, n/2 out, the lane with the mask bit
// set keeping the upper half. Every lane of the warp takes part.
template <int N>
__device__ __forceinline__ void sum_scatter_step(float* v, int mask, int lane) {
  const bool upper = (lane & mask) != 0;
#pragma unroll
  for (int i = 0; i < N / 2; ++i) {
    const float send = upper ? v[i] : v[i + N / 2];
    const float keep = upper ? v[i + N / 2] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, mask);
  }
}

constexpr int kNQ = 3;  // depth of the Q ring
constexpr int kNM = 4;  // depth of the metadata ring (prefetched two items ahead)

// kRows4: h == 4, cp.async gathers into the plain K-major layout.
// kTeacher: the index KL loss's teacher pass. `bound` holds each row's attention
// LSE, so P = exp(S - lse) are the per-head probabilities; no P.V is issued and
// the softmax warps write the mean over the token's h heads, p_T, for their
// 128 keys to `pt` (the lanes of one token sum-scatter the columns).
template <bool kRows4, bool kTeacher = false>
__global__ void __launch_bounds__(kFwdThreads, 1)
attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap, FwdArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  // Q ring: per stage 2 KB blocks of 8 head rows x (2 d-chunks x 128 B), one per
  // (token, head octet); descriptor SBO 2048, second d-chunk at +1024.
  uint8_t* sQ0 = smem;
  uint8_t* sK = smem + kNQ * 32768;  // K block: 2 d-chunks x 128 keys x 128 B (SBO 1024)
  uint8_t* sV = sK + 32768;          // V block, same layout (MN-major B operand of P.V)
  float* sX0 = reinterpret_cast<float*>(sV + 32768);  // per epilogue warp: 32 x 36 floats (transpose)
  __shared__ TileMeta meta[kNM];
  __shared__ uint64_t q_full[kNQ], q_empty[kNQ], meta_full[kNM], meta_empty[kNM];
  // TMEM stages: S (128 columns) + O_e (128) x 2; the teacher mode has no O_e, so
  // it runs 4 S-only stages and the S issuer keeps two items ahead of each warpgroup
  constexpr int kSt = kTeacher ? 4 : 2;
  constexpr int kStCols = kTeacher ? 128 : 256;
  // A second gathering warp (warp 3). Teacher mode: the TMA gathers (one 2 KB box per
  // token and head octet) are issued by the producer for the first half of each item's
  // chunk positions and by warp 3 for the second; the producer's serialised box issue
  // held the teacher's item rate (2.93K -> 2.66K cycles per item). The full forward at
  // 8+ heads per group is bound by its O drain instead, and there the helper measured
  // 10 % slower, so it keeps one issuing warp. 4 heads per group (cp.async, 64 16-byte
  // steps per item, ~5K cycles from one warp, the item rate of both modes): the
  // producer copies the first 64 columns of every row and warp 3 the second.
  constexpr bool kHelper = kRows4 || kTeacher;
  __shared__ uint64_t s_full[kSt], p_full[2], o_full[kSt], o_free[2];
  __shared__ uint64_t k_full, k_empty, v_full, v_empty;
  __shared__ int32_t pv_flags[2];
  __shared__ uint32_t tmem_base;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int j = 0; j < kNQ; ++j) {
      mbar_init(&q_full[j], kRows4 ? 64 : 1);  // cp.async: one arrival per lane of both gathering warps; TMA: expect_tx
      mbar_init(&q_empty[j], 1);
    }
    for (int j = 0; j < kNM; ++j) {
      mbar_init(&meta_full[j], 1);
      mbar_init(&meta_empty[j], kHelper ? 6 : 5);  // 4 softmax warps + the S issuer (+ the gather helper)
    }
    for (int j = 0; j < kSt; ++j) {
      mbar_init(&s_full[j], 1);
      mbar_init(&o_full[j], kTeacher ? 4 : 1);  // teacher: the 4 softmax warps release S
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&p_full[j], 4);
      mbar_init(&o_free[j], 4);
    }
    mbar_init(&k_full, 1);
    mbar_init(&k_empty, 1);
    mbar_init(&v_full, 1);
    mbar_init(&v_empty, 1);
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

  const int cells = a.n_waves * a.num_rows;
  const int total_items = a.work_ptr[cells];
  const int h = a.h;
  // h >= 8: TMA gathers each token's h rows as 8-row swizzle atoms (2 KB per 8
  // heads, SBO 2048). h = 4: 32 tokens x 4 heads, copied with cp.async into the
  // plain K-major layout (8-row groups 1024 B apart, halves 16 KB apart).
  constexpr bool rows4 = kRows4;
  const int hb = h;
  const int octets = hb / 8;  // 2 KB Q blocks per token (TMA path)

  if (warp == 0) {
    // ---------------------------------------------------------------- producer (whole warp)
    // Per item: its metadata block (bulk-copied two items ahead), then lane p
    // gathers the query rows of chunk position p with TMA.
    if (lane == 0) {
      tma_prefetch_desc(&qmap);
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
    }
    int kv_loads = 0, v_loads = 0;
    int pend_g = 0, pend_kb0 = 0;
    // V of a new key block loads once the previous block's last P.V is done; lane
    // 0 services it from its waits so Q gathers keep flowing meanwhile.
    auto service_v = [&](bool block) -> bool {
      if (kTeacher || v_loads == kv_loads) return true;  // the teacher mode reads no V
      if (v_loads > 0) {
        if (block) {
          if (!mbar_wait(&v_empty, (v_loads - 1) & 1, a.err, 14)) return false;
        } else if (!mbar_try_wait(&v_empty, (v_loads - 1) & 1)) {
          return true;
        }
      }
      mbar_arrive_expect_tx(&v_full, 32768);
      tma_load_3d(sV, &vmap, &v_full, 0, pend_g, pend_kb0);
      tma_load_3d(sV + 16384, &vmap, &v_full, 64, pend_g, pend_kb0);
      ++v_loads;
      return true;
    };
    auto wait_serviced = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
      for (uint32_t n = 0; n < kMaxPolls; ++n) {
        if (mbar_try_wait(bar, parity)) return true;
        if (!service_v(false)) return false;
        if ((n & 63) == 63 && *(volatile int*)a.err != 0) return false;
      }
      atomicCAS(a.err, 0, code);
      return false;
    };
    // metadata prefetch (lane 0): item ip into slot ip % kNM once that slot's previous item is released
    ItemIter itp;
    itp.start(total_items);
    int ip = 0;
    auto prefetch_meta = [&]() -> bool {
      if (!itp.valid()) return true;
      const int slot = ip % kNM;
      if (ip >= kNM && !wait_serviced(&meta_empty[slot], ((ip / kNM) - 1) & 1, 15)) return false;
      mbar_arrive_expect_tx(&meta_full[slot], sizeof(TileMeta));
      bulk_copy_g2s(&meta[slot], a.gmeta + itp.w, sizeof(TileMeta), &meta_full[slot]);
      ++ip;
      itp.next();
      return true;
    };
    bool ok = true;
    if (lane == 0) ok = prefetch_meta() && prefetch_meta();
    ItemIter it;
    it.start(total_items);
    for (int i = 0; it.valid() && __shfl_sync(0xffffffffu, ok, 0); ++i, it.next()) {
      const int qs = i % kNQ, ms = i % kNM;
      if (lane == 0) ok = prefetch_meta();
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      if (!mbar_wait_warp(&meta_full[ms], (i / kNM) & 1, a.err, 16)) {
        ok = false;
        break;
      }
      const TileMeta& m = meta[ms];
      const int t = m.tok[lane];
      const int g = m.g, kb0 = m.kb0, flags = m.flags;
      if (lane == 0) {
        if (flags & 1) {  // first chunk of a key block: K as soon as the old block's last S is done
          ok = service_v(true);
          if (ok && kv_loads > 0) ok = wait_serviced(&k_empty, (kv_loads - 1) & 1, 11);
          if (ok) {
            mbar_arrive_expect_tx(&k_full, 32768);
            tma_load_3d(sK, &kmap, &k_full, 0, g, kb0);
            tma_load_3d(sK + 16384, &kmap, &k_full, 64, g, kb0);
            ++kv_loads;
            pend_g = g;
            pend_kb0 = kb0;
          }
        }
        if (ok) ok = service_v(false);
        if (ok && i >= kNQ) ok = wait_serviced(&q_empty[qs], ((i / kNQ) - 1) & 1, 12);
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      if (rows4) {
        // cp.async gather; each lane's copies arrive on q_full when they land (32
        // arrivals complete the phase; the S issuer fences them for the async proxy)
        gather_rows4(smem_u32(sQ0 + qs * 32768), 16384, 128, a.q, (int64_t)a.hq * kD, g * 4, t, lane, 0, 1);
        cp_async_arrive_noinc(&q_full[qs]);
        continue;
      }
      const bool valid_pos = t >= 0;
      // the byte count covers the helper's boxes too (its completions may precede this
      // expect: the transaction count goes negative until it lands, never completing early)
      const uint32_t nv = __popc(__ballot_sync(0xffffffffu, valid_pos));
      if (lane == 0) mbar_arrive_expect_tx(&q_full[qs], nv * (uint32_t)hb * 256u);
      __syncwarp();
      if (valid_pos && (!kHelper || lane < (a.tpc >> 1))) {
        uint8_t* dst = sQ0 + qs * 32768 + lane * octets * 2048;
        for (int oc = 0; oc < octets; ++oc)
          tma_load_4d(dst + oc * 2048, &qmap, &q_full[qs], 0, g * h + oc * 8, 0, t);
      }
    }
    if (lane == 0 && ok) service_v(true);  // the last block's V
  } else if (kHelper && warp == 3) {
    // ---------------------------------------------------------------- gather helper
    // Second half of each item's chunk positions (TMA) or columns (cp.async) onto the
    // same q_full phase.
    const int octets = h / 8;
    ItemIter it;
    it.start(total_items);
    for (int i = 0; it.valid(); ++i, it.next()) {
      const int qs = i % kNQ, ms = i % kNM;
      if (!mbar_wait_warp(&meta_full[ms], (i / kNM) & 1, a.err, 17)) break;
      const int t = meta[ms].tok[lane];
      const int g = meta[ms].g;
      __syncwarp();
      if (lane == 0) mbar_arrive(&meta_empty[ms]);
      if (i >= kNQ && !mbar_wait_warp(&q_empty[qs], ((i / kNQ) - 1) & 1, a.err, 18)) break;
      if (kRows4) {  // the second 64 columns of every row
        gather_rows4(smem_u32(sQ0 + qs * 32768), 16384, 128, a.q, (int64_t)a.hq * kD, g * 4, t, lane, 1, 2);
        cp_async_arrive_noinc(&q_full[qs]);
        continue;
      }
      if (t >= 0 && lane >= (a.tpc >> 1)) {
        uint8_t* dst = sQ0 + qs * 32768 + lane * octets * 2048;
        for (int oc = 0; oc < octets; ++oc)
          tma_load_4d(dst + oc * 2048, &qmap, &q_full[qs], 0, g * h + oc * 8, 0, t);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------------------------------------------------------- S = Q K^T issuer
    const uint32_t id_s = idesc_f16(!a.f16, 128, 128, false, false);
    const uint32_t sk = smem_u32(sK);
    int k_loads = 0;
    ItemIter it;
    it.start(total_items);
    for (int i = 0; it.valid(); ++i, it.next()) {
      const int qs = i % kNQ, ms = i % kNM, ts = i % kSt;
      if (!mbar_wait(&q_full[qs], (i / kNQ) & 1, a.err, 21)) break;
      if (!mbar_wait(&meta_full[ms], (i / kNM) & 1, a.err, 24)) break;
      const int flags = meta[ms].flags;
      mbar_arrive(&meta_empty[ms]);
      const int last = (flags >> 1) & 1;
      if (flags & 1) {
        ++k_loads;
        if (!mbar_wait(&k_full, (k_loads - 1) & 1, a.err, 22)) break;
      }
      if (i >= kSt && !mbar_wait(&o_full[ts], ((i / kSt) - 1) & 1, a.err, 23)) break;  // stage ts's P consumed
      if (kRows4) fence_proxy_async_smem();  // cp.async-written Q tile -> the MMA's operand reads
      tc_fence_after();
      const uint32_t sq = smem_u32(sQ0 + qs * 32768);
      for (int ks = 0; ks < 8; ++ks) {
        const uint64_t da = kRows4 ? desc_kmajor_sw128(sq + (ks >> 2) * 16384 + (ks & 3) * 32)
                                   : desc_kmajor_sw128(sq + (ks >> 2) * 1024 + (ks & 3) * 32, 2048);
        umma_ss(tmem + ts * kStCols, da, desc_kmajor_sw128(sk + (ks >> 2) * 16384 + (ks & 3) * 32), id_s, ks > 0);
      }
      umma_commit(&s_full[ts]);
      umma_commit(&q_empty[qs]);
      if (last) umma_commit(&k_empty);
    }
  } else if (!kTeacher && warp == 2 && lane == 0) {
    // ---------------------------------------------------------------- O_e = P V issuer
    const uint32_t id_pv = idesc_f16(!a.f16, 128, 128, false, true);
    const uint32_t sv = smem_u32(sV);
    int v_loads = 0;
    ItemIter it;
    it.start(total_items);
    for (int i = 0; it.valid(); ++i, it.next()) {
      const int ts = i & 1;
      if (!mbar_wait(&p_full[ts], (i >> 1) & 1, a.err, 31)) break;
      const int flags = pv_flags[ts];
      const int last = (flags >> 1) & 1;
      if (flags & 1) {
        ++v_loads;
        if (!mbar_wait(&v_full, (v_loads - 1) & 1, a.err, 32)) break;
      }
      if (i >= 2 && !mbar_wait(&o_free[ts], ((i >> 1) - 1) & 1, a.err, 33)) break;
      tc_fence_after();
      for (int ks = 0; ks < 8; ++ks)
        umma_ts(tmem + ts * 256 + 128, tmem + ts * 256 + ks * 8, desc_mnmajor_sw128(sv + ks * 2048, 16384), id_pv,
                ks > 0);
      umma_commit(&o_full[ts]);
      if (last) umma_commit(&v_empty);
    }
  } else if (warp >= 4) {
    // ---------------------------------------------------------------- softmax + epilogue
    const int wg = (warp - 4) >> 2;
    const int qd = warp & 3;
    const int r = qd * 32 + lane;  // tile row == TMEM lane
    const int pos = r / hb, hh = r - (r / hb) * hb;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const uint32_t t_s = tmem + wg * 256 + lane_base, t_o = t_s + 128;
    float* xs = sX0 + (warp - 4) * 32 * 36;
    ItemIter it;
    it.start(total_items);
    for (int i = 0; it.valid(); ++i, it.next()) {
      if ((i & 1) != wg) continue;  // the other warpgroup takes this item
      const int ms = i % kNM;
      if (!mbar_wait_warp(&meta_full[ms], (i / kNM) & 1, a.err, 41)) break;
      const TileMeta& m = meta[ms];
      const int t = m.tok[pos];
      const int kb0 = m.kb0, g = m.g, flags = m.flags;
      __syncwarp();
      if (lane == 0) mbar_arrive(&meta_empty[ms]);
      const bool valid = t >= 0 && hh < h;
      const int64_t rowid = (int64_t)t * a.hq + g * h + hh;
      const float bnd = ld_early(a.bound + (valid ? rowid : 0));  // in flight during the S wait
      const int slot = kTeacher && valid ? a.gslot[(int64_t)it.w * 32 + pos] : 0;
      const int qoff = t - kb0;  // key c of the block is visible iff c <= qoff
      const int ts = kTeacher ? (i & 3) : wg;
      if (!mbar_wait_warp(&s_full[ts], (i / kSt) & 1, a.err, 42)) break;
      tc_fence_after();
      const float nbound = valid ? -bnd * kLog2e : 0.f;
      // P = 2^(s * scale * log2e - bound * log2e); keys past the query (diagonal
      // block only) and rows without a token give 0. ex2.approx: P is rounded to
      // the 16-bit operand type right after.
      float l = 0.f;
      const bool full = qoff >= 127;
      if (kTeacher) {
        float* dst = a.pt + (((int64_t)(valid ? t : 0) * a.groups + g) * a.topk + slot) * 128;
        const uint32_t t_st = tmem + ts * kStCols + lane_base;
        for (int half = 0; half < 2; ++half) {
          uint32_t sr0[32], sr1[32];
          tmem_ld32(t_st + (half * 2) * 32, sr0);
          tmem_ld32(t_st + (half * 2 + 1) * 32, sr1);
          tmem_wait_ld();
          if (half == 1) {  // all of S is in registers: the stage goes back to the S issuer
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&o_full[ts]);
          }
          const int k0 = half * 64 - qoff;  // key c visible iff c - qoff <= 0
          float v[64];
#pragma unroll
          for (int kk = 0; kk < 32; ++kk) {
            v[kk] = valid && kk + k0 <= 0 ? ex2_approx(fmaf(__uint_as_float(sr0[kk]), a.scale_log2, nbound)) : 0.f;
            v[kk + 32] =
                valid && kk + 32 + k0 <= 0 ? ex2_approx(fmaf(__uint_as_float(sr1[kk]), a.scale_log2, nbound)) : 0.f;
          }
          // sum over the token's h heads, each lane keeping 64 / h columns: hh * 64 / h + [0, 64 / h)
          sum_scatter_step<64>(v, h >> 1, lane);
          sum_scatter_step<32>(v, h >> 2, lane);
          const float inv_h = 1.f / (float)h;
          if (h == 4) {
            if (valid)
#pragma unroll
              for (int c = 0; c < 16; c += 4)
                *reinterpret_cast<float4*>(dst + half * 64 + hh * 16 + c) =
                    make_float4(v[c] * inv_h, v[c + 1] * inv_h, v[c + 2] * inv_h, v[c + 3] * inv_h);
          } else {
            sum_scatter_step<16>(v, h >> 3, lane);
            if (h == 8) {
              if (valid)
#pragma unroll
                for (int c = 0; c < 8; c += 4)
                  *reinterpret_cast<float4*>(dst + half * 64 + hh * 8 + c) =
                      make_float4(v[c] * inv_h, v[c + 1] * inv_h, v[c + 2] * inv_h, v[c + 3] * inv_h);
            } else {
              sum_scatter_step<8>(v, 1, lane);
              if (valid)
                *reinterpret_cast<float4*>(dst + half * 64 + hh * 4) =
                    make_float4(v[0] * inv_h, v[1] * inv_h, v[2] * inv_h, v[3] * inv_h);
            }
          }
        }
        continue;
      }
      for (int half = 0; half < 2; ++half) {
        uint32_t sr0[32], sr1[32], packed[32];
        tmem_ld32(t_s + (half * 2) * 32, sr0);
        tmem_ld32(t_s + (half * 2 + 1) * 32, sr1);
        tmem_wait_ld();
        if (!valid) {
#pragma unroll
          for (int kk = 0; kk < 32; ++kk) packed[kk] = 0u;
        } else if (full) {
#pragma unroll
          for (int kk = 0; kk < 32; kk += 2) {
            const float p0 = ex2_approx(fmaf(__uint_as_float(sr0[kk]), a.scale_log2, nbound));
            const float p1 = ex2_approx(fmaf(__uint_as_float(sr0[kk + 1]), a.scale_log2, nbound));
            const float p2 = ex2_approx(fmaf(__uint_as_float(sr1[kk]), a.scale_log2, nbound));
            const float p3 = ex2_approx(fmaf(__uint_as_float(sr1[kk + 1]), a.scale_log2, nbound));
            l += (p0 + p1) + (p2 + p3);
            packed[kk >> 1] = pack2(p0, p1, a.f16);
            packed[16 + (kk >> 1)] = pack2(p2, p3, a.f16);
          }
        } else {
          const int k0 = half * 64 - qoff;  // key c visible iff c - qoff <= 0
#pragma unroll
          for (int kk = 0; kk < 32; kk += 2) {
            const float p0 = kk + k0 <= 0 ? ex2_approx(fmaf(__uint_as_float(sr0[kk]), a.scale_log2, nbound)) : 0.f;
            const float p1 = kk + 1 + k0 <= 0 ? ex2_approx(fmaf(__uint_as_float(sr0[kk + 1]), a.scale_log2, nbound)) : 0.f;
            const float p2 = kk + 32 + k0 <= 0 ? ex2_approx(fmaf(__uint_as_float(sr1[kk]), a.scale_log2, nbound)) : 0.f;
            const float p3 = kk + 33 + k0 <= 0 ? ex2_approx(fmaf(__uint_as_float(sr1[kk + 1]), a.scale_log2, nbound)) : 0.f;
            l += (p0 + p1) + (p2 + p3);
            packed[kk >> 1] = pack2(p0, p1, a.f16);
            packed[16 + (kk >> 1)] = pack2(p2, p3, a.f16);
          }
        }
        tmem_st32(t_s + half * 32, packed);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (qd == 0) pv_flags[wg] = flags;
        mbar_arrive(&p_full[wg]);
      }
      if (valid) atomicAdd(a.l_acc + rowid, l);
      if (!mbar_wait_warp(&o_full[wg], (i >> 1) & 1, a.err, 43)) break;
      tc_fence_after();
      // O_e rows -> O accumulator. Each 32 x 32 block goes through a padded shared
      // transpose so that one red.v4 instruction covers four whole 128 B rows.
      const int64_t my_off = valid ? rowid * kD : -1;
      const int sub_row = lane >> 3, sub_col = (lane & 7) * 4;
      for (int cp = 0; cp < 2; ++cp) {
        uint32_t o2[2][32];
        tmem_ld32(t_o + (cp * 2) * 32, o2[0]);
        tmem_ld32(t_o + (cp * 2 + 1) * 32, o2[1]);
        tmem_wait_ld();
        if (cp == 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&o_free[wg]);
        }
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
          const int cb = cp * 2 + hb;
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<uint4*>(xs + lane * 36 + u * 4) =
                make_uint4(o2[hb][4 * u], o2[hb][4 * u + 1], o2[hb][4 * u + 2], o2[hb][4 * u + 3]);
          __syncwarp();
#pragma unroll
          for (int k4 = 0; k4 < 8; ++k4) {
            const int rr = k4 * 4 + sub_row;
            const int64_t off = __shfl_sync(0xffffffffu, my_off, rr);
            if (off >= 0) {
              const float4 v4 = *reinterpret_cast<const float4*>(xs + rr * 36 + sub_col);
              red_add_v4(a.o_acc + off + cb * 32 + sub_col, v4.x, v4.y, v4.z, v4.w);
            }
          }
          __syncwarp();
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

// ---------------------------------------------------------------- helpers
// Squared norm of 8 consecutive bf16/f16 elements (one 16-byte load).
__device__ __forceinline__ float sq8(const void* base, int64_t elem, int f16) {
  const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(base) + elem * 2);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = f16 ? __half22float2(*reinterpret_cast<const __half2*>(&w[i]))
                         : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
    s = fmaf(f.x, f.x, fmaf(f.y, f.y, s));
  }
  return s;
}

// Sum over the 16 lanes that share a row (lanes 0-15 / 16-31 of a warp).
__device__ __forceinline__ float sum16(float s) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}

// Largest |k| over the keys of each (key block, group) CSR row: one warp per
// row, 16 lanes x 8 elements per key, two keys at a time.
__global__ void block_key_norm_kernel(const void* __restrict__ k, int f16, const int32_t* __restrict__ cu,
                                      const int32_t* __restrict__ cbl, int nseq, int groups, int num_rows,
                                      float* __restrict__ kbmax) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < num_rows; row += warps) {
    const int gb = row / groups, g = row - gb * groups;
    const int s = block_sequence(cbl, nseq, gb);
    const int64_t kb0 = cu[s] + (int64_t)(gb - cbl[s]) * 128;
    const int nk = min(128, (int)(cu[s + 1] - kb0));
    float best = 0.f;
    for (int j = lane >> 4; j < nk; j += 2) {
      const float sq = sum16(sq8(k, ((kb0 + j) * groups + g) * kD + (lane & 15) * 8, f16));
      best = fmaxf(best, sqrtf(sq));
    }
    best = fmaxf(best, __shfl_xor_sync(0xffffffffu, best, 16));
    if (lane == 0) kbmax[row] = best;
  }
}

// Per (token, group): the largest key norm over the group's valid selected
// blocks (block ids are sequence-local, valid iff 0 <= b <= the token's block),
// or -1 when the pair selects no key at all.
__global__ void selected_key_norm_kernel(const int32_t* __restrict__ ids, const int32_t* __restrict__ cu,
                                         const int32_t* __restrict__ cbl, int nseq, int64_t p0, int64_t p1,
                                         int groups, int topk, const float* __restrict__ kbmax,
                                         float* __restrict__ selmax) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t p = p0 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < p1; p += stride) {
    const int t = (int)(p / groups), g = (int)(p - (int64_t)t * groups);
    int lo = 0, hi = nseq - 1;  // sequence of token t: last s with cu[s] <= t
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (cu[mid] <= t) lo = mid; else hi = mid - 1;
    }
    const int cur = (t - cu[lo]) / 128;
    float m = -1.f;
    for (int j = 0; j < topk; ++j) {
      const int b = ids[p * topk + j];
      if (b >= 0 && b <= cur) m = fmaxf(m, kbmax[(int64_t)(cbl[lo] + b) * groups + g]);
    }
    selmax[p] = m;
  }
}

// Per query row: bound = |scale| |q| max|k| over the row's selected blocks
// (slightly inflated so float rounding cannot put a logit above it), -inf for a
// row without keys. The same pass zeroes the row's O and l accumulators (no
// separate memset of the 1 GB-class accumulator).
__global__ void row_bound_kernel(const void* __restrict__ q, int f16, int64_t row0, int64_t rows, int hq, int h,
                                 const float* __restrict__ selmax, float abs_scale, float* __restrict__ bound,
                                 float* __restrict__ o_acc, float* __restrict__ l_acc) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int groups = hq / h;
  for (int64_t base = row0 + (((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5) * 2; base < rows;
       base += warps * 2) {
    const int64_t row = base + (lane >> 4);
    const bool in = row < rows;
    const float s = sum16(in ? sq8(q, row * kD + (lane & 15) * 8, f16) : 0.f);
    if (in) {
      float4* z = reinterpret_cast<float4*>(o_acc + row * kD + (lane & 15) * 8);
      z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
      z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (in && (lane & 15) == 0) {
      const int64_t t = row / hq;
      const int g = (int)(row - t * hq) / h;
      const float km = selmax[t * groups + g];
      bound[row] = km < 0.f ? -INFINITY : abs_scale * sqrtf(s) * km * 1.0001f + 1e-6f;
      l_acc[row] = 0.f;
    }
  }
}

// One warp per item: lane p takes chunk position p (token id, repeated-slot
// check against the previous CSR edge); item_cell gives the item's cell. With
// `gslot`, also each position's selection slot (from the CSR's slot_indices).
__global__ void item_meta_kernel(const int32_t* __restrict__ work_ptr, const int32_t* __restrict__ item_cell,
                                 const int32_t* __restrict__ wave_off, const int32_t* __restrict__ row_ptr,
                                 const int32_t* __restrict__ queries, const int32_t* __restrict__ cu,
                                 const int32_t* __restrict__ cbl, int nseq, int groups, int num_rows, int cells,
                                 int tpc, int grid, TileMeta* __restrict__ gmeta, const int32_t* __restrict__ slots,
                                 int32_t* __restrict__ gslot) {
  const int lane = threadIdx.x & 31;
  const int total = work_ptr[cells];
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < total; w += warps) {
    const int cell = item_cell[w];
    const int row = cell % num_rows;
    const int e0 = wave_off[cell] + (w - work_ptr[cell]) * tpc;
    const int n = min(tpc, wave_off[cell + num_rows] - e0);
    const int gb = row / groups, g = row - gb * groups;
    const int lo = block_sequence(cbl, nseq, gb);
    const int kb0 = cu[lo] + (gb - cbl[lo]) * 128;
    int t = lane < n ? queries[e0 + lane] : -1;
    int prev = __shfl_up_sync(0xffffffffu, t, 1);
    if (lane == 0) prev = e0 > row_ptr[row] ? queries[e0 - 1] : -1;
    t = (t >= 0 && t != prev) ? t : -1;
    TileMeta& m = gmeta[w];
    m.tok[lane] = t;
    if (gslot != nullptr) gslot[(int64_t)w * 32 + lane] = lane < n ? slots[e0 + lane] : -1;
    if (lane == 0) {
      m.kb0 = kb0;
      m.g = g;
      m.flags = item_run_flags(item_cell, num_rows, total, grid, w, row);
      m.pad = 0;
    }
  }
}

// out = O_acc / l (16 threads per row, 8 columns each) for rows [row0, rows);
// lse = bound + log(l). A kernel error word poisons the outputs with NaN instead of leaving stale data.
// Rows with keys but l < 2^-88 are left for the re-run: their (token, group)
// pair is flagged (and listed once) for the re-centred tensor-core pass.
__global__ void fwd_finalize_kernel(const float* __restrict__ o_acc, const float* __restrict__ l_acc,
                                    float* __restrict__ bound, int64_t row0, int64_t rows, int hq, int h, int f16,
                                    const int* __restrict__ err, uint32_t* __restrict__ flag_pair,
                                    int32_t* __restrict__ pair_list, int* __restrict__ fix_count,
                                    void* __restrict__ out, float* __restrict__ lse) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t row = row0 + (idx >> 4);
  const int c = (int)(idx & 15);
  if (row >= rows) return;
  const int64_t t = row / hq;
  const int64_t pair = t * (hq / h) + (row - t * hq) / h;
  const bool bad = *err != 0;
  const float l = l_acc[row];
  const float b = bound[row];
  if (!bad && b > -INFINITY && l < kMinRowMass) {  // a row with keys (finite bound) but too little mass
    if (c == 0) {
      if (atomicExch(flag_pair + pair, 1u) == 0u) pair_list[1 + atomicAdd(pair_list, 1)] = (int32_t)pair;
      atomicAdd(fix_count, 1);
    }
    return;
  }
  const float inv = bad ? __int_as_float(0x7fc00000) : (l > 0.f ? 1.f / l : 0.f);
  const float4 a = *reinterpret_cast<const float4*>(o_acc + row * kD + c * 8);
  const float4 bb = *reinterpret_cast<const float4*>(o_acc + row * kD + c * 8 + 4);
  uint4 packed;
  packed.x = pack2(a.x * inv, a.y * inv, f16);
  packed.y = pack2(a.z * inv, a.w * inv, f16);
  packed.z = pack2(bb.x * inv, bb.y * inv, f16);
  packed.w = pack2(bb.z * inv, bb.w * inv, f16);
  *reinterpret_cast<uint4*>(static_cast<uint8_t*>(out) + (row * kD + c * 8) * 2) = packed;
  if (c == 0) lse[row] = bad ? __int_as_float(0x7fc00000) : (l > 0.f ? b + logf(l) : -INFINITY);
}

// Finalize after the re-run, over the listed (token, group) pairs only (the
// first pass's finalize wrote every other row): out = O_acc / l, lse; a row still
// short of mass goes to the float64 row kernel's list. Grid-stride over (pair,
// head, 16-byte chunk), so an empty list costs one small launch.
__global__ void fix_finalize_kernel(const float* __restrict__ o_acc, const float* __restrict__ l_acc,
                                    const float* __restrict__ bound, int hq, int h, int f16, const int* __restrict__ err,
                                    const int32_t* __restrict__ pair_list, int32_t* __restrict__ fix_list,
                                    void* __restrict__ out, float* __restrict__ lse) {
  const int64_t n = (int64_t)pair_list[0] * h * 16;
  const int per_t = hq / h;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n; idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = idx / (h * 16);
    const int rem = (int)(idx - p * h * 16), i = rem >> 4, c = rem & 15;
    const int64_t pair = pair_list[1 + p];
    const int64_t t = pair / per_t;
    const int64_t row = t * hq + (pair - t * per_t) * h + i;
    const bool bad = *err != 0;
    const float l = l_acc[row];
    const float b = bound[row];
    if (!bad && b > -INFINITY && l < kMinRowMass) {
      if (c == 0) fix_list[1 + atomicAdd(fix_list, 1)] = (int32_t)row;
      continue;
    }
    const float inv = bad ? __int_as_float(0x7fc00000) : (l > 0.f ? 1.f / l : 0.f);
    const float4 a = *reinterpret_cast<const float4*>(o_acc + row * kD + c * 8);
    const float4 bb = *reinterpret_cast<const float4*>(o_acc + row * kD + c * 8 + 4);
    uint4 packed;
    packed.x = pack2(a.x * inv, a.y * inv, f16);
    packed.y = pack2(a.z * inv, a.w * inv, f16);
    packed.z = pack2(bb.x * inv, bb.y * inv, f16);
    packed.w = pack2(bb.z * inv, bb.w * inv, f16);
    *reinterpret_cast<uint4*>(static_cast<uint8_t*>(out) + (row * kD + c * 8) * 2) = packed;
    if (c == 0) lse[row] = bad ? __int_as_float(0x7fc00000) : (l > 0.f ? b + logf(l) : -INFINITY);
  }
}

// Re-run preparation, one CTA per listed (token, group) pair: every row of the
// pair that came out short (l < 2^-88) gets the exact maximum of its logits as
// its new centre (float32 dot products; thread c takes key c of every selected
// block, the pair's H query rows staged in shared memory), so exp(S - centre)
// <= 1 with the row maximum at 1; then O and l of all the pair's heads are
// zeroed (the unflagged heads are recomputed with their own bounds).
constexpr int kPrepThreads = 128;

template <int H>
__global__ void __launch_bounds__(kPrepThreads)
fix_prepare_kernel(const int32_t* __restrict__ pair_list, int groups, const void* __restrict__ q,
                   const void* __restrict__ k, int f16, const int32_t* __restrict__ ids, int topk,
                   const int32_t* __restrict__ cu, int nseq, float scale, float* __restrict__ bound,
                   float* __restrict__ o_acc, float* __restrict__ l_acc) {
  __shared__ __align__(16) float qs[H * kD];
  __shared__ float red_mx[kPrepThreads / 32][H], red_mn[kPrepThreads / 32][H];
  const int tid = threadIdx.x, lane = tid & 31, wib = tid >> 5;
  const int n = pair_list[0];
  for (int i = blockIdx.x; i < n; i += gridDim.x) {
    const int64_t p = pair_list[1 + i];
    const int64_t row0 = p * H;  // the group's heads are consecutive rows
    const int t = (int)(p / groups);
    const int g = (int)(p - (int64_t)t * groups);
    const int s = find_sequence(cu, nseq, t);
    const int seq0 = cu[s], pos = t - seq0, cur = pos / 128;
    for (int e = tid; e < H * kD / 2; e += kPrepThreads) {  // the pair's query rows as float32
      const uint32_t w2 = static_cast<const uint32_t*>(q)[(row0 * kD) / 2 + e];
      const float2 f = f16 ? __half22float2(*reinterpret_cast<const __half2*>(&w2))
                           : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w2));
      qs[2 * e] = f.x;
      qs[2 * e + 1] = f.y;
    }
    __syncthreads();
    float mx[H], mn[H];
#pragma unroll
    for (int hh = 0; hh < H; ++hh) {
      mx[hh] = -INFINITY;
      mn[hh] = INFINITY;
    }
    for (int j = 0; j < topk; ++j) {
      const int b = ids[p * topk + j];
      if (b < 0 || b > cur) continue;
      const int nk = b < cur ? 128 : pos - b * 128 + 1;  // causal: the diagonal block up to the token
      if (tid >= nk) continue;
      const int64_t key = (int64_t)(seq0 + b * 128 + tid) * groups + g;
      const uint4* kr = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(k) + key * kD * 2);
      float acc[H];
#pragma unroll
      for (int hh = 0; hh < H; ++hh) acc[hh] = 0.f;
      for (int d8 = 0; d8 < kD / 8; ++d8) {
        const uint4 u = kr[d8];
        const uint32_t wv[4] = {u.x, u.y, u.z, u.w};
        float kf[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = f16 ? __half22float2(*reinterpret_cast<const __half2*>(&wv[e]))
                               : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wv[e]));
          kf[2 * e] = f.x;
          kf[2 * e + 1] = f.y;
        }
#pragma unroll
        for (int hh = 0; hh < H; ++hh) {
          const float4 qa = *reinterpret_cast<const float4*>(qs + hh * kD + d8 * 8);
          const float4 qb = *reinterpret_cast<const float4*>(qs + hh * kD + d8 * 8 + 4);
          acc[hh] = fmaf(qa.x, kf[0], fmaf(qa.y, kf[1], fmaf(qa.z, kf[2], fmaf(qa.w, kf[3], acc[hh]))));
          acc[hh] = fmaf(qb.x, kf[4], fmaf(qb.y, kf[5], fmaf(qb.z, kf[6], fmaf(qb.w, kf[7], acc[hh]))));
        }
      }
#pragma unroll
      for (int hh = 0; hh < H; ++hh) {
        mx[hh] = fmaxf(mx[hh], acc[hh]);
        mn[hh] = fminf(mn[hh], acc[hh]);
      }
    }
#pragma unroll
    for (int hh = 0; hh < H; ++hh) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        mx[hh] = fmaxf(mx[hh], __shfl_xor_sync(0xffffffffu, mx[hh], o));
        mn[hh] = fminf(mn[hh], __shfl_xor_sync(0xffffffffu, mn[hh], o));
      }
      if (lane == 0) {
        red_mx[wib][hh] = mx[hh];
        red_mn[wib][hh] = mn[hh];
      }
    }
    __syncthreads();
    if (tid < H) {  // re-centre head tid if it came out short (its pass-1 l and bound are still in place)
      float a = red_mx[0][tid], z = red_mn[0][tid];
      for (int w2 = 1; w2 < kPrepThreads / 32; ++w2) {
        a = fmaxf(a, red_mx[w2][tid]);
        z = fminf(z, red_mn[w2][tid]);
      }
      const int64_t row = row0 + tid;
      const float b = bound[row];
      if (b > -INFINITY && l_acc[row] < kMinRowMass) bound[row] = scale >= 0.f ? scale * a : scale * z;
    }
    __syncthreads();
    float4* zo = reinterpret_cast<float4*>(o_acc + row0 * kD);
    for (int e = tid; e < H * kD / 4; e += kPrepThreads) zo[e] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (tid < H) l_acc[row0 + tid] = 0.f;
    __syncthreads();
  }
}

// Filtered CSR for the re-run: the edges of flagged (token, group) pairs only,
// in their original order. Pass 1 counts per row (all zero when nothing is
// flagged), a single-CTA scan makes the row pointers, pass 2 compacts.
__global__ void csr_filter_count_kernel(const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ queries,
                                        int num_rows, int groups, const uint32_t* __restrict__ flag_pair,
                                        const int* __restrict__ gate, int32_t* __restrict__ cnt) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const bool any = *gate != 0;
  for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < num_rows; row += warps) {
    int n = 0;
    if (any) {
      const int g = row % groups;
      for (int e = row_ptr[row] + lane, end = row_ptr[row + 1]; e - lane < end; e += 32) {
        const bool f = e < end && flag_pair[(int64_t)queries[e] * groups + g] != 0;
        n += __popc(__ballot_sync(0xffffffffu, f));
      }
    }
    if (lane == 0) cnt[row] = n;
  }
}

__global__ void __launch_bounds__(1024) row_scan_kernel(const int32_t* __restrict__ cnt, int num_rows,
                                                        int32_t* __restrict__ row_ptr) {
  __shared__ int32_t warp_tot[32];
  __shared__ int32_t carry;
  if (threadIdx.x == 0) {
    carry = 0;
    row_ptr[0] = 0;
  }
  __syncthreads();
  for (int base = 0; base < num_rows; base += 1024) {
    const int r = base + threadIdx.x;
    const int incl = block_inclusive_scan_1024(r < num_rows ? cnt[r] : 0, warp_tot);
    if (r < num_rows) row_ptr[r + 1] = carry + incl;
    __syncthreads();
    if (threadIdx.x == 1023) carry += incl;
    __syncthreads();
  }
}

__global__ void csr_filter_scatter_kernel(const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ queries,
                                          int num_rows, int groups, const uint32_t* __restrict__ flag_pair,
                                          const int* __restrict__ gate, const int32_t* __restrict__ row_ptr2,
                                          int32_t* __restrict__ queries2) {
  if (*gate == 0) return;
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < num_rows; row += warps) {
    const int g = row % groups;
    int dst = row_ptr2[row];
    for (int e = row_ptr[row] + lane, end = row_ptr[row + 1]; e - lane < end; e += 32) {
      const int t = e < end ? queries[e] : -1;
      const bool f = t >= 0 && flag_pair[(int64_t)t * groups + g] != 0;
      const unsigned m = __ballot_sync(0xffffffffu, f);
      if (f) queries2[dst + __popc(m & ((1u << lane) - 1))] = t;
      dst += __popc(m);
    }
  }
}

struct FwdWorkspace {
  float* o_acc;
  float* l_acc;
  float* bound;
  int32_t* wave_off;
  int32_t* work_ptr;
  int32_t* block_sums;
  int32_t* item_cell;
  TileMeta* gmeta;
  int32_t* fix_list;   // [1 + rows]: count, then rows for the float64 row kernel
  float* kbmax;        // [num_rows] max |k| per (key block, group)
  float* selmax;       // [pairs] max |k| over a (token, group)'s selected blocks
  uint32_t* flag_pair;  // [pairs] pair re-run by the tensor-core pass
  int32_t* pair_list;   // [1 + pairs]: count, then the flagged pairs
  int32_t* cnt;        // [num_rows] filtered CSR row lengths
  int32_t* row_ptr2;   // [num_rows + 1] filtered CSR
  int32_t* queries2;   // [edges]
  int* fix_count;      // flagged rows after the first pass
  int* err;
  size_t bytes;
};

inline size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

// Query tokens per wave: the wave's slice of the float32 O accumulator is ~32 MB.
inline int wave_tokens_for(int q_heads) {
  int wt = 128;
  while ((int64_t)wt * 2 * q_heads * kD * 4 <= (int64_t)32 << 20) wt *= 2;
  return wt;
}

FwdWorkspace carve_fwd(void* base, int64_t rows, int64_t num_rows, int64_t n_waves, int64_t max_items, int64_t pairs,
                       int64_t edges) {
  FwdWorkspace w{};
  char* b = static_cast<char*>(base);
  w.fix_count = reinterpret_cast<int*>(b);  // fixed header: re-run count, error word
  w.err = reinterpret_cast<int*>(b + 4);
  size_t off = 256;
  w.o_acc = reinterpret_cast<float*>(b + off);
  off = a256(off + sizeof(float) * rows * kD);
  w.l_acc = reinterpret_cast<float*>(b + off);
  off = a256(off + sizeof(float) * rows);
  w.bound = reinterpret_cast<float*>(b + off);
  off = a256(off + sizeof(float) * rows);
  w.fix_list = reinterpret_cast<int32_t*>(b + off);
  off = a256(off + sizeof(int32_t) * (rows + 1));
  w.wave_off = reinterpret_cast<int32_t*>(b + off);
  off = a256(off + sizeof(int32_t) * (n_waves + 1) * num_rows);
  w.work_ptr = reinterpret_cast<int32_t*>(b + off);
  off = a256(off + sizeof(int32_t) * (n_waves * num_rows + 1));
  w.block_sums = reinterpret_cast<int32_t*>(b + off);
  off = a256(off + sizeof(int32_t) * (n_waves * num_rows / kScanCells + 1));
  w.item_cell = reinterpret_cast<int32_t*>(b + off);
  off = a256(off + sizeof(int32_t) * std::max<int64_t>(max_items, 1));
  w.gmeta = reinterpret_cast<TileMeta*>(b + off);
  off = a256(off + sizeof(TileMeta) * std::max<int64_t>(max_items, 1));
  w.kbmax = reinterpret_cast<float*>(b + off);
  off = a256(off + sizeof(float) * std::max<int64_t>(num_rows, 1));
  w.selmax = reinterpret_cast<float*>(b + off);
  off = a256(off + sizeof(float) * std::max<int64_t>(pairs, 1));
  w.flag_pair = reinterpret_cast<uint32_t*>(b + off);
  off = a256(off + sizeof(uint32_t) * std::max<int64_t>(pairs, 1));
  w.pair_list = reinterpret_cast<int32_t*>(b + off);
  off = a256(off + sizeof(int32_t) * (pairs + 1));
  w.cnt = reinterpret_cast<int32_t*>(b + off);
  off = a256(off + sizeof(int32_t) * std::max<int64_t>(num_rows, 1));
  w.row_ptr2 = reinterpret_cast<int32_t*>(b + off);
  off = a256(off + sizeof(int32_t) * (num_rows + 1));
  w.queries2 = reinterpret_cast<int32_t*>(b + off);
  off = a256(off + sizeof(int32_t) * std::max<int64_t>(edges, 1));
  w.bytes = off;
  return w;
}

}  // namespace
}  // namespace msa

using namespace msa;

static int64_t waves_for(int64_t total_tokens, int32_t q_heads) {
  const int wt = wave_tokens_for(q_heads);
  return std::max<int64_t>(1, (total_tokens + wt - 1) / wt);
}

// Selector tokens per 128-row tile: each token takes h rows.
static int tokens_per_chunk(int h) { return 128 / h; }

// Upper bound of work items: every edge fills a chunk slot, every (wave, row) cell adds at most one partial chunk.
static int64_t max_items_for(int64_t total_tokens, int32_t q_heads, int32_t num_rows, int32_t groups, int32_t topk) {
  const int tpc = tokens_per_chunk(q_heads / groups);
  return total_tokens * groups * (int64_t)topk / tpc + waves_for(total_tokens, q_heads) * num_rows + 1;
}

extern "C" size_t msa_attn_fwd_tc_workspace_size(int64_t total_tokens, int32_t q_heads, int32_t num_rows,
                                                 int32_t groups, int32_t topk_blocks) {
  if (groups < 1 || q_heads % groups) return 0;
  return carve_fwd(nullptr, total_tokens * q_heads, num_rows, waves_for(total_tokens, q_heads),
                   max_items_for(total_tokens, q_heads, num_rows, groups, topk_blocks), total_tokens * groups,
                   total_tokens * groups * (int64_t)topk_blocks)
      .bytes;
}

namespace {

// The schedule (query waves x CSR rows -> items with metadata) and the kernel over one CSR.
// Teacher mode (index KL loss): `teacher_bound` is the attention LSE, `slots` the CSR's slot
// indices, `gslot` the per-item slot table and `pt` the output.
struct TeacherPass {
  const float* lse;
  const int32_t* slots;
  int32_t* gslot;
  float* pt;
  int topk;
};

int run_fwd_pass(const CUtensorMap& qmap, const CUtensorMap& kmap, const CUtensorMap& vmap, const FwdWorkspace& w,
                 const void* q, const int32_t* row_ptr, const int32_t* queries, const int32_t* cu_seqlens,
                 const int32_t* cu_block_lens, int nseq, int groups, int q_heads, int h, int tpc, int64_t n_waves,
                 int num_rows, double scale, int cd, int sms, cudaStream_t st, bool timed,
                 const TeacherPass* teacher = nullptr) {
  const int cells = (int)(n_waves * num_rows);
  wave_off_kernel<<<ceil_div((int64_t)(n_waves + 1) * num_rows, 256), 256, 0, st>>>(
      row_ptr, queries, num_rows, (int)n_waves, wave_tokens_for(q_heads), w.wave_off);
  const int scan_blocks = ceil_div((int64_t)cells, kScanCells);
  cell_scan_kernel<<<scan_blocks, kScanCells, 0, st>>>(w.wave_off, cells, num_rows, tpc, w.work_ptr, w.block_sums);
  cell_scan_add_kernel<<<scan_blocks, kScanCells, 0, st>>>(cells, w.block_sums, w.work_ptr);
  item_cell_kernel<<<ceil_div((int64_t)cells, 256), 256, 0, st>>>(w.work_ptr, cells, w.item_cell);
  item_meta_kernel<<<sms * 8, 256, 0, st>>>(w.work_ptr, w.item_cell, w.wave_off, row_ptr, queries, cu_seqlens,
                                            cu_block_lens, nseq, groups, num_rows, cells, tpc, sms, w.gmeta,
                                            teacher ? teacher->slots : nullptr, teacher ? teacher->gslot : nullptr);
  count_launches(5);
  FwdArgs fa{q,       row_ptr,      queries, w.work_ptr, w.wave_off, w.gmeta, cu_seqlens, cu_block_lens,
             teacher ? teacher->lse : w.bound,
             w.l_acc, w.o_acc,      w.err,   nseq,       num_rows,   groups,  q_heads,    h,
             tpc,     (int)n_waves, (float)(scale * 1.4426950408889634), cd,
             teacher ? teacher->gslot : nullptr, teacher ? teacher->pt : nullptr, teacher ? teacher->topk : 0};
  auto kern = teacher ? (h == 4 ? attn_fwd_tc_kernel<true, true> : attn_fwd_tc_kernel<false, true>)
                      : (h == 4 ? attn_fwd_tc_kernel<true> : attn_fwd_tc_kernel<false>);
  MSA_CUDA_RETURN(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemFwd));
  const int slot = timed ? timing_begin(st) : -1;
  kern<<<sms, kFwdThreads, kSmemFwd, st>>>(qmap, kmap, vmap, fa);
  if (timed) timing_end("attn_fwd_tc", slot, st);
  count_launches(1);
  return launch_status(teacher ? "index_kl_teacher_tc" : "attn_fwd_tc");
}

}  // namespace

extern "C" int msa_attn_fwd_tc_range(const void* q, const void* k, const void* v, int dtype, const int32_t* indices,
                                     const int32_t* cu_seqlens, const int32_t* cu_block_lens, const int32_t* row_ptr,
                                     const int32_t* query_indices, int32_t nseq, int64_t total_tokens,
                                     int32_t q_heads, int32_t groups, int32_t head_dim, int32_t topk_blocks,
                                     int32_t block_size, double scale, int32_t num_rows, int64_t q_lo, int64_t q_hi,
                                     void* out, float* lse, void* workspace, size_t workspace_bytes, void* stream) {
  MSA_CHECK_ARG(dtype == MSA_BF16 || dtype == MSA_F16, "msa_attn_fwd_tc: bf16/f16 only");
  MSA_CHECK_ARG(head_dim == kD && block_size == 128, "msa_attn_fwd_tc: head_dim and block_size must be 128");
  MSA_CHECK_ARG(groups >= 1 && q_heads % groups == 0, "msa_attn_fwd_tc: bad head counts");
  const int h = q_heads / groups;
  MSA_CHECK_ARG(h == 4 || h == 8 || h == 16, "msa_attn_fwd_tc: query heads per group must be 4, 8 or 16");
  MSA_CHECK_ARG(q_heads >= 8, "msa_attn_fwd_tc: at least 8 query heads");
  const int tpc = tokens_per_chunk(h);
  MSA_CHECK_ARG(total_tokens < (int64_t)1 << 31 && num_rows >= 0, "msa_attn_fwd_tc: size out of range");
  MSA_CHECK_ARG(0 <= q_lo && q_lo <= q_hi && q_hi <= total_tokens, "msa_attn_fwd_tc: bad query range");
  const int64_t rows = total_tokens * q_heads;
  if (q_hi == q_lo) return MSA_OK;
  const int64_t n_waves = waves_for(total_tokens, q_heads);
  const int64_t pairs = total_tokens * groups;
  const int64_t row0 = q_lo * q_heads, row1 = q_hi * q_heads;
  const FwdWorkspace w = carve_fwd(workspace, rows, num_rows, n_waves,
                                   max_items_for(total_tokens, q_heads, num_rows, groups, topk_blocks), pairs,
                                   pairs * topk_blocks);
  MSA_CHECK_ARG(workspace && workspace_bytes >= w.bytes, "msa_attn_fwd_tc: workspace too small");
  MSA_CHECK_ARG(n_waves * num_rows < (int64_t)1 << 31, "msa_attn_fwd_tc: schedule too large");
  cudaStream_t st = as_stream(stream);
  const int cd = tc::tma_dtype(dtype) == CU_TENSOR_MAP_DATA_TYPE_FLOAT16 ? 1 : 0;

  CUtensorMap qmap, kmap, vmap;
  {
    // Q as 4-D (d_in 64, head, d_out 2, token): one box = 8 head rows x both
    // 64-column halves of one token (2 KB), landing as [d_out][8 rows][128 B].
    const uint64_t dq[4] = {64, (uint64_t)q_heads, 2, (uint64_t)total_tokens};
    const uint64_t sq[3] = {(uint64_t)kD * 2, 128, (uint64_t)q_heads * kD * 2};
    const uint32_t bq[4] = {64, 8, 2, 1};
    if (int e = tc::encode_tensor_map(&qmap, tc::tma_dtype(dtype), 4, q, dq, sq, bq, CU_TENSOR_MAP_SWIZZLE_128B)) return e;
    const uint64_t dk[3] = {(uint64_t)kD, (uint64_t)groups, (uint64_t)total_tokens};
    const uint64_t sk[2] = {(uint64_t)kD * 2, (uint64_t)groups * kD * 2};
    const uint32_t bk[3] = {64, 1, 128};
    if (int e = tc::encode_tensor_map(&kmap, tc::tma_dtype(dtype), 3, k, dk, sk, bk, CU_TENSOR_MAP_SWIZZLE_128B)) return e;
    if (int e = tc::encode_tensor_map(&vmap, tc::tma_dtype(dtype), 3, v, dk, sk, bk, CU_TENSOR_MAP_SWIZZLE_128B)) return e;
  }
  // zero the header (re-run count, error word), the float64 row list count and the pair flags;
  // row_bound_kernel zeroes O_acc and l_acc
  MSA_CUDA_RETURN(cudaMemsetAsync(w.fix_count, 0, 8, st));
  MSA_CUDA_RETURN(cudaMemsetAsync(w.fix_list, 0, 4, st));
  MSA_CUDA_RETURN(cudaMemsetAsync(w.flag_pair, 0, sizeof(uint32_t) * pairs, st));
  MSA_CUDA_RETURN(cudaMemsetAsync(w.pair_list, 0, 4, st));
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (num_rows > 0)
    block_key_norm_kernel<<<ceil_div((int64_t)num_rows * 32, 256), 256, 0, st>>>(k, cd, cu_seqlens, cu_block_lens,
                                                                                nseq, groups, num_rows, w.kbmax);
  selected_key_norm_kernel<<<ceil_div((q_hi - q_lo) * groups, 256), 256, 0, st>>>(
      indices, cu_seqlens, cu_block_lens, nseq, q_lo * groups, q_hi * groups, groups, topk_blocks, w.kbmax, w.selmax);
  row_bound_kernel<<<sms * 8, 256, 0, st>>>(q, cd, row0, row1, q_heads, h, w.selmax, (float)fabs(scale), w.bound,
                                           w.o_acc, w.l_acc);
  count_launches(3);
  if (num_rows > 0) {
    if (int e = run_fwd_pass(qmap, kmap, vmap, w, q, row_ptr, query_indices, cu_seqlens, cu_block_lens, nseq, groups,
                             q_heads, h, tpc, n_waves, num_rows, scale, cd, sms, st, true))
      return e;
  }
  const unsigned fin_grid = (unsigned)ceil_div((row1 - row0) * 16, 256);
  fwd_finalize_kernel<<<fin_grid, 256, 0, st>>>(w.o_acc, w.l_acc, w.bound, row0, row1, q_heads, h, cd, w.err,
                                               w.flag_pair, w.pair_list, w.fix_count, out, lse);
  count_launches(1);
  if (num_rows > 0) {
    // rows whose bound sat too far above their logits: one more tensor-core pass over the
    // filtered CSR of their (token, group) pairs, re-centred (every kernel here returns at
    // once when no row was flagged)
    auto prep = h == 4 ? fix_prepare_kernel<4> : h == 8 ? fix_prepare_kernel<8> : fix_prepare_kernel<16>;
    prep<<<sms * 4, kPrepThreads, 0, st>>>(w.pair_list, groups, q, k, cd, indices, topk_blocks, cu_seqlens, nseq,
                                           (float)scale, w.bound, w.o_acc, w.l_acc);
    csr_filter_count_kernel<<<ceil_div((int64_t)num_rows * 32, 256), 256, 0, st>>>(
        row_ptr, query_indices, num_rows, groups, w.flag_pair, w.fix_count, w.cnt);
    row_scan_kernel<<<1, 1024, 0, st>>>(w.cnt, num_rows, w.row_ptr2);
    csr_filter_scatter_kernel<<<ceil_div((int64_t)num_rows * 32, 256), 256, 0, st>>>(
        row_ptr, query_indices, num_rows, groups, w.flag_pair, w.fix_count, w.row_ptr2, w.queries2);
    count_launches(4);
    if (int e = run_fwd_pass(qmap, kmap, vmap, w, q, w.row_ptr2, w.queries2, cu_seqlens, cu_block_lens, nseq, groups,
                             q_heads, h, tpc, n_waves, num_rows, scale, cd, sms, st, false))
      return e;
    fix_finalize_kernel<<<sms * 2, 256, 0, st>>>(w.o_acc, w.l_acc, w.bound, q_heads, h, cd, w.err, w.pair_list,
                                                 w.fix_list, out, lse);
    count_launches(1);
  }
  if (int e = launch_status("attn_fwd_tc")) return e;
  return launch_fwd_fixup(q, k, v, dtype, indices, cu_seqlens, nseq, q_heads, groups, head_dim, topk_blocks,
                          block_size, scale, w.fix_list, out, lse, st);
}

extern "C" int msa_attn_fwd_tc(const void* q, const void* k, const void* v, int dtype, const int32_t* indices,
                               const int32_t* cu_seqlens, const int32_t* cu_block_lens, const int32_t* row_ptr,
                               const int32_t* query_indices, int32_t nseq, int64_t total_tokens, int32_t q_heads,
                               int32_t groups, int32_t head_dim, int32_t topk_blocks, int32_t block_size, double scale,
                               int32_t num_rows, void* out, float* lse, void* workspace, size_t workspace_bytes,
                               void* stream) {
  return msa_attn_fwd_tc_range(q, k, v, dtype, indices, cu_seqlens, cu_block_lens, row_ptr, query_indices, nseq,
                               total_tokens, q_heads, groups, head_dim, topk_blocks, block_size, scale, num_rows, 0,
                               total_tokens, out, lse, workspace, workspace_bytes, stream);
}

extern "C" int msa_attn_fwd_tc_error(const void* workspace, int64_t total_tokens, int32_t q_heads, int32_t num_rows,
                                     int32_t* host_err) {
  const FwdWorkspace w = carve_fwd(const_cast<void*>(workspace), total_tokens * q_heads, num_rows,
                                   waves_for(total_tokens, q_heads), 0, 0, 0);
  MSA_CUDA_RETURN(cudaMemcpy(host_err, w.err, sizeof(int32_t), cudaMemcpyDeviceToHost));
  return MSA_OK;
}

extern "C" int msa_attn_fwd_tc_rerun_counts(const void* workspace, int64_t total_tokens, int32_t q_heads,
                                            int32_t num_rows, int32_t* rerun_rows, int32_t* f64_rows) {
  const FwdWorkspace w = carve_fwd(const_cast<void*>(workspace), total_tokens * q_heads, num_rows,
                                   waves_for(total_tokens, q_heads), 0, 0, 0);
  MSA_CUDA_RETURN(cudaMemcpy(rerun_rows, w.fix_count, sizeof(int32_t), cudaMemcpyDeviceToHost));
  MSA_CUDA_RETURN(cudaMemcpy(f64_rows, w.fix_list, sizeof(int32_t), cudaMemcpyDeviceToHost));
  return MSA_OK;
}

// ---------------------------------------------------------------- index KL loss: tensor-core teacher
// The KL's teacher probabilities p_T (the group mean of the main attention's
// per-head softmax over the selected keys) for every (pair, selection slot, key):
// the forward kernel in its teacher mode over the same k2q CSR, with the main
// attention's LSE as each row's exponent offset. pt: float32 [T*G][K][128];
// entries of invalid or repeated slots are not written. No counterpart in the
// reference (it specifies the KL loss without a kernel: docs/msa_training_flow.md:92-138).
static size_t teacher_bytes(int64_t total_tokens, int32_t q_heads, int32_t num_rows, int32_t groups,
                            int32_t topk_blocks, FwdWorkspace* w, void* base) {
  const int64_t n_waves = waves_for(total_tokens, q_heads);
  const int64_t items = max_items_for(total_tokens, q_heads, num_rows, groups, topk_blocks);
  FwdWorkspace c = carve_fwd(base, 0, num_rows, n_waves, items, 0, 0);
  const size_t slots_off = a256(c.bytes);
  if (w) {
    *w = c;
    w->cnt = reinterpret_cast<int32_t*>(static_cast<char*>(base) + slots_off);  // reused as the slot table
  }
  return slots_off + sizeof(int32_t) * 32 * (size_t)std::max<int64_t>(items, 1);
}

extern "C" size_t msa_index_kl_teacher_tc_workspace_size(int64_t total_tokens, int32_t q_heads, int32_t num_rows,
                                                         int32_t groups, int32_t topk_blocks) {
  if (groups < 1 || q_heads % groups) return 0;
  return teacher_bytes(total_tokens, q_heads, num_rows, groups, topk_blocks, nullptr, nullptr);
}

extern "C" int msa_index_kl_teacher_tc(const void* q, const void* k, int dtype, const float* lse,
                                       const int32_t* cu_seqlens, const int32_t* cu_block_lens,
                                       const int32_t* row_ptr, const int32_t* query_indices,
                                       const int32_t* slot_indices, int32_t nseq, int64_t total_tokens,
                                       int32_t q_heads, int32_t groups, int32_t head_dim, int32_t topk_blocks,
                                       int32_t block_size, double scale, int32_t num_rows, float* pt,
                                       void* workspace, size_t workspace_bytes, void* stream) {
  MSA_CHECK_ARG(dtype == MSA_BF16 || dtype == MSA_F16, "msa_index_kl_teacher_tc: bf16/f16 only");
  MSA_CHECK_ARG(head_dim == kD && block_size == 128, "msa_index_kl_teacher_tc: head_dim and block_size must be 128");
  MSA_CHECK_ARG(groups >= 1 && q_heads % groups == 0, "msa_index_kl_teacher_tc: bad head counts");
  const int h = q_heads / groups;
  MSA_CHECK_ARG(h == 4 || h == 8 || h == 16, "msa_index_kl_teacher_tc: query heads per group must be 4, 8 or 16");
  MSA_CHECK_ARG(q_heads >= 8, "msa_index_kl_teacher_tc: at least 8 query heads");
  MSA_CHECK_ARG(total_tokens < (int64_t)1 << 31 && num_rows >= 0, "msa_index_kl_teacher_tc: size out of range");
  if (total_tokens == 0 || num_rows == 0) return MSA_OK;
  FwdWorkspace w{};
  const size_t need = teacher_bytes(total_tokens, q_heads, num_rows, groups, topk_blocks, &w, workspace);
  MSA_CHECK_ARG(workspace && workspace_bytes >= need, "msa_index_kl_teacher_tc: workspace too small");
  const int64_t n_waves = waves_for(total_tokens, q_heads);
  MSA_CHECK_ARG(n_waves * num_rows < (int64_t)1 << 31, "msa_index_kl_teacher_tc: schedule too large");
  cudaStream_t st = as_stream(stream);
  const int cd = dtype == MSA_F16 ? 1 : 0;
  CUtensorMap qmap, kmap;
  {
    const uint64_t dq[4] = {64, (uint64_t)q_heads, 2, (uint64_t)total_tokens};
    const uint64_t sq[3] = {(uint64_t)kD * 2, 128, (uint64_t)q_heads * kD * 2};
    const uint32_t bq[4] = {64, 8, 2, 1};
    if (int e = tc::encode_tensor_map(&qmap, tc::tma_dtype(dtype), 4, q, dq, sq, bq, CU_TENSOR_MAP_SWIZZLE_128B)) return e;
    const uint64_t dk[3] = {(uint64_t)kD, (uint64_t)groups, (uint64_t)total_tokens};
    const uint64_t sk[2] = {(uint64_t)kD * 2, (uint64_t)groups * kD * 2};
    const uint32_t bk[3] = {64, 1, 128};
    if (int e = tc::encode_tensor_map(&kmap, tc::tma_dtype(dtype), 3, k, dk, sk, bk, CU_TENSOR_MAP_SWIZZLE_128B)) return e;
  }
  MSA_CUDA_RETURN(cudaMemsetAsync(w.err, 0, 4, st));
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // the teacher mode loads no V: kmap stands in for the V tensor map
  const TeacherPass tp{lse, slot_indices, w.cnt, pt, topk_blocks};
  return run_fwd_pass(qmap, kmap, kmap, w, q, row_ptr, query_indices, cu_seqlens, cu_block_lens, nseq, groups,
                      q_heads, h, 128 / h, n_waves, num_rows, scale, cd, sms, st, false, &tp);
}
