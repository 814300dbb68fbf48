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
// exp(S - bound) >= exp(-2 bound) must stay a normal float for the row maximum.
constexpr float kBoundLimit = 43.0f;
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
};

constexpr int kNQ = 3;  // depth of the Q ring
constexpr int kNM = 4;  // depth of the metadata ring (prefetched two items ahead)

template <bool kRows4>  // h == 4: cp.async gathers into the plain K-major layout
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
  __shared__ uint64_t s_full[2], p_full[2], o_full[2], o_free[2];
  __shared__ uint64_t k_full, k_empty, v_full, v_empty;
  __shared__ int32_t pv_flags[2];
  __shared__ uint32_t tmem_base;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int j = 0; j < kNQ; ++j) {
      mbar_init(&q_full[j], kRows4 ? 32 : 1);  // cp.async: one arrival per producer lane; TMA: expect_tx
      mbar_init(&q_empty[j], 1);
    }
    for (int j = 0; j < kNM; ++j) {
      mbar_init(&meta_full[j], 1);
      mbar_init(&meta_empty[j], 5);  // 4 softmax warps + the S issuer
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&s_full[j], 1);
      mbar_init(&p_full[j], 4);
      mbar_init(&o_full[j], 1);
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
      if (v_loads == kv_loads) return true;
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
        gather_rows4(smem_u32(sQ0 + qs * 32768), 16384, 128, a.q, (int64_t)a.hq * kD, g * 4, t, lane);
        cp_async_arrive_noinc(&q_full[qs]);
        continue;
      }
      const bool mine = t >= 0;
      const uint32_t nv = __popc(__ballot_sync(0xffffffffu, mine));
      if (lane == 0) mbar_arrive_expect_tx(&q_full[qs], nv * (uint32_t)hb * 256u);
      __syncwarp();
      if (mine) {
        uint8_t* dst = sQ0 + qs * 32768 + lane * octets * 2048;
        for (int oc = 0; oc < octets; ++oc)
          tma_load_4d(dst + oc * 2048, &qmap, &q_full[qs], 0, g * h + oc * 8, 0, t);
      }
    }
    if (lane == 0 && ok) service_v(true);  // the last block's V
  } else if (warp == 1 && lane == 0) {
    // ---------------------------------------------------------------- S = Q K^T issuer
    const uint32_t id_s = idesc_f16(!a.f16, 128, 128, false, false);
    const uint32_t sk = smem_u32(sK);
    int k_loads = 0;
    ItemIter it;
    it.start(total_items);
    for (int i = 0; it.valid(); ++i, it.next()) {
      const int qs = i % kNQ, ms = i % kNM, ts = i & 1;
      if (!mbar_wait(&q_full[qs], (i / kNQ) & 1, a.err, 21)) break;
      if (!mbar_wait(&meta_full[ms], (i / kNM) & 1, a.err, 24)) break;
      const int flags = meta[ms].flags;
      mbar_arrive(&meta_empty[ms]);
      const int last = (flags >> 1) & 1;
      if (flags & 1) {
        ++k_loads;
        if (!mbar_wait(&k_full, (k_loads - 1) & 1, a.err, 22)) break;
      }
      if (i >= 2 && !mbar_wait(&o_full[ts], ((i >> 1) - 1) & 1, a.err, 23)) break;  // stage ts's P consumed
      if (kRows4) fence_proxy_async_smem();  // cp.async-written Q tile -> the MMA's operand reads
      tc_fence_after();
      const uint32_t sq = smem_u32(sQ0 + qs * 32768);
      for (int ks = 0; ks < 8; ++ks) {
        const uint64_t da = kRows4 ? desc_kmajor_sw128(sq + (ks >> 2) * 16384 + (ks & 3) * 32)
                                   : desc_kmajor_sw128(sq + (ks >> 2) * 1024 + (ks & 3) * 32, 2048);
        umma_ss(tmem + ts * 256, da, desc_kmajor_sw128(sk + (ks >> 2) * 16384 + (ks & 3) * 32), id_s, ks > 0);
      }
      umma_commit(&s_full[ts]);
      umma_commit(&q_empty[qs]);
      if (last) umma_commit(&k_empty);
    }
  } else if (warp == 2 && lane == 0) {
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
      const int qoff = t - kb0;  // key c of the block is visible iff c <= qoff
      if (!mbar_wait_warp(&s_full[wg], (i >> 1) & 1, a.err, 42)) break;
      tc_fence_after();
      const float nbound = valid ? -bnd * kLog2e : 0.f;
      // P = 2^(s * scale * log2e - bound * log2e); keys past the query (diagonal
      // block only) and rows without a token give 0. ex2.approx: P is rounded to
      // the 16-bit operand type right after.
      float l = 0.f;
      const bool full = qoff >= 127;
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

// Largest |k| over all key rows (float bits are ordered for non-negative values).
// Each warp takes two rows at a time, 16 lanes x 8 elements per row.
__global__ void key_norm_max_kernel(const void* __restrict__ k, int f16, int64_t rows, unsigned* __restrict__ kmax) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  float best = 0.f;
  for (int64_t base = (((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5) * 2; base < rows; base += warps * 2) {
    const int64_t row = base + (lane >> 4);
    const bool in = row < rows;
    const float s = sum16(in ? sq8(k, row * kD + (lane & 15) * 8, f16) : 0.f);
    if (in) best = fmaxf(best, sqrtf(s));
  }
  best = fmaxf(best, __shfl_xor_sync(0xffffffffu, best, 16));
  if (lane == 0) atomicMax(kmax, __float_as_uint(best));
}

// Per query row: bound = |scale| |q| max|k| (slightly inflated so float
// rounding cannot put a logit above it); rows beyond the limit are listed.
// The same pass zeroes the row's O and l accumulators (no separate memset of
// the 1 GB-class accumulator).
__global__ void row_bound_kernel(const void* __restrict__ q, int f16, int64_t rows, const unsigned* __restrict__ kmax,
                                 float abs_scale, float* __restrict__ bound, int32_t* __restrict__ fix_list,
                                 float* __restrict__ o_acc, float* __restrict__ l_acc) {
  const int lane = threadIdx.x & 31;
  const float km = __uint_as_float(*kmax);
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t base = (((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5) * 2; base < rows; base += warps * 2) {
    const int64_t row = base + (lane >> 4);
    const bool in = row < rows;
    const float s = sum16(in ? sq8(q, row * kD + (lane & 15) * 8, f16) : 0.f);
    if (in) {
      float4* z = reinterpret_cast<float4*>(o_acc + row * kD + (lane & 15) * 8);
      z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
      z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (in && (lane & 15) == 0) {
      const float b = abs_scale * sqrtf(s) * km * 1.0001f + 1e-6f;
      bound[row] = b;
      l_acc[row] = 0.f;
      if (b > kBoundLimit) {
        const int slot = atomicAdd(fix_list, 1);
        fix_list[1 + slot] = (int32_t)row;
      }
    }
  }
}

// One warp per item: lane p takes chunk position p (token id, repeated-slot
// check against the previous CSR edge); item_cell gives the item's cell.
__global__ void item_meta_kernel(const int32_t* __restrict__ work_ptr, const int32_t* __restrict__ item_cell,
                                 const int32_t* __restrict__ wave_off, const int32_t* __restrict__ row_ptr,
                                 const int32_t* __restrict__ queries, const int32_t* __restrict__ cu,
                                 const int32_t* __restrict__ cbl, int nseq, int groups, int num_rows, int cells,
                                 int tpc, int grid, TileMeta* __restrict__ gmeta) {
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
    if (lane == 0) {
      m.kb0 = kb0;
      m.g = g;
      m.flags = item_run_flags(item_cell, num_rows, total, grid, w, row);
      m.pad = 0;
    }
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
  int32_t* wave_off;
  int32_t* work_ptr;
  int32_t* block_sums;
  int32_t* item_cell;
  TileMeta* gmeta;
  int32_t* fix_list;
  unsigned* kmax;
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

FwdWorkspace carve_fwd(void* base, int64_t rows, int64_t num_rows, int64_t n_waves, int64_t max_items) {
  FwdWorkspace w{};
  char* b = static_cast<char*>(base);
  w.kmax = reinterpret_cast<unsigned*>(b);  // fixed header: max |k|, error word
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
                   max_items_for(total_tokens, q_heads, num_rows, groups, topk_blocks))
      .bytes;
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
  MSA_CHECK_ARG(q_heads >= 8, "msa_attn_fwd_tc: at least 8 query heads");
  const int tpc = tokens_per_chunk(h);
  MSA_CHECK_ARG(total_tokens < (int64_t)1 << 31 && num_rows >= 0, "msa_attn_fwd_tc: size out of range");
  const int64_t rows = total_tokens * q_heads;
  if (rows == 0) return MSA_OK;
  const int64_t n_waves = waves_for(total_tokens, q_heads);
  const FwdWorkspace w =
      carve_fwd(workspace, rows, num_rows, n_waves, max_items_for(total_tokens, q_heads, num_rows, groups, topk_blocks));
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
  // zero the header (max |k|, error word) and the fixup count; row_bound_kernel zeroes O_acc and l_acc
  MSA_CUDA_RETURN(cudaMemsetAsync(w.kmax, 0, 8, st));
  MSA_CUDA_RETURN(cudaMemsetAsync(w.fix_list, 0, 4, st));
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  key_norm_max_kernel<<<sms * 4, 256, 0, st>>>(k, cd, total_tokens * groups, w.kmax);
  row_bound_kernel<<<sms * 8, 256, 0, st>>>(q, cd, rows, w.kmax, (float)fabs(scale), w.bound, w.fix_list, w.o_acc,
                                           w.l_acc);
  count_launches(2);
  if (num_rows > 0) {
    const int cells = (int)(n_waves * num_rows);
    wave_off_kernel<<<ceil_div((int64_t)(n_waves + 1) * num_rows, 256), 256, 0, st>>>(
        row_ptr, query_indices, num_rows, (int)n_waves, wave_tokens_for(q_heads), w.wave_off);
    const int scan_blocks = ceil_div((int64_t)cells, kScanCells);
    cell_scan_kernel<<<scan_blocks, kScanCells, 0, st>>>(w.wave_off, cells, num_rows, tpc, w.work_ptr, w.block_sums);
    cell_scan_add_kernel<<<scan_blocks, kScanCells, 0, st>>>(cells, w.block_sums, w.work_ptr);
    item_cell_kernel<<<ceil_div((int64_t)cells, 256), 256, 0, st>>>(w.work_ptr, cells, w.item_cell);
    item_meta_kernel<<<sms * 8, 256, 0, st>>>(w.work_ptr, w.item_cell, w.wave_off, row_ptr, query_indices,
                                              cu_seqlens, cu_block_lens, nseq, groups, num_rows, cells, tpc, sms,
                                              w.gmeta);
    count_launches(5);
    FwdArgs fa{q,        row_ptr,       query_indices, w.work_ptr, w.wave_off, w.gmeta, cu_seqlens, cu_block_lens, w.bound,
               w.l_acc,  w.o_acc,       w.err,      nseq,       num_rows, groups,     q_heads,       h,
               tpc,      (int)n_waves,  (float)(scale * 1.4426950408889634), cd};
    auto kern = h == 4 ? attn_fwd_tc_kernel<true> : attn_fwd_tc_kernel<false>;
    MSA_CUDA_RETURN(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemFwd));
    const int slot = timing_begin(st);
    kern<<<sms, kFwdThreads, kSmemFwd, st>>>(qmap, kmap, vmap, fa);
    timing_end("attn_fwd_tc", slot, st);
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
  const FwdWorkspace w = carve_fwd(const_cast<void*>(workspace), total_tokens * q_heads, num_rows,
                                   waves_for(total_tokens, q_heads), 0);
  MSA_CUDA_RETURN(cudaMemcpy(host_err, w.err, sizeof(int32_t), cudaMemcpyDeviceToHost));
  return MSA_OK;
}
