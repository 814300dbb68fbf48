// Sparse attention backward, tensor-core path (sm_100a: TMA + tcgen05 + TMEM).
//
// dK/dV -- key-block stationary, deterministic, no floating-point atomics
// (the role of _backward_kv_kernel, triton/sparse_attention.py:223-296). One
// CTA owns one k2q CSR row (128-key block b, group g) at a time and walks the
// row's selecting tokens in tiles of 64 rows ((token, head) pairs, gathered
// with TMA). Keys are the MMA's M:
//   S^T  = K_b Q^T,  dP^T = V_b dO^T                         TMEM (f32)
//   P^T  = exp(scale S^T - lse),  dS^T = P^T (dP^T - delta)    softmax warps
//   dV  += P^T dO,  dK += dS^T Q    (P^T, dS^T packed into TMEM: A operands)
// dV and dK stay in TMEM for the whole row; its last tile writes dK * scale and
// dV for the block's keys. Rows are taken from a global counter in CSR order.
//
// dQ -- the role of the query-owned dQ of _backward_kernel
// (triton/sparse_attention.py:87-199), on the forward's schedule (query waves x
// key blocks, chunks of 128 rows):
//   S = Q K_b^T, dP = dO V_b^T, dS = P (dP - delta) -> TMEM, dQ_e = dS K_b,
//   dQ_acc[t, heads] += dQ_e (float32 reductions), dq = scale * dQ_acc.
// delta = rowsum(dO * O) over the stored output (bwd_prep_kernel); the
// reference's center (sum(output * grad_output), sparse_attention.py:112).
#include <algorithm>

#include "attn_common.cuh"

namespace msa {
namespace {

using namespace tc;
using namespace attn;

constexpr int kD = 128;

// ---------------------------------------------------------------- prep
// delta[row] = sum_d dO * O, nlse2[row] = -lse * log2(e) (0 for rows without
// keys: every P of such a row is masked to 0). dq_acc (when dQ is requested):
// the same pass zeroes the row's float32 dQ accumulator.
__global__ void bwd_prep_kernel(const void* __restrict__ out, const void* __restrict__ dout,
                                const float* __restrict__ lse, int64_t row0, int64_t rows, int f16,
                                float* __restrict__ delta, float* __restrict__ nlse2, float* __restrict__ dq_acc) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t row = row0 + (idx >> 4);
  const int c = (int)(idx & 15);
  float acc = 0.f;
  if (row < rows && dq_acc) {
    float4* z = reinterpret_cast<float4*>(dq_acc + row * kD + c * 8);
    z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (row < rows) {
    const uint4 o = *reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(out) + (row * kD + c * 8) * 2);
    const uint4 g = *reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(dout) + (row * kD + c * 8) * 2);
    const uint32_t ov[4] = {o.x, o.y, o.z, o.w}, gv[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 a, b;
      if (f16) {
        a = __half22float2(*reinterpret_cast<const __half2*>(&ov[i]));
        b = __half22float2(*reinterpret_cast<const __half2*>(&gv[i]));
      } else {
        a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ov[i]));
        b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gv[i]));
      }
      acc = fmaf(a.x, b.x, fmaf(a.y, b.y, acc));
    }
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (row < rows && c == 0) {
    delta[row] = acc;
    const float l = lse[row];
    nlse2[row] = l == -INFINITY ? 0.f : -l * kLog2e;
  }
}

// ================================================================ dK / dV
constexpr int kKvThreads = 384;
constexpr int kKvNQ = 4;     // Q/dO tile ring (32 KB per tile)
constexpr int kKvNQDq = 3;   // the same ring when the kernel also produces dQ (two 16 KB dS tiles take the room)
constexpr int kKvNM = 8;     // metadata ring (the tile in softmax, the issuer's, the producer's look-ahead)
constexpr int kKvSmem = kKvNQ * 32768 + 2 * 32768 + 1024;
constexpr int kKvSmemDq = kKvNQDq * 32768 + 2 * 32768 + 2 * 16384 + 1024;
constexpr int kDone = 4;  // metadata flag: no more tiles for this CTA
constexpr int kFull = 8;  // metadata flag: every tile row has a token that sees the whole key block

// Tile metadata, built in shared memory by the kernel's metadata warp: a tile
// is 64 / h consecutive selecting tokens of one CSR row (tile row = position *
// h + head).
struct __align__(16) KvTileMeta {
  int32_t tok[16];   // token per tile position (-1: none, or a repeated selection)
  float nlse2[64];   // per tile row
  float delta[64];
  int32_t qoff[64];  // token - first key of the block; -1 for rows without a token
  int32_t kb0, g;
  int32_t flags;     // bit 0: first tile of the row, bit 1: last, bit 2: done, bit 3: full
  int32_t kend;      // keys of the block inside its sequence
};
static_assert(sizeof(KvTileMeta) % 16 == 0, "vector loads of the per-row arrays");
constexpr int kMetaBatch = 4;  // tiles whose metadata loads are issued together

struct KvArgs {
  const void* q;            // [T][Hq][128] and the output gradient, read directly by the
  const void* dout;         // 4-heads-per-group gather
  const int32_t* row_ptr;   // k2q CSR
  const int32_t* queries;
  const int32_t* cu;        // cu_seqlens
  const int32_t* cbl;       // cu_block_lens
  const float* nlse2;       // [T*Hq] -lse * log2(e)
  const float* delta;       // [T*Hq]
  int* row_counter;         // CSR rows taken so far (dynamic schedule)
  int* err;
  void* dk;
  void* dv;
  int nseq, num_rows, groups, hq, h;
  float scale_log2, scale;
  int f16;
  int kv_f32;     // 1: dk / dv are float32 (context-parallel partial sums), else the input dtype
  float* dq_acc;  // [T*Hq][128] float32 dS.K sums (the kDq variant only)
};

__device__ __forceinline__ void store_row32(void* base, int64_t elem_off, const uint32_t (&v)[32], float mul,
                                            int f16, int f32) {
  if (f32) {
    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(base) + elem_off);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      dst[i] = make_float4(__uint_as_float(v[4 * i]) * mul, __uint_as_float(v[4 * i + 1]) * mul,
                           __uint_as_float(v[4 * i + 2]) * mul, __uint_as_float(v[4 * i + 3]) * mul);
    return;
  }
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) w[i] = pack2(__uint_as_float(v[2 * i]) * mul, __uint_as_float(v[2 * i + 1]) * mul, f16);
  uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(base) + elem_off * 2);
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// Softmax of one 64-row tile for one key (thread): P^T and dS^T of its 64 rows,
// packed in pairs of rows. kMasked: rows without a token or with keys past
// their token (qoff < key) give 0.
template <bool kMasked>
__device__ __forceinline__ void kv_softmax_half(const KvTileMeta& m, int half, int key, float scale_log2, int f16,
                                                const uint32_t (&s)[32], const uint32_t (&dp)[32], uint32_t (&pp)[16],
                                                uint32_t (&ds)[16]) {
#pragma unroll
  for (int c = 0; c < 32; c += 4) {
    const int r = half * 32 + c;
    const float4 nl = *reinterpret_cast<const float4*>(&m.nlse2[r]);
    const float4 dl = *reinterpret_cast<const float4*>(&m.delta[r]);
    const float nls[4] = {nl.x, nl.y, nl.z, nl.w}, dls[4] = {dl.x, dl.y, dl.z, dl.w};
    int qos[4] = {0, 0, 0, 0};
    if (kMasked) {
      const int4 qo = *reinterpret_cast<const int4*>(&m.qoff[r]);
      qos[0] = qo.x; qos[1] = qo.y; qos[2] = qo.z; qos[3] = qo.w;
    }
    float p[4], d[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float e = ex2_approx(fmaf(__uint_as_float(s[c + u]), scale_log2, nls[u]));
      const float g = __uint_as_float(dp[c + u]) - dls[u];
      if (kMasked) {
        const bool v = key <= qos[u];
        p[u] = v ? e : 0.f;
        d[u] = v ? e * g : 0.f;
      } else {
        p[u] = e;
        d[u] = e * g;
      }
    }
    pp[c >> 1] = pack2(p[0], p[1], f16);
    pp[(c >> 1) + 1] = pack2(p[2], p[3], f16);
    ds[c >> 1] = pack2(d[0], d[1], f16);
    ds[(c >> 1) + 1] = pack2(d[2], d[3], f16);
  }
}

// Roles (384 threads): warp 0 = TMA producer, warp 1 (one lane) = S^T/dP^T
// issuer, warp 2 (one lane) = dV/dK issuer (two issuing threads keep the tensor
// pipe fed while either one waits), warps 4-7 and 8-11 = two softmax
// warpgroups (thread = key of the block) taking
// alternate tiles, each with its own TMEM stage; the warpgroup that takes a
// row's last tile writes the row's dK/dV.
// TMEM: stage j = tile parity: S^T at 128 j (64 columns), dP^T at 128 j + 64.
// The softmax packs P^T and dS^T (two rows per column) over the S^T columns it
// has read: rows 0-31 -> P^T at +0, dS^T at +16; rows 32-63 -> +32, +48. dV at
// 256, dK at 384. Both accumulation MMAs take A from TMEM.
// kDq (dQ in the same pass, no recomputation): the softmax also writes dS^T to
// shared memory (key-major rows of 64 tile rows, the MN-major B operand), the
// accumulation issuer adds dQ^T = K^T dS^T (M = 128 head dims, N = 64 tile
// rows; A = the K tile read MN-major) into the stage's dP^T columns, and the
// warpgroup drains it into the float32 dQ accumulator with red.global.add.
template <bool kDq, bool kRows4>
__global__ void __launch_bounds__(kKvThreads, 1)
attn_dkdv_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap domap,
                    const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, KvArgs a) {
  constexpr int kNQ = kDq ? kKvNQDq : kKvNQ;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  // ring tile: Q (8 blocks of 2 KB = 8 head rows x 2 d-chunks x 128 B) then dO, same layout
  uint8_t* sT0 = smem;
  uint8_t* sK = smem + kNQ * 32768;  // 2 d-chunks x 128 keys x 128 B
  uint8_t* sV = sK + 32768;
  // kDq: per stage, dS^T as 128 key rows x 128 B (64 tile rows), 128-byte swizzle;
  // after the stage's dQ MMA the same 16 KB holds the warpgroup's dQ transposes
  uint8_t* sDS = sV + 32768;
  __shared__ KvTileMeta meta[kKvNM];
  __shared__ int32_t tile_rowno[kKvNM];  // ordinal (in this CTA) of the row the slot's tile belongs to
  __shared__ uint64_t q_full[kNQ], q_empty[kNQ], meta_full[kKvNM], meta_empty[kKvNM];
  __shared__ uint64_t st_full[2], p_full[2], acc_done[2], acc_full[2], dq_free[2], kv_full, kv_empty, acc_free;
  __shared__ uint32_t tmem_base;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // h >= 8: TMA gathers each token's h rows of Q / dO as 8-row swizzle atoms (2 KB
  // per 8 heads, SBO 2048). h = 4: 16 tokens x 4 heads copied with cp.async into
  // the plain K-major layout (8-row groups 1024 B apart, halves 8 KB apart).
  constexpr bool rows4 = kRows4;  // h == 4
  const int h = a.h, hb = h, tpc = 64 / hb, octets = hb / 8;
  if (threadIdx.x == 0) {
    for (int j = 0; j < kNQ; ++j) {
      mbar_init(&q_full[j], kRows4 ? 64 : 1);  // cp.async: one arrival per lane of both copying warps; TMA: expect_tx
      mbar_init(&q_empty[j], 1);
    }
    for (int j = 0; j < kKvNM; ++j) {
      mbar_init(&meta_full[j], 1);
      mbar_init(&meta_empty[j], 6);  // the 4 warps of the tile's softmax warpgroup + both MMA issuers
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&st_full[j], 1);
      mbar_init(&p_full[j], 4);
      mbar_init(&acc_done[j], 1);
      mbar_init(&acc_full[j], 1);  // row parity: completes once per two rows
      mbar_init(&dq_free[j], 4);   // kDq: the warpgroup has read the stage's dQ^T
    }
    mbar_init(&kv_full, 1);
    mbar_init(&kv_empty, 1);
    mbar_init(&acc_free, 4);
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

  if (warp == 0) {
    // ---------------------------------------------------------------- producer (whole warp)
    // Per tile (metadata from warp 3): K/V on a new row, then one lane per token
    // gathers the tile's Q / dO rows.
    if (lane == 0) {
      tma_prefetch_desc(&qmap);
      tma_prefetch_desc(&domap);
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
    }
    bool ok = true;
    int kv_rows = 0;
    for (int ti = 0;; ++ti) {
      const int ms = ti % kKvNM, qs = ti % kNQ;
      if (!mbar_wait_warp(&meta_full[ms], (ti / kKvNM) & 1, a.err, 52)) break;
      const int flags = meta[ms].flags;
      if (flags & kDone) break;
      const int t = lane < (kRows4 ? 16 : 8) ? meta[ms].tok[lane] : -1;
      const int g = meta[ms].g, kb0 = meta[ms].kb0;
      if (lane == 0) {
        if (flags & 1) {  // new key block: K/V once the previous row's last S^T/dP^T are done
          if (kv_rows > 0) ok = mbar_wait(&kv_empty, (kv_rows - 1) & 1, a.err, 53);
          if (ok) {
            mbar_arrive_expect_tx(&kv_full, 65536);
            tma_load_3d(sK, &kmap, &kv_full, 0, g, kb0);
            tma_load_3d(sK + 16384, &kmap, &kv_full, 64, g, kb0);
            tma_load_3d(sV, &vmap, &kv_full, 0, g, kb0);
            tma_load_3d(sV + 16384, &vmap, &kv_full, 64, g, kb0);
          }
          ++kv_rows;
        }
        if (ok && ti >= kNQ) ok = mbar_wait(&q_empty[qs], ((ti / kNQ) - 1) & 1, a.err, 54);
        if (ok && !kRows4) mbar_arrive_expect_tx(&q_full[qs], (uint32_t)tpc * hb * 512u);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      if (kRows4) {
        // cp.async gather of Q here and of dO (16 KB further) by the metadata warp; each
        // lane's copies arrive on q_full when they land (the MMA issuers fence them for
        // the async proxy)
        gather_rows4(smem_u32(sT0 + qs * 32768), 8192, 64, a.q, (int64_t)a.hq * kD, g * 4, t, lane);
        cp_async_arrive_noinc(&q_full[qs]);
        continue;
      }
      if (lane < tpc) {
        // Positions without a token load from token -1: out of range, so their
        // rows are zero-filled and contribute nothing to dK/dV.
        uint8_t* dst = sT0 + qs * 32768 + lane * octets * 2048;
        for (int oc = 0; oc < octets; ++oc) {
          tma_load_4d(dst + oc * 2048, &qmap, &q_full[qs], 0, g * h + oc * 8, 0, t);
          tma_load_4d(dst + 16384 + oc * 2048, &domap, &q_full[qs], 0, g * h + oc * 8, 0, t);
        }
      }
    }
  } else if (warp == 3) {
    // ---------------------------------------------------------------- tile metadata (whole warp)
    // Takes CSR rows from the global counter and writes each tile's metadata
    // into the ring: up to kMetaBatch tiles at a time, lane j holding position
    // j % tpc of tile j / tpc, so the token loads and then the per-row lse /
    // delta loads of the batch each take one round trip.
    const uint32_t all = 0xffffffffu;
    int ip = 0, rowno = -1;
    bool ok = true;
    while (ok) {
      int r = 0;
      if (lane == 0) r = atomicAdd(a.row_counter, 1);
      r = __shfl_sync(all, r, 0);
      if (r >= a.num_rows) break;
      const int e_begin = a.row_ptr[r], e_end = a.row_ptr[r + 1];
      if (e_begin >= e_end) continue;
      ++rowno;
      const int gb = r / a.groups, g = r - gb * a.groups;
      const int sq = block_sequence(a.cbl, a.nseq, gb);
      const int kb0 = a.cu[sq] + (gb - a.cbl[sq]) * 128;
      const int kend = min(128, a.cu[sq + 1] - kb0);
      const int ntiles = (e_end - e_begin + tpc - 1) / tpc;
      constexpr int batch = kRows4 ? 2 : kMetaBatch;  // tiles per batch: batch * tpc <= 32 lanes
      for (int k0 = 0; k0 < ntiles; k0 += batch) {
        const int nb = min(batch, ntiles - k0);
        const int e0 = e_begin + k0 * tpc, e = e0 + lane;
        int t = (lane < nb * tpc && e < e_end) ? a.queries[e] : -1;
        int prev = __shfl_up_sync(all, t, 1);
        if (lane == 0) prev = e0 > e_begin ? a.queries[e0 - 1] : -1;
        t = (t >= 0 && t != prev) ? t : -1;  // a repeated selection of the block counts once
        float nl[kMetaBatch][2], dl[kMetaBatch][2];
        int qo[kMetaBatch][2];
#pragma unroll
        for (int kk = 0; kk < kMetaBatch; ++kk) {
#pragma unroll
          for (int hr = 0; hr < 2; ++hr) {
            const int rr = lane + hr * 32, pos = rr / hb, hh = rr - pos * hb;
            const int tr = __shfl_sync(all, t, (kk * tpc + pos) & 31);
            const bool real = kk < nb && tr >= 0 && hh < h;
            const int64_t rowid = (int64_t)tr * a.hq + g * h + hh;
            nl[kk][hr] = real ? a.nlse2[rowid] : 0.f;
            dl[kk][hr] = real ? a.delta[rowid] : 0.f;
            qo[kk][hr] = real ? tr - kb0 : -1;
          }
        }
        // kFull skips the per-row mask, so tiles with masked head rows never take it
        const unsigned sees_all = __ballot_sync(all, lane < nb * tpc && t >= 0 && t - kb0 >= 127 && hb == h);
        for (int kk = 0; kk < nb && ok; ++kk) {
          const int slot = ip + kk, ms = slot % kKvNM;
          if (slot >= kKvNM && !mbar_wait_warp(&meta_empty[ms], ((slot / kKvNM) - 1) & 1, a.err, 56)) {
            ok = false;
            break;
          }
          const int tk = __shfl_sync(all, t, (kk * tpc + (lane & 15)) & 31);
          KvTileMeta& m = meta[ms];
          if (lane < 16) m.tok[lane] = lane < tpc ? tk : -1;
#pragma unroll
          for (int q = 0; q < kMetaBatch; ++q) {
            if (q == kk) {  // static register indexing
              m.nlse2[lane] = nl[q][0];
              m.nlse2[lane + 32] = nl[q][1];
              m.delta[lane] = dl[q][0];
              m.delta[lane + 32] = dl[q][1];
              m.qoff[lane] = qo[q][0];
              m.qoff[lane + 32] = qo[q][1];
            }
          }
          if (lane == 0) {
            const unsigned tile_bits = (sees_all >> (kk * tpc)) & ((1u << tpc) - 1u);
            m.kb0 = kb0;
            m.g = g;
            m.kend = kend;
            m.flags = (k0 + kk == 0 ? 1 : 0) | (k0 + kk == ntiles - 1 ? 2 : 0) |
                      (tile_bits == (1u << tpc) - 1u ? kFull : 0);
            tile_rowno[ms] = rowno;
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&meta_full[ms]);  // releases the warp's stores above
          if (kRows4) {
            // 4 heads per group: this warp copies the tile's dO rows once its ring slot is
            // free (64 cp.async steps per tile from the producer alone set the tile rate)
            const int qs = slot % kNQ;
            if (slot >= kNQ && !mbar_wait_warp(&q_empty[qs], ((slot / kNQ) - 1) & 1, a.err, 58)) {
              ok = false;
              break;
            }
            gather_rows4(smem_u32(sT0 + qs * 32768) + 16384, 8192, 64, a.dout, (int64_t)a.hq * kD, g * 4,
                         lane < tpc ? tk : -1, lane);
            cp_async_arrive_noinc(&q_full[qs]);
          }
        }
        ip += nb;
        if (!ok) break;
      }
    }
    // End of work: "done" entries in the next two slots, one for each softmax warpgroup.
    for (int d = 0; d < 2 && ok; ++d, ++ip) {
      const int ms = ip % kKvNM;
      if (ip >= kKvNM && !mbar_wait_warp(&meta_empty[ms], ((ip / kKvNM) - 1) & 1, a.err, 55)) break;
      if (lane == 0) {
        meta[ms].flags = kDone;
        mbar_arrive(&meta_full[ms]);
      }
      __syncwarp();
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------------------------------------------------------- S^T = K Q^T, dP^T = V dO^T
    const uint32_t id_t = idesc_f16(!a.f16, 128, 64, false, false);  // M keys, N 64 rows, K d
    const uint32_t sk = smem_u32(sK), sv = smem_u32(sV);
    int rows = 0;
    for (int ti = 0;; ++ti) {
      const int ms = ti % kKvNM, qs = ti % kNQ, j = ti & 1;
      if (!mbar_wait(&meta_full[ms], (ti / kKvNM) & 1, a.err, 63)) break;
      const int flags = meta[ms].flags;
      if (flags & kDone) break;
      mbar_arrive(&meta_empty[ms]);
      if (flags & 1) {
        if (!mbar_wait(&kv_full, rows & 1, a.err, 64)) break;
        ++rows;
      }
      if (!mbar_wait(&q_full[qs], (ti / kNQ) & 1, a.err, 65)) break;
      // stage j was last used by tile ti - 2: its accumulation MMAs read its P^T and dS^T
      // (kDq: and its warpgroup has read the dQ^T that followed them)
      if (ti >= 2 && !mbar_wait(kDq ? &dq_free[j] : &acc_done[j], ((ti >> 1) - 1) & 1, a.err, 66)) break;
      if (kRows4) fence_proxy_async_smem();  // cp.async-written Q / dO tiles -> the MMAs' operand reads
      tc_fence_after();
      const uint32_t st = smem_u32(sT0 + qs * 32768);
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t ka = (ks >> 2) * 16384 + (ks & 3) * 32;
        constexpr uint32_t sbo = kRows4 ? 1024 : 2048;
        const uint32_t kb = kRows4 ? (ks >> 2) * 8192 + (ks & 3) * 32 : (ks >> 2) * 1024 + (ks & 3) * 32;
        umma_ss(tmem + 128 * j, desc_kmajor_sw128(sk + ka), desc_kmajor_sw128(st + kb, sbo), id_t, ks > 0);
        umma_ss(tmem + 128 * j + 64, desc_kmajor_sw128(sv + ka), desc_kmajor_sw128(st + 16384 + kb, sbo), id_t,
                ks > 0);
      }
      umma_commit(&st_full[j]);
      if (!kDq && (flags & 2)) umma_commit(&kv_empty);  // K/V are read by S^T/dP^T only (kDq: K also by dQ^T)
    }
  } else if (warp == 2 && lane == 0) {
    // ---------------------------------------------------------------- dV += P^T dO, dK += dS^T Q
    const uint32_t id_acc = idesc_f16(!a.f16, 128, 128, false, true);  // M keys, N d, K rows
    const uint32_t id_dq = idesc_f16(!a.f16, 128, 64, true, true);     // M d, N 64 rows, K keys
    const uint32_t sk = smem_u32(sK), sds = smem_u32(sDS);
    int rows_done = 0;
    for (int t = 0;; ++t) {
      const int ms = t % kKvNM, qs = t % kNQ, j = t & 1;
      if (!mbar_wait(&meta_full[ms], (t / kKvNM) & 1, a.err, 67)) break;
      const int flags = meta[ms].flags;
      if (flags & kDone) break;
      mbar_arrive(&meta_empty[ms]);
      if (!mbar_wait(&p_full[j], (t >> 1) & 1, a.err, 61)) break;
      if ((flags & 1) && rows_done > 0 && !mbar_wait(&acc_free, (rows_done - 1) & 1, a.err, 62)) break;
      if (kRows4) fence_proxy_async_smem();
      tc_fence_after();
      const uint32_t st = smem_u32(sT0 + qs * 32768);
      for (int ks = 0; ks < 4; ++ks) {  // K = 64 tile rows, 16 per step (two 8-row blocks of 2 KB)
        const uint32_t acc = ((flags & 1) && ks == 0) ? 0u : 1u;
        const uint32_t pcol = tmem + 128 * j + (ks >> 1) * 32 + (ks & 1) * 8;  // P^T; dS^T at +16
        // B = the dO / Q tile read MN-major (N = head dims, K = 16 tile rows per step)
        const uint64_t bdo = kRows4 ? desc_mnmajor_sw128(st + 16384 + ks * 2048, 8192, 1024)
                                   : desc_mnmajor_sw128(st + 16384 + ks * 4096, 1024, 2048);
        const uint64_t bq = kRows4 ? desc_mnmajor_sw128(st + ks * 2048, 8192, 1024)
                                  : desc_mnmajor_sw128(st + ks * 4096, 1024, 2048);
        umma_ts(tmem + 256, pcol, bdo, id_acc, acc);
        umma_ts(tmem + 384, pcol + 16, bq, id_acc, acc);
      }
      umma_commit(&q_empty[qs]);
      if (flags & 2) {
        umma_commit(&acc_full[rows_done & 1]);
        ++rows_done;
      }
      if (kDq) {  // dQ^T = K^T dS^T into the stage's dP^T columns (already read by the softmax)
        const uint32_t sb = sds + j * 16384;
        for (int ks = 0; ks < 8; ++ks)
          umma_ss(tmem + 128 * j + 64, desc_mnmajor_sw128(sk + ks * 2048, 16384), desc_mnmajor_sw128(sb + ks * 2048, 16384),
                  id_dq, ks > 0);
      }
      umma_commit(&acc_done[j]);
      if (kDq && (flags & 2)) umma_commit(&kv_empty);
    }
  } else if (warp >= 4) {
    // ---------------------------------------------------------------- softmax + dK/dV epilogue
    const int wg = (warp - 4) >> 2, qd = warp & 3;
    const int key = qd * 32 + lane;  // TMEM lane == key of the block
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const uint32_t t_st = tmem + 128 * wg + lane_base;
    uint8_t* my_ds = sDS + wg * 16384 + qd * 4096;  // kDq: this warp's 32 key rows of dS^T
    for (int ti = wg;; ti += 2) {
      const int ms = ti % kKvNM;
      if (!mbar_wait_warp(&meta_full[ms], (ti / kKvNM) & 1, a.err, 71)) break;
      const KvTileMeta& m = meta[ms];
      const int flags = m.flags;
      if (flags & kDone) break;
      const int kb0 = m.kb0, g = m.g, kend = m.kend, rowno = tile_rowno[ms];
      // kDq: dQ accumulator row of tile rows lane and lane + 32 (-1: no token or a masked head)
      int32_t dq_row0 = -1, dq_row1 = -1;
      if (kDq) {
        const int r0 = lane, r1 = lane + 32;
        const int t0 = m.tok[r0 / hb], t1 = m.tok[r1 / hb];
        const int h0 = r0 % hb, h1 = r1 % hb;
        dq_row0 = (t0 >= 0 && h0 < h) ? t0 * (a.groups * h) + g * h + h0 : -1;
        dq_row1 = (t1 >= 0 && h1 < h) ? t1 * (a.groups * h) + g * h + h1 : -1;
      }
      if (!mbar_wait_warp(&st_full[wg], (ti >> 1) & 1, a.err, 72)) break;
      tc_fence_after();
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        uint32_t s[32], dp[32], pp[16], ds[16];
        tmem_ld32(t_st + half * 32, s);
        tmem_ld32(t_st + 64 + half * 32, dp);
        tmem_wait_ld();
        if (flags & kFull)
          kv_softmax_half<false>(m, half, key, a.scale_log2, a.f16, s, dp, pp, ds);
        else
          kv_softmax_half<true>(m, half, key, a.scale_log2, a.f16, s, dp, pp, ds);
        // packed over S^T columns this thread already read, leaving dP^T's columns free for dQ^T
        tmem_st16(t_st + half * 32, pp);
        tmem_st16(t_st + half * 32 + 16, ds);
        if (kDq) {
          // key row: 64 tile rows = 8 chunks of 16 B, chunk u stored at u ^ (key & 7) (128-byte swizzle)
          uint8_t* row = my_ds + (lane >> 3) * 1024 + (lane & 7) * 128;
#pragma unroll
          for (int u = 0; u < 4; ++u)
            *reinterpret_cast<uint4*>(row + (((half * 4 + u) ^ (lane & 7)) << 4)) =
                make_uint4(ds[4 * u], ds[4 * u + 1], ds[4 * u + 2], ds[4 * u + 3]);
        }
      }
      tmem_wait_st();
      if (kDq) fence_proxy_async_smem();  // dS^T stores -> the dQ MMA's operand reads
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&p_full[wg]);
        mbar_arrive(&meta_empty[ms]);
      }
      if (flags & 2) {  // last tile of the row: dK, dV of this block's keys
        if (!mbar_wait_warp(&acc_full[rowno & 1], (rowno >> 1) & 1, a.err, 73)) break;
        tc_fence_after();
        const bool inside = key < kend;
        const int64_t off = ((int64_t)(kb0 + key) * a.groups + g) * kD;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          uint32_t vv[32], kk[32];
          tmem_ld32(tmem + 256 + lane_base + c4 * 32, vv);
          tmem_ld32(tmem + 384 + lane_base + c4 * 32, kk);
          tmem_wait_ld();
          if (inside) {
            if (a.dv) store_row32(a.dv, off + c4 * 32, vv, 1.f, a.f16, a.kv_f32);
            if (a.dk) store_row32(a.dk, off + c4 * 32, kk, a.scale, a.f16, a.kv_f32);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_free);
      }
      if (kDq) {
        // dQ^T (lane = head dim 32 qd + lane, column = tile row) -> dQ accumulator rows:
        // a 32 x 32 transpose through this warp's 4 KB of the stage's dS^T space (the
        // MMA that read it is complete), then one red.v4 covers 4 rows x 128 B.
        if (!mbar_wait_warp(&acc_done[wg], (ti >> 1) & 1, a.err, 74)) break;
        tc_fence_after();
        float* xs = reinterpret_cast<float*>(my_ds);
        const int sub_row = lane >> 3, sub_c = lane & 7;
        // both halves out of TMEM first, so the stage goes back to the S^T/dP^T issuer
        // before the transposes and reductions (the stage's cycle bounds the kernel)
        uint32_t v0[32], v1[32];
        tmem_ld32(t_st + 64, v0);
        tmem_ld32(t_st + 64 + 32, v1);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dq_free[wg]);
        auto drain_half = [&](const uint32_t (&v)[32], int32_t my_row) {
#pragma unroll
          for (int r = 0; r < 32; ++r) xs[r * 32 + lane] = __uint_as_float(v[r]);
          __syncwarp();
#pragma unroll
          for (int k4 = 0; k4 < 8; ++k4) {
            const int rr = k4 * 4 + sub_row;
            const int32_t drow = __shfl_sync(0xffffffffu, my_row, rr);
            const float4 v4 = *reinterpret_cast<const float4*>(xs + rr * 32 + sub_c * 4);
            if (drow >= 0) red_add_v4(a.dq_acc + (int64_t)drow * kD + qd * 32 + sub_c * 4, v4.x, v4.y, v4.z, v4.w);
          }
          __syncwarp();
        };
        drain_half(v0, dq_row0);
        drain_half(v1, dq_row1);
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

// ================================================================ dQ
constexpr int kDqThreads = 384;
constexpr int kDqSlots = 3;  // 32 KB slots; item i takes Q in slot 2i % 3 and dO in (2i + 1) % 3
constexpr int kDqNM = 4;
constexpr int kSmemDq = kDqSlots * 32768 + 3 * 32768 + 8 * 32 * 16 * 4 + 1024;

struct __align__(16) DqMeta {
  int32_t tok[32];  // token per chunk position, -1: past the chunk end or a repeated selection
  int32_t kb0, g;
  int32_t flags;    // set in shared memory by the producer: bit 0 first chunk of a K/V run, bit 1 last, bit 2 done
  int32_t row;      // CSR row (key block * G + group)
};
constexpr int kDqDone = 4;
static_assert(sizeof(DqMeta) % 16 == 0, "bulk copies move multiples of 16 bytes");

struct DqArgs {
  const int32_t* work_ptr;
  int* work_counter;  // groups of kGroupItems items taken so far (dynamic schedule)
  const DqMeta* gmeta;
  const float* nlse2;  // [T*Hq] -lse * log2(e)
  const float* delta;  // [T*Hq]
  float* dq_acc;
  int* err;
  int n_waves, num_rows, hq, h;
  float scale_log2;
  int f16;
};

__global__ void dq_item_meta_kernel(const int32_t* __restrict__ work_ptr, const int32_t* __restrict__ wave_off,
                                    const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ queries,
                                    const int32_t* __restrict__ cu, const int32_t* __restrict__ cbl, int nseq,
                                    int groups, int num_rows, int cells, int tpc, DqMeta* __restrict__ gmeta) {
  const int lane = threadIdx.x & 31;
  const int total = work_ptr[cells];
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < total; w += warps) {
    const int cell = first_cell_of(work_ptr, cells, w);
    const int row = cell % num_rows;
    const int e0 = wave_off[cell] + (w - work_ptr[cell]) * tpc;
    const int n = min(tpc, wave_off[cell + num_rows] - e0);
    const int gb = row / groups, g = row - gb * groups;
    const int sq = block_sequence(cbl, nseq, gb);
    const int kb0 = cu[sq] + (gb - cbl[sq]) * 128;
    int t = lane < n ? queries[e0 + lane] : -1;
    int prev = __shfl_up_sync(0xffffffffu, t, 1);
    if (lane == 0) prev = e0 > row_ptr[row] ? queries[e0 - 1] : -1;
    t = (t >= 0 && t != prev) ? t : -1;
    DqMeta& m = gmeta[w];
    m.tok[lane] = t;
    if (lane == 0) {
      m.kb0 = kb0;
      m.g = g;
      m.flags = 0;
      m.row = row;
    }
  }
}

// Roles (384 threads): warp 0 = TMA producer, warp 1 = S/dP issuer, warp 2 =
// dQ issuer, warps 4-7 and 8-11 = two softmax/epilogue warpgroups taking
// alternate chunks. Chunks are taken dynamically from a global counter, eight
// consecutive ones at a time (all CTAs stay in the same query wave; the eight
// mostly share one key block); the producer marks where a CTA's run on one key
// block starts and ends from its neighbours' CSR rows. TMEM stage j: S at 256 j (dS packed over its first 64
// columns after the softmax), dP at 256 j + 128 (dQ_e over it once dS is
// formed). K is double buffered: the dQ MMAs of a block's last chunk still
// read it while the next block's S runs. Shared memory: three Q/dO slots, two
// K buffers, V and the epilogue's transpose buffers.
__global__ void __launch_bounds__(kDqThreads, 1)
attn_dq_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap domap,
                  const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, DqArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sSlot0 = smem;                  // kDqSlots x 32 KB (one 128-row Q or dO tile each)
  uint8_t* sK0 = smem + kDqSlots * 32768;  // two K buffers
  uint8_t* sV = sK0 + 2 * 32768;
  float* sX0 = reinterpret_cast<float*>(sV + 32768);  // per epilogue warp: 32 x 16 floats (swizzled transpose)
  __shared__ DqMeta meta[kDqNM];
  __shared__ uint64_t slot_full[kDqSlots], slot_empty[kDqSlots], meta_full[kDqNM], meta_ready[kDqNM],
      meta_empty[kDqNM];
  __shared__ uint64_t s_full[2], p_full[2], o_full[2], o_free[2];
  __shared__ uint64_t k_full[2], k_empty[2], v_full, v_empty;
  __shared__ int32_t pv_flags[2];
  __shared__ uint32_t tmem_base;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int j = 0; j < kDqSlots; ++j) {
      mbar_init(&slot_full[j], 1);
      mbar_init(&slot_empty[j], 1);
    }
    for (int j = 0; j < kDqNM; ++j) {
      mbar_init(&meta_full[j], 1);   // the bulk copy landed (producer only)
      mbar_init(&meta_ready[j], 1);  // flags written: consumers may read the slot
      mbar_init(&meta_empty[j], 5);  // 4 softmax warps + the S/dP issuer
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&s_full[j], 1);
      mbar_init(&p_full[j], 4);
      mbar_init(&o_full[j], 1);
      mbar_init(&o_free[j], 4);
      mbar_init(&k_full[j], 1);
      mbar_init(&k_empty[j], 1);
    }
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
  const int h = a.h, hb = h < 8 ? 8 : h, octets = hb / 8;  // hb: tile rows per token (masked beyond h)

  if (warp == 0) {
    // ---------------------------------------------------------------- producer (whole warp)
    if (lane == 0) {
      tma_prefetch_desc(&qmap);
      tma_prefetch_desc(&domap);
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
    }
    int ip = 0;                  // items whose metadata was requested (lane 0)
    int end_i = 0x7fffffff;      // this CTA's item count, once the counter ran out (lane 0)
    int grp_w = 0, grp_end = 0;  // current group of consecutive items (lane 0)
    auto prefetch_meta = [&]() -> bool {
      if (ip >= end_i) return true;
      if (grp_w >= grp_end) {
        const int w0 = atomicAdd(a.work_counter, 1) * kGroupItems;
        if (w0 >= total_items) {
          end_i = ip;
          return true;
        }
        grp_w = w0;
        grp_end = min(w0 + kGroupItems, total_items);
      }
      const int slot = ip % kDqNM;
      if (ip >= kDqNM && !mbar_wait(&meta_empty[slot], ((ip / kDqNM) - 1) & 1, a.err, 81)) return false;
      mbar_arrive_expect_tx(&meta_full[slot], sizeof(DqMeta));
      bulk_copy_g2s(&meta[slot], a.gmeta + grp_w, sizeof(DqMeta), &meta_full[slot]);
      ++grp_w;
      ++ip;
      return true;
    };
    bool ok = true;
    if (lane == 0) ok = prefetch_meta() && prefetch_meta();
    int nblk = 0, prev_row = -1, i = 0;
    for (;; ++i) {
      if (lane == 0 && ok) ok = prefetch_meta();
      const int state = __shfl_sync(0xffffffffu, !ok ? 2 : (i >= end_i ? 1 : 0), 0);
      if (state == 2) {
        ok = false;
        break;
      }
      if (state == 1) break;
      const int ms = i % kDqNM;
      if (!mbar_wait_warp(&meta_full[ms], (i / kDqNM) & 1, a.err, 82)) {
        ok = false;
        break;
      }
      // the next item (requested two ahead) decides whether this one ends a K/V run
      int next_row = -1;
      if (lane == 0 && i + 1 < end_i) {
        const int ns = (i + 1) % kDqNM;
        if (mbar_wait(&meta_full[ns], ((i + 1) / kDqNM) & 1, a.err, 86)) next_row = meta[ns].row;
        else ok = false;
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      next_row = __shfl_sync(0xffffffffu, next_row, 0);
      const int row = meta[ms].row;
      const int flags = (row != prev_row ? 1 : 0) | (next_row != row ? 2 : 0);
      prev_row = row;
      const int t = meta[ms].tok[lane];
      const int g = meta[ms].g, kb0 = meta[ms].kb0;
      __syncwarp();
      if (lane == 0) {
        meta[ms].flags = flags;
        mbar_arrive(&meta_ready[ms]);
      }
      const bool mine = t >= 0;
      const uint32_t nv = __popc(__ballot_sync(0xffffffffu, mine));
      if (lane == 0 && (flags & 1)) {  // a new key block: K into the other buffer, V once free
        const int kb = nblk & 1;
        if (nblk >= 2) ok = mbar_wait(&k_empty[kb], ((nblk >> 1) - 1) & 1, a.err, 83);
        if (ok) {
          mbar_arrive_expect_tx(&k_full[kb], 32768);
          tma_load_3d(sK0 + kb * 32768, &kmap, &k_full[kb], 0, g, kb0);
          tma_load_3d(sK0 + kb * 32768 + 16384, &kmap, &k_full[kb], 64, g, kb0);
        }
        if (ok && nblk >= 1) ok = mbar_wait(&v_empty, (nblk - 1) & 1, a.err, 84);
        if (ok) {
          mbar_arrive_expect_tx(&v_full, 32768);
          tma_load_3d(sV, &vmap, &v_full, 0, g, kb0);
          tma_load_3d(sV + 16384, &vmap, &v_full, 64, g, kb0);
        }
        ++nblk;
      }
      for (int part = 0; part < 2; ++part) {  // Q tile, then dO tile
        const int u = 2 * i + part, s = u % kDqSlots;
        if (lane == 0) {
          if (ok && u >= kDqSlots) ok = mbar_wait(&slot_empty[s], ((u / kDqSlots) - 1) & 1, a.err, 85);
          if (ok) mbar_arrive_expect_tx(&slot_full[s], nv * (uint32_t)hb * 256u);
        }
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
        if (mine) {
          uint8_t* dst = sSlot0 + s * 32768 + lane * octets * 2048;
          const CUtensorMap* map = part ? &domap : &qmap;
          for (int oc = 0; oc < octets; ++oc) tma_load_4d(dst + oc * 2048, map, &slot_full[s], 0, g * h + oc * 8, 0, t);
        }
      }
    }
    // End of work: "done" entries in the next two slots, one for each softmax warpgroup.
    for (int d = 0; d < 2 && ok && lane == 0; ++d) {
      const int n = i + d, ms = n % kDqNM;
      if (n >= kDqNM && !mbar_wait(&meta_empty[ms], ((n / kDqNM) - 1) & 1, a.err, 87)) break;
      meta[ms].flags = kDqDone;
      mbar_arrive(&meta_ready[ms]);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------------------------------------------------------- S = Q K^T, dP = dO V^T
    const uint32_t id_s = idesc_f16(!a.f16, 128, 128, false, false);
    int nb = 0, kb = 0;
    for (int i = 0;; ++i) {
      const int ms = i % kDqNM, ts = i & 1;
      const int uq = 2 * i, uo = 2 * i + 1;
      if (!mbar_wait(&meta_ready[ms], (i / kDqNM) & 1, a.err, 91)) break;
      const int flags = meta[ms].flags;
      if (flags & kDqDone) break;
      mbar_arrive(&meta_empty[ms]);
      if (flags & 1) {
        kb = nb & 1;
        if (!mbar_wait(&k_full[kb], (nb >> 1) & 1, a.err, 92)) break;
        if (!mbar_wait(&v_full, nb & 1, a.err, 93)) break;
        ++nb;
      }
      if (!mbar_wait(&slot_full[uq % kDqSlots], (uq / kDqSlots) & 1, a.err, 94)) break;
      if (!mbar_wait(&slot_full[uo % kDqSlots], (uo / kDqSlots) & 1, a.err, 95)) break;
      if (i >= 2 && !mbar_wait(&o_free[ts], ((i >> 1) - 1) & 1, a.err, 96)) break;  // stage ts drained
      tc_fence_after();
      const uint32_t sq = smem_u32(sSlot0 + (uq % kDqSlots) * 32768);
      const uint32_t sdo = smem_u32(sSlot0 + (uo % kDqSlots) * 32768);
      const uint32_t sk = smem_u32(sK0 + kb * 32768), sv = smem_u32(sV);
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t qa = (ks >> 2) * 1024 + (ks & 3) * 32, ka = (ks >> 2) * 16384 + (ks & 3) * 32;
        umma_ss(tmem + ts * 256, desc_kmajor_sw128(sq + qa, 2048), desc_kmajor_sw128(sk + ka), id_s, ks > 0);
        umma_ss(tmem + ts * 256 + 128, desc_kmajor_sw128(sdo + qa, 2048), desc_kmajor_sw128(sv + ka), id_s, ks > 0);
      }
      umma_commit(&s_full[ts]);
      umma_commit(&slot_empty[uq % kDqSlots]);
      umma_commit(&slot_empty[uo % kDqSlots]);
      if (flags & 2) umma_commit(&v_empty);
    }
  } else if (warp == 2 && lane == 0) {
    // ---------------------------------------------------------------- dQ_e = dS K
    const uint32_t id_dq = idesc_f16(!a.f16, 128, 128, false, true);
    int nb = 0, kb = 0;
    for (int i = 0;; ++i) {
      const int ts = i & 1;
      if (!mbar_wait(&p_full[ts], (i >> 1) & 1, a.err, 101)) break;
      const int flags = pv_flags[ts];
      if (flags & kDqDone) break;
      if (flags & 1) {
        kb = nb & 1;
        ++nb;
      }
      tc_fence_after();
      const uint32_t sk = smem_u32(sK0 + kb * 32768);
      for (int ks = 0; ks < 8; ++ks)
        umma_ts(tmem + ts * 256 + 128, tmem + ts * 256 + ks * 8, desc_mnmajor_sw128(sk + ks * 2048, 16384), id_dq,
                ks > 0);
      umma_commit(&o_full[ts]);
      if (flags & 2) umma_commit(&k_empty[kb]);
    }
  } else if (warp >= 4) {
    // ---------------------------------------------------------------- softmax + epilogue
    const int wg = (warp - 4) >> 2;
    const int qd = warp & 3;
    const int r = qd * 32 + lane;  // tile row == TMEM lane
    const int pos = r / hb, hh = r - (r / hb) * hb;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const uint32_t t_s = tmem + wg * 256 + lane_base, t_p = t_s + 128;
    float* xs = sX0 + (warp - 4) * 32 * 16;
    const int sub_row = lane >> 2, sub_c = lane & 3;
    for (int i = wg;; i += 2) {  // the other warpgroup takes the other items
      const int ms = i % kDqNM;
      if (!mbar_wait_warp(&meta_ready[ms], (i / kDqNM) & 1, a.err, 111)) break;
      const DqMeta& m = meta[ms];
      const int flags = m.flags;
      if (flags & kDqDone) {  // tell the dQ issuer, which waits on this warpgroup's stage
        if (lane == 0) {
          if (qd == 0) pv_flags[wg] = kDqDone;
          mbar_arrive(&p_full[wg]);
        }
        break;
      }
      const int t = m.tok[pos];
      const int kb0 = m.kb0, g = m.g;
      __syncwarp();
      if (lane == 0) mbar_arrive(&meta_empty[ms]);
      const bool valid = t >= 0 && hh < h;
      const int64_t rowid = (int64_t)t * a.hq + g * h + hh;
      const float nl_raw = ld_early(a.nlse2 + (valid ? rowid : 0));  // in flight during the S wait
      const float dl_raw = ld_early(a.delta + (valid ? rowid : 0));
      const int lim = valid ? t - kb0 : -1;  // key c of the block is visible iff c <= lim
      if (!mbar_wait_warp(&s_full[wg], (i >> 1) & 1, a.err, 112)) break;
      tc_fence_after();
      const float nl = valid ? nl_raw : 0.f, dl = valid ? dl_raw : 0.f;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t packed[32];
#pragma unroll
        for (int qq = 0; qq < 2; ++qq) {
          const int c0 = half * 64 + qq * 32;
          uint32_t s[32], dp[32];
          tmem_ld32(t_s + c0, s);
          tmem_ld32(t_p + c0, dp);
          tmem_wait_ld();
          if (lim >= 127) {  // every key of the block is visible to this row
#pragma unroll
            for (int kk = 0; kk < 32; kk += 2) {
              const float p0 = ex2_approx(fmaf(__uint_as_float(s[kk]), a.scale_log2, nl));
              const float p1 = ex2_approx(fmaf(__uint_as_float(s[kk + 1]), a.scale_log2, nl));
              packed[qq * 16 + (kk >> 1)] =
                  pack2(p0 * (__uint_as_float(dp[kk]) - dl), p1 * (__uint_as_float(dp[kk + 1]) - dl), a.f16);
            }
          } else {
#pragma unroll
            for (int kk = 0; kk < 32; kk += 2) {
              const bool v0 = c0 + kk <= lim, v1 = c0 + kk + 1 <= lim;
              const float p0 = v0 ? ex2_approx(fmaf(__uint_as_float(s[kk]), a.scale_log2, nl)) : 0.f;
              const float p1 = v1 ? ex2_approx(fmaf(__uint_as_float(s[kk + 1]), a.scale_log2, nl)) : 0.f;
              const float d0 = v0 ? p0 * (__uint_as_float(dp[kk]) - dl) : 0.f;
              const float d1 = v1 ? p1 * (__uint_as_float(dp[kk + 1]) - dl) : 0.f;
              packed[qq * 16 + (kk >> 1)] = pack2(d0, d1, a.f16);
            }
          }
        }
        tmem_st32(t_s + half * 32, packed);  // dS packed over S columns [32 half, 32 half + 32): already read
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (qd == 0) pv_flags[wg] = flags;
        mbar_arrive(&p_full[wg]);
      }
      if (!mbar_wait_warp(&o_full[wg], (i >> 1) & 1, a.err, 113)) break;
      tc_fence_after();
      // dQ_e rows -> dQ accumulator through a swizzled 32 x 16 shared transpose
      // (16-byte chunk u of row x at position u ^ ((x >> 1) & 3): conflict-free
      // both ways); one red.v4 instruction then covers 8 rows x 64 B.
      for (int cp = 0; cp < 2; ++cp) {
        uint32_t o2[2][32];
        tmem_ld32(t_p + cp * 64, o2[0]);
        tmem_ld32(t_p + cp * 64 + 32, o2[1]);
        tmem_wait_ld();
        if (cp == 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&o_free[wg]);
        }
        const int64_t my_off = valid ? rowid * kD : -1;
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
#pragma unroll
          for (int q16 = 0; q16 < 2; ++q16) {
            const int col = cp * 64 + hb * 32 + q16 * 16;
#pragma unroll
            for (int u = 0; u < 4; ++u)
              *reinterpret_cast<uint4*>(xs + lane * 16 + ((u ^ ((lane >> 1) & 3)) << 2)) =
                  make_uint4(o2[hb][q16 * 16 + 4 * u], o2[hb][q16 * 16 + 4 * u + 1], o2[hb][q16 * 16 + 4 * u + 2],
                             o2[hb][q16 * 16 + 4 * u + 3]);
            __syncwarp();
#pragma unroll
            for (int k8 = 0; k8 < 4; ++k8) {
              const int rr = k8 * 8 + sub_row;
              const int64_t off = __shfl_sync(0xffffffffu, my_off, rr);
              const float4 v4 = *reinterpret_cast<const float4*>(xs + rr * 16 + ((sub_c ^ ((rr >> 1) & 3)) << 2));
              if (off >= 0) red_add_v4(a.dq_acc + off + col + sub_c * 4, v4.x, v4.y, v4.z, v4.w);
            }
            __syncwarp();
          }
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

// dq = scale * dQ_acc (16 threads per row); a kernel error word poisons dq with NaN.
__global__ void dq_finalize_kernel(const float* __restrict__ dq_acc, int64_t row0, int64_t rows, float scale,
                                   int f16, const int* __restrict__ err, void* __restrict__ dq) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t row = row0 + (idx >> 4);
  const int c = (int)(idx & 15);
  if (row >= rows) return;
  const float mul = *err != 0 ? __int_as_float(0x7fc00000) : scale;
  const float4 x = *reinterpret_cast<const float4*>(dq_acc + row * kD + c * 8);
  const float4 y = *reinterpret_cast<const float4*>(dq_acc + row * kD + c * 8 + 4);
  uint4 packed;
  packed.x = pack2(x.x * mul, x.y * mul, f16);
  packed.y = pack2(x.z * mul, x.w * mul, f16);
  packed.z = pack2(y.x * mul, y.y * mul, f16);
  packed.w = pack2(y.z * mul, y.w * mul, f16);
  *reinterpret_cast<uint4*>(static_cast<uint8_t*>(dq) + (row * kD + c * 8) * 2) = packed;
}

// After the dK/dV kernel: on a kernel error, poison dk/dv with NaN (no-op otherwise).
__global__ void kv_poison_kernel(const int* __restrict__ err, int64_t n_words, uint32_t nan2, uint32_t* __restrict__ dk,
                                 uint32_t* __restrict__ dv) {
  if (*err == 0) return;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_words; i += (int64_t)gridDim.x * blockDim.x) {
    if (dk) dk[i] = nan2;
    if (dv) dv[i] = nan2;
  }
}

struct BwdWorkspace {
  int* err;
  int* row_counter;
  int* work_counter;
  float* delta;
  float* nlse2;
  float* dq_acc;
  int32_t* wave_off;
  int32_t* work_ptr;
  DqMeta* dq_meta;
  size_t bytes;
};

inline size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

inline int wave_tokens_bwd(int q_heads) {  // the forward's wave: ~32 MB of float32 accumulator rows
  int wt = 128;
  while ((int64_t)wt * 2 * q_heads * kD * 4 <= (int64_t)32 << 20) wt *= 2;
  return wt;
}

inline int64_t waves_bwd(int64_t total_tokens, int32_t q_heads) {
  const int wt = wave_tokens_bwd(q_heads);
  return std::max<int64_t>(1, (total_tokens + wt - 1) / wt);
}

BwdWorkspace carve_bwd(void* base, int64_t total_tokens, int32_t q_heads, int32_t num_rows, int32_t groups,
                       int32_t topk) {
  const int64_t rows = total_tokens * q_heads;
  const int hb = std::max(q_heads / groups, 8);  // tile rows per token
  const int64_t edges = total_tokens * groups * (int64_t)topk;
  const int64_t n_waves = waves_bwd(total_tokens, q_heads);
  const int64_t max_items = edges / (128 / hb) + n_waves * num_rows + 1;
  BwdWorkspace w{};
  char* b = static_cast<char*>(base);
  w.err = reinterpret_cast<int*>(b);  // fixed header: error word, dK/dV row counter, dQ group counter
  w.row_counter = reinterpret_cast<int*>(b + 4);
  w.work_counter = reinterpret_cast<int*>(b + 8);
  size_t off = 256;
  w.dq_acc = reinterpret_cast<float*>(b + off);
  off = a256(off + sizeof(float) * rows * kD);
  w.delta = reinterpret_cast<float*>(b + off);
  off = a256(off + sizeof(float) * rows);
  w.nlse2 = reinterpret_cast<float*>(b + off);
  off = a256(off + sizeof(float) * rows);
  w.wave_off = reinterpret_cast<int32_t*>(b + off);
  off = a256(off + sizeof(int32_t) * (n_waves + 1) * num_rows);
  w.work_ptr = reinterpret_cast<int32_t*>(b + off);
  off = a256(off + sizeof(int32_t) * (n_waves * num_rows + 1));
  w.dq_meta = reinterpret_cast<DqMeta*>(b + off);
  off = a256(off + sizeof(DqMeta) * max_items);
  w.bytes = off;
  return w;
}

int encode_maps(const void* q, const void* dout, const void* k, const void* v, int dtype, int64_t total_tokens,
                int32_t q_heads, int32_t groups, CUtensorMap* qmap, CUtensorMap* domap, CUtensorMap* kmap,
                CUtensorMap* vmap) {
  // Q / dO as 4-D (d_in 64, head, d_out 2, token): one box = 8 head rows x both
  // 64-column halves of one token (2 KB), landing as [d_out][8 rows][128 B].
  const uint64_t dq[4] = {64, (uint64_t)q_heads, 2, (uint64_t)total_tokens};
  const uint64_t sq[3] = {(uint64_t)kD * 2, 128, (uint64_t)q_heads * kD * 2};
  const uint32_t bq[4] = {64, 8, 2, 1};
  const CUtensorMapDataType dt = tc::tma_dtype(dtype);
  if (int e = tc::encode_tensor_map(qmap, dt, 4, q, dq, sq, bq, CU_TENSOR_MAP_SWIZZLE_128B)) return e;
  if (int e = tc::encode_tensor_map(domap, dt, 4, dout, dq, sq, bq, CU_TENSOR_MAP_SWIZZLE_128B)) return e;
  const uint64_t dk[3] = {(uint64_t)kD, (uint64_t)groups, (uint64_t)total_tokens};
  const uint64_t sk[2] = {(uint64_t)kD * 2, (uint64_t)groups * kD * 2};
  const uint32_t bk[3] = {64, 1, 128};
  if (int e = tc::encode_tensor_map(kmap, dt, 3, k, dk, sk, bk, CU_TENSOR_MAP_SWIZZLE_128B)) return e;
  return tc::encode_tensor_map(vmap, dt, 3, v, dk, sk, bk, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace
}  // namespace msa

using namespace msa;

extern "C" size_t msa_attn_bwd_tc_workspace_size(int64_t total_tokens, int32_t q_heads, int32_t num_rows,
                                                 int32_t groups, int32_t topk_blocks) {
  if (groups < 1 || q_heads % groups || num_rows < 0) return 0;
  const int h = q_heads / groups;
  if ((h != 4 && h != 8 && h != 16) || q_heads < 8) return 0;
  return carve_bwd(nullptr, total_tokens, q_heads, num_rows, groups, topk_blocks).bytes;
}

extern "C" int msa_attn_bwd_tc_range(const void* q, const void* k, const void* v, const void* out,
                                     const void* dout, const float* lse, int dtype, const int32_t* cu_seqlens,
                                     const int32_t* cu_block_lens, const int32_t* row_ptr,
                                     const int32_t* query_indices, int32_t nseq, int64_t total_tokens,
                                     int32_t q_heads, int32_t groups, int32_t head_dim, int32_t topk_blocks,
                                     int32_t block_size, double scale, int32_t num_rows, int64_t q_lo, int64_t q_hi,
                                     void* dq, void* dk, void* dv, int kv_dtype, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  MSA_CHECK_ARG(dtype == MSA_BF16 || dtype == MSA_F16, "msa_attn_bwd_tc: bf16/f16 only");
  MSA_CHECK_ARG(head_dim == kD && block_size == 128, "msa_attn_bwd_tc: head_dim and block_size must be 128");
  MSA_CHECK_ARG(groups >= 1 && q_heads % groups == 0, "msa_attn_bwd_tc: bad head counts");
  const int h = q_heads / groups;
  MSA_CHECK_ARG(h == 4 || h == 8 || h == 16, "msa_attn_bwd_tc: query heads per group must be 4, 8 or 16");
  MSA_CHECK_ARG(q_heads >= 8, "msa_attn_bwd_tc: at least 8 query heads");
  const int hb = std::max(h, 8);  // tile rows per token
  MSA_CHECK_ARG(kv_dtype == dtype || kv_dtype == MSA_F32, "msa_attn_bwd_tc: dk/dv dtype must be the input's or f32");
  const int kv_f32 = kv_dtype == MSA_F32 ? 1 : 0;
  MSA_CHECK_ARG(total_tokens < (int64_t)1 << 31 && num_rows >= 0, "msa_attn_bwd_tc: size out of range");
  MSA_CHECK_ARG(0 <= q_lo && q_lo <= q_hi && q_hi <= total_tokens, "msa_attn_bwd_tc: bad query range");
  const int64_t rows = total_tokens * q_heads;
  const int64_t row0 = q_lo * q_heads, row1 = q_hi * q_heads;
  if (rows == 0 || (!dq && !dk && !dv)) return MSA_OK;
  const BwdWorkspace w = carve_bwd(workspace, total_tokens, q_heads, num_rows, groups, topk_blocks);
  MSA_CHECK_ARG(workspace && workspace_bytes >= w.bytes, "msa_attn_bwd_tc: workspace too small");
  const int64_t n_waves = waves_bwd(total_tokens, q_heads);
  MSA_CHECK_ARG(n_waves * num_rows < (int64_t)1 << 31, "msa_attn_bwd_tc: schedule too large");
  cudaStream_t st = as_stream(stream);
  const int cd = dtype == MSA_F16 ? 1 : 0;
  CUtensorMap qmap, domap, kmap, vmap;
  if (int e = encode_maps(q, dout, k, v, dtype, total_tokens, q_heads, groups, &qmap, &domap, &kmap, &vmap)) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const float scale_log2 = (float)(scale * 1.4426950408889634);

  MSA_CUDA_RETURN(cudaMemsetAsync(w.err, 0, 12, st));  // error word, row and group counters
  if (row1 > row0)
    bwd_prep_kernel<<<ceil_div((row1 - row0) * 16, 256), 256, 0, st>>>(out, dout, lse, row0, row1, cd, w.delta,
                                                                       w.nlse2, dq ? w.dq_acc : nullptr);
  count_launches(1);

  // dQ together with dK/dV: one key-block-stationary pass (dS computed once);
  // dQ alone: the query-wave dQ kernel
  const bool fused = dq && (dk || dv);
  if (dk || dv) {
    const size_t kv_bytes = (size_t)total_tokens * groups * kD * (kv_f32 ? 4 : 2);
    if (dk) MSA_CUDA_RETURN(cudaMemsetAsync(dk, 0, kv_bytes, st));  // keys no token selects keep zero gradients
    if (dv) MSA_CUDA_RETURN(cudaMemsetAsync(dv, 0, kv_bytes, st));
    if (num_rows > 0) {
      KvArgs ka{q, dout, row_ptr, query_indices, cu_seqlens, cu_block_lens, w.nlse2, w.delta, w.row_counter, w.err, dk, dv,
                nseq,    num_rows,      groups,     q_heads,       h,       scale_log2, (float)scale, cd, kv_f32,
                fused ? w.dq_acc : nullptr};
      auto kern = fused ? (h == 4 ? attn_dkdv_tc_kernel<true, true> : attn_dkdv_tc_kernel<true, false>)
                        : (h == 4 ? attn_dkdv_tc_kernel<false, true> : attn_dkdv_tc_kernel<false, false>);
      const int smem_bytes = fused ? kKvSmemDq : kKvSmem;
      MSA_CUDA_RETURN(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes));
      const int slot = timing_begin(st);
      kern<<<sms, kKvThreads, smem_bytes, st>>>(qmap, domap, kmap, vmap, ka);
      timing_end(fused ? "attn_bwd_tc" : "attn_dkdv_tc", slot, st);
      kv_poison_kernel<<<sms * 4, 256, 0, st>>>(w.err, (int64_t)kv_bytes / 4, kv_f32 ? 0x7fc00000u : 0x7fc07fc0u,
                                                static_cast<uint32_t*>(dk), static_cast<uint32_t*>(dv));
      count_launches(2);
    }
  }
  if (dq) {
    if (num_rows > 0 && !fused) {
      const int cells = (int)(n_waves * num_rows);
      const int tpc = 128 / hb;
      wave_off_kernel<<<ceil_div((int64_t)(n_waves + 1) * num_rows, 256), 256, 0, st>>>(
          row_ptr, query_indices, num_rows, (int)n_waves, wave_tokens_bwd(q_heads), w.wave_off);
      work_ptr_kernel<<<1, 1024, 0, st>>>(w.wave_off, cells, num_rows, tpc, w.work_ptr);
      dq_item_meta_kernel<<<sms * 8, 256, 0, st>>>(w.work_ptr, w.wave_off, row_ptr, query_indices, cu_seqlens,
                                                   cu_block_lens, nseq, groups, num_rows, cells, tpc, w.dq_meta);
      DqArgs da{w.work_ptr, w.work_counter, w.dq_meta, w.nlse2, w.delta, w.dq_acc, w.err, (int)n_waves, num_rows,
                q_heads, h, scale_log2, cd};
      MSA_CUDA_RETURN(cudaFuncSetAttribute(attn_dq_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemDq));
      const int slot = timing_begin(st);
      attn_dq_tc_kernel<<<sms, kDqThreads, kSmemDq, st>>>(qmap, domap, kmap, vmap, da);
      timing_end("attn_dq_tc", slot, st);
      count_launches(4);
    }
    if (row1 > row0)
      dq_finalize_kernel<<<ceil_div((row1 - row0) * 16, 256), 256, 0, st>>>(w.dq_acc, row0, row1, (float)scale, cd,
                                                                            w.err, dq);
    count_launches(1);
  }
  return launch_status("attn_bwd_tc");
}

extern "C" int msa_attn_bwd_tc(const void* q, const void* k, const void* v, const void* out, const void* dout,
                               const float* lse, int dtype, const int32_t* cu_seqlens, const int32_t* cu_block_lens,
                               const int32_t* row_ptr, const int32_t* query_indices, int32_t nseq,
                               int64_t total_tokens, int32_t q_heads, int32_t groups, int32_t head_dim,
                               int32_t topk_blocks, int32_t block_size, double scale, int32_t num_rows, void* dq,
                               void* dk, void* dv, int kv_dtype, void* workspace, size_t workspace_bytes,
                               void* stream) {
  return msa_attn_bwd_tc_range(q, k, v, out, dout, lse, dtype, cu_seqlens, cu_block_lens, row_ptr, query_indices,
                               nseq, total_tokens, q_heads, groups, head_dim, topk_blocks, block_size, scale,
                               num_rows, 0, total_tokens, dq, dk, dv, kv_dtype, workspace, workspace_bytes, stream);
}

extern "C" int msa_attn_bwd_tc_error(const void* workspace, int32_t* host_err) {
  MSA_CHECK_ARG(workspace && host_err, "msa_attn_bwd_tc_error: null pointer");
  MSA_CUDA_RETURN(cudaMemcpy(host_err, workspace, sizeof(int32_t), cudaMemcpyDeviceToHost));
  return MSA_OK;
}
