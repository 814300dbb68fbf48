// k2q CSR build: block -> query transpose of indices[T][G][K].
//
// Output contract of triton/k2q.py:39-128 (K2QCSR): row (cu_block_lens[seq] + b)
// * G + g lists every valid edge (query, slot) that selected sequence-local
// block b for group g, ordered by query then slot; row_ptr is the exclusive
// prefix of row counts; edge arrays have capacity T*G*K with a -1 tail. An edge
// is valid iff 0 <= b <= (t - seq_start) / block_size (k2q.py:101-106).
//
// The reference sorts a composite int64 key (k2q.py:117-127). Here the order
// comes from integer counting instead, in three stages:
//   1. histogram: each (query tile, group) warp counts its edges per block;
//   2. scans: per row, an exclusive prefix over the tiles of the sequence,
//      then an exclusive prefix over rows (row_ptr);
//   3. stable scatter: each warp replays its tile in (query, slot) order, with
//      cursors row_ptr[row] + tile prefix; duplicate blocks within one query
//      are ranked by slot with a warp match.
// Tiles never cross sequences, so block ids stay sequence-local.
#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace msa {
namespace {

constexpr int kCursorChunk = 2048;  // blocks per shared-memory cursor pass
constexpr int kWarps = 4;
constexpr int kScanThreads = 256;
constexpr int kScanTile = 4 * kScanThreads;  // elements per scan CTA
constexpr int64_t kMaxCountEntries = int64_t(1) << 25;
constexpr int kBatch = 8;  // tokens whose ids are loaded ahead of the replay

struct Tile { int32_t start, len, seq, count_off; };
struct SeqInfo { int32_t first_tile, num_tiles, count_off, pad; };

struct HostPlan {
  int tile_tokens = 128;
  int64_t num_tiles = 0, count_entries = 0, num_rows = 0;
  std::vector<int64_t> scan_levels;  // sizes of the recursive scan arrays
};

HostPlan make_plan(const int32_t* cu, int nseq, int groups, int block) {
  HostPlan p;
  int64_t total_blocks = 0;
  for (int s = 0; s < nseq; ++s) total_blocks += (cu[s + 1] - cu[s] + (int64_t)block - 1) / block;
  p.num_rows = total_blocks * groups;
  for (p.tile_tokens = 128;; p.tile_tokens *= 2) {
    int64_t tiles = 0, entries = 0;
    for (int s = 0; s < nseq; ++s) {
      const int64_t len = cu[s + 1] - cu[s];
      const int64_t nt = (len + p.tile_tokens - 1) / p.tile_tokens;
      tiles += nt;
      entries += nt * groups * ((len + block - 1) / block);
    }
    p.num_tiles = tiles;
    p.count_entries = entries;
    if (entries <= kMaxCountEntries || p.tile_tokens >= (1 << 30)) break;
  }
  for (int64_t n = p.num_rows; n > 1;) {
    n = (n + kScanTile - 1) / kScanTile;
    p.scan_levels.push_back(n);
  }
  return p;
}

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct Workspace {
  Tile* tiles = nullptr;
  SeqInfo* seqs = nullptr;
  int32_t* counts = nullptr;
  std::vector<int32_t*> levels;
  size_t bytes = 0;
};

Workspace carve(void* base, const HostPlan& p, int nseq) {
  Workspace w;
  size_t off = 0;
  char* b = static_cast<char*>(base);
  w.tiles = reinterpret_cast<Tile*>(b + off);
  off = align256(off + sizeof(Tile) * std::max<int64_t>(p.num_tiles, 1));
  w.seqs = reinterpret_cast<SeqInfo*>(b + off);
  off = align256(off + sizeof(SeqInfo) * nseq);
  w.counts = reinterpret_cast<int32_t*>(b + off);
  off = align256(off + sizeof(int32_t) * std::max<int64_t>(p.count_entries, 1));
  for (int64_t n : p.scan_levels) {
    w.levels.push_back(reinterpret_cast<int32_t*>(b + off));
    off = align256(off + sizeof(int32_t) * n);
  }
  w.bytes = off;
  return w;
}

// Tile and sequence tables, built on the device so the build is stream-ordered.
__global__ void plan_kernel(const int32_t* __restrict__ cu, int nseq, int groups, int block, int tile_tokens,
                            Tile* __restrict__ tiles, SeqInfo* __restrict__ seqs) {
  int32_t tile = 0, off = 0;
  for (int s = 0; s < nseq; ++s) {
    const int32_t start = cu[s], len = cu[s + 1] - cu[s];
    const int32_t nb = (int32_t)((len + (int64_t)block - 1) / block);
    const int32_t nt = (int32_t)((len + (int64_t)tile_tokens - 1) / tile_tokens);
    seqs[s] = SeqInfo{tile, nt, off, 0};
    for (int32_t i = 0; i < nt; ++i)
      tiles[tile + i] = Tile{start + i * tile_tokens, min(tile_tokens, len - i * tile_tokens), s,
                             off + i * groups * nb};
    tile += nt;
    off += nt * groups * nb;
  }
}

// Block selected by one lane's (token, slot); -1 - lane when there is no valid
// edge, so lanes without an edge never match each other in __match_any_sync.
__device__ __forceinline__ int edge_block(const int32_t* __restrict__ ids, int64_t t, int groups, int g,
                                          int k, int slot, int64_t cur, int lane) {
  if (slot >= k) return -1 - lane;
  const int b = __ldg(ids + (t * groups + g) * (int64_t)k + slot);
  return (b >= 0 && b <= cur) ? b : -1 - lane;
}

// Stage 1 (kScatter = false): per-(tile, group) block histogram into counts.
// Stage 3 (kScatter = true): counts holds exclusive tile prefixes; place edges.
template <bool kScatter>
__global__ void __launch_bounds__(kWarps * 32)
replay_kernel(const int32_t* __restrict__ ids, const int32_t* __restrict__ cu, const Tile* __restrict__ tiles,
              int64_t items, int groups, int k, int block, const int32_t* __restrict__ cu_block_lens,
              int32_t* __restrict__ counts, const int32_t* __restrict__ row_ptr,
              int32_t* __restrict__ query_out, int32_t* __restrict__ slot_out) {
  __shared__ int32_t cursor_all[kWarps][kCursorChunk];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t item = (int64_t)blockIdx.x * kWarps + warp;
  if (item >= items) return;
  const Tile tile = tiles[item / groups];
  const int g = (int)(item % groups);
  int32_t* cursor = cursor_all[warp];
  const int64_t seq_start = cu[tile.seq];
  const int32_t block_base = cu_block_lens[tile.seq];
  const int32_t nblocks = cu_block_lens[tile.seq + 1] - block_base;
  int32_t* my_counts = counts + tile.count_off + (int64_t)g * nblocks;
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int b0 = 0; b0 < nblocks; b0 += kCursorChunk) {
    const int bn = min(kCursorChunk, nblocks - b0);
    for (int i = lane; i < bn; i += 32)
      cursor[i] = kScatter ? row_ptr[((int64_t)block_base + b0 + i) * groups + g] + my_counts[b0 + i] : 0;
    __syncwarp();
    if (k <= 16) {
      // floor(32 / k) tokens per step, lane = (token p, slot s): one match over
      // all of them keeps the (query, slot) order, since earlier tokens sit in
      // lower lanes.
      const int per = 32 / k, p = lane / k, sl = lane - p * k;
      const bool act = p < per;
      for (int32_t i0 = 0; i0 < tile.len; i0 += per * kBatch) {
        int bv[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const int32_t ti = i0 + u * per + p;
          const int64_t t = tile.start + ti;
          bv[u] = (act && ti < tile.len) ? edge_block(ids, t, groups, g, k, sl, (t - seq_start) / block, lane)
                                         : -1 - lane;
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const int b = bv[u];
          const bool mine = b >= b0 && b < b0 + bn;
          const unsigned peers = __match_any_sync(0xffffffffu, mine ? b : -1 - lane);
          if (mine && kScatter) {
            const int pos = cursor[b - b0] + __popc(peers & lt_mask);
            query_out[pos] = (int32_t)(tile.start + i0 + u * per + p);
            slot_out[pos] = sl;
          }
          __syncwarp();
          if (mine && (peers & lt_mask) == 0) cursor[b - b0] += __popc(peers);
          __syncwarp();
        }
      }
    } else
    for (int32_t i0 = 0; i0 < tile.len; i0 += kBatch) {
      int first_chunk[kBatch];  // slots 0..31 of the batch's tokens, loaded ahead
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int64_t t = tile.start + i0 + u;
        first_chunk[u] = (i0 + u < tile.len)
                             ? edge_block(ids, t, groups, g, k, lane, (t - seq_start) / block, lane)
                             : -1 - lane;
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int64_t t = tile.start + i0 + u;
        for (int sc = 0; sc < k; sc += 32) {  // (query, slot) order: slot chunks inside the token
          int b = first_chunk[u];
          if (sc > 0)
            b = (i0 + u < tile.len) ? edge_block(ids, t, groups, g, k, sc + lane, (t - seq_start) / block, lane)
                                    : -1 - lane;
          const bool mine = b >= b0 && b < b0 + bn;
          const unsigned peers = __match_any_sync(0xffffffffu, mine ? b : -1 - lane);
          if (mine && kScatter) {
            const int pos = cursor[b - b0] + __popc(peers & lt_mask);
            query_out[pos] = (int32_t)t;
            slot_out[pos] = sc + lane;
          }
          __syncwarp();
          if (mine && (peers & lt_mask) == 0) cursor[b - b0] += __popc(peers);
          __syncwarp();
        }
      }
    }
    if (!kScatter)
      for (int i = lane; i < bn; i += 32) my_counts[b0 + i] = cursor[i];
    __syncwarp();
  }
}

// Stage 2a: per row (seq, b, g), exclusive prefix of its tile counts in place;
// the row total goes to row_ptr[row + 1]. One warp per row: 32 tile counts per
// step, warp-scanned, with a running carry.
__global__ void tile_prefix_kernel(int nseq, const int32_t* __restrict__ cu_block_lens, int groups,
                                   const SeqInfo* __restrict__ seqs, int64_t num_rows,
                                   int32_t* __restrict__ counts, int32_t* __restrict__ row_ptr) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= num_rows) return;  // whole warps leave together
  const int64_t gb = row / groups;
  const int g = (int)(row % groups);
  int lo = 0, hi = nseq - 1;  // sequence owning global block gb: largest s with cu_block_lens[s] <= gb
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu_block_lens[mid] <= gb) lo = mid; else hi = mid - 1;
  }
  const int32_t nb = cu_block_lens[lo + 1] - cu_block_lens[lo];
  const int64_t b = gb - cu_block_lens[lo];
  const SeqInfo si = seqs[lo];
  int32_t* p = counts + si.count_off + (int64_t)g * nb + b;
  const int64_t step = (int64_t)groups * nb;
  int32_t carry = 0;
  for (int32_t i0 = 0; i0 < si.num_tiles; i0 += 32) {
    const int32_t i = i0 + lane;
    const int32_t c = i < si.num_tiles ? p[i * step] : 0;
    int32_t x = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (i < si.num_tiles) p[i * step] = carry + x - c;
    carry += __shfl_sync(0xffffffffu, x, 31);
  }
  if (lane == 0) row_ptr[row + 1] = carry;
}

// Inclusive scan of one kScanTile slice per CTA; the slice total goes to sums.
__global__ void __launch_bounds__(kScanThreads)
scan_tiles_kernel(int32_t* __restrict__ data, int64_t n, int32_t* __restrict__ sums) {
  __shared__ int32_t warp_tot[kScanThreads / 32];
  const int64_t base = (int64_t)blockIdx.x * kScanTile + threadIdx.x * 4;
  int32_t v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = (base + i < n) ? data[base + i] : 0;
  v[1] += v[0]; v[2] += v[1]; v[3] += v[2];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int32_t x = v[3];
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int32_t w = lane < kScanThreads / 32 ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < kScanThreads / 32) warp_tot[lane] = w;
  }
  __syncthreads();
  const int32_t prefix = (x - v[3]) + (warp > 0 ? warp_tot[warp - 1] : 0);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (base + i < n) data[base + i] = v[i] + prefix;
  if (threadIdx.x == kScanThreads - 1 && sums) sums[blockIdx.x] = warp_tot[kScanThreads / 32 - 1];
}

__global__ void add_tile_offsets_kernel(int32_t* __restrict__ data, int64_t n, const int32_t* __restrict__ sums) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t tile = i / kScanTile;
  if (i < n && tile > 0) data[i] += sums[tile - 1];
}

// Recursive inclusive scan of data[0, n) using the plan's level buffers.
void inclusive_scan(int32_t* data, int64_t n, const std::vector<int32_t*>& levels, size_t level,
                    cudaStream_t st) {
  if (n <= 0) return;
  const int64_t tiles = (n + kScanTile - 1) / kScanTile;
  int32_t* sums = tiles > 1 ? levels[level] : nullptr;
  scan_tiles_kernel<<<(unsigned)tiles, kScanThreads, 0, st>>>(data, n, sums); count_launches(1);
  if (tiles > 1) {
    inclusive_scan(sums, tiles, levels, level + 1, st);
    add_tile_offsets_kernel<<<ceil_div(n, 256), 256, 0, st>>>(data, n, sums); count_launches(1);
  }
}

__global__ void tail_fill_kernel(const int32_t* __restrict__ row_ptr, int64_t num_rows, int64_t capacity,
                                 int32_t* __restrict__ query_out, int32_t* __restrict__ slot_out) {
  const int64_t used = row_ptr[num_rows];
  for (int64_t i = used + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < capacity;
       i += (int64_t)gridDim.x * blockDim.x) {
    query_out[i] = -1;
    slot_out[i] = -1;
  }
}

}  // namespace
}  // namespace msa

using namespace msa;

extern "C" size_t msa_k2q_workspace_size(const int32_t* host_cu_seqlens, int32_t nseq, int32_t groups,
                                         int32_t block_size) {
  if (!host_cu_seqlens || nseq < 1 || groups < 1 || block_size < 1) return 0;
  const HostPlan p = make_plan(host_cu_seqlens, nseq, groups, block_size);
  return carve(nullptr, p, nseq).bytes;
}

extern "C" int msa_k2q_build(const int32_t* indices, const int32_t* cu_seqlens, const int32_t* host_cu_seqlens,
                             const int32_t* cu_block_lens, int32_t nseq, int64_t total_tokens, int32_t groups,
                             int32_t topk_blocks, int32_t block_size, int32_t* row_ptr, int32_t* query_indices,
                             int32_t* slot_indices, void* workspace, size_t workspace_bytes, void* stream) {
  MSA_CHECK_ARG(host_cu_seqlens && nseq >= 1 && groups >= 1 && block_size >= 1 && topk_blocks >= 0,
                "msa_k2q_build: bad sizes");
  const int64_t capacity = total_tokens * groups * (int64_t)topk_blocks;
  MSA_CHECK_ARG(capacity <= 0x7fffffffLL, "msa_k2q_build: T * G * K exceeds int32 edge capacity");
  const HostPlan p = make_plan(host_cu_seqlens, nseq, groups, block_size);
  MSA_CHECK_ARG(p.count_entries <= 0x7fffffffLL, "msa_k2q_build: tile histogram exceeds int32 indexing");
  cudaStream_t st = as_stream(stream);
  MSA_CUDA_RETURN(cudaMemsetAsync(row_ptr, 0, sizeof(int32_t) * (p.num_rows + 1), st));
  // rows == 0 implies T == 0 (every non-empty sequence owns a block), so no edges.
  if (capacity == 0 || p.num_rows == 0) return launch_status("k2q_memset");
  const Workspace w = carve(workspace, p, nseq);
  MSA_CHECK_ARG(workspace && workspace_bytes >= w.bytes, "msa_k2q_build: workspace too small (%zu < %zu)",
                workspace_bytes, w.bytes);
  plan_kernel<<<1, 1, 0, st>>>(cu_seqlens, nseq, groups, block_size, p.tile_tokens, w.tiles, w.seqs); count_launches(1);
  const int64_t items = p.num_tiles * groups;
  const unsigned replay_grid = ceil_div(items, kWarps);
  replay_kernel<false><<<replay_grid, kWarps * 32, 0, st>>>(indices, cu_seqlens, w.tiles, items, groups,
                                                           topk_blocks, block_size, cu_block_lens, w.counts,
                                                           nullptr, nullptr, nullptr); count_launches(1);
  tile_prefix_kernel<<<ceil_div(p.num_rows * 32, 256), 256, 0, st>>>(nseq, cu_block_lens, groups, w.seqs, p.num_rows,
                                                                   w.counts, row_ptr); count_launches(1);
  inclusive_scan(row_ptr + 1, p.num_rows, w.levels, 0, st);
  replay_kernel<true><<<replay_grid, kWarps * 32, 0, st>>>(indices, cu_seqlens, w.tiles, items, groups,
                                                          topk_blocks, block_size, cu_block_lens, w.counts,
                                                          row_ptr, query_indices, slot_indices); count_launches(1);
  const int64_t fill_blocks = std::min<int64_t>(1024, std::max<int64_t>(1, capacity / 2048));
  tail_fill_kernel<<<(unsigned)fill_blocks, 256, 0, st>>>(row_ptr, p.num_rows, capacity, query_indices,
                                                          slot_indices); count_launches(1);
  return launch_status("k2q_build");
}

// ------------------------------------------------------------------ no-alloc variant
// msa_k2q_build with its scratch (tile table, per-tile histograms, scan
// levels) in a fixed device array instead of a caller workspace: the call
// allocates nothing. Every scratch word a call reads it first writes itself,
// so the array needs no zeroing; row_ptr is zeroed by the call as in
// msa_k2q_build. All calls on one device share the array: calls whose
// execution overlaps (different streams, or threads without ordering) race on
// it; calls ordered on one stream do not.
namespace msa {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // 4 MiB: T = 32K at G = 8 needs ~2.1 MB
static __device__ __align__(256) unsigned char g_k2q_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

}  // namespace
}  // namespace msa

extern "C" int msa_k2q_build_noalloc(const int32_t* indices, const int32_t* cu_seqlens,
                                     const int32_t* host_cu_seqlens, const int32_t* cu_block_lens, int32_t nseq,
                                     int64_t total_tokens, int32_t groups, int32_t topk_blocks, int32_t block_size,
                                     int32_t* row_ptr, int32_t* query_indices, int32_t* slot_indices, void* stream) {
  MSA_CHECK_ARG(host_cu_seqlens && nseq >= 1 && groups >= 1 && block_size >= 1 && topk_blocks >= 0,
                "msa_k2q_build_noalloc: bad sizes");
  const int64_t capacity = total_tokens * groups * (int64_t)topk_blocks;
  MSA_CHECK_ARG(capacity <= 0x7fffffffLL, "msa_k2q_build_noalloc: T * G * K exceeds int32 edge capacity");
  const HostPlan p = make_plan(host_cu_seqlens, nseq, groups, block_size);
  MSA_CHECK_ARG(p.count_entries <= 0x7fffffffLL, "msa_k2q_build_noalloc: tile histogram exceeds int32 indexing");
  const size_t need = carve(nullptr, p, nseq).bytes;
  MSA_CHECK_ARG(need <= kNoAllocScratchBytes,
                "msa_k2q_build_noalloc: this problem needs %zu bytes of scratch, more than the fixed %zu-byte "
                "device buffer; use msa_k2q_build with a workspace",
                need, kNoAllocScratchBytes);
  // Set-up, once per device with that device current: the buffer's device address.
  int dev = 0;
  MSA_CUDA_RETURN(cudaGetDevice(&dev));
  MSA_CHECK_ARG(dev >= 0 && dev < kMaxDevices, "msa_k2q_build_noalloc: device ordinal %d out of range", dev);
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
      void* addr = nullptr;
      MSA_CUDA_RETURN(cudaGetSymbolAddress(&addr, g_k2q_scratch));
      g_scratch_addr[dev] = addr;
    }
    scratch = g_scratch_addr[dev];
  }
  cudaStream_t st = as_stream(stream);
  MSA_CUDA_RETURN(cudaMemsetAsync(row_ptr, 0, sizeof(int32_t) * (p.num_rows + 1), st));
  if (capacity == 0 || p.num_rows == 0) return launch_status("k2q_noalloc_memset");
  const Workspace w = carve(scratch, p, nseq);
  plan_kernel<<<1, 1, 0, st>>>(cu_seqlens, nseq, groups, block_size, p.tile_tokens, w.tiles, w.seqs); count_launches(1);
  const int64_t items = p.num_tiles * groups;
  const unsigned replay_grid = ceil_div(items, kWarps);
  replay_kernel<false><<<replay_grid, kWarps * 32, 0, st>>>(indices, cu_seqlens, w.tiles, items, groups,
                                                           topk_blocks, block_size, cu_block_lens, w.counts,
                                                           nullptr, nullptr, nullptr); count_launches(1);
  tile_prefix_kernel<<<ceil_div(p.num_rows * 32, 256), 256, 0, st>>>(nseq, cu_block_lens, groups, w.seqs, p.num_rows,
                                                                   w.counts, row_ptr); count_launches(1);
  inclusive_scan(row_ptr + 1, p.num_rows, w.levels, 0, st);
  replay_kernel<true><<<replay_grid, kWarps * 32, 0, st>>>(indices, cu_seqlens, w.tiles, items, groups,
                                                          topk_blocks, block_size, cu_block_lens, w.counts,
                                                          row_ptr, query_indices, slot_indices); count_launches(1);
  const int64_t fill_blocks = std::min<int64_t>(1024, std::max<int64_t>(1, capacity / 2048));
  tail_fill_kernel<<<(unsigned)fill_blocks, 256, 0, st>>>(row_ptr, p.num_rows, capacity, query_indices,
                                                          slot_indices); count_launches(1);
  return launch_status("k2q_build_noalloc");
}
