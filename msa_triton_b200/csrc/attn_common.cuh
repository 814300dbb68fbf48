// Device helpers shared by the tensor-core attention kernels (forward and
// backward): work schedule over the k2q CSR, operand packing, reductions.
#pragma once

#include "tc_common.cuh"

namespace msa {
namespace attn {
namespace {  // internal linkage: every translation unit gets its own kernels

using namespace tc;

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Work items are chunks of up to tpc selector tokens of one (wave, row) cell,
// where a row is one (key block, group) of the k2q CSR and a wave is a range of
// query tokens. Cells are numbered wave-major (cell = wave * num_rows + row)
// and work_ptr is the exclusive prefix of their chunk counts.
__device__ __forceinline__ int first_cell_of(const int32_t* work_ptr, int cells, int w) {
  int lo = 0, hi = cells - 1;  // largest cell with work_ptr[cell] <= w (empty cells skipped)
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (work_ptr[mid] <= w) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// CTAs take groups of kGroupItems consecutive items round-robin, so at any time
// all CTAs work inside the same wave (its slice of the O accumulator and of Q
// stays resident in L2) while consecutive items of a group share K/V.
constexpr int kGroupItems = 8;

struct ItemIter {
  int w, group_end, total;
  bool group_start;  // first item of a group: the cell must be searched, not advanced to
  __device__ void start(int total_items) {
    total = total_items;
    w = blockIdx.x * kGroupItems;
    group_end = min(w + kGroupItems, total);
    group_start = true;
  }
  __device__ bool valid() const { return w < total; }
  __device__ void next() {
    ++w;
    group_start = false;
    if (w >= group_end) {
      w += (gridDim.x - 1) * kGroupItems;
      group_end = min(w + kGroupItems, total);
      group_start = true;
    }
  }
};

// Sequence of a CSR row's key block and the block's first key token.
__device__ __forceinline__ int block_sequence(const int32_t* cbl, int nseq, int gb) {
  int lo = 0, hi = nseq - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cbl[mid] <= gb) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi, int f16) {
  if (f16) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Global load issued where it stands (volatile asm is not moved across the
// barrier-wait asm that follows it), so its latency overlaps the wait.
__device__ __forceinline__ float ld_early(const float* p) {
  float v;
  asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// wave_off[c][row] = first edge of CSR row `row` whose query is >= c * wave_tokens
// (rows are sorted by query); c = n_waves gives the row end.
__global__ void wave_off_kernel(const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ queries, int num_rows,
                                int n_waves, int wave_tokens, int32_t* __restrict__ wave_off) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)(n_waves + 1) * num_rows) return;
  const int c = (int)(idx / num_rows), row = (int)(idx - (int64_t)c * num_rows);
  int lo = row_ptr[row], hi = row_ptr[row + 1];
  if (c == n_waves) {
    lo = hi;
  } else if (c > 0) {
    const int key = c * wave_tokens;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (queries[mid] < key) lo = mid + 1; else hi = mid;
    }
  }
  wave_off[idx] = lo;
}

// work_ptr[cell] = exclusive prefix over cells (wave-major) of ceil(edges / tpc);
// one CTA of 1024 threads.
__global__ void __launch_bounds__(1024) work_ptr_kernel(const int32_t* __restrict__ wave_off, int cells, int num_rows,
                                                        int tpc, int32_t* __restrict__ work_ptr) {
  __shared__ int32_t warp_tot[32];
  __shared__ int32_t carry;
  if (threadIdx.x == 0) {
    carry = 0;
    work_ptr[0] = 0;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int base = 0; base < cells; base += 1024) {
    const int cell = base + threadIdx.x;
    const int c = cell < cells ? (wave_off[cell + num_rows] - wave_off[cell] + tpc - 1) / tpc : 0;
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
    if (cell < cells) work_ptr[cell + 1] = carry + incl;
    __syncthreads();
    if (threadIdx.x == 1023) carry += incl;
    __syncthreads();
  }
}

// Parallel form of work_ptr_kernel for many cells, two passes of 1024-cell
// CTAs: cell_scan_kernel writes each CTA's local inclusive prefix and its total
// (block_sums); cell_scan_add_kernel adds the totals of the CTAs before it.
constexpr int kScanCells = 1024;

__device__ __forceinline__ int block_inclusive_scan_1024(int x, int32_t* warp_tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
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
  return x + (warp > 0 ? warp_tot[warp - 1] : 0);
}

__global__ void __launch_bounds__(kScanCells) cell_scan_kernel(const int32_t* __restrict__ wave_off, int cells,
                                                               int num_rows, int tpc, int32_t* __restrict__ work_ptr,
                                                               int32_t* __restrict__ block_sums) {
  __shared__ int32_t warp_tot[32];
  const int cell = blockIdx.x * kScanCells + threadIdx.x;
  const int c = cell < cells ? (wave_off[cell + num_rows] - wave_off[cell] + tpc - 1) / tpc : 0;
  const int incl = block_inclusive_scan_1024(c, warp_tot);
  if (cell < cells) work_ptr[cell + 1] = incl;
  if (threadIdx.x == kScanCells - 1) block_sums[blockIdx.x] = incl;
  if (cell == 0) work_ptr[0] = 0;
}

__global__ void __launch_bounds__(kScanCells) cell_scan_add_kernel(int cells, const int32_t* __restrict__ block_sums,
                                                                   int32_t* __restrict__ work_ptr) {
  __shared__ int32_t part[32];
  if (blockIdx.x == 0) return;
  int s = 0;
  for (int i = threadIdx.x; i < (int)blockIdx.x; i += kScanCells) s += block_sums[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  int off = 0;
#pragma unroll
  for (int i = 0; i < 32; ++i) off += part[i];
  const int cell = blockIdx.x * kScanCells + threadIdx.x;
  if (cell < cells) work_ptr[cell + 1] += off;
}

// item_cell[w] = the cell of work item w (one thread per cell fills its items).
__global__ void item_cell_kernel(const int32_t* __restrict__ work_ptr, int cells, int32_t* __restrict__ item_cell) {
  const int stride = gridDim.x * blockDim.x;
  for (int cell = blockIdx.x * blockDim.x + threadIdx.x; cell < cells; cell += stride)
    for (int w = work_ptr[cell], end = work_ptr[cell + 1]; w < end; ++w) item_cell[w] = cell;
}

// Flags of item w (CSR row `row`) against the items its CTA takes just before
// and after it under ItemIter: bit 0 = first of a run on one key block (load
// K/V), bit 1 = last (release them). item_cell: the cell of every item.
__device__ __forceinline__ int item_run_flags(const int32_t* item_cell, int num_rows, int total, int grid, int w,
                                                  int row) {
  const int grp = w / kGroupItems;
  const int w_prev = (w % kGroupItems) ? w - 1 : (grp >= grid ? (grp - grid) * kGroupItems + kGroupItems - 1 : -1);
  const int w_next = (w % kGroupItems != kGroupItems - 1 && w + 1 < total) ? w + 1 : (grp + grid) * kGroupItems;
  const bool first = w_prev < 0 || item_cell[w_prev] % num_rows != row;
  const bool last = w_next >= total || item_cell[w_next] % num_rows != row;
  return (first ? 1 : 0) | (last ? 2 : 0);
}

}  // namespace
}  // namespace attn
}  // namespace msa
