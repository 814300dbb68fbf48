// Self-test of the tcgen05 building blocks: one 128 x nw output tile per CTA,
//   C = A * B^T  (B stored [N][K], K-major)      when layout bit 0 is clear
//   C = A * B    (B stored [K][N], N contiguous) when layout bit 0 is set
// with A stored [M][K] (K-major), or [K][M] (M contiguous, MN-major) when
// layout bit 1 is set; nw = 64 when layout bit 2 is set, else 128; K in
// {64, 128}, bf16/f16 in, f32 out. It drives the
// same TMA 128-byte-swizzle loads, UMMA descriptors, TMEM allocation and
// TMEM loads as the score and attention kernels, so a GPU test can pin the
// descriptor encodings against torch.matmul before those kernels run.
#include "tc_common.cuh"

namespace msa {
namespace {

using namespace tc;

constexpr int kTile = 128;

__global__ void __launch_bounds__(128)
selftest_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, float* c,
                int n_total, int k, int layout, uint32_t idesc, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;                        // k/64 chunks x 16 KB
  uint8_t* sb = smem + (k / 64) * 16384;     // same size
  __shared__ uint64_t full_bar, mma_bar;
  __shared__ uint32_t tmem_base;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b_mn_major = layout & 1, a_mn_major = (layout >> 1) & 1, nw = (layout & 4) ? 64 : 128;
  const int m0 = blockIdx.x * kTile, n0 = blockIdx.y * nw;
  if (threadIdx.x == 0) {
    mbar_init(&full_bar, 1);
    mbar_init(&mma_bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) { tmem_alloc(&tmem_base, 128); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  bool ok = true;
  if (threadIdx.x == 0) {
    const uint32_t bytes = 2u * (uint32_t)(k / 64) * 16384u;
    mbar_arrive_expect_tx(&full_bar, bytes);
    if (a_mn_major) {
      for (int mc = 0; mc < 2; ++mc) tma_load_2d(sa + mc * (k * 128), &map_a, &full_bar, m0 + mc * 64, 0);
    } else {
      for (int kc = 0; kc < k / 64; ++kc) tma_load_2d(sa + kc * 16384, &map_a, &full_bar, kc * 64, m0);
    }
    if (b_mn_major) {
      for (int nc = 0; nc < 2; ++nc) tma_load_2d(sb + nc * (k * 128), &map_b, &full_bar, n0 + nc * 64, 0);
    } else {
      for (int kc = 0; kc < k / 64; ++kc) tma_load_2d(sb + kc * 16384, &map_b, &full_bar, kc * 64, n0);
    }
    ok = mbar_wait(&full_bar, 0, err, 1);
    if (ok) {
      tc_fence_after();
      for (int ks = 0; ks < k / 16; ++ks) {
        const uint64_t da = a_mn_major ? desc_mnmajor_sw128(smem_u32(sa + ks * 2048), (uint32_t)k * 128)
                                       : desc_kmajor_sw128(smem_u32(sa + (ks / 4) * 16384 + (ks % 4) * 32));
        const uint64_t db = b_mn_major ? desc_mnmajor_sw128(smem_u32(sb + ks * 2048), (uint32_t)k * 128)
                                       : desc_kmajor_sw128(smem_u32(sb + (ks / 4) * 16384 + (ks % 4) * 32));
        umma_ss(tmem, da, db, idesc, ks > 0 ? 1u : 0u);
      }
      umma_commit(&mma_bar);
    }
  }
  __syncwarp();
  ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0 || warp != 0;
  if (ok && mbar_wait(&mma_bar, 0, err, 2)) {
    tc_fence_after();
    const int row = m0 + warp * 32 + lane;
    for (int cc = 0; cc < nw / 32; ++cc) {
      uint32_t r[32];
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + cc * 32, r);
      tmem_wait_ld();
      float* dst = c + (int64_t)row * n_total + n0 + cc * 32;
#pragma unroll
      for (int i = 0; i < 32; ++i) dst[i] = __uint_as_float(r[i]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

}  // namespace
}  // namespace msa

using namespace msa;

extern "C" int msa_selftest_umma(const void* a, const void* b, int dtype, int32_t m_tiles, int32_t n_tiles, int32_t k,
                                 int32_t layout, float* c, int32_t* err, void* stream) {
  MSA_CHECK_ARG(dtype == MSA_BF16 || dtype == MSA_F16, "msa_selftest_umma: bf16/f16 only");
  MSA_CHECK_ARG(k == 64 || k == 128, "msa_selftest_umma: k must be 64 or 128");
  MSA_CHECK_ARG(m_tiles >= 1 && n_tiles >= 1, "msa_selftest_umma: bad tiles");
  MSA_CHECK_ARG(layout >= 0 && layout < 8, "msa_selftest_umma: layout bits 0-2 only");
  const int b_mn_major = layout & 1, a_mn_major = (layout >> 1) & 1, nw = (layout & 4) ? 64 : 128;
  const uint64_t m = 128ull * m_tiles, n = (uint64_t)nw * n_tiles;
  CUtensorMap ma, mb;
  const uint32_t box_a[2] = {64, 128};
  if (a_mn_major) {
    const uint64_t da[2] = {m, (uint64_t)k}, sa[1] = {m * 2};
    const uint32_t box_am[2] = {64, (uint32_t)k};
    if (int st = tc::encode_tensor_map(&ma, tc::tma_dtype(dtype), 2, a, da, sa, box_am, CU_TENSOR_MAP_SWIZZLE_128B)) return st;
  } else {
    const uint64_t da[2] = {(uint64_t)k, m}, sa[1] = {(uint64_t)k * 2};
    if (int st = tc::encode_tensor_map(&ma, tc::tma_dtype(dtype), 2, a, da, sa, box_a, CU_TENSOR_MAP_SWIZZLE_128B)) return st;
  }
  if (b_mn_major) {
    const uint64_t db[2] = {n, (uint64_t)k}, sb[1] = {n * 2};
    const uint32_t box_b[2] = {64, (uint32_t)k};
    if (int st = tc::encode_tensor_map(&mb, tc::tma_dtype(dtype), 2, b, db, sb, box_b, CU_TENSOR_MAP_SWIZZLE_128B)) return st;
  } else {
    const uint64_t db[2] = {(uint64_t)k, n}, sb[1] = {(uint64_t)k * 2};
    if (int st = tc::encode_tensor_map(&mb, tc::tma_dtype(dtype), 2, b, db, sb, box_a, CU_TENSOR_MAP_SWIZZLE_128B)) return st;
  }
  const size_t smem = 2 * (k / 64) * 16384 + 1024;
  auto kern = selftest_kernel;
  MSA_CUDA_RETURN(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const uint32_t idesc = tc::idesc_f16(dtype == MSA_BF16, 128, nw, a_mn_major != 0, b_mn_major != 0);
  kern<<<dim3(m_tiles, n_tiles), 128, smem, as_stream(stream)>>>(ma, mb, c, (int)n, k, layout, idesc, err);
  count_launches(1);
  return launch_status("selftest_umma");
}
