// Tensor-pipe throughput of the block-scaled FP8 x FP4 MMA this library's GEMMs issue
// (tcgen05.mma kind::mxf8f6f4.block_scale: A = E4M3, B = E2M1 in its 8-bit container, UE8M0
// 1x32 scales), measured without memory traffic: the operand tiles and their scales stay
// resident in shared memory / TMEM and one thread per CTA (or CTA pair) issues `iters`
// 128-deep k blocks (4 MMAs of K = 32 each) into one accumulator, with the descriptors of
// moe_gemm_kernel's tokens-on-M tiles. It is the denominator of the tensor-bound GEMM
// rooflines (the block-scaled peak is not the bf16 one).
#pragma once
#include <cstdint>
#include "ptx.cuh"

namespace gptoss {

constexpr uint32_t kMpBTileBytes = 256u * 128u;   // up to 256 B rows of 128 bytes
constexpr uint32_t kMpSmemBytes = 1024u + 16384u + kMpBTileBytes + 3u * 512u;

// PAIR: a CTA pair (cluster of 2, cta_group::2): M = 256 (each CTA's 128 A rows), N = n
// (each CTA holds n / 2 B rows). Otherwise M = 128, N = n. n: a multiple of 16 up to 256.
template <bool PAIR>
__global__ void __launch_bounds__(128, 1) mma_peak_kernel(int n, int iters, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint32_t s_tmem;
  __shared__ __align__(8) uint64_t s_bar;
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t a_s = base, b_s = base + 16384u, sf_s = b_s + kMpBTileBytes;
  uint8_t* gen = smem_raw + (base - smem_u32(smem_raw));
  for (uint32_t i = threadIdx.x; i < (16384u + kMpBTileBytes + 3u * 512u) / 16u; i += blockDim.x)
    reinterpret_cast<uint4*>(gen)[i] = make_uint4(0, 0, 0, 0);   // zero operands and scales
  fence_proxy_async_shared();
  const uint32_t bar = smem_u32(&s_bar);
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  if (threadIdx.x < 32) {
    if constexpr (PAIR) {
      tmem_alloc_pair(smem_u32(&s_tmem), 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_u32(&s_tmem), 512);
      tmem_relinquish();
    }
  }
  if constexpr (PAIR) cluster_sync();
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  const bool leader = !PAIR || (cluster_ctarank() & 1u) == 0u;
  if (threadIdx.x == 0) {
    if (leader) {
      // TMEM: accumulator in columns [0, n); A scales at 256, B scales (two 128-row chunks) at 260
      const uint32_t t_sfa = tmem + 256u, t_sfb = tmem + 260u;
      if constexpr (PAIR) {
        tc_cp_32x128b_warpx4_pair(t_sfa, desc_sf_block(sf_s));
        tc_cp_32x128b_warpx4_pair(t_sfb, desc_sf_block(sf_s + 512u));
        tc_cp_32x128b_warpx4_pair(t_sfb + 4u, desc_sf_block(sf_s + 1024u));
      } else {
        tc_cp_32x128b_warpx4(t_sfa, desc_sf_block(sf_s));
        tc_cp_32x128b_warpx4(t_sfb, desc_sf_block(sf_s + 512u));
        tc_cp_32x128b_warpx4(t_sfb + 4u, desc_sf_block(sf_s + 1024u));
      }
      const uint32_t idesc0 = idesc_mxf8f6f4(0, 5, PAIR ? 256u : 128u, static_cast<uint32_t>(n), 0, 0);
      const uint64_t dA = desc_kmajor_sw128(a_s), dB = desc_kmajor_sw128(b_s);
      for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t idesc = idesc0 | (static_cast<uint32_t>(k) << 4) | (static_cast<uint32_t>(k) << 29);
          const uint32_t acc = (it != 0 || k != 0) ? 1u : 0u;
          if constexpr (PAIR) mma_mxf8f6f4_pair(tmem, dA + 2u * k, dB + 2u * k, idesc, t_sfa, t_sfb, acc);
          else mma_mxf8f6f4(tmem, dA + 2u * k, dB + 2u * k, idesc, t_sfa, t_sfb, acc);
        }
      }
      if constexpr (PAIR) tc_commit_pair(bar, 0x3);
      else tc_commit(bar);
    }
    (void)mbar_wait(bar, 0u, err, kDevTimeoutMma);   // every MMA done (both CTAs of a pair)
  }
  if constexpr (PAIR) cluster_sync();
  else __syncthreads();
  if (threadIdx.x < 32) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem, 512);
    else tmem_dealloc(tmem, 512);
  }
}

}  // namespace gptoss
