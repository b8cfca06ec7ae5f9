// Tensor-pipe throughput of the block-scaled MMAs this library's GEMMs issue, measured
// without memory traffic: the operand tiles and their scales stay resident in shared
// memory / TMEM and one thread per CTA (or CTA pair) issues `iters` k blocks of 4 MMAs into
// one accumulator, with the descriptors of moe_gemm_kernel's tokens-on-M tiles.
//   NVF4 = false: kind::mxf8f6f4.block_scale (A = E4M3, B = E2M1 in its 8-bit container,
//                 UE8M0 1x32 scales); a k block is 128 codes, 4 MMAs of K = 32.
//   NVF4 = true:  kind::mxf4nvf4.block_scale.scale_vec::4X (packed E2M1 x E2M1, UE4M3 1x16
//                 scales, the W4A4 mode); a k block is 256 codes, 4 MMAs of K = 64.
// It is the denominator of the tensor-bound GEMM rooflines (the block-scaled peaks are not
// the bf16 one).
#pragma once
#include <cstdint>
#include "ptx.cuh"

namespace gptoss {

constexpr uint32_t kMpBTileBytes = 256u * 128u;   // up to 256 B rows of 128 bytes
constexpr uint32_t kMpSfBytes = 3u * 2048u;       // A: 4 atoms; B: 2 row blocks x 4 atoms
constexpr uint32_t kMpSmemBytes = 1024u + 16384u + kMpBTileBytes + kMpSfBytes;

// PAIR: a CTA pair (cluster of 2, cta_group::2): M = 256 (each CTA's 128 A rows), N = n
// (each CTA holds n / 2 B rows). Otherwise M = 128, N = n. n: a multiple of 16 up to 256.
template <bool PAIR, bool NVF4>
__global__ void __launch_bounds__(128, 1) mma_peak_kernel(int n, int iters, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint32_t s_tmem;
  __shared__ __align__(8) uint64_t s_bar;
  constexpr uint32_t kAtoms = NVF4 ? 4u : 1u;   // 512-byte scale atoms per 128 rows per k block
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t a_s = base, b_s = base + 16384u, sf_s = b_s + kMpBTileBytes;
  uint8_t* gen = smem_raw + (base - smem_u32(smem_raw));
  for (uint32_t i = threadIdx.x; i < (16384u + kMpBTileBytes + kMpSfBytes) / 16u; i += blockDim.x)
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
      // TMEM: accumulator in columns [0, n); A scales from 256 (4 per atom), B scales from
      // 256 + 4 atoms (two 128-row blocks, atom-major: 8 columns per atom)
      const uint32_t t_sfa = tmem + 256u, t_sfb = tmem + 256u + 4u * kAtoms;
      const uint32_t sf_b_s = sf_s + 512u * kAtoms;
      for (uint32_t a = 0; a < kAtoms; ++a) {
        const uint64_t da = desc_sf_block(sf_s + 512u * a);
        const uint64_t db0 = desc_sf_block(sf_b_s + 512u * a), db1 = desc_sf_block(sf_b_s + 512u * (kAtoms + a));
        if constexpr (PAIR) {
          tc_cp_32x128b_warpx4_pair(t_sfa + 4u * a, da);
          tc_cp_32x128b_warpx4_pair(t_sfb + 8u * a, db0);
          tc_cp_32x128b_warpx4_pair(t_sfb + 8u * a + 4u, db1);
        } else {
          tc_cp_32x128b_warpx4(t_sfa + 4u * a, da);
          tc_cp_32x128b_warpx4(t_sfb + 8u * a, db0);
          tc_cp_32x128b_warpx4(t_sfb + 8u * a + 4u, db1);
        }
      }
      const uint32_t M = PAIR ? 256u : 128u;
      const uint32_t idesc0 = NVF4 ? idesc_mxf4nvf4(M, static_cast<uint32_t>(n))
                                   : idesc_mxf8f6f4(0, 5, M, static_cast<uint32_t>(n), 0, 0);
      const uint64_t dA = desc_kmajor_sw128(a_s), dB = desc_kmajor_sw128(b_s);
      for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (uint32_t k = 0; k < 4; ++k) {
          const uint32_t acc = (it != 0 || k != 0) ? 1u : 0u;
          if constexpr (NVF4) {
            // the 4 scales of this K = 64 step are one column (per row group)
            if constexpr (PAIR) mma_mxf4nvf4_pair(tmem, dA + 2u * k, dB + 2u * k, idesc0, t_sfa + 4u * k, t_sfb + 8u * k, acc);
            else mma_mxf4nvf4(tmem, dA + 2u * k, dB + 2u * k, idesc0, t_sfa + 4u * k, t_sfb + 8u * k, acc);
          } else {
            // byte k of the scale column: the scale of this K = 32 step
            const uint32_t idesc = idesc0 | (k << 4) | (k << 29);
            if constexpr (PAIR) mma_mxf8f6f4_pair(tmem, dA + 2u * k, dB + 2u * k, idesc, t_sfa, t_sfb, acc);
            else mma_mxf8f6f4(tmem, dA + 2u * k, dB + 2u * k, idesc, t_sfa, t_sfb, acc);
          }
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
