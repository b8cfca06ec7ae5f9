// Decode-sized MoE layer in one persistent launch (one CTA per SM): router, top-k,
// stable counting sort, FP8 quantisation, GEMM1 (+ bias + SwiGLU + FP8 requantisation)
// and GEMM2 (+ bias x routing weight, bf16 scatter-add). It replaces the three-launch
// decode path (decode_prologue_kernel -> GEMM1 -> GEMM2) for batches whose experts hold
// at most a few rows each (16-row activation chunks, weights on the MMA's M side).
//
// A decode step is a weight stream (13.25 MB per touched expert at GPT-OSS-20B shapes)
// with a few microseconds of dependent routing work in front of it. Here the stream
// starts at launch:
//   * before waiting on the previous kernel, the producer warp issues the weight and
//     weight-scale copies of the first kDlPreStages ring stages of the tile this CTA most
//     likely starts with (tile b when every expert is touched once); the activation half of those stages
//     is issued once the routing is known. A wrong guess costs those stages' bytes only
//     (the MMA warps release them unused);
//   * the routing runs on every CTA's idle warps: CTA b computes a 1/G share of the
//     router dot products (exact bf16 products summed in fp64, rounded once to bf16, so
//     the result does not depend on the summation order), a grid-wide counter publishes
//     them, and every CTA then runs the top-k, softmax and stable counting sort of all
//     tokens redundantly in its shared memory (identical inputs and code: identical
//     results), zeroes its slice of `out`, and quantises sorted rows b, b + G, ...
//     (per-expert counters publish the rows);
//   * GEMM1 and GEMM2 tiles run back to back on the same ring and TMEM accumulators: one
//     list holds every GEMM1 tile (expert-major) followed by every GEMM2 tile; CTA b starts
//     with tile b and then takes the next unclaimed tile from a global counter (one tile
//     ahead of its MMA), so the experts finish GEMM1 one after another, a GEMM2 tile comes up
//     several waves after the last GEMM1 tile of its expert, and CTAs that stream faster
//     take more tiles. A GEMM1 tile's activation loads wait until its expert's rows are all quantised; a
//     GEMM2 tile's wait until all of its expert's GEMM1 tiles have published their FP8
//     intermediate rows (a per-expert counter) -- in practice they never wait.
// Synchronisation words live in the workspace and are zeroed by decode_reset_kernel,
// launched right before this kernel (programmatic serialisation lets both start early).
// Every global write happens after griddepcontrol.wait; before it only the expert
// weights and their scales are read. Every wait is bounded (kWaitTimeoutNs): a role that
// gives up records an error word and the kernel still exits. The CTAs wait on each other,
// so the kernel expects all of its CTAs to become resident (grid = SM count, one CTA per
// SM), as every launch of this library does.
//
// Semantics are those of the three-launch path (cutlass_experts.py:376-452 with the router
// of GptOssTopKRouter in front); the router logits are the exactly rounded F.linear value.
// With `out_prefilled` the kernel adds into `out` as it is (the residual rows of a decoder
// block, gptoss_moe_block_forward) instead of zeroing it first.
//
// decode_layer_kernel<true> is the same kernel as one rank of an expert-parallel layer: the
// sort, quantisation and combine phases become dispatch / receive / combine over NVLink peer
// memory (see the comment at the kernel), the GEMMs run the rank's local experts on the rows
// it received, and GEMM2 stores into the sources' return rows.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include "ptx.cuh"
#include "numerics.cuh"
#include "routing.cuh"
#include "gemm.cuh"
#include "prologue.cuh"
#include "ep_p2p.cuh"

namespace gptoss {

constexpr int kDlMaxTokens = 64;
constexpr int kDlMaxAssign = 256;
constexpr int kDlMaxExperts = 128;
constexpr int kDlPreStages = 3;   // ring stages whose weights load before the routing is known

using DlCfg = GemmConfig<true, true, false>;
static_assert(kDlPreStages < DlCfg::kStages, "the routing scratch lives in the ring stages past the pre-loaded ones");

// Synchronisation words (int32, zeroed before every launch):
//   [0]              CTAs past the routing phase (their slice of `out` zeroed, their share
//                    of the activation rows quantised)
//   [1]              CTAs whose router dot products are written
//   [2, 2 + E)       GEMM1 tiles of expert e whose intermediate rows are written
//   [2 + E]          tiles handed out past every CTA's first one (dynamic scheduling)
__host__ __device__ constexpr int dl_sync_words(int E) { return 3 + E; }

constexpr int kDlQueue = 16;   // tile indices the producer publishes ahead of the MMA and epilogue

struct DecodeLayerParams {
  const __nv_bfloat16* x;          // [T, H]
  const __nv_bfloat16* router_w;   // [E, H]; nullptr: the routing is an input
  const __nv_bfloat16* router_b;   // [E]
  const int64_t* ridx_in;          // [T, K] (router_w == nullptr)
  const float* rw_in;              // [T, K]
  int T, H, I, E, K;
  int64_t* ridx_out;               // [T, K] (router mode)
  __nv_bfloat16* scores_out;       // [T, K] or nullptr
  float* rw_out;                   // [T, K] (router mode)
  __nv_bfloat16* out;              // [T, H]
  // workspace
  float* logits;                   // [T, E] bf16-rounded logits (router mode)
  int64_t* sorted_token;
  int64_t* sorted_expert;
  float* sorted_weight;
  int32_t* counts;
  int32_t* offsets;
  int32_t* sf_offsets_a;
  int32_t* sf_offsets_b;
  uint8_t* act_codes;              // [A, H] FP8
  uint8_t* act_sf;                 // blocked, SPREAD rows
  uint8_t* inter_codes;            // [A, I] FP8
  uint8_t* inter_sf;
  int32_t* sync;                   // dl_sync_words(E)
  // expert weights (scales in the blocked layout)
  const uint8_t* sfb_gu;
  int64_t sfb_stride_gu;
  const float* bias_gu;            // [E, 2I]
  const uint8_t* sfb_dn;
  int64_t sfb_stride_dn;
  const float* bias_dn;            // [E, H]
  float swiglu_alpha, swiglu_limit;
  int kb1, kb2;                    // 128-deep k blocks of GEMM1 (H padded) and GEMM2 (I padded)
  int n_tiles1, n_tiles2;          // 128-row weight tiles of GEMM1 (2I rows) and GEMM2 (H rows)
  int* err;
  // expert parallelism over peer memory (decode_layer_kernel<true>): E is the global expert
  // count (the router's), the GEMMs run the ep_epr local experts of rank ep_rank; the
  // exchange buffers, row format and flag protocol are those of ep_p2p.cuh
  int ep_world, ep_rank, ep_epr, ep_rb;
  int64_t ep_cap;                  // rows per (source, owner) segment
  uint8_t* ep_local;               // this rank's exchange buffer
  const uint64_t* ep_peer_bases;   // [W] every rank's exchange buffer (this rank's included)
  int32_t ep_epoch;
  int32_t* ep_send_counts;         // [W] rows sent to each owner (output)
  int32_t* ep_pos_of;              // [T, K] the assignment's row in the exchange (output)
  // L2 warm-up while the routing and the exchange run: the first l2_prefetch_bytes of the
  // local experts' weights in the order the tiles consume them (gate_up experts 0.., then
  // down experts 0..), each CTA a 1/G share (0: none)
  const uint8_t* wgu;              // [E, 2I, H/2]
  const uint8_t* wdn;              // [E, H, I/2]
  int64_t wgu_bytes, wdn_bytes;    // all local experts of each tensor
  int64_t l2_prefetch_bytes;
  int out_prefilled;               // `out` already holds the rows GEMM2 adds into (a residual)
};

// Received rows one rank of the expert-parallel kernel can hold (W x cap <= this).
constexpr int kEpMaxRecv = 1024;
static_assert(3 * kEpMaxRecv * 4 <= DlCfg::kEpiStageBytes, "received-row headers are staged in the epilogue buffer");

// Per-CTA routing state in shared memory.
template <bool EP>
struct DlSharedT {
  int cnt[kDlMaxExperts], off[kDlMaxExperts], sfa[kDlMaxExperts], sfb[kDlMaxExperts];
  int chunks[kDlMaxExperts], prefix[kDlMaxExperts + 1], run[kDlMaxExperts];
  int64_t tok[kDlMaxAssign];       // sorted position -> token
  float w[kDlMaxAssign];           // sorted position -> routing weight
  int sexp[kDlMaxAssign];          // sorted position -> expert
  int64_t ridx[kDlMaxAssign];      // assignment -> expert (-1: out of range)
  float rw[kDlMaxAssign];          // assignment -> routing weight
  uint64_t tq_bar[kDlQueue];       // tile queue: slot (i - 1) % kDlQueue holds the CTA's tile i >= 1
  int tq[kDlQueue];                // (tile 0 is the CTA index itself); -1 ends the list
};
// Expert parallelism: the sorted positions index the rows this rank received (up to
// kEpMaxRecv), and every local assignment keeps its row in the exchange.
template <>
struct DlSharedT<true> {
  int cnt[kDlMaxExperts], off[kDlMaxExperts], sfa[kDlMaxExperts], sfb[kDlMaxExperts];
  int chunks[kDlMaxExperts], prefix[kDlMaxExperts + 1], run[kDlMaxExperts];
  int32_t tok[kEpMaxRecv];         // sorted position -> received row (segment x cap + slot)
  float w[kEpMaxRecv];             // sorted position -> routing weight
  uint8_t sexp[kEpMaxRecv];        // sorted position -> local expert
  int64_t ridx[kDlMaxAssign];      // local assignment -> global expert (-1: out of range)
  float rw[kDlMaxAssign];          // local assignment -> routing weight
  int32_t dslot[kDlMaxAssign];     // local assignment -> owner x cap + slot (-1: not sent)
  int dcnt[kP2pMaxWorld];          // rows sent to each owner
  int rpre[kP2pMaxWorld + 1];      // received rows: exclusive prefix of the sources' counts
  uint64_t tq_bar[kDlQueue];
  int tq[kDlQueue];
};
using DlShared = DlSharedT<false>;

template <bool EP = false>
__host__ __device__ constexpr uint32_t dl_smem_bytes() {
  return 1024u + DlCfg::kStages * DlCfg::kStageBytes + ((DlCfg::kBarrierBytes + 255u) & ~255u) +
         DlCfg::kEpiStageBytes + static_cast<uint32_t>((sizeof(DlSharedT<EP>) + 255) & ~size_t(255));
}
static_assert(dl_smem_bytes<true>() <= 227u * 1024u, "expert-parallel decode layer: shared memory");

__device__ __forceinline__ int32_t ld_acquire_gpu(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Bounded wait until *p >= target (acquire). Returns false (and records `code`) on a
// timeout or when another role already reported an error.
__device__ __forceinline__ bool spin_wait_geq(const int32_t* p, int32_t target, int* err, int code) {
  if (ld_acquire_gpu(p) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (ld_acquire_gpu(p) >= target) return true;
    if ((it & 63u) == 0u) {
      if (*reinterpret_cast<volatile int*>(err) != 0) return false;
      if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
        atomicCAS(err, 0, code);
        return false;
      }
    }
  }
}

// Order-preserving key of a router logit for torch.topk order: larger floats -> larger keys,
// every NaN the largest key, -0 equal to +0; 0 is below every real key.
__device__ __forceinline__ uint32_t topk_key(float v) {
  if (v != v) return 0xffffffffu;
  const uint32_t b = __float_as_uint(v == 0.0f ? 0.0f : v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

enum DlError : int { kDlTimeoutGrid = 0x106, kDlTimeoutAct = 0x107, kDlTimeoutInter = 0x108 };

__global__ void decode_reset_kernel(int32_t* sync, int n) {
  pdl_trigger();
  pdl_wait();
  for (int i = threadIdx.x; i < n; i += blockDim.x) sync[i] = 0;
}

// grid = SM count, blockDim = DlCfg::kThreads (producer, MMA issuer, 4 epilogue warps,
// second MMA issuer), dynamic smem = dl_smem_bytes<EP>().
//
// EP = true: one rank of an expert-parallel layer over NVLink peer memory, the whole step
// in this launch (the five launches of the ep_p2p.cuh path): the router and top-k on this
// rank's tokens as above; then dispatch -- every CTA quantises its share of the local
// assignments straight into the owning ranks' receive rows (segment = this rank, slot =
// the assignment's stable rank among those to that owner), the last CTA raises this rank's
// dispatch flag on every peer; receive -- every CTA waits for all W dispatch flags, sorts
// the W x cap received rows by local expert in its shared memory and copies its share
// into the GEMM's activation layout; the GEMM tiles of the ep_epr local experts as above,
// GEMM2's epilogue storing each output row into its source rank's return rows; the last
// CTA raises this rank's return flag on every peer; combine -- every CTA waits for all W
// return flags and sums its tokens' k returned rows (ascending expert, fp32, one bf16
// rounding) into `out`. The weight stream of the first tiles still starts at launch, under
// the routing and the exchange.
template <bool EP>
__global__ void __launch_bounds__(DlCfg::kThreads, 1)
    decode_layer_kernel(const __grid_constant__ CUtensorMap tm_act, const __grid_constant__ CUtensorMap tm_inter,
                        const __grid_constant__ CUtensorMap tm_wgu, const __grid_constant__ CUtensorMap tm_wdn,
                        const DecodeLayerParams p, const GemmParams pg1_in, const GemmParams pg2_in) {
  using C = DlCfg;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint32_t s_tmem_base;
  __shared__ int s_epi_tile;   // the epilogue warps' tile, read from the queue by one thread
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int G = static_cast<int>(gridDim.x), cta = static_cast<int>(blockIdx.x);
  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* const smem_gen = smem_raw + (smem_base - smem_u32(smem_raw));   // generic view of smem_base
  const uint32_t bar_base = smem_base + C::kStages * C::kStageBytes;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (C::kStages + s); };
  auto accf_bar = [&](int b) { return bar_base + 8u * (2 * C::kStages + b); };
  auto acce_bar = [&](int b) { return bar_base + 8u * (2 * C::kStages + C::kAccBufs + b); };
  const uint32_t drain_bar = bar_base + 8u * (2 * C::kStages + 2 * C::kAccBufs);
  const uint32_t epi_off = C::kStages * C::kStageBytes + ((C::kBarrierBytes + 255u) & ~255u);
  float* const epi_f = reinterpret_cast<float*>(smem_gen + epi_off);
  DlSharedT<EP>& S = *reinterpret_cast<DlSharedT<EP>*>(smem_gen + epi_off + C::kEpiStageBytes);

  const int T = p.T, H = p.H, E = p.E, K = p.K, A = T * K;
  const int EG = EP ? p.ep_epr : E;   // experts the GEMMs run (this rank's, under expert parallelism)
  const bool router = p.router_w != nullptr;
  constexpr uint32_t kTxSub = C::kActRows * 128u + C::kWgtRowsCta * 64u + C::kSfActBytes + 512u;

  // ---- set-up: barriers, TMEM, descriptor prefetch
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_act);
    tma_prefetch_desc(&tm_inter);
    tma_prefetch_desc(&tm_wgu);
    tma_prefetch_desc(&tm_wdn);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), C::kIssuers);
    }
    for (int b = 0; b < C::kAccBufs; ++b) {
      mbar_init(accf_bar(b), C::kIssuers);
      mbar_init(acce_bar(b), C::kEpiWarps);
    }
    mbar_init(drain_bar, C::kIssuers);
    for (int j = 0; j < kDlQueue; ++j) mbar_init(smem_u32(&S.tq_bar[j]), 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&s_tmem_base), C::kTmemCols);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = s_tmem_base;

  // ---- weights of the likely first tile, before the routing (and the previous kernel)
  // are known: CTA b starts with GEMM1 tile b, (expert b / n1, weight tile b % n1) when every
  // expert is touched once.
  const bool guess_live = cta < EG * p.n_tiles1;
  const int e_g = cta / p.n_tiles1, nt_g = cta - e_g * p.n_tiles1;
  // The routing scratch (logits, their keys, top-k slots) lives in the epilogue staging buffer when
  // it fits -- then the whole ring is loaded ahead -- else in the ring stages past the
  // first kDlPreStages.
  const bool scratch_in_epi = static_cast<uint32_t>(T) * (2 * E + K) * 4u <= C::kEpiStageBytes;
  const int pre = guess_live ? min(scratch_in_epi ? C::kStages : kDlPreStages, (p.kb1 + C::kSubs - 1) / C::kSubs) : 0;
  auto sfb_gu_at = [&](int e, int nt, int kb) {
    return p.sfb_gu + static_cast<int64_t>(e) * p.sfb_stride_gu +
           static_cast<int64_t>((nt * C::kWgtRows) >> 7) * p.kb1 * 512 + static_cast<int64_t>(kb) * 512;
  };
  auto sfb_dn_at = [&](int e, int nt, int kb) {
    return p.sfb_dn + static_cast<int64_t>(e) * p.sfb_stride_dn +
           static_cast<int64_t>((nt * C::kWgtRows) >> 7) * p.kb2 * 512 + static_cast<int64_t>(kb) * 512;
  };
  if (warp == 0 && elect_one()) {
    const uint64_t pol_w = policy_evict_first();
    for (int s = 0; s < pre; ++s) {
      const int nsub = min(C::kSubs, p.kb1 - s * C::kSubs);
      mbar_arrive_expect_tx(full_bar(s), kTxSub * static_cast<uint32_t>(nsub));
      for (int j = 0; j < nsub; ++j) {
        const int kb = s * C::kSubs + j;
        const uint32_t sb = smem_base + s * C::kStageBytes + j * C::kSubBytes;
        tma_load_3d(sb, &tm_wgu, full_bar(s), kb * 128, nt_g * C::kWgtRows, e_g, pol_w);
        bulk_load(sb + C::kWgtTileBytes + C::kActTileBytes + C::kSfActBytes, sfb_gu_at(e_g, nt_g, kb), 512,
                  full_bar(s), pol_w);
      }
    }
  }
  if (router) {   // the router weight rows this CTA's dot products read (not written upstream)
    const int np = T * E;
    const int plo = static_cast<int>(static_cast<int64_t>(np) * cta / G);
    const int phi = static_cast<int>(static_cast<int64_t>(np) * (cta + 1) / G);
    for (int pr = plo + warp; pr < phi; pr += nthr / 32)
      if (lane == 0) bulk_prefetch_l2(p.router_w + static_cast<int64_t>(pr % E) * H, static_cast<uint32_t>(H) * 2u);
  }
  if constexpr (EP) {
    // Expert-parallel steps stream only this rank's experts: up to a budget that L2 holds,
    // pull them into L2 under the routing and the exchange (the tiles that follow the
    // pre-loaded first stages then read L2 instead of HBM). Weights are not written upstream.
    if (warp == 3 && lane == 0 && p.l2_prefetch_bytes > 0) {
      const int64_t total = min(p.l2_prefetch_bytes, p.wgu_bytes + p.wdn_bytes);
      const int64_t lo = (total * cta / G) & ~static_cast<int64_t>(15);
      const int64_t hi = cta == G - 1 ? total : (total * (cta + 1) / G) & ~static_cast<int64_t>(15);
      constexpr int64_t kPiece = 64 * 1024;
      for (int64_t o = lo; o < hi; o += kPiece) {
        const int64_t n = min(kPiece, hi - o);
        if (o < p.wgu_bytes) {
          bulk_prefetch_l2(p.wgu + o, static_cast<uint32_t>(min(n, p.wgu_bytes - o)));
        } else {
          bulk_prefetch_l2(p.wdn + (o - p.wgu_bytes), static_cast<uint32_t>(n));
        }
      }
    }
  }
  pdl_trigger();
  pdl_wait();

  // ================================================================ routing (all warps)
  // zero this CTA's slice of `out` (GEMM2 adds into it; expert-parallel: the combine writes it;
  // a prefilled `out` -- the residual of a block -- is added into as it is)
  if (!EP && !p.out_prefilled) {
    const int64_t n16 = static_cast<int64_t>(T) * H / 8;
    const int64_t lo = n16 * cta / G, hi = n16 * (cta + 1) / G;
    uint4* z = reinterpret_cast<uint4*>(p.out);
    for (int64_t i = lo + tid; i < hi; i += nthr) z[i] = make_uint4(0, 0, 0, 0);
  }
  if (router) {
    // this CTA's share of the T*E router dot products, one warp per (token, expert):
    // exact bf16 x bf16 products (exact in fp32) summed in fp64 with a fixed butterfly,
    // + bias, one rounding to bf16 (the exactly rounded value of F.linear)
    const int np = T * E;
    const int plo = static_cast<int>(static_cast<int64_t>(np) * cta / G);
    const int phi = static_cast<int>(static_cast<int64_t>(np) * (cta + 1) / G);
    const int nwarps = nthr / 32;
    for (int pr = plo + warp; pr < phi; pr += nwarps) {
      const int t = pr / E, e = pr - t * E;
      const uint4* xr = reinterpret_cast<const uint4*>(p.x + static_cast<int64_t>(t) * H);
      const uint4* wr = reinterpret_cast<const uint4*>(p.router_w + static_cast<int64_t>(e) * H);
      // four 16-byte vectors of each operand in flight per lane, one fp64 partial each
      double part[4] = {0.0, 0.0, 0.0, 0.0};
      const int nv = H / 8;
      for (int v0 = lane; v0 < nv; v0 += 4 * 32) {
        uint4 a[4], w4[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int v = v0 + 32 * u;
          a[u] = v < nv ? __ldg(xr + v) : make_uint4(0, 0, 0, 0);
          w4[u] = v < nv ? __ldg(wr + v) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint32_t av[4] = {a[u].x, a[u].y, a[u].z, a[u].w}, wv[4] = {w4[u].x, w4[u].y, w4[u].z, w4[u].w};
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            part[u] += static_cast<double>(__fmul_rn(bf16_bits_lo(av[h]), bf16_bits_lo(wv[h])));
            part[u] += static_cast<double>(__fmul_rn(bf16_bits_hi(av[h]), bf16_bits_hi(wv[h])));
          }
        }
      }
      double acc = (part[0] + part[1]) + (part[2] + part[3]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0)
        p.logits[pr] = __bfloat162float(__double2bfloat16(acc + static_cast<double>(__bfloat162float(p.router_b[e]))));
    }
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      atomicAdd(p.sync + 1, 1);
      (void)spin_wait_geq(p.sync + 1, G, p.err, kDlTimeoutGrid);
    }
    __syncthreads();
    // every CTA: all logits (L2, bypassing L1) -> the routing scratch in ring stages the
    // pre-loads do not use, then one thread per token: top-k + softmax
    float* lg = scratch_in_epi ? epi_f : reinterpret_cast<float*>(smem_gen + kDlPreStages * C::kStageBytes);
    float* slot_v = lg + np;
    uint32_t* keys = reinterpret_cast<uint32_t*>(slot_v + T * K);
    for (int i = tid; i < np; i += nthr) {
      const float v = __ldcg(p.logits + i);
      lg[i] = v;
      keys[i] = topk_key(v);
    }
    __syncthreads();
    // top-k in torch.topk order (larger first, NaN above every number, equal values by
    // ascending expert id): thread per (token, expert) counts the experts ranked ahead of
    // it on order-preserving integer keys (loads batched by the unrolled loop), so slot
    // `rank` of token t holds its rank-th choice; then one thread per token applies the
    // softmax over the K values in rank order (the operation order of router_topk_token)
    for (int q = tid; q < np; q += nthr) {
      const int t = q / E, e = q - t * E;
      const uint32_t* kr = keys + t * E;
      const uint32_t ke = kr[e];
      int rk = 0;
#pragma unroll 8
      for (int f = 0; f < E; ++f) {
        const uint32_t kf = kr[f];
        rk += (kf > ke || (kf == ke && f < e)) ? 1 : 0;
      }
      if (rk < K) {
        S.ridx[t * K + rk] = e;
        slot_v[t * K + rk] = lg[q];
      }
    }
    __syncthreads();
    for (int t = tid; t < T; t += nthr) {
      const float m = slot_v[t * K];
      float ex[kMaxTopK], sum = 0.0f;
#pragma unroll
      for (int j = 0; j < kMaxTopK; ++j)
        if (j < K) { ex[j] = expf(__fsub_rn(slot_v[t * K + j], m)); sum = __fadd_rn(sum, ex[j]); }
      const float inv = __frcp_rn(sum);
#pragma unroll
      for (int j = 0; j < kMaxTopK; ++j)
        if (j < K) S.rw[t * K + j] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(ex[j], inv)));
    }
  } else {
    for (int i = tid; i < A; i += nthr) {
      const int64_t v = p.ridx_in[i];
      if (v < 0 || v >= E) {
        if (cta == 0) atomicCAS(p.err, 0, 0x201);
        S.ridx[i] = -1;
      } else {
        S.ridx[i] = v;
      }
      S.rw[i] = p.rw_in[i];
    }
  }
  // exclusive scans of the GEMM experts' row counts (warp 0): row offsets, scale offsets
  // (SPREAD rows), 16-row chunks
  auto scan_counts = [&]() {
    const int per = (EG + 31) / 32, q0 = lane * per;
    int c_run = 0, a_run = 0, b_run = 0, k_run = 0;
    for (int i = 0; i < per; ++i) {
      const int q = q0 + i;
      if (q < EG) {
        c_run += S.cnt[q];
        a_run += static_cast<int>(act_sf_cosize(S.cnt[q], p.kb1 * 4, true));
        b_run += static_cast<int>(act_sf_cosize(S.cnt[q], p.kb2 * 4, true));
        k_run += (S.cnt[q] + C::kActRows - 1) / C::kActRows;
      }
    }
    int ci = c_run, ai = a_run, bi = b_run, ki = k_run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int c2 = __shfl_up_sync(0xffffffffu, ci, o), a2 = __shfl_up_sync(0xffffffffu, ai, o);
      const int b2 = __shfl_up_sync(0xffffffffu, bi, o), k2 = __shfl_up_sync(0xffffffffu, ki, o);
      if (lane >= o) { ci += c2; ai += a2; bi += b2; ki += k2; }
    }
    int ce = ci - c_run, ae = ai - a_run, be = bi - b_run, ke = ki - k_run;
    for (int i = 0; i < per; ++i) {
      const int q = q0 + i;
      if (q < EG) {
        const int m = S.cnt[q];
        S.off[q] = ce; S.run[q] = ce; S.sfa[q] = ae; S.sfb[q] = be;
        S.chunks[q] = (m + C::kActRows - 1) / C::kActRows;
        S.prefix[q] = ke;
        ce += m;
        ae += static_cast<int>(act_sf_cosize(m, p.kb1 * 4, true));
        be += static_cast<int>(act_sf_cosize(m, p.kb2 * 4, true));
        ke += S.chunks[q];
      }
    }
    if (lane == 31) S.prefix[EG] = ki;
    __syncwarp();
  };
  // expert parallelism: the exchange rows of this rank's receive buffer
  const uint8_t* const recv = EP ? p.ep_local + p2p_recv_offset(0, p.ep_cap, p.ep_rb) : nullptr;
  if constexpr (!EP) {
    for (int e = tid; e < E; e += nthr) S.cnt[e] = 0;
    __syncthreads();
    for (int i = tid; i < A; i += nthr)
      if (S.ridx[i] >= 0) atomicAdd(&S.cnt[S.ridx[i]], 1);
    __syncthreads();
    if (warp == 0) {
      scan_counts();
      // stable positions, 32 assignments at a time (lanes of one expert rank by lane order)
      for (int i0 = 0; i0 < A; i0 += 32) {
        const int i = i0 + lane;
        const int e = i < A ? static_cast<int>(S.ridx[i]) : -2;
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        if (e >= 0) {
          const int pos = S.run[e] + __popc(peers & ((1u << lane) - 1u));
          S.tok[pos] = i / K;
          S.w[pos] = S.rw[i];
          S.sexp[pos] = e;
        }
        __syncwarp();
        if (e >= 0 && lane == __ffs(peers) - 1) S.run[e] += __popc(peers);
        __syncwarp();
      }
    }
    __syncthreads();
  } else {
    // ================================================================ dispatch
    const int W = p.ep_world, epr = p.ep_epr, rb = p.ep_rb;
    const int64_t cap = p.ep_cap;
    __syncthreads();   // every thread's S.ridx / S.rw (the top-k's or the given routing) is in
    // owner q = expert / epr; slot j = the assignment's stable rank among those to q
    if (warp == 0) {
      for (int q = lane; q < W; q += 32) S.dcnt[q] = 0;
      __syncwarp();
      for (int i0 = 0; i0 < A; i0 += 32) {
        const int i = i0 + lane;
        const int q = (i < A && S.ridx[i] >= 0) ? static_cast<int>(S.ridx[i] / epr) : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, q);
        if (q >= 0) {
          const int j = S.dcnt[q] + __popc(peers & ((1u << lane) - 1u));
          S.dslot[i] = j < cap ? static_cast<int32_t>(q * cap + j) : -1;
        } else if (i < A) {
          S.dslot[i] = -1;
        }
        __syncwarp();
        if (q >= 0 && lane == __ffs(peers) - 1) S.dcnt[q] += __popc(peers);
        __syncwarp();
      }
    }
    __syncthreads();
    if (cta == 0) {   // the routing outputs of the API
      if (router) {
        for (int i = tid; i < A; i += nthr) {
          p.ridx_out[i] = S.ridx[i];
          if (p.scores_out) p.scores_out[i] = __float2bfloat16_rn(S.rw[i]);
          p.rw_out[i] = S.rw[i];
        }
      }
      for (int q = tid; q < W; q += nthr) {
        const int32_t c = static_cast<int32_t>(min(static_cast<int64_t>(S.dcnt[q]), cap));
        p.ep_send_counts[q] = c;
        // the owner reads how many rows this rank sent (published by the dispatch flag)
        reinterpret_cast<int32_t*>(p.ep_peer_bases[q])[kP2pSendCounts + p.ep_rank] = c;
      }
      for (int i = tid; i < A; i += nthr) p.ep_pos_of[i] = S.dslot[i];
    }
    // this CTA's local assignments cta, cta + G, ...: FP8 codes and UE8M0 scales straight into
    // the owner's receive row (a row per assignment, in the ep_pack_p2p_row format)
    {
      const int gv = H / 32;
      const int nmine = cta < A ? (A - cta + G - 1) / G : 0;
      for (int q = tid; q < nmine * gv; q += nthr) {
        const int r = q / gv, g = q - r * gv;
        const int i = cta + r * G;
        const int slot = S.dslot[i];
        if (slot < 0) continue;
        const int own = static_cast<int>(slot / cap);
        const int64_t j = slot - static_cast<int64_t>(own) * cap;
        uint8_t* row = reinterpret_cast<uint8_t*>(p.ep_peer_bases[own]) + p2p_recv_offset(p.ep_rank, cap, rb) + j * rb;
        const uint4* src = reinterpret_cast<const uint4*>(p.x + static_cast<int64_t>(i / K) * H + 32 * g);
        float v[32];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint4 w4 = __ldg(src + u);
          const uint32_t wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            v[8 * u + 2 * h] = bf16_bits_lo(wv[h]);
            v[8 * u + 2 * h + 1] = bf16_bits_hi(wv[h]);
          }
        }
        uint32_t cw[8];
        const uint8_t sc = quantize_group32(v, cw);
        uint4* dst = reinterpret_cast<uint4*>(row + 32 * g);
        dst[0] = make_uint4(cw[0], cw[1], cw[2], cw[3]);
        dst[1] = make_uint4(cw[4], cw[5], cw[6], cw[7]);
        row[H + g] = sc;
        if (g == 0) {
          for (int b = H + gv; b < rb - 8; ++b) row[b] = 0;   // padding travels as zeros
          int32_t* meta = reinterpret_cast<int32_t*>(row + rb - 8);
          meta[0] = static_cast<int32_t>(S.ridx[i] % epr);
          meta[1] = __float_as_int(S.rw[i]);
        }
      }
      // every owner's slots past this rank's count carry the empty-slot marker
      for (int64_t f = static_cast<int64_t>(cta) * nthr + tid; f < W * cap; f += static_cast<int64_t>(G) * nthr) {
        const int own = static_cast<int>(f / cap);
        const int64_t j = f - static_cast<int64_t>(own) * cap;
        if (j < S.dcnt[own]) continue;
        int32_t* meta = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(p.ep_peer_bases[own]) +
                                                   p2p_recv_offset(p.ep_rank, cap, rb) + j * rb + rb - 8);
        meta[0] = -1;
        meta[1] = 0;
      }
    }
    __syncthreads();
    if (tid < 32)
      p2p_last_cta_signal(reinterpret_cast<int32_t*>(p.ep_local) + kP2pCounterDispatch, p.ep_peer_bases, W,
                          p.ep_rank, p.ep_epoch);
    // ================================================================ receive
    p2p_wait_flags(reinterpret_cast<const int32_t*>(p.ep_local), 0, W, p.ep_epoch, p.err);
    // the valid rows: source s sent rows [0, count_s) of its segment (its count travels with
    // its flag), so only those headers are read, in (source, slot) order
    if (tid == 0) {
      int acc = 0;
      for (int src = 0; src < W; ++src) {
        S.rpre[src] = acc;
        acc += min(max(__ldcg(reinterpret_cast<const int32_t*>(p.ep_local) + kP2pSendCounts + src), 0),
                   static_cast<int>(cap));
      }
      S.rpre[W] = acc;
    }
    for (int e = tid; e < EG; e += nthr) S.cnt[e] = 0;
    __syncthreads();
    const int nvalid = S.rpre[W];
    // row headers (local expert, routing weight, row) in the epilogue staging, free until the GEMMs
    int* hexp = reinterpret_cast<int*>(epi_f);
    float* hw = epi_f + kEpMaxRecv;
    int* hrow = reinterpret_cast<int*>(epi_f + 2 * kEpMaxRecv);
    for (int v = tid; v < nvalid; v += nthr) {
      int src = 0;
      while (S.rpre[src + 1] <= v) ++src;
      const int r = static_cast<int>(src * cap) + (v - S.rpre[src]);
      const int32_t* meta = reinterpret_cast<const int32_t*>(recv + static_cast<int64_t>(r) * rb + rb - 8);
      int e = __ldcg(meta);
      const float wv = __int_as_float(__ldcg(meta + 1));
      if (e >= EG || e < -1) {
        if (cta == 0) atomicCAS(p.err, 0, 0x201);
        e = -1;
      }
      hexp[v] = e;
      hw[v] = wv;
      hrow[v] = r;
      if (e >= 0) atomicAdd(&S.cnt[e], 1);
    }
    __syncthreads();
    if (warp == 0) {
      scan_counts();
      // stable positions over the received rows (source rank, then slot)
      for (int i0 = 0; i0 < nvalid; i0 += 32) {
        const int v = i0 + lane;
        const int e = v < nvalid ? hexp[v] : -2;
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        if (e >= 0) {
          const int pos = S.run[e] + __popc(peers & ((1u << lane) - 1u));
          S.tok[pos] = hrow[v];
          S.w[pos] = hw[v];
          S.sexp[pos] = static_cast<uint8_t>(e);
        }
        __syncwarp();
        if (e >= 0 && lane == __ffs(peers) - 1) S.run[e] += __popc(peers);
        __syncwarp();
      }
    }
    __syncthreads();
  }
  const int total = S.off[EG - 1] + S.cnt[EG - 1];     // rows with a valid expert
  const int nchunks = S.prefix[EG];
  // one tile list: GEMM1 tiles [0, q1), then GEMM2 tiles [q1, q1 + q2); CTA b takes b, b + G, ...
  const int q1 = nchunks * p.n_tiles1, q2 = nchunks * p.n_tiles2;
  const int qall = q1 + q2;
  // Tile schedule: CTA b's first tile is tile b (what its pre-loaded stages guessed); every
  // later one comes from a global counter (first come, first served), so CTAs that stream
  // faster take more tiles. The producer publishes each tile index through S.tq.
  const int t_first = cta < qall ? cta : -1;
  auto queued_tile = [&](int i, bool& ok) -> int {   // tile i >= 1 of this CTA, or -1
    const int slot = (i - 1) % kDlQueue;
    if (!mbar_wait(smem_u32(&S.tq_bar[slot]), static_cast<uint32_t>((i - 1) / kDlQueue) & 1u, p.err,
                   kDevTimeoutMma)) {
      ok = false;
      return -1;
    }
    return *reinterpret_cast<volatile int*>(&S.tq[slot]);
  };

  // CTA 0: the routing outputs of the API and the routed layout of the workspace
  if constexpr (!EP) {
    if (cta == 0) {
      if (router) {
        for (int i = tid; i < A; i += nthr) {
          p.ridx_out[i] = S.ridx[i];
          if (p.scores_out) p.scores_out[i] = __float2bfloat16_rn(S.rw[i]);
          p.rw_out[i] = S.rw[i];
        }
      }
      for (int i = tid; i < A; i += nthr) {
        const bool v = i < total;
        p.sorted_token[i] = v ? S.tok[i] : -1;
        p.sorted_expert[i] = v ? S.sexp[i] : -1;
        p.sorted_weight[i] = v ? S.w[i] : 0.0f;
      }
      for (int e = tid; e < E; e += nthr) {
        p.counts[e] = S.cnt[e];
        p.offsets[e] = S.off[e];
        p.sf_offsets_a[e] = S.sfa[e];
        p.sf_offsets_b[e] = S.sfb[e];
      }
    }
  }
  // tile t of a GEMM's list -> (expert, weight tile, 16-row chunk); chunks innermost
  auto decode = [&](int t, int n_tiles, int& e, int& nt, int& ch) {
    const int cidx = t / n_tiles;
    int lo = 0, hi = EG - 1;
    while (lo < hi) {                         // last e with prefix[e] <= cidx
      const int mid = (lo + hi + 1) >> 1;
      if (S.prefix[mid] <= cidx) lo = mid; else hi = mid - 1;
    }
    e = lo;
    const int local = t - S.prefix[e] * n_tiles;
    const int nch = S.chunks[e];
    nt = local / nch;
    ch = local - nt * nch;
  };
  // tile t of the combined list (GEMM1 tiles, then GEMM2 tiles)
  auto tile_of = [&](int t, bool& g2, int& e, int& nt, int& ch) {
    g2 = t >= q1;
    if (g2) decode(t - q1, p.n_tiles2, e, nt, ch);
    else decode(t, p.n_tiles1, e, nt, ch);
  };
  // quantise sorted rows cta, cta + G, ... (expert parallelism: copy the received rows): each
  // row's codes and blocked scales; the CTA then counts itself into sync[0] (the activation
  // loads wait until every CTA has: one wait per CTA instead of one acquire round trip per
  // expert on the producer's path)
  {
    const int gp = 4 * p.kb1;                 // scale groups per row incl. K padding
    const int gv = H / 32;                    // valid groups
    const int nmine = cta < total ? (total - cta + G - 1) / G : 0;
    if constexpr (!EP) {
      for (int q = tid; q < nmine * gp; q += nthr) {
        const int r = q / gp, g = q - r * gp;
        const int pos = cta + r * G;
        const int e = S.sexp[pos], j = pos - S.off[e];
        uint8_t sc = 0;
        if (g < gv) {
          const uint4* src = reinterpret_cast<const uint4*>(p.x + S.tok[pos] * H + 32 * g);
          float v[32];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const uint4 w4 = __ldg(src + u);
            const uint32_t wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              v[8 * u + 2 * h] = bf16_bits_lo(wv[h]);
              v[8 * u + 2 * h + 1] = bf16_bits_hi(wv[h]);
            }
          }
          uint32_t cw[8];
          sc = quantize_group32(v, cw);
          uint4* dst = reinterpret_cast<uint4*>(p.act_codes + static_cast<int64_t>(pos) * H + 32 * g);
          dst[0] = make_uint4(cw[0], cw[1], cw[2], cw[3]);
          dst[1] = make_uint4(cw[4], cw[5], cw[6], cw[7]);
        }
        p.act_sf[S.sfa[e] + blocked_sf_offset(act_sf_row<true>(j), g, p.kb1)] = sc;   // K padding: 0
      }
    } else {
      const int64_t rb = p.ep_rb;
      const int nv = H / 16;
      for (int q = tid; q < nmine * nv; q += nthr) {
        const int r = q / nv, v = q - r * nv;
        const int pos = cta + r * G;
        reinterpret_cast<uint4*>(p.act_codes + static_cast<int64_t>(pos) * H)[v] =
            __ldcg(reinterpret_cast<const uint4*>(recv + static_cast<int64_t>(S.tok[pos]) * rb) + v);
      }
      for (int q = tid; q < nmine * gp; q += nthr) {
        const int r = q / gp, g = q - r * gp;
        const int pos = cta + r * G;
        const int e = S.sexp[pos], j = pos - S.off[e];
        const uint8_t sc = g < gv ? __ldcg(recv + static_cast<int64_t>(S.tok[pos]) * rb + H + g) : uint8_t{0};
        p.act_sf[S.sfa[e] + blocked_sf_offset(act_sf_row<true>(j), g, p.kb1)] = sc;   // K padding: 0
      }
    }
    fence_proxy_async_global();               // the rows are read by other CTAs' TMA copies
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      atomicAdd(p.sync + 0, 1);               // this CTA's slice of `out` is zero
    }
  }

  // the first real tile and whether the pre-loaded stages belong to it
  bool match = false;
  if (pre > 0 && cta < q1) {
    int e0, nt0, ch0;
    decode(cta, p.n_tiles1, e0, nt0, ch0);
    match = e0 == e_g && nt0 == nt_g && ch0 == 0;
  }

  if (warp == 0) {
    // ================================================================ producer
    if (elect_one()) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_a = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int ready_e2 = -1;
      bool all_rows = false;   // every CTA's activation rows quantised and its slice of `out` zeroed
      // activation half of the pre-loaded stages: the first tile's rows, or (the guess was
      // wrong) any in-range rows -- the MMA warps release those stages unused
      if (pre > 0) {
        int e0 = 0, ch0 = 0;
        if (match) {
          int nt0;
          decode(cta, p.n_tiles1, e0, nt0, ch0);
          ok = spin_wait_geq(p.sync + 0, G, p.err, kDlTimeoutAct);
          fence_proxy_async_global();
          all_rows = true;
        }
        const int row = match ? S.off[e0] : 0;
        const int64_t sfa_base = match ? S.sfa[e0] : 0;
        for (int s = 0; s < pre; ++s) {
          const int nsub = min(C::kSubs, p.kb1 - s * C::kSubs);
          for (int j = 0; j < nsub; ++j) {
            const int kb = s * C::kSubs + j;
            const uint32_t sb = smem_base + s * C::kStageBytes + j * C::kSubBytes;
            tma_load_2d(sb + C::kWgtTileBytes, &tm_act, full_bar(s), kb * 128, row, pol_a);
            bulk_load(sb + C::kWgtTileBytes + C::kActTileBytes, p.act_sf + sfa_base + static_cast<int64_t>(kb) * 512,
                      512, full_bar(s), pol_a);
          }
        }
        stage = pre;   // pre <= kStages: the next stage wraps to 0 when every stage was pre-loaded
        if (stage == C::kStages) { stage = 0; phase ^= 1u; }
      }
      int t_next = -1;
      for (int i = 0; ok; ++i) {
        const int t = i == 0 ? t_first : (t_next < qall ? t_next : -1);
        if (i > 0) {                          // publish tile i (or the end of the list)
          const int slot = (i - 1) % kDlQueue;
          *reinterpret_cast<volatile int*>(&S.tq[slot]) = t;
          mbar_arrive(smem_u32(&S.tq_bar[slot]));
        }
        if (t < 0) break;
        t_next = G + atomicAdd(p.sync + 2 + EG, 1);   // the next tile, one tile ahead
        bool g2;
        int e, nt, ch;
        tile_of(t, g2, e, nt, ch);
        const int num_kb = g2 ? p.kb2 : p.kb1;
        // One wait per CTA for the activation rows (every CTA counts itself into sync[0] once
        // its share is quantised): an acquire load is a blocking L2 round trip on the
        // producer's path, so it is not repeated per expert. GEMM2 tiles wait per expert for
        // the expert's GEMM1 tiles (in practice they are long done).
        if (!all_rows) {
          if (!spin_wait_geq(p.sync + 0, G, p.err, kDlTimeoutAct)) { ok = false; break; }
          fence_proxy_async_global();
          all_rows = true;
        }
        if (g2 && e != ready_e2) {
          if (!spin_wait_geq(p.sync + 2 + e, p.n_tiles1 * S.chunks[e], p.err, kDlTimeoutInter)) {
            ok = false;
            break;
          }
          fence_proxy_async_global();
          ready_e2 = e;
        }
        const CUtensorMap* wmap = g2 ? &tm_wdn : &tm_wgu;
        const CUtensorMap* amap = g2 ? &tm_inter : &tm_act;
        const uint8_t* asf = g2 ? p.inter_sf : p.act_sf;
        const int row = S.off[e] + ch * C::kActRows;
        const int64_t sfa_off = (g2 ? S.sfb[e] : S.sfa[e]) +
                                static_cast<int64_t>(act_sf_row<true>(static_cast<int64_t>(ch) * C::kActRows) >> 7) *
                                    num_kb * 512;
        for (int kb0 = (i == 0 && match) ? pre * C::kSubs : 0; kb0 < num_kb; kb0 += C::kSubs) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.err, kDevTimeoutProducer)) { ok = false; break; }
          const int nsub = min(C::kSubs, num_kb - kb0);
          mbar_arrive_expect_tx(full_bar(stage), kTxSub * static_cast<uint32_t>(nsub));
          for (int j = 0; j < nsub; ++j) {
            const int kb = kb0 + j;
            const uint32_t sb = smem_base + stage * C::kStageBytes + j * C::kSubBytes;
            const uint32_t s_a = sb + C::kWgtTileBytes, s_sfa = s_a + C::kActTileBytes, s_sfw = s_sfa + C::kSfActBytes;
            tma_load_3d(sb, wmap, full_bar(stage), kb * 128, nt * C::kWgtRows, e, pol_w);
            bulk_load(s_sfw, g2 ? sfb_dn_at(e, nt, kb) : sfb_gu_at(e, nt, kb), 512, full_bar(stage), pol_w);
            tma_load_2d(s_a, amap, full_bar(stage), kb * 128, row, pol_a);
            bulk_load(s_sfa, asf + sfa_off + static_cast<int64_t>(kb) * 512, 512, full_bar(stage), pol_a);
          }
          if (++stage == C::kStages) { stage = 0; phase ^= 1u; }
        }
      }
      // drain: no copy may still be landing in shared memory at exit
      for (int s = 0; s < C::kStages; ++s) {
        const uint32_t ph = (s < stage) ? phase : (phase ^ 1u);
        (void)mbar_wait(full_bar(s), ph, p.err, kDevTimeoutDrain);
      }
    }
  } else if (warp == 1 || warp == 2 + C::kEpiWarps) {
    // ================================================================ MMA issuers
    const int issuer = warp == 1 ? 0 : 1;
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      if (pre > 0 && !match) {   // the pre-loaded stages of a wrong guess: release them unused
        for (int s = 0; s < pre && ok; ++s) {
          if (!mbar_wait(full_bar(s), 0u, p.err, kDevTimeoutMma)) { ok = false; break; }
          tc_commit(empty_bar(s));
        }
        stage = pre;   // pre <= kStages: the next stage wraps to 0 when every stage was pre-loaded
        if (stage == C::kStages) { stage = 0; phase ^= 1u; }
      }
      for (int i = 0; ok; ++i) {
        const int t = i == 0 ? t_first : queued_tile(i, ok);
        if (t < 0) break;
        bool g2;
        int e, nt, ch;
        tile_of(t, g2, e, nt, ch);
        const int num_kb = g2 ? p.kb2 : p.kb1;
        const int b = i % C::kAccBufs;
        const uint32_t acc_phase = static_cast<uint32_t>(i / C::kAccBufs) & 1u;
        if (!mbar_wait(acce_bar(b), acc_phase ^ 1u, p.err, kDevTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * C::kAccStride + issuer * C::kAccCols;
        const uint32_t ashift = static_cast<uint32_t>((act_sf_row<true>(static_cast<int64_t>(ch) * C::kActRows) & 127) >> 5);
        const uint32_t t_sfa = tmem_base + C::kSfActCol + issuer * C::kSfCols;
        const uint32_t t_sfw = tmem_base + C::kSfWgtCol + issuer * C::kSfCols;
        const uint32_t idesc0 = idesc_mxf8f6f4(5, 0, C::kMmaM, C::kActRows, 0, 0);
        const uint32_t sf_a_t = t_sfw, sf_b_t = t_sfa + ashift;
        for (int kb0 = 0; kb0 < num_kb; kb0 += C::kSubs) {
          if (!mbar_wait(full_bar(stage), phase, p.err, kDevTimeoutMma)) { ok = false; break; }
          tc_fence_after();
          const int nsub = min(C::kSubs, num_kb - kb0);
          const uint32_t sb0 = smem_base + stage * C::kStageBytes;
          const uint64_t dw0 = desc_kmajor_sw128(sb0);
          const uint64_t da0 = desc_kmajor_sw128(sb0 + C::kWgtTileBytes);
          const uint64_t dsa0 = desc_sf_block(sb0 + C::kWgtTileBytes + C::kActTileBytes);
          const uint64_t dsw0 = dsa0 + (C::kSfActBytes >> 4);
#pragma unroll
          for (int j = 0; j < C::kSubs; ++j) {
            if (j >= nsub) break;
            if (j % C::kIssuers != issuer) continue;
            const uint64_t joff = (static_cast<uint64_t>(j) * C::kSubBytes) >> 4;
            tc_cp_32x128b_warpx4(t_sfa, dsa0 + joff);
            tc_cp_32x128b_warpx4(t_sfw, dsw0 + joff);
            const uint64_t dA = dw0 + joff, dB = da0 + joff;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint32_t idesc = idesc0 | (static_cast<uint32_t>(k) << 4) | (static_cast<uint32_t>(k) << 29);
              const uint32_t acc = (kb0 != 0 || j >= C::kIssuers || k != 0) ? 1u : 0u;
              mma_mxf8f6f4(d_tmem, dA + 2u * k, dB + 2u * k, idesc, sf_a_t, sf_b_t, acc);
            }
          }
          tc_commit(empty_bar(stage));
          if (++stage == C::kStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        tc_commit(accf_bar(b));
      }
      tc_commit(drain_bar);
      (void)mbar_wait(drain_bar, 0u, p.err, kDevTimeoutDrain);
    }
  } else {
    // ================================================================ epilogue
    GemmParams pg1 = pg1_in, pg2 = pg2_in;
    pg1.out_sf_offsets = S.sfb;               // shared-memory copies of the routed layout
    if constexpr (EP) pg2.token_idx32 = S.tok;   // received rows: GEMM2 stores into their sources
    else pg2.token_idx = S.tok;
    pg2.row_weights = S.w;
    const int q = warp & 3;
    bool ok = true;
    bool out_ready = false;
    for (int i = 0;; ++i) {
      // one thread reads the queue and the four warps take the same decision (the named
      // barriers of the epilogue must stay matched even when a wait gives up)
      int t = t_first;
      if (i > 0) {
        if (tid == 64) {
          bool okq = true;
          const int v = queued_tile(i, okq);
          *reinterpret_cast<volatile int*>(&s_epi_tile) = okq ? v : -2;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        t = *reinterpret_cast<volatile int*>(&s_epi_tile);
        if (t == -2) ok = false;
      }
      if (t < 0) break;
      bool g2;
      int e, nt, ch;
      tile_of(t, g2, e, nt, ch);
      const int b = i % C::kAccBufs;
      const uint32_t acc_phase = static_cast<uint32_t>(i / C::kAccBufs) & 1u;
      if (ok) ok = mbar_wait(accf_bar(b), acc_phase, p.err, kDevTimeoutEpilogue);
      if (ok && g2 && !out_ready) {           // every CTA's zeroing of `out` is visible
        if (lane == 0) ok = spin_wait_geq(p.sync + 0, G, p.err, kDlTimeoutGrid);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        out_ready = true;
      }
      if (!ok) {                               // keep the named barriers matched
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (!g2) asm volatile("bar.sync 1, 128;" ::: "memory");
        continue;
      }
      tc_fence_after();
      const uint32_t t_acc = tmem_base + (static_cast<uint32_t>(32 * q) << 16) + b * C::kAccStride;
      const bool has_b = (g2 ? p.kb2 : p.kb1) > 1;
      if (!g2) {
        // GEMM1 stages 4 KB per buffer, GEMM2 8 KB: tile i uses buffer i % 2, so GEMM1's
        // odd buffer moves to the 8 KB mark and never overlaps the neighbouring GEMM2 tile's
        float* const epi_g1 = epi_f + ((i & 1) ? 1024 : 0);
        swap_epilogue_tile<true, kEpiGemm1>(pg1, t_acc, acce_bar(b), e, nt, ch, S.cnt[e], S.off[e], i, epi_g1, has_b,
                                            q, lane);
        // publish this tile's intermediate rows to the GEMM2 tiles of other CTAs
        fence_proxy_async_global();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (tid == 64) {
          __threadfence();
          atomicAdd(p.sync + 2 + e, 1);
        }
      } else {
        swap_epilogue_tile<true, kEpiGemm2>(pg2, t_acc, acce_bar(b), e, nt, ch, S.cnt[e], S.off[e], i, epi_f, has_b,
                                            q, lane);
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
  if constexpr (EP) {
    // ================================================================ return + combine
    // every GEMM2 store of this CTA is behind the barrier above: the last CTA raises this
    // rank's return flag on every peer; then every CTA waits for all owners' flags and sums
    // its tokens' returned rows
    if (tid < 32)
      p2p_last_cta_signal(reinterpret_cast<int32_t*>(p.ep_local) + kP2pCounterReturn, p.ep_peer_bases, p.ep_world,
                          p.ep_world + p.ep_rank, p.ep_epoch);
    p2p_wait_flags(reinterpret_cast<const int32_t*>(p.ep_local), p.ep_world, p.ep_world, p.ep_epoch, p.err);
    const __nv_bfloat16* ret =
        reinterpret_cast<const __nv_bfloat16*>(p.ep_local + p2p_ret_offset(p.ep_world, 0, p.ep_cap, p.ep_rb, H));
    for (int t = cta; t < T; t += G) {
      int order[kMaxTopK];
      for (int j = 0; j < K; ++j) order[j] = j;
      for (int a = 1; a < K; ++a)             // insertion sort by expert id
        for (int b = a; b > 0 && S.ridx[t * K + order[b]] < S.ridx[t * K + order[b - 1]]; --b) {
          const int tmp = order[b]; order[b] = order[b - 1]; order[b - 1] = tmp;
        }
      for (int h2 = tid; h2 < H / 2; h2 += nthr) {
        float a0 = 0.0f, a1 = 0.0f;
        for (int j = 0; j < K; ++j) {
          const int pr = S.dslot[t * K + order[j]];
          if (pr < 0) continue;
          const __nv_bfloat162 v = __ldcg(reinterpret_cast<const __nv_bfloat162*>(ret + static_cast<int64_t>(pr) * H) + h2);
          a0 += __bfloat162float(v.x);
          a1 += __bfloat162float(v.y);
        }
        reinterpret_cast<__nv_bfloat162*>(p.out + static_cast<int64_t>(t) * H)[h2] = __floats2bfloat162_rn(a0, a1);
      }
    }
  }
}

}  // namespace gptoss
