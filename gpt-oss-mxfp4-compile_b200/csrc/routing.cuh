// Routing kernels of the MoE expert path.
//
//  router_mma_kernel    logits = x W^T + b (bf16 out, fp32 accumulate), top-k, softmax
//                       over the k selected logits; HF GptOssTopKRouter semantics
//                       (F.linear -> torch.topk -> softmax(dtype=bf16)).
//  route_sort_kernel    one CTA per expert: histogram of all assignments, exclusive
//                       offsets, then a stable compaction of this expert's assignments
//                       in (token, k) order. Replaces the reference's atomic-slot
//                       counting sort (kernels/matmul_mxfp4_cutlass.cu:1010-1095); the
//                       result equals torch.argsort(stable=True), the order
//                       benchmark_optimizations.py:170-187 uses.
//  gather_quant_kernel  hidden[sorted_token] -> FP8 rows + UE8M0 scales written straight
//                       into the blocked layout the MMA reads
//                       (cutlass_experts.py:405-408 + matmul_mxfp4_cutlass.cu:881-908).
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include "ptx.cuh"
#include "numerics.cuh"

namespace gptoss {

constexpr int kMaxExperts = 256;
constexpr int kMaxTopK = 8;

// ----------------------------------------------------------------------------------
// Router. logits = x W^T + b is a [T, H] x [H, E] projection with E <= 256: it moves x
// once and does ~2*E flops per byte, so it runs on warp-level bf16 MMAs (m16n8k16,
// fp32 accumulate) fed by cp.async -- the tensor pipe is not its bound, HBM is.
// A CTA owns 16 tokens; its 4 warps split the experts (NT n-tiles of 8 each). When there
// are too few token blocks to cover the SMs the K dimension is split over the CTAs of a
// thread-block cluster and the fp32 partial logits are summed by the cluster's rank 0
// through distributed shared memory, in rank order (deterministic).
// Then: bias add and one bf16 rounding (F.linear), top-k with the lower expert id first
// on ties, softmax over the k selected logits (HF GptOssTopKRouter).
constexpr int kRtTok = 16;            // tokens per CTA
constexpr int kRtKc = 128;            // K elements per shared-memory chunk
constexpr int kRtLd = kRtKc + 8;      // padded row: conflict-free 4-byte fragment loads
// Ring depth: 4 chunks (three in flight, ~39 KB at E <= 32); 2 for E > 64 so the ring
// of a 256-expert W slice still fits in shared memory.
__host__ __device__ constexpr int router_stages(int nt) { return nt <= 2 ? 4 : 2; }

// K-split ranks of a cluster: at most 8, and at most 8 / nt so the leader's buffer of
// the ranks' partial logits stays at 16 KB.
__host__ __device__ constexpr int router_max_split(int nt) { return 8 / nt; }

__host__ __device__ constexpr size_t router_smem_bytes(int nt) {
  // x ring, W ring, fp32 partial logits [max split][16][32*nt]
  return static_cast<size_t>(router_stages(nt)) * (kRtTok + 32 * nt) * kRtLd * 2 +
         sizeof(float) * router_max_split(nt) * kRtTok * 32 * nt;
}

// One token's top-k + softmax by one thread: an insertion pass over the bf16-rounded
// logits `lg` keeps the k largest in descending order, equal values by ascending expert
// id, NaN above every number (torch.topk's NaN order).
__device__ __forceinline__ void router_topk_token(const float* lg, int E, int K, int64_t tg,
                                                  int64_t* __restrict__ out_idx,
                                                  __nv_bfloat16* __restrict__ out_scores,
                                                  float* __restrict__ out_weights_f32) {
  float bv[kMaxTopK];
  int be[kMaxTopK];
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) { bv[j] = -INFINITY; be[j] = -1; }
  for (int e = 0; e < E; ++e) {
    float cv = lg[e];
    int ce = e;
#pragma unroll
    for (int j = 0; j < kMaxTopK; ++j) {
      if (j < K) {
        // larger, or NaN over a number, or equal (both NaN counts) with the lower id --
        // the last case only arises for an entry displaced further down the list
        const bool cnan = cv != cv, bnan = bv[j] != bv[j];
        const bool better = be[j] < 0 || cv > bv[j] || (cnan && !bnan) ||
                            ((cv == bv[j] || (cnan && bnan)) && ce < be[j]);
        if (better) {
          const float tv = bv[j]; bv[j] = cv; cv = tv;
          const int te = be[j]; be[j] = ce; ce = te;
        }
      }
    }
  }
  const float m = bv[0];
  float ex[kMaxTopK], s = 0.0f;
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j)
    if (j < K) { ex[j] = expf(__fsub_rn(bv[j], m)); s = __fadd_rn(s, ex[j]); }
  const float inv = __frcp_rn(s);
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) {
    if (j < K) {
      const __nv_bfloat16 pr = __float2bfloat16_rn(__fmul_rn(ex[j], inv));
      out_idx[tg * K + j] = be[j];
      if (out_scores) out_scores[tg * K + j] = pr;
      if (out_weights_f32) out_weights_f32[tg * K + j] = __bfloat162float(pr);
    }
  }
}

// Top-k + softmax of given bf16 logits [T, E] (router_topk_token, the second half of the
// router): 32 tokens per CTA, their rows staged in shared memory (padded to E + 1 floats).
// dynamic smem = 32 * (E + 1) * 4 bytes.
__global__ void __launch_bounds__(32) router_topk_logits_kernel(const __nv_bfloat16* __restrict__ logits, int T, int E,
                                                                int K, int64_t* __restrict__ out_idx,
                                                                __nv_bfloat16* __restrict__ out_scores,
                                                                float* __restrict__ out_weights_f32) {
  extern __shared__ float s_rows[];
  pdl_trigger();
  pdl_wait();
  const int t0 = blockIdx.x * 32;
  const int nt = min(32, T - t0);
  for (int i = threadIdx.x; i < nt * E; i += 32) {
    const int r = i / E, e = i - r * E;
    s_rows[r * (E + 1) + e] = __bfloat162float(logits[static_cast<int64_t>(t0 + r) * E + e]);
  }
  __syncwarp();
  if (static_cast<int>(threadIdx.x) < nt)
    router_topk_token(s_rows + threadIdx.x * (E + 1), E, K, t0 + threadIdx.x, out_idx, out_scores, out_weights_f32);
}

// grid = (ceil(T / 16), S); cluster = (1, S, 1) when S > 1; blockDim = 128.
template <int NT>
__global__ void __launch_bounds__(128) router_mma_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
    const __nv_bfloat16* __restrict__ bias, int T, int H, int E, int K, int chunks_per_cta,
    int64_t* __restrict__ out_idx, __nv_bfloat16* __restrict__ out_scores,
    float* __restrict__ out_weights_f32, __nv_bfloat16* __restrict__ out_logits,
    __nv_bfloat16* __restrict__ zero_rows, int64_t zero_row_elems) {
  constexpr int kEp = 32 * NT;                           // expert rows held (>= E)
  constexpr int kRtStages = router_stages(NT);
  extern __shared__ __align__(16) uint8_t router_smem[];
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(router_smem);                    // [stages][16][kRtLd]
  __nv_bfloat16* ws = xs + kRtStages * kRtTok * kRtLd;                               // [stages][kEp][kRtLd]
  float* part = reinterpret_cast<float*>(ws + kRtStages * kEp * kRtLd);              // [S][16][kEp]
  pdl_trigger();
  // A CTA may write into another CTA's shared memory only once that CTA runs: every
  // rank arrives here and waits before its remote stores.
  if (gridDim.y > 1) cluster_arrive_relaxed();
  pdl_wait();

  const int S = gridDim.y, split = blockIdx.y;
  const int t0 = blockIdx.x * kRtTok;
  const int ntok = min(kRtTok, T - t0);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int nchunks = (H + kRtKc - 1) / kRtKc;
  const int c_begin = split * chunks_per_cta;
  const int c_end = min(nchunks, c_begin + chunks_per_cta);

  if (zero_rows != nullptr) {          // the combine adds into these rows
    const int64_t vz = zero_row_elems >> 3;
    const uint4 z = make_uint4(0, 0, 0, 0);
    uint4* zr = reinterpret_cast<uint4*>(zero_rows + static_cast<int64_t>(t0) * zero_row_elems);
    for (int64_t i = static_cast<int64_t>(split) * blockDim.x + tid; i < ntok * vz; i += static_cast<int64_t>(S) * blockDim.x)
      zr[i] = z;
  }

  auto load_chunk = [&](int ck, int stage) {
    const int k0 = ck * kRtKc;
    constexpr int kVec = kRtKc / 8;     // 16-byte vectors per row chunk
#pragma unroll
    for (int i = 0; i < kRtTok * kVec / 128; ++i) {   // x: 16 rows
      const int idx = tid + 128 * i;
      const int r = idx / kVec, v = idx % kVec;
      const int k = k0 + 8 * v;
      const bool in = r < ntok && k < H;
      const __nv_bfloat16* src = in ? x + static_cast<int64_t>(t0 + r) * H + k : x;
      cp_async_16(smem_u32(xs + (stage * kRtTok + r) * kRtLd + 8 * v), src, in ? 16u : 0u);
    }
#pragma unroll
    for (int i = 0; i < kEp * kVec / 128; ++i) {   // W: kEp rows
      const int idx = tid + 128 * i;
      const int r = idx / kVec, v = idx % kVec;
      const int k = k0 + 8 * v;
      const bool in = r < E && k < H;
      const __nv_bfloat16* src = in ? w + static_cast<int64_t>(r) * H + k : w;
      cp_async_16(smem_u32(ws + (stage * kEp + r) * kRtLd + 8 * v), src, in ? 16u : 0u);
    }
  };

  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;

#pragma unroll
  for (int s = 0; s < kRtStages - 1; ++s) {
    if (c_begin + s < c_end) load_chunk(c_begin + s, s);
    cp_async_commit();
  }
  for (int ck = c_begin; ck < c_end; ++ck) {
    cp_async_wait<kRtStages - 2>();
    __syncthreads();
    const int nxt = ck + kRtStages - 1;
    if (nxt < c_end) load_chunk(nxt, (nxt - c_begin) % kRtStages);
    cp_async_commit();
    const int st = (ck - c_begin) % kRtStages;
    const __nv_bfloat16* xa = xs + st * kRtTok * kRtLd;
    const __nv_bfloat16* wb = ws + st * kEp * kRtLd;
    // Each 64-deep chunk accumulates from zero on the tensor pipe and is then added to
    // the running fp32 sums with round-to-nearest adds: the running sums never go
    // through the MMA's internal adder, whose alignment of small terms to a large
    // accumulator loses low bits.
    float cacc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) cacc[j][0] = cacc[j][1] = cacc[j][2] = cacc[j][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < kRtKc / 16; ++kk) {
      const int kb = kk * 16 + 2 * c;
      const uint32_t a0 = *reinterpret_cast<const uint32_t*>(xa + g * kRtLd + kb);
      const uint32_t a1 = *reinterpret_cast<const uint32_t*>(xa + (g + 8) * kRtLd + kb);
      const uint32_t a2 = *reinterpret_cast<const uint32_t*>(xa + g * kRtLd + kb + 8);
      const uint32_t a3 = *reinterpret_cast<const uint32_t*>(xa + (g + 8) * kRtLd + kb + 8);
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const __nv_bfloat16* wr = wb + ((warp * NT + j) * 8 + g) * kRtLd + kb;
        mma_bf16_16816(cacc[j], a0, a1, a2, a3, *reinterpret_cast<const uint32_t*>(wr),
                       *reinterpret_cast<const uint32_t*>(wr + 8));
      }
    }
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[j][q] = __fadd_rn(acc[j][q], cacc[j][q]);
  }
  cp_async_wait<0>();

  // fp32 partial logits of this CTA's K range -> slot [split] of rank 0's buffer (remote
  // stores into the leader's shared memory when the K dimension is split).
  float* slot = part + split * (kRtTok * kEp);
  if (S > 1) cluster_wait();
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int n = (warp * NT + j) * 8 + 2 * c;
    const int idx[4] = {g * kEp + n, g * kEp + n + 1, (g + 8) * kEp + n, (g + 8) * kEp + n + 1};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (S > 1) dsmem_st_f32(dsmem_map(smem_u32(slot + idx[q]), 0), acc[j][q]);
      else slot[idx[q]] = acc[j][q];
    }
  }
  if (S > 1) {
    cluster_sync();                    // the partials are in rank 0's shared memory
    if (cluster_ctarank() != 0) return;
  } else {
    __syncthreads();
  }
  // rank 0: sum the ranks' partials in rank order, add the bias, round once to bf16
  for (int i = tid; i < kRtTok * kEp; i += blockDim.x) {
    float a = part[i];
    for (int r = 1; r < S; ++r) a = __fadd_rn(a, part[r * (kRtTok * kEp) + i]);
    const int e = i % kEp;
    if (e < E) a = bf16_round(a + __bfloat162float(bias[e]));
    part[i] = a;                       // only this thread touches element i
  }
  __syncthreads();
  if (tid < ntok) router_topk_token(part + tid * kEp, E, K, t0 + tid, out_idx, out_scores, out_weights_f32);
  if (out_logits)
    for (int i = tid; i < ntok * E; i += blockDim.x)
      out_logits[static_cast<int64_t>(t0) * E + i] = __float2bfloat16_rn(part[(i / E) * kEp + i % E]);
}

// ----------------------------------------------------------------------------------
// Per-expert stable counting sort. blockDim = 1024, gridDim = E.
struct RouteSortParams {
  const int64_t* router_indices;   // [A] expert of assignment i = t*K + k
  const float* routing_weights;    // [A]
  int A, K, E;
  int64_t* sorted_token;           // [A]
  int64_t* sorted_expert;          // [A]
  float* sorted_weight;            // [A]
  int32_t* counts;                 // [E]
  int32_t* offsets;                // [E]
  // Optional blocked-scale bookkeeping for the fused path (nullptr to skip). The
  // padding rows of the scale blocks are left as they are: a padding row only feeds its
  // own accumulator row (or column) of the GEMMs, which no epilogue stores.
  int32_t* sf_offsets_a;           // [E] bytes, act layout with g4_a k-atoms
  int g4_a, groups_a;              // k-atoms / valid groups of the GEMM1 A operand
  uint8_t* sf_a;
  int32_t* sf_offsets_b;           // [E] bytes, intermediate layout
  int g4_b, groups_b;
  uint8_t* sf_b;
  int spread;                      // activation scales in the SPREAD row layout
  int divisor;                     // bucket of assignment i = router_indices[i] / divisor (0, 1: expert)
  int32_t* sorted_src;             // optional [A]: assignment index i of each sorted entry
  int allow_empty;                 // index -1 marks an empty slot: skipped without an error
  int* err;                        // set if an index is outside [0, E)
};

// Assignments whose buckets one pass keeps in shared memory (uint16 codes, 32 KB).
constexpr int kSortChunk = 16384;
constexpr uint16_t kBktEmpty = 0xFFFF, kBktBad = 0xFFFE;

__global__ void __launch_bounds__(1024) route_sort_kernel(RouteSortParams p) {
  __shared__ int hist[kMaxExperts];
  __shared__ int warp_tot[32];
  __shared__ int s_chunk_total;
  __shared__ uint16_t s_bkt[kSortChunk];
  pdl_trigger();
  pdl_wait();
  const int e = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nthr = static_cast<int>(blockDim.x);
  const int64_t dv = p.divisor > 1 ? p.divisor : 1;
  auto bucket = [&](int64_t v) -> uint16_t {
    if (v < 0) return (p.allow_empty && v == -1) ? kBktEmpty : kBktBad;
    const int64_t b = dv == 1 ? v : v / dv;
    return b < p.E ? static_cast<uint16_t>(b) : kBktBad;
  };
  for (int i = tid; i < p.E; i += nthr) hist[i] = 0;
  __syncthreads();
  // Pass 1 (coalesced, 8 loads in flight per thread): full histogram -- every CTA
  // builds it; A is small next to the GEMMs -- caching the first chunk's buckets.
  for (int i0 = tid; i0 < p.A; i0 += 8 * nthr) {
    int64_t v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = i0 + j * nthr;
      v[j] = i < p.A ? p.router_indices[i] : -1;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = i0 + j * nthr;
      if (i >= p.A) break;
      const uint16_t b = bucket(v[j]);
      if (i < kSortChunk) s_bkt[i] = b;
      if (b == kBktBad) {
        if (p.err) atomicCAS(p.err, 0, 0x201);
      } else if (b != kBktEmpty) {
        atomicAdd(&hist[b], 1);
      }
    }
  }
  __syncthreads();
  // Exclusive prefixes of the counts and of both scale-region sizes, once, by warp 0
  // (E <= 256: eight values per lane, then a warp scan).
  __shared__ int s_off[kMaxExperts];
  __shared__ int64_t s_sfa[kMaxExperts], s_sfb[kMaxExperts];
  if (warp == 0) {
    int c_run = 0;
    int64_t a_run = 0, b_run = 0;
    const int per = (p.E + 31) / 32;
    const int q0 = lane * per;
    int cl[8];
    int64_t al[8], bl[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int q = q0 + i;
      const bool v = i < per && q < p.E;
      const int c = v ? hist[q] : 0;
      cl[i] = c;
      al[i] = (v && p.sf_offsets_a) ? act_sf_cosize(c, p.g4_a * 4, p.spread != 0) : 0;
      bl[i] = (v && p.sf_offsets_a) ? act_sf_cosize(c, p.g4_b * 4, p.spread != 0) : 0;
      c_run += c; a_run += al[i]; b_run += bl[i];
    }
    int c_inc = c_run;
    int64_t a_inc = a_run, b_inc = b_run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int c2 = __shfl_up_sync(0xffffffffu, c_inc, o);
      const int64_t a2 = __shfl_up_sync(0xffffffffu, a_inc, o);
      const int64_t b2 = __shfl_up_sync(0xffffffffu, b_inc, o);
      if (lane >= o) { c_inc += c2; a_inc += a2; b_inc += b2; }
    }
    int c_ex = c_inc - c_run;
    int64_t a_ex = a_inc - a_run, b_ex = b_inc - b_run;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int q = q0 + i;
      if (i < per && q < p.E) { s_off[q] = c_ex; s_sfa[q] = a_ex; s_sfb[q] = b_ex; }
      c_ex += cl[i]; a_ex += al[i]; b_ex += bl[i];
    }
  }
  __syncthreads();
  const int off = s_off[e];
  const int cnt = hist[e];
  if (tid == 0) {
    p.counts[e] = cnt;
    p.offsets[e] = off;
    if (p.sf_offsets_a != nullptr) {
      p.sf_offsets_a[e] = static_cast<int32_t>(s_sfa[e]);
      p.sf_offsets_b[e] = static_cast<int32_t>(s_sfb[e]);
    }
  }
  // Entries past the last valid one (only when some index was out of range or an
  // empty slot) get the sentinel -1, which every consumer of the sorted arrays skips.
  if (e == p.E - 1) {
    for (int i = off + cnt + tid; i < p.A; i += nthr) {
      p.sorted_token[i] = -1;
      p.sorted_expert[i] = -1;
      p.sorted_weight[i] = 0.0f;
      if (p.sorted_src) p.sorted_src[i] = -1;
    }
  }
  // Pass 2, chunk by chunk: each thread owns a contiguous segment of the chunk; an
  // exclusive scan of the per-thread counts of expert e gives stable positions.
  int run = off;
  for (int c0 = 0; c0 < p.A; c0 += kSortChunk) {
    const int len = min(kSortChunk, p.A - c0);
    if (c0 > 0) {
      __syncthreads();                 // the previous chunk is consumed
      for (int i0 = tid; i0 < len; i0 += 8 * nthr) {
        int64_t v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int i = i0 + j * nthr;
          v[j] = i < len ? p.router_indices[c0 + i] : -1;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int i = i0 + j * nthr;
          if (i < len) s_bkt[i] = bucket(v[j]);
        }
      }
      __syncthreads();
    }
    const int seg = (len + nthr - 1) / nthr;
    const int j0 = min(len, tid * seg), j1 = min(len, j0 + seg);
    int mine = 0;
    for (int j = j0; j < j1; ++j) mine += (s_bkt[j] == e);
    int incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const int nw = nthr >> 5;
      const int tot = lane < nw ? warp_tot[lane] : 0;
      int x = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += v;
      }
      if (lane < nw) warp_tot[lane] = x - tot;    // exclusive
      if (lane == 31) s_chunk_total = x;
    }
    __syncthreads();
    if (mine > 0) {
      int pos = run + warp_tot[warp] + incl - mine;
      for (int j = j0; j < j1; ++j) {
        if (s_bkt[j] != e) continue;
        const int i = c0 + j;
        p.sorted_token[pos] = i / p.K;
        p.sorted_expert[pos] = e;
        if (p.sorted_src) p.sorted_src[pos] = i;
        p.sorted_weight[pos] = p.routing_weights[i];
        ++pos;
      }
    }
    run += s_chunk_total;
  }
}

// ----------------------------------------------------------------------------------
// Gather + quantise. `tpr` threads share a row (one 32-element group each per pass);
// a block of 256 threads covers 256 / tpr rows. Writes FP8 codes into a compact [A, H]
// buffer and the UE8M0 scales into the blocked layout at sf_offsets[expert] (row index =
// position inside the expert's group). When sorted_token is null the rows are taken in
// order (plain quantiser) and scales go row-major into sf_rowmajor.
template <typename InT>
__global__ void __launch_bounds__(256) gather_quant_kernel(
    const InT* __restrict__ src, int64_t rows, int H, int tpr, const int64_t* __restrict__ sorted_token,
    const int64_t* __restrict__ sorted_expert, const int32_t* __restrict__ offsets,
    const int32_t* __restrict__ sf_offsets, int g4, int spread, uint8_t* __restrict__ out_codes,
    uint8_t* __restrict__ sf_blocked, uint8_t* __restrict__ sf_rowmajor) {
  pdl_trigger();
  pdl_wait();
  const int rows_per_block = blockDim.x / tpr;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * rows_per_block + threadIdx.x / tpr;
  if (row >= rows) return;
  const int sub = threadIdx.x % tpr;
  const int G = H >> 5;
  int64_t src_row = row;
  int64_t sf_base = 0, r_in = 0;
  if (sorted_token != nullptr) {
    src_row = sorted_token[row];
    if (src_row < 0) return;   // sentinel of an out-of-range router index
    const int ex = static_cast<int>(sorted_expert[row]);
    r_in = row - offsets[ex];
    if (spread) r_in = act_sf_row<true>(r_in);
    sf_base = sf_offsets[ex];
  }
  const InT* xr = src + src_row * H;
  uint8_t* orow = out_codes + row * H;
  for (int g = sub; g < G; g += tpr) {
    float v[32];
    if constexpr (sizeof(InT) == 2) {
      const uint4* pp = reinterpret_cast<const uint4*>(xr + g * 32);
      uint4 u[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) u[q] = __ldg(pp + q);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t w4[4] = {u[q].x, u[q].y, u[q].z, u[q].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          v[q * 8 + 2 * j] = bf16_bits_lo(w4[j]);
          v[q * 8 + 2 * j + 1] = bf16_bits_hi(w4[j]);
        }
      }
    } else {
      const float4* pp = reinterpret_cast<const float4*>(xr + g * 32);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 f = __ldg(pp + q);
        v[4 * q] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
      }
    }
    uint32_t codes[8];
    const uint8_t sc = quantize_group32(v, codes);
    uint4* o = reinterpret_cast<uint4*>(orow + g * 32);
    o[0] = make_uint4(codes[0], codes[1], codes[2], codes[3]);
    o[1] = make_uint4(codes[4], codes[5], codes[6], codes[7]);
    if (sorted_token != nullptr) sf_blocked[sf_base + blocked_sf_offset(r_in, g, g4)] = sc;
    else sf_rowmajor[row * G + g] = sc;
  }
}

// |x| max of a packed bf16 pair word into a running packed maximum; NaN propagates like
// torch.max (abs and max are exact in bf16, so the group maximum equals the fp32 one).
__device__ __forceinline__ uint32_t bf16x2_absmax(uint32_t m, uint32_t w) {
  uint32_t a, r;
  asm("abs.bf16x2 %0, %1;" : "=r"(a) : "r"(w));
  asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(m), "r"(a));
  return r;
}

// One bf16 row of H elements quantised by one warp, 1024 elements (32 groups of 32) per
// pass. Lane l loads 16 bytes at 256q + 8l for q = 0..3 (512-byte coalesced warp loads);
// the four lanes sharing a group combine their maxima with shuffles; lane g then
// computes the UE8M0 scale of group g of the pass, so the division and reciprocal run
// once per 32 groups; the scales go back to the lanes by shuffle, and lane 4a writes
// k-atom a's four scale bytes as one 32-bit word at blocked row r_in (the blocked layout
// keeps them contiguous; bytes of groups past H/32 are the zero padding).
__device__ __forceinline__ void quantize_row_warp(const __nv_bfloat16* __restrict__ xr, int H,
                                                  uint8_t* __restrict__ orow, uint8_t* __restrict__ sf_base,
                                                  int64_t r_in, int g4, int lane) {
  for (int base = 0; base < H; base += 1024) {
    uint4 u[4];
    float am[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int e0 = base + 256 * q + 8 * lane;
      u[q] = e0 < H ? __ldg(reinterpret_cast<const uint4*>(xr + e0)) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t m = bf16x2_absmax(0u, u[q].x);
      m = bf16x2_absmax(m, u[q].y);
      m = bf16x2_absmax(m, u[q].z);
      m = bf16x2_absmax(m, u[q].w);
      m = bf16x2_absmax(m, m >> 16);        // low half now holds the maximum of all 8
      float a = bf16_bits_lo(m);
#pragma unroll
      for (int o = 1; o <= 2; o <<= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, a, o);
        a = (ob > a || ob != ob) ? ob : a;
      }
      am[q] = a;                            // group 8q + lane/4 of this pass
    }
    // lane g <- maximum of group g = 8q + j (q = g / 8, j = g % 8), held by lane 4j
    float mine = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float v = __shfl_sync(0xffffffffu, am[q], 4 * (lane & 7));
      if ((lane >> 3) == q) mine = v;
    }
    const uint32_t rb = ue8m0_rounded_bits(mine);
    const float inv_mine = inv_scale(scale_from_bits(rb));
    const uint32_t sc = (rb >> 23) & 0xFFu;  // zero for groups past H/32 (their max is 0)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float inv = __shfl_sync(0xffffffffu, inv_mine, 8 * q + (lane >> 2));
      const int e0 = base + 256 * q + 8 * lane;
      if (e0 < H) {
        const uint32_t w4[4] = {u[q].x, u[q].y, u[q].z, u[q].w};
        uint32_t c[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float a = clamp_fp8(__fmul_rn(bf16_bits_lo(w4[2 * j]), inv));
          const float b = clamp_fp8(__fmul_rn(bf16_bits_hi(w4[2 * j]), inv));
          const float cc = clamp_fp8(__fmul_rn(bf16_bits_lo(w4[2 * j + 1]), inv));
          const float d = clamp_fp8(__fmul_rn(bf16_bits_hi(w4[2 * j + 1]), inv));
          c[j] = static_cast<uint32_t>(cvt_e4m3x2(a, b)) | (static_cast<uint32_t>(cvt_e4m3x2(cc, d)) << 16);
        }
        *reinterpret_cast<uint2*>(orow + e0) = make_uint2(c[0], c[1]);
      }
    }
    const uint32_t s1 = __shfl_down_sync(0xffffffffu, sc, 1);
    const uint32_t s2 = __shfl_down_sync(0xffffffffu, sc, 2);
    const uint32_t s3 = __shfl_down_sync(0xffffffffu, sc, 3);
    const int g0 = (base >> 5) + lane;      // first group of atom lane/4 when lane % 4 == 0
    if ((lane & 3) == 0 && 32 * g0 < H)
      *reinterpret_cast<uint32_t*>(sf_base + blocked_sf_offset(r_in, g0, g4)) =
          sc | (s1 << 8) | (s2 << 16) | (s3 << 24);
  }
}

// Fused-pipeline gather + quantise (bf16 input): one warp per expert-sorted row.
__global__ void __launch_bounds__(256) gather_quant_rows_kernel(
    const __nv_bfloat16* __restrict__ src, int64_t rows, int H, const int64_t* __restrict__ sorted_token,
    const int64_t* __restrict__ sorted_expert, const int32_t* __restrict__ offsets,
    const int32_t* __restrict__ sf_offsets, int g4, int spread, uint8_t* __restrict__ out_codes,
    uint8_t* __restrict__ sf_blocked) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;                  // warp-uniform
  const int64_t src_row = sorted_token[row];
  if (src_row < 0) return;                  // sentinel of an out-of-range router index
  const int ex = static_cast<int>(sorted_expert[row]);
  int64_t r_in = row - offsets[ex];
  if (spread) r_in = act_sf_row<true>(r_in);
  quantize_row_warp(src + src_row * H, H, out_codes + row * H, sf_blocked + sf_offsets[ex], r_in, g4, lane);
}

// Threads per row for gather_quant_kernel: a multiple of 32 covering the row's groups,
// at most 128.
__host__ __forceinline__ int quant_threads_per_row(int H) {
  const int G = H / 32;
  const int t = ((G + 31) / 32) * 32;
  return t > 128 ? 128 : t;
}

// ----------------------------------------------------------------------------------
// Row-major [rows, G] scales -> one blocked buffer (zero padded), grid-stride over the
// padded domain. Restates convert_scales_w4a8_impl (matmul_mxfp4_cutlass.cu:666-749).
__global__ void convert_scales_kernel(const uint8_t* __restrict__ in, int64_t rows, int G, int g4,
                                      uint8_t* __restrict__ out) {
  const int gp = g4 * 4;
  const int64_t total = ((rows + 127) & ~int64_t(127)) * gp;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / gp;
    const int g = static_cast<int>(i - r * gp);
    out[blocked_sf_offset(r, g, g4)] = (r < rows && g < G) ? in[r * G + g] : 0;
  }
}

// Per-expert blocked conversion (batch_convert_a_scales_for_w4a8_gpu,
// matmul_mxfp4_cutlass.cu:881-1004) with the per-expert byte offsets computed on the
// device. grid = E, block = 256.
__global__ void batch_convert_scales_kernel(const uint8_t* __restrict__ in,
                                            const int32_t* __restrict__ counts,
                                            const int32_t* __restrict__ offsets, int E, int G,
                                            int g4, uint8_t* __restrict__ out,
                                            int32_t* __restrict__ sf_offsets) {
  const int e = blockIdx.x;
  const int gp = g4 * 4;
  int64_t base = 0;
  for (int q = 0; q < e; ++q) base += blocked_sf_cosize(counts[q], gp);
  if (threadIdx.x == 0) sf_offsets[e] = static_cast<int32_t>(base);
  const int m = counts[e];
  const int64_t total = static_cast<int64_t>((m + 127) & ~127) * gp;
  const int64_t in_base = static_cast<int64_t>(offsets[e]) * G;
  for (int64_t i = threadIdx.x; i < total; i += blockDim.x) {
    const int64_t r = i / gp;
    const int g = static_cast<int>(i - r * gp);
    out[base + blocked_sf_offset(r, g, g4)] = (r < m && g < G) ? in[in_base + r * G + g] : 0;
  }
}

// ----------------------------------------------------------------------------------
// Standalone SwiGLU (cutlass_experts.py:258-276) for [rows, 2n] interleaved gate/up.
// bf16 inputs follow torch's per-op rounding (every elementwise op of the reference
// rounds its bf16 result); fp32 inputs use swiglu_pair.
template <typename T>
__global__ void swiglu_kernel(const T* __restrict__ in, int64_t rows, int64_t n, T* __restrict__ out,
                              float alpha, float limit) {
  const int64_t total = rows * n;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / n, c = i - r * n;
    const T* row = in + r * 2 * n;
    if constexpr (sizeof(T) == 4) {
      out[i] = swiglu_pair(row[2 * c], row[2 * c + 1], alpha, limit);
    } else {
      float g = __bfloat162float(row[2 * c]), u = __bfloat162float(row[2 * c + 1]);
      g = g > limit ? limit : g;
      u = u < -limit ? -limit : (u > limit ? limit : u);
      const float ga = bf16_round(__fmul_rn(g, alpha));
      const float sg = bf16_round(__frcp_rn(__fadd_rn(1.0f, expf(-ga))));
      const float gs = bf16_round(__fmul_rn(g, sg));
      const float u1 = bf16_round(__fadd_rn(u, 1.0f));
      out[i] = __float2bfloat16_rn(__fmul_rn(gs, u1));
    }
  }
}

// ----------------------------------------------------------------------------------
// Expert parallelism. A dispatched row carries everything the receiving rank needs:
//   [FP8 codes H | UE8M0 scales H/32 | pad | local expert int32 | routing weight f32]
// padded to a multiple of 16 bytes (H = 2880: 2992 bytes). Rows are quantised before they
// are sent (quantisation is per row, so the codes equal the single-GPU ones).
__host__ __device__ __forceinline__ int64_t ep_row_bytes(int H) {
  // the scale bytes are padded to whole k-atoms (4 groups) so a receiver can read them as
  // 32-bit words
  return ((static_cast<int64_t>(H) + (H / 32 + 3) / 4 * 4 + 8 + 15) / 16) * 16;
}

// Pack: entry p of the destination-sorted order (route_sort_kernel with divisor =
// experts per rank) -> quantised send row; pos_of[i] remembers which row assignment i
// went to so the combine can find its returned row.
//   cap == 0: compact rows, row p (per-destination splits are variable);
//   cap > 0:  W fixed segments of cap rows, entry j of destination q in row q*cap + j;
//             unused rows carry local expert -1 (an empty slot the receiver skips), so the
//             exchange has equal splits and needs no host-visible counts.
__global__ void __launch_bounds__(256) ep_pack_kernel(
    const __nv_bfloat16* __restrict__ hidden, int H, int K, int experts_per_rank, int64_t A,
    const int64_t* __restrict__ router_indices, const float* __restrict__ routing_weights,
    const int32_t* __restrict__ sorted_src, int64_t cap, int world, const int32_t* __restrict__ dest_counts,
    const int32_t* __restrict__ dest_offsets, int tpr, uint8_t* __restrict__ send_rows,
    int32_t* __restrict__ pos_of) {
  pdl_trigger();
  pdl_wait();
  const int rows_per_block = blockDim.x / tpr;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * rows_per_block + threadIdx.x / tpr;
  const int64_t rows_total = cap > 0 ? cap * world : A;
  if (r >= rows_total) return;
  const int sub = threadIdx.x % tpr;
  const int G = H >> 5;
  const int64_t rb = ep_row_bytes(H);
  uint8_t* row = send_rows + r * rb;
  int64_t p = r;
  if (cap > 0) {
    const int q = static_cast<int>(r / cap);
    const int64_t j = r - static_cast<int64_t>(q) * cap;
    if (j >= dest_counts[q]) {
      if (sub == 0) {
        int32_t* meta = reinterpret_cast<int32_t*>(row + rb - 8);
        meta[0] = -1;
        meta[1] = 0;
      }
      return;
    }
    p = dest_offsets[q] + j;
  }
  const int i = sorted_src[p];
  if (i < 0) return;   // sentinel of an out-of-range router index
  const int64_t t = i / K;
  const __nv_bfloat16* xr = hidden + t * H;
  for (int g = sub; g < G; g += tpr) {
    const uint4* pp = reinterpret_cast<const uint4*>(xr + g * 32);
    uint4 u[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) u[q] = __ldg(pp + q);
    float v[32];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t w4[4] = {u[q].x, u[q].y, u[q].z, u[q].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[q * 8 + 2 * j] = bf16_bits_lo(w4[j]);
        v[q * 8 + 2 * j + 1] = bf16_bits_hi(w4[j]);
      }
    }
    uint32_t codes[8];
    const uint8_t sc = quantize_group32(v, codes);
    uint4* o = reinterpret_cast<uint4*>(row + g * 32);
    o[0] = make_uint4(codes[0], codes[1], codes[2], codes[3]);
    o[1] = make_uint4(codes[4], codes[5], codes[6], codes[7]);
    row[H + g] = sc;
  }
  if (sub == 0) {
    for (int64_t b = H + G; b < rb - 8; ++b) row[b] = 0;   // padding travels as zeros
    int32_t* meta = reinterpret_cast<int32_t*>(row + rb - 8);
    meta[0] = static_cast<int32_t>(router_indices[i] % experts_per_rank);
    meta[1] = __float_as_int(routing_weights[i]);
    pos_of[i] = static_cast<int32_t>(r);
  }
}

// Receiving rank: row r's (local expert, weight) -> arrays route_sort_kernel reads.
__global__ void ep_unpack_meta_kernel(const uint8_t* __restrict__ recv_rows, int64_t R, int H,
                                      int64_t* __restrict__ expert, float* __restrict__ weight) {
  pdl_trigger();
  pdl_wait();
  const int64_t rb = ep_row_bytes(H);
  for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; r < R;
       r += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t* meta = reinterpret_cast<const int32_t*>(recv_rows + r * rb + rb - 8);
    expert[r] = meta[0];
    weight[r] = __int_as_float(meta[1]);
  }
}

// Expert-sorted position p <- received row sorted_token[p]: copy its codes into the
// GEMM's activation rows and scatter its scales into the blocked layout.
__global__ void __launch_bounds__(256) ep_gather_kernel(
    const uint8_t* __restrict__ recv_rows, int64_t R, int H, const int64_t* __restrict__ sorted_row,
    const int64_t* __restrict__ sorted_expert, const int32_t* __restrict__ offsets,
    const int32_t* __restrict__ sf_offsets, int g4, int spread, uint8_t* __restrict__ act_codes,
    uint8_t* __restrict__ act_sf) {
  pdl_trigger();
  pdl_wait();
  const int64_t p = blockIdx.x;
  if (p >= R) return;
  const int64_t rb = ep_row_bytes(H);
  if (sorted_row[p] < 0) return;   // sentinel of an out-of-range local expert id
  const uint8_t* src = recv_rows + sorted_row[p] * rb;
  const int ex = static_cast<int>(sorted_expert[p]);
  int64_t r_in = p - offsets[ex];
  if (spread) r_in = act_sf_row<true>(r_in);
  const int64_t base = sf_offsets[ex];
  for (int v = threadIdx.x; v < H / 16; v += blockDim.x)
    reinterpret_cast<uint4*>(act_codes + p * H)[v] = reinterpret_cast<const uint4*>(src)[v];
  for (int g = threadIdx.x; g < 4 * g4; g += blockDim.x)   // K padding groups: zero
    act_sf[base + blocked_sf_offset(r_in, g, g4)] = g < H / 32 ? src[H + g] : 0;
}

// Combine: out[t] = bf16 of the fp32 sum of the token's k returned rows, added in ascending
// expert order -- what the reference's scatter_add_ of expert-sorted bf16 rows into a zero
// bf16 tensor gives on the CPU (cutlass_experts.py:445-450; fp32 accumulation, one
// rounding).
__global__ void __launch_bounds__(256) ep_combine_kernel(const __nv_bfloat16* __restrict__ back_rows,
                                                         const int32_t* __restrict__ pos_of,
                                                         const int64_t* __restrict__ router_indices, int64_t T,
                                                         int K, int H, int64_t rows,
                                                         __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int64_t t = blockIdx.x;
  if (t >= T) return;
  int order[kMaxTopK];
  for (int j = 0; j < K; ++j) order[j] = j;
  for (int a = 1; a < K; ++a)                      // insertion sort by expert id
    for (int b = a; b > 0 && router_indices[t * K + order[b]] < router_indices[t * K + order[b - 1]]; --b) {
      const int tmp = order[b]; order[b] = order[b - 1]; order[b - 1] = tmp;
    }
  for (int h2 = threadIdx.x; h2 < H / 2; h2 += blockDim.x) {
    float a0 = 0.0f, a1 = 0.0f;
    for (int j = 0; j < K; ++j) {
      const int64_t pr = pos_of[t * K + order[j]];
      if (pr < 0 || pr >= rows) continue;   // assignment with an out-of-range expert id
      const __nv_bfloat162 v = reinterpret_cast<const __nv_bfloat162*>(back_rows + pr * H)[h2];
      a0 += __bfloat162float(v.x);
      a1 += __bfloat162float(v.y);
    }
    reinterpret_cast<__nv_bfloat162*>(out + t * H)[h2] = __floats2bfloat162_rn(a0, a1);
  }
}


// RMSNorm in front of a MoE block (GptOssRMSNorm / F.rms_norm: fp32 mean of squares,
// rsqrt(mean + eps), x * rsqrt * weight, one rounding to bf16), fused with the residual:
// one warp per token reads its row once for the sum of squares and once more (from L1/L2)
// to write the normalised row `xn` and, when `res` is set, a copy of the input into `res` --
// the rows GEMM2 then adds the expert outputs into, so the block's residual add needs no
// kernel of its own. x may alias res.
__global__ void __launch_bounds__(256) rmsnorm_residual_kernel(const __nv_bfloat16* x, const __nv_bfloat16* w,
                                                               float eps, int T, int H, __nv_bfloat16* xn,
                                                               __nv_bfloat16* res) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + t * H);
  const int nv = H / 8;
  float ss = 0.0f;
  for (int v = lane; v < nv; v += 32) {
    const uint4 u = xr[v];
    const uint32_t a[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float lo = bf16_bits_lo(a[h]), hi = bf16_bits_hi(a[h]);
      ss = fmaf(lo, lo, ss);
      ss = fmaf(hi, hi, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(H)), eps));
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* yr = reinterpret_cast<uint4*>(xn + t * H);
  uint4* cr = res != nullptr ? reinterpret_cast<uint4*>(res + t * H) : nullptr;
  for (int v = lane; v < nv; v += 32) {
    const uint4 u = xr[v], g = __ldg(wr + v);
    const uint32_t a[4] = {u.x, u.y, u.z, u.w}, b[4] = {g.x, g.y, g.z, g.w};
    uint32_t o[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const __nv_bfloat162 y = __floats2bfloat162_rn(__fmul_rn(__fmul_rn(bf16_bits_lo(a[h]), r), bf16_bits_lo(b[h])),
                                                     __fmul_rn(__fmul_rn(bf16_bits_hi(a[h]), r), bf16_bits_hi(b[h])));
      o[h] = *reinterpret_cast<const uint32_t*>(&y);
    }
    yr[v] = make_uint4(o[0], o[1], o[2], o[3]);
    if (cr != nullptr) cr[v] = u;
  }
}

}  // namespace gptoss
