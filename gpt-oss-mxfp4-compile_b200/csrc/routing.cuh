// Routing kernels of the MoE expert path.
//
//  router_topk_kernel   logits = x W^T + b (bf16 out, fp32 accumulate), top-k, softmax
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
// Router: each CTA owns TB tokens; their rows are staged in shared memory. Warp w
// handles experts w, w + nwarps, ...; lane l accumulates the 8-element slices
// l, l + 32, ... of the dot product in a fixed order (deterministic), with the weight
// slices of a chunk loaded before any arithmetic so their latencies overlap, then a
// fixed-order warp tree.
constexpr int kRouterVecChunk = 12;   // 8-element slices per lane per pass (H <= 3072 in one pass)

template <int TB>
__global__ void __launch_bounds__(TB == 1 ? 1024 : 512) router_topk_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
    const __nv_bfloat16* __restrict__ bias, int T, int H, int E, int K,
    int64_t* __restrict__ out_idx, __nv_bfloat16* __restrict__ out_scores,
    float* __restrict__ out_weights_f32, __nv_bfloat16* __restrict__ out_logits,
    __nv_bfloat16* __restrict__ zero_rows, int64_t zero_row_elems) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem_raw);      // [TB][H]
  float* logits = reinterpret_cast<float*>(smem_raw + sizeof(__nv_bfloat16) * TB * H);  // [TB][E]
  pdl_trigger();
  pdl_wait();

  const int t0 = blockIdx.x * TB;
  const int ntok = min(TB, T - t0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;

  const int vec_per_row = H >> 3;     // H % 8 == 0 (host check)
  for (int i = threadIdx.x; i < ntok * vec_per_row; i += blockDim.x) {
    const int t = i / vec_per_row, v = i - t * vec_per_row;
    reinterpret_cast<uint4*>(xs + t * H)[v] =
        reinterpret_cast<const uint4*>(x + static_cast<int64_t>(t0 + t) * H)[v];
  }
  if (zero_rows != nullptr) {          // the combine adds into these rows
    const int64_t vz = zero_row_elems >> 3;
    const uint4 z = make_uint4(0, 0, 0, 0);
    for (int64_t i = threadIdx.x; i < ntok * vz; i += blockDim.x)
      reinterpret_cast<uint4*>(zero_rows + static_cast<int64_t>(t0) * zero_row_elems)[i] = z;
  }
  __syncthreads();

  for (int e = warp; e < E; e += nwarps) {
    float acc[TB];
#pragma unroll
    for (int t = 0; t < TB; ++t) acc[t] = 0.0f;
    const uint4* wr = reinterpret_cast<const uint4*>(w + static_cast<int64_t>(e) * H);
    for (int v0 = 0; v0 < vec_per_row; v0 += 32 * kRouterVecChunk) {
      uint4 wv[kRouterVecChunk];
#pragma unroll
      for (int i = 0; i < kRouterVecChunk; ++i) {
        const int v = v0 + lane + 32 * i;
        wv[i] = v < vec_per_row ? __ldg(wr + v) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int i = 0; i < kRouterVecChunk; ++i) {
        const int v = v0 + lane + 32 * i;
        if (v < vec_per_row) {
          const uint32_t wq[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
#pragma unroll
          for (int t = 0; t < TB; ++t) {
            if (t < ntok) {
              const uint4 xv = reinterpret_cast<const uint4*>(xs + t * H)[v];
              const uint32_t xq[4] = {xv.x, xv.y, xv.z, xv.w};
              float a = acc[t];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                a = fmaf(bf16_bits_lo(xq[j]), bf16_bits_lo(wq[j]), a);
                a = fmaf(bf16_bits_hi(xq[j]), bf16_bits_hi(wq[j]), a);
              }
              acc[t] = a;
            }
          }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < TB; ++t) {
      float a = acc[t];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      if (lane == 0 && t < ntok) {
        // F.linear in bf16: fp32 accumulate, add the bias, round once to bf16.
        logits[t * E + e] = bf16_round(a + __bfloat162float(bias[e]));
      }
    }
  }
  __syncthreads();

  // Top-k (ties -> lower expert index first) and softmax over the selected logits; one
  // warp per token, each lane holding experts lane, lane + 32, ...
  for (int t = warp; t < ntok; t += nwarps) {
    const float* lg = logits + t * E;
    float lv[kMaxExperts / 32];
#pragma unroll
    for (int i = 0; i < kMaxExperts / 32; ++i) {
      const int e = lane + 32 * i;
      lv[i] = e < E ? lg[e] : -INFINITY;
    }
    int sel[kMaxTopK];
    float val[kMaxTopK];
    for (int j = 0; j < K; ++j) {
      // lane-local best (NaN counts as largest, like torch.topk), then a warp argmax
      float bv = -INFINITY;
      int be = 0x7fffffff;                 // no candidate yet
#pragma unroll
      for (int i = 0; i < kMaxExperts / 32; ++i) {
        const int e = lane + 32 * i;       // ascending, so a tie keeps the lower id
        const bool better = lv[i] > bv || (lv[i] != lv[i] && bv == bv);
        if (e < E && (be == 0x7fffffff || better)) { bv = lv[i]; be = e; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oe = __shfl_xor_sync(0xffffffffu, be, o);
        const bool better = (ov > bv) || (ov != ov && bv == bv) || ((ov == bv || (ov != ov && bv != bv)) && oe < be);
        if (better) { bv = ov; be = oe; }
      }
      sel[j] = be;
      val[j] = bv;
#pragma unroll
      for (int i = 0; i < kMaxExperts / 32; ++i)
        if (lane + 32 * i == be) lv[i] = -INFINITY;   // selected
    }
    if (lane == 0) {
      const float m = val[0];
      float ex[kMaxTopK], s = 0.0f;
      for (int j = 0; j < K; ++j) { ex[j] = expf(__fsub_rn(val[j], m)); s = __fadd_rn(s, ex[j]); }
      const float inv = __frcp_rn(s);
      const int64_t tg = t0 + t;
      for (int j = 0; j < K; ++j) {
        const __nv_bfloat16 pr = __float2bfloat16_rn(__fmul_rn(ex[j], inv));
        out_idx[tg * K + j] = sel[j];
        if (out_scores) out_scores[tg * K + j] = pr;
        if (out_weights_f32) out_weights_f32[tg * K + j] = __bfloat162float(pr);
      }
    }
    if (out_logits)
      for (int e = lane; e < E; e += 32) out_logits[(t0 + t) * static_cast<int64_t>(E) + e] = __float2bfloat16_rn(lg[e]);
  }
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
  // Optional blocked-scale bookkeeping for the fused path (nullptr to skip).
  int32_t* sf_offsets_a;           // [E] bytes, act layout with g4_a k-atoms
  int g4_a, groups_a;              // k-atoms / valid groups of the GEMM1 A operand
  uint8_t* sf_a;                   // zero the padding of this buffer
  int32_t* sf_offsets_b;           // [E] bytes, intermediate layout
  int g4_b, groups_b;
  uint8_t* sf_b;
  int spread;                      // activation scales in the SPREAD row layout
  int divisor;                     // bucket of assignment i = router_indices[i] / divisor (0, 1: expert)
  int32_t* sorted_src;             // optional [A]: assignment index i of each sorted entry
  int allow_empty;                 // index -1 marks an empty slot: skipped without an error
  int* err;                        // set if an index is outside [0, E)
};

__global__ void __launch_bounds__(1024) route_sort_kernel(RouteSortParams p) {
  __shared__ int hist[kMaxExperts];
  __shared__ int warp_cnt[32];
  __shared__ int s_base;
  pdl_trigger();
  pdl_wait();
  const int e = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t dv = p.divisor > 1 ? p.divisor : 1;
  for (int i = tid; i < p.E; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  // Pass 1: full histogram (every CTA builds it; A is small next to the GEMMs).
  for (int i = tid; i < p.A; i += blockDim.x) {
    const int64_t ex = p.router_indices[i] / dv;
    if (p.allow_empty && p.router_indices[i] == -1) continue;
    if (p.router_indices[i] < 0 || ex >= p.E) {
      if (p.err) atomicCAS(p.err, 0, 0x201);
      continue;
    }
    atomicAdd(&hist[ex], 1);
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
    for (int i = 0; i < per; ++i) {
      const int q = q0 + i;
      const int c = q < p.E ? hist[q] : 0;
      cl[i] = c;
      al[i] = (q < p.E && p.sf_offsets_a) ? act_sf_cosize(c, p.g4_a * 4, p.spread != 0) : 0;
      bl[i] = (q < p.E && p.sf_offsets_a) ? act_sf_cosize(c, p.g4_b * 4, p.spread != 0) : 0;
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
    for (int i = 0; i < per; ++i) {
      const int q = q0 + i;
      if (q < p.E) { s_off[q] = c_ex; s_sfa[q] = a_ex; s_sfb[q] = b_ex; }
      c_ex += cl[i]; a_ex += al[i]; b_ex += bl[i];
    }
  }
  __syncthreads();
  const int off = s_off[e];
  const int cnt = hist[e];
  if (tid == 0) {
    p.counts[e] = cnt;
    p.offsets[e] = off;
    s_base = 0;
    if (p.sf_offsets_a != nullptr) {
      p.sf_offsets_a[e] = static_cast<int32_t>(s_sfa[e]);
      p.sf_offsets_b[e] = static_cast<int32_t>(s_sfb[e]);
    }
  }
  // Zero this expert's blocked scale regions (16-byte stores); the quantisers that run
  // after this kernel overwrite the valid entries, so the padding ends up zero.
  if (p.sf_offsets_a != nullptr) {
    for (int pass = 0; pass < 2; ++pass) {
      uint8_t* buf = pass == 0 ? p.sf_a : p.sf_b;
      const int gp = (pass == 0 ? p.g4_a : p.g4_b) * 4;
      if (buf == nullptr) continue;
      uint4* dst = reinterpret_cast<uint4*>(buf + (pass == 0 ? s_sfa[e] : s_sfb[e]));   // multiple of 512
      const int64_t n16 = act_sf_cosize(cnt, gp, p.spread != 0) >> 4;
      const uint4 z = make_uint4(0, 0, 0, 0);
      for (int64_t i = tid; i < n16; i += blockDim.x) dst[i] = z;
    }
  }
  // Entries past the last valid one (only when some index was out of range) get the
  // sentinel -1, which every consumer of the sorted arrays skips.
  if (e == p.E - 1) {
    for (int i = off + cnt + tid; i < p.A; i += blockDim.x) {
      p.sorted_token[i] = -1;
      p.sorted_expert[i] = -1;
      p.sorted_weight[i] = 0.0f;
      if (p.sorted_src) p.sorted_src[i] = -1;
    }
  }
  __syncthreads();
  // Pass 2: stable compaction of this expert's assignments, 1024 at a time.
  for (int c0 = 0; c0 < p.A; c0 += blockDim.x) {
    const int i = c0 + tid;
    const bool mine = (i < p.A) && (p.router_indices[i] >= 0) && (p.router_indices[i] / dv == e);
    const unsigned bal = __ballot_sync(0xffffffffu, mine);
    if (lane == 0) warp_cnt[warp] = __popc(bal);
    __syncthreads();
    int before = 0;
    for (int q = 0; q < warp; ++q) before += warp_cnt[q];
    int chunk_total = 0;
    if (tid == 0)
      for (int q = 0; q < 32; ++q) chunk_total += warp_cnt[q];
    if (mine) {
      const int pos = off + s_base + before + __popc(bal & ((1u << lane) - 1u));
      p.sorted_token[pos] = i / p.K;
      p.sorted_expert[pos] = e;
      if (p.sorted_src) p.sorted_src[pos] = i;
      p.sorted_weight[pos] = p.routing_weights[i];
    }
    __syncthreads();
    if (tid == 0) s_base += chunk_total;
    __syncthreads();
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
  return ((static_cast<int64_t>(H) + H / 32 + 8 + 15) / 16) * 16;
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
  for (int g = threadIdx.x; g < H / 32; g += blockDim.x)
    act_sf[base + blocked_sf_offset(r_in, g, g4)] = src[H + g];
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

}  // namespace gptoss
