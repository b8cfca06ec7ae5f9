// Decode-sized prologue in one launch: router + top-k + stable counting sort + gather /
// FP8 quantisation into the blocked scale layout, run by one thread-block cluster.
//
// At decode sizes (T <= 64 tokens) the three separate kernels (router_mma_kernel,
// route_sort_kernel, gather_quant_rows_kernel) are each a few microseconds of dependent
// memory latency plus a launch gap. Here a cluster of kDpCluster CTAs does all of it,
// exchanging intermediate results through distributed shared memory:
//   phase 1  every rank stages its 1/kDpCluster slice of K of x (and of W) in shared
//            memory with cp.async, quantises that slice of every token (FP8 codes +
//            UE8M0 scales, kept in shared memory) and computes bf16 MMA partial logits;
//   phase 2  rank r owns tokens r, r + kDpCluster, ...: sums their partial logits over the
//            ranks in rank order, adds the bias, rounds to bf16, takes the top-k by
//            counting, per (token, expert), the experts ranked ahead (torch.topk
//            order), applies the softmax, and sends the routing to every rank;
//   phase 3  every rank (redundantly): the stable counting sort of the T*k assignments
//            (same order as route_sort_kernel) with warp match_any ranks; rank 0 writes
//            the routed layout to global memory;
//   phase 4  every rank writes its K slice of every expert-sorted row (codes and scale
//            words) straight from shared memory.
// Two cluster barriers; no rank touches another's shared memory after the second.
// Semantics and outputs are those of router_mma_kernel + route_sort_kernel +
// gather_quant_rows_kernel. With `w == nullptr` the routing is an input (phases 1-2 are
// skipped and rank 0 reads ridx_in / rw_in).
//
// Expert-parallel dispatch mode (ep_world > 0) replaces the local layout with the
// peer-memory dispatch of ep_pack_p2p_kernel: phase 3 sorts the assignments by owning rank
// (stable, as route_sort_kernel with divisor = experts per rank), phase 4 stores each rank's
// K slice of every row straight into the owner's receive rows (segment ep_rank), rank 0
// adds the row metadata, the empty-slot markers, pos_of and send_counts, and after a third
// cluster barrier rank 0 raises dispatch flag[ep_rank] of every peer to the epoch.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include "ptx.cuh"
#include "numerics.cuh"
#include "routing.cuh"
#include "ep_p2p.cuh"

namespace gptoss {

constexpr int kDpCluster = 8;          // CTAs of the cluster (portable size)
constexpr int kDpThreads = 256;
constexpr int kDpMaxTokens = 64;
constexpr int kDpMaxAssign = 512;
constexpr size_t kDpMaxSmem = 200 * 1024;

struct DecodePrologueParams {
  const __nv_bfloat16* x;       // [T, H]
  const __nv_bfloat16* w;       // [E, H] router weight; nullptr: routing is given
  const __nv_bfloat16* bias;    // [E]
  const int64_t* ridx_in;       // [T, K] (w == nullptr)
  const float* rw_in;           // [T, K] (w == nullptr)
  int T, H, E, K;
  int slice_chunks;             // 64-element K chunks per rank
  int64_t* ridx_out;            // [T, K] (w != nullptr)
  __nv_bfloat16* scores_out;    // [T, K] or nullptr
  float* rw_out;                // [T, K] (w != nullptr)
  int64_t* sorted_token;
  int64_t* sorted_expert;
  float* sorted_weight;
  int32_t* counts;
  int32_t* offsets;
  int32_t* sf_offsets_a;
  int32_t* sf_offsets_b;
  uint8_t* act_codes;
  uint8_t* act_sf;
  uint8_t* inter_sf;
  int g4_a, g4_b, spread;
  __nv_bfloat16* zero_out;      // [T, H] zeroed for the GEMM2 combine, or nullptr
  int* err;
  // expert-parallel dispatch mode (ep_world > 0)
  int ep_world, ep_rank, ep_epr, ep_rb;
  int64_t ep_cap;
  const uint64_t* peer_bases;   // [ep_world] exchange buffers, this rank's own included
  int32_t* send_counts;         // [ep_world]
  int32_t* pos_of;              // [T, K] assignment -> row of the return layout (-1: none)
  int32_t epoch;
};

struct DpLayout {
  uint32_t xs, ws, part, lg, codes, sfs, slot_e, slot_v, sel, wts, run, cnt, off, sfa, sfb, srow, sexp, total;
  int ld, tp, ep, sl;
};

// slice_chunks: 64-element K chunks per rank (even, so a slice is whole 128-wide k-atoms).
__host__ __device__ inline DpLayout dp_layout(int T, int E, int K, int slice_chunks, bool router) {
  DpLayout L{};
  L.sl = slice_chunks * 64;
  L.ld = L.sl + 8;                            // padded bf16 row: conflict-free fragment loads
  L.tp = ((T + 15) / 16) * 16;
  L.ep = ((E + 7) / 8) * 8;
  const int A = T * K;
  uint32_t o = 0;
  auto take = [&](uint32_t bytes) { const uint32_t r = o; o = (o + bytes + 15u) & ~15u; return r; };
  L.xs = take(static_cast<uint32_t>(L.tp * L.ld * 2));
  L.ws = take(router ? static_cast<uint32_t>(L.ep * L.ld * 2) : 0u);
  L.part = take(router ? static_cast<uint32_t>(L.tp * L.ep * 4) : 0u);
  L.lg = take(router ? static_cast<uint32_t>(L.tp * L.ep * 4) : 0u);
  L.codes = take(static_cast<uint32_t>(T * L.sl));
  L.sfs = take(static_cast<uint32_t>(T * (L.sl / 32)));
  L.slot_e = take(router ? static_cast<uint32_t>(A * 4) : 0u);
  L.slot_v = take(router ? static_cast<uint32_t>(A * 4) : 0u);
  L.sel = take(static_cast<uint32_t>(A * 4));
  L.wts = take(static_cast<uint32_t>(A * 4));
  L.run = take(static_cast<uint32_t>(E * 4));
  L.cnt = take(static_cast<uint32_t>(E * 4));
  L.off = take(static_cast<uint32_t>(E * 4));
  L.sfa = take(static_cast<uint32_t>(E * 4));
  L.sfb = take(static_cast<uint32_t>(E * 4));
  L.srow = take(static_cast<uint32_t>(A * 4));
  L.sexp = take(static_cast<uint32_t>(A * 4));
  L.total = o;
  return L;
}

// True when expert e (value a) ranks ahead of expert f (value b) in torch.topk order:
// larger first, NaN above every number, equal values (NaN with NaN) by ascending id.
__device__ __forceinline__ bool topk_ahead(float a, int e, float b, int f) {
  const bool an = a != a, bn = b != b;
  return a > b || (an && !bn) || ((a == b || (an && bn)) && e < f);
}

// Expert-parallel phase 4: this rank's K slice of every row (codes, then the slice's
// UE8M0 bytes) into row j of peer q's receive rows, segment ep_rank; rank 0 writes the
// padding bytes, the (local expert, weight) metadata and the empty-slot markers. Then the
// cluster barrier orders every rank's peer stores (fenced at system scope) before rank 0
// raises flag[ep_rank] of every peer.
__device__ __forceinline__ void ep_dispatch_phase4(const DecodePrologueParams& p, uint32_t rank,
                                                   const uint8_t* codes, const uint8_t* sfs, const int* srow,
                                                   const int* sasg, const int* sel, const float* wts,
                                                   const int* cnt, const int* off, int sl, int slv, int gs,
                                                   int k0) {
  const int tid = threadIdx.x;
  const int H = p.H, W = p.ep_world, G = H >> 5;
  const int64_t rb = p.ep_rb, cap = p.ep_cap;
  const int total = off[W - 1] + cnt[W - 1];
  auto row_of = [&](int pos, int& q) -> uint8_t* {
    const int i = sasg[pos];
    q = sel[i] / p.ep_epr;
    const int64_t j = pos - off[q];
    return reinterpret_cast<uint8_t*>(p.peer_bases[q]) + p2p_recv_offset(p.ep_rank, cap, rb) + j * rb;
  };
  if (slv > 0) {
    const int v16 = slv / 16;
    for (int q2 = tid; q2 < total * v16; q2 += kDpThreads) {
      const int pos = q2 / v16, v = q2 - pos * v16;
      int q;
      uint8_t* row = row_of(pos, q);
      reinterpret_cast<uint4*>(row + k0)[v] = reinterpret_cast<const uint4*>(codes + srow[pos] * sl)[v];
    }
    const int gv = slv / 32;
    for (int q2 = tid; q2 < total * gv; q2 += kDpThreads) {
      const int pos = q2 / gv, gi = q2 - pos * gv;
      int q;
      uint8_t* row = row_of(pos, q);
      row[H + (k0 >> 5) + gi] = sfs[srow[pos] * gs + gi];
    }
  }
  if (rank == 0) {
    for (int pos = tid; pos < total; pos += kDpThreads) {
      int q;
      uint8_t* row = row_of(pos, q);
      const int i = sasg[pos];
      for (int64_t b = H + G; b < rb - 8; ++b) row[b] = 0;   // padding travels as zeros
      int32_t* meta = reinterpret_cast<int32_t*>(row + rb - 8);
      meta[0] = sel[i] - q * p.ep_epr;
      meta[1] = __float_as_int(wts[i]);
    }
    for (int64_t r = tid; r < cap * W; r += kDpThreads) {     // empty slots past each count
      const int q = static_cast<int>(r / cap);
      const int64_t j = r - static_cast<int64_t>(q) * cap;
      if (j >= cnt[q]) {
        int32_t* meta = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(p.peer_bases[q]) +
                                                   p2p_recv_offset(p.ep_rank, cap, rb) + j * rb + rb - 8);
        meta[0] = -1;
        meta[1] = 0;
      }
    }
  }
  __threadfence_system();
  cluster_sync();
  if (rank == 0 && tid < 32) p2p_raise_flags_warp(p.peer_bases, W, p.ep_rank, p.epoch);
}

// grid = kDpCluster CTAs forming one cluster; blockDim = kDpThreads.
__global__ void __launch_bounds__(kDpThreads, 1) decode_prologue_kernel(const DecodePrologueParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const bool router = p.w != nullptr;
  const DpLayout L = dp_layout(p.T, p.E, p.K, p.slice_chunks, router);
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem + L.xs);
  __nv_bfloat16* wsm = reinterpret_cast<__nv_bfloat16*>(smem + L.ws);
  float* part = reinterpret_cast<float*>(smem + L.part);
  float* lg = reinterpret_cast<float*>(smem + L.lg);
  uint8_t* codes = smem + L.codes;
  uint8_t* sfs = smem + L.sfs;
  int* slot_e = reinterpret_cast<int*>(smem + L.slot_e);
  float* slot_v = reinterpret_cast<float*>(smem + L.slot_v);
  int* sel = reinterpret_cast<int*>(smem + L.sel);
  float* wts = reinterpret_cast<float*>(smem + L.wts);
  int* run = reinterpret_cast<int*>(smem + L.run);
  int* cnt = reinterpret_cast<int*>(smem + L.cnt);
  int* off = reinterpret_cast<int*>(smem + L.off);
  int* sfa = reinterpret_cast<int*>(smem + L.sfa);
  int* sfb = reinterpret_cast<int*>(smem + L.sfb);
  int* srow = reinterpret_cast<int*>(smem + L.srow);
  int* sexp = reinterpret_cast<int*>(smem + L.sexp);
  pdl_trigger();
  pdl_wait();

  const uint32_t rank = cluster_ctarank();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int T = p.T, H = p.H, E = p.E, K = p.K, A = T * K;
  const int ld = L.ld, ep = L.ep, sl = L.sl;
  const int k0 = static_cast<int>(rank) * sl;            // this rank's K slice [k0, k0 + slv)
  const int slv = max(0, min(sl, H - k0));
  const int gs = sl / 32;                                 // groups per slice

  if (p.zero_out != nullptr) {                    // the GEMM2 combine adds into these rows
    const int64_t n16 = static_cast<int64_t>(T) * H / 8;
    uint4* z = reinterpret_cast<uint4*>(p.zero_out);
    for (int64_t i = static_cast<int64_t>(rank) * kDpThreads + tid; i < n16; i += kDpCluster * kDpThreads)
      z[i] = make_uint4(0, 0, 0, 0);
  }

  // ---- phase 1: stage the x slice (and the W slice)
  const int vec = sl / 8;
  for (int idx = tid; idx < L.tp * vec; idx += kDpThreads) {
    const int r = idx / vec, v = idx - r * vec;
    const int k = k0 + 8 * v;
    const bool in = r < T && k < H;
    cp_async_16(smem_u32(xs + r * ld + 8 * v), in ? p.x + static_cast<int64_t>(r) * H + k : p.x, in ? 16u : 0u);
  }
  cp_async_commit();
  if (router) {
    for (int idx = tid; idx < ep * vec; idx += kDpThreads) {
      const int r = idx / vec, v = idx - r * vec;
      const int k = k0 + 8 * v;
      const bool in = r < E && k < H;
      cp_async_16(smem_u32(wsm + r * ld + 8 * v), in ? p.w + static_cast<int64_t>(r) * H + k : p.w, in ? 16u : 0u);
    }
  }
  cp_async_commit();
  cp_async_wait<1>();                             // the x slice; W may still be landing
  __syncthreads();
  // (a) FP8 codes and UE8M0 scales of the slice for every token: one thread per group
  for (int q = tid; q < T * gs; q += kDpThreads) {
    const int t = q / gs, gi = q - t * gs;
    uint8_t sc = 0;
    if (32 * gi < slv) {
      const uint4* src = reinterpret_cast<const uint4*>(xs + t * ld + 32 * gi);
      float v[32];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 u = src[j];
        const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          v[8 * j + 2 * h] = bf16_bits_lo(w4[h]);
          v[8 * j + 2 * h + 1] = bf16_bits_hi(w4[h]);
        }
      }
      uint32_t cw[8];
      sc = quantize_group32(v, cw);
      uint4* dst = reinterpret_cast<uint4*>(codes + t * sl + 32 * gi);
      dst[0] = make_uint4(cw[0], cw[1], cw[2], cw[3]);
      dst[1] = make_uint4(cw[4], cw[5], cw[6], cw[7]);
    }
    sfs[t * gs + gi] = sc;                              // zero past H (padding groups)
  }
  // (b) partial logits over the slice
  cp_async_wait<0>();
  __syncthreads();
  if (router) {
    const int ntile = ep / 8;
    const int npairs = (L.tp / 16) * ntile;
    for (int pr = warp; pr < npairs; pr += kDpThreads / 32) {
      const int mi = pr / ntile, nj = pr - mi * ntile;
      const __nv_bfloat16* xa = xs + (16 * mi) * ld;
      const __nv_bfloat16* wb = wsm + (8 * nj + g) * ld;
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      for (int ch = 0; ch < p.slice_chunks; ++ch) {
        // 64-deep chunks accumulate from zero on the tensor pipe and are added with
        // round-to-nearest adds (the running sums never go through the MMA adder)
        float cacc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const int kb = ch * 64 + kk * 16 + 2 * c;
          const uint32_t a0 = *reinterpret_cast<const uint32_t*>(xa + g * ld + kb);
          const uint32_t a1 = *reinterpret_cast<const uint32_t*>(xa + (g + 8) * ld + kb);
          const uint32_t a2 = *reinterpret_cast<const uint32_t*>(xa + g * ld + kb + 8);
          const uint32_t a3 = *reinterpret_cast<const uint32_t*>(xa + (g + 8) * ld + kb + 8);
          mma_bf16_16816(cacc, a0, a1, a2, a3, *reinterpret_cast<const uint32_t*>(wb + kb),
                         *reinterpret_cast<const uint32_t*>(wb + kb + 8));
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[q] = __fadd_rn(acc[q], cacc[q]);
      }
      const int n = 8 * nj + 2 * c;
      const int t0 = 16 * mi + g;
      part[t0 * ep + n] = acc[0];
      part[t0 * ep + n + 1] = acc[1];
      part[(t0 + 8) * ep + n] = acc[2];
      part[(t0 + 8) * ep + n + 1] = acc[3];
    }
    cluster_sync();                               // partials complete on every rank
    // ---- phase 2: tokens t = rank, rank + kDpCluster, ...: logits summed over the ranks
    // in rank order + bias, one bf16 rounding; top-k by counting the experts ranked
    // ahead; softmax; the routing goes to global memory and to rank 0's sort inputs
    const int nt_r = T > static_cast<int>(rank) ? (T - static_cast<int>(rank) + kDpCluster - 1) / kDpCluster : 0;
    for (int q = tid; q < nt_r * E; q += kDpThreads) {
      const int i = q / E, e = q - i * E;
      const int t = static_cast<int>(rank) + kDpCluster * i;
      const uint32_t a_loc = smem_u32(part + t * ep + e);
      float v[kDpCluster];
#pragma unroll
      for (int r = 0; r < kDpCluster; ++r) v[r] = dsmem_ld_f32(dsmem_map(a_loc, r));
      float a = v[0];
#pragma unroll
      for (int r = 1; r < kDpCluster; ++r) a = __fadd_rn(a, v[r]);
      lg[i * ep + e] = bf16_round(a + __bfloat162float(p.bias[e]));
    }
    __syncthreads();
    for (int q = tid; q < nt_r * E; q += kDpThreads) {
      const int i = q / E, e = q - i * E;
      const float* row = lg + i * ep;
      const float v = row[e];
      int rk = 0;
#pragma unroll 8
      for (int f = 0; f < E; ++f) rk += topk_ahead(row[f], f, v, e) ? 1 : 0;
      if (rk < K) { slot_e[i * K + rk] = e; slot_v[i * K + rk] = v; }
    }
    __syncthreads();
    const uint32_t sel0 = smem_u32(sel), wts0 = smem_u32(wts);
    for (int i = tid; i < nt_r; i += kDpThreads) {
      const int t = static_cast<int>(rank) + kDpCluster * i;
      const float m = slot_v[i * K];
      float ex[kMaxTopK], s = 0.0f;
#pragma unroll
      for (int j = 0; j < kMaxTopK; ++j)
        if (j < K) { ex[j] = expf(__fsub_rn(slot_v[i * K + j], m)); s = __fadd_rn(s, ex[j]); }
      const float inv = __frcp_rn(s);
#pragma unroll
      for (int j = 0; j < kMaxTopK; ++j) {
        if (j < K) {
          const __nv_bfloat16 pr = __float2bfloat16_rn(__fmul_rn(ex[j], inv));
          const int e = slot_e[i * K + j];
          p.ridx_out[t * K + j] = e;
          if (p.scores_out) p.scores_out[t * K + j] = pr;
          p.rw_out[t * K + j] = __bfloat162float(pr);
          for (int r = 0; r < kDpCluster; ++r) {   // every rank sorts the assignments
            dsmem_st_s32(dsmem_map(sel0 + 4u * (t * K + j), r), e);
            dsmem_st_f32(dsmem_map(wts0 + 4u * (t * K + j), r), __bfloat162float(pr));
          }
        }
      }
    }
  }
  cluster_sync();                                 // every rank holds every token's routing;
                                                  // no shared memory is accessed remotely after this
  // ---- phase 3 (every rank, redundantly): the stable counting sort of the assignments;
  // rank 0 writes the routed layout to global memory
  const bool writer = rank == 0;
  const bool epm = p.ep_world > 0;
  const int nb = epm ? p.ep_world : E;           // sort buckets: owning ranks or experts
  const int epr = epm ? p.ep_epr : 1;
  if (!router) {
    for (int i = tid; i < A; i += kDpThreads) {
      const int64_t v = p.ridx_in[i];
      if (v < 0 || v >= E) {
        if (writer && p.err) atomicCAS(p.err, 0, 0x201);
        sel[i] = -1;
      } else {
        sel[i] = static_cast<int>(v);
      }
      wts[i] = p.rw_in[i];
    }
  }
  for (int e = tid; e < nb; e += kDpThreads) cnt[e] = 0;
  __syncthreads();
  for (int i = tid; i < A; i += kDpThreads)
    if (sel[i] >= 0) atomicAdd(&cnt[sel[i] / epr], 1);
  __syncthreads();
  if (warp == 0) {                                // exclusive scans over the buckets
    int c_run = 0, a_run = 0, b_run = 0;
    const int per = (nb + 31) / 32;
    const int q0 = lane * per;
    for (int i = 0; i < per; ++i) {
      const int q = q0 + i;
      if (q < nb) {
        c_run += cnt[q];
        if (!epm) {
          a_run += static_cast<int>(act_sf_cosize(cnt[q], p.g4_a * 4, p.spread != 0));
          b_run += static_cast<int>(act_sf_cosize(cnt[q], p.g4_b * 4, p.spread != 0));
        }
      }
    }
    int ci = c_run, ai = a_run, bi = b_run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int c2 = __shfl_up_sync(0xffffffffu, ci, o);
      const int a2 = __shfl_up_sync(0xffffffffu, ai, o);
      const int b2 = __shfl_up_sync(0xffffffffu, bi, o);
      if (lane >= o) { ci += c2; ai += a2; bi += b2; }
    }
    int ce = ci - c_run, ae = ai - a_run, be = bi - b_run;
    for (int i = 0; i < per; ++i) {
      const int q = q0 + i;
      if (q < nb) {
        off[q] = ce; run[q] = ce;
        if (epm) {
          if (writer) p.send_counts[q] = cnt[q];
        } else {
          sfa[q] = ae; sfb[q] = be;
          if (writer) { p.counts[q] = cnt[q]; p.offsets[q] = ce; p.sf_offsets_a[q] = ae; p.sf_offsets_b[q] = be; }
          ae += static_cast<int>(act_sf_cosize(cnt[q], p.g4_a * 4, p.spread != 0));
          be += static_cast<int>(act_sf_cosize(cnt[q], p.g4_b * 4, p.spread != 0));
        }
        ce += cnt[q];
      }
    }
    __syncwarp();
    // stable positions, 32 assignments at a time: lanes with the same bucket rank
    // themselves by lane order on top of the bucket's running count
    for (int i0 = 0; i0 < A; i0 += 32) {
      const int i = i0 + lane;
      const int e = i < A ? (sel[i] >= 0 ? sel[i] / epr : -1) : -2;
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      if (e >= 0) {
        const int pos = run[e] + __popc(peers & ((1u << lane) - 1u));
        if (epm) {
          srow[pos] = i / K;
          sexp[pos] = i;                          // the assignment itself
          if (writer) p.pos_of[i] = e * static_cast<int>(p.ep_cap) + (pos - off[e]);
        } else {
          if (writer) {
            p.sorted_token[pos] = i / K;
            p.sorted_expert[pos] = e;
            p.sorted_weight[pos] = wts[i];
          }
          srow[pos] = i / K;
          sexp[pos] = e;
        }
      } else if (e == -1 && epm && writer) {
        p.pos_of[i] = -1;                         // out-of-range expert id: nothing returns
      }
      __syncwarp();
      if (e >= 0 && lane == __ffs(peers) - 1) run[e] += __popc(peers);
      __syncwarp();
    }
  }
  __syncthreads();
  if (epm) {
    ep_dispatch_phase4(p, rank, codes, sfs, srow, sexp, sel, wts, cnt, off, sl, slv, gs, k0);
    return;
  }
  if (writer) {
    const int total = off[E - 1] + cnt[E - 1];
    for (int i = total + tid; i < A; i += kDpThreads) {   // out-of-range indices: sentinel
      p.sorted_token[i] = -1;
      p.sorted_expert[i] = -1;
      p.sorted_weight[i] = 0.0f;
    }
  }
  // ---- phase 4: this rank's K slice of every expert-sorted row (codes and scale words)
  // straight from shared memory. The scale bytes of the blocks' padding rows stay as they
  // are: a padding row only feeds its own accumulator row (or column) of the GEMMs, which
  // no epilogue stores, and every valid row's words, K padding included, are written.
  const int a_lo = k0 / 128, a_hi = min(p.g4_a, (k0 + sl) / 128);
  const int total = off[E - 1] + cnt[E - 1];
  if (slv > 0) {
    const int v16 = slv / 16;
    for (int q = tid; q < total * v16; q += kDpThreads) {
      const int pos = q / v16, v = q - pos * v16;
      const int t = srow[pos];
      reinterpret_cast<uint4*>(p.act_codes + static_cast<int64_t>(pos) * H + k0)[v] =
          reinterpret_cast<const uint4*>(codes + t * sl)[v];
    }
    const int na = a_hi - a_lo;
    for (int q = tid; q < total * na; q += kDpThreads) {
      const int pos = q / na, a = a_lo + (q - pos * na);
      const int t = srow[pos], e = sexp[pos];
      const int j = pos - off[e];
      const int64_t r_in = p.spread ? act_sf_row<true>(j) : j;
      const uint8_t* sc = sfs + t * gs + 4 * (a - a_lo);
      const uint32_t word = sc[0] | (static_cast<uint32_t>(sc[1]) << 8) | (static_cast<uint32_t>(sc[2]) << 16) |
                            (static_cast<uint32_t>(sc[3]) << 24);
      *reinterpret_cast<uint32_t*>(p.act_sf + sfa[e] + blocked_sf_offset(r_in, 4 * a, p.g4_a)) = word;
    }
  }
}

}  // namespace gptoss
