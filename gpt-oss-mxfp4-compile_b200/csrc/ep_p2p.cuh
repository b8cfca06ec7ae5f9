// Expert-parallel exchange over NVLink peer memory (no collective library on the data
// path). Every rank owns one peer-mapped exchange buffer (cudaIpc, mapped on every other
// rank of the node):
//
//   [ header: flags + counters (1 KB) | recv rows [W][cap][row_bytes] | ret rows [W][cap][H] bf16 ]
//
//   dispatch  rank s packs (quantises) each assignment's row straight into the receive
//             rows of the owning rank q at segment s (st.global to q's memory); rows of
//             the segment past the count carry the empty-slot marker; then it raises
//             flag[s] of every peer to the call's epoch (release, system scope).
//   expert    rank q waits (bounded) until flag[s] >= epoch for every s, runs the local
//             expert forward on its W * cap received rows, and each valid output row goes
//             back into the ret rows of its source rank s at segment q (stored by GEMM2's
//             epilogue for weights-on-M tiles, else copied by ep_return_p2p_kernel); then
//             the last CTA of that kernel raises flag[W + q] of every peer.
//   combine   rank s waits (bounded) until flag[W + q] >= epoch for every q and sums each
//             token's k returned rows (ascending expert, fp32, one bf16 rounding).
//
// Reuse of the buffers across calls needs no barrier: a rank starts dispatch n + 1 only
// after its combine n saw every owner's return flag n, which each owner raises after it
// finished reading its receive rows of call n; and an owner writes ret rows of call n + 1
// only after seeing the dispatch flags of call n + 1. Epochs only grow.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include "ptx.cuh"
#include "numerics.cuh"
#include "routing.cuh"

namespace gptoss {

constexpr int kP2pMaxWorld = 64;
constexpr int kDevTimeoutPeer = 0x301;    // a peer's flag did not arrive within the timeout
// header (int32 words): dispatch flags [0, 64), return flags [64, 128), completion counters
// [128, 130), rows each source sent in the current call [192, 256) (written before its flag)
constexpr uint32_t kP2pFlagBytes = 4 * kP2pMaxWorld * 4;
constexpr int kP2pCounterDispatch = 2 * kP2pMaxWorld;
constexpr int kP2pCounterReturn = 2 * kP2pMaxWorld + 1;
constexpr int kP2pSendCounts = 3 * kP2pMaxWorld;

__host__ __device__ __forceinline__ int64_t p2p_recv_offset(int rank_s, int64_t cap, int64_t rb) {
  return kP2pFlagBytes + static_cast<int64_t>(rank_s) * cap * rb;
}
__host__ __device__ __forceinline__ int64_t p2p_ret_offset(int world, int rank_q, int64_t cap, int64_t rb, int H) {
  return kP2pFlagBytes + world * cap * rb + static_cast<int64_t>(rank_q) * cap * H * 2;
}
__host__ __device__ __forceinline__ int64_t p2p_buffer_bytes(int world, int64_t cap, int H) {
  const int64_t rb = ep_row_bytes(H);
  return kP2pFlagBytes + world * cap * rb + world * cap * static_cast<int64_t>(H) * 2;
}

__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(int32_t* p, int32_t v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys(int32_t* p, int32_t v) {
  asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Raise flags[slot] of every peer to `epoch`, called by the 32 lanes of one warp after a
// system-scope fence of everything the caller published: one fence, then the W flag stores
// in parallel from separate lanes (W release stores from one thread would each wait for the
// previous one's NVLink round trip).
__device__ __forceinline__ void p2p_raise_flags_warp(const uint64_t* peer_bases, int world, int slot, int32_t epoch) {
  __threadfence_system();
  for (int q = static_cast<int>(threadIdx.x & 31u); q < world; q += 32)
    st_relaxed_sys(reinterpret_cast<int32_t*>(peer_bases[q]) + slot, epoch);
}

// Thread 0 waits until flags[first .. first + n) all reach `epoch` (bounded by
// kWaitTimeoutNs; on a timeout it records kDevTimeoutPeer and gives up), then the CTA
// proceeds. The acquire loads order the CTA's later reads after the peers' writes.
__device__ __forceinline__ void p2p_wait_flags(const int32_t* flags, int first, int n, int32_t epoch, int* err) {
  if (threadIdx.x == 0) {
    const uint64_t t0 = globaltimer_ns();
    for (int i = 0; i < n; ++i) {
      while (ld_acquire_sys(flags + first + i) < epoch) {
        if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
          if (err) atomicCAS(err, 0, kDevTimeoutPeer);
          i = n;
          break;
        }
      }
    }
  }
  __syncthreads();
}

// Called by the 32 lanes of warp 0 of every CTA after the CTA's stores to the peers (behind
// a CTA barrier): the last CTA to get here raises flags[slot] on every peer to `epoch` (the
// threadfence-reduction pattern: every CTA fences its stores at system scope before counting
// itself) and resets the counter for the next call.
__device__ __forceinline__ void p2p_last_cta_signal(int32_t* counter, const uint64_t* peer_bases, int world,
                                                    int slot, int32_t epoch) {
  int prev = 0;
  if ((threadIdx.x & 31u) == 0) {
    __threadfence_system();
    prev = atomicAdd(counter, 1);
  }
  prev = __shfl_sync(0xffffffffu, prev, 0);
  if (prev == static_cast<int>(gridDim.x * gridDim.y * gridDim.z) - 1) {
    p2p_raise_flags_warp(peer_bases, world, slot, epoch);
    __syncwarp();
    if ((threadIdx.x & 31u) == 0) atomicExch(counter, 0);
  }
}

// Row r of the fixed-capacity send layout (destination q = r / cap, slot j = r % cap):
// quantised into peer q's receive rows, segment `rank`, or marked empty past the count.
__device__ __forceinline__ void ep_pack_p2p_row(
    const __nv_bfloat16* __restrict__ hidden, int H, int K, int experts_per_rank,
    const int64_t* __restrict__ router_indices, const float* __restrict__ routing_weights,
    const int32_t* __restrict__ sorted_src, int64_t cap, int world, int rank,
    const int32_t* __restrict__ dest_counts, const int32_t* __restrict__ dest_offsets, int tpr,
    const uint64_t* __restrict__ peer_bases, int32_t* __restrict__ pos_of) {
  const int rows_per_block = blockDim.x / tpr;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * rows_per_block + threadIdx.x / tpr;
  if (r >= cap * world) return;
  const int sub = threadIdx.x % tpr;
  const int G = H >> 5;
  const int64_t rb = ep_row_bytes(H);
  const int q = static_cast<int>(r / cap);
  const int64_t j = r - static_cast<int64_t>(q) * cap;
  uint8_t* row = reinterpret_cast<uint8_t*>(peer_bases[q]) + p2p_recv_offset(rank, cap, rb) + j * rb;
  if (j >= dest_counts[q]) {
    if (sub == 0) {
      int32_t* meta = reinterpret_cast<int32_t*>(row + rb - 8);
      meta[0] = -1;
      meta[1] = 0;
    }
    return;
  }
  const int i = sorted_src[dest_offsets[q] + j];
  if (i < 0) return;   // sentinel of an out-of-range router index
  const int64_t t = i / K;
  const __nv_bfloat16* xr = hidden + t * H;
  for (int g = sub; g < G; g += tpr) {
    const uint4* pp = reinterpret_cast<const uint4*>(xr + g * 32);
    uint4 u[4];
#pragma unroll
    for (int qq = 0; qq < 4; ++qq) u[qq] = __ldg(pp + qq);
    float v[32];
#pragma unroll
    for (int qq = 0; qq < 4; ++qq) {
      const uint32_t w4[4] = {u[qq].x, u[qq].y, u[qq].z, u[qq].w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        v[qq * 8 + 2 * h] = bf16_bits_lo(w4[h]);
        v[qq * 8 + 2 * h + 1] = bf16_bits_hi(w4[h]);
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

// Dispatch: like ep_pack_kernel with the fixed-capacity layout, but row j of destination q
// goes to peer q's receive rows, segment `rank`.
__global__ void __launch_bounds__(256) ep_pack_p2p_kernel(
    const __nv_bfloat16* __restrict__ hidden, int H, int K, int experts_per_rank, int64_t A,
    const int64_t* __restrict__ router_indices, const float* __restrict__ routing_weights,
    const int32_t* __restrict__ sorted_src, int64_t cap, int world, int rank,
    const int32_t* __restrict__ dest_counts, const int32_t* __restrict__ dest_offsets, int tpr,
    const uint64_t* __restrict__ peer_bases, int32_t* __restrict__ pos_of, int32_t* __restrict__ counter,
    int32_t epoch) {
  pdl_trigger();
  pdl_wait();
  ep_pack_p2p_row(hidden, H, K, experts_per_rank, router_indices, routing_weights, sorted_src, cap, world, rank,
                  dest_counts, dest_offsets, tpr, peer_bases, pos_of);
  __syncthreads();
  if (threadIdx.x < 32) p2p_last_cta_signal(counter, peer_bases, world, rank, epoch);
}


// Receiving rank: wait for every sender's dispatch flag, then row r's (local expert,
// weight) -> the arrays route_sort_kernel reads (empty slots carry expert -1).
__global__ void ep_unpack_meta_p2p_kernel(const uint8_t* __restrict__ recv_rows, int64_t R, int H,
                                          const int32_t* __restrict__ flags, int world, int32_t epoch,
                                          int* err, int64_t* __restrict__ expert, float* __restrict__ weight) {
  pdl_trigger();
  pdl_wait();
  p2p_wait_flags(flags, 0, world, epoch, err);
  const int64_t rb = ep_row_bytes(H);
  for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; r < R;
       r += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t* meta = reinterpret_cast<const int32_t*>(recv_rows + r * rb + rb - 8);
    expert[r] = meta[0];
    weight[r] = __int_as_float(meta[1]);
  }
}

// Owner: output row r of the local expert forward (received row r = segment s, slot j)
// -> ret rows of source rank s, segment `rank`, slot j. One CTA per row; empty rows skip.
// The last CTA raises return flag[W + rank] on every peer.
__global__ void __launch_bounds__(256) ep_return_p2p_kernel(const __nv_bfloat16* __restrict__ back_rows,
                                                            const int64_t* __restrict__ expert, int64_t cap,
                                                            int world, int rank, int H,
                                                            const uint64_t* __restrict__ peer_bases,
                                                            int32_t* __restrict__ counter, int32_t epoch) {
  pdl_trigger();
  pdl_wait();
  const int64_t r = blockIdx.x;
  if (r < cap * world && expert[r] >= 0) {
    const int s = static_cast<int>(r / cap);
    const int64_t j = r - static_cast<int64_t>(s) * cap;
    const int64_t rb = ep_row_bytes(H);
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(peer_bases[s]) +
                                          p2p_ret_offset(world, rank, cap, rb, H) + j * H * 2);
    const uint4* src = reinterpret_cast<const uint4*>(back_rows + r * H);
    for (int v = threadIdx.x; v < H / 8; v += blockDim.x) dst[v] = src[v];
  }
  __syncthreads();
  if (threadIdx.x < 32) p2p_last_cta_signal(counter, peer_bases, world, world + rank, epoch);
}

// ---------------------------------------------------------------- receiving rank, one launch
// Wait for every sender's flag, then (every CTA, redundantly) read the W * cap row
// headers into shared memory and run the stable counting sort by local expert (empty slots
// skipped; the order of route_sort_kernel); CTA 0 writes the routed layout. Then CTA c
// copies the sorted rows c, c + gridDim.x, ... -- FP8 codes into the GEMM's activation
// rows, the row's UE8M0 bytes as 32-bit words into the blocked layout (the padding groups
// of the last k-atom travel as zeros) -- and every CTA zeroes a share of the output rows the
// GEMM2 combine adds into.
constexpr int kRpMaxRows = 8192;

struct RecvPrologueParams {
  const uint8_t* recv;         // [R, row_bytes]
  int64_t R;
  int H, E, world;
  int32_t epoch;
  const int32_t* flags;
  int* err;
  int64_t* lexp;               // [R] local expert of each row (-1: empty), for the return
  float* lw;                   // [R]
  int64_t* sorted_token;       // sorted position -> received row
  int64_t* sorted_expert;
  float* sorted_weight;
  int32_t* counts;
  int32_t* offsets;
  int32_t* sf_offsets_a;
  int32_t* sf_offsets_b;
  int g4_a, g4_b, spread;
  uint8_t* act_codes;
  uint8_t* act_sf;
  __nv_bfloat16* back_rows;    // [R, H], zeroed here (nullptr: not needed)
};

__host__ __device__ inline size_t recv_prologue_smem(int64_t R, int E) {
  return static_cast<size_t>(R) * 12 + static_cast<size_t>(E) * 20 + 64;
}

__global__ void __launch_bounds__(256) ep_recv_prologue_kernel(const RecvPrologueParams p) {
  extern __shared__ __align__(16) uint8_t rp_smem[];
  const int R = static_cast<int>(p.R), E = p.E;
  int* s_e = reinterpret_cast<int*>(rp_smem);
  float* s_w = reinterpret_cast<float*>(s_e + R);
  int* srow = reinterpret_cast<int*>(s_w + R);
  int* cnt = srow + R;
  int* off = cnt + E;
  int* sfa = off + E;
  int* sfb = sfa + E;
  int* run = sfb + E;
  pdl_trigger();
  pdl_wait();
  p2p_wait_flags(p.flags, 0, p.world, p.epoch, p.err);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool writer = blockIdx.x == 0;
  const int64_t rb = ep_row_bytes(p.H);
  for (int e = tid; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int r = tid; r < R; r += blockDim.x) {
    const int32_t* meta = reinterpret_cast<const int32_t*>(p.recv + r * rb + rb - 8);
    int e = meta[0];
    const float w = __int_as_float(meta[1]);
    if (e >= E || e < -1) {
      if (writer && p.err) atomicCAS(p.err, 0, 0x201);
      e = -1;
    }
    s_e[r] = e;
    s_w[r] = w;
    if (e >= 0) atomicAdd(&cnt[e], 1);
    if (writer) { p.lexp[r] = e; p.lw[r] = w; }
  }
  __syncthreads();
  if (warp == 0) {
    int c_run = 0, a_run = 0, b_run = 0;
    const int per = (E + 31) / 32;
    const int q0 = lane * per;
    for (int i = 0; i < per; ++i) {
      const int q = q0 + i;
      if (q < E) {
        c_run += cnt[q];
        a_run += static_cast<int>(act_sf_cosize(cnt[q], p.g4_a * 4, p.spread != 0));
        b_run += static_cast<int>(act_sf_cosize(cnt[q], p.g4_b * 4, p.spread != 0));
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
      if (q < E) {
        off[q] = ce; run[q] = ce; sfa[q] = ae; sfb[q] = be;
        if (writer) { p.counts[q] = cnt[q]; p.offsets[q] = ce; p.sf_offsets_a[q] = ae; p.sf_offsets_b[q] = be; }
        ce += cnt[q];
        ae += static_cast<int>(act_sf_cosize(cnt[q], p.g4_a * 4, p.spread != 0));
        be += static_cast<int>(act_sf_cosize(cnt[q], p.g4_b * 4, p.spread != 0));
      }
    }
    __syncwarp();
    for (int i0 = 0; i0 < R; i0 += 32) {
      const int r = i0 + lane;
      const int e = r < R ? s_e[r] : -1;
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      if (e >= 0) {
        const int pos = run[e] + __popc(peers & ((1u << lane) - 1u));
        srow[pos] = r;
        if (writer) {
          p.sorted_token[pos] = r;
          p.sorted_expert[pos] = e;
          p.sorted_weight[pos] = s_w[r];
        }
      }
      __syncwarp();
      if (e >= 0 && lane == __ffs(peers) - 1) run[e] += __popc(peers);
      __syncwarp();
    }
  }
  __syncthreads();
  const int total = E > 0 ? off[E - 1] + cnt[E - 1] : 0;
  if (writer) {
    for (int i = total + tid; i < R; i += blockDim.x) {
      p.sorted_token[i] = -1;
      p.sorted_expert[i] = -1;
      p.sorted_weight[i] = 0.0f;
    }
  }
  const int H = p.H;
  for (int pos = blockIdx.x; pos < total; pos += gridDim.x) {
    const int r = srow[pos];
    const int e = s_e[r];
    const int j = pos - off[e];
    const int64_t r_in = p.spread ? act_sf_row<true>(j) : j;
    const uint8_t* src = p.recv + r * rb;
    for (int v = tid; v < H / 16; v += blockDim.x)
      reinterpret_cast<uint4*>(p.act_codes + static_cast<int64_t>(pos) * H)[v] = reinterpret_cast<const uint4*>(src)[v];
    for (int a = tid; a < p.g4_a; a += blockDim.x)   // bytes past H/32 are the zero padding of the row
      *reinterpret_cast<uint32_t*>(p.act_sf + sfa[e] + blocked_sf_offset(r_in, 4 * a, p.g4_a)) =
          *reinterpret_cast<const uint32_t*>(src + H + 4 * a);
  }
  if (p.back_rows != nullptr) {   // null: GEMM2 stores the rows straight into the sources' buffers
    const int64_t n16 = static_cast<int64_t>(R) * H / 8;
    uint4* z = reinterpret_cast<uint4*>(p.back_rows);
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + tid; i < n16;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
      z[i] = make_uint4(0, 0, 0, 0);
  }
}

// Source: wait for every owner's return flag, then the combine of ep_combine_kernel over
// this rank's ret rows.
__global__ void __launch_bounds__(256) ep_combine_p2p_kernel(const __nv_bfloat16* __restrict__ ret_rows,
                                                             const int32_t* __restrict__ flags, int world,
                                                             int32_t epoch, int* err,
                                                             const int32_t* __restrict__ pos_of,
                                                             const int64_t* __restrict__ router_indices,
                                                             int64_t T, int K, int H, int64_t rows,
                                                             __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  p2p_wait_flags(flags, world, world, epoch, err);
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
      const __nv_bfloat162 v = reinterpret_cast<const __nv_bfloat162*>(ret_rows + pr * H)[h2];
      a0 += __bfloat162float(v.x);
      a1 += __bfloat162float(v.y);
    }
    reinterpret_cast<__nv_bfloat162*>(out + t * H)[h2] = __floats2bfloat162_rn(a0, a1);
  }
}

}  // namespace gptoss
