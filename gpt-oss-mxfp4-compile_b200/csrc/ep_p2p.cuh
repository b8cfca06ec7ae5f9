// Expert-parallel exchange over NVLink peer memory (no collective library on the data
// path). Every rank owns one peer-mapped exchange buffer (cudaIpc, mapped on every other
// rank of the node):
//
//   [ flags: 2 * kP2pMaxWorld int32 | recv rows [W][cap][row_bytes] | ret rows [W][cap][H] bf16 ]
//
//   dispatch  rank s packs (quantises) each assignment's row straight into the receive
//             rows of the owning rank q at segment s (st.global to q's memory); rows of
//             the segment past the count carry the empty-slot marker; then it raises
//             flag[s] of every peer to the call's epoch (release, system scope).
//   expert    rank q waits (bounded) until flag[s] >= epoch for every s, runs the local
//             expert forward on its W * cap received rows, and copies each valid output
//             row back into the ret rows of its source rank s at segment q; then it
//             raises flag[W + q] of every peer.
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
constexpr uint32_t kP2pFlagBytes = 2 * kP2pMaxWorld * 4;

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

// One CTA, blockDim >= world: after the previous kernel on the stream (whose stores went to
// the peers) completed, raise flags[slot] on every peer to `epoch`.
__global__ void p2p_signal_kernel(const uint64_t* __restrict__ peer_bases, int world, int slot, int32_t epoch) {
  pdl_trigger();
  pdl_wait();
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  const int q = threadIdx.x;
  if (q < world) st_release_sys(reinterpret_cast<int32_t*>(peer_bases[q]) + slot, epoch);
}

// Dispatch: like ep_pack_kernel with the fixed-capacity layout, but row j of destination q
// goes to peer q's receive rows, segment `rank`.
__global__ void __launch_bounds__(256) ep_pack_p2p_kernel(
    const __nv_bfloat16* __restrict__ hidden, int H, int K, int experts_per_rank, int64_t A,
    const int64_t* __restrict__ router_indices, const float* __restrict__ routing_weights,
    const int32_t* __restrict__ sorted_src, int64_t cap, int world, int rank,
    const int32_t* __restrict__ dest_counts, const int32_t* __restrict__ dest_offsets, int tpr,
    const uint64_t* __restrict__ peer_bases, int32_t* __restrict__ pos_of) {
  pdl_trigger();
  pdl_wait();
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
__global__ void __launch_bounds__(256) ep_return_p2p_kernel(const __nv_bfloat16* __restrict__ back_rows,
                                                            const int64_t* __restrict__ expert, int64_t cap,
                                                            int world, int rank, int H,
                                                            const uint64_t* __restrict__ peer_bases) {
  pdl_trigger();
  pdl_wait();
  const int64_t r = blockIdx.x;
  if (r >= cap * world || expert[r] < 0) return;
  const int s = static_cast<int>(r / cap);
  const int64_t j = r - static_cast<int64_t>(s) * cap;
  const int64_t rb = ep_row_bytes(H);
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(peer_bases[s]) +
                                        p2p_ret_offset(world, rank, cap, rb, H) + j * H * 2);
  const uint4* src = reinterpret_cast<const uint4*>(back_rows + r * H);
  for (int v = threadIdx.x; v < H / 8; v += blockDim.x) dst[v] = src[v];
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
