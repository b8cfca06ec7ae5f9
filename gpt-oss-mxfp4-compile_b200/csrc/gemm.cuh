// Grouped W4A8 GEMM for sm_100a: FP8 e4m3 activations x E2M1 weights, UE8M0 1x32 block
// scales, fp32 accumulation in TMEM via tcgen05.mma kind::mxf8f6f4.block_scale.
//
// One persistent CTA per SM (or CTA pair) walks a ragged tile list built on the device
// from the per-expert row counts (no host sync). Warp roles:
//   warp 0     TMA producer: activation tile (2-D map, fp8), weight tile (3-D map,
//              packed e2m1 expanded to the 8-bit smem container by the TMA unit),
//              plus the 512-byte blocked scale chunks (bulk copies, or 256-byte-row
//              tensor maps for CTA pairs); SWAP tiles load two K blocks per stage.
//   warp 1     TMEM allocator + MMA issuer: tcgen05.cp of the scale chunks into TMEM,
//              then 4 MMAs (K = 32 each) per 128-deep K block. SWAP tiles add a second
//              issuer warp (the last warp) that takes the odd K blocks into a second
//              partial accumulator.
//   warps 2+   epilogue: tcgen05.ld of the accumulator and one of three fused tails;
//              4 warps (SWAP; two passes through shared memory) or 12 warps, three per
//              TMEM lane quarter, each warpgroup taking one 64-column slice of the
//              192-column tile (SWAP = false).
//
// Two orientations:
//   SWAP = false  M = 128 activation rows, N = 192 weight rows (prefill-sized groups;
//                 PAIR: M = 256 over a CTA pair).
//   SWAP = true   M = 128 weight rows, N = 16 (SPREAD) or 16/32/64 activation rows
//                 (decode: the weights stream through the M side so a group of a few
//                 rows wastes little MMA).
//
// Epilogues (all restate cutlass_experts.py:414-450 for the rows a tile owns):
//   kEpiPlain  D = bf16(alpha[e] * acc) stored row-major (the fp4_group_mm op,
//              matmul_mxfp4_cutlass.cu:1118-1171 with beta = 0).
//   kEpiGemm1  h = swiglu(float(bf16(acc)) + b_gu[e]) on (even, odd) column pairs,
//              then FP8 + UE8M0 requantisation written as the next GEMM's A operand
//              (codes compact row-major, scales in the blocked layout).
//   kEpiGemm2  y = bf16((float(bf16(acc)) + b_dn[e]) * w_row) added into out[token]
//              with bf16x2 vector reductions (the scatter_add_ of :445-450), or stored
//              into the source rank's return rows over peer memory (expert parallelism).
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include "ptx.cuh"
#include "numerics.cuh"
#include "ep_p2p.cuh"

namespace gptoss {

enum EpilogueKind : int { kEpiPlain = 0, kEpiGemm1 = 1, kEpiGemm2 = 2 };

struct GemmParams {
  int num_experts;
  int N;                        // weight rows (output features) per expert
  int K;                        // padded reduction depth, multiple of 128
  int num_kb;                   // K / 128
  const int32_t* m_sizes;       // rows of expert e at m_sizes[e * m_stride]
  int m_stride;
  const int32_t* row_offsets;   // first activation / output row of each expert
  const int32_t* sfa_offsets;   // byte offset of each expert's activation scales
  const uint8_t* sfa;           // activation scales, blocked layout
  const uint8_t* sfb;           // weight scales, blocked layout
  int64_t sfb_stride;           // bytes between experts in sfb
  int n_tiles;                  // ceil(N / weight rows per tile)
  int* err;                     // device status word (0 = ok)
  // epilogue
  void* out;
  int64_t ld_out;               // elements per output row
  const float* alphas;          // kEpiPlain
  const float* bias;            // [E, N] fp32 (kEpiGemm1, kEpiGemm2)
  uint8_t* out_sf;              // kEpiGemm1: blocked scales of the intermediate
  const int32_t* out_sf_offsets;
  int out_g4;
  int out_features;             // kEpiGemm1: intermediate width (N / 2)
  const int64_t* token_idx;     // kEpiGemm2
  const int32_t* token_idx32;   // kEpiGemm2 on weights-on-M tiles: 32-bit row indices when set
  const float* row_weights;     // kEpiGemm2
  float swiglu_alpha, swiglu_limit;
  // Weights-on-M tiles: weight tiles each CTA prefetches into L2 before waiting on the
  // previous kernel (0: none). The tiles are guessed assuming one activation chunk per
  // expert -- the decode case; a wrong guess only costs bandwidth.
  int prefetch_tiles;
  // kEpiGemm2 on weights-on-M tiles, expert parallelism over peer memory (ep_world > 0):
  // output row r is a received row (segment s = r / ep_cap, slot j); its values go straight
  // into source rank s's return rows (ep_ret_off bytes into s's exchange buffer, row j)
  // with 16-byte stores instead of being added into `out`, and the last CTA to finish
  // raises return flag [ep_world + ep_rank] on every peer.
  const uint64_t* ep_peer_bases;
  int64_t ep_ret_off;
  int64_t ep_cap;
  int32_t* ep_counter;
  int ep_world, ep_rank;
  int32_t ep_epoch;
};

// PAIR: tokens-on-M tiles computed by a CTA pair (cluster of 2, tcgen05 cta_group::2):
// M = 256 activation rows (128 per CTA), N = 192 weight rows (each CTA loads 96 of them,
// the MMA reads both halves), so per SM the weight bytes per MMA halve and the ring holds
// 7 stages instead of 5. Each CTA still loads its activation-row scales and the full
// tile's weight scales.
//
// NVF4: the W4A4 mode (NVFP4 x NVFP4: packed E2M1 activations and weights, UE4M3 scales
// per 16 codes; tcgen05.mma kind::mxf4nvf4 scale_vec::4X, K = 64 per MMA). A k block is
// still 128 bytes of every operand row (256 codes), so tiles, TMA boxes and descriptors
// are those of the W4A8 mode; a k block's scales are 4 blocked atoms (64 codes each) per
// 128 rows instead of one, copied into 4 TMEM column groups that the 4 MMAs read in turn.
template <bool SWAP, bool SPREAD = false, bool PAIR = false, bool NVF4 = false>
struct GemmConfig {
  static_assert(SWAP || !SPREAD, "spread activation scales are a SWAP-mode layout");
  static_assert(!(SWAP && PAIR), "CTA pairs are a tokens-on-M layout");
  static_assert(!(NVF4 && (SPREAD || PAIR)), "NVFP4 tiles: reference scale rows, single CTAs");
  static constexpr int kWgtRows = SWAP ? 128 : 192;   // weight rows per tile
  static constexpr int kWgtRowsCta = PAIR ? kWgtRows / 2 : kWgtRows;   // weight rows this CTA loads
  // Activation rows per tile. SWAP with reference-layout scales uses 64-row chunks that
  // start 0 or 64 rows into a 128-row scale block (TMEM column offset 0 or 2); SPREAD
  // uses 16-row chunks (a 2 KB activation slot per K block).
  static constexpr int kActRows = SWAP ? (SPREAD ? 16 : 64) : 128;
  static constexpr int kColChunks = (kActRows + 31) / 32;   // 32-column TMEM loads per tile
  static constexpr int kTileM = PAIR ? 2 * kActRows : kActRows;   // activation rows per tile
  static constexpr int kMmaM = PAIR ? 256 : 128;
  static constexpr int kMmaN = SWAP ? kActRows : kWgtRows;
  // K blocks (128 codes each) per pipeline stage. The TMA engine completes about one
  // mbarrier transaction group per ~300 ns per SM whatever its size (measured on B200:
  // 8 KB fp4 weight boxes stream at ~4 TB/s one per stage and ~6.7 TB/s two per stage,
  // at any ring depth), so weights-on-M tiles load two k blocks behind each barrier.
  static constexpr int kSubs = SWAP ? 2 : 1;
  static constexpr int kStages = SWAP ? (SPREAD ? 5 : (NVF4 ? 3 : 4)) : (PAIR ? 7 : (NVF4 ? 4 : 5));
  static constexpr int kKbCodes = NVF4 ? 256 : 128;   // K codes per k block
  static constexpr int kSfAtoms = NVF4 ? 4 : 1;       // 512-byte scale atoms per 128 rows per k block
  // global bytes of one weight row per k block (W4A8: 64 packed bytes the TMA expands to 128)
  static constexpr uint32_t kWgtRowGlobalBytes = NVF4 ? 128u : 64u;
  // MMA issuing threads. A small-N block-scaled MMA costs ~75 cycles of issue, so one
  // thread cannot keep up with the weight stream of weights-on-M tiles: two warps issue
  // alternate k blocks of each stage into two partial accumulators that the epilogue adds.
  static constexpr int kIssuers = SWAP ? 2 : 1;
  static constexpr int kAccBufs = SWAP ? (SPREAD ? 4 : 3) : 2;
  static constexpr int kAccCols = kMmaN;              // fp32 columns per partial accumulator
  static constexpr int kAccStride = kIssuers * kAccCols;   // columns per accumulator buffer
  static constexpr int kWgtSfChunks = SWAP ? 1 : 2;   // 128-row scale blocks per tile
  static constexpr uint32_t kWgtTileBytes = kWgtRowsCta * 128;   // 8-bit container in smem
  static constexpr uint32_t kActTileBytes = kActRows * 128;
  static constexpr uint32_t kSfActBytes = 512 * kSfAtoms;
  static constexpr uint32_t kSfWgtBytes = 512 * kSfAtoms * kWgtSfChunks;
  static constexpr uint32_t kSubBytes =   // one k block: weights | activations | scales
      ((kWgtTileBytes + kActTileBytes + kSfActBytes + kSfWgtBytes + 1023) / 1024) * 1024;
  static constexpr uint32_t kStageBytes = kSubs * kSubBytes;
  static constexpr uint32_t kTmemAccCols = kAccBufs * kAccStride;
  // scale columns of each issuer: activation 4 per atom, then weights 4 per atom and chunk
  // (atom-major: the chunks of one atom are adjacent, so a tile that starts 64 rows into a
  // 128-row block reads across them)
  static constexpr uint32_t kSfCols = 4 * kSfAtoms * (1 + kWgtSfChunks);
  static constexpr uint32_t kSfActCol = kTmemAccCols;
  static constexpr uint32_t kSfWgtCol = kTmemAccCols + 4 * kSfAtoms;
  static constexpr uint32_t kTmemUsed = kTmemAccCols + kIssuers * kSfCols;
  static constexpr uint32_t kTmemCols = kTmemUsed <= 128 ? 128 : kTmemUsed <= 256 ? 256 : 512;
  static_assert(kTmemUsed <= 512, "TMEM budget");
  static constexpr uint32_t kBarrierBytes = 8 * (2 * kStages + 2 * kAccBufs + 1) + 16;
  static constexpr uint32_t kEpiStageBytes = SWAP ? 16384 : 0;   // weights-on-M epilogue staging
  static constexpr uint32_t kSmemBytes =
      1024 + kStages * kStageBytes + ((kBarrierBytes + 127) & ~127u) + kEpiStageBytes + 2048;
  // Epilogue warps: one warpgroup for weights-on-M tiles (their two-pass epilogue
  // regroups rows through shared memory across the warpgroup); tokens-on-M tiles give
  // each warpgroup one 64-column slice, so three warps share every TMEM lane quarter and
  // hide each other's latency.
  static constexpr int kEpiWarps = SWAP ? 4 : 4 * (kWgtRows / 64);
  static constexpr int kThreads = 64 + 32 * kEpiWarps + 32 * (kIssuers - 1);   // 2nd issuer: last warp
};

constexpr int kMaxExpertsGemm = 256;

// 32 consecutive fp32 bias values (16-byte vector loads when all are in range; zero past
// `valid`). `b` is 16-byte aligned whenever valid >= 32 (N and the column are multiples
// of 32).
__device__ __forceinline__ void load_bias32(const float* b, int valid, float (&out)[32]) {
  if (valid >= 32) {
    const float4* b4 = reinterpret_cast<const float4*>(b);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 v = __ldg(b4 + i);
      out[4 * i] = v.x; out[4 * i + 1] = v.y; out[4 * i + 2] = v.z; out[4 * i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) out[i] = i < valid ? b[i] : 0.0f;
  }
}

// Weights-on-M (SWAP) GEMM1 / GEMM2 epilogue of one tile, run by the four epilogue warps
// (warps 2..5: TMEM lane quarter q = warp % 4). t_acc: the tile's accumulator buffer at this
// warp's lane quarter; acce_bar_b: the barrier that hands the buffer back to the MMA.
// out_sf_offsets, token_idx and row_weights may point to shared memory (generic addresses).
template <bool SPREAD, int EPI>
__device__ __forceinline__ void swap_epilogue_tile(const GemmParams& p, uint32_t t_acc, uint32_t acce_bar_b, int e,
                                                   int nt, int ch, int m_e, int row0, int local, float* epi_f,
                                                   bool has_b, int q, int lane) {
  using C = GemmConfig<true, SPREAD, false>;
  constexpr int kEpiTok = C::kActRows < 32 ? C::kActRows : 32;
  constexpr int kEpiFeat = EPI == kEpiGemm1 ? C::kWgtRows / 2 : C::kWgtRows;
  constexpr uint32_t kEpiBufBytes = static_cast<uint32_t>(kEpiTok * kEpiFeat * 4);
  constexpr int kEpiBufs = 2 * kEpiBufBytes <= C::kEpiStageBytes ? 2 : 1;
  static_assert(kEpiBufBytes <= C::kEpiStageBytes, "epilogue staging too small");
  // Weights-on-M GEMM1 / GEMM2 epilogue in two passes per chunk of kEpiTok activation
  // rows. Pass 1 (thread <-> weight row = TMEM lane): accumulator -> bf16 rounding +
  // bias (GEMM1: SwiGLU of the gate/up lane pair, the two lanes splitting the rows)
  // into shared memory, and the accumulator goes back to the MMA right after its last
  // load. Pass 2 regroups by activation row: GEMM1 quantises each 32-feature group in a
  // team of 4 lanes (8 features each, one 8-byte store); GEMM2 scales 8 outputs by the
  // routing weight and adds them with one 16-byte bf16x2 reduction.
  const int wrow_i = nt * C::kWgtRows + 32 * q + lane;    // weight row
  const bool vcol = wrow_i < p.N;
  const float bsv = vcol ? p.bias[static_cast<int64_t>(e) * p.N + wrow_i] : 0.0f;
  const int a_end = min(m_e, ch * C::kActRows + C::kActRows);
  const int etid = static_cast<int>(threadIdx.x) - 64;   // 0..127
#pragma unroll 1
  for (int c = 0; c < C::kColChunks; ++c) {
    const int a0 = ch * C::kActRows + c * kEpiTok;        // first row inside expert
    const bool live = a0 < a_end;                         // uniform over the CTA
    const int nv = min(kEpiTok, a_end - a0);
    float* sh = epi_f + ((local * C::kColChunks + c) % kEpiBufs) * (kEpiBufBytes / 4);
    if (live) {
      float v[kEpiTok];   // accumulator column j (the two issuers' partial sums added)
      __syncwarp();
      if constexpr (kEpiTok == 16) {
        static_assert(kEpiTok != 16 || C::kAccCols == 16, "16-row chunks fill one partial accumulator");
        uint32_t r[32];   // partial accumulators of both issuers are adjacent: one load
        tmem_ld_32x32b_x32(t_acc, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j)
          v[j] = has_b ? __fadd_rn(__uint_as_float(r[j]), __uint_as_float(r[16 + j])) : __uint_as_float(r[j]);
      } else {
        uint32_t r[32], r2[32];
        tmem_ld_32x32b_x32(t_acc + c * 32, r);
        if (has_b) tmem_ld_32x32b_x32(t_acc + C::kAccCols + c * 32, r2);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j)
          v[j] = has_b ? __fadd_rn(__uint_as_float(r[j]), __uint_as_float(r2[j])) : __uint_as_float(r[j]);
      }
      if (c == C::kColChunks - 1 || a0 + kEpiTok >= a_end) {   // last load of this tile
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acce_bar_b);
      }
      if constexpr (EPI == kEpiGemm1) {
        // lanes (2f, 2f+1) hold gate / up of feature f: the even lane finishes rows
        // [0, kHalf), the odd lane rows [kHalf, kEpiTok), one exchange per row pair
        constexpr int kHalf = kEpiTok / 2;
        const bool odd = (lane & 1) != 0;
        const int fl = (32 * q + lane) >> 1;
#pragma unroll
        for (int j = 0; j < kHalf; ++j) {
          const float vlo = __fadd_rn(bf16_round(v[j]), bsv);
          const float vhi = __fadd_rn(bf16_round(v[kHalf + j]), bsv);
          const float other = __shfl_xor_sync(0xffffffffu, odd ? vlo : vhi, 1);
          const float h = odd ? swiglu_pair(other, vhi, p.swiglu_alpha, p.swiglu_limit)
                              : swiglu_pair(vlo, other, p.swiglu_alpha, p.swiglu_limit);
          sh[(odd ? kHalf + j : j) * kEpiFeat + fl] = h;
        }
      } else {
        const int fl = 32 * q + lane;
#pragma unroll
        for (int j = 0; j < kEpiTok; ++j) sh[j * kEpiFeat + fl] = __fadd_rn(bf16_round(v[j]), bsv);
      }
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (live) {
      if constexpr (EPI == kEpiGemm1) {
        constexpr int kGroups = kEpiFeat / 32;                // quantisation groups per row
        uint8_t* codes_out = static_cast<uint8_t*>(p.out);
        uint8_t* sfb_e = p.out_sf + p.out_sf_offsets[e];
#pragma unroll 1
        for (int i0 = 0; i0 < kEpiTok * kGroups * 4; i0 += 128) {
          const int idx = i0 + etid;
          const int unit = idx >> 2, sub = idx & 3;
          const int tok = unit / kGroups, grp = unit % kGroups;
          const float* src = sh + tok * kEpiFeat + grp * 32 + sub * 8;
          const float4 x0 = *reinterpret_cast<const float4*>(src);
          const float4 x1 = *reinterpret_cast<const float4*>(src + 4);
          float amax = 0.0f;
          amax = torch_max_abs(amax, x0.x); amax = torch_max_abs(amax, x0.y);
          amax = torch_max_abs(amax, x0.z); amax = torch_max_abs(amax, x0.w);
          amax = torch_max_abs(amax, x1.x); amax = torch_max_abs(amax, x1.y);
          amax = torch_max_abs(amax, x1.z); amax = torch_max_abs(amax, x1.w);
#pragma unroll
          for (int o = 1; o < 4; o <<= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, amax, o);
            amax = (ob > amax || ob != ob) ? ob : amax;
          }
          const uint32_t rb = ue8m0_rounded_bits(amax);
          const float inv = inv_scale(scale_from_bits(rb));
          const int f0 = nt * (C::kWgtRows / 2) + grp * 32 + sub * 8;   // intermediate feature
          if (tok < nv && f0 < p.out_features) {
            const uint32_t lo = static_cast<uint32_t>(cvt_e4m3x2(clamp_fp8(__fmul_rn(x0.x, inv)),
                                                                 clamp_fp8(__fmul_rn(x0.y, inv)))) |
                                (static_cast<uint32_t>(cvt_e4m3x2(clamp_fp8(__fmul_rn(x0.z, inv)),
                                                                  clamp_fp8(__fmul_rn(x0.w, inv)))) << 16);
            const uint32_t hi = static_cast<uint32_t>(cvt_e4m3x2(clamp_fp8(__fmul_rn(x1.x, inv)),
                                                                 clamp_fp8(__fmul_rn(x1.y, inv)))) |
                                (static_cast<uint32_t>(cvt_e4m3x2(clamp_fp8(__fmul_rn(x1.z, inv)),
                                                                  clamp_fp8(__fmul_rn(x1.w, inv)))) << 16);
            const int64_t grow = static_cast<int64_t>(row0) + a0 + tok;
            *reinterpret_cast<uint2*>(codes_out + grow * p.ld_out + f0) = make_uint2(lo, hi);
            if (sub == 0) {
              const int64_t srow = act_sf_row<SPREAD>(a0 + tok);
              const int g = f0 >> 5;
              sfb_e[blocked_sf_offset(srow, g, p.out_g4)] = static_cast<uint8_t>((rb >> 23) & 0xFFu);
              // the K padding groups of the row's last k-atom read as zero scales in GEMM2
              if (g == (p.out_features >> 5) - 1)
                for (int gz = p.out_features >> 5; gz < 4 * p.out_g4; ++gz)
                  sfb_e[blocked_sf_offset(srow, gz, p.out_g4)] = 0;
            }
          }
        }
      } else {
        constexpr int kSegs = kEpiFeat / 8;                   // 8-output segments per row
        __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.out);
#pragma unroll 1
        for (int i0 = 0; i0 < kEpiTok * kSegs; i0 += 128) {
          const int idx = i0 + etid;
          const int tok = idx / kSegs, seg = idx % kSegs;
          const int n0 = nt * C::kWgtRows + seg * 8;           // output feature
          if (tok < nv && n0 < p.N) {
            const int64_t grow = static_cast<int64_t>(row0) + a0 + tok;
            const int64_t tk = p.token_idx32 != nullptr ? static_cast<int64_t>(p.token_idx32[grow]) : p.token_idx[grow];
            const float wr = p.row_weights[grow];
            const float* src = sh + tok * kEpiFeat + seg * 8;
            const float4 z0 = *reinterpret_cast<const float4*>(src);
            const float4 z1 = *reinterpret_cast<const float4*>(src + 4);
            const __nv_bfloat162 v0 = __floats2bfloat162_rn(__fmul_rn(z0.x, wr), __fmul_rn(z0.y, wr));
            const __nv_bfloat162 v1 = __floats2bfloat162_rn(__fmul_rn(z0.z, wr), __fmul_rn(z0.w, wr));
            const __nv_bfloat162 v2 = __floats2bfloat162_rn(__fmul_rn(z1.x, wr), __fmul_rn(z1.y, wr));
            const __nv_bfloat162 v3 = __floats2bfloat162_rn(__fmul_rn(z1.z, wr), __fmul_rn(z1.w, wr));
            const uint4 pk4 = make_uint4(*reinterpret_cast<const uint32_t*>(&v0), *reinterpret_cast<const uint32_t*>(&v1),
                                         *reinterpret_cast<const uint32_t*>(&v2), *reinterpret_cast<const uint32_t*>(&v3));
            if (p.ep_world > 0) {   // one received row per output row: a plain store into the source's rows
              const int s = static_cast<int>(tk / p.ep_cap);
              const int64_t j = tk - static_cast<int64_t>(s) * p.ep_cap;
              __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<uint8_t*>(p.ep_peer_bases[s]) +
                                                                   p.ep_ret_off) + j * p.ld_out + n0;
              *reinterpret_cast<uint4*>(dst) = pk4;
            } else {
              asm volatile("red.global.add.noftz.v4.bf16x2 [%0], {%1,%2,%3,%4};" ::"l"(o + tk * p.ld_out + n0),
                           "r"(pk4.x), "r"(pk4.y), "r"(pk4.z), "r"(pk4.w)
                           : "memory");
            }
          }
        }
      }
    }
    // single staging buffer: the next chunk's pass 1 waits for this pass 2
    if constexpr (kEpiBufs == 1) asm volatile("bar.sync 1, 128;" ::: "memory");
  }
}

// tm_aux0 / tm_aux1: SWAP: the 32- and 16-row activation maps; PAIR: the activation and
// weight scale buffers viewed as rows of 256 bytes (512-byte chunks = 2 rows).
// NVF4: the W4A4 mode (plain epilogue only): p.num_kb counts 256-code k blocks, the
// activation scales of expert e start p.sfa_offsets[e] ROWS into p.sfa (K / 16 bytes a row,
// matmul_mxfp4_cutlass.cu:95), and a partial last k block issues only its K / 64 MMAs.
template <bool SWAP, bool SPREAD, int EPI, bool PAIR = false, bool NVF4 = false>
__global__ void __launch_bounds__(GemmConfig<SWAP, SPREAD, PAIR, NVF4>::kThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tm_act,
                    const __grid_constant__ CUtensorMap tm_aux0,
                    const __grid_constant__ CUtensorMap tm_aux1,
                    const __grid_constant__ CUtensorMap tm_wgt, const GemmParams p) {
  using C = GemmConfig<SWAP, SPREAD, PAIR, NVF4>;
  static_assert(!NVF4 || EPI == kEpiPlain, "the W4A4 mode is the plain grouped GEMM");
  // scale atoms per 128-row block along K, and those of k block kb (fewer in a partial last block)
  const int g4 = NVF4 ? (p.K >> 6) : p.num_kb;
  auto atoms_of = [&](int kb) -> int { return NVF4 ? min(C::kSfAtoms, g4 - C::kSfAtoms * kb) : 1; };
  // CTA pair: rank inside the pair, pair index and count (a plain CTA is its own "pair")
  const uint32_t prank = PAIR ? (cluster_ctarank() & 1u) : 0u;
  const int unit = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int nunits = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  const bool leader = prank == 0;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ int s_chunk_prefix[kMaxExpertsGemm + 1];
  __shared__ int s_chunks[kMaxExpertsGemm];
  // per-expert metadata read once per CTA: a global load per tile on the producer's path
  // (under a full memory system, microseconds each) would delay every tile's first stage
  __shared__ int s_msize[kMaxExpertsGemm];
  __shared__ int s_row_off[kMaxExpertsGemm];
  __shared__ long long s_sfa_base[kMaxExpertsGemm];
  __shared__ uint32_t s_tmem_base;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t bar_base = smem_base + C::kStages * C::kStageBytes;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (C::kStages + s); };
  auto accf_bar = [&](int b) { return bar_base + 8u * (2 * C::kStages + b); };
  auto acce_bar = [&](int b) { return bar_base + 8u * (2 * C::kStages + C::kAccBufs + b); };
  const uint32_t drain_bar = bar_base + 8u * (2 * C::kStages + 2 * C::kAccBufs);
  const uint32_t epi_base = bar_base + ((C::kBarrierBytes + 127u) & ~127u);   // epilogue staging

  pdl_trigger();
  // ---- barriers, TMEM and descriptor prefetch overlap the previous kernel's tail
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_act);
    if constexpr (SWAP || PAIR) {
      tma_prefetch_desc(&tm_aux0);
      tma_prefetch_desc(&tm_aux1);
    }
    tma_prefetch_desc(&tm_wgt);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), C::kIssuers);   // one commit per MMA issuer
    }
    for (int b = 0; b < C::kAccBufs; ++b) {
      mbar_init(accf_bar(b), C::kIssuers);
      mbar_init(acce_bar(b), PAIR ? 2 * C::kEpiWarps : C::kEpiWarps);   // both CTAs' epilogues
    }
    mbar_init(drain_bar, C::kIssuers);
    fence_barrier_init();
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(smem_u32(&s_tmem_base), C::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_u32(&s_tmem_base), C::kTmemCols);
      tmem_relinquish();
    }
  }
  if constexpr (SWAP) {
    // The weights do not depend on the previous kernel: while it (the routing prologue)
    // runs, pull the weight tiles this CTA will most likely stream first into L2.
    if (warp == 0 && p.prefetch_tiles > 0 && elect_one()) {
      for (int j = 0; j < p.prefetch_tiles; ++j) {
        const int t = blockIdx.x + j * gridDim.x;
        const int e = t / p.n_tiles, nt = t - e * p.n_tiles;
        if (e >= p.num_experts) break;
        for (int kb = 0; kb < p.num_kb; ++kb) tma_prefetch_3d(&tm_wgt, kb * 128, nt * C::kWgtRows, e);
        bulk_prefetch_l2(p.sfb + static_cast<int64_t>(e) * p.sfb_stride +
                             static_cast<int64_t>((nt * C::kWgtRows) >> 7) * g4 * 512,
                         static_cast<uint32_t>(g4) * 512u);
      }
    }
  }
  pdl_wait();
  // ---- per-CTA tile map from the device-side counts
  for (int i = threadIdx.x; i < p.num_experts; i += blockDim.x) {
    const int m = p.m_sizes[i * p.m_stride];
    s_chunks[i] = m > 0 ? (m + C::kTileM - 1) / C::kTileM : 0;
    s_msize[i] = m;
    s_row_off[i] = p.row_offsets[i];
    int64_t sfa_base = NVF4 ? static_cast<int64_t>(p.sfa_offsets[i]) * (p.K >> 4) : p.sfa_offsets[i];
    if (sfa_base & 15) {   // a bulk copy needs 16-byte alignment: report, then read aligned
      if (m > 0 && p.err) atomicCAS(p.err, 0, static_cast<int>(kDevMisalignedScales));
      sfa_base &= ~static_cast<int64_t>(15);
    }
    s_sfa_base[i] = sfa_base;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < p.num_experts; ++e) { s_chunk_prefix[e] = acc; acc += s_chunks[e]; }
    s_chunk_prefix[p.num_experts] = acc;
  }
  __syncthreads();
  // barriers initialised and TMEM allocated in both CTAs before any cross-CTA signal
  if constexpr (PAIR) cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = s_tmem_base;
  const int total_tiles = s_chunk_prefix[p.num_experts] * p.n_tiles;

  // Activation rows a tile loads and multiplies: SWAP tiles load only 16 or 32 rows when
  // the chunk holds that few (the MMA N follows); the chunk still starts on a 64-row
  // boundary, so the scale TMEM shift stays 0 or 2 columns.
  auto act_rows_of = [&](int e, int ch) -> int {
    if constexpr (!SWAP || SPREAD) {
      return C::kActRows;
    } else {
      const int left = s_msize[e] - ch * C::kActRows;
      return left <= 16 ? 16 : (left <= 32 ? 32 : C::kActRows);
    }
  };

  // tile t -> (expert, weight tile, activation chunk)
  auto decode = [&](int t, int& e, int& nt, int& ch) {
    const int cidx = t / p.n_tiles;           // global chunk-major index
    int lo = 0, hi = p.num_experts - 1;
    while (lo < hi) {                         // last e with prefix[e] <= cidx
      const int mid = (lo + hi + 1) >> 1;
      if (s_chunk_prefix[mid] <= cidx) lo = mid; else hi = mid - 1;
    }
    e = lo;
    const int local = t - s_chunk_prefix[e] * p.n_tiles;
    const int nch = s_chunks[e];
    nt = local / nch;
    ch = local - nt * nch;
  };

  if (warp == 0) {
    // ================================================================ producer
    if (elect_one()) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_a = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = unit; t < total_tiles && ok; t += nunits) {
        int e, nt, ch;
        decode(t, e, nt, ch);
        // this CTA's activation rows (PAIR: its 128-row half of the 256-row tile) and the
        // weight rows it loads (PAIR: its 96-row half of the 192-row tile)
        const int act_in0 = ch * C::kTileM + static_cast<int>(prank) * C::kActRows;
        const int act_row0 = s_row_off[e] + act_in0;
        const int wgt_row0 = nt * C::kWgtRows + static_cast<int>(prank) * C::kWgtRowsCta;
        const int act_blk = static_cast<int>(act_sf_row<SPREAD>(static_cast<int64_t>(act_in0)) >> 7);
        const int64_t sfa_off = s_sfa_base[e] + static_cast<int64_t>(act_blk) * g4 * 512;
        const int wblk0 = (nt * C::kWgtRows) >> 7;   // scale blocks of the whole tile
        const int nwblk_total = (p.N + 127) >> 7;
        const int nwchunks = min(C::kWgtSfChunks, nwblk_total - wblk0);
        const int64_t sfb_off = static_cast<int64_t>(e) * p.sfb_stride + static_cast<int64_t>(wblk0) * g4 * 512;
        const int arows = act_rows_of(e, ch);
        const CUtensorMap* amap = arows == 16 ? &tm_aux1 : (arows == 32 ? &tm_aux0 : &tm_act);
        const uint32_t tx_fixed = arows * 128u + C::kWgtRowsCta * C::kWgtRowGlobalBytes;
        for (int kb0 = 0; kb0 < p.num_kb; kb0 += C::kSubs) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.err, kDevTimeoutProducer)) { ok = false; break; }
          const int nsub = min(C::kSubs, p.num_kb - kb0);
          uint32_t tx = 0;
          for (int j = 0; j < nsub; ++j)
            tx += (tx_fixed + 512u * static_cast<uint32_t>(atoms_of(kb0 + j) * (1 + nwchunks))) * (PAIR ? 2u : 1u);
          if (leader) mbar_arrive_expect_tx(full_bar(stage), tx);
          for (int j = 0; j < nsub; ++j) {
            const int kb = kb0 + j;
            const uint32_t sb = smem_base + stage * C::kStageBytes + j * C::kSubBytes;
            const uint32_t s_w = sb, s_a = sb + C::kWgtTileBytes;
            const uint32_t s_sfa = s_a + C::kActTileBytes, s_sfw = s_sfa + C::kSfActBytes;
            if constexpr (PAIR) {
              // every load of both CTAs completes on the even CTA's full barrier
              const uint32_t fb = dsmem_map(full_bar(stage), 0);
              tma_load_2d_pair(s_a, &tm_act, fb, kb * 128, act_row0, pol_a);
              tma_load_3d_pair(s_w, &tm_wgt, fb, kb * 128, wgt_row0, e, pol_w);
              tma_load_2d_pair(s_sfa, &tm_aux0, fb, 0, static_cast<int32_t>((sfa_off + kb * 512) >> 8), pol_a);
              for (int c = 0; c < nwchunks; ++c)
                tma_load_2d_pair(s_sfw + 512u * c, &tm_aux1, fb, 0,
                                 static_cast<int32_t>((sfb_off + static_cast<int64_t>(c) * p.num_kb * 512 + kb * 512) >> 8),
                                 pol_w);
            } else {
              // x = 128 smem bytes per k block either way: 128 fp8 codes / 128 E2M1 codes
              // expanded by the TMA (W4A8), or 128 packed bytes (W4A4)
              // this k block's atoms: kSfAtoms * 512 bytes into each 128-row block's scales
              const uint32_t sf_bytes = 512u * static_cast<uint32_t>(atoms_of(kb));
              const int64_t kb_sf = static_cast<int64_t>(kb) * C::kSfAtoms * 512;
              tma_load_2d(s_a, amap, full_bar(stage), kb * 128, act_row0, pol_a);
              tma_load_3d(s_w, &tm_wgt, full_bar(stage), kb * 128, wgt_row0, e, pol_w);
              bulk_load(s_sfa, p.sfa + sfa_off + kb_sf, sf_bytes, full_bar(stage), pol_a);
              for (int c = 0; c < nwchunks; ++c)
                bulk_load(s_sfw + 512u * C::kSfAtoms * c, p.sfb + sfb_off + static_cast<int64_t>(c) * g4 * 512 + kb_sf,
                          sf_bytes, full_bar(stage), pol_w);
            }
          }
          if (++stage == C::kStages) { stage = 0; phase ^= 1u; }
        }
      }
      // Drain: make sure no copy is still landing in shared memory before exit (in a pair
      // the even CTA's barriers count both CTAs' copies; the odd CTA is held by the
      // closing cluster barrier until then).
      if (leader) {
        for (int s = 0; s < C::kStages; ++s) {
          // Stage s last received the load of phase (phase if s < stage else phase ^ 1).
          const uint32_t ph = (s < stage) ? phase : (phase ^ 1u);
          (void)mbar_wait(full_bar(s), ph, p.err, kDevTimeoutDrain);
        }
      }
    }
  } else if (warp == 1 || (C::kIssuers > 1 && warp == 2 + C::kEpiWarps)) {
    // ================================================================ MMA issuer(s)
    // issuer i takes the k blocks j of each stage with j % kIssuers == i
    const int issuer = warp == 1 ? 0 : 1;
    if (elect_one() && !(PAIR && !leader)) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = unit; t < total_tiles && ok; t += nunits, ++local) {
        int e, nt, ch;
        decode(t, e, nt, ch);
        const int b = local % C::kAccBufs;
        const uint32_t acc_phase = static_cast<uint32_t>(local / C::kAccBufs) & 1u;
        if (!mbar_wait(acce_bar(b), acc_phase ^ 1u, p.err, kDevTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * C::kAccStride + issuer * C::kAccCols;
        // Column shift selecting the 32-row groups this tile starts at inside the
        // copied 128-row scale blocks.
        const uint32_t wshift = SWAP ? 0u : static_cast<uint32_t>(((nt * C::kWgtRows) & 127) >> 5);
        const uint32_t ashift =
            SWAP ? static_cast<uint32_t>((act_sf_row<SPREAD>(static_cast<int64_t>(ch) * C::kActRows) & 127) >> 5) : 0u;
        const uint32_t t_sfa = tmem_base + C::kSfActCol + issuer * C::kSfCols;
        const uint32_t t_sfw = tmem_base + C::kSfWgtCol + issuer * C::kSfCols;
        const uint32_t mma_n = SWAP ? static_cast<uint32_t>(act_rows_of(e, ch)) : static_cast<uint32_t>(C::kMmaN);
        // The issue loop is lean on purpose (small-N block-scaled MMAs cost ~75 cycles of
        // issue each): descriptors and the instruction word are formed once per tile /
        // stage and advanced by adds (a 32-byte K step is +2 in the descriptor's 16-byte
        // address field).
        const uint32_t idesc0 = NVF4 ? idesc_mxf4nvf4(C::kMmaM, mma_n)
                                : SWAP ? idesc_mxf8f6f4(5, 0, C::kMmaM, mma_n, 0, 0)
                                       : idesc_mxf8f6f4(0, 5, C::kMmaM, mma_n, 0, 0);
        const uint32_t sf_a_t = SWAP ? t_sfw : t_sfa;                       // scales of MMA operand A
        const uint32_t sf_b_t = SWAP ? t_sfa + ashift : t_sfw + wshift;     // scales of MMA operand B
        for (int kb0 = 0; kb0 < p.num_kb; kb0 += C::kSubs) {
          if (!mbar_wait(full_bar(stage), phase, p.err, kDevTimeoutMma)) { ok = false; break; }
          tc_fence_after();
          const int nsub = min(C::kSubs, p.num_kb - kb0);
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
            if constexpr (NVF4) {
              // atom a of the activation scales -> columns 4a; of weight chunk c -> 4 (chunks a + c)
              const int na = atoms_of(kb0 + j);
              for (int a = 0; a < na; ++a) {
                tc_cp_32x128b_warpx4(t_sfa + 4u * a, dsa0 + joff + 32u * a);
#pragma unroll
                for (int c = 0; c < C::kWgtSfChunks; ++c)
                  tc_cp_32x128b_warpx4(t_sfw + 4u * (C::kWgtSfChunks * a + c), dsw0 + joff + 32u * (C::kSfAtoms * c + a));
              }
              const uint64_t dw = dw0 + joff, da = da0 + joff;
              const uint64_t dA = SWAP ? dw : da, dB = SWAP ? da : dw;
              for (int k = 0; k < na; ++k) {
                const uint32_t sfa_k = t_sfa + 4u * k, sfw_k = t_sfw + 4u * C::kWgtSfChunks * k;
                const uint32_t acc = (kb0 != 0 || j >= C::kIssuers || k != 0) ? 1u : 0u;
                // a 64-code (32-byte) K step is +2 in the descriptor's 16-byte address field
                mma_mxf4nvf4(d_tmem, dA + 2u * k, dB + 2u * k, idesc0, SWAP ? sfw_k : sfa_k,
                             SWAP ? sfa_k + ashift : sfw_k + wshift, acc);
              }
              continue;
            }
            if constexpr (PAIR) {
              // each CTA's scale chunks go from its own shared memory into its own TMEM
              tc_cp_32x128b_warpx4_pair(t_sfa, dsa0 + joff);
#pragma unroll
              for (int c = 0; c < C::kWgtSfChunks; ++c) tc_cp_32x128b_warpx4_pair(t_sfw + 4u * c, dsw0 + joff + 32u * c);
            } else {
              tc_cp_32x128b_warpx4(t_sfa, dsa0 + joff);
#pragma unroll
              for (int c = 0; c < C::kWgtSfChunks; ++c) tc_cp_32x128b_warpx4(t_sfw + 4u * c, dsw0 + joff + 32u * c);
            }
            const uint64_t dw = dw0 + joff, da = da0 + joff;
            // operand A / B descriptors: weights are A in SWAP tiles, activations otherwise
            const uint64_t dA = SWAP ? dw : da, dB = SWAP ? da : dw;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint32_t idesc = idesc0 | (static_cast<uint32_t>(k) << 4) | (static_cast<uint32_t>(k) << 29);
              // the first MMA of each issuer in a tile starts its partial accumulator
              const uint32_t acc = (kb0 != 0 || j >= C::kIssuers || k != 0) ? 1u : 0u;
              if constexpr (PAIR) {
                mma_mxf8f6f4_pair(d_tmem, dA + 2u * k, dB + 2u * k, idesc, sf_a_t, sf_b_t, acc);
              } else {
                mma_mxf8f6f4(d_tmem, dA + 2u * k, dB + 2u * k, idesc, sf_a_t, sf_b_t, acc);
              }
            }
          }
          if constexpr (PAIR) tc_commit_pair(empty_bar(stage), 0x3);   // both CTAs' producers
          else tc_commit(empty_bar(stage));
          if (++stage == C::kStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        if constexpr (PAIR) tc_commit_pair(accf_bar(b), 0x3);   // both CTAs' epilogues
        else tc_commit(accf_bar(b));
      }
      // Wait for every tcgen05 operation the issuers issued before TMEM is released.
      if constexpr (PAIR) tc_commit_pair(drain_bar, 0x3);
      else tc_commit(drain_bar);
      (void)mbar_wait(drain_bar, 0u, p.err, kDevTimeoutDrain);
    } else if (PAIR && !leader && elect_one()) {
      // odd CTA of a pair: its TMEM is written by the even CTA's MMAs; wait for them
      (void)mbar_wait(drain_bar, 0u, p.err, kDevTimeoutDrain);
    }
  } else {
    // ================================================================ epilogue
    // staging of the weights-on-M GEMM1 / GEMM2 epilogue: kEpiTok activation rows x kEpiFeat
    // fp32 values per buffer, double-buffered when two fit
    constexpr int kEpiTok = C::kActRows < 32 ? C::kActRows : 32;
    constexpr int kEpiFeat = EPI == kEpiGemm1 ? C::kWgtRows / 2 : C::kWgtRows;
    constexpr uint32_t kEpiBufBytes = static_cast<uint32_t>(kEpiTok * kEpiFeat * 4);
    constexpr int kEpiBufs = 2 * kEpiBufBytes <= C::kEpiStageBytes ? 2 : 1;
    static_assert(!SWAP || EPI == kEpiPlain || kEpiBufBytes <= C::kEpiStageBytes, "epilogue staging too small");
    float* const epi_f = reinterpret_cast<float*>(smem_raw + (epi_base - smem_u32(smem_raw)));
    // the second issuer's partial accumulator holds something once a tile has 2 k blocks
    const bool has_b = C::kIssuers > 1 && p.num_kb > 1;
    const int q = warp & 3;                 // TMEM lane quarter of this warp
    const int wg = (warp - 2) >> 2;         // epilogue warpgroup
    constexpr int kWgs = C::kEpiWarps / 4;
    int local = 0;
    bool ok = true;   // after a timeout keep walking the tiles (named barriers stay
                      // matched across the four warps) but touch no TMEM or memory
    for (int t = unit; t < total_tiles; t += nunits, ++local) {
      int e, nt, ch;
      decode(t, e, nt, ch);
      const int b = local % C::kAccBufs;
      const uint32_t acc_phase = static_cast<uint32_t>(local / C::kAccBufs) & 1u;
      if (ok) ok = mbar_wait(accf_bar(b), acc_phase, p.err, kDevTimeoutEpilogue);
      if (!ok) {
        if constexpr (SWAP && EPI != kEpiPlain) {
          for (int c = 0; c < C::kColChunks * (kEpiBufs == 1 ? 2 : 1); ++c) asm volatile("bar.sync 1, 128;" ::: "memory");
        }
        continue;
      }
      tc_fence_after();
      const uint32_t t_acc = tmem_base + (static_cast<uint32_t>(32 * q) << 16) + b * C::kAccStride;
      const int m_e = s_msize[e];
      const int row0 = s_row_off[e];
      if constexpr (!SWAP) {
        // thread <-> activation row
        const int r_in = ch * C::kTileM + static_cast<int>(prank) * C::kActRows + 32 * q + lane;   // row in expert
        const bool vrow = r_in < m_e;
        const int64_t grow = static_cast<int64_t>(row0) + r_in;
        const int n_tile0 = nt * C::kWgtRows;
        if constexpr (EPI == kEpiGemm1) {
#pragma unroll 1
          for (int gi = wg; gi < C::kWgtRows / 64; gi += kWgs) {
            float h[32];
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              uint32_t r[32];
              __syncwarp();
              tmem_ld_32x32b_x32(t_acc + (2 * gi + half) * 32, r);
              const int nb = n_tile0 + (2 * gi + half) * 32;
              float bsv[32];
              load_bias32(p.bias + static_cast<int64_t>(e) * p.N + nb, p.N - nb, bsv);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const float g = __fadd_rn(bf16_round(__uint_as_float(r[2 * j])), bsv[2 * j]);
                const float u = __fadd_rn(bf16_round(__uint_as_float(r[2 * j + 1])), bsv[2 * j + 1]);
                h[half * 16 + j] = swiglu_pair(g, u, p.swiglu_alpha, p.swiglu_limit);
              }
            }
            const int f0 = (n_tile0 >> 1) + 32 * gi;   // first intermediate feature
            if (vrow && f0 < p.out_features) {
              uint32_t codes[8];
              const uint8_t s = quantize_group32(h, codes);
              uint4* o = reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.out) + grow * p.ld_out + f0);
              o[0] = make_uint4(codes[0], codes[1], codes[2], codes[3]);
              o[1] = make_uint4(codes[4], codes[5], codes[6], codes[7]);
              uint8_t* sfb_e = p.out_sf + p.out_sf_offsets[e];
              sfb_e[blocked_sf_offset(r_in, f0 >> 5, p.out_g4)] = s;
              // the K padding groups of the row's last k-atom read as zero scales in GEMM2
              if ((f0 >> 5) == (p.out_features >> 5) - 1)
                for (int gz = p.out_features >> 5; gz < 4 * p.out_g4; ++gz)
                  sfb_e[blocked_sf_offset(r_in, gz, p.out_g4)] = 0;
            }
          }
        } else {
          float alpha = 1.0f, wrow = 0.0f;
          int64_t tok = 0;
          if constexpr (EPI == kEpiPlain) alpha = p.alphas ? p.alphas[e] : 1.0f;
          if constexpr (EPI == kEpiGemm2) {
            if (vrow) { tok = p.token_idx[grow]; wrow = p.row_weights[grow]; }
          }
#pragma unroll 1
          for (int c = wg; c < C::kWgtRows / 32; c += kWgs) {
            uint32_t r[32];
            __syncwarp();
            tmem_ld_32x32b_x32(t_acc + c * 32, r);
            tmem_ld_wait();
            const int nb = n_tile0 + c * 32;
            if (vrow && nb < p.N) {
            const bool full = nb + 32 <= p.N;
            if constexpr (EPI == kEpiPlain) {
              __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.out) + grow * p.ld_out + nb;
              if (full) {
                uint32_t pk[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  const __nv_bfloat162 v2 = __floats2bfloat162_rn(__fmul_rn(alpha, __uint_as_float(r[2 * j])),
                                                                  __fmul_rn(alpha, __uint_as_float(r[2 * j + 1])));
                  pk[j] = *reinterpret_cast<const uint32_t*>(&v2);
                }
                uint4* o4 = reinterpret_cast<uint4*>(o);
#pragma unroll
                for (int j = 0; j < 4; ++j) o4[j] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
              } else {
                // unrolled with a predicate: a runtime loop bound would index r[] dynamically
                // and put the whole array in local memory for every tile
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (nb + j < p.N) o[j] = __float2bfloat16_rn(__fmul_rn(alpha, __uint_as_float(r[j])));
              }
            } else {  // kEpiGemm2
              float bsv[32];
              load_bias32(p.bias + static_cast<int64_t>(e) * p.N + nb, p.N - nb, bsv);
              __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.out) + tok * p.ld_out + nb;
              uint32_t pk[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const float y0 = __fmul_rn(__fadd_rn(bf16_round(__uint_as_float(r[2 * j])), bsv[2 * j]), wrow);
                const float y1 = __fmul_rn(__fadd_rn(bf16_round(__uint_as_float(r[2 * j + 1])), bsv[2 * j + 1]), wrow);
                const __nv_bfloat162 v2 = __floats2bfloat162_rn(y0, y1);
                pk[j] = *reinterpret_cast<const uint32_t*>(&v2);
              }
              if (full) {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                  asm volatile("red.global.add.noftz.v4.bf16x2 [%0], {%1,%2,%3,%4};" ::"l"(o + 8 * j),
                               "r"(pk[4 * j]), "r"(pk[4 * j + 1]), "r"(pk[4 * j + 2]), "r"(pk[4 * j + 3])
                               : "memory");
              } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) {   // unrolled with a predicate, as above (pk[])
                  if (nb + 2 * j < p.N) {
                    const __nv_bfloat162 v2 = *reinterpret_cast<const __nv_bfloat162*>(&pk[j]);
                    if (nb + 2 * j + 1 < p.N) {
                      atomicAdd(reinterpret_cast<__nv_bfloat162*>(o + 2 * j), v2);
                    } else {
                      atomicAdd(o + 2 * j, v2.x);
                    }
                  }
                }
              }
            }
            }  // vrow && nb < N
          }
        }
      } else if constexpr (EPI == kEpiPlain) {
        // thread <-> weight row (output feature); column j = activation row ch*64 + j,
        // walked in two 32-column halves.
        const int wrow_i = nt * C::kWgtRows + 32 * q + lane;    // weight row / feature
        const bool vcol = wrow_i < p.N;
#pragma unroll 1
        for (int c = 0; c < C::kColChunks; ++c) {
          const int a0 = ch * C::kActRows + c * 32;             // first row inside expert
          const int a_end = min(m_e, ch * C::kActRows + C::kActRows);
          const bool live = a0 < a_end;                         // uniform over the CTA
          uint32_t r[32];
          if (live) {
            __syncwarp();
            tmem_ld_32x32b_x32(t_acc + c * 32, r);
            if (has_b) {
              uint32_t r2[32];
              tmem_ld_32x32b_x32(t_acc + C::kAccCols + c * 32, r2);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__fadd_rn(__uint_as_float(r[j]), __uint_as_float(r2[j])));
            } else {
              tmem_ld_wait();
            }
          }
          {
            if (live) {
              const float alpha = p.alphas ? p.alphas[e] : 1.0f;
              __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.out);
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (vcol && a0 + j < a_end)
                  o[(static_cast<int64_t>(row0) + a0 + j) * p.ld_out + wrow_i] =
                      __float2bfloat16_rn(__fmul_rn(alpha, __uint_as_float(r[j])));
              }
            }
          }
        }
      } else {
        swap_epilogue_tile<SPREAD, EPI>(p, t_acc, acce_bar(b), e, nt, ch, m_e, row0, local, epi_f, has_b, q, lane);
        continue;   // the accumulator went back to the MMA after its last load
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR) mbar_arrive_cluster(dsmem_map(acce_bar(b), 0));   // the even CTA's MMA
        else mbar_arrive(acce_bar(b));
      }
    }
  }

  // A pair stays alive until both CTAs are done: the even CTA's MMAs write the odd CTA's
  // TMEM and the odd CTA's epilogue arrives on the even CTA's barriers.
  if constexpr (PAIR) cluster_sync();
  else __syncthreads();
  if constexpr (EPI == kEpiGemm2 && SWAP) {
    // every epilogue store of this CTA is behind the barrier: publish them (one fence per
    // CTA, then the last CTA raises the return flags)
    if (p.ep_world > 0 && threadIdx.x < 32)
      p2p_last_cta_signal(p.ep_counter, p.ep_peer_bases, p.ep_world, p.ep_world + p.ep_rank, p.ep_epoch);
  }
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, C::kTmemCols);
    else tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

}  // namespace gptoss
