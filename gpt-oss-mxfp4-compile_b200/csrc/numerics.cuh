// Device numerics shared by the quantiser, the router and the GEMM epilogues.
//
// quantize_group32 restates kernels/cutlass_experts.py:197-251
// (quantize_activations_to_fp8) operation by operation so the FP8 codes and UE8M0
// scales are bit-identical to the reference's eager PyTorch result:
//   amax  = max |x|                     (fp32, NaN propagates like torch.max)
//   ds    = amax / 448                  (IEEE round-to-nearest division)
//   r     = (bits(ds) + 0x7FFFFF) & 0x7F800000   (round the scale up to a power of 2)
//   scale = r == 0 ? 2^-126 : float(r)
//   code  = e4m3(clamp(x / scale, -448, 448))    (round-to-nearest-even)
//   ue8m0 = r >> 23
// swiglu restates cutlass_experts.py:258-276 (clamp, sigmoid(1.702 g), (up + 1)).
#pragma once
#include <cstdint>
#include <cuda_bf16.h>

namespace gptoss {

constexpr float kFp8Max = 448.0f;

// Byte offset of scale factor (row r, k-group g) inside one expert's blocked scale
// buffer: 128-row x 4-group atoms of 512 bytes, k-atoms innermost. This is the layout of
// CUTLASS's Sm1xxBlockScaledConfig<32>::tile_atom_to_shape_SFA/SFB (checked offset by
// offset against CuTe), which is also the smem image tcgen05.cp 32x128b.warpx4 expects.
__host__ __device__ __forceinline__ int64_t blocked_sf_offset(int64_t r, int g, int g4) {
  return (r >> 7) * (static_cast<int64_t>(g4) << 9) + ((g >> 2) << 9) + ((r & 31) << 4) +
         (((r & 127) >> 5) << 2) + (g & 3);
}

// Bytes of one blocked scale buffer holding `rows` rows and ceil(groups/4) k-atoms.
__host__ __device__ __forceinline__ int64_t blocked_sf_cosize(int64_t rows, int groups) {
  return ((rows + 127) / 128) * static_cast<int64_t>((groups + 3) / 4) * 512;
}

// Activation scale rows. SPREAD places real row r at scale row 64*(r/16) + r%16, so every
// 16-row chunk starts at scale row 0 or 64 of a 128-row block: its scales sit at a TMEM
// column offset of 0 or 2 (the even offsets CUTLASS uses for N=64 / N=192 tiles).
template <bool SPREAD>
__host__ __device__ __forceinline__ int64_t act_sf_row(int64_t r) {
  if constexpr (SPREAD) return ((r >> 4) << 6) + (r & 15);
  else return r;
}

// Scale rows (padded to 128) one expert of m rows occupies.
__host__ __device__ __forceinline__ int64_t act_sf_rows(int64_t m, bool spread) {
  const int64_t rows = spread ? ((m + 15) / 16) * 64 : m;
  return (rows + 127) / 128 * 128;
}

// Bytes of one expert's activation scale region for m rows.
__host__ __device__ __forceinline__ int64_t act_sf_cosize(int64_t m, int groups, bool spread) {
  return m > 0 ? act_sf_rows(m, spread) / 128 * static_cast<int64_t>((groups + 3) / 4) * 512 : 0;
}

__device__ __forceinline__ float torch_max_abs(float m, float x) {
  // torch.max propagates NaN; fmaxf would drop it.
  const float a = fabsf(x);
  return (a > m || a != a) ? a : m;
}

__device__ __forceinline__ uint32_t ue8m0_rounded_bits(float amax) {
  const float ds = __fdiv_rn(amax, kFp8Max);
  return (__float_as_uint(ds) + 0x007FFFFFu) & 0x7F800000u;
}

__device__ __forceinline__ float scale_from_bits(uint32_t rbits) {
  return rbits == 0u ? 1.1754944e-38f : __uint_as_float(rbits);
}

// 1 / scale for a power-of-two scale in [2^-126, 2^127]. The reciprocal is exact
// (2^-127 is a subnormal, still exact), so x * inv equals the reference's x / scale
// bit for bit, including results that round into the subnormal range.
__device__ __forceinline__ float inv_scale(float scale) { return __frcp_rn(scale); }

__device__ __forceinline__ float clamp_fp8(float v) {
  // torch.clamp keeps NaN: the .NaN forms of max / min return NaN when an input is NaN.
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(v), "f"(-kFp8Max));
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(r), "f"(kFp8Max));
  return r;
}

// Two floats -> two e4m3 bytes, round-to-nearest-even (low byte = lo).
__device__ __forceinline__ uint16_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// Quantise 32 fp32 values; writes 32 codes into out[0..7] (little-endian bytes) and
// returns the UE8M0 scale byte.
__device__ __forceinline__ uint8_t quantize_group32(const float (&x)[32], uint32_t (&out)[8]) {
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = torch_max_abs(amax, x[i]);
  const uint32_t rb = ue8m0_rounded_bits(amax);
  const float inv = inv_scale(scale_from_bits(rb));
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float a = clamp_fp8(__fmul_rn(x[4 * i + 0], inv));
    const float b = clamp_fp8(__fmul_rn(x[4 * i + 1], inv));
    const float c = clamp_fp8(__fmul_rn(x[4 * i + 2], inv));
    const float d = clamp_fp8(__fmul_rn(x[4 * i + 3], inv));
    out[i] = static_cast<uint32_t>(cvt_e4m3x2(a, b)) | (static_cast<uint32_t>(cvt_e4m3x2(c, d)) << 16);
  }
  return static_cast<uint8_t>((rb >> 23) & 0xFFu);
}

// SwiGLU on one (gate, up) pair, fp32, same operation order as the reference.
__device__ __forceinline__ float swiglu_pair(float gate, float up, float alpha, float limit) {
  gate = gate > limit ? limit : gate;                       // clamp(max=limit)
  up = up < -limit ? -limit : (up > limit ? limit : up);    // clamp(-limit, limit)
  // 1 / (1 + e): a correctly rounded reciprocal equals the IEEE quotient 1.0f / y.
  const float sig = __frcp_rn(__fadd_rn(1.0f, expf(-__fmul_rn(gate, alpha))));
  return __fmul_rn(__fmul_rn(gate, sig), __fadd_rn(up, 1.0f));
}

__device__ __forceinline__ float bf16_bits_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_bits_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

}  // namespace gptoss
