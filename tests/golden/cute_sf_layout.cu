// Dumps CuTe's blocked scale-factor layout (CUTLASS Sm1xxBlockScaledConfig<VEC>, the
// layout the reference builds its scale buffers with, kernels/matmul_mxfp4_cutlass.cu:
// 716-746 for VEC = 32; the NVFP4 mode's ScaleConfig, :200-260, for VEC = 16) for a few
// shapes, so the closed form used by the oracle and the kernels is pinned to CuTe itself.
// Host-only; build and run in a container that has the CUTLASS headers:
//   nvcc -std=c++17 -I<cutlass>/include -x cu cute_sf_layout.cu -o /tmp/cute_sf
//   /tmp/cute_sf 32 > cute_sf_layout.txt
//   /tmp/cute_sf 16 > cute_sf_layout16.txt
// Output: one line per shape "rows K cosize_sfa cosize_sfb" followed by the SFA offsets of
// every (row, k-group) in row-major order (K / VEC groups per row).
#include <cstdio>
#include <cstdlib>
#include <cute/tensor.hpp>
#include <cutlass/detail/sm100_blockscaled_layout.hpp>

template <int VEC>
void dump() {
  using Cfg = cutlass::detail::Sm1xxBlockScaledConfig<VEC>;
  const int shapes32[][2] = {{1, 256}, {64, 256}, {129, 384}, {200, 2944}, {5, 2880}};
  const int shapes16[][2] = {{1, 64}, {64, 256}, {129, 512}, {200, 640}, {5, 320}};
  for (int i = 0; i < 5; ++i) {
    const int rows = VEC == 16 ? shapes16[i][0] : shapes32[i][0];
    const int K = VEC == 16 ? shapes16[i][1] : shapes32[i][1];
    auto la = Cfg::tile_atom_to_shape_SFA(cute::make_shape(rows, 128, K, 1));
    auto lb = Cfg::tile_atom_to_shape_SFB(cute::make_shape(128, rows, K, 1));
    std::printf("%d %d %ld %ld\n", rows, K, (long)cute::cosize(la), (long)cute::cosize(lb));
    for (int r = 0; r < rows; ++r) {
      for (int g = 0; g < K / VEC; ++g) std::printf("%ld ", (long)la(r, g * VEC, 0));
      std::printf("\n");
    }
  }
}

int main(int argc, char** argv) {
  const int vec = argc > 1 ? std::atoi(argv[1]) : 32;
  if (vec == 16) dump<16>();
  else dump<32>();
  return 0;
}
