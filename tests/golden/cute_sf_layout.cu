// Dumps CuTe's blocked scale-factor layout (CUTLASS Sm1xxBlockScaledConfig<32>, the
// layout the reference builds its scale buffers with, kernels/matmul_mxfp4_cutlass.cu:
// 716-746) for a few shapes, so the closed form used by the oracle and the kernels is
// pinned to CuTe itself. Host-only; build and run in a container that has the CUTLASS
// headers:
//   nvcc -std=c++17 -I<cutlass>/include -x cu cute_sf_layout.cu -o /tmp/cute_sf && /tmp/cute_sf > cute_sf_layout.txt
// Output: one line per shape "rows K cosize_sfa cosize_sfb" followed by the SFA offsets of
// every (row, k-group) in row-major order.
#include <cstdio>
#include <cute/tensor.hpp>
#include <cutlass/detail/sm100_blockscaled_layout.hpp>

int main() {
  using Cfg = cutlass::detail::Sm1xxBlockScaledConfig<32>;
  const int shapes[][2] = {{1, 256}, {64, 256}, {129, 384}, {200, 2944}, {5, 2880}};
  for (const auto& s : shapes) {
    const int rows = s[0], K = s[1];
    auto la = Cfg::tile_atom_to_shape_SFA(cute::make_shape(rows, 128, K, 1));
    auto lb = Cfg::tile_atom_to_shape_SFB(cute::make_shape(128, rows, K, 1));
    std::printf("%d %d %ld %ld\n", rows, K, (long)cute::cosize(la), (long)cute::cosize(lb));
    for (int r = 0; r < rows; ++r) {
      for (int g = 0; g < K / 32; ++g) std::printf("%ld ", (long)la(r, g * 32, 0));
      std::printf("\n");
    }
  }
  return 0;
}
