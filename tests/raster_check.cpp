// Host check of the persistent GEMM's tile order (welvet.metal_b200/csrc/
// gemm_raster.cuh, the function the kernel calls, compiled here for the CPU): for
// every grid of up to 96 x 96 tiles and every panel width gn, the tile indices
// cover each output tile exactly once, and each panel's N-tiles are consecutive.
// Test infrastructure, built and run by tests/test_gemm_raster.py.
#include <cstdio>
#include <vector>

#include "gemm_raster.cuh"

int main() {
  long bad = 0, grids = 0;
  std::vector<int> seen;
  for (int mt = 1; mt <= 96; ++mt)
    for (int nt = 1; nt <= 96; ++nt)
      for (int gn = 1; gn <= nt + 1; ++gn) {
        seen.assign((size_t)mt * nt, 0);
        int prev_panel = 0;
        for (int t = 0; t < mt * nt; ++t) {
          int mb = -1, nb = -1;
          wv::raster_tile(t, gn, mt, nt, mb, nb);
          if (mb < 0 || mb >= mt || nb < 0 || nb >= nt) {
            ++bad;
            continue;
          }
          ++seen[(size_t)mb * nt + nb];
          const int panel = nb / gn;  // panels are swept in order
          if (panel < prev_panel) ++bad;
          prev_panel = panel;
        }
        for (int v : seen) bad += v != 1;
        ++grids;
      }
  std::printf("%ld grids, %ld mismatches\n", grids, bad);
  return bad == 0 ? 0 : 1;
}
