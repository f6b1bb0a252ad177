// Tile order of the persistent GEMM (gemm_tc.cu), shared with a host-side check.
//
// Grouped rasterisation over N: a panel of gn N-tiles of B (the weights, sized on
// the host) is swept by every M-tile before the next panel, N fastest within the
// panel; the last panel holds the n_tiles % gn remaining N-tiles. Tile index t in
// [0, m_tiles * n_tiles) maps to one (mb, nb) each, every output tile exactly once,
// for any gn >= 1.
#pragma once

#ifdef __CUDACC__
#define WV_RASTER_FN __host__ __device__ __forceinline__
#else
#define WV_RASTER_FN inline
#endif

namespace wv {

WV_RASTER_FN void raster_tile(int t, int gn, int m_tiles, int n_tiles, int& mb, int& nb) {
  const int group = gn * m_tiles;
  const int g = t / group, r = t % group;
  const int first = g * gn;
  const int w = n_tiles - first < gn ? n_tiles - first : gn;
  nb = first + r % w;
  mb = r / w;
}

}  // namespace wv
