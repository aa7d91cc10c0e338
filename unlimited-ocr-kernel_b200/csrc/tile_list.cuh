// tile_list.cuh — the tile assignment of the persistent tensor-core GEMMs
// (q8_tc.cu), shared by the kernels and the CPU test that checks it
// (tests/test_tile_list.py compiles this header with the host compiler).
//
// Tiles are 64 activation rows x 128 weight rows.  Row tiles are numbered
// over the groups in order (a group of c rows has ceil(c / 64) of them; a
// single matrix is one group of M rows) and the linear order is
// L = row tile * ntn + weight tile (ntn = N / 128).  CTA c of `ctas` takes
// L = c, c + ctas, c + 2 ctas, ...: the CTAs working at the same time share
// activation tiles and a group's weight tiles.
#pragma once

#if !defined(__CUDACC__) && !defined(__host__)
#define __host__
#define __device__
#endif

namespace uocr {

struct TileSpec {
  int group, row0, rows, nx;  // rows <= row_tile
};

// Writes CTA `cta`'s tiles through emit(index, spec), at most max_tiles of
// them, and returns how many.  counts/offsets: the groups' rows and first
// rows (counts null: one group of M rows from row 0).
template <typename Emit>
__host__ __device__ inline int cta_tile_list(int cta, int ctas, int ntn, int M, const int* counts,
                                             const int* offsets, int groups, int row_tile,
                                             int max_tiles, Emit emit) {
  int n = 0, g = 0, before = 0;  // `before`: row tiles of the groups before g
  const int single_tiles = (M + row_tile - 1) / row_tile;
  for (long long L = cta; n < max_tiles; L += ctas) {
    const int ty = static_cast<int>(L / ntn), nx = static_cast<int>(L % ntn);
    TileSpec t;
    t.nx = nx;
    if (counts) {
      while (g < groups && ty >= before + (counts[g] + row_tile - 1) / row_tile) {
        before += (counts[g] + row_tile - 1) / row_tile;
        ++g;
      }
      if (g >= groups) break;
      t.group = g;
      t.row0 = offsets[g] + (ty - before) * row_tile;
      t.rows = counts[g] - (ty - before) * row_tile;
    } else {
      if (ty >= single_tiles) break;
      t.group = 0;
      t.row0 = ty * row_tile;
      t.rows = M - t.row0;
    }
    if (t.rows > row_tile) t.rows = row_tile;
    emit(n, t);
    ++n;
  }
  return n;
}

// CTAs for `tiles` (an upper bound on the tiles) with `sms` SMs: one per SM,
// more only if a CTA would otherwise own more than max_per_cta tiles (the
// length of its list).
__host__ __device__ inline int persistent_ctas(long long tiles, int sms, int max_per_cta) {
  long long g = tiles < sms ? tiles : sms;
  if (g < 1) g = 1;
  if ((tiles + g - 1) / g > max_per_cta) g = (tiles + max_per_cta - 1) / max_per_cta;
  return static_cast<int>(g);
}

}  // namespace uocr
