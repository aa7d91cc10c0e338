// Host check of the persistent GEMMs' tile assignment (tile_list.cuh, the
// header the kernels include): over random group layouts, tile-list lengths
// and SM counts, every tile of the launch is listed by exactly one CTA, with
// the rows of its group, and no CTA's list is cut short.  Built and run by
// tests/test_tile_list.py; prints "ok" and exits 0, or prints the first
// violation and exits 1.
#include <cstdio>
#include <random>
#include <vector>

#include "tile_list.cuh"

using uocr::TileSpec;

static int fail(const char* what, int a, int b, int c) {
  std::printf("violation: %s (%d, %d, %d)\n", what, a, b, c);
  return 1;
}

// One launch: counts (empty: a single matrix of M rows), ntn weight tiles.
static int check(const std::vector<int>& counts, int M, int ntn, int max_per_cta, int sms,
                 int slack) {
  const int kRowTile = 64;
  const bool grouped = !counts.empty();
  std::vector<int> offsets(counts.size() + 1, 0);
  int row_tiles = 0;
  for (size_t g = 0; g < counts.size(); ++g) {
    offsets[g + 1] = offsets[g] + counts[g];
    row_tiles += (counts[g] + kRowTile - 1) / kRowTile;
  }
  if (!grouped) row_tiles = (M + kRowTile - 1) / kRowTile;
  // the launchers pass an upper bound on the row tiles (the grouped prefill's
  // max_tiles); `slack` more than the actual count
  const long long upper = static_cast<long long>(ntn) * (row_tiles + slack);
  const int ctas = uocr::persistent_ctas(upper, sms, max_per_cta);
  std::vector<int> seen(static_cast<size_t>(row_tiles) * ntn, 0);
  for (int c = 0; c < ctas; ++c) {
    std::vector<TileSpec> list(max_per_cta);
    const int n = uocr::cta_tile_list(c, ctas, ntn, M, grouped ? counts.data() : nullptr,
                                      offsets.data(), static_cast<int>(counts.size()), kRowTile,
                                      max_per_cta,
                                      [&](int i, const TileSpec& t) { list[i] = t; });
    if (n > max_per_cta) return fail("list longer than its bound", c, n, max_per_cta);
    // a full list must not hide tiles: the next tile in this CTA's order is past the end
    if (n == max_per_cta) {
      const long long next = c + static_cast<long long>(n) * ctas;
      if (next < static_cast<long long>(row_tiles) * ntn) return fail("list cut short", c, n, ctas);
    }
    for (int i = 0; i < n; ++i) {
      const TileSpec& t = list[i];
      const long long L = c + static_cast<long long>(i) * ctas;
      const int ty = static_cast<int>(L / ntn), nx = static_cast<int>(L % ntn);
      if (t.nx != nx) return fail("weight tile", c, i, t.nx);
      if (ty >= row_tiles) return fail("row tile past the end", c, i, ty);
      if (t.rows < 1 || t.rows > kRowTile) return fail("rows", c, i, t.rows);
      if (grouped) {
        if (t.group < 0 || t.group >= static_cast<int>(counts.size()))
          return fail("group", c, i, t.group);
        const int first = offsets[t.group], end = offsets[t.group + 1];
        if (t.row0 < first || t.row0 + t.rows > end || (t.row0 - first) % kRowTile)
          return fail("rows outside the group", c, i, t.row0);
        if (t.rows != (end - t.row0 < kRowTile ? end - t.row0 : kRowTile))
          return fail("rows of the group's tile", c, i, t.rows);
      } else {
        if (t.group != 0 || t.row0 != ty * kRowTile) return fail("single row0", c, i, t.row0);
        if (t.rows != (M - t.row0 < kRowTile ? M - t.row0 : kRowTile))
          return fail("single rows", c, i, t.rows);
      }
      ++seen[static_cast<size_t>(ty) * ntn + nx];
    }
  }
  for (size_t j = 0; j < seen.size(); ++j)
    if (seen[j] != 1) return fail("tile listed other than once", static_cast<int>(j), seen[j], ctas);
  return 0;
}

int main() {
  std::mt19937 rng(12345);
  auto uni = [&](int lo, int hi) { return std::uniform_int_distribution<int>(lo, hi)(rng); };
  int cases = 0;
  for (int it = 0; it < 3000; ++it) {
    const int max_per_cta = uni(0, 1) ? 128 : 64;  // the int8 and FP32 kernels' list lengths
    const int sms = uni(0, 3) ? 148 : uni(1, 200);
    const int ntn = uni(1, 40);
    const int slack = uni(0, 3) ? uni(0, 4) : uni(0, 200);
    std::vector<int> counts;
    int M = 0;
    if (uni(0, 4)) {
      const int groups = uni(1, 256);
      counts.resize(groups);
      for (int& c : counts) {
        const int kind = uni(0, 9);
        c = kind == 0 ? 0 : kind < 7 ? uni(1, 130) : uni(1, 2000);
      }
    } else {
      M = uni(1, 70000);
    }
    bool any = !counts.empty() ? false : M > 0;
    for (int c : counts) any = any || c > 0;
    if (!any) continue;
    if (check(counts, M, ntn, max_per_cta, sms, slack)) {
      std::printf("case %d: groups %zu, M %d, ntn %d, list %d, sms %d, slack %d\n", it,
                  counts.size(), M, ntn, max_per_cta, sms, slack);
      return 1;
    }
    ++cases;
  }
  // the shapes the benchmarks launch: grouped prefill at 1024 tokens, lm_head rows
  std::vector<int> prefill(64, 96);
  if (check(prefill, 0, 7, 128, 148, 30) || check(prefill, 0, 10, 64, 148, 30) ||
      check({}, 64, 1010, 128, 148, 0) || check({}, 65535, 30, 64, 148, 0))
    return 1;
  std::printf("ok %d cases\n", cases + 4);
  return 0;
}
