// Launch planning of the tensor-core GEMM: tile shape and K splitting.  Pure host functions of
// the problem's tile counts and the GPU's SM count, shared by the launcher (b2g_api.cu) and
// b2g_plan_preview (which the CPU tests use to pin the choices).
#pragma once
#include <algorithm>
#include <cstdint>

namespace b2g {

struct TileChoice {
  int cg;    // CTAs per tile (1 or 2)
  int bn;    // tile width in columns (128, 256 or 512)
  bool half; // CG = 2 half-height pair tile: 128 x 256 over the pair, 64 A rows per CTA
};

// Split count of one-CTA (cg = 1) or half-height pair (half) tiles of a small problem: what
// choose_splits gives when every tile is split (at least 16 K blocks per split, at most 8
// one-CTA splits or 4 pair splits: the largest cluster of the cluster fix-up is 8 CTAs).
inline int64_t small_splits(int64_t tiles, int64_t kit, int64_t groups, bool half) {
  int64_t sp = std::min<int64_t>({groups / std::max<int64_t>(1, tiles), kit / 16, half ? 4 : 8});
  if (2 * tiles > groups || kit < 32) sp = 1;
  return std::max<int64_t>(1, sp);
}

// nmt: 128-row M tiles; kit: K blocks of one tile; sms: SMs; opt_cg / opt_bn: forced values
// (0 = choose); opt_rows: 64 = half-height pair tiles whenever the shape allows, 0 or 128 =
// never (the planner does not choose them: measured on B200 they stream B more slowly than
// one-CTA tiles on every skinny shape tried, although their split-K reduction is smaller).
inline TileChoice choose_tiles(int64_t nmt, int64_t N, int64_t kit, int sms, int opt_cg,
                               int opt_bn, int opt_rows = 0) {
  int cg = opt_cg, bn = opt_bn;
  if (bn == 128) cg = 1;  // the 128-column tile exists for one CTA only
  const bool half_ok = (bn == 0 || bn == 256) && cg != 1;
  if (opt_rows == 64 && half_ok) return {2, 256, true};
  if (cg != 1 && cg != 2) {
    // Small problems (fewer 128x256 tiles than SMs) take one-CTA tiles.  The width is the one
    // whose work units (tiles times the split count choose_splits would give) fill the SMs
    // best; on a tie the 128x256 tile, which moves a quarter fewer bytes per FLOP.
    if (bn == 0 && nmt * ((N + 255) / 256) < sms) {
      cg = 1;
      auto fill = [&](int w, int64_t* splits) {
        const int64_t tiles = nmt * ((N + w - 1) / w);
        const int64_t sp = small_splits(tiles, kit, sms, false);
        const int64_t units = tiles * sp;
        const int64_t waves = (units + sms - 1) / sms;
        *splits = sp;
        return (double)units / (double)(waves * sms);
      };
      int64_t sp128 = 1, sp256 = 1;
      const double f128 = fill(128, &sp128), f256 = fill(256, &sp256);
      bn = f128 > f256 + 1e-9 ? 128 : 256;
    } else {
      cg = (nmt >= 2) ? 2 : 1;
    }
  }
  if (bn != 128 && bn != 256 && bn != 512) {
    // 512-wide pair tiles pull a quarter fewer operand bytes from L2 per FLOP; use them when
    // there are enough of them to fill every CTA pair at least twice.
    const int64_t pairs = std::max(1, sms / 2);
    const int64_t t512 = ((nmt + 1) / 2) * ((N + 511) / 512);
    bn = (cg == 2 && t512 >= 2 * pairs) ? 512 : 256;
  }
  if (cg == 1 && bn == 512) bn = 256;  // one CTA: at most 256 columns (two accumulators)
  if (cg == 2 && bn == 128) bn = 256;
  return {cg, bn, false};
}

struct SplitChoice {
  int num_full;     // tiles done as one unit over all of K (the first ones in tile order)
  int k_splits;     // units per remaining tile
  int k_per_split;  // K blocks per split unit
};

// Split-K for under-filled grids and for the tail wave.  group_cap: CTA groups resident at
// once (SMs, or CTA pairs); opt_split: forced split count (0 = choose); half: half-height pair
// tiles (at most 4 splits, and never a tail split: they split only with the cluster fix-up).
inline SplitChoice choose_splits(int num_tiles, int k_iters, int group_cap, int cg, int opt_split,
                                 bool tail_split, bool half = false) {
  int splits = opt_split;
  int full = 0;
  if (splits <= 0) {
    splits = 1;
    full = num_tiles;
    const int waves = num_tiles / std::max(1, group_cap);
    const int rem = num_tiles - waves * group_cap;
    // every split keeps >= 16 K blocks: below that the fixed cost of a unit (pipeline fill,
    // partial write, fix-up) outweighs the shorter main loop.  One-CTA tiles split at most 8
    // ways, the largest cluster of the cluster fix-up.
    if (2 * num_tiles <= group_cap && k_iters >= 32) {
      splits = std::min({group_cap / std::max(1, num_tiles), k_iters / 16,
                         half ? 4 : (cg == 1 ? 8 : 16)});
      full = 0;
    } else if (!half && tail_split && waves >= 1 && rem > 0 && group_cap / rem >= 2 &&
               k_iters >= 32) {
      // whole waves plus a partial one: split only the partial wave's tiles
      splits = std::min({group_cap / rem, 4, k_iters / 16});
      full = waves * group_cap;
    }
  }
  splits = std::max(1, std::min(splits, std::max(1, k_iters)));
  SplitChoice c;
  c.k_per_split = (k_iters + splits - 1) / splits;
  c.k_splits = c.k_per_split > 0 ? (k_iters + c.k_per_split - 1) / c.k_per_split : 1;  // no empty split
  if (c.k_splits < 1) c.k_splits = 1;
  c.num_full = c.k_splits == 1 ? num_tiles : full;
  return c;
}

}  // namespace b2g
