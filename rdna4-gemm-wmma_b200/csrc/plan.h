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

// Fraction of the resident CTA groups that `units` work units keep busy over their waves.
inline double wave_fill(int64_t units, int64_t groups) {
  groups = std::max<int64_t>(1, groups);
  const int64_t waves = (units + groups - 1) / groups;
  return (double)units / (double)(std::max<int64_t>(1, waves) * groups);
}

// Split count when every tile of a small problem is split (fewer than half as many tiles as
// CTA groups): at most 8 one-CTA splits or 4 half-height pair splits (the largest cluster of
// the cluster fix-up is 8 CTAs), 16 for pairs, each split keeping at least 16 K blocks.  One-CTA
// tiles may keep 8 K blocks a split instead, when that fills strictly more CTA groups
// (measured on B200: 1024^3 in two splits of 8 blocks, 512x512x2048 and 256x1024x2048 in four,
// 5-22% faster than with 16).  *short_split tells whether the 8-block rule was taken.
inline int64_t small_splits(int64_t tiles, int64_t kit, int64_t groups, int cg, bool half,
                            bool* short_split = nullptr) {
  if (short_split) *short_split = false;
  if (2 * tiles > groups) return 1;
  const int64_t cap = half ? 4 : (cg == 1 ? 8 : 16);
  const int64_t per = std::max<int64_t>(1, groups / std::max<int64_t>(1, tiles));
  const int64_t sp16 = kit >= 32 ? std::max<int64_t>(1, std::min<int64_t>({per, kit / 16, cap})) : 1;
  if (cg != 1 || half || kit < 16) return sp16;
  const int64_t sp8 = std::max<int64_t>(1, std::min<int64_t>({per, kit / 8, cap}));
  if (wave_fill(tiles * sp8, groups) > wave_fill(tiles * sp16, groups) + 1e-9) {
    if (short_split) *short_split = true;
    return sp8;
  }
  return sp16;
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
  const int64_t pairs = std::max(1, sms / 2);
  if (cg != 1 && cg != 2) {
    // Small problems (fewer 128x256 tiles than SMs).  When split-K applies, one-CTA tiles (the
    // cluster fix-up), of the width whose work units (tiles times the split count) fill the
    // SMs best; on a tie the 128x256 tile, which moves a quarter fewer bytes per FLOP.  When
    // no width splits, 256x256 pair tiles if they fill the SMs as well: the same CTAs, each
    // loading half as many B bytes per FLOP (measured on B200: 2048^3 and 4096x1024x4096
    // 10-15% faster than 128x256 one-CTA tiles).
    if (bn == 0 && nmt * ((N + 255) / 256) < sms) {
      auto fill = [&](int w, int64_t* splits, bool* short_split) {
        const int64_t tiles = nmt * ((N + w - 1) / w);
        const int64_t sp = small_splits(tiles, kit, sms, 1, false, short_split);
        *splits = sp;
        return wave_fill(tiles * sp, sms);
      };
      int64_t sp128 = 1, sp256 = 1;
      bool s128 = false, s256 = false;
      const double f128 = fill(128, &sp128, &s128), f256 = fill(256, &sp256, &s256);
      if (sp128 == 1 && sp256 == 1 && nmt >= 2 &&
          wave_fill(((nmt + 1) / 2) * ((N + 255) / 256), pairs) >= std::max(f128, f256) - 1e-9)
        return {2, 256, false};
      cg = 1;
      // on a tie, the width that needs no 8-block splits (measured: 4096x512x1024 unsplit
      // 128x128 tiles beat 128x256 tiles in two splits of 8 blocks), then 128x256
      if (f128 > f256 + 1e-9 || (f128 > f256 - 1e-9 && s256 && !s128))
        bn = 128;
      else
        bn = 256;
    } else {
      cg = (nmt >= 2) ? 2 : 1;
    }
  }
  if (bn != 128 && bn != 256 && bn != 512) {
    // 512-wide pair tiles pull a quarter fewer operand bytes from L2 per FLOP; use them when
    // there are enough of them to fill every CTA pair at least twice, or when their waves fill
    // the pairs as well as 256-wide tiles' do (measured on B200: 2048x4096x4096, 3072^3 and
    // 4096x4096x2048 10-13% faster with one or two waves of 512-wide tiles).
    const int64_t mp = (nmt + 1) / 2;
    const int64_t t512 = mp * ((N + 511) / 512), t256 = mp * ((N + 255) / 256);
    bn = (cg == 2 && (t512 >= 2 * pairs || wave_fill(t512, pairs) >= wave_fill(t256, pairs) - 1e-9))
             ? 512
             : 256;
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
    // Every tile split when the tiles fill at most half the CTA groups (small_splits: each
    // split keeps 16 K blocks, or 8 for one-CTA tiles when that fills more groups; below that
    // the fixed cost of a unit, pipeline fill, partial write and fix-up, outweighs the shorter
    // main loop).
    const int64_t sp = small_splits(num_tiles, k_iters, group_cap, cg, half);
    if (sp > 1) {
      splits = (int)sp;
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
