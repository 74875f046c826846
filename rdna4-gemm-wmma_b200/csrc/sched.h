// Persistent-kernel tile order shared by the device kernel and the host (the host
// copy is exported as b2g_tile_coord so the bijection can be tested without a GPU).
//
// Tiles are visited in grouped column order: `group` consecutive M-tile rows form a
// strip, and a strip is walked N-tile by N-tile with its M-tiles innermost.  CTAs that
// run at the same time therefore share a small set of A row-panels and B column-panels
// in L2.  The last strip may hold fewer than `group` rows; its width is clipped, so the
// map t -> (tm, tn) is a bijection on [0, num_m*num_n) for every grid shape.  (The
// strip remap of the reference, mmm.cpp:1219-1236, falls back to blockIdx when the grid
// width is not a multiple of its strip width and then repeats some tiles and skips
// others; this map has no fallback.)
#pragma once

#if defined(__CUDACC__)
#define B2G_HD __host__ __device__ __forceinline__
#else
#define B2G_HD static inline
#endif

B2G_HD void b2g_sched_tile(int t, int num_m, int num_n, int group, int* tm, int* tn) {
  if (group < 1) group = 1;
  const int per_strip = group * num_n;
  const int strip = t / per_strip;
  const int first_m = strip * group;
  const int rows = (num_m - first_m) < group ? (num_m - first_m) : group;
  const int r = t - strip * per_strip;
  *tm = first_m + r % rows;
  *tn = r / rows;
}
