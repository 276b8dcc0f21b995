// mask_geom.cuh -- integer mask geometry shared by host and device.
//
// Every mask of the reference operators (extra_bench.py:55-61: causal,
// dilated, local, block-diagonal, prefix-LM, sliding window) is one instance
// of
//
//   vis(i, j) = j < prefix  ||  ( lo(i) <= j <= hi(i)  &&  (i - j) % dil == 0 )
//   lo(i) = max(0,        i - left  [left  >= 0],  block_start(i) [block > 0],
//               seq_start(i) [packed sequences])
//   hi(i) = min(S_kv - 1, i + right [right >= 0],  block_end(i)   [block > 0],
//               seq_end(i) - 1 [packed sequences])
//
// lo(i) and hi(i) are non-decreasing in i, so the keys any row of a query
// tile [r0, r1] can see lie in [lo(r0), hi(r1)] (plus [0, prefix)). That hull
// is the key-tile range the kernel visits; tiles inside it that every row
// sees completely skip the element-wise mask.
#pragma once
#include <cstdint>

#ifndef CHIA_HD
#define CHIA_HD __host__ __device__ __forceinline__
#endif

namespace chia {

struct MaskGeom {
  int64_t sq;      // query rows
  int64_t skv;     // keys
  int64_t left;    // max i - j, -1 = unbounded
  int64_t right;   // max j - i, -1 = unbounded
  int64_t block;   // block size, 0 = none
  int64_t prefix;  // always-visible key prefix, already clipped to skv
  int64_t dil;     // dilation >= 1
  // packed sequences: nseg + 1 cumulative offsets (device memory), or null
  const int32_t *seg;
  int64_t nseg;
};

// Sequence s of row i: seg[s] <= i < seg[s + 1] (binary search, seg[0] = 0).
CHIA_HD int64_t seq_of(const MaskGeom &g, int64_t i) {
  int64_t lo = 0, hi = g.nseg;
  while (hi - lo > 1) {
    const int64_t mid = (lo + hi) >> 1;
    if (g.seg[mid] <= i)
      lo = mid;
    else
      hi = mid;
  }
  return lo;
}

CHIA_HD int64_t imax64(int64_t a, int64_t b) { return a > b ? a : b; }
CHIA_HD int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }

// Band [lo, hi] of row i (empty when lo > hi). SEG: packed sequences (the
// kernels are instantiated with and without, so calls without them carry no
// sequence code at all).
template <bool SEG = false>
CHIA_HD void row_band(const MaskGeom &g, int64_t i, int64_t &lo, int64_t &hi) {
  lo = 0;
  hi = g.skv - 1;
  if (g.left >= 0) lo = imax64(lo, i - g.left);
  if (g.right >= 0) hi = imin64(hi, i + g.right);
  if (g.block > 0) {
    const int64_t b0 = (i / g.block) * g.block;
    lo = imax64(lo, b0);
    hi = imin64(hi, b0 + g.block - 1);
  }
  if (SEG) {
    const int64_t s = seq_of(g, i);
    lo = imax64(lo, g.seg[s]);
    hi = imin64(hi, static_cast<int64_t>(g.seg[s + 1]) - 1);
  }
}

// Key-tile range [tlo, thi) of width tn visited by query rows [r0, r1].
template <bool SEG = false>
CHIA_HD void tile_range(const MaskGeom &g, int64_t r0, int64_t r1, int tn, int64_t &tlo,
                        int64_t &thi) {
  tlo = thi = 0;
  if (r1 > g.sq - 1) r1 = g.sq - 1;
  if (r0 > r1 || g.skv <= 0) return;
  int64_t lo0, hi0, lo1, hi1;
  row_band<SEG>(g, r0, lo0, hi0);
  row_band<SEG>(g, r1, lo1, hi1);
  int64_t lo = lo0, hi = hi1;
  const bool band_empty = lo > hi;
  if (g.prefix > 0) {
    lo = 0;
    hi = band_empty ? g.prefix - 1 : imax64(hi, g.prefix - 1);
  } else if (band_empty) {
    return;
  }
  tlo = lo / tn;
  thi = hi / tn + 1;
}

// True when every (i, j) with i in [r0, r1] and j in key tile t is visible,
// so the kernel can skip the element-wise mask for that tile.
CHIA_HD bool tile_full(const MaskGeom &g, int64_t r0, int64_t r1, int tn, int64_t t) {
  if (r1 > g.sq - 1) r1 = g.sq - 1;
  const int64_t c0 = t * tn, c1 = c0 + tn - 1;
  if (c1 > g.skv - 1) return false;  // ragged last tile: mask the padding keys
  if (c1 < g.prefix) return true;
  if (g.dil != 1) return false;
  int64_t lo_last, hi_last, lo_first, hi_first;
  row_band(g, r1, lo_last, hi_last);
  row_band(g, r0, lo_first, hi_first);
  return lo_last <= c0 && hi_first >= c1;
}

// tile_full() for every key tile of one query tile [r0, r1], computed once:
// the comparisons of tile_full() turned into tile-index bounds. Because lo()
// and hi() are non-decreasing, the fully visible tiles are the prefix tiles
// plus one contiguous band range, all within the tiles that end inside S_kv.
struct FullTiles {
  int32_t kv_end;   // tiles t < kv_end end inside S_kv
  int32_t pre_end;  // tiles t < pre_end lie inside the prefix
  int32_t band_lo, band_hi;  // band tiles [band_lo, band_hi) (dilation 1 only)
  CHIA_HD bool full(int64_t t) const {
    return t < kv_end && (t < pre_end || (t >= band_lo && t < band_hi));
  }
};

template <bool SEG = false>
CHIA_HD FullTiles full_tiles(const MaskGeom &g, int64_t r0, int64_t r1, int tn) {
  if (r1 > g.sq - 1) r1 = g.sq - 1;
  FullTiles f;
  f.kv_end = static_cast<int32_t>(g.skv / tn);     // (t + 1) tn <= skv
  f.pre_end = static_cast<int32_t>(g.prefix / tn);  // (t + 1) tn <= prefix
  f.band_lo = f.band_hi = 0;
  if (g.dil == 1) {
    int64_t lo_last, hi_last, lo_first, hi_first;
    row_band<SEG>(g, r1, lo_last, hi_last);
    row_band<SEG>(g, r0, lo_first, hi_first);
    // lo(r1) <= t tn  and  t tn + tn - 1 <= hi(r0)
    f.band_lo = static_cast<int32_t>((imax64(lo_last, 0) + tn - 1) / tn);
    f.band_hi = static_cast<int32_t>(imax64(hi_first + 1, 0) / tn);
  }
  return f;
}

// Element visibility with the row band already known.
CHIA_HD bool visible(const MaskGeom &g, int64_t i, int64_t j, int64_t lo, int64_t hi) {
  if (j < g.prefix) return true;
  if (j < lo || j > hi) return false;
  return g.dil == 1 || ((i - j) % g.dil) == 0;
}

// Number of j in [a, b] with (i - j) % d == 0 (a, b, i >= 0).
CHIA_HD int64_t count_congruent(int64_t a, int64_t b, int64_t i, int64_t d) {
  if (a > b) return 0;
  if (d == 1) return b - a + 1;
  const int64_t r = i % d;
  // j = r + d * m, m in [ceil((a - r)/d), floor((b - r)/d)]
  auto fdiv = [](int64_t x, int64_t y) { return x >= 0 ? x / y : -((-x + y - 1) / y); };
  const int64_t mlo = -fdiv(-(a - r), d);
  const int64_t mhi = fdiv(b - r, d);
  return mhi >= mlo ? mhi - mlo + 1 : 0;
}

// Visible pairs of one (batch, head): the mask-aware work unit.
inline int64_t visible_pairs(const MaskGeom &g) {
  int64_t total = 0;
  for (int64_t i = 0; i < g.sq; ++i) {
    int64_t lo, hi;
    row_band(g, i, lo, hi);
    int64_t n = g.prefix;  // keys [0, prefix)
    const int64_t a = imax64(lo, g.prefix);
    n += count_congruent(a, hi, i, g.dil);
    total += n;
  }
  return total;
}

}  // namespace chia
