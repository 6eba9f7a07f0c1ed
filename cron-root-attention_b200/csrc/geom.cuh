// geom.cuh -- index geometry of the causal 3-phase sqrt(N) attention, shared by
// every kernel and by the host-side launch code.
//
// Semantics (reference: cron_root_attention/core.py, forward kernel
// _cron_root_attn_fwd_v14_tiled, lines 907-1158):
//   W  = ceil(sqrt(S))                                         core.py:3479
//   query m, ls(m) = max(m - W + 1, 0)
//   local keys    j in [ls, m]                                 core.py:993-994
//   strided keys  j = s*W with j < ls                          core.py:1059
//   relay token t of block r = t / TOP_K visible iff
//                 (r + 1) * W - 1 < ls                         core.py:1115-1116
//
// Global list.  The strided and relay keys of every W-block r are stored as one
// contiguous run of R rows per block ("global rows", G):
//   G[r*R + 0]       = k[r*W]             (strided key of block r)
//   G[r*R + 1 + t]   = k[src(r, t)]       (relay token t of block r, t < TOP_K)
// with R = 1 + TOP_K when the relay is active, else R = 1.  Row r*R is visible
// iff r*W < ls, i.e. r < ceil(ls/W); the relay rows of block r are visible iff
// r < floor(ls/W).  So the rows a query sees are exactly the PREFIX
//   gcount(m) = R * floor(ls/W) + (ls % W != 0)
// of its (b, h) list: phases 2 and 3 become a dense attention against a prefix
// of one contiguous matrix, with no gather in the inner loop.
#pragma once
#include <stdint.h>

namespace cra {

constexpr int kTile = 128;  // query rows per tile and key rows per tile
constexpr int kUnit = 64;   // backward work unit: 64 keys (dQ pass) or 64 queries (key passes)

struct Geom {
  int S;   // sequence length
  int W;   // window = block size = stride
  int R;   // global rows per block (1 + TOP_K with relay, else 1)
  int NB;  // number of W-blocks, ceil(S / W)
  int NG;  // global rows per (b, h) = NB * R
};

__host__ __device__ __forceinline__ int local_start(int m, int W) { return m - W + 1 > 0 ? m - W + 1 : 0; }

__host__ __device__ __forceinline__ int gcount(int m, int W, int R) {
  const int ls = local_start(m, W);
  return R * (ls / W) + (ls % W != 0 ? 1 : 0);
}

// Number of 128-key band tiles a 128-query tile starting at m0 needs.  Band
// tile t covers keys [m0 - 128 t, m0 - 128 t + 128); tile 0 is the diagonal.
__host__ __device__ __forceinline__ int band_tiles(int m0, int W) {
  const int back = (W - 1 < m0) ? W - 1 : m0;
  return 1 + (back + kTile - 1) / kTile;
}

// Number of 128-row global tiles a 128-query tile starting at m0 needs.
__host__ __device__ __forceinline__ int global_tiles(int m0, int S, int W, int R) {
  const int last = (m0 + kTile - 1 < S - 1) ? m0 + kTile - 1 : S - 1;
  const int c = gcount(last, W, R);
  return (c + kTile - 1) / kTile;
}

// First query that sees global row g (gcount(m) > g); S if none.
__host__ __device__ __forceinline__ int first_query_seeing(int g, int S, int W, int R) {
  // gcount(m) > g  <=>  R*floor(ls/W) + [ls%W!=0] > g.
  // Smallest ls: block r = g / R, row in block i = g % R.
  //   i == 0 (strided row): need ls > r*W          -> ls = r*W + 1
  //   i >  0 (relay row):   need floor(ls/W) > r   -> ls = (r+1)*W
  const int r = g / R, i = g % R;
  const long long ls = (i == 0) ? (long long)r * W + 1 : (long long)(r + 1) * W;
  const long long m = ls + W - 1;
  return m < S ? (int)m : S;
}

// Key-tile schedule of a CTA that owns TWO consecutive 128-query tiles
// A = [m0, m0+128) and B = [m0+128, m0+256) of one (b, h), sharing one stream
// of 128-row key tiles.  Band tile t (t < nband) covers keys
// [m0 + 128 - 128 t, m0 + 256 - 128 t) -- t = 0 is B's diagonal, t = 1 A's --
// down to A's lowest local key (without a valid B, the list starts at t = 1).  Global tile g (after the band) covers global
// rows [128 g, 128 g + 128).  use_a / use_b say which query tile needs the key
// tile; every listed tile is needed by at least one of them.  Queries at or
// after q_end (the sequence end, or the end of this GPU's shard) are absent.
struct PairSchedule {
  int m0, t0, nband, ntiles, lb, ca, cb;
  bool valid_b;
  __host__ __device__ __forceinline__ PairSchedule(int m0_, int q_end, int W, int R) : m0(m0_) {
    const int S = q_end;
    valid_b = m0 + kTile < S;
    const int la = local_start(m0, W);
    lb = local_start(m0 + kTile, W);
    t0 = valid_b ? 0 : 1;  // without B, B's diagonal tile is not needed
    nband = (m0 + 2 * kTile - la + kTile - 1) / kTile - t0;
    ca = gcount(min(m0 + kTile - 1, S - 1), W, R);
    cb = valid_b ? gcount(min(m0 + 2 * kTile - 1, S - 1), W, R) : 0;
    const int cmax = ca > cb ? ca : cb;
    ntiles = nband + (cmax + kTile - 1) / kTile;
  }
  // row0: first key position (band) or first global row; g: global tile
  __host__ __device__ __forceinline__ void tile(int j, int& row0, bool& g, bool& use_a, bool& use_b) const {
    if (j < nband) {
      g = false;
      row0 = m0 + kTile - (j + t0) * kTile;
      use_a = j + t0 >= 1;
      use_b = valid_b && row0 + kTile > lb;
    } else {
      g = true;
      row0 = (j - nband) * kTile;
      use_a = row0 < ca;
      use_b = row0 < cb;
    }
  }
};

}  // namespace cra
