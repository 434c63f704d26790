// Work schedule of the persistent GEMM kernels.
//
// A problem of T output tiles, each kb k-blocks deep, runs on P persistent
// CTAs (or CTA pairs) that take work units u = blockIdx, blockIdx + P, ...
// Whole waves of tiles run over all of K and store final results: units
// [0, whole) are tiles [0, whole) in raster order. The R = T - whole tiles of
// the last, partial wave would leave SMs idle, so each of them is cut into
// `pieces` K-ranges of kbp k-blocks: unit whole + piece * R + r is piece
// `piece` of tile whole + r. A piece writes raw partial sums to a tile-local
// buffer part[piece][r][BM][BN]; a reduction pass adds the pieces of each
// tile in piece order (deterministic), then applies the epilogue.
//
// make_sched picks `pieces` from a wave model: time = whole / P tile-times
// + ceil(R * pieces / P) / pieces tile-times + the partial-sum traffic, which
// is (pieces + 1) * R * BM * BN * element bytes through HBM.
#pragma once
#include <cstdint>

namespace b200 {

struct Sched {
  int tiles_m, tiles_n;
  int whole;   // tiles run over all of K
  int rest;    // tiles cut into pieces
  int pieces;  // K-ranges per cut tile (1 when rest == 0)
  int kb;      // k-blocks per tile
  int kbp;     // k-blocks per piece
  int units;   // whole + rest * pieces
  int group_m; // raster: group_m M-tiles share each N sweep
};

struct Unit {
  int m0, n0;  // tile origin (elements)
  int kb0, nkb;
  int piece;   // -1: whole tile (final result); else the piece index
  int r;       // cut-tile index (piece >= 0)
};

// Tile index -> tile coordinates in the grouped raster (group_m M-tiles per
// N sweep, so CTAs running at the same time share A rows and B columns in L2).
__host__ __device__ inline void tile_coords(const Sched& s, int tile, int& mt, int& nt) {
  const int tiles_per_group = s.group_m * s.tiles_n;
  const int group = tile / tiles_per_group;
  const int first_m = group * s.group_m;
  const int group_rows = (s.tiles_m - first_m) < s.group_m ? (s.tiles_m - first_m) : s.group_m;
  const int in_group = tile - group * tiles_per_group;
  mt = first_m + in_group % group_rows;
  nt = in_group / group_rows;
}

__host__ __device__ inline Unit unit_at(const Sched& s, int u, int bm, int bn) {
  Unit w;
  int tile;
  if (u < s.whole) {
    tile = u;
    w.kb0 = 0;
    w.nkb = s.kb;
    w.piece = -1;
    w.r = 0;
  } else {
    const int v = u - s.whole;
    w.r = v % s.rest;
    w.piece = v / s.rest;
    tile = s.whole + w.r;
    w.kb0 = w.piece * s.kbp;
    w.nkb = (s.kb - w.kb0) < s.kbp ? (s.kb - w.kb0) : s.kbp;
  }
  int mt, nt;
  tile_coords(s, tile, mt, nt);
  w.m0 = mt * bm;
  w.n0 = nt * bn;
  return w;
}

// procs: concurrent CTAs (pairs); t_tile: seconds for one tile over all of K
// on one of them; elem_bytes: partial-sum element size; max_kbp: most
// k-blocks one unit may cover (0: no limit); max_pieces: cap on pieces (1:
// no cutting unless max_kbp forces it); min_kbp: fewest k-blocks per piece.
inline Sched make_sched(int64_t M, int64_t N, int64_t K, int bm, int bn, int bk, int procs,
                        double t_tile, int elem_bytes, int max_kbp, int max_pieces, int min_kbp,
                        int group_m) {
  Sched s;
  s.tiles_m = (int)((M + bm - 1) / bm);
  s.tiles_n = (int)((N + bn - 1) / bn);
  s.group_m = group_m;
  s.kb = (int)((K + bk - 1) / bk);
  const int T = s.tiles_m * s.tiles_n;
  const int P = procs > 0 ? procs : 1;
  // pieces needed so that no unit exceeds max_kbp k-blocks
  const int min_pieces = (max_kbp > 0 && s.kb > max_kbp) ? (s.kb + max_kbp - 1) / max_kbp : 1;
  auto finish = [&](int whole, int pieces) {
    s.whole = whole;
    s.rest = T - whole;
    s.kbp = (s.kb + pieces - 1) / pieces;
    s.pieces = s.rest > 0 ? (s.kb + s.kbp - 1) / s.kbp : 1;  // every piece non-empty
    if (s.rest == 0) s.kbp = s.kb;
    s.units = s.whole + s.rest * s.pieces;
    return s;
  };
  const double tile_bytes = (double)bm * bn * elem_bytes;
  if (min_pieces > 1) {  // every tile is cut
    double best_t = 1e30;
    int best = min_pieces;
    for (int p = min_pieces; p <= (max_pieces > min_pieces ? max_pieces : min_pieces); ++p) {
      if (p > min_pieces && s.kb / p < min_kbp) break;
      const double t = (double)(((int64_t)T * p + P - 1) / P) / p * t_tile +
                       (p + 1) * T * tile_bytes / 6.0e12;
      if (t < best_t * 0.97) {
        best_t = t;
        best = p;
      }
    }
    return finish(0, best);
  }
  const int whole = (T / P) * P;
  const int R = T - whole;
  if (R == 0) return finish(T, 1);
  double best_t = (double)(whole / P + 1) * t_tile;  // the partial wave run whole
  int best = 1;
  for (int p = 2; p <= max_pieces; ++p) {
    if (s.kb / p < min_kbp) break;
    const double t = (double)(whole / P) * t_tile +
                     (double)(((int64_t)R * p + P - 1) / P) / p * t_tile +
                     (p + 1) * R * tile_bytes / 6.0e12;
    if (t < best_t * 0.97) {
      best_t = t;
      best = p;
    }
  }
  return best == 1 ? finish(T, 1) : finish(whole, best);
}

}  // namespace b200
