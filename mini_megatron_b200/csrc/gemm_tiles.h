// Work-unit -> tile mapping of the persistent tcgen05 GEMM (gemm_sm100.cu).
//
// Plain C++ with __host__ __device__ under nvcc, so the same code is compiled into the
// kernel and into host-side checks (tests/test_gemm_schedule.py verifies that every
// output tile and K split is produced exactly once, for CTA pairs, odd m-tile counts
// and the all-gather rotation included).
#pragma once

#if defined(__CUDACC__)
#define MMB_TILES_FN __host__ __device__ __forceinline__
#else
#define MMB_TILES_FN inline
#endif

namespace mmb {
namespace tiles {

constexpr int kBM = 128;     // rows of A per CTA tile
constexpr int kGroupM = 16;  // m-tiles walked down each n column before moving right

// Grouped rasterisation: walk kGroupM m-tiles down each n column so the B tile and a
// band of A tiles stay hot in L2.
MMB_TILES_FN void tile_coords(int t, int mtiles, int ntiles, int& tm, int& tn) {
  const int per_group = kGroupM * ntiles;
  const int g = t / per_group;
  const int first_m = g * kGroupM;
  const int left = mtiles - first_m;
  const int gsz = left < kGroupM ? left : kGroupM;
  const int r = t - g * per_group;
  tm = first_m + r % gsz;
  tn = r / gsz;
}

// All-gather consumer: the 128-row tiles of each S-row sequence are rotated by this
// rank's shard (rank * Sl rows), so a rank starts on the rows it produced itself
// (already local) while the peers' shards are still arriving.
MMB_TILES_FN int ag_rotate(int tm, int S, int Sl, int rank) {
  const int tps = S / kBM;
  const int b = tm / tps, k = tm % tps;
  return b * tps + (k + rank * (Sl / kBM)) % tps;
}

// This CTA's 128-row m-tile and n-tile of work unit u (u / splits is the output tile).
// CG = 2 (CTA pair): the output tile is the pair of m-tiles 2p, 2p + 1 sharing one
// n-tile, and CTA `crank` of the pair takes m-tile 2p + crank (>= mtiles: outside the
// matrix, computed on zero-filled rows and not stored).  The all-gather rotation is
// applied per 128-row m-tile: the pair MMA needs the two CTAs to share B, not to hold
// adjacent rows of A.
template <int CG>
MMB_TILES_FN void unit_tile(int u, int splits, int mtiles, int ntiles, int crank, bool ag, int ag_S, int ag_Sl,
                            int ag_rank, int& tm, int& tn) {
  if (CG == 1) {
    tile_coords(u / splits, mtiles, ntiles, tm, tn);
    if (ag) tm = ag_rotate(tm, ag_S, ag_Sl, ag_rank);
  } else {
    tile_coords(u / splits, (mtiles + 1) >> 1, ntiles, tm, tn);
    tm = 2 * tm + crank;
    if (ag && tm < mtiles) tm = ag_rotate(tm, ag_S, ag_Sl, ag_rank);
  }
}

// Work units of a launch: output tiles (pairs of m-tiles for CG = 2) x K splits.
MMB_TILES_FN int num_units(int mtiles, int ntiles, int splits, int cg) {
  return (cg == 1 ? mtiles : (mtiles + 1) >> 1) * ntiles * splits;
}

}  // namespace tiles
}  // namespace mmb
