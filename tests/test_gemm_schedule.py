"""The persistent GEMM's work-unit -> tile mapping (csrc/gemm_tiles.h), checked on the host.

The header is compiled with the host C++ compiler into a small program that walks every
work unit of a launch the way the kernel does (each CTA of a pair included) and checks
that every (m-tile, n-tile, K split) of the output is produced exactly once: one-CTA and
CTA-pair tiles, odd m-tile counts (the second CTA of the last pair falls outside the
matrix) and the all-gather consumer's per-rank rotation of each sequence's m-tiles.
"""
import os
import shutil
import subprocess

import pytest

CSRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "mini_megatron_b200", "csrc")

PROGRAM = r"""
#include "gemm_tiles.h"
#include <cstdio>
#include <vector>
using namespace mmb::tiles;

template <int CG>
static int check(int mtiles, int ntiles, int splits, bool ag, int S, int Sl, int rank) {
  const int units = num_units(mtiles, ntiles, splits, CG);
  std::vector<int> seen((size_t)mtiles * ntiles * splits, 0);
  for (int u = 0; u < units; ++u)
    for (int cr = 0; cr < CG; ++cr) {
      int tm, tn;
      unit_tile<CG>(u, splits, mtiles, ntiles, cr, ag, S, Sl, rank, tm, tn);
      if (tn < 0 || tn >= ntiles || tm < 0) return 1;
      if (tm >= mtiles) {                 // only the second CTA of an odd last pair
        if (CG != 2 || cr != 1 || tm != mtiles) return 2;
        continue;
      }
      ++seen[((size_t)tm * ntiles + tn) * splits + (u % splits)];
    }
  for (int v : seen)
    if (v != 1) return 3;
  return 0;
}

int main() {
  long cases = 0;
  for (int mt = 1; mt <= 70; ++mt)
    for (int nt = 1; nt <= 7; ++nt)
      for (int sp = 1; sp <= 3; ++sp) {
        int rc = check<1>(mt, nt, sp, false, 0, 0, 0);
        if (!rc) rc = check<2>(mt, nt, sp, false, 0, 0, 0);
        ++cases;
        if (rc) { printf("FAIL plain mt=%d nt=%d sp=%d rc=%d\n", mt, nt, sp, rc); return 1; }
      }
  // all-gather consumer: M = batch * S rows, each rank holds Sl rows of every sequence
  const int seqs[][2] = {{1024, 512}, {1024, 256}, {2048, 256}, {2048, 1024}, {1024, 128}, {512, 128}, {384, 128}};
  for (const auto& q : seqs) {
    const int S = q[0], Sl = q[1], world = S / Sl, tps = S / kBM;
    for (int batch = 1; batch <= 5; ++batch)
      for (int rank = 0; rank < world; ++rank)
        for (int nt = 1; nt <= 4; ++nt) {
          int rc = check<1>(batch * tps, nt, 1, true, S, Sl, rank);
          if (!rc) rc = check<2>(batch * tps, nt, 1, true, S, Sl, rank);
          ++cases;
          if (rc) { printf("FAIL ag S=%d Sl=%d batch=%d rank=%d nt=%d rc=%d\n", S, Sl, batch, rank, nt, rc); return 1; }
        }
  }
  printf("OK %ld\n", cases);
  return 0;
}
"""


def test_every_tile_and_split_is_produced_exactly_once(tmp_path):
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        pytest.skip("no host C++ compiler")
    src = tmp_path / "tiles_check.cpp"
    src.write_text(PROGRAM)
    exe = tmp_path / "tiles_check"
    subprocess.run([cxx, "-std=c++17", "-O1", "-I", CSRC, str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0 and out.stdout.startswith("OK"), out.stdout + out.stderr
