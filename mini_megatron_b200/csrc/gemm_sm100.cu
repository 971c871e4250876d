// Persistent warp-specialised bf16 GEMM for sm_100a (tcgen05 + TMEM + TMA).
//
//   D[M,N] = alpha * sum_k A(m,k) * B(n,k)      (fp32 accumulation in TMEM)
//
// Operand storage (row-major, leading dimension in elements):
//   A K-major  : A[M,K]           A MN-major : At[K,M]
//   B K-major  : B[N,K]           B MN-major : Bt[K,N]
// which covers the three GEMMs of a linear layer without any transpose copy:
//   forward  Y  = X  W^T   (A=X  K-major,  B=W  K-major)
//   dgrad    dX = dY W     (A=dY K-major,  B=W  MN-major)
//   wgrad    dW = dY^T X   (A=dY MN-major, B=X  MN-major)
//
// The reference computes these with library GEMMs behind F.linear
// (parallel/tensor_parallel.py:57,79; model/transformer.py:46).  Here the
// epilogue also fuses the element-wise work that follows each GEMM in the
// model: GELU (fc1), GELU-backward (fc2 dgrad), residual add (attn.o / fc2),
// and fp32 gradient accumulation into the flat main-grad buffer (wgrad).
//
// CTA = 10 warps: warp 0 issues TMA loads, warp 1 owns TMEM and issues
// tcgen05.mma from one thread, warps 2-9 drain the accumulator (tcgen05.ld)
// and run the epilogue.  Two TMEM accumulators let the epilogue of tile i
// overlap the main loop of tile i+1.  Tiles are 128 x BN x 64 per CTA.
//
// CTA pairs (CG = 2): a 2-CTA cluster on one TPC computes a 256 x 256 tile.
// Each CTA TMA-loads its own 128 rows of A and 128 of the 256 B rows (no tile is
// copied between the two CTAs), with the transaction bytes completing on the even
// CTA's barrier; that CTA alone issues tcgen05.mma.cta_group::2, which reads both
// CTAs' shared memory and writes each CTA's 128 x 256 accumulator into its own
// TMEM.  Per SM, a 64-deep k-block then moves 32 KB of operands instead of 48 KB
// for the same MMA work.
#include "common.cuh"
#include "gemm_sm100.h"
#include "gemm_tiles.h"
#include "peer.cuh"

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <unordered_map>

namespace mmb {

constexpr int BM = 128;
constexpr int BK = 64;
static_assert(BM == tiles::kBM, "tile mapping and kernel disagree on the m-tile height");
constexpr int kGemmThreads = 320;  // 2 producer/MMA warps + 8 epilogue warps
constexpr int kEpiWarps = 8;

// CG = CTAs per output tile: 1, or 2 for a CTA pair (2-CTA cluster) that computes a
// 256 x BN tile with pair MMAs, each CTA holding 128 rows of A and BN/2 rows of B.
template <int BN, int CG = 1>
struct GemmCfg {
  static_assert(CG == 1 || (CG == 2 && BN == 256), "CTA pairs use 256-wide tiles");
  static constexpr int STAGES = (BN == 256 && CG == 1) ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2;          // 16 KB
  static constexpr int B_BYTES = (BN / CG) * BK * 2;   // 32 KB / 16 KB (this CTA's share)
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;             // double-buffered accumulator
  static constexpr int SMEM_BYTES = 1024 /*align slack*/ + STAGES * STAGE_BYTES + 8 * 4096 /*epilogue*/ + 256;  // one 4 KB stage per epilogue warp
};

// Work-unit -> tile mapping (gemm_tiles.h), with the all-gather parameters of the launch.
template <int CG>
__device__ __forceinline__ void unit_tile(const GemmArgs& args, int u, int splits, int mtiles, int ntiles, int crank,
                                          int& tm, int& tn) {
  tiles::unit_tile<CG>(u, splits, mtiles, ntiles, crank, args.ag_flags != nullptr, args.ag_S, args.ag_Sl,
                       args.ag_rank, tm, tn);
}

// ---------------------------------------------------------------- epilogue helpers
// Each epilogue warp owns 32 accumulator rows (one per lane).  A chunk of its
// rows is staged in shared memory as 32 rows x 128 bytes in the TMA 128-byte
// swizzle (16-byte unit u of row r lives at unit u ^ (r % 8)), then written by
// ONE bulk tensor store (or reduce-add) issued by lane 0.
constexpr int kStageBytes = 32 * 128;

__device__ __forceinline__ uint8_t* stage_unit(uint8_t* stg, int row, int unit) {
  return stg + row * 128 + ((unit ^ (row & 7)) << 4);
}

// Cooperative, coalesced copy of a 32-row x 128-byte window of a row-major
// global matrix into the swizzled stage (8 lanes per row, 4 rows per step).
// Rows >= rows_valid or bytes past col_bytes_valid are skipped.
__device__ __forceinline__ void stage_load(uint8_t* stg, const uint8_t* gbase, long ld_bytes, int rows_valid,
                                           int col_bytes_valid, int lane) {
  const int unit = lane & 7;
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int row = it * 4 + (lane >> 3);
    if (row < rows_valid && unit * 16 < col_bytes_valid)
      *reinterpret_cast<uint4*>(stage_unit(stg, row, unit)) =
          *reinterpret_cast<const uint4*>(gbase + (size_t)row * ld_bytes + unit * 16);
  }
}

// Register prefetch of the same 32-row x 128-byte window (the side input of the
// residual / GELU-backward epilogues): lane l holds rows it*4 + l/8, unit l%8.
// Issued one chunk ahead, so the global-load latency hides behind the current
// chunk's TMEM load, math and store.
__device__ __forceinline__ void side_prefetch(uint4 (&buf)[8], const uint8_t* gbase, long ld_bytes, int rows_valid,
                                              int col_bytes_valid, int lane) {
  const int unit = lane & 7;
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int row = it * 4 + (lane >> 3);
    buf[it] = (row < rows_valid && unit * 16 < col_bytes_valid)
                  ? *reinterpret_cast<const uint4*>(gbase + (size_t)row * ld_bytes + unit * 16)
                  : make_uint4(0u, 0u, 0u, 0u);
  }
}

__device__ __forceinline__ void side_to_stage(uint8_t* stg, const uint4 (&buf)[8], int lane) {
  const int unit = lane & 7;
#pragma unroll
  for (int it = 0; it < 8; ++it) *reinterpret_cast<uint4*>(stage_unit(stg, it * 4 + (lane >> 3), unit)) = buf[it];
}

template <int BN, bool A_MN, bool B_MN, int EPI, int CG>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_sm100(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmAux,
                    const GemmArgs args) {
  pdl_trigger();
  using C = GemmCfg<BN, CG>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::A_BYTES;
  uint8_t* sStage = smem + STAGES * C::STAGE_BYTES;  // 8 epilogue warps x 4 KB staging
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStage + 8 * kStageBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* acc_empty = bars + 2 * STAGES + 2;
  uint64_t* drain = bars + 2 * STAGES + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // CTA pair: rank 0 (leader) owns the stage-full and accumulator-empty barriers
  // and issues the MMAs; both CTAs load their own operand halves and drain their
  // own accumulator rows.
  const uint32_t crank = (CG == 2) ? cluster_ctarank() : 0u;
  const bool leader = (crank == 0);
  const int u0 = blockIdx.x / CG;      // first work unit of this CTA (pair)
  const int ustep = gridDim.x / CG;    // CTAs (pairs) in the persistent grid
  // a failed wait in one CTA of a pair also stops the other one
  auto raise_abort = [&]() {
    *abort_flag = 1;
    if constexpr (CG == 2) st_cluster_u32(cluster_addr((const void*)abort_flag, crank ^ 1u), 1u);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      // 1 CTA: every epilogue thread arrives; pair: one arrival per epilogue warp of both CTAs
      mbar_init(&acc_empty[b], CG == 1 ? 32 * kEpiWarps : 2 * kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmD);
  }
  if (warp == 1) {
    if constexpr (CG == 1) {
      tmem_alloc(tmem_slot, C::TMEM_COLS);
      tmem_relinquish();
    } else {
      tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
      tmem_relinquish_pair();
    }
  }
  tc_fence_before();
  if constexpr (CG == 1) {
    __syncthreads();
  } else {
    cluster_sync_all();  // the peer's barriers are initialised before any remote arrive
  }
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // set-up above touched no global memory; everything below may depend on the previous kernel

  const int mtiles = (args.M + BM - 1) / BM;
  const int ntiles = (args.N + BN - 1) / BN;
  const int kblocks_total = (args.K + BK - 1) / BK;
  // Work unit = (output tile, K split).  Splits > 1 only with the atomic epilogue.
  const int splits = args.splits > 0 ? args.splits : 1;
  const int kb_per_split = (kblocks_total + splits - 1) / splits;
  const int num_tiles = tiles::num_units(mtiles, ntiles, splits, CG);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_par = 0;
      bool ok = true;
      uint32_t ag_ready = 0;  // source ranks whose rows are known to have arrived
      for (int t = u0; t < num_tiles && ok; t += ustep) {
        int tm, tn;
        unit_tile<CG>(args, t, splits, mtiles, ntiles, (int)crank, tm, tn);
        const int m0 = tm * BM, n0 = tn * BN + (int)crank * (BN / CG);
        if (args.ag_flags != nullptr && tm < mtiles) {
          const int src = (m0 % args.ag_S) / args.ag_Sl;
          if (!((ag_ready >> src) & 1u)) {
            if (!wait_flag_ge(args.ag_flags + src, args.ag_epoch, args.err)) {
              raise_abort();
              ok = false;
              break;
            }
            ag_ready |= 1u << src;
          }
        }
        const int kb_lo = (t % splits) * kb_per_split;
        const int kb_hi = min(kblocks_total, kb_lo + kb_per_split);
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, args.err, kErrGemmEmptyWait, abort_flag)) {
            raise_abort();
            ok = false;
            break;
          }
          uint8_t* a_dst = sA + stage * C::A_BYTES;
          uint8_t* b_dst = sB + stage * C::B_BYTES;
          const int k0 = kb * BK;
          if constexpr (CG == 1) {
            mbar_expect_tx(&full[stage], C::STAGE_BYTES);
            issued_mask |= 1u << stage;
            issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
            if constexpr (!A_MN) {
              tma_load_2d(a_dst, &tmA, &full[stage], k0, m0);
            } else {
#pragma unroll
              for (int j = 0; j < BM / 64; ++j) tma_load_2d(a_dst + j * 8192, &tmA, &full[stage], m0 + 64 * j, k0);
            }
            if constexpr (!B_MN) {
              tma_load_2d(b_dst, &tmB, &full[stage], k0, n0);
            } else {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j) tma_load_2d(b_dst + j * 8192, &tmB, &full[stage], n0 + 64 * j, k0);
            }
          } else {
            // both CTAs' bytes complete on the leader's barrier, which expects them all
            if (leader) {
              mbar_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
              issued_mask |= 1u << stage;
              issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
            }
            const uint32_t fb = cluster_addr(&full[stage], 0);
            if constexpr (!A_MN) {
              tma_load_2d_pair(a_dst, &tmA, fb, k0, m0);
            } else {
#pragma unroll
              for (int j = 0; j < BM / 64; ++j) tma_load_2d_pair(a_dst + j * 8192, &tmA, fb, m0 + 64 * j, k0);
            }
            if constexpr (!B_MN) {
              tma_load_2d_pair(b_dst, &tmB, fb, k0, n0);
            } else {
#pragma unroll
              for (int j = 0; j < (BN / CG) / 64; ++j) tma_load_2d_pair(b_dst + j * 8192, &tmB, fb, n0 + 64 * j, k0);
            }
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Let loads already in flight land before the CTA (and its smem) goes
        // away: stage s completes the phase with the parity it was issued in.
        // (A pair's follower has no barrier of its own to watch; the closing
        // cluster barrier keeps it alive until the leader has drained.)
        for (int s = 0; s < STAGES; ++s) {
          if (!((issued_mask >> s) & 1u)) continue;
          const uint32_t par = (issued_par >> s) & 1u;
          const unsigned long long t0 = globaltimer();
          while (!mbar_try_wait(&full[s], par) && globaltimer() - t0 < 10000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (pair: leader only)
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = make_idesc_bf16(BM * CG, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int t = u0; t < num_tiles && ok; t += ustep, ++it) {
        const int buf = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&acc_empty[buf], acc_phase ^ 1u, args.err, kErrGemmAccEmptyWait, abort_flag)) {
          raise_abort();
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        const int kb_lo = (t % splits) * kb_per_split;
        const int kb_hi = min(kblocks_total, kb_lo + kb_per_split);
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(&full[stage], phase, args.err, kErrGemmFullWait, abort_flag)) {
            raise_abort();
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = A_MN ? make_sdesc_sw128(a_addr + k * 2048, 8192, 1024)
                                        : make_sdesc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? make_sdesc_sw128(b_addr + k * 2048, 8192, 1024)
                                        : make_sdesc_sw128(b_addr + k * 32, 16, 1024);
            if constexpr (CG == 1)
              umma_bf16_ss(d_tmem, adesc, bdesc, idesc, (kb != kb_lo || k != 0) ? 1u : 0u);
            else
              umma_bf16_ss_pair(d_tmem, adesc, bdesc, idesc, (kb != kb_lo || k != 0) ? 1u : 0u);
          }
          // frees the smem stage (of both CTAs) once these MMAs have read it
          if constexpr (CG == 1) {
            umma_commit(&empty[stage]);
          } else {
            umma_commit_pair(cluster_addr(&empty[stage], 0));
            umma_commit_pair(cluster_addr(&empty[stage], 1));
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        // accumulator ready for the epilogue(s)
        if constexpr (CG == 1) {
          umma_commit(&acc_full[buf]);
        } else {
          umma_commit_pair(cluster_addr(&acc_full[buf], 0));
          umma_commit_pair(cluster_addr(&acc_full[buf], 1));
        }
      }
      if (!ok) {
        // Drain: wait (bounded) until every MMA issued so far has completed.
        if constexpr (CG == 1)
          umma_commit(drain);
        else
          umma_commit_pair(cluster_addr(drain, 0));
        const unsigned long long t0 = globaltimer();
        while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < 10000000ull) {
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..9)
    // bf16 outputs go out in 64-column chunks, fp32 outputs in 32-column
    // chunks (128 bytes per row either way).  Warps w and w+4 share a TMEM lane
    // quarter and take alternate chunks, so two warps per scheduler run the
    // epilogue math.
    constexpr bool OUT_BF16 = (EPI == EPI_BF16 || EPI == EPI_GELU || EPI == EPI_DGELU || EPI == EPI_PUSH_BF16 ||
                               EPI == EPI_CE_STATS);
    constexpr int W = OUT_BF16 ? 64 : 32;
    const int q = warp & 3;             // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;   // which alternate chunks this warp takes
    uint8_t* stg = sStage + (warp - 2) * kStageBytes;
    // side input (residual fp32 / gelu' bf16) of chunk ch of tile t, prefetched one chunk ahead
    constexpr bool SIDE = (EPI == EPI_RESID || EPI == EPI_DGELU);
    constexpr int SIDE_ES = (EPI == EPI_RESID) ? 4 : 2;
    const uint8_t* side_base = SIDE ? reinterpret_cast<const uint8_t*>(EPI == EPI_RESID ? (const void*)args.resid
                                                                                        : (const void*)args.aux)
                                    : nullptr;
    const long side_ld = (EPI == EPI_RESID) ? args.ld_resid : args.ld_aux;
    uint4 side[8];
    auto prefetch_side = [&](int tt, int ch) {
      int pm, pn;
      unit_tile<CG>(args, tt, splits, mtiles, ntiles, (int)crank, pm, pn);
      const int pr0 = pm * BM + q * 32, pc0 = pn * BN + ch * W;
      side_prefetch(side, side_base + ((size_t)pr0 * side_ld + pc0) * SIDE_ES, side_ld * SIDE_ES,
                    min(32, args.M - pr0), (args.N - pc0) * SIDE_ES, lane);
    };
    // the chunk this warp handles after (t, ch): the next alternate chunk of this
    // tile, else its first chunk of the next tile of this CTA (if any)
    auto prefetch_next_side = [&](int tt, int ch) {
      int nt = tt, nch = ch + 2, cm, cn;
      unit_tile<CG>(args, tt, splits, mtiles, ntiles, (int)crank, cm, cn);
      if (nch >= BN / W || cn * BN + nch * W >= args.N) {
        nt = tt + ustep;
        nch = half;
      }
      if (nt < num_tiles) prefetch_side(nt, nch);
    };
    if constexpr (SIDE) {
      if (u0 < num_tiles) prefetch_side(u0, half);
    }
    int it = 0;
    for (int t = u0; t < num_tiles; t += ustep, ++it) {
      const int buf = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      // One lane waits, the warp follows: tcgen05.ld below is warp-collective,
      // so the whole warp must agree on whether to continue.
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&acc_full[buf], acc_phase, args.err, kErrGemmAccFullWait, abort_flag) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) raise_abort();
        break;
      }
      tc_fence_after();
      int tm, tn;
      unit_tile<CG>(args, t, splits, mtiles, ntiles, (int)crank, tm, tn);
      const int r0 = tm * BM + q * 32;                 // first row of this warp
      const int n0 = tn * BN;
      const int rows_valid = min(32, args.M - r0);
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + buf * BN;
      const int nchunks = BN / W;
      float ce_m = -INFINITY, ce_s = 0.f;  // EPI_CE_STATS: this lane's row over this warp's chunks of the tile
#pragma unroll 1
      for (int ch = half; ch < nchunks; ch += 2) {
        const int col0 = n0 + ch * W;
        if (col0 >= args.N) {  // warp-uniform
          if constexpr (SIDE) prefetch_next_side(t, ch);
          break;
        }
        float v[W];
        {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + ch * W, r);
          if constexpr (W == 64) {
            uint32_t r2[32];
            tmem_ld_32x32b_x32(t_row + ch * W + 32, r2);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              v[i] = __uint_as_float(r[i]) * args.alpha;
              v[32 + i] = __uint_as_float(r2[i]) * args.alpha;
            }
          } else {
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * args.alpha;
          }
        }
        if (rows_valid <= 0) {
          if constexpr (SIDE) prefetch_next_side(t, ch);
          continue;
        }
        const int colb_valid = (args.N - col0) * (OUT_BF16 ? 2 : 4);
        // the previous store from this warp's stage must have finished reading it
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
        if constexpr (EPI == EPI_BF16 || EPI == EPI_PUSH_BF16) {
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<uint4*>(stage_unit(stg, lane, u)) =
                make_uint4(pack_bf16x2(v[8 * u], v[8 * u + 1]), pack_bf16x2(v[8 * u + 2], v[8 * u + 3]),
                           pack_bf16x2(v[8 * u + 4], v[8 * u + 5]), pack_bf16x2(v[8 * u + 6], v[8 * u + 7]));
        } else if constexpr (EPI == EPI_CE_STATS) {
          // store the bf16 logits and fold this chunk's (max, sumexp) of the ROUNDED values into the row's
          // running pair, so the statistics match the logits the backward reads
          constexpr float kLog2e = 1.4426950408889634f;
          const int nv = args.ce_n_valid - col0;  // valid columns in this chunk (may be <= 0 or >= 64)
          float xb[W];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const uint4 w4 = make_uint4(pack_bf16x2(v[8 * u], v[8 * u + 1]), pack_bf16x2(v[8 * u + 2], v[8 * u + 3]),
                                        pack_bf16x2(v[8 * u + 4], v[8 * u + 5]),
                                        pack_bf16x2(v[8 * u + 6], v[8 * u + 7]));
            *reinterpret_cast<uint4*>(stage_unit(stg, lane, u)) = w4;
            const float2 f0 = unpack_bf16x2(w4.x), f1 = unpack_bf16x2(w4.y), f2 = unpack_bf16x2(w4.z),
                         f3 = unpack_bf16x2(w4.w);
            xb[8 * u + 0] = f0.x; xb[8 * u + 1] = f0.y; xb[8 * u + 2] = f1.x; xb[8 * u + 3] = f1.y;
            xb[8 * u + 4] = f2.x; xb[8 * u + 5] = f2.y; xb[8 * u + 6] = f3.x; xb[8 * u + 7] = f3.y;
          }
          float cm[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int i = 0; i < W; ++i)
            if (i < nv) cm[i & 3] = fmaxf(cm[i & 3], xb[i]);
          const float mc = fmaxf(fmaxf(cm[0], cm[1]), fmaxf(cm[2], cm[3]));
          if (mc > -INFINITY) {
            float cs[4] = {0.f, 0.f, 0.f, 0.f};
            const float mcl = mc * kLog2e;
#pragma unroll
            for (int i = 0; i < W; ++i)
              if (i < nv) cs[i & 3] += fast_exp2(fmaf(xb[i], kLog2e, -mcl));
            const float sc = (cs[0] + cs[1]) + (cs[2] + cs[3]);
            if (mc > ce_m) {
              ce_s = ce_s * fast_exp2((ce_m - mc) * kLog2e) + sc;
              ce_m = mc;
            } else {
              ce_s += sc * fast_exp2((mc - ce_m) * kLog2e);
            }
          }
        } else if constexpr (EPI == EPI_GELU) {
          // gelu and gelu' share one erf evaluation; gelu' is stored (aux) for the backward
          uint32_t act[W / 2], grd[W / 2];
#pragma unroll
          for (int i = 0; i < W; i += 2) {
            const GeluTerms g0 = gelu_terms(v[i]), g1 = gelu_terms(v[i + 1]);
            act[i >> 1] = pack_bf16x2(v[i] * g0.cdf, v[i + 1] * g1.cdf);
            grd[i >> 1] = pack_bf16x2(g0.cdf + v[i] * g0.pdf, g1.cdf + v[i + 1] * g1.pdf);
          }
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<uint4*>(stage_unit(stg, lane, u)) =
                make_uint4(grd[4 * u], grd[4 * u + 1], grd[4 * u + 2], grd[4 * u + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmAux, stg, col0, r0);
            bulk_commit();
            bulk_wait_read<0>();
          }
          __syncwarp();
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<uint4*>(stage_unit(stg, lane, u)) =
                make_uint4(act[4 * u], act[4 * u + 1], act[4 * u + 2], act[4 * u + 3]);
        } else if constexpr (EPI == EPI_DGELU) {
          // stage <- prefetched gelu'(pre) chunk, prefetch the next one, then out = acc * gelu' in place
          side_to_stage(stg, side, lane);
          prefetch_next_side(t, ch);
          __syncwarp();
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            uint4* pu = reinterpret_cast<uint4*>(stage_unit(stg, lane, u));
            uint4 gp = *pu;
            const uint32_t* gw = reinterpret_cast<const uint32_t*>(&gp);
            uint32_t o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 gf = unpack_bf16x2(gw[e]);
              o[e] = pack_bf16x2(v[8 * u + 2 * e] * gf.x, v[8 * u + 2 * e + 1] * gf.y);
            }
            *pu = make_uint4(o[0], o[1], o[2], o[3]);
          }
        } else if constexpr (EPI == EPI_RESID) {
          // stage <- prefetched residual chunk, prefetch the next one, then out = resid + acc in place
          side_to_stage(stg, side, lane);
          prefetch_next_side(t, ch);
          __syncwarp();
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            float4* pu = reinterpret_cast<float4*>(stage_unit(stg, lane, u));
            float4 c = *pu;
            c.x += v[4 * u]; c.y += v[4 * u + 1]; c.z += v[4 * u + 2]; c.w += v[4 * u + 3];
            *pu = c;
          }
        } else {  // EPI_F32, EPI_F32_ACC, EPI_F32_ATOMIC
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<float4*>(stage_unit(stg, lane, u)) =
                make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
        }
        if constexpr (EPI == EPI_PUSH_BF16) {
          // reduce-scatter: coalesced NVLink stores of the staged 32-row chunk into the owner's slot
          __syncwarp();
          const int owner = (r0 % args.push_S) / args.push_Sl;
          const long lr0 = (long)(r0 / args.push_S) * args.push_Sl + (r0 % args.push_S) - owner * args.push_Sl;
          uint8_t* dst = reinterpret_cast<uint8_t*>(args.push_dst[owner]) + (lr0 * args.ldd + col0) * 2;
          const int unit = lane & 7;
#pragma unroll
          for (int itr = 0; itr < 8; ++itr) {
            const int row = itr * 4 + (lane >> 3);
            if (row < rows_valid && unit * 16 < colb_valid)
              *reinterpret_cast<uint4*>(dst + (size_t)row * args.ldd * 2 + unit * 16) =
                  *reinterpret_cast<const uint4*>(stage_unit(stg, row, unit));
          }
          __syncwarp();
          continue;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if constexpr (EPI == EPI_F32_ACC || EPI == EPI_F32_ATOMIC) {
            tma_reduce_add_2d(&tmD, stg, col0, r0);
          } else {
            tma_store_2d(&tmD, stg, col0, r0);
          }
          bulk_commit();
        }
      }
      if constexpr (EPI == EPI_CE_STATS) {
        if (lane < rows_valid)
          args.ce_part[(size_t)(r0 + lane) * args.ce_ld + 2 * tn + half] = make_float2(ce_m, ce_s);
      }
      tc_fence_before();
      if constexpr (CG == 1) {
        mbar_arrive(&acc_empty[buf]);
      } else {
        __syncwarp();  // the whole warp's TMEM reads are done
        if (lane == 0) mbar_arrive_remote(cluster_addr(&acc_empty[buf], 0));
      }
    }
    if (lane == 0) bulk_wait<0>();
    __syncwarp();
  }

  tc_fence_before();
  if constexpr (CG == 1) {
    __syncthreads();
  } else {
    // neither CTA of a pair leaves while the other may still signal its barriers,
    // read its shared memory or write its tensor memory
    cluster_sync_all();
  }
  if constexpr (EPI == EPI_PUSH_BF16) {
    // every tile of this rank has been pushed: the last CTA tells each owner
    if (!*abort_flag)
      grid_done_signal(args.push_flags, args.push_world, args.push_rank, args.push_epoch, args.push_counter);
  }
  if (warp == 1) {
    tc_fence_after();
    if constexpr (CG == 1)
      tmem_dealloc(tmem_base, C::TMEM_COLS);
    else
      tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

// ============================================================================ host side

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled get_encode_fn() {
  static PFN_encodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  });
  return fn;
}

// Encoded tensor maps, cached per host thread.  A map is a pure function of its
// parameters (address, shape, leading dimension, box, element type), so a hit can be
// reused whatever the memory holds now; the eager (un-captured) training step launches
// the same few hundred GEMM / attention shapes on the same buffers every step.
struct TmapKey {
  const void* base;
  long rows, cols, ld;
  int box_cols, box_rows, dt;
  bool operator==(const TmapKey& o) const {
    return base == o.base && rows == o.rows && cols == o.cols && ld == o.ld && box_cols == o.box_cols &&
           box_rows == o.box_rows && dt == o.dt;
  }
};
struct TmapKeyHash {
  size_t operator()(const TmapKey& k) const {
    uint64_t h = reinterpret_cast<uintptr_t>(k.base) * 0x9E3779B97F4A7C15ull;
    for (uint64_t v : {(uint64_t)k.rows, (uint64_t)k.cols, (uint64_t)k.ld,
                       ((uint64_t)k.box_cols << 32) | (uint32_t)k.box_rows, (uint64_t)k.dt})
      h = (h ^ v) * 0x100000001B3ull;
    return (size_t)(h ^ (h >> 29));
  }
};
constexpr size_t kTmapCacheMax = 4096;  // cleared when full (a step uses far fewer)

static bool tmap_cache_enabled() {
  static const bool on = [] {
    const char* e = getenv("MMB_TMAP_CACHE");
    return e == nullptr || e[0] != '0';
  }();
  return on;
}

// 2-D tensor map over a row-major matrix [rows, cols] with leading dimension
// `ld` (elements), 128-byte swizzle, box {box_cols, box_rows}.
static int make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* base, long rows, long cols,
                        long ld, int box_cols, int box_rows) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return -2;
  if ((ld * esize) % 16 != 0) return -3;
  thread_local std::unordered_map<TmapKey, CUtensorMap, TmapKeyHash> cache;
  const TmapKey key{base, rows, cols, ld, box_cols, box_rows, (int)dt};
  const bool use_cache = tmap_cache_enabled();
  if (use_cache) {
    const auto it = cache.find(key);
    if (it != cache.end()) {
      *map = it->second;
      return 0;
    }
  }
  PFN_encodeTiled enc = get_encode_fn();
  if (!enc) return -1;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * esize)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return -4;
  if (use_cache) {
    if (cache.size() >= kTmapCacheMax) cache.clear();
    cache.emplace(key, *map);
  }
  return 0;
}

int make_tmap_bf16_2d(CUtensorMap* map, const void* base, long rows, long cols, long ld, int box_cols,
                      int box_rows) {
  return make_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, rows, cols, ld, box_cols, box_rows);
}

int make_tmap_f32_2d(CUtensorMap* map, const void* base, long rows, long cols, long ld, int box_cols, int box_rows) {
  return make_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, rows, cols, ld, box_cols, box_rows);
}

// Launch of one instantiation.  `grid` is in CTAs (even for CTA pairs); pairs are
// launched as 2-CTA clusters, capped at the number of clusters that fit at once.
template <int BN, bool A_MN, bool B_MN, int EPI, int CG>
static cudaError_t launch_one(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td,
                              const CUtensorMap& tx, const GemmArgs& args, int grid, cudaStream_t stream) {
  auto kern = gemm_bf16_sm100<BN, A_MN, B_MN, EPI, CG>;
  constexpr int smem = GemmCfg<BN, CG>::SMEM_BYTES;
  static bool attr_set = false;  // per instantiation
  static int max_pairs = 0;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if constexpr (CG == 2) {
      cudaLaunchConfig_t q = {};
      q.gridDim = dim3(2 * 74);
      q.blockDim = dim3(kGemmThreads);
      q.dynamicSmemBytes = smem;
      cudaLaunchAttribute ca[1];
      ca[0].id = cudaLaunchAttributeClusterDimension;
      ca[0].val.clusterDim.x = 2;
      ca[0].val.clusterDim.y = 1;
      ca[0].val.clusterDim.z = 1;
      q.attrs = ca;
      q.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &q) != cudaSuccess || n <= 0) {
        (void)cudaGetLastError();
        return cudaErrorInvalidConfiguration;
      }
      max_pairs = n;
    }
    attr_set = true;
  }
  if constexpr (CG == 1) {
    launch_k(kern, grid, kGemmThreads, smem, stream, ta, tb, td, tx, args);
  } else {
    const int pairs = std::max(1, std::min(grid / 2, max_pairs));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    int na = 1;
    if (pdl_enabled()) {
      attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[1].val.programmaticStreamSerializationAllowed = 1;
      na = 2;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, td, tx, args);
    if (e != cudaSuccess) return e;
  }
  return cudaGetLastError();
}

template <int BN, bool A_MN, bool B_MN, int CG>
static cudaError_t dispatch_epi(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td,
                                const CUtensorMap& tx, const GemmArgs& args, int grid, cudaStream_t s) {
  switch (args.epi) {
    case EPI_BF16: return launch_one<BN, A_MN, B_MN, EPI_BF16, CG>(ta, tb, td, tx, args, grid, s);
    case EPI_F32: return launch_one<BN, A_MN, B_MN, EPI_F32, CG>(ta, tb, td, tx, args, grid, s);
    case EPI_F32_ACC: return launch_one<BN, A_MN, B_MN, EPI_F32_ACC, CG>(ta, tb, td, tx, args, grid, s);
    case EPI_GELU: return launch_one<BN, A_MN, B_MN, EPI_GELU, CG>(ta, tb, td, tx, args, grid, s);
    case EPI_RESID: return launch_one<BN, A_MN, B_MN, EPI_RESID, CG>(ta, tb, td, tx, args, grid, s);
    case EPI_DGELU: return launch_one<BN, A_MN, B_MN, EPI_DGELU, CG>(ta, tb, td, tx, args, grid, s);
    case EPI_CE_STATS: return launch_one<BN, A_MN, B_MN, EPI_CE_STATS, CG>(ta, tb, td, tx, args, grid, s);
    case EPI_F32_ATOMIC: return launch_one<BN, A_MN, B_MN, EPI_F32_ATOMIC, CG>(ta, tb, td, tx, args, grid, s);
    case EPI_PUSH_BF16: return launch_one<BN, A_MN, B_MN, EPI_PUSH_BF16, CG>(ta, tb, td, tx, args, grid, s);
  }
  return cudaErrorInvalidValue;
}

template <int BN, int CG>
static cudaError_t dispatch_major(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td,
                                  const CUtensorMap& tx, const GemmArgs& args, bool a_mn, bool b_mn, int grid,
                                  cudaStream_t s) {
  if (!a_mn && !b_mn) return dispatch_epi<BN, false, false, CG>(ta, tb, td, tx, args, grid, s);
  if (!a_mn && b_mn) return dispatch_epi<BN, false, true, CG>(ta, tb, td, tx, args, grid, s);
  if (a_mn && b_mn) return dispatch_epi<BN, true, true, CG>(ta, tb, td, tx, args, grid, s);
  return dispatch_epi<BN, true, false, CG>(ta, tb, td, tx, args, grid, s);
}

int choose_bn(int M, int N, int num_sms) {
  if (N <= 128) return 128;
  const long mt = (M + BM - 1) / BM;
  const long t256 = mt * ((N + 255) / 256), t128 = mt * ((N + 127) / 128);
  const double w256 = (double)((t256 + num_sms - 1) / num_sms) * 256.0;
  const double w128 = (double)((t128 + num_sms - 1) / num_sms) * 128.0 * 1.15;  // lower intensity per column
  return (w128 < w256) ? 128 : 256;
}

// Pick (tile width, K splits) for GEMMs whose output tiles cannot fill the
// machine (weight gradients: small M x N, long K).  Cost model in units of
// one 128x256x64 k-block: per wave, the longest unit's k-blocks plus a fixed
// epilogue charge; narrower tiles cost 15% more per column.
static void choose_split(int M, int N, int K, int num_sms, int& bn, int& splits) {
  const int kblocks = (K + BK - 1) / BK;
  double best = 1e30;
  for (int b : {256, 128}) {
    if (b == 256 && N <= 128) continue;
    const long tiles = (long)((M + BM - 1) / BM) * ((N + b - 1) / b);
    for (int sp = 1; sp <= 32; ++sp) {
      if (sp > 1 && kblocks / sp < 4) break;
      const int kps = (kblocks + sp - 1) / sp;
      const int real_sp = (kblocks + kps - 1) / kps;
      const long units = tiles * real_sp;
      const long waves = (units + num_sms - 1) / num_sms;
      const double per_unit = (b / 256.0) * (b == 128 ? 1.15 : 1.0) * (kps + (real_sp > 1 ? 4.0 : 2.0));
      const double cost = waves * per_unit;
      if (cost < best - 1e-9) {
        best = cost;
        bn = b;
        splits = real_sp;
      }
    }
  }
}

// Returns 0 on success, a negative host-side validation code, or a positive cudaError_t.
int gemm_bf16_launch(const GemmProblem& p, cudaStream_t stream) {
  if (p.M <= 0 || p.N <= 0 || p.K <= 0) return -10;
  if (p.N % 8 != 0) return -11;
  if ((reinterpret_cast<uintptr_t>(p.args.D) & 15) != 0) return -12;
  const int sms = p.num_sms > 0 ? p.num_sms : 148;
  GemmArgs args = p.args;
  args.M = p.M;
  args.N = p.N;
  args.K = p.K;
  args.splits = 1;
  int bn = p.bn > 0 ? p.bn : choose_bn(p.M, p.N, sms);
  const bool can_split = (args.epi == EPI_F32_ACC || args.epi == EPI_F32_ATOMIC) && p.allow_split;
  // CTA pairs (256 x 256 output tiles over two SMs) for 256-wide tiles with at
  // least two m-tiles; the default is in gemm_pairs_default.
  const int want_cg = p.cg > 0 ? p.cg : gemm_pairs_default(p.K, p.args.epi);
  int cg = (want_cg == 2 && p.M > BM && sms >= 2) ? 2 : 1;
  if (can_split) {
    int sbn = bn, sp = 1;
    if (cg == 2) {
      // pair units: ceil(M / 256) x n-tiles over sms / 2 pairs (same cost model, in pairs)
      choose_split((int)(((p.M + 2 * BM - 1) / (2 * BM)) * BM), p.N, p.K, sms / 2, sbn, sp);
      if ((p.bn > 0 ? p.bn : sbn) != 256) cg = 1;
    }
    if (cg == 1) {
      sbn = bn;
      sp = 1;
      choose_split(p.M, p.N, p.K, sms, sbn, sp);
    }
    if (p.bn <= 0) bn = sbn;
    if (sp > 1) {
      args.splits = sp;
      args.epi = EPI_F32_ATOMIC;
    }
  }
  if (bn != 256) cg = 1;
  CUtensorMap ta, tb;
  int rc;
  if (!p.a_mn) rc = make_tmap_bf16_2d(&ta, p.A, p.M, p.K, p.lda, 64, BM);
  else rc = make_tmap_bf16_2d(&ta, p.A, p.K, p.M, p.lda, 64, 64);
  if (rc) return rc - 20;
  // K-major B: each CTA of a pair loads its bn / 2 rows
  if (!p.b_mn) rc = make_tmap_bf16_2d(&tb, p.B, p.N, p.K, p.ldb, 64, bn / cg);
  else rc = make_tmap_bf16_2d(&tb, p.B, p.K, p.N, p.ldb, 64, 64);
  if (rc) return rc - 30;
  // output (and GELU pre-activation) maps for the TMA-store epilogue
  CUtensorMap td, tx;
  const bool out_bf16 = (args.epi == EPI_BF16 || args.epi == EPI_GELU || args.epi == EPI_DGELU ||
                         args.epi == EPI_CE_STATS);
  if (args.epi == EPI_CE_STATS && (args.ce_part == nullptr || bn != 256 || args.ce_ld < 2L * ((p.N + 255) / 256)))
    return -70;
  if (args.epi == EPI_PUSH_BF16) {
    // the epilogue writes peer slots with plain stores; this map only keeps the launch well-formed
    if (args.push_world < 1 || args.push_world > 8 || args.push_Sl % 32 != 0 || args.push_S % args.push_Sl != 0)
      return -60;
    rc = make_tmap_2d(&td, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, args.push_dst[args.push_rank], 32, p.N, args.ldd, 64,
                      32);
  } else if (out_bf16)
    rc = make_tmap_2d(&td, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, args.D, p.M, p.N, args.ldd, 64, 32);
  else rc = make_tmap_2d(&td, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, args.D, p.M, p.N, args.ldd, 32, 32);
  if (rc) return rc - 40;
  if (args.epi == EPI_GELU) {
    rc = make_tmap_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, args.aux, p.M, p.N, args.ld_aux, 64, 32);
    if (rc) return rc - 50;
  } else {
    tx = td;
  }
  const long mt = (p.M + BM - 1) / BM;
  const long units = (cg == 2 ? (mt + 1) / 2 : mt) * ((p.N + bn - 1) / bn) * args.splits;
  cudaError_t e;
  if (cg == 2) {
    const int grid = 2 * (int)std::min<long>(units, sms / 2);
    e = dispatch_major<256, 2>(ta, tb, td, tx, args, p.a_mn, p.b_mn, grid, stream);
  } else {
    const int grid = (int)std::min<long>(units, sms);
    e = (bn == 256) ? dispatch_major<256, 1>(ta, tb, td, tx, args, p.a_mn, p.b_mn, grid, stream)
                    : dispatch_major<128, 1>(ta, tb, td, tx, args, p.a_mn, p.b_mn, grid, stream);
  }
  return e == cudaSuccess ? 0 : (int)e;
}

// Default for GemmProblem::cg == 0.  MMB_GEMM_PAIRS=0: single-CTA tiles only;
// MMB_GEMM_PAIRS=1: pairs wherever eligible.  Unset: pairs for K < 32768 and the
// epilogues in MMB_GEMM_PAIR_EPI_MASK (bit e = GemmEpilogue e), except the residual
// epilogue at K <= 1024.  The default mask leaves out GELU and GELU-backward.
// Measured on B200 (GPT-125M shapes, CUDA events): the two CTAs of a pair release
// their accumulator together, so a pair runs at the pace of its slower epilogue, and
// where the epilogue is heavy against a short main loop one CTA per tile is faster
// (fc1 + GELU 90 against 96 us, fc2 dgrad + GELU-backward 74 against 80 us,
// attn-out + residual at K = 768 39 against 41 us); elsewhere pairs are faster
// (fc2 + residual at K = 3072 70 against 77 us, weight gradients 57 against 64 us),
// except for the vocabulary-long K of the lm_head input gradient.
int gemm_pairs_default(int K, int epi) {
  static const int mode = [] {
    const char* e = getenv("MMB_GEMM_PAIRS");
    if (e == nullptr || e[0] == 0) return -1;
    return e[0] == '1' ? 1 : 0;
  }();
  static const unsigned mask = [] {
    const char* e = getenv("MMB_GEMM_PAIR_EPI_MASK");
    return (e != nullptr && e[0] != 0) ? (unsigned)strtoul(e, nullptr, 0)
                                       : 0x1FFu & ~((1u << EPI_GELU) | (1u << EPI_DGELU));
  }();
  if (mode >= 0) return mode == 1 ? 2 : 1;
  if (K >= 32768 || !((mask >> epi) & 1u)) return 1;
  if (epi == EPI_RESID && K <= 1024) return 1;
  return 2;
}

}  // namespace mmb
