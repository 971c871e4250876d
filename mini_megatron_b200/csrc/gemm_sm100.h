// Host-visible interface of the tcgen05 GEMM (no torch headers here so the
// kernel translation units compile quickly and can be reused by plain C/C++).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

namespace mmb {

enum GemmEpilogue : int {
  EPI_BF16 = 0,     // D(bf16)  = alpha*acc
  EPI_F32 = 1,      // D(fp32)  = alpha*acc
  EPI_F32_ACC = 2,  // D(fp32) += alpha*acc            (gradient accumulation)
  EPI_GELU = 3,     // x = alpha*acc: D(bf16) = gelu(x), aux(bf16) = gelu'(x)  (saved for the backward)
  EPI_RESID = 4,    // D(fp32)  = resid(fp32) + alpha*acc (resid may alias D)
  EPI_DGELU = 5,    // D(bf16)  = alpha*acc * aux(bf16)          (aux = gelu'(pre) from EPI_GELU)
  EPI_F32_ATOMIC = 6,  // D(fp32) += alpha*acc with atomics (split-K partial sums)
  EPI_PUSH_BF16 = 7,   // bf16 tile -> owning TP rank's reduce-scatter slot (NVLink stores), then signal
  EPI_CE_STATS = 8,    // D(bf16) = alpha*acc, plus per-row (max, sum exp(x - max)) of the stored bf16 values of
                       // columns < ce_n_valid, one partial per (row, 256-column tile, epilogue half) in ce_part
};

struct GemmArgs {
  int M, N, K;
  int epi;
  void* D;
  long ldd;
  void* aux;
  long ld_aux;
  const float* resid;
  long ld_resid;
  float alpha;
  int* err;     // device error word (bounded-wait timeouts)
  int splits;   // K splits (set by the launcher)
  // all-gather consumer: rows of A from source rank o = (m % ag_S) / ag_Sl are
  // loaded only after ag_flags[o] >= ag_epoch (nullptr: no waiting)
  const int* ag_flags;
  int ag_epoch, ag_S, ag_Sl;
  int ag_rank;  // this rank: its own rows are computed first
  // reduce-scatter producer (EPI_PUSH_BF16): row m goes to owner o = (m % push_S) / push_Sl,
  // local row (m / push_S) * push_Sl + m % push_Sl of push_dst[o] (ld = ldd)
  void* push_dst[8];
  int* push_flags[8];
  int push_world, push_rank, push_epoch, push_S, push_Sl;
  unsigned* push_counter;
  // cross-entropy statistics (EPI_CE_STATS): ce_part[row * ce_ld + 2 * n_tile + half] = (max, sumexp)
  float2* ce_part;
  long ce_ld;
  int ce_n_valid;
};

struct GemmProblem {
  const void* A;
  long lda;
  bool a_mn;
  const void* B;
  long ldb;
  bool b_mn;
  int M, N, K;
  int bn;       // 0 = heuristic, else 128 / 256
  int num_sms;  // persistent grid size cap
  bool allow_split;  // accumulate epilogues may split K across CTAs (atomics)
  int cg;            // CTAs per output tile: 0 = default, 1 = one CTA (128 x bn), 2 = a CTA pair (256 x 256)
  GemmArgs args;
};

int make_tmap_bf16_2d(CUtensorMap* map, const void* base, long rows, long cols, long ld, int box_cols,
                      int box_rows);
int make_tmap_f32_2d(CUtensorMap* map, const void* base, long rows, long cols, long ld, int box_cols, int box_rows);
int gemm_bf16_launch(const GemmProblem& p, cudaStream_t stream);
int choose_bn(int M, int N, int num_sms);
int gemm_pairs_default(int K, int epi);

}  // namespace mmb
