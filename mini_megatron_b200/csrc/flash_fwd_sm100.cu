// Causal flash attention forward for sm_100a: two query tiles per work item,
// scores, probabilities and output accumulators all resident in TMEM.
//
// The reference calls F.scaled_dot_product_attention(is_causal=True) on
// [B, nh, S, d] views of its fused QKV projection (model/transformer.py:27-33).
// This kernel reads Q, K and V tiles straight out of the packed [B*S, 3*nh*d]
// bf16 QKV activation with TMA and writes the context in the [B*S, nh*d]
// layout the output projection consumes, plus the log-sum-exp per row for the
// backward.
//
// Persistent grid (one CTA per SM).  A work item is (batch, head, pair of
// adjacent 128-row query tiles t0 = t1 - 1, t1); items are taken heaviest
// first (longest causal rows), round-robin over the CTAs.  The two tiles share
// every K/V tile they both see.  Roles (10 warps):
//
//   warp 0     TMA: Q0, Q1 per item; K_j / V_j into an NS-stage ring
//   warp 1     TMEM allocation; one thread issues every tcgen05.mma:
//                S_i  = Q_i K_j^T              (128 x 128 fp32, TMEM)
//                O_i += P_i V_j                (128 x d fp32, TMEM; P_i read from TMEM)
//              in the order  PV0_j, S0_{j+1}, PV1_j, S1_{j+1}  so that tile 0's
//              softmax runs while the tensor core works for tile 1 and back.
//   warps 2-5  softmax of tile 0, warps 6-9 softmax of tile 1: thread r owns
//              query row r (TMEM lane r).  It loads its 128 scores, takes the
//              row maximum, writes P = exp2(S * scale * log2 e - m) as bf16
//              over the first 64 columns of its own S row, and keeps the
//              running row sum.  O is rescaled in TMEM only when the row
//              maximum grew by more than kRescaleLog2 (= a factor 256): until
//              then the stale maximum is kept, P stays <= 256 and O and the
//              row sum share the same reference, so the result is exact.  At
//              the end of the item the same warps divide O by the row sum,
//              store bf16 rows and the natural-log LSE.
//
// Ordering facts the pipeline relies on: tcgen05.mma operations of one thread
// complete in issue order, and tcgen05.commit tracks all earlier ones.  So when
// S_i(j) is complete, PV_i(j-1) (issued before it) is too, which is what lets a
// softmax warp rescale O_i after waiting only for S_i(j); and writing S_i(j+1)
// over P_i(j) is safe because PV_i(j), which reads P_i(j), was issued first.
//
// Every mbarrier wait is bounded.  On a time-out the kernel records an error
// code, every role winds down, the TMA thread waits (bounded) for the loads it
// has in flight, the MMA thread for its MMAs, TMEM is freed and the CTA returns.
#include "common.cuh"
#include "ops.h"

#include <algorithm>

namespace mmb {
namespace attn2 {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int kThreads = 320;
constexpr float kRescaleLog2 = 8.0f;

template <int D>
struct Cfg {
  static constexpr int CHUNKS = D / 64;           // 64-column (128 B) chunks per row
  static constexpr int TILE = BM * D * 2;         // bytes of one 128-row Q / K / V tile
  static constexpr int NS = (D == 64) ? 4 : 2;    // K/V ring stages
  // d = 64: P has its own TMEM columns, so S_i(j+1) can be computed while the softmax of S_i(j)
  // runs, and Q is double-buffered so the next item's tiles load during this one.  d = 128 has
  // no TMEM left for that (S 2x128 + O 2x128 = 512 columns): P overwrites S and Q is single.
  static constexpr bool SEP = (D == 64);
  static constexpr int Q_BUFS = SEP ? 2 : 1;
  static constexpr int Q_OFF = 0;                 // [Q_BUFS][Q0, Q1]
  static constexpr int K_OFF = Q_BUFS * 2 * TILE;
  static constexpr int V_OFF = K_OFF + NS * TILE;
  static constexpr int BAR_OFF = V_OFF + NS * TILE;
  static constexpr int SMEM = 1024 + BAR_OFF + 512;
  static constexpr uint32_t T_S0 = 0, T_S1 = 128, T_O0 = 256, T_O1 = 256 + D;
  static constexpr uint32_t T_P0 = SEP ? 384 : T_S0, T_P1 = SEP ? 448 : T_S1;
};

struct Args {
  int B, S, nh;
  int q_col0, k_col0, v_col0;
  __nv_bfloat16* out;
  long ld_out;
  float* lse;  // [B, nh, S], natural log
  float scale_log2;
  int* err;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void tmem_st_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Warp-wide bounded wait: every lane polls the barrier (cheaper than one lane polling while
// the others wait on a shuffle); the warp proceeds only if every lane saw the phase complete.
__device__ __forceinline__ bool wwait(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag) {
  const bool ok = mbar_wait(bar, parity, err, kErrAttnWait, abort_flag);
  return __all_sync(0xffffffffu, ok) != 0;
}

// Bounded wait used while winding down after an abort (does not look at the abort flag).
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity) && globaltimer() - t0 < 20000000ull) {
  }
}

// One arrival per warp on `bar`, after every lane's tcgen05 loads / stores are ordered before it.
__device__ __forceinline__ void warp_arrive(uint64_t* bar) {
  tc_fence_before();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

struct Item {
  int b, h, t0, t1;  // t0 < 0: the item has only tile t1 (odd number of query tiles)
};

__device__ __forceinline__ Item decode(int item, int BH, int nh, int n_qt) {
  const int n_pairs = (n_qt + 1) / 2;
  const int pr = item / BH, bh = item % BH;
  const int p = n_pairs - 1 - pr;  // heaviest pair first
  Item it;
  it.b = bh / nh;
  it.h = bh % nh;
  it.t1 = (n_qt & 1) ? 2 * p : 2 * p + 1;
  it.t0 = it.t1 - 1;
  return it;
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)  // 10 warps: 3 on some SM sub-partitions -> <= 168 registers
    flash_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_qkv, const Args a) {
  pdl_trigger();
  using C = Cfg<D>;
  constexpr int NS = C::NS;
  constexpr int QB = C::Q_BUFS;
  constexpr bool SEP = C::SEP;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sQ = smem + C::Q_OFF;
  uint8_t* sK = smem + C::K_OFF;
  uint8_t* sV = smem + C::V_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* q_full = bars + 0;            // [2]
  uint64_t* q_empty = bars + 2;           // [2]
  uint64_t* k_full = bars + 4;            // [NS]
  uint64_t* k_empty = k_full + NS;        // [NS]
  uint64_t* v_full = k_empty + NS;        // [NS]
  uint64_t* v_empty = v_full + NS;        // [NS]
  uint64_t* s_full = v_empty + NS;        // [2]  S_i computed
  uint64_t* s_free = s_full + 2;          // [2]  S_i read into registers (SEP only; one arrival per warp)
  uint64_t* p_full = s_free + 2;          // [2]  P_i written (one arrival per softmax warp)
  uint64_t* p_free = p_full + 2;          // [2]  PV_i that read P_i complete (SEP only)
  uint64_t* o_full = p_free + 2;          // [2]  last PV_i of the item complete
  uint64_t* o_free = o_full + 2;          // [2]  O_i read by the epilogue (one arrival per softmax warp)
  uint64_t* drain = o_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = a.S / BM;
  const int BH = a.B * a.nh;
  const int n_items = BH * ((n_qt + 1) / 2);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&p_free[i], 1);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 4);
    }
    for (int s = 0; s < NS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_qkv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();  // the set-up above touched no global memory
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int kv = 0, it = 0;
      bool ok = true;
      int q_issued = -1;  // item count of the last Q load
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++it) {
        const Item w = decode(item, BH, a.nh, n_qt);
        const int row0 = w.b * a.S;
        const int qx = a.q_col0 + w.h * D, kx = a.k_col0 + w.h * D, vx = a.v_col0 + w.h * D;
        const int qb = it % QB;
        if (it >= QB && !mbar_wait(&q_empty[qb], ((it / QB) - 1) & 1, a.err, kErrAttnWait, abort_flag)) {
          ok = false;
          break;
        }
        uint8_t* qd = sQ + qb * 2 * C::TILE;
        mbar_expect_tx(&q_full[qb], (w.t0 >= 0 ? 2 : 1) * C::TILE);
#pragma unroll
        for (int c = 0; c < C::CHUNKS; ++c) {
          if (w.t0 >= 0) tma_load_2d(qd + c * 16384, &tm_qkv, &q_full[qb], qx + 64 * c, row0 + w.t0 * BM);
          tma_load_2d(qd + C::TILE + c * 16384, &tm_qkv, &q_full[qb], qx + 64 * c, row0 + w.t1 * BM);
        }
        q_issued = it;
        const int J = w.t1 + 1;
        for (int j = 0; j < J; ++j, ++kv) {
          const int s = kv % NS, n = kv / NS;
          if (n > 0 && !mbar_wait(&k_empty[s], (n - 1) & 1, a.err, kErrAttnWait, abort_flag)) { ok = false; break; }
          mbar_expect_tx(&k_full[s], C::TILE);
#pragma unroll
          for (int c = 0; c < C::CHUNKS; ++c)
            tma_load_2d(sK + s * C::TILE + c * 16384, &tm_qkv, &k_full[s], kx + 64 * c, row0 + j * BN);
          if (n > 0 && !mbar_wait(&v_empty[s], (n - 1) & 1, a.err, kErrAttnWait, abort_flag)) {
            ++kv;  // the K load of this slot is in flight
            ok = false;
            break;
          }
          mbar_expect_tx(&v_full[s], C::TILE);
#pragma unroll
          for (int c = 0; c < C::CHUNKS; ++c)
            tma_load_2d(sV + s * C::TILE + c * 16384, &tm_qkv, &v_full[s], vx + 64 * c, row0 + j * BN);
        }
      }
      if (!ok) {
        // let the loads this thread issued land before the CTA's shared memory goes away
        for (int u = std::max(0, q_issued - QB + 1); u <= q_issued; ++u) drain_wait(&q_full[u % QB], (u / QB) & 1);
        for (int u = std::max(0, kv - NS); u < kv; ++u) {
          drain_wait(&k_full[u % NS], (u / NS) & 1);
          drain_wait(&v_full[u % NS], (u / NS) & 1);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(BM, BN, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16(BM, D, false, true);
      int kv = 0, it = 0;
      int sc[2] = {0, 0};  // S_i issued per group (s_free phases)
      int pc[2] = {0, 0};  // P_i consumed per group (p_full phases)
      int ic[2] = {0, 0};  // items with an active tile per group (o_free phases)
      bool ok = true;
      // S_i = Q_i K^T into the S columns of group i (SEP: once the softmax has read the previous S_i)
      auto issue_s = [&](int i, uint32_t qa, int stage) -> bool {
        if (SEP && sc[i] > 0 && !mbar_wait(&s_free[i], (sc[i] - 1) & 1, a.err, kErrAttnWait, abort_flag))
          return false;
        ++sc[i];
        tc_fence_after();
        const uint32_t dst = tmem + (i == 0 ? C::T_S0 : C::T_S1);
        // the start-address field is (address >> 4) in the low 14 bits: per-step offsets are added to it
        const uint64_t qd = make_sdesc_sw128(qa, 16, 1024);
        const uint64_t kd = make_sdesc_sw128(smem_u32(sK + stage * C::TILE), 16, 1024);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off16 = ((k >> 2) * 16384 + (k & 3) * 32) >> 4;
          umma_bf16_ss(dst, qd + off16, kd + off16, idesc_s, k != 0 ? 1u : 0u);
        }
        umma_commit(&s_full[i]);
        return true;
      };
      // O_i (+)= P_i V once the softmax has written P_i (and, for the first tile of an item, once the
      // previous item's epilogue has read O_i)
      auto issue_pv = [&](int i, int stage, bool first, bool last) -> bool {
        if (!mbar_wait(&p_full[i], pc[i] & 1, a.err, kErrAttnWait, abort_flag)) return false;
        ++pc[i];
        if (first && ic[i] > 0 && !mbar_wait(&o_free[i], (ic[i] - 1) & 1, a.err, kErrAttnWait, abort_flag))
          return false;
        tc_fence_after();
        const uint64_t vd = make_sdesc_sw128(smem_u32(sV + stage * C::TILE), 16384, 1024);
        const uint32_t p_t = tmem + (i == 0 ? C::T_P0 : C::T_P1);
        const uint32_t o_t = tmem + (i == 0 ? C::T_O0 : C::T_O1);
#pragma unroll
        for (int k = 0; k < BN / 16; ++k)
          umma_bf16_ts(o_t, p_t + k * 8, vd + (uint64_t)(k * (2048 >> 4)), idesc_o, (!first || k != 0) ? 1u : 0u);
        if (SEP) umma_commit(&p_free[i]);
        if (last) umma_commit(&o_full[i]);
        return true;
      };
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++it) {
        const Item w = decode(item, BH, a.nh, n_qt);
        const bool act0 = w.t0 >= 0;
        const int J = w.t1 + 1;
        const int qb = it % QB;
        const uint32_t q0 = smem_u32(sQ + qb * 2 * C::TILE), q1 = q0 + C::TILE;
        if (!mbar_wait(&q_full[qb], (it / QB) & 1, a.err, kErrAttnWait, abort_flag)) { ok = false; break; }
        if (!mbar_wait(&k_full[kv % NS], (kv / NS) & 1, a.err, kErrAttnWait, abort_flag)) { ok = false; break; }
        if (act0 && !issue_s(0, q0, kv % NS)) { ok = false; break; }
        if (!issue_s(1, q1, kv % NS)) { ok = false; break; }
        umma_commit(&k_empty[kv % NS]);
        for (int j = 0; j < J && ok; ++j) {
          const int st = (kv + j) % NS, ph = ((kv + j) / NS) & 1;
          const int st1 = (kv + j + 1) % NS, ph1 = ((kv + j + 1) / NS) & 1;
          const bool t0_now = act0 && j <= w.t0, t0_next = act0 && j + 1 <= w.t0;
          if (SEP) {
            // next scores first: they only need the softmax to have read the current ones
            if (j + 1 < J) {
              if (!mbar_wait(&k_full[st1], ph1, a.err, kErrAttnWait, abort_flag)) { ok = false; break; }
              if (t0_next && !issue_s(0, q0, st1)) { ok = false; break; }
              if (!issue_s(1, q1, st1)) { ok = false; break; }
              umma_commit(&k_empty[st1]);
            }
            if (!mbar_wait(&v_full[st], ph, a.err, kErrAttnWait, abort_flag)) { ok = false; break; }
            if (t0_now && !issue_pv(0, st, j == 0, j == w.t0)) { ok = false; break; }
            if (!issue_pv(1, st, j == 0, j == J - 1)) { ok = false; break; }
            umma_commit(&v_empty[st]);
          } else {
            // P_i overwrites S_i: order PV0_j, S0_{j+1}, PV1_j, S1_{j+1} (tile 0's softmax overlaps tile 1's MMAs)
            if (!mbar_wait(&v_full[st], ph, a.err, kErrAttnWait, abort_flag)) { ok = false; break; }
            if (t0_now) {
              if (!issue_pv(0, st, j == 0, j == w.t0)) { ok = false; break; }
              if (t0_next) {
                if (!mbar_wait(&k_full[st1], ph1, a.err, kErrAttnWait, abort_flag)) { ok = false; break; }
                if (!issue_s(0, q0, st1)) { ok = false; break; }
              }
            }
            if (!issue_pv(1, st, j == 0, j == J - 1)) { ok = false; break; }
            umma_commit(&v_empty[st]);
            if (j + 1 < J) {
              if (!mbar_wait(&k_full[st1], ph1, a.err, kErrAttnWait, abort_flag)) { ok = false; break; }
              if (!issue_s(1, q1, st1)) { ok = false; break; }
              umma_commit(&k_empty[st1]);
            }
          }
        }
        umma_commit(&q_empty[qb]);  // every S MMA of this item has been issued
        kv += J;
        if (act0) ++ic[0];
        ++ic[1];
      }
      if (!ok) {
        umma_commit(drain);
        drain_wait(drain, 0);
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    const int grp = (warp - 2) >> 2;          // 0: tile t0, 1: tile t1
    const int q = warp & 3;                   // TMEM lane quarter of this warp
    const int r = q * 32 + lane;              // query row within the tile (TMEM lane)
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const uint32_t t_s = tmem + (grp == 0 ? C::T_S0 : C::T_S1) + lane_off;
    const uint32_t t_p = tmem + (grp == 0 ? C::T_P0 : C::T_P1) + lane_off;
    const uint32_t t_o = tmem + (grp == 0 ? C::T_O0 : C::T_O1) + lane_off;
    const float sl2 = a.scale_log2;
    int sc = 0, pc = 0, ic = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      const Item w = decode(item, BH, a.nh, n_qt);
      const int t = grp == 0 ? w.t0 : w.t1;
      if (t < 0) continue;
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j <= t; ++j) {
        if (!wwait(&s_full[grp], sc & 1, a.err, abort_flag)) { ok = false; break; }
        ++sc;
        tc_fence_after();
        uint32_t s[128];
        tmem_ld_32x32b_x32(t_s + 0, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
        tmem_ld_32x32b_x32(t_s + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32]));
        tmem_ld_32x32b_x32(t_s + 64, *reinterpret_cast<uint32_t(*)[32]>(&s[64]));
        tmem_ld_32x32b_x32(t_s + 96, *reinterpret_cast<uint32_t(*)[32]>(&s[96]));
        tmem_wait_ld();
        if (SEP) warp_arrive(&s_free[grp]);  // the next S_i may now be computed into these columns
        if (j == t) {  // diagonal tile: key column c is visible to query row r iff c <= r
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c > r) s[c] = __float_as_uint(-INFINITY);
        }
        float mx[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) mx[k] = __uint_as_float(s[k]);
#pragma unroll
        for (int c = 8; c < 128; ++c) mx[c & 7] = fmaxf(mx[c & 7], __uint_as_float(s[c]));
        const float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                               fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * sl2;
        const bool need = mt > m + kRescaleLog2;
        const bool any_need = __any_sync(0xffffffffu, need) != 0;
        float alpha = 1.f;
        if (need) {
          alpha = ex2(m - mt);  // m = -inf on the first tile: alpha = 0
          m = mt;
        }
        if (SEP) {
          // the PV that read the previous P_i (and last wrote O_i) must be complete
          if (pc > 0 && !wwait(&p_free[grp], (pc - 1) & 1, a.err, abort_flag)) { ok = false; break; }
          tc_fence_after();
        }
        ++pc;
        // P = exp2(S * sl2 - m) as bf16 pairs (64 TMEM columns: SEP its own, else over the first half of S)
        float rs[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) rs[k] = 0.f;
#pragma unroll
        for (int hcol = 0; hcol < 2; ++hcol) {
          uint32_t pk[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int c = hcol * 64 + 2 * e;
            const float p0 = ex2(fmaf(__uint_as_float(s[c]), sl2, -m));
            const float p1 = ex2(fmaf(__uint_as_float(s[c + 1]), sl2, -m));
            rs[e & 7] += p0 + p1;
            pk[e] = pack_bf16x2(p0, p1);
          }
          tmem_st_x32(t_p + hcol * 32, pk);
        }
        l = l * alpha + (((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7])));
        if (any_need && j > 0) {
          // PV_i(j-1) is complete (SEP: waited above; otherwise it was issued before S_i(j)):
          // rescale this row of O in place before PV_i(j) adds the new tile
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            tmem_ld_32x32b_x32(t_o + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st_x32(t_o + c * 32, o);
          }
        }
        tmem_wait_st();
        warp_arrive(&p_full[grp]);
      }
      if (!ok) break;
      // epilogue: O / l -> bf16 row, LSE
      if (!wwait(&o_full[grp], ic & 1, a.err, abort_flag)) { ok = false; break; }
      ++ic;
      tc_fence_after();
      const float inv = 1.f / l;
      const long row = (long)w.b * a.S + (long)t * BM + r;
      __nv_bfloat16* orow = a.out + row * a.ld_out + w.h * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(t_o + c * 32, o);
        tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 v;
          v.x = pack_bf16x2(__uint_as_float(o[8 * u + 0]) * inv, __uint_as_float(o[8 * u + 1]) * inv);
          v.y = pack_bf16x2(__uint_as_float(o[8 * u + 2]) * inv, __uint_as_float(o[8 * u + 3]) * inv);
          v.z = pack_bf16x2(__uint_as_float(o[8 * u + 4]) * inv, __uint_as_float(o[8 * u + 5]) * inv);
          v.w = pack_bf16x2(__uint_as_float(o[8 * u + 6]) * inv, __uint_as_float(o[8 * u + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + c * 32 + 8 * u) = v;
        }
      }
      a.lse[((size_t)w.b * a.nh + w.h) * a.S + (size_t)t * BM + r] = m * 0.69314718055994531f + logf(l);
      warp_arrive(&o_free[grp]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace attn2

int flash_attn_fwd_sm100(const __nv_bfloat16* qkv, long ld_qkv, int B, int S, int nh, int d, __nv_bfloat16* out,
                         long ld_out, float* lse, float softmax_scale, int* err, int num_sms, cudaStream_t stream) {
  using namespace attn2;
  if (S % BM != 0 || (d != 64 && d != 128)) return -1;
  if ((reinterpret_cast<uintptr_t>(out) & 15) || (ld_out % 8)) return -2;
  CUtensorMap tm;
  const long rows = (long)B * S, cols = 3L * nh * d;
  int rc = make_tmap_bf16_2d(&tm, qkv, rows, cols, ld_qkv, 64, BM);
  if (rc) return rc - 10;
  Args a;
  a.B = B;
  a.S = S;
  a.nh = nh;
  a.q_col0 = 0;
  a.k_col0 = nh * d;
  a.v_col0 = 2 * nh * d;
  a.out = out;
  a.ld_out = ld_out;
  a.lse = lse;
  a.scale_log2 = softmax_scale * 1.4426950408889634f;
  a.err = err;
  const int n_items = B * nh * ((S / BM + 1) / 2);
  const int grid = std::max(1, std::min(n_items, num_sms));
  if (d == 64) {
    auto k = flash_fwd_sm100_kernel<64>;
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<64>::SMEM);
      set = true;
    }
    launch_k(k, grid, kThreads, Cfg<64>::SMEM, stream, tm, a);
  } else {
    auto k = flash_fwd_sm100_kernel<128>;
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<128>::SMEM);
      set = true;
    }
    launch_k(k, grid, kThreads, Cfg<128>::SMEM, stream, tm, a);
  }
  return (int)cudaGetLastError();
}

}  // namespace mmb
