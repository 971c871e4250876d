// Causal flash attention backward for head_dim 64 on sm_100a: persistent,
// key/value-stationary, with the next query tile's score MMAs running while
// the current tile's softmax gradient is computed.
//
// The reference differentiates F.scaled_dot_product_attention(is_causal=True)
// through autograd (model/transformer.py:27-33).  Inputs here are the packed
// [B*S, 3*nh*64] bf16 QKV activation, dO [B*S, nh*64], the forward's LSE and
// Delta = rowsum(dO * O); dK and dV are written into the packed dQKV output,
// dQ is accumulated in fp32 with TMA bulk reduce-adds (converted afterwards).
//
// Work item = (batch, head, key tile j): K_j and V_j stay in shared memory
// while the CTA walks the query tiles i = j .. S/128-1 that see them; items
// are taken heaviest first (j = 0 has the most query tiles), round-robin over
// one CTA per SM.  Roles (10 warps):
//
//   warp 0     TMA: K_j, V_j per item; Q_i, dO_i and their LSE / Delta rows
//              into a 3-stage ring
//   warp 1     TMEM allocation; one thread issues the tcgen05.mma:
//                S^T  = K_j Q_i^T,  dP^T = V_j dO_i^T        (128 x 128 fp32 each)
//                dV  += P^T dO_i   (P^T read from TMEM)      (128 x 64)
//                dK  += dS^T Q_i,  dQ_i = dS K_j             (dS^T from shared memory)
//              S^T / dP^T of tile i+1 are issued as soon as the softmax warps
//              have read tile i's into registers.
//   warps 2-9  softmax gradient: warps w and w+4 share a TMEM lane quarter
//              (key rows) and split the 128 query columns.  P^T = exp2(S^T *
//              scale * log2 e - LSE * log2 e) (causal mask on the diagonal
//              tile), dS^T = P^T * (dP^T - Delta); P^T goes to TMEM as bf16,
//              dS^T to 128B-swizzled shared memory (read K-major for dK and
//              MN-major for dQ).  Before writing tile i they drain dQ_{i-1}
//              from TMEM through a per-warp staging tile into a TMA reduce-add,
//              and at the end of an item they store dK (scaled) and dV.
//
// TMEM columns: S^T [0,128) dP^T [128,256) dV [256,320) dK [320,384)
// dQ [384,448) P^T [448,512).  Every mbarrier wait is bounded; on a time-out
// the kernel records an error code, all roles wind down, the TMA thread waits
// (bounded) for its loads in flight, the MMA thread for its MMAs, TMEM is
// freed and the CTA returns.
#include "common.cuh"
#include "ops.h"

#include <algorithm>

namespace mmb {
namespace attnb {

constexpr int D = 64;
constexpr int BM = 128;  // query rows per tile
constexpr int BN = 128;  // key rows per tile
constexpr int kThreads = 320;
constexpr int TILE = BM * D * 2;  // 16 KB
constexpr int QS = 3;             // Q / dO ring stages (loads of tile i+3 overlap tiles i+1, i+2)
constexpr int KB = 1;             // K / V buffer (a new item's K / V load after the last tile's MMAs)
constexpr int K_OFF = 0;                        // [KB][K, V]
constexpr int Q_OFF = K_OFF + KB * 2 * TILE;    // [QS][Q, dO]
constexpr int DS_OFF = Q_OFF + QS * 2 * TILE;   // dS^T [128 keys x 128 queries] bf16: 2 chunks of 16 KB
constexpr int LD_OFF = DS_OFF + 2 * TILE;       // [QS][lse 128, delta 128] fp32
constexpr int ST_OFF = LD_OFF + QS * 1024;      // 8 warps x 4 KB dQ staging
constexpr int BAR_OFF = ST_OFF + 8 * 4096;
constexpr int SMEM = 1024 + BAR_OFF + 512;
constexpr uint32_t T_ST = 0, T_DPT = 128, T_DV = 256, T_DK = 320, T_DQ = 384, T_PT = 448;

struct Args {
  int B, S, nh;
  int q_col0, k_col0, v_col0;
  const float* lse;     // [B, nh, S] natural log
  const float* delta;   // [B, nh, S]
  __nv_bfloat16* dqkv;  // [B*S, 3*nh*D]
  long ld_dqkv;
  float scale;
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

__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity) && globaltimer() - t0 < 20000000ull) {
  }
}

__device__ __forceinline__ void warp_arrive(uint64_t* bar) {
  tc_fence_before();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

struct Item {
  int b, h, j;
};

__device__ __forceinline__ Item decode(int item, int BH, int nh) {
  Item it;
  it.j = item / BH;  // key tile: j = 0 (the most query tiles) first
  const int bh = item % BH;
  it.b = bh / nh;
  it.h = bh % nh;
  return it;
}

__global__ void __launch_bounds__(kThreads, 1)
    flash_bwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_do,
                           const __grid_constant__ CUtensorMap tm_dq, const Args a) {
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sKV = smem + K_OFF;
  uint8_t* sQ = smem + Q_OFF;
  uint8_t* sDS = smem + DS_OFF;
  float* sLD = reinterpret_cast<float*>(smem + LD_OFF);
  uint8_t* sST = smem + ST_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* kv_full = bars + 0;    // [KB]
  uint64_t* kv_empty = bars + 2;   // [KB]
  uint64_t* q_full = bars + 4;     // [QS]
  uint64_t* q_empty = bars + 8;    // [QS]
  uint64_t* st_full = bars + 12;   // S^T, dP^T computed
  uint64_t* st_free = bars + 13;   // S^T, dP^T read into registers (8 warps)
  uint64_t* ps_full = bars + 14;   // P^T (TMEM) and dS^T (smem) written (8 warps)
  uint64_t* grads = bars + 15;     // dV, dK, dQ MMAs of a tile complete (commit)
  uint64_t* dq_free = bars + 16;   // dQ drained from TMEM (8 warps)
  uint64_t* dkv_free = bars + 17;  // dK, dV of an item read by the epilogue (8 warps)
  uint64_t* drain = bars + 18;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 19);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = a.S / BM;
  const int BH = a.B * a.nh;
  const int n_items = BH * n_qt;

  if (threadIdx.x == 0) {
    for (int i = 0; i < KB; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < QS; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    mbar_init(st_full, 1);
    mbar_init(st_free, 8);
    mbar_init(ps_full, 8);
    mbar_init(grads, 1);
    mbar_init(dq_free, 8);
    mbar_init(dkv_free, 8);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_qkv);
    prefetch_tmap(&tm_do);
    prefetch_tmap(&tm_dq);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0, qi = 0;  // items, query tiles loaded by this CTA
      bool ok = true;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++it) {
        const Item w = decode(item, BH, a.nh);
        const int row0 = w.b * a.S;
        const int kb = it % KB;
        if (it >= KB && !mbar_wait(&kv_empty[kb], ((it / KB) - 1) & 1, a.err, kErrAttnWait, abort_flag)) {
          ok = false;
          break;
        }
        mbar_expect_tx(&kv_full[kb], 2 * TILE);
        tma_load_2d(sKV + kb * 2 * TILE, &tm_qkv, &kv_full[kb], a.k_col0 + w.h * D, row0 + w.j * BN);
        tma_load_2d(sKV + kb * 2 * TILE + TILE, &tm_qkv, &kv_full[kb], a.v_col0 + w.h * D, row0 + w.j * BN);
        const size_t ld_off = ((size_t)w.b * a.nh + w.h) * a.S;
        for (int i = w.j; i < n_qt; ++i, ++qi) {
          const int st = qi % QS;
          if (qi >= QS && !mbar_wait(&q_empty[st], ((qi / QS) - 1) & 1, a.err, kErrAttnWait, abort_flag)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&q_full[st], 2 * TILE + 1024);
          tma_load_2d(sQ + st * 2 * TILE, &tm_qkv, &q_full[st], a.q_col0 + w.h * D, row0 + i * BM);
          tma_load_2d(sQ + st * 2 * TILE + TILE, &tm_do, &q_full[st], w.h * D, row0 + i * BM);
          bulk_load(sLD + st * 256, a.lse + ld_off + (size_t)i * BM, 512, &q_full[st]);
          bulk_load(sLD + st * 256 + 128, a.delta + ld_off + (size_t)i * BM, 512, &q_full[st]);
        }
      }
      if (!ok) {
        for (int u = std::max(0, it - KB + 1); u <= it; ++u) drain_wait(&kv_full[u % KB], (u / KB) & 1);
        for (int u = std::max(0, qi - QS); u < qi; ++u) drain_wait(&q_full[u % QS], (u / QS) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(BN, BM, false, false);   // S^T, dP^T
      constexpr uint32_t idesc_kv = make_idesc_bf16(BN, D, false, true);    // dV (A in TMEM), dK
      constexpr uint32_t idesc_q = make_idesc_bf16(BM, D, true, true);      // dQ: A = dS (MN-major view)
      const uint64_t ds_k = make_sdesc_sw128(smem_u32(sDS), 16, 1024);      // dS^T, K-major
      const uint64_t ds_mn = make_sdesc_sw128(smem_u32(sDS), 16384, 1024);  // dS^T read as dS (MN-major)
      int it = 0, qi = 0, g = 0;  // items, query tiles issued, tiles whose grads were issued
      bool ok = true;
      auto issue_st = [&](int qtile, int kb) -> bool {
        const int st = qtile % QS;
        if (!mbar_wait(&q_full[st], (qtile / QS) & 1, a.err, kErrAttnWait, abort_flag)) return false;
        if (qtile > 0 && !mbar_wait(st_free, (qtile - 1) & 1, a.err, kErrAttnWait, abort_flag)) return false;
        tc_fence_after();
        const uint64_t kd = make_sdesc_sw128(smem_u32(sKV + kb * 2 * TILE), 16, 1024);
        const uint64_t vd = make_sdesc_sw128(smem_u32(sKV + kb * 2 * TILE + TILE), 16, 1024);
        const uint64_t qd = make_sdesc_sw128(smem_u32(sQ + st * 2 * TILE), 16, 1024);
        const uint64_t od = make_sdesc_sw128(smem_u32(sQ + st * 2 * TILE + TILE), 16, 1024);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) umma_bf16_ss(tmem + T_ST, kd + 2 * k, qd + 2 * k, idesc_s, k != 0);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) umma_bf16_ss(tmem + T_DPT, vd + 2 * k, od + 2 * k, idesc_s, k != 0);
        umma_commit(st_full);
        return true;
      };
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++it) {
        const Item w = decode(item, BH, a.nh);
        const int kb = it % KB;
        const int NI = n_qt - w.j;
        if (!mbar_wait(&kv_full[kb], (it / KB) & 1, a.err, kErrAttnWait, abort_flag)) { ok = false; break; }
        if (!issue_st(qi, kb)) { ok = false; break; }
        const uint64_t kmn = make_sdesc_sw128(smem_u32(sKV + kb * 2 * TILE), 16384, 1024);
        for (int i = 0; i < NI; ++i, ++qi, ++g) {
          const int st = qi % QS;
          if (i + 1 < NI && !issue_st(qi + 1, kb)) { ok = false; break; }
          if (!mbar_wait(ps_full, g & 1, a.err, kErrAttnWait, abort_flag)) { ok = false; break; }
          if (g > 0 && !mbar_wait(dq_free, (g - 1) & 1, a.err, kErrAttnWait, abort_flag)) { ok = false; break; }
          if (i == 0 && it > 0 && !mbar_wait(dkv_free, (it - 1) & 1, a.err, kErrAttnWait, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t qmn = make_sdesc_sw128(smem_u32(sQ + st * 2 * TILE), 16384, 1024);
          const uint64_t omn = make_sdesc_sw128(smem_u32(sQ + st * 2 * TILE + TILE), 16384, 1024);
#pragma unroll
          for (int k = 0; k < BM / 16; ++k) {  // reduction over the 128 query rows of tile i
            const uint32_t a_off16 = ((k >> 2) * 16384 + (k & 3) * 32) >> 4;
            umma_bf16_ts(tmem + T_DV, tmem + T_PT + k * 8, omn + k * (2048 >> 4), idesc_kv, (i > 0 || k > 0));
            umma_bf16_ss(tmem + T_DK, ds_k + a_off16, qmn + k * (2048 >> 4), idesc_kv, (i > 0 || k > 0));
          }
#pragma unroll
          for (int k = 0; k < BN / 16; ++k)  // reduction over the 128 key rows of tile j
            umma_bf16_ss(tmem + T_DQ, ds_mn + k * (2048 >> 4), kmn + k * (2048 >> 4), idesc_q, k != 0);
          umma_commit(grads);
          umma_commit(&q_empty[st]);
        }
        if (ok) umma_commit(&kv_empty[kb]);
      }
      if (!ok) {
        umma_commit(drain);
        drain_wait(drain, 0);
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax gradient, dQ drain, dK/dV
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;          // which 64 query columns (and which 32 of the 64 dQ/dK/dV columns)
    const int c = q * 32 + lane;               // key row within the tile (TMEM lane)
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const float sl2 = a.scale_log2;
    uint8_t* stg = sST + (warp - 2) * 4096;
    int qi = 0, g = 0, it = 0;
    bool ok = true;

    // dQ of a finished tile: TMEM -> per-warp 32x32 fp32 staging tile -> one TMA bulk reduce-add
    auto drain_dq = [&](int qrow0, int h) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(tmem + T_DQ + lane_off + half * 32, v);
      tmem_wait_ld();
      if (lane == 0) bulk_wait_read<0>();  // the staging tile's previous reduce-add has read it
      __syncwarp();
#pragma unroll
      for (int u = 0; u < 8; ++u)
        *reinterpret_cast<float4*>(stg + lane * 128 + ((u ^ (lane & 7)) << 4)) =
            make_float4(__uint_as_float(v[4 * u]) * a.scale, __uint_as_float(v[4 * u + 1]) * a.scale,
                        __uint_as_float(v[4 * u + 2]) * a.scale, __uint_as_float(v[4 * u + 3]) * a.scale);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_reduce_add_2d(&tm_dq, stg, h * D + half * 32, qrow0 + q * 32);
        bulk_commit();
      }
    };

    int prev_qrow = -1, prev_h = 0;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++it) {
      const Item w = decode(item, BH, a.nh);
      const int NI = n_qt - w.j;
      const int row0 = w.b * a.S;
      for (int i = 0; i < NI; ++i, ++qi, ++g) {
        const int st = qi % QS;
        if (!wwait(st_full, qi & 1, a.err, abort_flag)) { ok = false; break; }
        if (!wwait(&q_full[st], (qi / QS) & 1, a.err, abort_flag)) { ok = false; break; }  // LSE / Delta rows
        tc_fence_after();
        const float* lse = sLD + st * 256 + half * 64;
        const float* dlt = lse + 128;
        const bool diag = (i == 0);
        uint32_t pp[32], dd[32];
        // two passes of 32 query columns keep the live registers near 128 (no spills at 168)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t sv[32], dv[32];
          tmem_ld_32x32b_x32(tmem + T_ST + lane_off + half * 64 + hh * 32, sv);
          tmem_ld_32x32b_x32(tmem + T_DPT + lane_off + half * 64 + hh * 32, dv);
          tmem_wait_ld();
          if (hh == 1) warp_arrive(st_free);  // the next tile's S^T / dP^T may now be computed
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const int col = hh * 32 + e;       // column within this warp's 64
            const int qc = half * 64 + col;    // query column within the tile
            float p0 = ex2(fmaf(__uint_as_float(sv[e]), sl2, -lse[col] * 1.4426950408889634f));
            float p1 = ex2(fmaf(__uint_as_float(sv[e + 1]), sl2, -lse[col + 1] * 1.4426950408889634f));
            if (diag && qc < c) p0 = 0.f;
            if (diag && qc + 1 < c) p1 = 0.f;
            const float d0 = p0 * (__uint_as_float(dv[e]) - dlt[col]);
            const float d1 = p1 * (__uint_as_float(dv[e + 1]) - dlt[col + 1]);
            pp[col >> 1] = pack_bf16x2(p0, p1);
            dd[col >> 1] = pack_bf16x2(d0, d1);
          }
        }
        // the previous tile's dV/dK/dQ MMAs must be done reading P^T and dS^T; within an item, its dQ
        // is drained here (the last tile of an item was waited for and drained at the item's end)
        if (i > 0) {
          if (!wwait(grads, (g - 1) & 1, a.err, abort_flag)) { ok = false; break; }
          tc_fence_after();
          drain_dq(prev_qrow, prev_h);
          warp_arrive(dq_free);
        }
        // P^T -> TMEM (bf16 pairs of query columns), dS^T -> swizzled shared memory
        tmem_st_x32(tmem + T_PT + lane_off + half * 32, pp);
        uint8_t* ds_row = sDS + half * 16384 + c * 128;
#pragma unroll
        for (int u = 0; u < 8; ++u)
          *reinterpret_cast<uint4*>(ds_row + ((u ^ (c & 7)) << 4)) =
              make_uint4(dd[4 * u], dd[4 * u + 1], dd[4 * u + 2], dd[4 * u + 3]);
        tmem_wait_st();
        fence_proxy_async_smem();
        warp_arrive(ps_full);
        prev_qrow = row0 + (w.j + i) * BM;
        prev_h = w.h;
      }
      if (!ok) break;
      // end of the item: the last tile's dQ, then dK (scaled) and dV
      if (!wwait(grads, (g - 1) & 1, a.err, abort_flag)) { ok = false; break; }
      tc_fence_after();
      drain_dq(prev_qrow, prev_h);
      {
        uint32_t kv[32], vv[32];
        tmem_ld_32x32b_x32(tmem + T_DK + lane_off + half * 32, kv);
        tmem_ld_32x32b_x32(tmem + T_DV + lane_off + half * 32, vv);
        tmem_wait_ld();
        warp_arrive(dq_free);   // dQ columns read
        warp_arrive(dkv_free);  // dK / dV columns read
        const size_t row = (size_t)(row0 + w.j * BN + c);
        __nv_bfloat16* dk = a.dqkv + row * a.ld_dqkv + a.k_col0 + w.h * D + half * 32;
        __nv_bfloat16* dvp = a.dqkv + row * a.ld_dqkv + a.v_col0 + w.h * D + half * 32;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 wk, wv;
          wk.x = pack_bf16x2(__uint_as_float(kv[8 * u + 0]) * a.scale, __uint_as_float(kv[8 * u + 1]) * a.scale);
          wk.y = pack_bf16x2(__uint_as_float(kv[8 * u + 2]) * a.scale, __uint_as_float(kv[8 * u + 3]) * a.scale);
          wk.z = pack_bf16x2(__uint_as_float(kv[8 * u + 4]) * a.scale, __uint_as_float(kv[8 * u + 5]) * a.scale);
          wk.w = pack_bf16x2(__uint_as_float(kv[8 * u + 6]) * a.scale, __uint_as_float(kv[8 * u + 7]) * a.scale);
          wv.x = pack_bf16x2(__uint_as_float(vv[8 * u + 0]), __uint_as_float(vv[8 * u + 1]));
          wv.y = pack_bf16x2(__uint_as_float(vv[8 * u + 2]), __uint_as_float(vv[8 * u + 3]));
          wv.z = pack_bf16x2(__uint_as_float(vv[8 * u + 4]), __uint_as_float(vv[8 * u + 5]));
          wv.w = pack_bf16x2(__uint_as_float(vv[8 * u + 6]), __uint_as_float(vv[8 * u + 7]));
          *reinterpret_cast<uint4*>(dk + 8 * u) = wk;
          *reinterpret_cast<uint4*>(dvp + 8 * u) = wv;
        }
      }
    }
    if (lane == 0) bulk_wait<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace attnb

int flash_attn_bwd_sm100_d64(const __nv_bfloat16* dout, long ld_do, const __nv_bfloat16* qkv, long ld_qkv,
                             const float* lse, const float* delta, float* dq_acc, __nv_bfloat16* dqkv, long ld_dqkv,
                             int B, int S, int nh, float softmax_scale, int* err, int num_sms, cudaStream_t stream) {
  using namespace attnb;
  if (S % BM != 0) return -1;
  const long rows = (long)B * S;
  CUtensorMap tm_qkv, tm_do, tm_dq;
  int rc = make_tmap_bf16_2d(&tm_qkv, qkv, rows, 3L * nh * D, ld_qkv, 64, BM);
  if (rc) return rc - 10;
  rc = make_tmap_bf16_2d(&tm_do, dout, rows, (long)nh * D, ld_do, 64, BM);
  if (rc) return rc - 20;
  rc = make_tmap_f32_2d(&tm_dq, dq_acc, rows, (long)nh * D, (long)nh * D, 32, 32);
  if (rc) return rc - 30;
  Args a;
  a.B = B;
  a.S = S;
  a.nh = nh;
  a.q_col0 = 0;
  a.k_col0 = nh * D;
  a.v_col0 = 2 * nh * D;
  a.lse = lse;
  a.delta = delta;
  a.dqkv = dqkv;
  a.ld_dqkv = ld_dqkv;
  a.scale = softmax_scale;
  a.scale_log2 = softmax_scale * 1.4426950408889634f;
  a.err = err;
  const int n_items = B * nh * (S / BM);
  const int grid = std::max(1, std::min(n_items, num_sms));
  static bool set = false;
  if (!set) {
    cudaFuncSetAttribute(flash_bwd_sm100_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    set = true;
  }
  launch_k(flash_bwd_sm100_kernel, grid, kThreads, SMEM, stream, tm_qkv, tm_do, tm_dq, a);
  return (int)cudaGetLastError();
}

}  // namespace mmb
