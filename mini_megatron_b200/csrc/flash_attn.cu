// Causal flash attention (forward and backward) for sm_100a on tcgen05 / TMEM / TMA.
//
// The reference calls F.scaled_dot_product_attention(is_causal=True) on
// [B, nh, S, d] views of its fused QKV projection (model/transformer.py:27-33).
// Here the kernels read Q, K and V tiles directly out of the packed
// [B*S, 3*nh*d] bf16 output of the QKV GEMM with TMA (no reshape/transpose
// copies) and write the context in the [B*S, nh*d] layout the O projection
// consumes.
//
// Forward, one CTA per (128-query tile, head, batch), 6 warps:
//   warp 0      TMA producer: Q once, then K_j / V_j into a 2-stage ring
//   warp 1      TMEM owner + single-thread tcgen05.mma issuer:
//                 S   = Q K_j^T          (128 x 128, fp32 in TMEM)
//                 O_j = P_j V_j          (128 x d,   fp32 in TMEM, 2 buffers)
//   warps 2-5   softmax: thread i owns query row i (TMEM lane i); reads S with
//               tcgen05.ld, keeps the running max / sum in registers, writes
//               P_j (bf16) to shared memory in the 128B-swizzled K-major
//               layout the next MMA reads, and accumulates
//               o = o * exp2(m_old - m_new) + O_j in registers.
// S_{j+1} is computed while the softmax warps finish tile j, and PV_j runs
// while they start tile j+1.  Scores are kept in log2 units
// (scale * log2(e) folded in), LSE is written in natural-log units.
//
// Every mbarrier wait is bounded; on time-out the kernel records an error
// code, winds down all roles, frees TMEM and returns.
#include "common.cuh"
#include "ops.h"

#include <algorithm>
#include <mutex>

namespace mmb {

namespace attn {

constexpr int BM = 128;  // query rows per tile
constexpr int BN = 128;  // key rows per tile
constexpr int kThreads = 192;

template <int D>
struct FwdCfg {
  static constexpr int CHUNKS = D / 64;                 // 64-column (128 B) chunks per row
  static constexpr int TILE_BYTES = BM * D * 2;         // one Q / K / V tile
  static constexpr int P_BUFS = 1;
  static constexpr int V_STAGES = (D == 64) ? 1 : 2;    // d=64: two CTAs per SM, so keep smem <= ~100 KB
  static constexpr int P_BYTES = BM * BN * 2;           // 32 KB
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + TILE_BYTES;
  static constexpr int V_OFF = K_OFF + 2 * TILE_BYTES;
  static constexpr int P_OFF = V_OFF + V_STAGES * TILE_BYTES;
  static constexpr int BAR_OFF = P_OFF + P_BUFS * P_BYTES;
  static constexpr int SMEM = 1024 + BAR_OFF + 256;
  static constexpr int TMEM_COLS = (BN + 2 * D) <= 256 ? 256 : 512;
  static constexpr int MIN_CTAS = (D == 64) ? 2 : 1;
};

struct FwdArgs {
  int B, S, nh;
  int q_col0, k_col0, v_col0;  // column offsets of the Q / K / V blocks in the qkv rows
  __nv_bfloat16* out;
  long ld_out;
  float* lse;                  // [B, nh, S]
  float scale_log2;
  int* err;
};

__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Warp-uniform bounded wait: lane 0 polls, the result is broadcast.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int code,
                                          volatile int* abort_flag) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, err, code, abort_flag) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

template <int D>
__global__ void __launch_bounds__(kThreads, FwdCfg<D>::MIN_CTAS)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, const FwdArgs a) {
  pdl_trigger();
  using C = FwdCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sQ = smem + C::Q_OFF;
  uint8_t* sK = smem + C::K_OFF;
  uint8_t* sV = smem + C::V_OFF;
  uint8_t* sP = smem + C::P_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2]  K stage loaded
  uint64_t* v_full = bars + 3;    // [2]  V stage loaded
  uint64_t* k_empty = bars + 5;   // [2]  S MMA that read the K stage is done
  uint64_t* s_full = bars + 7;
  uint64_t* s_free = bars + 8;
  uint64_t* p_full = bars + 9;    // [2]
  uint64_t* p_free = bars + 11;   // [2]
  uint64_t* o_full = bars + 13;   // [2]
  uint64_t* o_free = bars + 15;   // [2]
  uint64_t* drain = bars + 17;
  uint64_t* v_empty = bars + 18;  // [2]  PV MMA that read the V stage is done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 20);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int b = bh / a.nh, h = bh % a.nh;
  const int n_qt = a.S / BM;
  const int qt = n_qt - 1 - blockIdx.y;  // heaviest (longest causal row) tiles first
  const int J = qt + 1;                  // key tiles 0..qt
  const int row0 = b * a.S;              // first qkv row of this sequence

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&p_free[i], 1);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 128);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 128);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_qkv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();  // set-up above touched no global memory
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s = tmem;            // S: columns [0, 128)
  const uint32_t t_o = tmem + BN;       // O buffers: [128, 128 + 2D)

  if (warp == 0) {
    if (lane == 0) {
      const int qx = a.q_col0 + h * D, kx = a.k_col0 + h * D, vx = a.v_col0 + h * D;
      mbar_expect_tx(q_full, C::TILE_BYTES);
#pragma unroll
      for (int c = 0; c < C::CHUNKS; ++c) tma_load_2d(sQ + c * 16384, &tm_qkv, q_full, qx + 64 * c, row0 + qt * BM);
      for (int j = 0; j < J; ++j) {
        const int st = j & 1;
        const int vs = j % C::V_STAGES;
        if (j >= 2 && !mbar_wait(&k_empty[st], ((j >> 1) - 1) & 1, a.err, kErrAttnWait, abort_flag)) break;
        uint8_t* kd = sK + st * C::TILE_BYTES;
        mbar_expect_tx(&k_full[st], C::TILE_BYTES);
#pragma unroll
        for (int c = 0; c < C::CHUNKS; ++c) tma_load_2d(kd + c * 16384, &tm_qkv, &k_full[st], kx + 64 * c, row0 + j * BN);
        if (j >= C::V_STAGES &&
            !mbar_wait(&v_empty[vs], ((j / C::V_STAGES) - 1) & 1, a.err, kErrAttnWait, abort_flag))
          break;
        uint8_t* vd = sV + vs * C::TILE_BYTES;
        mbar_expect_tx(&v_full[vs], C::TILE_BYTES);
#pragma unroll
        for (int c = 0; c < C::CHUNKS; ++c) tma_load_2d(vd + c * 16384, &tm_qkv, &v_full[vs], vx + 64 * c, row0 + j * BN);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(BM, BN, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16(BM, D, false, true);
      bool ok = mbar_wait(q_full, 0, a.err, kErrAttnWait, abort_flag);
      const uint32_t q_addr = smem_u32(sQ);
      auto issue_pv = [&](int t) -> bool {
        const int vs = t % C::V_STAGES, pb = t % C::P_BUFS, ob = t & 1;
        if (!mbar_wait(&v_full[vs], (t / C::V_STAGES) & 1, a.err, kErrAttnWait, abort_flag)) return false;
        if (!mbar_wait(&p_full[pb], (t / C::P_BUFS) & 1, a.err, kErrAttnWait, abort_flag)) return false;
        if (t >= 2 && !mbar_wait(&o_free[ob], ((t - 2) >> 1) & 1, a.err, kErrAttnWait, abort_flag)) return false;
        tc_fence_after();
        const uint32_t p_addr = smem_u32(sP + pb * C::P_BYTES);
        const uint32_t v_addr = smem_u32(sV + vs * C::TILE_BYTES);
#pragma unroll
        for (int k = 0; k < BN / 16; ++k) {
          const uint64_t ad = make_sdesc_sw128(p_addr + (k >> 2) * 16384 + (k & 3) * 32, 16, 1024);
          const uint64_t bd = make_sdesc_sw128(v_addr + k * 2048, 16384, 1024);
          umma_bf16_ss(t_o + ob * D, ad, bd, idesc_o, k != 0 ? 1u : 0u);
        }
        umma_commit(&o_full[ob]);
        umma_commit(&p_free[pb]);
        umma_commit(&v_empty[vs]);
        return true;
      };
      for (int j = 0; j < J && ok; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&k_full[st], (j >> 1) & 1, a.err, kErrAttnWait, abort_flag)) { ok = false; break; }
        if (j >= 1 && !mbar_wait(s_free, (j - 1) & 1, a.err, kErrAttnWait, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + st * C::TILE_BYTES);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint64_t ad = make_sdesc_sw128(q_addr + (k >> 2) * 16384 + (k & 3) * 32, 16, 1024);
          const uint64_t bd = make_sdesc_sw128(k_addr + (k >> 2) * 16384 + (k & 3) * 32, 16, 1024);
          umma_bf16_ss(t_s, ad, bd, idesc_s, k != 0 ? 1u : 0u);
        }
        umma_commit(s_full);
        umma_commit(&k_empty[st]);
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok) ok = issue_pv(J - 1);
      if (!ok) {
        umma_commit(drain);
        const unsigned long long t0 = globaltimer();
        while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < 10000000ull) {
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax warps
    const int q = warp & 3;
    const int r = q * 32 + lane;                 // row within the tile == TMEM lane
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const float sl2 = a.scale_log2;
    float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
    float o[D];
#pragma unroll
    for (int i = 0; i < D; ++i) o[i] = 0.f;
    bool ok = true;

    auto accumulate_o = [&](int t) -> bool {
      const int ob = t & 1;
      if (!warp_wait(&o_full[ob], (t >> 1) & 1, a.err, kErrAttnWait, abort_flag)) return false;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(t_o + lane_off + ob * D + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) o[c * 32 + e] = o[c * 32 + e] * alpha_prev + __uint_as_float(v[e]);
      }
      tc_fence_before();
      mbar_arrive(&o_free[ob]);
      return true;
    };

    for (int j = 0; j < J; ++j) {
      if (!warp_wait(s_full, j & 1, a.err, kErrAttnWait, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const bool diag = (j == qt);
      // pass 1: row max of this tile (causal mask on the diagonal tile).  Eight
      // independent partial maxima keep the reduction off one serial chain.
      float mx[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mx[k] = -INFINITY;
#pragma unroll
      for (int cc = 0; cc < BN / 32; ++cc) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(t_s + lane_off + cc * 32, v);
        tmem_wait_ld();
        if (diag) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (cc * 32 + e <= r) mx[e & 7] = fmaxf(mx[e & 7], __uint_as_float(v[e]));
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) mx[e & 7] = fmaxf(mx[e & 7], __uint_as_float(v[e]));
        }
      }
      const float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                             fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
      const float m_new = fmaxf(m, mt * sl2);
      const float alpha = exp2_approx(m - m_new);
      const int pb = j % C::P_BUFS;
      if (j >= C::P_BUFS && !warp_wait(&p_free[pb], ((j / C::P_BUFS) - 1) & 1, a.err, kErrAttnWait, abort_flag)) {
        ok = false;
        break;
      }
      // pass 2: P = exp2(S*scale_log2 - m_new) -> bf16 -> swizzled smem (eight partial row sums)
      float rs8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) rs8[k] = 0.f;
      uint8_t* prow = sP + pb * C::P_BYTES + r * 128;
#pragma unroll
      for (int cc = 0; cc < BN / 32; ++cc) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(t_s + lane_off + cc * 32, v);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const int c0 = cc * 32 + e;
          float p0 = exp2_approx(__uint_as_float(v[e]) * sl2 - m_new);
          float p1 = exp2_approx(__uint_as_float(v[e + 1]) * sl2 - m_new);
          if (diag) {
            if (c0 > r) p0 = 0.f;
            if (c0 + 1 > r) p1 = 0.f;
          }
          rs8[(e >> 1) & 7] += p0 + p1;
          pk[e >> 1] = pack_bf16x2(p0, p1);
        }
        uint8_t* chunk = prow + (cc >> 1) * 16384;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int unit = (cc & 1) * 4 + u;
          *reinterpret_cast<uint4*>(chunk + ((unit ^ (r & 7)) << 4)) =
              make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(s_free);
      fence_proxy_async_smem();
      mbar_arrive(&p_full[pb]);
      const float rowsum = ((rs8[0] + rs8[1]) + (rs8[2] + rs8[3])) + ((rs8[4] + rs8[5]) + (rs8[6] + rs8[7]));
      l = l * alpha + rowsum;
      m = m_new;
      if (j >= 1 && !accumulate_o(j - 1)) { ok = false; break; }
      alpha_prev = alpha;
    }
    if (ok && accumulate_o(J - 1)) {
      const int pos = qt * BM + r;
      const float inv = 1.f / l;
      __nv_bfloat16* orow = a.out + (size_t)(row0 + pos) * a.ld_out + h * D;
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        uint4 w;
        w.x = pack_bf16x2(o[8 * c + 0] * inv, o[8 * c + 1] * inv);
        w.y = pack_bf16x2(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
        w.z = pack_bf16x2(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
        w.w = pack_bf16x2(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
        *reinterpret_cast<uint4*>(orow + 8 * c) = w;
      }
      a.lse[((size_t)b * a.nh + h) * a.S + pos] = m * 0.69314718055994531f + logf(l);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace attn

int flash_attn_fwd(const __nv_bfloat16* qkv, long ld_qkv, int B, int S, int nh, int d, __nv_bfloat16* out,
                   long ld_out, float* lse, float softmax_scale, int* err, cudaStream_t stream) {
  using namespace attn;
  if (S % BM != 0 || (d != 64 && d != 128)) return -1;
  if ((reinterpret_cast<uintptr_t>(out) & 15) || (ld_out % 8)) return -2;
  CUtensorMap tm;
  const long rows = (long)B * S, cols = 3L * nh * d;
  int rc = make_tmap_bf16_2d(&tm, qkv, rows, cols, ld_qkv, 64, BM);
  if (rc) return rc - 10;
  FwdArgs a;
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
  dim3 grid(B * nh, S / BM);
  if (d == 64) {
    auto k = flash_fwd_kernel<64>;
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, FwdCfg<64>::SMEM);
      set = true;
    }
    launch_k(k, grid, kThreads, FwdCfg<64>::SMEM, stream, tm, a);
  } else {
    auto k = flash_fwd_kernel<128>;
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, FwdCfg<128>::SMEM);
      set = true;
    }
    launch_k(k, grid, kThreads, FwdCfg<128>::SMEM, stream, tm, a);
  }
  return (int)cudaGetLastError();
}

// ============================================================================ backward
//
// One CTA per (128-key tile j, head, batch); it loops over the query tiles
// i >= j that see tile j under the causal mask.  Roles as in the forward:
//   warp 0      TMA: K_j, V_j once; Q_i, dO_i (+ LSE_i, Delta_i by bulk copy) per i
//   warp 1      tcgen05.mma:   S^T  = K_j Q_i^T,   dP^T = V_j dO_i^T
//                              dV  += P^T dO_i,    dK  += dS^T Q_i,   dQ_i = dS K_j
//   warps 2-5   thread c owns key row c:  P^T = exp2(S^T*scale_log2 - LSE2),
//               dS^T = P^T * (dP^T - Delta)  -> bf16 swizzled smem (the dS^T
//               buffer is read K-major for dK and MN-major for dQ), then they
//               drain dQ_i (thread r = query row r) into an fp32 accumulator
//               with vector atomics, and finally write dK_j (scaled) and dV_j.
namespace attn {

template <int D>
struct BwdCfg {
  static constexpr int CHUNKS = D / 64;
  static constexpr int TILE = BM * D * 2;
  static constexpr int STAGES = (D == 64) ? 2 : 1;
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = TILE;
  static constexpr int Q_OFF = 2 * TILE;
  static constexpr int DO_OFF = Q_OFF + STAGES * TILE;
  static constexpr int PT_OFF = DO_OFF + STAGES * TILE;
  static constexpr int DS_OFF = PT_OFF + BM * BN * 2;
  static constexpr int LD_OFF = DS_OFF + BM * BN * 2;   // per stage: lse[128], delta[128]
  static constexpr int DQ_OFF = LD_OFF + STAGES * 1024;  // 8 warps x 4 KB dQ staging for the bulk reduce-add
  static constexpr int BAR_OFF = DQ_OFF + 8 * 4096;
  static constexpr int SMEM = 1024 + BAR_OFF + 256;
  // TMEM columns
  static constexpr int T_ST = 0, T_DPT = 128, T_DV = 256, T_DK = 256 + D;
  static constexpr int T_DQ = (D == 64) ? 384 : 128;   // D=128: dQ reuses the dP^T columns
};

constexpr int kBwdThreads = 320;  // TMA warp, MMA warp, 8 softmax-gradient warps

struct BwdArgs {
  int B, S, nh;
  int q_col0, k_col0, v_col0;
  const float* lse;     // [B, nh, S] natural log
  const float* delta;   // [B, nh, S]
  float* dq_acc;        // [B*S, nh*D] fp32, pre-zeroed
  long ld_dq;
  __nv_bfloat16* dqkv;  // [B*S, 3*nh*D]
  long ld_dqkv;
  float scale;          // softmax scale
  float scale_log2;
  int* err;
};

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

template <int D>
__global__ void __launch_bounds__(kBwdThreads, 1)
    flash_bwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_do,
                     const __grid_constant__ CUtensorMap tm_dq, const BwdArgs a) {
  pdl_trigger();
  using C = BwdCfg<D>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sK = smem + C::K_OFF;
  uint8_t* sV = smem + C::V_OFF;
  uint8_t* sQ = smem + C::Q_OFF;
  uint8_t* sDO = smem + C::DO_OFF;
  uint8_t* sPT = smem + C::PT_OFF;
  uint8_t* sDS = smem + C::DS_OFF;
  float* sLD = reinterpret_cast<float*>(smem + C::LD_OFF);
  uint8_t* sDQ = smem + C::DQ_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;    // [2]
  uint64_t* q_empty = bars + 3;   // [2]
  uint64_t* st_full = bars + 5;
  uint64_t* st_free = bars + 6;
  uint64_t* ps_full = bars + 7;
  uint64_t* ps_free = bars + 8;
  uint64_t* dq_full = bars + 9;
  uint64_t* dq_free = bars + 10;
  uint64_t* dkv_full = bars + 11;
  uint64_t* drain = bars + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int b = bh / a.nh, h = bh % a.nh;
  const int n_qt = a.S / BM;
  const int j = blockIdx.y;          // key tile (j = 0 has the most query tiles: scheduled first)
  const int NI = n_qt - j;           // query tiles j .. n_qt-1
  const int row0 = b * a.S;
  const size_t ld_off = ((size_t)b * a.nh + h) * a.S;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    mbar_init(st_full, 1);
    mbar_init(st_free, 256);
    mbar_init(ps_full, 256);
    mbar_init(ps_free, 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 256);
    mbar_init(dkv_full, 1);
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
  pdl_wait();  // set-up above touched no global memory
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const int qx = a.q_col0 + h * D, kx = a.k_col0 + h * D, vx = a.v_col0 + h * D, ox = h * D;
      mbar_expect_tx(kv_full, 2 * C::TILE);
#pragma unroll
      for (int c = 0; c < C::CHUNKS; ++c) {
        tma_load_2d(sK + c * 16384, &tm_qkv, kv_full, kx + 64 * c, row0 + j * BN);
        tma_load_2d(sV + c * 16384, &tm_qkv, kv_full, vx + 64 * c, row0 + j * BN);
      }
      for (int i = 0; i < NI; ++i) {
        const int st = i % STAGES;
        if (i >= STAGES && !mbar_wait(&q_empty[st], ((i / STAGES) - 1) & 1, a.err, kErrAttnWait, abort_flag)) break;
        const int qrow = row0 + (j + i) * BM;
        mbar_expect_tx(&q_full[st], 2 * C::TILE + 1024);
#pragma unroll
        for (int c = 0; c < C::CHUNKS; ++c) {
          tma_load_2d(sQ + st * C::TILE + c * 16384, &tm_qkv, &q_full[st], qx + 64 * c, qrow);
          tma_load_2d(sDO + st * C::TILE + c * 16384, &tm_do, &q_full[st], ox + 64 * c, qrow);
        }
        bulk_load(sLD + st * 256, a.lse + ld_off + (size_t)(j + i) * BM, 512, &q_full[st]);
        bulk_load(sLD + st * 256 + 128, a.delta + ld_off + (size_t)(j + i) * BM, 512, &q_full[st]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(BM, BN, false, false);
      constexpr uint32_t idesc_kv = make_idesc_bf16(BN, D, false, true);  // dV, dK: A K-major smem, B MN-major
      constexpr uint32_t idesc_q = make_idesc_bf16(BM, D, true, true);    // dQ: A = dS (MN-major view)
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      const uint32_t pt_addr = smem_u32(sPT), ds_addr = smem_u32(sDS);
      bool ok = mbar_wait(kv_full, 0, a.err, kErrAttnWait, abort_flag);

      auto issue_s = [&](int i) -> bool {
        const int st = i % STAGES;
        if (!mbar_wait(&q_full[st], (i / STAGES) & 1, a.err, kErrAttnWait, abort_flag)) return false;
        if (i >= 1 && !mbar_wait(st_free, (i - 1) & 1, a.err, kErrAttnWait, abort_flag)) return false;
        if (D == 128 && i >= 1 && !mbar_wait(dq_free, (i - 1) & 1, a.err, kErrAttnWait, abort_flag)) return false;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sQ + st * C::TILE), do_addr = smem_u32(sDO + st * C::TILE);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
          umma_bf16_ss(tmem + C::T_ST, make_sdesc_sw128(k_addr + off, 16, 1024),
                       make_sdesc_sw128(q_addr + off, 16, 1024), idesc_s, k != 0);
        }
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
          umma_bf16_ss(tmem + C::T_DPT, make_sdesc_sw128(v_addr + off, 16, 1024),
                       make_sdesc_sw128(do_addr + off, 16, 1024), idesc_s, k != 0);
        }
        umma_commit(st_full);
        return true;
      };
      auto issue_grads = [&](int t) -> bool {
        const int st = t % STAGES;
        if (!mbar_wait(ps_full, t & 1, a.err, kErrAttnWait, abort_flag)) return false;
        if (D == 64 && t >= 1 && !mbar_wait(dq_free, (t - 1) & 1, a.err, kErrAttnWait, abort_flag)) return false;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sQ + st * C::TILE), do_addr = smem_u32(sDO + st * C::TILE);
#pragma unroll
        for (int k = 0; k < BM / 16; ++k) {   // reduction over the 128 query rows of tile t
          const uint32_t a_off = (k >> 2) * 16384 + (k & 3) * 32;
          umma_bf16_ss(tmem + C::T_DV, make_sdesc_sw128(pt_addr + a_off, 16, 1024),
                       make_sdesc_sw128(do_addr + k * 2048, 16384, 1024), idesc_kv, (t > 0 || k > 0));
          umma_bf16_ss(tmem + C::T_DK, make_sdesc_sw128(ds_addr + a_off, 16, 1024),
                       make_sdesc_sw128(q_addr + k * 2048, 16384, 1024), idesc_kv, (t > 0 || k > 0));
        }
#pragma unroll
        for (int k = 0; k < BN / 16; ++k) {   // reduction over the 128 key rows of tile j
          umma_bf16_ss(tmem + C::T_DQ, make_sdesc_sw128(ds_addr + k * 2048, 16384, 1024),
                       make_sdesc_sw128(k_addr + k * 2048, 16384, 1024), idesc_q, k != 0);
        }
        umma_commit(dq_full);
        umma_commit(ps_free);
        umma_commit(&q_empty[st]);
        return true;
      };
      for (int i = 0; i <= NI && ok; ++i) {
        if (i < NI && D == 64 && !issue_s(i)) { ok = false; break; }
        if (i >= 1 && !issue_grads(i - 1)) { ok = false; break; }
        if (i < NI && D == 128 && !issue_s(i)) { ok = false; break; }
      }
      if (ok) umma_commit(dkv_full);
      else {
        umma_commit(drain);
        const unsigned long long t0 = globaltimer();
        while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < 10000000ull) {
        }
      }
    }
  } else {
    // warps 2..9: w and w+4 share a TMEM lane quarter; `half` selects which 64 query columns
    // of S^T / dP^T (and which half of the dQ / dK / dV columns) this warp handles.
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int c = q * 32 + lane;               // key row (TMEM lane) for S^T / dP^T / dK / dV
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const float sl2 = a.scale_log2;
    uint8_t* stg = sDQ + (warp - 2) * 4096;
    bool ok = true;

    // dQ_t (TMEM lane = query row) -> per-warp 32x32 fp32 stage -> one bulk tensor reduce-add into dq_acc
    auto drain_dq = [&](int t) -> bool {
      if (!warp_wait(dq_full, t & 1, a.err, kErrAttnWait, abort_flag)) return false;
      tc_fence_after();
      const int qrow0 = row0 + (j + t) * BM + q * 32;
#pragma unroll
      for (int cc = half; cc < D / 32; cc += 2) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem + C::T_DQ + lane_off + cc * 32, v);
        tmem_wait_ld();
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
#pragma unroll
        for (int u = 0; u < 8; ++u)
          *reinterpret_cast<float4*>(stg + lane * 128 + ((u ^ (lane & 7)) << 4)) =
              make_float4(__uint_as_float(v[4 * u]) * a.scale, __uint_as_float(v[4 * u + 1]) * a.scale,
                          __uint_as_float(v[4 * u + 2]) * a.scale, __uint_as_float(v[4 * u + 3]) * a.scale);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_2d(&tm_dq, stg, h * D + cc * 32, qrow0);
          bulk_commit();
        }
      }
      tc_fence_before();
      mbar_arrive(dq_free);
      return true;
    };

    for (int i = 0; i < NI; ++i) {
      const int st = i % STAGES;
      // D = 128: dQ_{i-1} lives in the dP^T columns, and the MMA computing dP^T_i
      // waits for it to be drained -- so drain first.  D = 64: dQ has its own
      // columns and is drained after P^T_i / dS^T_i are handed over.
      if (D == 128 && i >= 1 && !drain_dq(i - 1)) { ok = false; break; }
      if (!warp_wait(&q_full[st], (i / STAGES) & 1, a.err, kErrAttnWait, abort_flag)) { ok = false; break; }
      if (!warp_wait(st_full, i & 1, a.err, kErrAttnWait, abort_flag)) { ok = false; break; }
      if (i >= 1 && !warp_wait(ps_free, (i - 1) & 1, a.err, kErrAttnWait, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const float* lse = sLD + st * 256;
      const float* dlt = lse + 128;
      const bool diag = (i == 0);
      uint8_t* pt_row = sPT + half * 16384 + c * 128;
      uint8_t* ds_row = sDS + half * 16384 + c * 128;
#pragma unroll
      for (int k2 = 0; k2 < 2; ++k2) {
        const int cc = half * 2 + k2;            // 32-column chunk of the 128 query columns
        uint32_t sv[32], dv[32];
        tmem_ld_32x32b_x32(tmem + C::T_ST + lane_off + cc * 32, sv);
        tmem_ld_32x32b_x32(tmem + C::T_DPT + lane_off + cc * 32, dv);
        tmem_wait_ld();
        uint32_t pp[16], dd[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const int r0 = cc * 32 + e;
          float p0 = exp2_approx(__uint_as_float(sv[e]) * sl2 - lse[r0] * 1.4426950408889634f);
          float p1 = exp2_approx(__uint_as_float(sv[e + 1]) * sl2 - lse[r0 + 1] * 1.4426950408889634f);
          if (diag && r0 < c) p0 = 0.f;
          if (diag && r0 + 1 < c) p1 = 0.f;
          const float d0 = p0 * (__uint_as_float(dv[e]) - dlt[r0]);
          const float d1 = p1 * (__uint_as_float(dv[e + 1]) - dlt[r0 + 1]);
          pp[e >> 1] = pack_bf16x2(p0, p1);
          dd[e >> 1] = pack_bf16x2(d0, d1);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int sw = (((k2 * 4 + u) ^ (c & 7)) << 4);
          *reinterpret_cast<uint4*>(pt_row + sw) = make_uint4(pp[4 * u], pp[4 * u + 1], pp[4 * u + 2], pp[4 * u + 3]);
          *reinterpret_cast<uint4*>(ds_row + sw) = make_uint4(dd[4 * u], dd[4 * u + 1], dd[4 * u + 2], dd[4 * u + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(st_free);
      fence_proxy_async_smem();
      mbar_arrive(ps_full);
      if (D == 64 && i >= 1 && !drain_dq(i - 1)) { ok = false; break; }
    }
    if (ok) ok = drain_dq(NI - 1);
    if (ok && warp_wait(dkv_full, 0, a.err, kErrAttnWait, abort_flag)) {
      tc_fence_after();
      const size_t row = (size_t)(row0 + j * BN + c);
      __nv_bfloat16* dk = a.dqkv + row * a.ld_dqkv + a.k_col0 + h * D;
      __nv_bfloat16* dv = a.dqkv + row * a.ld_dqkv + a.v_col0 + h * D;
#pragma unroll
      for (int cc = half; cc < D / 32; cc += 2) {
        uint32_t kv[32], vv[32];
        tmem_ld_32x32b_x32(tmem + C::T_DK + lane_off + cc * 32, kv);
        tmem_ld_32x32b_x32(tmem + C::T_DV + lane_off + cc * 32, vv);
        tmem_wait_ld();
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
          *reinterpret_cast<uint4*>(dk + cc * 32 + 8 * u) = wk;
          *reinterpret_cast<uint4*>(dv + cc * 32 + 8 * u) = wv;
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

// delta[b, h, pos] = sum_d dO[row, h*D + d] * O[row, h*D + d]
// One thread per 8 elements (16 bytes); the D/8 threads of a (row, head) reduce with shuffles.
// The same thread also zeroes the 8 matching fp32 elements of the dQ accumulator (same
// [B*S, nh*D] layout), which the backward then fills with bulk reduce-adds.
__global__ void attn_delta_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ out,
                                  long ld, int B, int S, int nh, int D, float* __restrict__ delta,
                                  float* __restrict__ dq_zero) {
  pdl_trigger();
  pdl_wait();
  const int g = D / 8;  // threads per (row, head): 8 or 16
  const long tid = blockIdx.x * (long)blockDim.x + threadIdx.x;
  const long pair = tid / g;  // (row, head) index
  const int part = (int)(tid % g);
  const bool valid = pair < (long)B * S * nh;
  float acc = 0.f;
  long row = 0;
  int h = 0;
  if (valid) {
    row = pair / nh;
    h = (int)(pair % nh);
    const uint4 x = *reinterpret_cast<const uint4*>(dout + row * ld + h * D + part * 8);
    const uint4 y = *reinterpret_cast<const uint4*>(out + row * ld + h * D + part * 8);
    if (dq_zero) {
      float4* z = reinterpret_cast<float4*>(dq_zero + row * ld + h * D + part * 8);
      z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
      z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(&x);
    const uint32_t* yw = reinterpret_cast<const uint32_t*>(&y);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 p = unpack_bf16x2(xw[e]), q = unpack_bf16x2(yw[e]);
      acc += p.x * q.x + p.y * q.y;
    }
  }
  for (int o = g / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (valid && part == 0) {
    const long b = row / S, pos = row % S;
    delta[((size_t)b * nh + h) * S + pos] = acc;
  }
}

// dqkv[:, q block] = bf16(dq_acc)
__global__ void attn_dq_convert_kernel(const float* __restrict__ dq, long ld_dq, __nv_bfloat16* __restrict__ dqkv,
                                       long ld_dqkv, long rows, int width) {
  pdl_trigger();
  pdl_wait();
  const long n4 = rows * (width / 4);
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
    const long r = i / (width / 4), c = (i % (width / 4)) * 4;
    const float4 v = *reinterpret_cast<const float4*>(dq + r * ld_dq + c);
    uint2 o;
    o.x = pack_bf16x2(v.x, v.y);
    o.y = pack_bf16x2(v.z, v.w);
    *reinterpret_cast<uint2*>(dqkv + r * ld_dqkv + c) = o;
  }
}

}  // namespace attn

int flash_attn_bwd(const __nv_bfloat16* dout, long ld_do, const __nv_bfloat16* qkv, long ld_qkv,
                   const __nv_bfloat16* out, const float* lse, float* delta, float* dq_acc, __nv_bfloat16* dqkv,
                   long ld_dqkv, int B, int S, int nh, int d, float softmax_scale, int* err, int num_sms,
                   cudaStream_t stream, bool one_tile_per_cta) {
  using namespace attn;
  if (S % BM != 0 || (d != 64 && d != 128)) return -1;
  if (ld_do != (long)nh * d) return -2;
  const long rows = (long)B * S;
  // Delta = rowsum(dO * O)
  {
    const long threads = rows * nh * (d / 8);
    launch_k(attn_delta_kernel, (unsigned)((threads + 255) / 256), 256, 0, stream, dout, out, ld_do, B, S, nh, d, delta,
             dq_acc);
  }
  const long n4 = rows * nh * d / 4;
  if (d == 64 && !one_tile_per_cta) {
    // persistent key/value-stationary kernel (flash_bwd_sm100.cu)
    const int rc = flash_attn_bwd_sm100_d64(dout, ld_do, qkv, ld_qkv, lse, delta, dq_acc, dqkv, ld_dqkv, B, S, nh,
                                            softmax_scale, err, num_sms, stream);
    if (rc) return rc;
    launch_k(attn_dq_convert_kernel, (unsigned)std::min<long>((n4 + 255) / 256, (long)num_sms * 8), 256, 0, stream,
             dq_acc, (long)nh * d, dqkv, ld_dqkv, rows, nh * d);
    return (int)cudaGetLastError();
  }
  CUtensorMap tm_qkv, tm_do;
  int rc = make_tmap_bf16_2d(&tm_qkv, qkv, rows, 3L * nh * d, ld_qkv, 64, BM);
  if (rc) return rc - 10;
  rc = make_tmap_bf16_2d(&tm_do, dout, rows, (long)nh * d, ld_do, 64, BM);
  if (rc) return rc - 20;
  CUtensorMap tm_dq;
  rc = make_tmap_f32_2d(&tm_dq, dq_acc, rows, (long)nh * d, (long)nh * d, 32, 32);
  if (rc) return rc - 30;
  BwdArgs a;
  a.B = B;
  a.S = S;
  a.nh = nh;
  a.q_col0 = 0;
  a.k_col0 = nh * d;
  a.v_col0 = 2 * nh * d;
  a.lse = lse;
  a.delta = delta;
  a.dq_acc = dq_acc;
  a.ld_dq = (long)nh * d;
  a.dqkv = dqkv;
  a.ld_dqkv = ld_dqkv;
  a.scale = softmax_scale;
  a.scale_log2 = softmax_scale * 1.4426950408889634f;
  a.err = err;
  dim3 grid(B * nh, S / BN);
  if (d == 64) {
    auto k = flash_bwd_kernel<64>;
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, BwdCfg<64>::SMEM);
      set = true;
    }
    launch_k(k, grid, kBwdThreads, BwdCfg<64>::SMEM, stream, tm_qkv, tm_do, tm_dq, a);
  } else {
    auto k = flash_bwd_kernel<128>;
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, BwdCfg<128>::SMEM);
      set = true;
    }
    launch_k(k, grid, kBwdThreads, BwdCfg<128>::SMEM, stream, tm_qkv, tm_do, tm_dq, a);
  }
  launch_k(attn_dq_convert_kernel, (unsigned)std::min<long>((n4 + 255) / 256, (long)num_sms * 8), 256, 0, stream, 
      dq_acc, (long)nh * d, dqkv, ld_dqkv, rows, nh * d);
  return (int)cudaGetLastError();
}

}  // namespace mmb
