// Causal / sliding-window GQA attention forward on the 5th-generation tensor
// cores (tcgen05 + TMEM), head dims 64 and 128 (model/attention.py:136-224
// semantics: query i sees key j iff j <= i and, with a window W > 0, i - j < W).
//
// Head dim H: every K-major tile (Q, K, V rows of H bf16) is stored as H / 64
// swizzle atoms of 128-byte rows (one TMA box each); a K step of 16 inside
// atom a = k / 64 starts at atom a's base + (k % 64) * 2 bytes.  The MN-major
// operands (V, dO, Q, K as the B of P V, dS K, P^T dO, dS^T Q) are 64-row
// tiles whose 64-column atoms lie 8 KB apart, the descriptor's leading-byte
// offset, so the same descriptor covers N = 64 and N = 128.
//
// CTA = 128 query rows of one head; key/value tiles of 64.  Warp roles:
//   warp 0     TMA producer: Q once, then K_j / V_j into a 3-deep ring
//   warp 1     MMA issuer (one elected lane):
//                S_j  = Q K_j^T   M 128 x N 64 x K 64   -> TMEM S buffer j % 2
//                O   += P_j V_j   M 128 x N 64 x K 64   -> TMEM O
//              S_{j+2} is issued as soon as softmax j has consumed S_j, so the
//              tensor core computes the next score tile during the softmax
//   warps 2-9  softmax / epilogue, two threads per query row (32 keys each):
//              read S from TMEM (tcgen05.ld), online softmax in the exp2 domain
//              (row max exchanged through shared memory), write P_j (bf16) into
//              P buffer j % 2, a 128B-swizzled shared tile that is the A operand
//              of the P V MMA; at the end O / l -> bf16 and the row lse (log2).
// The running max used for the exponentials is raised only when a tile's max
// exceeds it by more than 8 (log2 units), so P <= 256 and O in TMEM is
// rescaled (tcgen05.ld / st, warp-uniform: the whole warp takes that path when
// any of its rows needs it) only on those rare steps.  Double-buffered
// barriers (s_full, p_full, pv_done per buffer) keep every mbarrier at most
// one phase ahead of its waiter.  Head dim 64: two CTAs share an SM (97 KB of
// shared memory, 256 TMEM columns each); head dim 128: one CTA (161 KB).
// Every wait is bounded (status word).
#include <torch/extension.h>

#include "../common/host.h"
#include "../common/sm100.cuh"

namespace hb {
namespace fatc {

constexpr int BQ = 128;
constexpr int BK = 64;
constexpr int THREADS = 320;   // producer, MMA, 8 softmax warps
constexpr int P_BYTES = BQ * BK * 2;         // 16 KB
constexpr int KV_STAGES = 3;
constexpr int TMEM_COLS = 256;
constexpr int S_COL = 0, O_COL = 128;   // S buffers at columns 0 and 64; O: H columns
template <int H>
struct Fwd {
  static constexpr int Q_BYTES = BQ * H * 2;   // 16 / 32 KB
  static constexpr int K_BYTES = BK * H * 2;   // 8 / 16 KB
  static constexpr int V_BYTES = BK * H * 2;
  static constexpr int SMEM = Q_BYTES + KV_STAGES * (K_BYTES + V_BYTES) + 2 * P_BYTES + 1024 + 256 + 6 * BQ * 4;
};

// K-major descriptor of K step kk (16 elements) of a tile of `rows` rows of H
// bf16 stored as H / 64 swizzle atoms of rows x 128 bytes.
HB_DEVICE uint64_t kdesc(uint32_t base, int rows, int kk) {
  return make_smem_desc(base + (kk >> 2) * rows * 128 + (kk & 3) * 32, 16, 1024);
}
// TMA of a rows x H tile: one 64-column box per atom.
template <int H>
HB_DEVICE void load_tile(uint32_t dst, const CUtensorMap* m, uint32_t bar, int col, int row, int rows) {
#pragma unroll
  for (int a = 0; a < H / 64; ++a) tma_load_2d(dst + a * rows * 128, m, bar, col + 64 * a, row);
}

// 2^x on the special-function unit (PTX ex2.approx, flush-to-zero).
HB_DEVICE float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float LOG2E = 1.4426950408889634f;

struct TcParams {
  int B, S, Nq, Nkv, window;
  float sl2;            // scale * log2(e)
  long long q_row;      // elements between consecutive tokens of q / out
  __nv_bfloat16* out;
  float* lse;
  int* status;
  unsigned long long budget_ns;
};

HB_DEVICE bool visible(const TcParams& p, int qi, int kj) {
  return kj <= qi && (p.window <= 0 || qi - kj < p.window) && kj < p.S && qi < p.S;
}

template <int H>
__global__ void __launch_bounds__(THREADS, H == 64 ? 2 : 1)
    fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const TcParams p) {
  constexpr int Q_BYTES = Fwd<H>::Q_BYTES, K_BYTES = Fwd<H>::K_BYTES, V_BYTES = Fwd<H>::V_BYTES;
  constexpr int HC = H / 64;   // 32-column chunks per half row of O
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + Q_BYTES;                 // KV_STAGES stages of K, then of V
  const uint32_t sV0 = sK0 + KV_STAGES * K_BYTES;
  const uint32_t sP0 = sV0 + KV_STAGES * V_BYTES;    // two P buffers
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Q_BYTES + KV_STAGES * (K_BYTES + V_BYTES) + 2 * P_BYTES);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;                 // [KV_STAGES]
  uint64_t* kv_empty = kv_full + KV_STAGES;     // [KV_STAGES]
  uint64_t* s_full = kv_empty + KV_STAGES;      // [2]
  uint64_t* p_full = s_full + 2;                // [2]
  uint64_t* pv_done = p_full + 2;               // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pv_done + 2);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nqt = (p.S + BQ - 1) / BQ;
  const int qt = nqt - 1 - blockIdx.x;  // longest causal rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Nq / p.Nkv);
  const int q0 = qt * BQ;
  const int hi = min(p.S, q0 + BQ);
  const int lo = p.window > 0 ? max(0, q0 - p.window + 1) : 0;
  const int jb0 = lo / BK, jb1 = (hi + BK - 1) / BK;
  const int nkt = jb1 - jb0;
  const int row0 = b * p.S;  // first token row of this sequence in the 2-D views

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    for (int s = 0; s < KV_STAGES; ++s) {
      mbar_init(smem_u32(&kv_full[s]), 1);
      mbar_init(smem_u32(&kv_empty[s]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&s_full[i]), 1);
      mbar_init(smem_u32(&p_full[i]), 256);
      mbar_init(smem_u32(&pv_done[i]), 1);
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      mbar_expect_tx(smem_u32(q_full), Q_BYTES);
      load_tile<H>(sQ, &tmQ, smem_u32(q_full), h * H, row0 + q0, BQ);
      for (int j = 0; j < nkt; ++j) {
        const int st = j % KV_STAGES;
        if (!mbar_wait(smem_u32(&kv_empty[st]), ((j / KV_STAGES) & 1) ^ 1, p.status, kErrTimeoutProducer,
                       p.budget_ns))
          break;
        const uint32_t fb = smem_u32(&kv_full[st]);
        mbar_expect_tx(fb, K_BYTES + V_BYTES);
        const int k0 = (jb0 + j) * BK;
        load_tile<H>(sK0 + st * K_BYTES, &tmK, fb, hk * H, row0 + k0, BK);
        load_tile<H>(sV0 + st * V_BYTES, &tmV, fb, hk * H, row0 + k0, BK);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc_s = make_idesc_bf16(BQ, BK, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16(BQ, H, false, true);
      bool ok = mbar_wait(smem_u32(q_full), 0, p.status, kErrTimeoutMma, p.budget_ns);
      auto issue_s = [&](int j) -> bool {
        const int st = j % KV_STAGES;
        if (!mbar_wait(smem_u32(&kv_full[st]), (j / KV_STAGES) & 1, p.status, kErrTimeoutMma, p.budget_ns))
          return false;
        tc_fence_after();
        const uint32_t sk = sK0 + st * K_BYTES;
#pragma unroll
        for (int kk = 0; kk < H / 16; ++kk)
          umma_f16(tmem + S_COL + (j & 1) * BK, kdesc(sQ, BQ, kk), kdesc(sk, BK, kk), idesc_s,
                   kk != 0 ? 1u : 0u);
        umma_commit(smem_u32(&s_full[j & 1]));
        return true;
      };
      if (ok && nkt > 0) ok = issue_s(0);
      if (ok && nkt > 1) ok = issue_s(1);
      for (int j = 0; ok && j < nkt; ++j) {
        if (!mbar_wait(smem_u32(&p_full[j & 1]), (j >> 1) & 1, p.status, kErrTimeoutMma, p.budget_ns)) break;
        tc_fence_after();
        const uint32_t sv = sV0 + (j % KV_STAGES) * V_BYTES;
        const uint32_t sp = sP0 + (j & 1) * P_BYTES;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t ad = make_smem_desc(sp + kk * 32, 16, 1024);
          const uint64_t bd = make_smem_desc(sv + kk * 2048, 8192, 1024);
          umma_f16(tmem + O_COL, ad, bd, idesc_o, (j | kk) != 0 ? 1u : 0u);
        }
        umma_commit(smem_u32(&pv_done[j & 1]));
        umma_commit(smem_u32(&kv_empty[j % KV_STAGES]));
        if (j + 2 < nkt) ok = issue_s(j + 2);   // S buffer j % 2 was consumed by softmax j
      }
    }
  } else {
    // ------------------------------------------------------------ softmax / epilogue
    // Warps 2-9: two threads per query row.  Warp w reads TMEM lane quadrant
    // w % 4 (rows 32 (w % 4) ..) and owns key / output columns half * 32 ..,
    // half = (w - 2) / 4.  The two halves of a row exchange their maxima
    // through xmax (double-buffered by tile parity, one named barrier per tile).
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quad * 32 + lane;     // row of the tile == TMEM lane
    const int qi = q0 + r;
    const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
    float* xmax = reinterpret_cast<float*>(tmem_slot + 4);   // [2 parity][2 half][BQ]
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkt; ++j) {
      // After a timeout the loop keeps running without waiting, so every warp
      // still reaches the named barriers below; nothing is written at the end.
      if (ok) ok = mbar_wait(smem_u32(&s_full[j & 1]), (j >> 1) & 1, p.status, kErrTimeoutEpilogue, p.budget_ns);
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
      const int k0 = (jb0 + j) * BK + half * 32;   // this thread's 32 keys
      const bool need_mask = (k0 + 32 > q0) || p.window > 0 || (k0 + 32 > p.S);
      uint32_t sv[32];
      tmem_ld_32x32b_x32(trow + S_COL + (j & 1) * BK + half * 32, sv);
      tmem_ld_wait();
      // pass 1: row max of the raw scores (the scale is positive), both halves
      float mraw = -INFINITY;
      if (!need_mask) {
#pragma unroll
        for (int e = 0; e < 32; ++e) mraw = fmaxf(mraw, __uint_as_float(sv[e]));
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (visible(p, qi, k0 + e)) mraw = fmaxf(mraw, __uint_as_float(sv[e]));
      }
      xmax[((j & 1) * 2 + half) * BQ + r] = mraw;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      mraw = fmaxf(mraw, xmax[((j & 1) * 2 + (half ^ 1)) * BQ + r]);
      const float mt = mraw * p.sl2;
      float alpha = 1.f;
      const bool raise = mt > m_used + 8.f;
      if (raise) {
        alpha = m_used == -INFINITY ? 0.f : ex2(m_used - mt);
        m_used = mt;
        l *= alpha;
      }
      // tcgen05.ld / st are warp-collective: the rescale runs for the whole warp
      const bool warp_raise = __any_sync(0xffffffffu, raise);
      // O rescale: needs P V_{j-1} complete (and P V_j not yet issued)
      if (warp_raise && j > 0) {
        if (ok)
          ok = mbar_wait(smem_u32(&pv_done[(j - 1) & 1]), ((j - 1) >> 1) & 1, p.status, kErrTimeoutEpilogue,
                         p.budget_ns);
        ok = __all_sync(0xffffffffu, ok);
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < HC; ++c) {
          uint32_t v[32];
          const uint32_t col = O_COL + half * (H / 2) + 32 * c;
          tmem_ld_32x32b_x32(trow + col, v);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
          tmem_st_32x32b_x32(trow + col, v);
        }
        tmem_st_wait();
      }
      // P buffer j % 2 is free once P V_{j-2} is complete
      if (j >= 2) {
        if (ok) ok = mbar_wait(smem_u32(&pv_done[j & 1]), ((j - 2) >> 1) & 1, p.status, kErrTimeoutEpilogue, p.budget_ns);
        ok = __all_sync(0xffffffffu, ok);
      }
      // pass 2: P = exp2(s * scale * log2e - m_used) -> bf16 into the swizzled A tile
      {
        const float nm = -m_used;
        const bool live = m_used != -INFINITY;   // otherwise no key of this row is visible yet
        float pv[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          float x = live ? ex2(fmaf(__uint_as_float(sv[e]), p.sl2, nm)) : 0.f;
          if (need_mask && !visible(p, qi, k0 + e)) x = 0.f;
          pv[e] = x;
          l += x;
        }
        const uint32_t prow = sP0 + (j & 1) * P_BYTES + r * 128;
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          const int chunk = half * 4 + q8;
          const uint32_t addr = prow + ((chunk ^ (r & 7)) << 4);
          const uint32_t w0 = pack_bf16x2(pv[q8 * 8 + 0], pv[q8 * 8 + 1]);
          const uint32_t w1 = pack_bf16x2(pv[q8 * 8 + 2], pv[q8 * 8 + 3]);
          const uint32_t w2 = pack_bf16x2(pv[q8 * 8 + 4], pv[q8 * 8 + 5]);
          const uint32_t w3 = pack_bf16x2(pv[q8 * 8 + 6], pv[q8 * 8 + 7]);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(w0), "r"(w1), "r"(w2), "r"(w3)
                       : "memory");
        }
      }
      fence_proxy_async();   // generic-proxy P stores -> visible to the tensor core
      tc_fence_before();
      mbar_arrive(smem_u32(&p_full[j & 1]));
    }
    // epilogue: O / l with l summed over the row's two halves
    if (ok && nkt > 0)
      ok = mbar_wait(smem_u32(&pv_done[(nkt - 1) & 1]), ((nkt - 1) >> 1) & 1, p.status, kErrTimeoutEpilogue,
                     p.budget_ns);
    const bool all_ok = __all_sync(0xffffffffu, ok) && nkt > 0;
    float* xl = xmax + 4 * BQ;   // [2 half][BQ]
    xl[half * BQ + r] = l;
    asm volatile("bar.sync 1, 256;" ::: "memory");
    l += xl[(half ^ 1) * BQ + r];
    if (all_ok) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
      for (int c = 0; c < HC; ++c) {
        const int col = half * (H / 2) + 32 * c;
        __nv_bfloat16* og = p.out + ((long long)b * p.S + qi) * p.q_row + h * H + col;
        uint32_t v[32];
        tmem_ld_32x32b_x32(trow + O_COL + col, v);
        tmem_ld_wait();
        if (qi < p.S) {
          uint4* o4 = reinterpret_cast<uint4*>(og);
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(v[q8 * 8 + 0]) * inv, __uint_as_float(v[q8 * 8 + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(v[q8 * 8 + 2]) * inv, __uint_as_float(v[q8 * 8 + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(v[q8 * 8 + 4]) * inv, __uint_as_float(v[q8 * 8 + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(v[q8 * 8 + 6]) * inv, __uint_as_float(v[q8 * 8 + 7]) * inv);
            o4[q8] = w;
          }
        }
      }
      if (qi < p.S && half == 0)
        p.lse[((long long)b * p.Nq + h) * p.S + qi] = l > 0.f ? m_used + log2f(l) : INFINITY;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}


// ============================================================== backward dK / dV
// CTA = 128 keys of one KV head; loops over every query head of the GQA group
// and every query tile of 64 that sees these keys.  Per query tile i:
//   S^T  = K Q_i^T,  dP^T = V dO_i^T          (M 128 keys x N 64 queries, TMEM)
//   P^T  = exp2(S^T * scale * log2e - lse),  dS^T = P^T (dP^T - delta)
//          (two threads per key row, 32 queries each; bf16 into swizzled A tiles)
//   dV  += P^T dO_i,  dK += dS^T Q_i           (M 128 x N 64 x K 64, TMEM)
// then dK * scale and dV -> bf16.  The producer warp stages lse / delta of the
// tile into shared memory (bounds-checked loads) beside the TMA loads of Q_i and
// dO_i.  dQ is produced by the Q-major kernel in flash_attn.cu.
constexpr int KBT = 128;    // keys per CTA
constexpr int QBT = 64;     // queries per tile
constexpr int BWD_THREADS = 320;
constexpr int PT_BYTES = KBT * QBT * 2;   // 16 KB
constexpr int ST_COL = 0, DPT_COL = 64, DV_COL = 128;   // dK at DV_COL + H
template <int H>
struct BwdKV {
  static constexpr int QT_BYTES = QBT * H * 2;   // 8 / 16 KB
  static constexpr int KT_BYTES = KBT * H * 2;   // 16 / 32 KB
  static constexpr int SMEM = 2 * KT_BYTES + 2 * 2 * QT_BYTES + 2 * PT_BYTES + 2 * 2 * QBT * 4 + 1024 + 256;
  static constexpr int TMEM = H == 64 ? 256 : 512;
};

struct BwdParams {
  int B, S, Nq, Nkv, window;
  float scale, sl2;
  const float *lse, *delta;
  __nv_bfloat16 *dk, *dv;
  long long kv_row;
  int* status;
  unsigned long long budget_ns;
};

HB_DEVICE bool visible_b(const BwdParams& p, int qi, int kj) {
  return kj <= qi && (p.window <= 0 || qi - kj < p.window) && kj < p.S && qi < p.S;
}

template <int H>
__global__ void __launch_bounds__(BWD_THREADS, H == 64 ? 2 : 1)
    bwd_kv_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                     const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmD,
                     const BwdParams p) {
  constexpr int QT_BYTES = BwdKV<H>::QT_BYTES, KT_BYTES = BwdKV<H>::KT_BYTES, BWD_TMEM = BwdKV<H>::TMEM;
  constexpr int DK_COL = DV_COL + H;
  constexpr int HC = H / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sK = smem_u32(smem);
  const uint32_t sV = sK + KT_BYTES;
  const uint32_t sQ0 = sV + KT_BYTES;                // 2 stages
  const uint32_t sD0 = sQ0 + 2 * QT_BYTES;           // 2 stages (dO)
  const uint32_t sPt = sD0 + 2 * QT_BYTES;           // P^T tile
  const uint32_t sSt = sPt + PT_BYTES;               // dS^T tile
  float* sLse = reinterpret_cast<float*>(smem + 2 * KT_BYTES + 4 * QT_BYTES + 2 * PT_BYTES);  // [2][QBT]
  float* sDel = sLse + 2 * QBT;                                                               // [2][QBT]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDel + 2 * QBT);
  uint64_t* kv_full = bars;
  uint64_t* qd_full = bars + 1;    // [2]
  uint64_t* qd_empty = bars + 3;   // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* p_full = bars + 6;
  uint64_t* pv_done = bars + 7;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int kb = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int k0 = kb * KBT;
  const int rep = p.Nq / p.Nkv;
  const int qlo = k0;
  const int qhi = p.window > 0 ? min(p.S, k0 + KBT - 1 + p.window) : p.S;
  const int ib0 = qlo / QBT, ib1 = (qhi + QBT - 1) / QBT;
  const int nq = max(0, ib1 - ib0);
  const int total = nq * rep;
  const int row0 = b * p.S;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(kv_full), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&qd_full[s]), 32);
      mbar_init(smem_u32(&qd_empty[s]), 1);
    }
    mbar_init(smem_u32(s_full), 1);
    mbar_init(smem_u32(p_full), 256);
    mbar_init(smem_u32(pv_done), 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), BWD_TMEM);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (whole warp)
    if (lane == 0) {
      mbar_expect_tx(smem_u32(kv_full), 2 * KT_BYTES);
      load_tile<H>(sK, &tmK, smem_u32(kv_full), hk * H, row0 + k0, KBT);
      load_tile<H>(sV, &tmV, smem_u32(kv_full), hk * H, row0 + k0, KBT);
    }
    for (int it = 0; it < total; ++it) {
      const int st = it & 1;
      bool ok = true;
      if (lane == 0) ok = mbar_wait(smem_u32(&qd_empty[st]), ((it >> 1) & 1) ^ 1, p.status, kErrTimeoutProducer, p.budget_ns);
      if (!__all_sync(0xffffffffu, __shfl_sync(0xffffffffu, ok, 0))) break;
      const int hq = hk * rep + it / nq;
      const int q0 = (ib0 + it % nq) * QBT;
      for (int i = lane; i < QBT; i += 32) {
        const bool in = q0 + i < p.S;
        const long long idx = ((long long)b * p.Nq + hq) * p.S + q0 + i;
        sLse[st * QBT + i] = in ? p.lse[idx] : INFINITY;
        sDel[st * QBT + i] = in ? p.delta[idx] : 0.f;
      }
      const uint32_t fb = smem_u32(&qd_full[st]);
      if (lane == 0) {
        mbar_expect_tx(fb, 2 * QT_BYTES);
        load_tile<H>(sQ0 + st * QT_BYTES, &tmQ, fb, hq * H, row0 + q0, QBT);
        load_tile<H>(sD0 + st * QT_BYTES, &tmD, fb, hq * H, row0 + q0, QBT);
      } else {
        mbar_arrive(fb);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc_s = make_idesc_bf16(KBT, QBT, false, false);   // K-major A and B
      constexpr uint32_t idesc_a = make_idesc_bf16(KBT, H, false, true);      // B MN-major
      bool ok = mbar_wait(smem_u32(kv_full), 0, p.status, kErrTimeoutMma, p.budget_ns);
      auto issue_s = [&](int it) -> bool {
        const int st = it & 1;
        if (!mbar_wait(smem_u32(&qd_full[st]), (it >> 1) & 1, p.status, kErrTimeoutMma, p.budget_ns)) return false;
        tc_fence_after();
        const uint32_t sq = sQ0 + st * QT_BYTES, sd = sD0 + st * QT_BYTES;
#pragma unroll
        for (int kk = 0; kk < H / 16; ++kk) {
          umma_f16(tmem + ST_COL, kdesc(sK, KBT, kk), kdesc(sq, QBT, kk), idesc_s, kk != 0 ? 1u : 0u);
          umma_f16(tmem + DPT_COL, kdesc(sV, KBT, kk), kdesc(sd, QBT, kk), idesc_s, kk != 0 ? 1u : 0u);
        }
        umma_commit(smem_u32(s_full));
        return true;
      };
      if (ok && total > 0) ok = issue_s(0);
      for (int it = 0; ok && it < total; ++it) {
        if (!mbar_wait(smem_u32(p_full), it & 1, p.status, kErrTimeoutMma, p.budget_ns)) break;
        tc_fence_after();
        const int st = it & 1;
        const uint32_t sq = sQ0 + st * QT_BYTES, sd = sD0 + st * QT_BYTES;
#pragma unroll
        for (int kk = 0; kk < QBT / 16; ++kk) {
          umma_f16(tmem + DV_COL, make_smem_desc(sPt + kk * 32, 16, 1024), make_smem_desc(sd + kk * 2048, 8192, 1024),
                   idesc_a, (it | kk) != 0 ? 1u : 0u);
          umma_f16(tmem + DK_COL, make_smem_desc(sSt + kk * 32, 16, 1024), make_smem_desc(sq + kk * 2048, 8192, 1024),
                   idesc_a, (it | kk) != 0 ? 1u : 0u);
        }
        umma_commit(smem_u32(pv_done));
        umma_commit(smem_u32(&qd_empty[st]));
        if (it + 1 < total) ok = issue_s(it + 1);
      }
    }
  } else {
    // ------------------------------------------------------------ P^T / dS^T, epilogue
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quad * 32 + lane;        // key row of the tile == TMEM lane
    const int kj = k0 + r;
    const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
    bool ok = true;
    for (int it = 0; it < total; ++it) {
      if (ok) ok = mbar_wait(smem_u32(s_full), it & 1, p.status, kErrTimeoutEpilogue, p.budget_ns);
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
      const int st = it & 1;
      const int q0 = (ib0 + it % nq) * QBT + half * 32;   // this thread's 32 queries
      const bool need_mask = q0 < k0 + KBT || p.window > 0 || q0 + 32 > p.S;
      uint32_t sv[32], dv[32];
      tmem_ld_32x32b_x32(trow + ST_COL + half * 32, sv);
      tmem_ld_32x32b_x32(trow + DPT_COL + half * 32, dv);
      tmem_ld_wait();
      // the P^T / dS^T tiles are free once the previous tile's dV / dK MMAs are done
      if (it > 0) {
        if (ok) ok = mbar_wait(smem_u32(pv_done), (it - 1) & 1, p.status, kErrTimeoutEpilogue, p.budget_ns);
        ok = __all_sync(0xffffffffu, ok);
      }
      const float* lse = sLse + st * QBT + half * 32;
      const float* del = sDel + st * QBT + half * 32;
      float pt[32], ds[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        float pv = ex2(fmaf(__uint_as_float(sv[e]), p.sl2, -lse[e]));
        if (need_mask && !visible_b(p, q0 + e, kj)) pv = 0.f;
        pt[e] = pv;
        ds[e] = pv * (__uint_as_float(dv[e]) - del[e]);
      }
      const uint32_t off = r * 128;
#pragma unroll
      for (int q8 = 0; q8 < 4; ++q8) {
        const int chunk = half * 4 + q8;
        const uint32_t sw = off + ((chunk ^ (r & 7)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(sPt + sw),
                     "r"(pack_bf16x2(pt[q8 * 8 + 0], pt[q8 * 8 + 1])), "r"(pack_bf16x2(pt[q8 * 8 + 2], pt[q8 * 8 + 3])),
                     "r"(pack_bf16x2(pt[q8 * 8 + 4], pt[q8 * 8 + 5])), "r"(pack_bf16x2(pt[q8 * 8 + 6], pt[q8 * 8 + 7]))
                     : "memory");
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(sSt + sw),
                     "r"(pack_bf16x2(ds[q8 * 8 + 0], ds[q8 * 8 + 1])), "r"(pack_bf16x2(ds[q8 * 8 + 2], ds[q8 * 8 + 3])),
                     "r"(pack_bf16x2(ds[q8 * 8 + 4], ds[q8 * 8 + 5])), "r"(pack_bf16x2(ds[q8 * 8 + 6], ds[q8 * 8 + 7]))
                     : "memory");
      }
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(smem_u32(p_full));
    }
    if (ok && total > 0) ok = mbar_wait(smem_u32(pv_done), (total - 1) & 1, p.status, kErrTimeoutEpilogue, p.budget_ns);
    if (__all_sync(0xffffffffu, ok)) {
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < HC; ++c) {
      const int col = half * (H / 2) + 32 * c;
      uint32_t vv[32], kv[32];
      tmem_ld_32x32b_x32(trow + DV_COL + col, vv);
      tmem_ld_32x32b_x32(trow + DK_COL + col, kv);
      tmem_ld_wait();
      if (kj < p.S) {
        const long long o = ((long long)b * p.S + kj) * p.kv_row + hk * H + col;
        uint4* dv4 = reinterpret_cast<uint4*>(p.dv + o);
        uint4* dk4 = reinterpret_cast<uint4*>(p.dk + o);
        const bool any = total > 0;
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          uint4 w, u;
          const float* fv = reinterpret_cast<const float*>(vv) + q8 * 8;
          const float* fk = reinterpret_cast<const float*>(kv) + q8 * 8;
          w.x = pack_bf16x2(any ? fv[0] : 0.f, any ? fv[1] : 0.f);
          w.y = pack_bf16x2(any ? fv[2] : 0.f, any ? fv[3] : 0.f);
          w.z = pack_bf16x2(any ? fv[4] : 0.f, any ? fv[5] : 0.f);
          w.w = pack_bf16x2(any ? fv[6] : 0.f, any ? fv[7] : 0.f);
          u.x = pack_bf16x2(any ? fk[0] * p.scale : 0.f, any ? fk[1] * p.scale : 0.f);
          u.y = pack_bf16x2(any ? fk[2] * p.scale : 0.f, any ? fk[3] * p.scale : 0.f);
          u.z = pack_bf16x2(any ? fk[4] * p.scale : 0.f, any ? fk[5] * p.scale : 0.f);
          u.w = pack_bf16x2(any ? fk[6] * p.scale : 0.f, any ? fk[7] * p.scale : 0.f);
          dv4[q8] = w;
          dk4[q8] = u;
        }
      }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, BWD_TMEM);
}


// ============================================================== backward dQ
// CTA = 128 queries of one head; loops over the key tiles of 64 they see:
//   S = Q K_j^T,  dP = dO V_j^T                  (M 128 x N 64, TMEM)
//   dS = P (dP - delta),  P = exp2(S * scale * log2e - lse)  (two threads per row)
//   dQ += dS K_j                                 (M 128 x N 64 x K 64, TMEM)
// then dQ * scale -> bf16.
constexpr int DQ_THREADS = 320;
constexpr int DQ_KB = 64;
constexpr int DQ_TMEM = 256;
constexpr int DQ_S = 0, DQ_DP = 64, DQ_ACC = 128;
template <int H>
struct BwdQ {
  static constexpr int Q_BYTES = BQ * H * 2;
  static constexpr int KT = DQ_KB * H * 2;      // 8 / 16 KB
  static constexpr int SMEM = 2 * Q_BYTES + 2 * 2 * KT + BQ * DQ_KB * 2 + 1024 + 256;
};

struct DqParams {
  int B, S, Nq, Nkv, window;
  float scale, sl2;
  const float *lse, *delta;
  __nv_bfloat16* dq;
  long long q_row;
  int* status;
  unsigned long long budget_ns;
};

HB_DEVICE bool visible_q(const DqParams& p, int qi, int kj) {
  return kj <= qi && (p.window <= 0 || qi - kj < p.window) && kj < p.S && qi < p.S;
}

template <int H>
__global__ void __launch_bounds__(DQ_THREADS, H == 64 ? 2 : 1)
    bwd_q_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmD,
                    const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                    const DqParams p) {
  constexpr int Q_BYTES = BwdQ<H>::Q_BYTES, DQ_KT = BwdQ<H>::KT;
  constexpr int HC = H / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sD = sQ + Q_BYTES;
  const uint32_t sK0 = sD + Q_BYTES;           // 2 stages of K then of V
  const uint32_t sV0 = sK0 + 2 * DQ_KT;
  const uint32_t sS = sV0 + 2 * DQ_KT;         // dS tile
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 2 * Q_BYTES + 4 * DQ_KT + BQ * DQ_KB * 2);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;    // [2]
  uint64_t* kv_empty = bars + 3;   // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* p_full = bars + 6;
  uint64_t* pv_done = bars + 7;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nqt = (p.S + BQ - 1) / BQ;
  const int qt = nqt - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Nq / p.Nkv);
  const int q0 = qt * BQ;
  const int hi = min(p.S, q0 + BQ);
  const int lo = p.window > 0 ? max(0, q0 - p.window + 1) : 0;
  const int jb0 = lo / DQ_KB, jb1 = (hi + DQ_KB - 1) / DQ_KB;
  const int nkt = jb1 - jb0;
  const int row0 = b * p.S;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    for (int st = 0; st < 2; ++st) {
      mbar_init(smem_u32(&kv_full[st]), 1);
      mbar_init(smem_u32(&kv_empty[st]), 1);
    }
    mbar_init(smem_u32(s_full), 1);
    mbar_init(smem_u32(p_full), 256);
    mbar_init(smem_u32(pv_done), 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), DQ_TMEM);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      mbar_expect_tx(smem_u32(q_full), 2 * Q_BYTES);
      load_tile<H>(sQ, &tmQ, smem_u32(q_full), h * H, row0 + q0, BQ);
      load_tile<H>(sD, &tmD, smem_u32(q_full), h * H, row0 + q0, BQ);
      for (int j = 0; j < nkt; ++j) {
        const int st = j & 1;
        if (!mbar_wait(smem_u32(&kv_empty[st]), ((j >> 1) & 1) ^ 1, p.status, kErrTimeoutProducer, p.budget_ns))
          break;
        const uint32_t fb = smem_u32(&kv_full[st]);
        mbar_expect_tx(fb, 2 * DQ_KT);
        const int k0 = (jb0 + j) * DQ_KB;
        load_tile<H>(sK0 + st * DQ_KT, &tmK, fb, hk * H, row0 + k0, DQ_KB);
        load_tile<H>(sV0 + st * DQ_KT, &tmV, fb, hk * H, row0 + k0, DQ_KB);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc_s = make_idesc_bf16(BQ, DQ_KB, false, false);
      constexpr uint32_t idesc_q = make_idesc_bf16(BQ, H, false, true);
      bool ok = mbar_wait(smem_u32(q_full), 0, p.status, kErrTimeoutMma, p.budget_ns);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(smem_u32(&kv_full[st]), (j >> 1) & 1, p.status, kErrTimeoutMma, p.budget_ns)) return false;
        tc_fence_after();
        const uint32_t sk = sK0 + st * DQ_KT, sv = sV0 + st * DQ_KT;
#pragma unroll
        for (int kk = 0; kk < H / 16; ++kk) {
          umma_f16(tmem + DQ_S, kdesc(sQ, BQ, kk), kdesc(sk, DQ_KB, kk), idesc_s, kk != 0 ? 1u : 0u);
          umma_f16(tmem + DQ_DP, kdesc(sD, BQ, kk), kdesc(sv, DQ_KB, kk), idesc_s, kk != 0 ? 1u : 0u);
        }
        umma_commit(smem_u32(s_full));
        return true;
      };
      if (ok && nkt > 0) ok = issue_s(0);
      for (int j = 0; ok && j < nkt; ++j) {
        if (!mbar_wait(smem_u32(p_full), j & 1, p.status, kErrTimeoutMma, p.budget_ns)) break;
        tc_fence_after();
        const uint32_t sk = sK0 + (j & 1) * DQ_KT;
#pragma unroll
        for (int kk = 0; kk < DQ_KB / 16; ++kk)
          umma_f16(tmem + DQ_ACC, make_smem_desc(sS + kk * 32, 16, 1024), make_smem_desc(sk + kk * 2048, 8192, 1024),
                   idesc_q, (j | kk) != 0 ? 1u : 0u);
        umma_commit(smem_u32(pv_done));
        umma_commit(smem_u32(&kv_empty[j & 1]));
        if (j + 1 < nkt) ok = issue_s(j + 1);
      }
    }
  } else {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quad * 32 + lane;
    const int qi = q0 + r;
    const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
    const bool qin = qi < p.S;
    const long long li = ((long long)b * p.Nq + h) * p.S + (qin ? qi : 0);
    const float lse = qin ? p.lse[li] : INFINITY;
    const float del = qin ? p.delta[li] : 0.f;
    bool ok = true;
    for (int j = 0; j < nkt; ++j) {
      // after a timeout the loop keeps going without waiting (no early exit)
      if (ok) ok = mbar_wait(smem_u32(s_full), j & 1, p.status, kErrTimeoutEpilogue, p.budget_ns);
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
      const int k0 = (jb0 + j) * DQ_KB + half * 32;
      const bool need_mask = (k0 + 32 > q0) || p.window > 0 || (k0 + 32 > p.S);
      uint32_t sv[32], dv[32];
      tmem_ld_32x32b_x32(trow + DQ_S + half * 32, sv);
      tmem_ld_32x32b_x32(trow + DQ_DP + half * 32, dv);
      tmem_ld_wait();
      if (j > 0) {   // the dS tile is free once the previous dQ MMA is done
        if (ok) ok = mbar_wait(smem_u32(pv_done), (j - 1) & 1, p.status, kErrTimeoutEpilogue, p.budget_ns);
        ok = __all_sync(0xffffffffu, ok);
      }
      float ds[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        float pv = ex2(fmaf(__uint_as_float(sv[e]), p.sl2, -lse));
        if (need_mask && !visible_q(p, qi, k0 + e)) pv = 0.f;
        ds[e] = pv * (__uint_as_float(dv[e]) - del);
      }
      const uint32_t off = r * 128;
#pragma unroll
      for (int q8 = 0; q8 < 4; ++q8) {
        const int chunk = half * 4 + q8;
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(sS + off + ((chunk ^ (r & 7)) << 4)),
                     "r"(pack_bf16x2(ds[q8 * 8 + 0], ds[q8 * 8 + 1])), "r"(pack_bf16x2(ds[q8 * 8 + 2], ds[q8 * 8 + 3])),
                     "r"(pack_bf16x2(ds[q8 * 8 + 4], ds[q8 * 8 + 5])), "r"(pack_bf16x2(ds[q8 * 8 + 6], ds[q8 * 8 + 7]))
                     : "memory");
      }
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(smem_u32(p_full));
    }
    if (ok && nkt > 0) ok = mbar_wait(smem_u32(pv_done), (nkt - 1) & 1, p.status, kErrTimeoutEpilogue, p.budget_ns);
    if (__all_sync(0xffffffffu, ok) && nkt > 0) {
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < HC; ++c) {
      const int col = half * (H / 2) + 32 * c;
      uint32_t v[32];
      tmem_ld_32x32b_x32(trow + DQ_ACC + col, v);
      tmem_ld_wait();
      if (qin) {
        uint4* o4 = reinterpret_cast<uint4*>(p.dq + ((long long)b * p.S + qi) * p.q_row + h * H + col);
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          const float* f = reinterpret_cast<const float*>(v) + q8 * 8;
          uint4 w;
          w.x = pack_bf16x2(f[0] * p.scale, f[1] * p.scale);
          w.y = pack_bf16x2(f[2] * p.scale, f[3] * p.scale);
          w.z = pack_bf16x2(f[4] * p.scale, f[5] * p.scale);
          w.w = pack_bf16x2(f[6] * p.scale, f[7] * p.scale);
          o4[q8] = w;
        }
      }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, DQ_TMEM);
}

}  // namespace fatc

namespace {
template <int H>
void fwd_tc_launch(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor lse,
                   int64_t window) {
  const int B = q.size(0), S = q.size(1), Nq = q.size(2), Nkv = k.size(2);
  fatc::TcParams p{};
  p.B = B;
  p.S = S;
  p.Nq = Nq;
  p.Nkv = Nkv;
  p.window = (int)window;
  p.sl2 = (1.f / std::sqrt((float)H)) * fatc::LOG2E;
  p.q_row = (long long)Nq * H;
  p.out = (__nv_bfloat16*)out.data_ptr();
  p.lse = lse.data_ptr<float>();
  p.status = status_ptr();
  p.budget_ns = wait_budget_ns();
  const uint64_t rows = (uint64_t)B * S;
  CUtensorMap tq = tmap_bf16_2d(q.data_ptr(), rows, (uint64_t)Nq * H, (uint64_t)Nq * H, 64, fatc::BQ);
  CUtensorMap tk = tmap_bf16_2d(k.data_ptr(), rows, (uint64_t)Nkv * H, (uint64_t)Nkv * H, 64, fatc::BK);
  CUtensorMap tv = tmap_bf16_2d(v.data_ptr(), rows, (uint64_t)Nkv * H, (uint64_t)Nkv * H, 64, fatc::BK);
  static bool configured = false;
  if (!configured) {
    HB_CUDA_CHECK(cudaFuncSetAttribute(fatc::fwd_tc_kernel<H>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       fatc::Fwd<H>::SMEM));
    configured = true;
  }
  dim3 grid((S + fatc::BQ - 1) / fatc::BQ, Nq, B);
  fatc::fwd_tc_kernel<H><<<grid, fatc::THREADS, fatc::Fwd<H>::SMEM, cur_stream()>>>(tq, tk, tv, p);
  HB_CUDA_CHECK(cudaGetLastError());
}

template <int H>
void bwd_kv_tc_launch(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor dout, torch::Tensor lse,
                      torch::Tensor delta, torch::Tensor dk, torch::Tensor dv, int64_t window) {
  const int B = q.size(0), S = q.size(1), Nq = q.size(2), Nkv = k.size(2);
  fatc::BwdParams p{};
  p.B = B;
  p.S = S;
  p.Nq = Nq;
  p.Nkv = Nkv;
  p.window = (int)window;
  p.scale = 1.f / std::sqrt((float)H);
  p.sl2 = p.scale * fatc::LOG2E;
  p.lse = lse.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  p.dk = (__nv_bfloat16*)dk.data_ptr();
  p.dv = (__nv_bfloat16*)dv.data_ptr();
  p.kv_row = (long long)Nkv * H;
  p.status = status_ptr();
  p.budget_ns = wait_budget_ns();
  const uint64_t rows = (uint64_t)B * S;
  CUtensorMap tk = tmap_bf16_2d(k.data_ptr(), rows, (uint64_t)Nkv * H, (uint64_t)Nkv * H, 64, fatc::KBT);
  CUtensorMap tv = tmap_bf16_2d(v.data_ptr(), rows, (uint64_t)Nkv * H, (uint64_t)Nkv * H, 64, fatc::KBT);
  CUtensorMap tq = tmap_bf16_2d(q.data_ptr(), rows, (uint64_t)Nq * H, (uint64_t)Nq * H, 64, fatc::QBT);
  CUtensorMap td = tmap_bf16_2d(dout.data_ptr(), rows, (uint64_t)Nq * H, (uint64_t)Nq * H, 64, fatc::QBT);
  static bool configured = false;
  if (!configured) {
    HB_CUDA_CHECK(cudaFuncSetAttribute(fatc::bwd_kv_tc_kernel<H>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       fatc::BwdKV<H>::SMEM));
    configured = true;
  }
  dim3 grid((S + fatc::KBT - 1) / fatc::KBT, Nkv, B);
  fatc::bwd_kv_tc_kernel<H><<<grid, fatc::BWD_THREADS, fatc::BwdKV<H>::SMEM, cur_stream()>>>(tk, tv, tq, td, p);
  HB_CUDA_CHECK(cudaGetLastError());
}

template <int H>
void bwd_q_tc_launch(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor dout, torch::Tensor lse,
                     torch::Tensor delta, torch::Tensor dq, int64_t window) {
  const int B = q.size(0), S = q.size(1), Nq = q.size(2), Nkv = k.size(2);
  fatc::DqParams p{};
  p.B = B;
  p.S = S;
  p.Nq = Nq;
  p.Nkv = Nkv;
  p.window = (int)window;
  p.scale = 1.f / std::sqrt((float)H);
  p.sl2 = p.scale * fatc::LOG2E;
  p.lse = lse.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  p.dq = (__nv_bfloat16*)dq.data_ptr();
  p.q_row = (long long)Nq * H;
  p.status = status_ptr();
  p.budget_ns = wait_budget_ns();
  const uint64_t rows = (uint64_t)B * S;
  CUtensorMap tq = tmap_bf16_2d(q.data_ptr(), rows, (uint64_t)Nq * H, (uint64_t)Nq * H, 64, fatc::BQ);
  CUtensorMap td = tmap_bf16_2d(dout.data_ptr(), rows, (uint64_t)Nq * H, (uint64_t)Nq * H, 64, fatc::BQ);
  CUtensorMap tk = tmap_bf16_2d(k.data_ptr(), rows, (uint64_t)Nkv * H, (uint64_t)Nkv * H, 64, fatc::DQ_KB);
  CUtensorMap tv = tmap_bf16_2d(v.data_ptr(), rows, (uint64_t)Nkv * H, (uint64_t)Nkv * H, 64, fatc::DQ_KB);
  static bool configured = false;
  if (!configured) {
    HB_CUDA_CHECK(cudaFuncSetAttribute(fatc::bwd_q_tc_kernel<H>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       fatc::BwdQ<H>::SMEM));
    configured = true;
  }
  dim3 grid((S + fatc::BQ - 1) / fatc::BQ, Nq, B);
  fatc::bwd_q_tc_kernel<H><<<grid, fatc::DQ_THREADS, fatc::BwdQ<H>::SMEM, cur_stream()>>>(tq, td, tk, tv, p);
  HB_CUDA_CHECK(cudaGetLastError());
}
}  // namespace

// q [B,S,Nq,H], k/v [B,S,Nkv,H] bf16 contiguous (H = 64 or 128); out like q;
// lse [B,Nq,S] fp32.
void flash_fwd_tc(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor lse,
                  int64_t window) {
  const c10::cuda::CUDAGuard guard(q.device());
  if (q.size(3) == 64) fwd_tc_launch<64>(q, k, v, out, lse, window);
  else if (q.size(3) == 128) fwd_tc_launch<128>(q, k, v, out, lse, window);
  else HB_CHECK(false, "flash_fwd_tc: head dim 64 or 128");
}

// dK, dV of the attention backward on tcgen05; lse / delta as produced by the
// forward and the delta kernel.
void flash_bwd_kv_tc(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor dout, torch::Tensor lse,
                     torch::Tensor delta, torch::Tensor dk, torch::Tensor dv, int64_t window) {
  const c10::cuda::CUDAGuard guard(q.device());
  if (q.size(3) == 64) bwd_kv_tc_launch<64>(q, k, v, dout, lse, delta, dk, dv, window);
  else if (q.size(3) == 128) bwd_kv_tc_launch<128>(q, k, v, dout, lse, delta, dk, dv, window);
  else HB_CHECK(false, "flash_bwd_kv_tc: head dim 64 or 128");
}

// dQ of the attention backward on tcgen05.
void flash_bwd_q_tc(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor dout, torch::Tensor lse,
                    torch::Tensor delta, torch::Tensor dq, int64_t window) {
  const c10::cuda::CUDAGuard guard(q.device());
  if (q.size(3) == 64) bwd_q_tc_launch<64>(q, k, v, dout, lse, delta, dq, window);
  else if (q.size(3) == 128) bwd_q_tc_launch<128>(q, k, v, dout, lse, delta, dq, window);
  else HB_CHECK(false, "flash_bwd_q_tc: head dim 64 or 128");
}

}  // namespace hb
