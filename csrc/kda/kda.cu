// Kimi Delta Attention: chunk-parallel gated delta rule, forward and backward,
// plus the fused front-end (ShortConv4 + SiLU + L2 norm, decay gate, beta).
//
// Recurrence (model/kda.py:305-323), per token t with state S [K, V]:
//   S <- diag(e^{g_t}) S;  v' = v_t - b_t S^T k_t;  S <- S + b_t k_t v'^T;
//   o_t = scale * S^T q_t          (readout after the update)
// Chunk form (chunk C, incoming state S0, G = cumsum(g) inside the chunk):
//   A_ts = sum_c k_t k_s e^{G_t-G_s} (s<t),  P_ts = scale sum_c q_t k_s e^{G_t-G_s} (s<=t)
//   L = I + diag(b^2) A;  Ut = L^{-1} diag(b) V;  Wt = L^{-1} diag(b^2) (K*e^G)
//   U = Ut - Wt S0;  O = scale (Q*e^G) S0 + P U;  S_C = e^{G_C} S0 + (K*e^{G_C-G})^T U
// Pairwise decays are evaluated as exp(G_t - G_s) of the difference, never as
// exp(G_t) / exp(G_s), so strongly negative cumulative decays cannot underflow
// into 0/0.  All arithmetic is fp32.
//
// Kernels
//   kda_intra_fwd   grid (chunks, H, B): everything that does not depend on S0
//   kda_state_fwd   grid (H, B): the sequential chunk recurrence; stores S0 of
//                   every chunk for the backward
//   kda_state_bwd   grid (H, B): reverse recurrence of dS (state gradient)
//   kda_intra_bwd   grid (chunks, H, B): recomputes the chunk and emits dq, dk,
//                   dv, dg, dbeta given S0, dS_C and dO
#include <torch/extension.h>

#include <mutex>

#include "../common/host.h"
#include "../common/sm100.cuh"
#include "kda_common.cuh"

namespace hb {
namespace kda {

// Pairwise products with log-space decay, for rows t >= columns s:
//   A_ts = sum_c k_t k_s e^{G_t-G_s} (s < t, else 0),  N = diag(b^2) A,
//   P_ts = scale sum_c q_t k_s e^{G_t-G_s} (s <= t, else 0).
// Lane = row t (C == 32); warp w owns columns s = w, w + nw, ...  Each lane
// streams its own row in 16-byte pieces and accumulates against the warp's
// columns (broadcast reads): no cross-lane reductions.  Pairs with s > t are
// computed and discarded by a select, never multiplied in.
template <int DK, int C, bool WRITE_A>
HB_DEVICE void pair_products(const float* q, const float* k, const float* G, const float* bet, float* A,
                             float* N, float* P, float scale) {
  static_assert(C == 32, "one lane per chunk row");
  constexpr int L = LDK<DK>(), LC = LDC<C>();
  constexpr int MS = 4;
  const int nw = blockDim.x >> 5, warp = threadIdx.x >> 5, t = threadIdx.x & 31;
  for (int s0 = warp; s0 < C; s0 += nw * MS) {
    float a[MS], pp[MS];
#pragma unroll
    for (int j = 0; j < MS; ++j) a[j] = pp[j] = 0.f;
    for (int c = 0; c < DK; c += 4) {
      const float4 kt = ld4(k + t * L + c), gt = ld4(G + t * L + c), qt = ld4(q + t * L + c);
#pragma unroll
      for (int j = 0; j < MS; ++j) {
        const int s = s0 + j * nw;
        if (s >= C) break;
        const float4 ks = ld4(k + s * L + c), gs = ld4(G + s * L + c);
        const float e0 = exp2_fast(gt.x - gs.x) * ks.x, e1 = exp2_fast(gt.y - gs.y) * ks.y;
        const float e2 = exp2_fast(gt.z - gs.z) * ks.z, e3 = exp2_fast(gt.w - gs.w) * ks.w;
        a[j] += kt.x * e0 + kt.y * e1 + kt.z * e2 + kt.w * e3;
        pp[j] += qt.x * e0 + qt.y * e1 + qt.z * e2 + qt.w * e3;
      }
    }
#pragma unroll
    for (int j = 0; j < MS; ++j) {
      const int s = s0 + j * nw;
      if (s >= C) break;
      const float av = s < t ? a[j] : 0.f;
      if (WRITE_A) A[t * LC + s] = av;
      N[t * LC + s] = bet[t] * bet[t] * av;
      P[t * LC + s] = s <= t ? pp[j] * scale : 0.f;
    }
  }
  __syncthreads();
}


// ------------------------------------------------------------------ intra fwd
template <int DK, int C>
__global__ void __launch_bounds__(256) intra_fwd_kernel(Ptrs p) {
  constexpr int L = LDK<DK>(), LC = LDC<C>(), D4 = DK / 4;
  extern __shared__ float sm[];
  float* q = sm;
  float* k = q + C * L;
  float* v = k + C * L;          // v, then Ut
  float* G = v + C * L;
  float* Wt = G + C * L;
  float* N = Wt + C * L;         // C x LC
  float* P = N + C * LC;         // C x LC
  float* bet = P + C * LC;       // C
  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  load_chunk<DK, C>(p, b, h, n, q, k, v, G, bet);
  pair_products<DK, C, false>(q, k, G, bet, nullptr, N, P, p.scale);
  // Ut = L^{-1} b v (in place),  Wt = L^{-1} b^2 k e^G
  solve_cols<C, false>(
      2 * DK, N,
      [&](int t, int col) {
        return col < DK ? bet[t] * v[t * L + col]
                        : bet[t] * bet[t] * k[t * L + col - DK] * exp2_fast(G[t * L + col - DK]);
      },
      [&](int t, int col, float x) {
        if (col < DK) v[t * L + col] = x;
        else Wt[t * L + col - DK] = x;
      });
  __syncthreads();
  const long long co = chunk_off(p, b, h, n, C * DK);
  const float* GC = G + (C - 1) * L;
  for (int i = threadIdx.x; i < C * D4; i += blockDim.x) {
    const int r = i / D4, c = (i % D4) * 4;
    const int si = r * L + c;
    const float4 kk = ld4(k + si), gg = ld4(G + si), qq = ld4(q + si), gc = ld4(GC + c);
    st4(p.Ut + co + r * DK + c, ld4(v + si));
    st4(p.Wt + co + r * DK + c, ld4(Wt + si));
    st4(p.Kh + co + r * DK + c, make_float4(kk.x * exp2_fast(gc.x - gg.x), kk.y * exp2_fast(gc.y - gg.y),
                                            kk.z * exp2_fast(gc.z - gg.z), kk.w * exp2_fast(gc.w - gg.w)));
    const float sc = p.scale;
    st4(p.Qg + co + r * DK + c, make_float4(sc * qq.x * exp2_fast(gg.x), sc * qq.y * exp2_fast(gg.y),
                                            sc * qq.z * exp2_fast(gg.z), sc * qq.w * exp2_fast(gg.w)));
  }
  const long long po = chunk_off(p, b, h, n, C * C);
  for (int i = threadIdx.x; i < C * C / 4; i += blockDim.x) {
    const int r = i / (C / 4), c = (i % (C / 4)) * 4;
    st4(p.Pm + po + r * C + c, ld4(P + r * LC + c));
  }
  for (int c = threadIdx.x; c < DK; c += blockDim.x) p.gC[chunk_off(p, b, h, n, DK) + c] = exp2_fast(GC[c]);
}


// ------------------------------------------------------------------ intra bwd
// Rows of the [DK, DK] state matrices streamed per step (two panels in smem).
template <int DK>
constexpr int PANEL() { return DK >= 128 ? 16 : 8; }

// Recomputes the chunk (A, N, P, Ut, Wt, U) and emits dq, dk, dv, dg, dbeta
// given S0 (state entering the chunk), dS_C (gradient of the state leaving
// it) and dO.  S0 and dS_C are read in row panels, twice (the second pass
// needs the completed U and dU):
//   pass 1: U -= Wt S0,  dU += Kh dS_C,  dQg = dO S0^T,  dgC = rowsum(dS_C * S0)
//   pass 2: dWt = -dU S0^T,  dKh = U dS_C^T
template <int DK, int C>
__global__ void __launch_bounds__(NTB<DK>(), DK >= 128 ? 1 : 2) intra_bwd_kernel(Ptrs p) {
  constexpr int L = LDK<DK>(), LC = LDC<C>(), D4 = DK / 4, PR = PANEL<DK>();
  extern __shared__ float sm[];
  float* q = sm;                 // C x L each
  float* k = q + C * L;
  float* v = k + C * L;          // v, later dv
  float* G = v + C * L;
  float* dO = G + C * L;         // dO, later X = L^{-T} dU
  float* U = dO + C * L;         // Ut -> U, later dG
  float* dU = U + C * L;         // dU, later Ut / Wt (recomputed)
  float* T0 = dU + C * L;        // Wt -> dWt -> Y = L^{-T} dWt
  float* T1 = T0 + C * L;        // Kh -> dKh -> dk
  float* T2 = T1 + C * L;        // dQg -> dq
  float* S0p = T2 + C * L;       // PR x L
  float* dSp = S0p + PR * L;     // PR x L
  float* A = dSp + PR * L;       // C x LC
  float* N = A + C * LC;         // C x LC
  float* P = N + C * LC;         // C x LC, later dP
  float* dA = P + C * LC;        // C x LC
  float* bet = dA + C * LC;      // C
  float* dbt = bet + C;          // C
  float* red = dbt + C;          // DK
  float* dgc = red + DK;         // DK
  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const float scale = p.scale;
  load_rows<DK, C>(p, p.dout, b, h, n, dO);
  load_chunk<DK, C>(p, b, h, n, q, k, v, G, bet);
  pair_products<DK, C, true>(q, k, G, bet, A, N, P, scale);
  const float* GC = G + (C - 1) * L;
  // Ut -> U, Wt -> T0;  Kh -> T1
  solve_cols<C, false>(
      2 * DK, N,
      [&](int t, int col) {
        return col < DK ? bet[t] * v[t * L + col]
                        : bet[t] * bet[t] * k[t * L + col - DK] * exp2_fast(G[t * L + col - DK]);
      },
      [&](int t, int col, float x) {
        if (col < DK) U[t * L + col] = x;
        else T0[t * L + col - DK] = x;
      });
  for (int e = threadIdx.x; e < C * DK; e += blockDim.x) {
    const int t = e / DK, c = e % DK;
    T1[t * L + c] = k[t * L + c] * exp2_fast(GC[c] - G[t * L + c]);
  }
  __syncthreads();
  // dU = P^T dO
  mm<C, DK, C, true, false>(dU, L, P, LC, dO, L, 1.f, false);
  __syncthreads();
  const long long so = chunk_off(p, b, h, n, DK * DK);
  // panel rows are fetched into registers one panel ahead (the loads overlap
  // the current panel's math) and stored to shared memory between barriers
  static_assert(PR * D4 <= NTB<DK>(), "one 16-byte piece of each panel per thread");
  const bool pl = threadIdx.x < PR * D4;
  const int pr = threadIdx.x / D4, pc = (threadIdx.x % D4) * 4;
  float4 nx_s = make_float4(0.f, 0.f, 0.f, 0.f), nx_d = nx_s;
  auto fetch_panel = [&](int kp) {
    if (pl && kp < DK) {
      const long long g = so + (long long)(kp + pr) * DK + pc;
      nx_s = ld4(p.states + g);
      nx_d = ld4(p.dstates + g);
    }
  };
  auto put_panel = [&]() {
    if (pl) {
      st4(S0p + pr * L + pc, nx_s);
      st4(dSp + pr * L + pc, nx_d);
    }
  };
  fetch_panel(0);
  for (int kp = 0; kp < DK; kp += PR) {
    put_panel();
    __syncthreads();
    fetch_panel(kp + PR < DK ? kp + PR : 0);  // pass 2 starts again at panel 0
    mm<C, DK, PR, false, false>(U, L, T0 + kp, L, S0p, L, -1.f, true);
    mm<C, DK, PR, false, false>(dU, L, T1 + kp, L, dSp, L, 1.f, true);
    mm<C, PR, DK, false, true>(T2 + kp, L, dO, L, S0p, L, 1.f, false);
    for (int r = warp; r < PR; r += nw) {
      float s = 0.f;
      for (int c = lane; c < DK; c += 32) s += dSp[r * L + c] * S0p[r * L + c];
      s = warp_sum(s);
      if (lane == 0) dgc[kp + r] = s;
    }
    __syncthreads();
  }
  // dP = dO U^T (into P; masked to s <= t below)
  mm<C, C, DK, false, true>(P, LC, dO, L, U, L, 1.f, false);
  for (int kp = 0; kp < DK; kp += PR) {
    put_panel();
    __syncthreads();
    fetch_panel(kp + PR);
    mm<C, PR, DK, false, true>(T0 + kp, L, dU, L, S0p, L, -1.f, false);
    mm<C, PR, DK, false, true>(T1 + kp, L, U, L, dSp, L, 1.f, false);
    __syncthreads();
  }
  for (int e = threadIdx.x; e < C * C; e += blockDim.x) {
    const int t = e / C, s = e % C;
    if (s > t) P[t * LC + s] = 0.f;
  }
  // red[c] = sum_t dKh Kh
  for (int c = threadIdx.x; c < DK; c += blockDim.x) {
    float s = 0.f;
#pragma unroll 8
    for (int t = 0; t < C; ++t) s += T1[t * L + c] * k[t * L + c] * exp2_fast(GC[c] - G[t * L + c]);
    red[c] = s;
  }
  __syncthreads();
  // dk = dKh e^{G_C-G} (T1);  dG = -dKh Kh + dQg scale q e^G (U);  dq = dQg scale e^G (T2)
  for (int e = threadIdx.x; e < C * DK; e += blockDim.x) {
    const int t = e / DK, c = e % DK;
    const int si = t * L + c;
    const float dkh = T1[si], dqg = T2[si];
    const float ed = exp2_fast(GC[c] - G[si]), eg = exp2_fast(G[si]);
    T1[si] = dkh * ed;
    U[si] = -dkh * k[si] * ed + dqg * scale * q[si] * eg;
    T2[si] = dqg * scale * eg;
  }
  // X = L^{-T} dU (into dO) and Y = L^{-T} dWt (in place in T0), one phase
  solve_cols<C, true>(
      2 * DK, N, [&](int t, int col) { return col < DK ? dU[t * L + col] : T0[t * L + col - DK]; },
      [&](int t, int col, float x) {
        if (col < DK) dO[t * L + col] = x;
        else T0[t * L + col - DK] = x;
      });
  __syncthreads();
  float* X = dO;
  float* Y = T0;
  // dL_ts = -(X Ut^T + Y Wt^T)_ts for s < t; Ut is recomputed into dU, then Wt
  solve_cols<C, false>(
      DK, N, [&](int t, int c) { return bet[t] * v[t * L + c]; },
      [&](int t, int c, float x) { dU[t * L + c] = x; });
  __syncthreads();
  mm<C, C, DK, false, true>(dA, LC, X, L, dU, L, -1.f, false);
  __syncthreads();
  solve_cols<C, false>(
      DK, N, [&](int t, int c) { return bet[t] * bet[t] * k[t * L + c] * exp2_fast(G[t * L + c]); },
      [&](int t, int c, float x) { dU[t * L + c] = x; });
  __syncthreads();
  mm<C, C, DK, false, true>(dA, LC, Y, L, dU, L, -1.f, true);
  __syncthreads();
  for (int e = threadIdx.x; e < C * C; e += blockDim.x) {
    const int t = e / C, s = e % C;
    if (s >= t) dA[t * LC + s] = 0.f;
  }
  __syncthreads();
  // dbeta_t = v_t . X_t + 2 b_t (sum_s A_ts dL_ts + sum_c k e^G Y)   (one warp per t)
  for (int t = warp; t < C; t += nw) {
    float s1 = 0.f, s2 = 0.f, s3 = 0.f;
    for (int s = lane; s < t; s += 32) s1 += A[t * LC + s] * dA[t * LC + s];
    for (int c = lane; c < DK; c += 32) {
      const int si = t * L + c;
      s2 += k[si] * exp2_fast(G[si]) * Y[si];
      s3 += v[si] * X[si];
    }
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    s3 = warp_sum(s3);
    if (lane == 0) dbt[t] = s3 + 2.f * bet[t] * (s1 + s2);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < C * C; e += blockDim.x) {
    const int t = e / C, s = e % C;
    dA[t * LC + s] *= bet[t] * bet[t];
  }
  // dv = b X ; dKg = b^2 Y: dk += dKg e^G, dG += dKg k e^G
  for (int e = threadIdx.x; e < C * DK; e += blockDim.x) {
    const int t = e / DK, c = e % DK;
    const int si = t * L + c;
    const float eg = exp2_fast(G[si]);
    const float dkg = bet[t] * bet[t] * Y[si];
    T1[si] += dkg * eg;
    U[si] += dkg * k[si] * eg;
    v[si] = bet[t] * X[si];
  }
  __syncthreads();
  // t-side: dq_t += scale sum_{s<=t} dP_ts k_s e_ts ; dk_t += sum_{s<t} dA_ts k_s e_ts
  for (int e = threadIdx.x; e < C * DK; e += blockDim.x) {
    const int t = e / DK, c = e % DK;
    const int si = t * L + c;
    const float gt = G[si];
    float sp = 0.f, sa = 0.f;
    for (int s = 0; s <= t; ++s) {
      const float ks = k[s * L + c] * exp2_fast(gt - G[s * L + c]);
      sp += P[t * LC + s] * ks;
      sa += dA[t * LC + s] * ks;
    }
    sp *= scale;
    T2[si] += sp;
    T1[si] += sa;
    U[si] += q[si] * sp + k[si] * sa;
  }
  __syncthreads();
  // s-side: dk_s += sum_{t>=s} (scale dP_ts q_t + dA_ts k_t) e_ts ; dG_s -= k_s * that
  for (int e = threadIdx.x; e < C * DK; e += blockDim.x) {
    const int s = e / DK, c = e % DK;
    const int si = s * L + c;
    const float gs = G[si];
    float acc = 0.f;
    for (int t = s; t < C; ++t) {
      const float ee = exp2_fast(G[t * L + c] - gs);
      acc += (scale * P[t * LC + s] * q[t * L + c] + dA[t * LC + s] * k[t * L + c]) * ee;
    }
    T1[si] += acc;
    U[si] -= k[si] * acc;
  }
  __syncthreads();
  // dG_C += red + dgC e^{G_C};  dg = reverse cumsum of dG
  for (int c = threadIdx.x; c < DK; c += blockDim.x) {
    float x[C];
#pragma unroll
    for (int r = 0; r < C; ++r) x[r] = U[r * L + c];
    x[C - 1] += red[c] + dgc[c] * exp2_fast(GC[c]);
#pragma unroll
    for (int r = C - 2; r >= 0; --r) x[r] += x[r + 1];
#pragma unroll
    for (int r = 0; r < C; ++r) U[r * L + c] = x[r];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < C * D4; i += blockDim.x) {
    const int r = i / D4, c = (i % D4) * 4;
    const int t = n * C + r;
    if (t >= p.S) continue;
    const long long o = tok_off(p, b, t, h, DK) + c;
    const int si = r * L + c;
    st4(p.dq + o, ld4(T2 + si));
    st4(p.dk + o, ld4(T1 + si));
    st4(p.dv + o, ld4(v + si));
    st4(p.dg + o, ld4(U + si));
  }
  for (int r = threadIdx.x; r < C; r += blockDim.x) {
    const int t = n * C + r;
    if (t < p.S) p.dbeta[((long long)b * p.S + t) * p.H + h] = dbt[r];
  }
}

template <int DK, int C>
constexpr int intra_fwd_smem() { return (5 * C * LDK<DK>() + 2 * C * LDC<C>() + C) * 4; }
template <int DK, int C>
constexpr int intra_bwd_smem() {
  return (10 * C * LDK<DK>() + 2 * PANEL<DK>() * LDK<DK>() + 4 * C * LDC<C>() + 2 * C + 2 * DK) * 4;
}

// ================================================================ front-end
// Blocks per head, two adjacent channels per lane: bf16x2 loads of the
// projection taps, float2 loads and stores of the fp32 rows.
// raw: [T, 3*HK] bf16 rows (q | k | v projections, row stride ld_raw); conv
// weights [HK, 4] fp32 each; outputs fp32 [T, H, K].
HB_DEVICE float2 ld_bf2(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}
HB_DEVICE float tap(const float4& w, int i) { return i == 0 ? w.x : i == 1 ? w.y : i == 2 ? w.z : w.w; }
HB_DEVICE float rbf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
// softplus(y) = max(y, 0) + log1p(exp(-|y|)) never overflows
HB_DEVICE float softplus_f(float y) { return fmaxf(y, 0.f) + log1pf(__expf(-fabsf(y))); }

// sigmoid by the hardware exponential and an approximate divide (2 ulp);
// 1 / (1 + inf) = 0 gives the right limit for very negative x
HB_DEVICE float sigm(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

// The conv taps of one head's channels (c, c+1) of projection `which`.
struct Taps2 { float4 a, b; };
HB_DEVICE Taps2 load_taps(const float* w, int ch) {
  return {*reinterpret_cast<const float4*>(w + ch * 4), *reinterpret_cast<const float4*>(w + ch * 4 + 4)};
}
// Causal 4-tap conv of channels (c, c+1) at offset `off` of the token rows
// rows[i] = row of token t - 3 + i (nullptr before the sequence start),
// rounded to the compute dtype (model/kda.py:136, 257-259).
HB_DEVICE float2 conv_taps(const __nv_bfloat16* const (&rows)[4], int off, const Taps2& w) {
  float a0 = 0.f, a1 = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (!rows[i]) continue;
    const float2 x = ld_bf2(rows[i] + off);
    a0 += tap(w.a, i) * x.x;
    a1 += tap(w.b, i) * x.y;
  }
  return make_float2(rbf(a0), rbf(a1));
}

// Forward (block per head, warp per token row of that head): the head's conv
// taps, dt_bias and A stay in registers across the block's rows.
template <int DK>
__global__ void __launch_bounds__(256) prep_fwd_kernel(const __nv_bfloat16* __restrict__ raw, long long ld_raw,
                                const float* __restrict__ wq, const float* __restrict__ wk,
                                const float* __restrict__ wv, const float* __restrict__ f,
                                const float* __restrict__ a_log, const float* __restrict__ dt_bias,
                                const float* __restrict__ braw, int gate_mode, int T, int S, int H,
                                float* __restrict__ q, float* __restrict__ k, float* __restrict__ v,
                                float* __restrict__ g, float* __restrict__ beta) {
  constexpr int NP = (DK + 63) / 64;
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  const int HK = H * DK, h = blockIdx.y;
  const float A = gate_mode == 0 ? -__expf(a_log[h]) : 0.f;
  Taps2 tq[NP], tk[NP], tv[NP];
  float2 db[NP];
#pragma unroll
  for (int j = 0; j < NP; ++j) {
    const int ch = h * DK + min(2 * lane + 64 * j, DK - 2);
    tq[j] = load_taps(wq, ch);
    tk[j] = load_taps(wk, ch);
    tv[j] = load_taps(wv, ch);
    db[j] = *reinterpret_cast<const float2*>(dt_bias + ch);
  }
  for (long long t = blockIdx.x * (long long)warps + (threadIdx.x >> 5); t < T; t += (long long)gridDim.x * warps) {
    const int pos = t % S;
    const __nv_bfloat16* rows[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) rows[i] = pos - (3 - i) >= 0 ? raw + (t - (3 - i)) * ld_raw : nullptr;
    float2 qv[NP], kv[NP];
    float ssq = 0.f, ssk = 0.f;
#pragma unroll
    for (int j = 0; j < NP; ++j) {
      const int c = 2 * lane + 64 * j;
      qv[j] = kv[j] = make_float2(0.f, 0.f);
      if (c >= DK) continue;
      const int ch = h * DK + c;
      const float2 cq = conv_taps(rows, ch, tq[j]), ck = conv_taps(rows, HK + ch, tk[j]),
                   cv = conv_taps(rows, 2 * HK + ch, tv[j]);
      qv[j] = make_float2(cq.x * sigm(cq.x), cq.y * sigm(cq.y));
      kv[j] = make_float2(ck.x * sigm(ck.x), ck.y * sigm(ck.y));
      ssq += qv[j].x * qv[j].x + qv[j].y * qv[j].y;
      ssk += kv[j].x * kv[j].x + kv[j].y * kv[j].y;
      const long long o = t * HK + ch;
      *reinterpret_cast<float2*>(v + o) = make_float2(cv.x * sigm(cv.x), cv.y * sigm(cv.y));
      const float2 fz = *reinterpret_cast<const float2*>(f + o);
      const float z0 = fz.x + db[j].x, z1 = fz.y + db[j].y;
      float2 gg;
      if (gate_mode == 0) {
        gg = make_float2(A * softplus_f(z0), A * softplus_f(z1));
      } else {
        gg = make_float2(-softplus_f(-z0), -softplus_f(-z1));
      }
      *reinterpret_cast<float2*>(g + o) = gg;
    }
    ssq = warp_sum(ssq);
    ssk = warp_sum(ssk);
    const float rq = rsqrtf(ssq + 1e-6f), rk = rsqrtf(ssk + 1e-6f);
#pragma unroll
    for (int j = 0; j < NP; ++j) {
      const int c = 2 * lane + 64 * j;
      if (c >= DK) continue;
      const long long o = t * HK + h * DK + c;
      *reinterpret_cast<float2*>(q + o) = make_float2(qv[j].x * rq, qv[j].y * rq);
      *reinterpret_cast<float2*>(k + o) = make_float2(kv[j].x * rk, kv[j].y * rk);
    }
    if (lane == 0) beta[t * H + h] = sigm(braw[t * H + h]);
  }
}

// Fused backward (block per head, persistent over token tiles of R rows):
// the gradient at the conv outputs never leaves shared memory.
//   stage 0: the raw projection rows t0-3 .. t0+R+2 of the block's head
//            (q | k | v columns, bf16) into shared memory;
//   stage 1: warp per row r in [0, R+3): conv + SiLU (+ L2 norm) recomputed from
//            the staged taps, dconv of rows t0 .. t0+R+2 into shared memory (the
//            last three rows are the next tile's, recomputed here); rows < R also
//            write df, dbraw and sum the bias gradients;
//   stage 2: thread per channel, sliding 4-row windows over dconv and raw:
//            draw[t] = sum_i w[i] dconv[t+3-i] (same sequence) for the R rows,
//            dw[i] += dconv[t] raw[t-3+i] in registers across tiles.
// One atomic per channel and tap per block at the end.  The kernel is
// instruction-bound, so sigmoids use the approximate divide, the L2-norm
// backward one reciprocal square root per row, and the sequence position
// is advanced instead of divided.
template <int DK>
struct PrepTile {
  static constexpr int ROWS = 2048 / DK;       // dconv rows per tile: a multiple of the 8 warps
  static constexpr int R = ROWS - 3;           // rows the tile owns (3 halo rows recomputed)
  static constexpr int C3 = 3 * DK;            // channels per head
  static constexpr int NC = (C3 + 255) / 256;  // channels per thread in stage 2
  static constexpr int smem = (R + 3) * C3 * 4 + (R + 6) * C3 * 2 + C3 * 16;
};

template <int DK>
__global__ void __launch_bounds__(256, 4) prep_bwd_fused_kernel(
    const __nv_bfloat16* __restrict__ raw, long long ld_raw, const float* __restrict__ wq,
    const float* __restrict__ wk, const float* __restrict__ wv, const float* __restrict__ f,
    const float* __restrict__ a_log, const float* __restrict__ dt_bias, const float* __restrict__ beta,
    int gate_mode, int T, int S, int H, const float* __restrict__ dq, const float* __restrict__ dk,
    const float* __restrict__ dv, const float* __restrict__ dg, const float* __restrict__ dbeta,
    __nv_bfloat16* __restrict__ df, float* __restrict__ dbraw, float* __restrict__ d_alog,
    float* __restrict__ d_dtb, __nv_bfloat16* __restrict__ draw, float* __restrict__ dwq,
    float* __restrict__ dwk, float* __restrict__ dwv) {
  using P = PrepTile<DK>;
  constexpr int R = P::R, C3 = P::C3, NP = (DK + 63) / 64;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* sdc = reinterpret_cast<float*>(smem_raw);                                      // [R+3][C3]
  __nv_bfloat16* sraw = reinterpret_cast<__nv_bfloat16*>(smem_raw + (R + 3) * C3 * 4);  // [R+6][C3]
  float4* sw = reinterpret_cast<float4*>(smem_raw + (R + 3) * C3 * 4 + (R + 6) * C3 * 2);  // [C3] taps
  __shared__ float s_dtb[DK + 1];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, warps = blockDim.x >> 5;
  const int HK = H * DK, h = blockIdx.y;
  const float A = gate_mode == 0 ? __expf(a_log[h]) : 0.f;
  for (int c = tid; c < C3; c += blockDim.x) {
    const int which = c / DK;
    const float* w = which == 0 ? wq : (which == 1 ? wk : wv);
    sw[c] = *reinterpret_cast<const float4*>(w + (h * DK + c % DK) * 4);
  }
  float2 dtb[NP], acc_dtb[NP];
#pragma unroll
  for (int j = 0; j < NP; ++j) {
    dtb[j] = *reinterpret_cast<const float2*>(dt_bias + h * DK + min(2 * lane + 64 * j, DK - 2));
    acc_dtb[j] = make_float2(0.f, 0.f);
  }
  float acc_al = 0.f;
  float dwacc[P::NC][4];
#pragma unroll
  for (int n = 0; n < P::NC; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) dwacc[n][i] = 0.f;
  for (int i = tid; i < DK + 1; i += blockDim.x) s_dtb[i] = 0.f;
  const int ntiles = (T + R - 1) / R;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int t0 = tile * R;
    const int pos0 = t0 % S;
    // ---- stage 0: raw rows t0-3 .. t0+R+2 (16-byte vectors; zero outside [0, T))
    {
      constexpr int VPR = C3 * 2 / 16;  // vectors per row
      for (int idx = tid; idx < (R + 6) * VPR; idx += blockDim.x) {
        const int r = idx / VPR, v = idx % VPR;
        const int c = v * 8, which = c / DK, cc = c % DK;
        const int t = t0 - 3 + r;
        uint4 val = make_uint4(0, 0, 0, 0);
        if (t >= 0 && t < T)
          val = *reinterpret_cast<const uint4*>(raw + (long long)t * ld_raw + which * HK + h * DK + cc);
        *reinterpret_cast<uint4*>(sraw + r * C3 + c) = val;
      }
    }
    __syncthreads();
    // ---- stage 1: dconv rows (warp per row)
    for (int r = warp; r < R + 3; r += warps) {
      const int t = t0 + r;
      float* drow = sdc + r * C3;
      if (t >= T) {
        for (int c = lane; c < C3; c += 32) drow[c] = 0.f;
        continue;
      }
      int pos = pos0 + r;
      if (pos >= S) pos %= S;
      const bool own = r < R;
      const long long orow = (long long)t * HK + h * DK;
      float2 sq[NP], sk[NP], dsq[NP], dsk[NP], gq[NP], gk[NP];
      float ssq = 0.f, ssk = 0.f, dotq = 0.f, dotk = 0.f;
#pragma unroll
      for (int j = 0; j < NP; ++j) {
        const int c = 2 * lane + 64 * j;
        sq[j] = sk[j] = dsq[j] = dsk[j] = gq[j] = gk[j] = make_float2(0.f, 0.f);
        if (c >= DK) continue;
        const long long o = orow + c;
        float2 cq = make_float2(0.f, 0.f), ck = cq, cv = cq;
        {
          const float4 wa = sw[c], wb = sw[c + 1], ka = sw[DK + c], kb = sw[DK + c + 1],
                       va = sw[2 * DK + c], vb = sw[2 * DK + c + 1];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            if (pos - 3 + i < 0) continue;
            const __nv_bfloat16* row = sraw + (r + i) * C3;
            const float2 xq = ld_bf2(row + c), xk = ld_bf2(row + DK + c), xv = ld_bf2(row + 2 * DK + c);
            cq.x += tap(wa, i) * xq.x;  cq.y += tap(wb, i) * xq.y;
            ck.x += tap(ka, i) * xk.x;  ck.y += tap(kb, i) * xk.y;
            cv.x += tap(va, i) * xv.x;  cv.y += tap(vb, i) * xv.y;
          }
        }
        cq = make_float2(rbf(cq.x), rbf(cq.y));
        ck = make_float2(rbf(ck.x), rbf(ck.y));
        cv = make_float2(rbf(cv.x), rbf(cv.y));
        // silu(x) = x s, silu'(x) = s (1 + x (1 - s)), s = sigmoid(x)
        {
          const float s0 = sigm(cq.x), s1 = sigm(cq.y);
          sq[j] = make_float2(cq.x * s0, cq.y * s1);
          dsq[j] = make_float2(s0 * (1.f + cq.x * (1.f - s0)), s1 * (1.f + cq.y * (1.f - s1)));
        }
        {
          const float s0 = sigm(ck.x), s1 = sigm(ck.y);
          sk[j] = make_float2(ck.x * s0, ck.y * s1);
          dsk[j] = make_float2(s0 * (1.f + ck.x * (1.f - s0)), s1 * (1.f + ck.y * (1.f - s1)));
        }
        ssq += sq[j].x * sq[j].x + sq[j].y * sq[j].y;
        ssk += sk[j].x * sk[j].x + sk[j].y * sk[j].y;
        gq[j] = *reinterpret_cast<const float2*>(dq + o);
        gk[j] = *reinterpret_cast<const float2*>(dk + o);
        dotq += gq[j].x * sq[j].x + gq[j].y * sq[j].y;
        dotk += gk[j].x * sk[j].x + gk[j].y * sk[j].y;
        {
          const float2 gv = *reinterpret_cast<const float2*>(dv + o);
          const float s0 = sigm(cv.x), s1 = sigm(cv.y);
          *reinterpret_cast<float2*>(drow + 2 * DK + c) =
              make_float2(gv.x * s0 * (1.f + cv.x * (1.f - s0)), gv.y * s1 * (1.f + cv.y * (1.f - s1)));
        }
        if (own) {
          const float2 fz = *reinterpret_cast<const float2*>(f + o);
          const float2 gg = *reinterpret_cast<const float2*>(dg + o);
          const float z[2] = {fz.x + dtb[j].x, fz.y + dtb[j].y}, dgv[2] = {gg.x, gg.y};
          float dz[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float sig = sigm(z[e]);
            if (gate_mode == 0) {
              dz[e] = dgv[e] * (-A) * sig;
              acc_al += dgv[e] * (-A * softplus_f(z[e]));
            } else {
              dz[e] = dgv[e] * (1.f - sig);
            }
          }
          *reinterpret_cast<__nv_bfloat162*>(df + o) = __floats2bfloat162_rn(dz[0], dz[1]);
          acc_dtb[j].x += dz[0];
          acc_dtb[j].y += dz[1];
        }
      }
      ssq = warp_sum(ssq);
      ssk = warp_sum(ssk);
      dotq = warp_sum(dotq);
      dotk = warp_sum(dotk);
      // y = x / n, n = sqrt(|x|^2 + eps): dx = (dy - y (dy . y)) / n
      const float iq = rsqrtf(ssq + 1e-6f), ik = rsqrtf(ssk + 1e-6f);
      const float cqf = dotq * iq * iq, ckf = dotk * ik * ik;
#pragma unroll
      for (int j = 0; j < NP; ++j) {
        const int c = 2 * lane + 64 * j;
        if (c >= DK) continue;
        *reinterpret_cast<float2*>(drow + c) =
            make_float2((gq[j].x - sq[j].x * cqf) * iq * dsq[j].x, (gq[j].y - sq[j].y * cqf) * iq * dsq[j].y);
        *reinterpret_cast<float2*>(drow + DK + c) =
            make_float2((gk[j].x - sk[j].x * ckf) * ik * dsk[j].x, (gk[j].y - sk[j].y * ckf) * ik * dsk[j].y);
      }
      if (own && lane == 0) {
        const float bt = beta[(long long)t * H + h];
        dbraw[(long long)t * H + h] = dbeta[(long long)t * H + h] * bt * (1.f - bt);
      }
    }
    __syncthreads();
    // ---- stage 2: thread per channel, sliding windows over the tile's rows
    const int rn = min(R, T - t0);
#pragma unroll
    for (int n = 0; n < P::NC; ++n) {
      const int c = tid + 256 * n;
      if (c >= C3) continue;
      const float4 wt = sw[c];
      const long long col = (c / DK) * HK + h * DK + c % DK;
      // d0..d3 = dconv rows r..r+3; x0..x3 = staged raw rows r..r+3 (tokens t-3..t)
      float d0 = sdc[c], d1 = sdc[C3 + c], d2 = sdc[2 * C3 + c], d3;
      float x0 = __bfloat162float(sraw[c]), x1 = __bfloat162float(sraw[C3 + c]),
            x2 = __bfloat162float(sraw[2 * C3 + c]), x3;
      int pos = pos0;
      for (int r = 0; r < rn; ++r) {
        d3 = sdc[(r + 3) * C3 + c];
        x3 = __bfloat162float(sraw[(r + 3) * C3 + c]);
        float acc = wt.w * d0;
        if (pos + 1 < S) acc += wt.z * d1;
        if (pos + 2 < S) acc += wt.y * d2;
        if (pos + 3 < S) acc += wt.x * d3;
        draw[(long long)(t0 + r) * ld_raw + col] = __float2bfloat16_rn(acc);
        dwacc[n][3] += d0 * x3;
        if (pos >= 1) dwacc[n][2] += d0 * x2;
        if (pos >= 2) dwacc[n][1] += d0 * x1;
        if (pos >= 3) dwacc[n][0] += d0 * x0;
        d0 = d1; d1 = d2; d2 = d3;
        x0 = x1; x1 = x2; x2 = x3;
        if (++pos == S) pos = 0;
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int n = 0; n < P::NC; ++n) {
    const int c = tid + 256 * n;
    if (c >= C3) continue;
    const int which = c / DK, cc = h * DK + c % DK;
    float* dw = which == 0 ? dwq : (which == 1 ? dwk : dwv);
#pragma unroll
    for (int i = 0; i < 4; ++i) atomicAdd(dw + cc * 4 + i, dwacc[n][i]);
  }
#pragma unroll
  for (int j = 0; j < NP; ++j) {
    const int c = 2 * lane + 64 * j;
    if (c < DK) {
      atomicAdd(s_dtb + c, acc_dtb[j].x);
      atomicAdd(s_dtb + c + 1, acc_dtb[j].y);
    }
  }
  if (gate_mode == 0) {
    acc_al = warp_sum(acc_al);
    if (lane == 0) atomicAdd(s_dtb + DK, acc_al);
  }
  __syncthreads();
  for (int i = tid; i < DK; i += blockDim.x)
    if (s_dtb[i] != 0.f) atomicAdd(d_dtb + h * DK + i, s_dtb[i]);
  if (tid == 0 && s_dtb[DK] != 0.f) atomicAdd(d_alog + h, s_dtb[DK]);
}

}  // namespace kda

using kda::Ptrs;

#define KDA_DISPATCH(DKV, ...)                     \
  if (DKV == 16) {                                 \
    constexpr int DK = 16;                         \
    constexpr int C = 32;                          \
    __VA_ARGS__                                    \
  } else if (DKV == 32) {                          \
    constexpr int DK = 32;                         \
    constexpr int C = 32;                          \
    __VA_ARGS__                                    \
  } else if (DKV == 64) {                          \
    constexpr int DK = 64;                         \
    constexpr int C = 32;                          \
    __VA_ARGS__                                    \
  } else if (DKV == 128) {                         \
    constexpr int DK = 128;                        \
    constexpr int C = 32;                          \
    __VA_ARGS__                                    \
  } else {                                         \
    HB_CHECK(false, "KDA head_dim must be 16, 32, 64 or 128"); \
  }

int64_t kda_chunk_size(int64_t dk) { return 32; }

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static void set_smem(const void* f, int bytes) {
  HB_CUDA_CHECK(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

// q,k,v,g: [B,S,H,K] fp32; beta [B,S,H]; outputs o [B,S,H,K];
// scratch: Wt,Ut,Kh,Qg [B,H,NC,C,K], Pm [B,H,NC,C,C], gC [B,H,NC,K], states [B,H,NC,K,K]
void kda_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g, torch::Tensor beta,
             double scale, torch::Tensor o, torch::Tensor Wt, torch::Tensor Ut, torch::Tensor Kh,
             torch::Tensor Qg, torch::Tensor Pm, torch::Tensor gC, torch::Tensor states,
             c10::optional<torch::Tensor> init_state, c10::optional<torch::Tensor> final_state) {
  Ptrs p{};
  p.B = q.size(0);
  p.S = q.size(1);
  p.H = q.size(2);
  const int DKV = q.size(3);
  p.q = q.data_ptr<float>();
  p.k = k.data_ptr<float>();
  p.v = v.data_ptr<float>();
  p.g = g.data_ptr<float>();
  p.beta = beta.data_ptr<float>();
  p.o = o.data_ptr<float>();
  p.Wt = Wt.data_ptr<float>();
  p.Ut = Ut.data_ptr<float>();
  p.Kh = Kh.data_ptr<float>();
  p.Qg = Qg.data_ptr<float>();
  p.Pm = Pm.data_ptr<float>();
  p.gC = gC.data_ptr<float>();
  p.states = states.data_ptr<float>();
  p.scale = (float)scale;
  p.init_state = init_state.has_value() ? init_state->data_ptr<float>() : nullptr;
  p.final_state = final_state.has_value() ? final_state->data_ptr<float>() : nullptr;
  HB_CHECK(al16(p.q) && al16(p.k) && al16(p.v) && al16(p.g) && al16(p.o) && al16(p.Wt) && al16(p.Ut) &&
               al16(p.Kh) && al16(p.Qg) && al16(p.Pm) && al16(p.states),
           "kda_fwd: 16-byte aligned buffers required");
  KDA_DISPATCH(DKV, {
    p.NC = (p.S + C - 1) / C;
    HB_CHECK(Pm.size(-1) == C, "kda_fwd: scratch chunk size mismatch");
    constexpr int VS = DK >= 32 ? 32 : DK;
    const int s1 = kda::intra_fwd_smem<DK, C>(), s2 = kda::state_fwd_smem<DK, C, VS>();
    static bool cfg = false;
    if (!cfg) {
      set_smem((const void*)kda::intra_fwd_kernel<DK, C>, s1);
      set_smem((const void*)kda::state_fwd_kernel<DK, C, VS>, s2);
      cfg = true;
    }
    kda::intra_fwd_kernel<DK, C><<<dim3(p.NC, p.H, p.B), kda::NT, s1, cur_stream()>>>(p);
    HB_CUDA_CHECK(cudaGetLastError());
    kda::state_fwd_kernel<DK, C, VS><<<dim3(DK / VS, p.H, p.B), kda::NT, s2, cur_stream()>>>(p);
    HB_CUDA_CHECK(cudaGetLastError());
  })
}

void kda_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g, torch::Tensor beta,
             double scale, torch::Tensor dout, torch::Tensor Wt, torch::Tensor Kh, torch::Tensor Qg,
             torch::Tensor Pm, torch::Tensor gC, torch::Tensor states, torch::Tensor dstates,
             torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor dg, torch::Tensor dbeta) {
  Ptrs p{};
  p.B = q.size(0);
  p.S = q.size(1);
  p.H = q.size(2);
  const int DKV = q.size(3);
  p.q = q.data_ptr<float>();
  p.k = k.data_ptr<float>();
  p.v = v.data_ptr<float>();
  p.g = g.data_ptr<float>();
  p.beta = beta.data_ptr<float>();
  p.dout = dout.data_ptr<float>();
  p.Wt = Wt.data_ptr<float>();
  p.Kh = Kh.data_ptr<float>();
  p.Qg = Qg.data_ptr<float>();
  p.Pm = Pm.data_ptr<float>();
  p.gC = gC.data_ptr<float>();
  p.states = states.data_ptr<float>();
  p.dstates = dstates.data_ptr<float>();
  p.dq = dq.data_ptr<float>();
  p.dk = dk.data_ptr<float>();
  p.dv = dv.data_ptr<float>();
  p.dg = dg.data_ptr<float>();
  p.dbeta = dbeta.data_ptr<float>();
  p.scale = (float)scale;
  HB_CHECK(dout.is_contiguous(), "kda_bwd: contiguous dout");
  HB_CHECK(al16(p.q) && al16(p.k) && al16(p.v) && al16(p.g) && al16(p.dout) && al16(p.states) &&
               al16(p.dstates) && al16(p.dq) && al16(p.dk) && al16(p.dv) && al16(p.dg),
           "kda_bwd: 16-byte aligned buffers required");
  KDA_DISPATCH(DKV, {
    p.NC = (p.S + C - 1) / C;
    constexpr int VS = DK >= 32 ? 32 : DK;
    const int s1 = kda::state_bwd_smem<DK, C, VS>(), s2 = kda::intra_bwd_smem<DK, C>();
    static bool cfg = false;
    if (!cfg) {
      set_smem((const void*)kda::state_bwd_kernel<DK, C, VS>, s1);
      set_smem((const void*)kda::intra_bwd_kernel<DK, C>, s2);
      cfg = true;
    }
    kda::state_bwd_kernel<DK, C, VS><<<dim3(DK / VS, p.H, p.B), kda::NT, s1, cur_stream()>>>(p);
    HB_CUDA_CHECK(cudaGetLastError());
    kda::intra_bwd_kernel<DK, C><<<dim3(p.NC, p.H, p.B), kda::NTB<DK>(), s2, cur_stream()>>>(p);
    HB_CUDA_CHECK(cudaGetLastError());
  })
}

void kda_prep_fwd(torch::Tensor raw, torch::Tensor wq, torch::Tensor wk, torch::Tensor wv, torch::Tensor f,
                  torch::Tensor a_log, torch::Tensor dt_bias, torch::Tensor braw, int64_t gate_mode,
                  int64_t S, torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g,
                  torch::Tensor beta) {
  const int T = q.size(0), H = q.size(1), DKV = q.size(2);
  HB_CHECK(raw.stride(0) % 2 == 0 && DKV % 2 == 0, "kda_prep: even row stride and head dim");
  // blocks: (token runs) x (heads), about 8 resident blocks per SM in all
  const int gx = (int)std::max<long long>(
      1, std::min<long long>(((long long)T + 7) / 8, ((long long)num_sms() * 8 + H - 1) / H));
  const dim3 grid(gx, H);
  auto launch = [&](auto dk) {
    constexpr int DK = decltype(dk)::value;
    kda::prep_fwd_kernel<DK><<<grid, 256, 0, cur_stream()>>>(
        (const __nv_bfloat16*)raw.data_ptr(), raw.stride(0), wq.data_ptr<float>(), wk.data_ptr<float>(),
        wv.data_ptr<float>(), f.data_ptr<float>(), a_log.data_ptr<float>(), dt_bias.data_ptr<float>(),
        braw.data_ptr<float>(), (int)gate_mode, T, (int)S, H, q.data_ptr<float>(), k.data_ptr<float>(),
        v.data_ptr<float>(), g.data_ptr<float>(), beta.data_ptr<float>());
  };
  if (DKV == 16) launch(std::integral_constant<int, 16>{});
  else if (DKV == 32) launch(std::integral_constant<int, 32>{});
  else if (DKV == 64) launch(std::integral_constant<int, 64>{});
  else if (DKV == 128) launch(std::integral_constant<int, 128>{});
  else HB_CHECK(false, "kda_prep: unsupported head dim");
  HB_CUDA_CHECK(cudaGetLastError());
}

void kda_prep_bwd(torch::Tensor raw, torch::Tensor wq, torch::Tensor wk, torch::Tensor wv, torch::Tensor f,
                  torch::Tensor a_log, torch::Tensor dt_bias, torch::Tensor beta, int64_t gate_mode,
                  int64_t S, torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor dg,
                  torch::Tensor dbeta, torch::Tensor df, torch::Tensor dbraw,
                  torch::Tensor d_alog, torch::Tensor d_dtb, torch::Tensor draw, torch::Tensor dwq,
                  torch::Tensor dwk, torch::Tensor dwv) {
  const int T = dq.size(0), H = dq.size(1), DKV = dq.size(2);
  HB_CHECK(raw.stride(0) % 2 == 0 && DKV % 2 == 0, "kda_prep: even row stride and head dim");
  HB_CHECK(df.scalar_type() == at::kBFloat16 && df.is_contiguous(), "kda_prep_bwd: df must be contiguous bf16");
  {
    HB_CHECK(raw.stride(0) % 8 == 0 && al16(raw.data_ptr()) && draw.stride(0) == raw.stride(0),
             "kda_prep_bwd: 16-byte aligned raw rows");
    auto launch = [&](auto dkc) {
      constexpr int DK = decltype(dkc)::value;
      using PT = kda::PrepTile<DK>;
      static bool cfg = false;
      if (!cfg) {
        set_smem((const void*)kda::prep_bwd_fused_kernel<DK>, PT::smem);
        cfg = true;
      }
      int per_sm = 0;
      HB_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
          &per_sm, kda::prep_bwd_fused_kernel<DK>, 256, PT::smem));
      const int ntiles = (T + PT::R - 1) / PT::R;
      const int gx = (int)std::max<long long>(
          1, std::min<long long>(ntiles, ((long long)num_sms() * std::max(per_sm, 1) + H - 1) / H));
      kda::prep_bwd_fused_kernel<DK><<<dim3(gx, H), 256, PT::smem, cur_stream()>>>(
          (const __nv_bfloat16*)raw.data_ptr(), raw.stride(0), wq.data_ptr<float>(), wk.data_ptr<float>(),
          wv.data_ptr<float>(), f.data_ptr<float>(), a_log.data_ptr<float>(), dt_bias.data_ptr<float>(),
          beta.data_ptr<float>(), (int)gate_mode, T, (int)S, H, dq.data_ptr<float>(), dk.data_ptr<float>(),
          dv.data_ptr<float>(), dg.data_ptr<float>(), dbeta.data_ptr<float>(), (__nv_bfloat16*)df.data_ptr(),
          dbraw.data_ptr<float>(), d_alog.data_ptr<float>(), d_dtb.data_ptr<float>(),
          (__nv_bfloat16*)draw.data_ptr(), dwq.data_ptr<float>(), dwk.data_ptr<float>(), dwv.data_ptr<float>());
    };
    if (DKV == 16) launch(std::integral_constant<int, 16>{});
    else if (DKV == 32) launch(std::integral_constant<int, 32>{});
    else if (DKV == 64) launch(std::integral_constant<int, 64>{});
    else if (DKV == 128) launch(std::integral_constant<int, 128>{});
    else HB_CHECK(false, "kda_prep: unsupported head dim");
    HB_CUDA_CHECK(cudaGetLastError());
  }
}

}  // namespace hb

// ============================================================================
// Allocation-free entry point (declared in kda_noalloc.h).
//
// For callers that cannot allocate device memory themselves: code running
// inside a CUDA-graph capture that must not see a cudaMalloc, host runtimes
// with their own fixed memory pools, and plugins loaded into a process whose
// allocator they do not own.  The chunk intermediates live in the file-scope
// array below, 64 MiB on every GPU that loads this library, held until the
// process exits.  The host side cannot use the array's name as a device
// address (there it is only a host-side stand-in); the device address is
// obtained once per device with cudaGetSymbolAddress, with that device
// current, the first time the entry point is called on it.
// ============================================================================
namespace hb {
namespace kda_noalloc {

constexpr long long kScratchFloats = 16LL * 1024 * 1024;  // 64 MiB of fp32
__device__ __align__(256) float g_scratch[kScratchFloats];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
float* g_dev_ptr[kMaxDevices] = {nullptr};
CUcontext g_dev_ctx[kMaxDevices] = {nullptr};  // context the cached address belongs to

// cuCtxGetCurrent through the runtime's driver entry point, so the library
// does not link libcuda directly (it must import on machines without a GPU).
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
bool current_context(CUcontext* ctx) {
  static CtxGetCurrentFn fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || f == nullptr)
      return false;
    fn = reinterpret_cast<CtxGetCurrentFn>(f);
  }
  return fn(ctx) == CUDA_SUCCESS;
}

// Scratch floats needed for [B, S, H, DK] inputs (chunk size 32).
long long scratch_floats(int B, int S, int H, int DK) {
  const long long C = 32;
  const long long NC = (S + C - 1) / C;
  const long long bhn = (long long)B * H * NC;
  return bhn * (4 * C * DK + C * C + DK + (long long)DK * DK);
}

}  // namespace kda_noalloc
}  // namespace hb

#include "kda_noalloc.h"

extern "C" __attribute__((visibility("default"))) int hb_kda_fwd_noalloc(
    const float* q, const float* k, const float* v, const float* g, const float* beta, float* o,
    int B, int S, int H, int DK, float scale, cudaStream_t stream) {
  using namespace hb;
  using namespace hb::kda_noalloc;
  if (!(DK == 16 || DK == 32 || DK == 64)) return HB_NOALLOC_BAD_HEAD_DIM;
  if (B <= 0 || S <= 0 || H <= 0) return HB_NOALLOC_BAD_SHAPE;
  for (const void* ptr : {(const void*)q, (const void*)k, (const void*)v, (const void*)g, (const void*)o})
    if (reinterpret_cast<uintptr_t>(ptr) & 15) return HB_NOALLOC_BAD_SHAPE;
  if (scratch_floats(B, S, H, DK) > kScratchFloats) return HB_NOALLOC_TOO_LARGE;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return HB_NOALLOC_CUDA_ERROR;
  float* base = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    CUcontext ctx = nullptr;
    if (!current_context(&ctx)) return HB_NOALLOC_CUDA_ERROR;
    if (!g_dev_ptr[dev] || g_dev_ctx[dev] != ctx) {  // first call, or the context was rebuilt
      void* ptr = nullptr;
      if (cudaGetSymbolAddress(&ptr, g_scratch) != cudaSuccess || ptr == nullptr)
        return HB_NOALLOC_CUDA_ERROR;
      if (!current_context(&ctx)) return HB_NOALLOC_CUDA_ERROR;
      g_dev_ptr[dev] = static_cast<float*>(ptr);
      g_dev_ctx[dev] = ctx;
    }
    base = g_dev_ptr[dev];
  }
  Ptrs p{};
  p.B = B;
  p.S = S;
  p.H = H;
  p.q = q;
  p.k = k;
  p.v = v;
  p.g = g;
  p.beta = beta;
  p.o = o;
  p.scale = scale;
  const long long C = 32;
  const long long NC = (S + C - 1) / C;
  p.NC = (int)NC;
  const long long bhn = (long long)B * H * NC;
  // carve the scratch: every region is written before it is read, so nothing
  // has to be cleared between calls
  float* cur = base;
  p.Wt = cur; cur += bhn * C * DK;
  p.Ut = cur; cur += bhn * C * DK;
  p.Kh = cur; cur += bhn * C * DK;
  p.Qg = cur; cur += bhn * C * DK;
  p.Pm = cur; cur += bhn * C * C;
  p.gC = cur; cur += bhn * DK;
  p.states = cur;
  p.init_state = nullptr;
  p.final_state = nullptr;
  auto run = [&](auto dkc) -> int {
    constexpr int DKc = decltype(dkc)::value;
    constexpr int Cc = 32;
    constexpr int VS = DKc >= 32 ? 32 : DKc;
    const int s1 = kda::intra_fwd_smem<DKc, Cc>(), s2 = kda::state_fwd_smem<DKc, Cc, VS>();
    if (cudaFuncSetAttribute((const void*)kda::intra_fwd_kernel<DKc, Cc>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, s1) != cudaSuccess ||
        cudaFuncSetAttribute((const void*)kda::state_fwd_kernel<DKc, Cc, VS>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, s2) != cudaSuccess)
      return HB_NOALLOC_CUDA_ERROR;
    kda::intra_fwd_kernel<DKc, Cc><<<dim3(p.NC, p.H, p.B), kda::NT, s1, stream>>>(p);
    if (cudaGetLastError() != cudaSuccess) return HB_NOALLOC_CUDA_ERROR;
    kda::state_fwd_kernel<DKc, Cc, VS><<<dim3(DKc / VS, p.H, p.B), kda::NT, s2, stream>>>(p);
    if (cudaGetLastError() != cudaSuccess) return HB_NOALLOC_CUDA_ERROR;
    return HB_NOALLOC_OK;
  };
  if (DK == 16) return run(std::integral_constant<int, 16>{});
  if (DK == 32) return run(std::integral_constant<int, 32>{});
  return run(std::integral_constant<int, 64>{});
}
