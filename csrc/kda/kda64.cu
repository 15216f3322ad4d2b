// Kimi Delta Attention, chunk 64 with 16-row sub-blocks (head dim 64).
//
// Same recurrence and chunk form as kda.cu (model/kda.py:305-323); what
// changes is how the decay-weighted pair products are evaluated and what the
// forward keeps for the backward.
//
// Pair products with per-channel decays.  For rows t of a later sub-block than
// the column block j (s in [16j, 16j+16), e = 16j + 15 its last row):
//   e^{G_t - G_s} = e^{G_t - G_e} e^{G_e - G_s},  both factors <= 1,
// so   A[t, blk j] = (K_t e^{G_t-G_e}) (K_blk e^{G_e-G_blk})^T   is a plain
// matmul, and so are P and every backward contraction through the decays
// (dq / dk "t-side" from dP and dA, and the "s-side" sums over later rows).
// Only the four 16x16 diagonal blocks are evaluated pair by pair.  No factor
// exceeds 1, so strongly negative decays underflow to 0 instead of overflowing.
//
// The forward stores Linv = (I + diag(b^2) A)^{-1} and A besides Wt, Ut, Kh,
// Qg, P, gC: the backward then needs no triangular solve (X = Linv^T dU is a
// matmul) and no recomputed pair products.
//
// The two sequential recurrences carry only what the chunk-to-chunk dependency
// needs (forward: U = Ut - Wt S, S <- gC S + Kh^T U; backward: dU = P^T dO +
// Kh dS, dS <- gC dS + Qg^T dO - Wt^T dU with both dO products precomputed),
// so four CTAs fit on an SM and every (batch, head, value slice) is resident
// at once; everything else runs chunk-parallel.
//
// Kernels (grid (NC, H, B) unless noted):
//   intra_fwd64_kernel        A, P, Linv, Ut, Wt, Kh, Qg, gC per chunk
//   state_fwd64_kernel        grid (64 / VS, H, B): S per chunk (states) and U
//   out64_kernel              O = Qg S0 + P U
//   bwd_pre64_kernel          P^T dO and Qg^T dO
//   state_bwd64_kernel        grid (64 / VS, H, B): dS per chunk (dstates) and dU
//   state_products64_kernel   dQg, dKh, dWt, dP, dgC (the S0 / dS products)
// The S0 / dS state products also have a tcgen05 version (kda64_tc.cu).
//   intra_bwd64_kernel        X, Y, dN, dbeta, dv and the decay contractions
// All products are 3xTF32 warp-tile matmuls (fp32-level accuracy).
#include <torch/extension.h>

#include "../common/host.h"
#include "kda_common.cuh"

namespace hb {
namespace kda64 {
using namespace hb::kda;

constexpr int C = 64;         // chunk
constexpr int D = 64;         // head dim (key = value)
constexpr int BS = 16;        // sub-block rows
constexpr int NB = C / BS;
constexpr int L = D + 4;      // smem row stride of every [64, 64] tile (4 mod 32)
constexpr int TILE = C * L;   // floats
constexpr int NTF = 512;      // threads of the intra kernels
constexpr int NTP = 256;      // threads of the state-product kernel
static_assert(C == D, "the C x C and C x D tiles share one layout");

// Off-diagonal column blocks j = 0, 1, 2: rows after block j and their offsets
// in the forward's staging area.
HB_DEVICE constexpr int rows_after(int j) { return C - BS * (j + 1); }  // 48, 32, 16
HB_DEVICE constexpr int stage_off(int j) { return j == 0 ? 0 : j == 1 ? 48 : 80; }

// [64, 64] tile of a chunk-layout tensor (row stride 64) -> smem (cp.async)
HB_DEVICE void cp_chunk_tile(float* s, const float* g) { cp_tile<C, D>(s, L, g, D); }

// Chunk n's rows of a token-layout [B, S, H, D] tensor (zeros past S), cp.async.
HB_DEVICE void cp_token_rows(const Ptrs& p, const float* x, int b, int h, int n, float* dst) {
  for (int i = threadIdx.x; i < C * (D / 4); i += blockDim.x) {
    const int r = i / (D / 4), c = (i % (D / 4)) * 4;
    const int t = n * C + r;
    const bool ok = t < p.S;
    cp_async16(dst + r * L + c, ok ? x + tok_off(p, b, t, h, D) + c : x, ok);
  }
}

HB_DEVICE void load_beta(const Ptrs& p, int b, int h, int n, float* bet) {
  for (int r = threadIdx.x; r < C; r += blockDim.x) {
    const int t = n * C + r;
    bet[r] = t < p.S ? p.beta[((long long)b * p.S + t) * p.H + h] : 0.f;
  }
}

// g -> G = cumsum(g) log2(e) in place (the chunk kernels evaluate every decay
// as one ex2.approx of a difference of these base-2 log decays).
HB_DEVICE void cumsum_log2(float* G) {
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float acc = 0.f;
#pragma unroll 16
    for (int r = 0; r < C; ++r) {
      acc += G[r * L + c];
      G[r * L + c] = acc * kLog2e;
    }
  }
}

// Phase timing of the intra kernels, off unless a counter array is set
// (kda64_set_profile): thread 0 of every CTA adds the cycles since its previous
// mark to slot i, so each slot sums one phase over all CTAs.
HB_DEVICE long long cycle_count() {
  long long c;
  asm volatile("mov.u64 %0, %%clock64;" : "=l"(c));
  return c;
}
struct PhaseClock {
  unsigned long long* prof;
  long long t;
  HB_DEVICE explicit PhaseClock(unsigned long long* p) : prof(p), t(cycle_count()) {}
  HB_DEVICE void mark(int i) {
    if (prof && threadIdx.x == 0) {
      const long long now = cycle_count();
      atomicAdd(prof + i, (unsigned long long)(now - t));
      t = now;
    }
  }
};

// (t, s) of pair r of a 16x16 lower triangle with the diagonal (r < 136)
HB_DEVICE void tri_pair(int r, int& t, int& s) {
  int tt = (int)((sqrtf(8.f * r + 1.f) - 1.f) * 0.5f);
  while ((tt + 1) * (tt + 2) / 2 <= r) ++tt;
  while (tt * (tt + 1) / 2 > r) --tt;
  t = tt;
  s = r - tt * (tt + 1) / 2;
}

// Linv = (I + N)^{-1} for N strictly lower [64, 64] (row stride L), by 16-row
// blocks: the diagonal blocks D_i by column substitution (one thread per
// column), then the block rows at distance d = 1, 2, 3 from the diagonal,
//   Linv_ij = -D_i sum_{k=j}^{i-1} N_ik Linv_kj,
// each level a pair of small products over all threads.  T: 768 floats.
HB_DEVICE void block_inverse(const float* N, float* Li, float* T) {
  for (int i = threadIdx.x; i < C * C; i += blockDim.x) {
    const int r = i / C, c = i % C;
    if ((c >> 4) > (r >> 4)) Li[r * L + c] = 0.f;
  }
  if (threadIdx.x < C) {
    const int base = (threadIdx.x >> 4) * BS, col = threadIdx.x & (BS - 1);
    float x[BS];
#pragma unroll
    for (int t = 0; t < BS; ++t) x[t] = t == col ? 1.f : 0.f;
#pragma unroll
    for (int q = 0; q < BS - 1; ++q) {
#pragma unroll
      for (int t = q + 1; t < BS; ++t) x[t] = fmaf(-N[(base + t) * L + base + q], x[q], x[t]);
    }
#pragma unroll
    for (int t = 0; t < BS; ++t) Li[(base + t) * L + base + col] = x[t];
  }
  __syncthreads();
  for (int d = 1; d < NB; ++d) {
    const int nb = NB - d;
    for (int e = threadIdx.x; e < nb * BS * BS; e += blockDim.x) {
      const int bi = e / (BS * BS), r = (e / BS) % BS, c = e % BS;
      const int i = d + bi, j = i - d;
      const float* nrow = N + (i * BS + r) * L;
      float acc = 0.f;
      for (int kk = j * BS; kk < i * BS; ++kk) acc = fmaf(nrow[kk], Li[kk * L + j * BS + c], acc);
      T[e] = acc;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < nb * BS * BS; e += blockDim.x) {
      const int bi = e / (BS * BS), r = (e / BS) % BS, c = e % BS;
      const int i = d + bi, j = i - d;
      const float* drow = Li + (i * BS + r) * L + i * BS;
      float acc = 0.f;
      for (int kk = 0; kk <= r; ++kk) acc = fmaf(drow[kk], T[bi * BS * BS + kk * BS + c], acc);
      Li[(i * BS + r) * L + j * BS + c] = -acc;
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------ forward
// Six [64, 64] tiles (q, k, G, A, P, staging) and beta: 104 KB, two CTAs of
// 256 threads per SM.  The staging tile holds, per off-diagonal column block j,
// Zr_j (16 rows) and then Zk_j or Zq_j (up to 48 rows), later Linv; the P tile
// holds the block inversion's scratch and then b V once P is stored.
constexpr int NTFW = 256;
constexpr int fwd_smem() { return (6 * TILE + C) * 4; }

__global__ void __launch_bounds__(NTFW, 2) intra_fwd64_kernel(Ptrs p) {
  extern __shared__ float sm[];
  float* q = sm;           // q, later b^2 K e^G
  float* k = q + TILE;
  float* G = k + TILE;
  float* A = G + TILE;     // A, then N = diag(b^2) A
  float* P = A + TILE;     // P, then inversion scratch, then b V
  float* Z = P + TILE;     // staging, then Linv
  float* bet = Z + TILE;
  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const float scale = p.scale;
  PhaseClock pc(p.prof);
  cp_token_rows(p, p.q, b, h, n, q);
  cp_token_rows(p, p.k, b, h, n, k);
  cp_token_rows(p, p.g, b, h, n, G);
  cp_async_commit();
  load_beta(p, b, h, n, bet);
  for (int i = threadIdx.x; i < 2 * TILE; i += blockDim.x) A[i] = 0.f;  // A and P
  cp_async_wait_all();
  __syncthreads();
  pc.mark(0);
  cumsum_log2(G);
  __syncthreads();
  pc.mark(1);
  const long long co = chunk_off(p, b, h, n, C * D);
  const float* GC = G + (C - 1) * L;
  // Kh = K e^{G_C - G},  Qg = scale Q e^G,  gC = e^{G_C}
  for (int i = threadIdx.x; i < C * D / 4; i += blockDim.x) {
    const int r = i / (D / 4), c = (i % (D / 4)) * 4;
    const int si = r * L + c;
    const float4 kk = ld4(k + si), gg = ld4(G + si), qq = ld4(q + si), gc = ld4(GC + c);
    st4(p.Kh + co + r * D + c, make_float4(kk.x * exp2_fast(gc.x - gg.x), kk.y * exp2_fast(gc.y - gg.y),
                                           kk.z * exp2_fast(gc.z - gg.z), kk.w * exp2_fast(gc.w - gg.w)));
    st4(p.Qg + co + r * D + c, make_float4(scale * qq.x * exp2_fast(gg.x), scale * qq.y * exp2_fast(gg.y),
                                           scale * qq.z * exp2_fast(gg.z), scale * qq.w * exp2_fast(gg.w)));
  }
  if (threadIdx.x < D) p.gC[chunk_off(p, b, h, n, D) + threadIdx.x] = exp2_fast(GC[threadIdx.x]);
  // off-diagonal column blocks: A[t > e, blk j] = Zk_j Zr_j^T,  P = scale Zq_j Zr_j^T
  float* Zr = Z;
  float* Zt = Z + BS * L;
  auto offdiag = [&](auto jc) {
    constexpr int j = decltype(jc)::value;
    constexpr int r0 = BS * (j + 1), M = C - r0, e = BS * j + BS - 1;
    // (a barrier separates this from the previous round's readers of Z)
    for (int i = threadIdx.x; i < BS * D / 4; i += blockDim.x) {
      const int s4 = i / (D / 4), c = (i % (D / 4)) * 4;
      const int si = (BS * j + s4) * L + c;
      const float4 kk = ld4(k + si), gs = ld4(G + si), ge = ld4(G + e * L + c);
      st4(Zr + s4 * L + c, make_float4(kk.x * exp2_fast(ge.x - gs.x), kk.y * exp2_fast(ge.y - gs.y),
                                       kk.z * exp2_fast(ge.z - gs.z), kk.w * exp2_fast(ge.w - gs.w)));
    }
    auto stage_rows = [&](const float* src) {
      for (int i = threadIdx.x; i < M * D / 4; i += blockDim.x) {
        const int tt = i / (D / 4), c = (i % (D / 4)) * 4;
        const int si = (r0 + tt) * L + c;
        const float4 x = ld4(src + si), gt = ld4(G + si), ge = ld4(G + e * L + c);
        st4(Zt + tt * L + c, make_float4(x.x * exp2_fast(gt.x - ge.x), x.y * exp2_fast(gt.y - ge.y),
                                         x.z * exp2_fast(gt.z - ge.z), x.w * exp2_fast(gt.w - ge.w)));
      }
    };
    stage_rows(k);
    __syncthreads();
    mm<M, BS, D, false, true>(A + r0 * L + BS * j, L, Zt, L, Zr, L, 1.f, false);
    __syncthreads();
    stage_rows(q);
    __syncthreads();
    mm<M, BS, D, false, true>(P + r0 * L + BS * j, L, Zt, L, Zr, L, scale, false);
    __syncthreads();
  };
  offdiag(std::integral_constant<int, 0>{});
  offdiag(std::integral_constant<int, 1>{});
  offdiag(std::integral_constant<int, 2>{});
  pc.mark(2);
  // diagonal blocks pair by pair (s <= t inside a sub-block)
  for (int pi = threadIdx.x; pi < NB * 136; pi += blockDim.x) {
    const int blk = pi / 136;
    int tt, ss;
    tri_pair(pi % 136, tt, ss);
    const int t = blk * BS + tt, s = blk * BS + ss;
    float a = 0.f, pp = 0.f;
#pragma unroll 4
    for (int c = 0; c < D; c += 4) {
      const float4 kt = ld4(k + t * L + c), ks = ld4(k + s * L + c), qt = ld4(q + t * L + c);
      const float4 gt = ld4(G + t * L + c), gs = ld4(G + s * L + c);
      const float e0 = exp2_fast(gt.x - gs.x) * ks.x, e1 = exp2_fast(gt.y - gs.y) * ks.y;
      const float e2 = exp2_fast(gt.z - gs.z) * ks.z, e3 = exp2_fast(gt.w - gs.w) * ks.w;
      a += kt.x * e0 + kt.y * e1 + kt.z * e2 + kt.w * e3;
      pp += qt.x * e0 + qt.y * e1 + qt.z * e2 + qt.w * e3;
    }
    A[t * L + s] = s < t ? a : 0.f;
    P[t * L + s] = scale * pp;
  }
  __syncthreads();
  pc.mark(3);
  // store P and A; N = diag(b^2) A in place
  const long long po = chunk_off(p, b, h, n, C * C);
  for (int i = threadIdx.x; i < C * C / 4; i += blockDim.x) {
    const int r = i / (C / 4), c = (i % (C / 4)) * 4;
    st4(p.Pm + po + r * C + c, ld4(P + r * L + c));
    const float4 a = ld4(A + r * L + c);
    st4(p.Am + po + r * C + c, a);
    const float b2 = bet[r] * bet[r];
    st4(A + r * L + c, make_float4(b2 * a.x, b2 * a.y, b2 * a.z, b2 * a.w));
  }
  __syncthreads();
  pc.mark(4);
  // Linv = (I + N)^{-1} into the staging tile (scratch in the P tile)
  float* Li = Z;
  block_inverse(A, Li, P);
  pc.mark(5);
  // v rows into the P tile; store Linv; b V (in P) and b^2 K e^G (in q)
  cp_token_rows(p, p.v, b, h, n, P);
  cp_async_commit();
  for (int i = threadIdx.x; i < C * C / 4; i += blockDim.x) {
    const int r = i / (C / 4), c = (i % (C / 4)) * 4;
    st4(p.Linv + po + r * C + c, ld4(Li + r * L + c));
  }
  for (int i = threadIdx.x; i < C * D / 4; i += blockDim.x) {
    const int r = i / (D / 4), c = (i % (D / 4)) * 4;
    const int si = r * L + c;
    const float b2 = bet[r] * bet[r];
    const float4 kk = ld4(k + si), gg = ld4(G + si);
    st4(q + si, make_float4(b2 * kk.x * exp2_fast(gg.x), b2 * kk.y * exp2_fast(gg.y),
                            b2 * kk.z * exp2_fast(gg.z), b2 * kk.w * exp2_fast(gg.w)));
  }
  cp_async_wait_all();
  __syncthreads();
  for (int i = threadIdx.x; i < C * D / 4; i += blockDim.x) {
    const int r = i / (D / 4), c = (i % (D / 4)) * 4;
    const float bt = bet[r];
    const float4 vv = ld4(P + r * L + c);
    st4(P + r * L + c, make_float4(bt * vv.x, bt * vv.y, bt * vv.z, bt * vv.w));
  }
  __syncthreads();
  pc.mark(6);
  // Ut = Linv b V,  Wt = Linv b^2 K e^G  (written straight to global)
  mm<C, D, C, false, false>(p.Ut + co, D, Li, L, P, L, 1.f, false);
  mm<C, D, C, false, false>(p.Wt + co, D, Li, L, q, L, 1.f, false);
  pc.mark(7);
}

// ------------------------------------------------------ state recurrences
// Value-column slice of the recurrences and its smem row stride.
constexpr int VS = 16;
constexpr int LV = VS + 4;

// Forward, one CTA per (value slice, head, batch), chunks in order:
//   states[n] = S;  U = Ut - Wt S (saved);  S <- gC * S + Kh^T U.
// Wt / Ut (first product) and Kh (second) have one buffer each; the next
// chunk's Wt / Ut are fetched while Kh^T U runs, its Kh after that.
constexpr int state_fwd64_smem() { return (D * LV + C * LV + 2 * C * L + D) * 4; }

__global__ void __launch_bounds__(256, 4) state_fwd64_kernel(Ptrs p) {
  extern __shared__ float sm[];
  float* S = sm;              // D x LV
  float* U = S + D * LV;      // C x LV (Ut slice, then U)
  float* Wt = U + C * LV;     // C x L
  float* Kh = Wt + C * L;     // C x L
  float* gc = Kh + C * L;     // D
  const int vs = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int v0 = vs * VS;
  // Wt of chunk n+1 is fetched as soon as U = Ut - Wt S of chunk n is done,
  // so that copy overlaps the rest of the step; Ut, gC and Kh after the step.
  auto fetch_w = [&](int n) { cp_tile<C, D>(Wt, L, p.Wt + chunk_off(p, b, h, n, C * D), D); };
  auto fetch_uk = [&](int n) {
    const long long co = chunk_off(p, b, h, n, C * D);
    cp_tile<C, VS>(U, LV, p.Ut + co + v0, D);
    cp_tile<1, D>(gc, D, p.gC + chunk_off(p, b, h, n, D), D);
    cp_tile<C, D>(Kh, L, p.Kh + co, D);
  };
  for (int i = threadIdx.x; i < D * VS; i += blockDim.x) {
    const int r = i / VS, c = i % VS;
    S[r * LV + c] = p.init_state ? p.init_state[((long long)b * p.H + h) * D * D + r * D + v0 + c] : 0.f;
  }
  fetch_w(0);
  fetch_uk(0);
  cp_async_commit();
  for (int n = 0; n < p.NC; ++n) {
    cp_async_wait_all();
    __syncthreads();
    const long long so = chunk_off(p, b, h, n, D * D), co = chunk_off(p, b, h, n, C * D);
    for (int i = threadIdx.x; i < D * VS / 4; i += blockDim.x) {
      const int r = i / (VS / 4), c = (i % (VS / 4)) * 4;
      st4(p.states + so + r * D + v0 + c, ld4(S + r * LV + c));
    }
    mm<C, VS, D, false, false>(U, LV, Wt, L, S, LV, -1.f, true);   // U = Ut - Wt S
    __syncthreads();
    if (n + 1 < p.NC) {
      fetch_w(n + 1);
      cp_async_commit();
    }
    for (int i = threadIdx.x; i < C * VS / 4; i += blockDim.x) {
      const int r = i / (VS / 4), c = (i % (VS / 4)) * 4;
      st4(p.Usv + co + r * D + v0 + c, ld4(U + r * LV + c));
    }
    for (int e = threadIdx.x; e < D * VS; e += blockDim.x) S[(e / VS) * LV + e % VS] *= gc[e / VS];
    __syncthreads();
    mm<D, VS, C, true, false>(S, LV, Kh, L, U, LV, 1.f, true);      // S += Kh^T U
    __syncthreads();
    if (n + 1 < p.NC) {
      fetch_uk(n + 1);
      cp_async_commit();
    }
  }
  __syncthreads();
  if (p.final_state)
    for (int i = threadIdx.x; i < D * VS; i += blockDim.x) {
      const int r = i / VS, c = i % VS;
      p.final_state[((long long)b * p.H + h) * D * D + r * D + v0 + c] = S[r * LV + c];
    }
}

// O = Qg S0 + P U, chunk-parallel; rows past S are not stored.
constexpr int out64_smem() { return 5 * TILE * 4; }

__global__ void __launch_bounds__(256, 2) out64_kernel(Ptrs p) {
  extern __shared__ float sm[];
  float* S0 = sm;
  float* Qg = S0 + TILE;
  float* P = Qg + TILE;
  float* U = P + TILE;
  float* O = U + TILE;
  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const long long co = chunk_off(p, b, h, n, C * D);
  cp_chunk_tile(S0, p.states + chunk_off(p, b, h, n, D * D));
  cp_chunk_tile(Qg, p.Qg + co);
  cp_chunk_tile(P, p.Pm + chunk_off(p, b, h, n, C * C));
  cp_chunk_tile(U, p.Usv + co);
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();
  mm<C, D, D, false, false>(O, L, Qg, L, S0, L, 1.f, false);
  mm<C, D, C, false, false>(O, L, P, L, U, L, 1.f, true);   // same warp tiles: no barrier
  __syncthreads();
  for (int i = threadIdx.x; i < C * D / 4; i += blockDim.x) {
    const int r = i / (D / 4), c = (i % (D / 4)) * 4;
    const int t = n * C + r;
    if (t < p.S) st4(p.o + tok_off(p, b, t, h, D) + c, ld4(O + r * L + c));
  }
}

// dUp = P^T dO,  dSq = Qg^T dO  (state-independent halves of the backward recurrence)
constexpr int bwd_pre64_smem() { return 3 * TILE * 4; }

__global__ void __launch_bounds__(256, 3) bwd_pre64_kernel(Ptrs p) {
  extern __shared__ float sm[];
  float* P = sm;
  float* Qg = P + TILE;
  float* dO = Qg + TILE;
  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const long long co = chunk_off(p, b, h, n, C * D);
  cp_chunk_tile(P, p.Pm + chunk_off(p, b, h, n, C * C));
  cp_chunk_tile(Qg, p.Qg + co);
  cp_token_rows(p, p.dout, b, h, n, dO);
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();
  mm<C, D, C, true, false>(p.dUp + co, D, P, L, dO, L, 1.f, false);
  mm<D, D, C, true, false>(p.dSq + chunk_off(p, b, h, n, D * D), D, Qg, L, dO, L, 1.f, false);
}

// Backward, one CTA per (value slice, head, batch), chunks in reverse:
//   dstates[n] = dS;  dU = dUp + Kh dS (exported);  dS <- gC * dS + dSq - Wt^T dU.
constexpr int state_bwd64_smem() { return (2 * D * LV + C * LV + 2 * C * L + D) * 4; }

__global__ void __launch_bounds__(256, 4) state_bwd64_kernel(Ptrs p) {
  extern __shared__ float sm[];
  float* dS = sm;             // D x LV
  float* dU = dS + D * LV;    // C x LV (dUp slice, then dU)
  float* Sq = dU + C * LV;    // D x LV (dSq slice)
  float* Kh = Sq + D * LV;    // C x L
  float* Wt = Kh + C * L;     // C x L
  float* gc = Wt + C * L;     // D
  const int vs = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int v0 = vs * VS;
  // Kh of chunk n-1 is fetched as soon as dU = dUp + Kh dS of chunk n is
  // done, so that copy overlaps the rest of the step; the others after it.
  auto fetch_k = [&](int n) { cp_tile<C, D>(Kh, L, p.Kh + chunk_off(p, b, h, n, C * D), D); };
  auto fetch_rest = [&](int n) {
    const long long co = chunk_off(p, b, h, n, C * D);
    cp_tile<C, VS>(dU, LV, p.dUp + co + v0, D);
    cp_tile<D, VS>(Sq, LV, p.dSq + chunk_off(p, b, h, n, D * D) + v0, D);
    cp_tile<C, D>(Wt, L, p.Wt + co, D);
    cp_tile<1, D>(gc, D, p.gC + chunk_off(p, b, h, n, D), D);
  };
  for (int i = threadIdx.x; i < D * LV; i += blockDim.x) dS[i] = 0.f;
  fetch_k(p.NC - 1);
  fetch_rest(p.NC - 1);
  cp_async_commit();
  for (int n = p.NC - 1; n >= 0; --n) {
    cp_async_wait_all();
    __syncthreads();
    const long long so = chunk_off(p, b, h, n, D * D), co = chunk_off(p, b, h, n, C * D);
    for (int i = threadIdx.x; i < D * VS / 4; i += blockDim.x) {
      const int r = i / (VS / 4), c = (i % (VS / 4)) * 4;
      st4(p.dstates + so + r * D + v0 + c, ld4(dS + r * LV + c));
    }
    mm<C, VS, D, false, false>(dU, LV, Kh, L, dS, LV, 1.f, true);   // dU = dUp + Kh dS
    __syncthreads();
    if (n > 0) {
      fetch_k(n - 1);
      cp_async_commit();
    }
    for (int i = threadIdx.x; i < C * VS / 4; i += blockDim.x) {
      const int r = i / (VS / 4), c = (i % (VS / 4)) * 4;
      st4(p.dU + co + r * D + v0 + c, ld4(dU + r * LV + c));
    }
    for (int e = threadIdx.x; e < D * VS; e += blockDim.x) {
      const int si = (e / VS) * LV + e % VS;
      dS[si] = gc[e / VS] * dS[si] + Sq[si];
    }
    __syncthreads();
    mm<D, VS, C, true, false>(dS, LV, Wt, L, dU, LV, -1.f, true);  // dS -= Wt^T dU
    __syncthreads();
    if (n > 0) {
      fetch_rest(n - 1);
      cp_async_commit();
    }
  }
}

// ----------------------------------------------------------- state products
// dQg = dO S0^T;  dWt = -dU S0^T;  dKh = U dS^T;  dP = dO U^T (unmasked, masked
// by the consumer);  dgC = rowsum(dS * S0).  U is the forward's saved U.
constexpr int prod_smem() { return 5 * TILE * 4; }

__global__ void __launch_bounds__(NTP, 2) state_products64_kernel(Ptrs p) {
  extern __shared__ float sm[];
  float* S0 = sm;
  float* dS = S0 + TILE;
  float* dO = dS + TILE;
  float* U = dO + TILE;
  float* dU = U + TILE;
  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const long long co = chunk_off(p, b, h, n, C * D), so = chunk_off(p, b, h, n, D * D);
  cp_chunk_tile(S0, p.states + so);
  cp_chunk_tile(dS, p.dstates + so);
  cp_token_rows(p, p.dout, b, h, n, dO);
  cp_chunk_tile(U, p.Usv + co);
  cp_chunk_tile(dU, p.dU + co);
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();
  mm<C, D, D, false, true>(p.dQg + co, D, dO, L, S0, L, 1.f, false);
  mm<C, D, D, false, true>(p.dWt + co, D, dU, L, S0, L, -1.f, false);
  mm<C, D, D, false, true>(p.dKh + co, D, U, L, dS, L, 1.f, false);
  mm<C, C, D, false, true>(p.dP + chunk_off(p, b, h, n, C * C), C, dO, L, U, L, 1.f, false);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int r = warp; r < D; r += nw) {
    float sv = dS[r * L + lane] * S0[r * L + lane] + dS[r * L + lane + 32] * S0[r * L + lane + 32];
    sv = warp_sum(sv);
    if (lane == 0) p.dgC[chunk_off(p, b, h, n, D) + r] = sv;
  }
}

// --------------------------------------------------------------- intra bwd
constexpr int bwd_smem() { return (12 * TILE + 2 * C + D) * 4; }

// float4 helpers for the per-channel loops below
HB_DEVICE float4 f4(float x) { return make_float4(x, x, x, x); }
HB_DEVICE float4 exp2_4(float4 a, float4 b) {  // 2^(a - b) per lane
  return make_float4(exp2_fast(a.x - b.x), exp2_fast(a.y - b.y), exp2_fast(a.z - b.z), exp2_fast(a.w - b.w));
}
HB_DEVICE float4 mul4(float4 a, float4 b) { return make_float4(a.x * b.x, a.y * b.y, a.z * b.z, a.w * b.w); }
HB_DEVICE float4 fma4(float4 a, float4 b, float4 c) {
  return make_float4(fmaf(a.x, b.x, c.x), fmaf(a.y, b.y, c.y), fmaf(a.z, b.z, c.z), fmaf(a.w, b.w, c.w));
}
HB_DEVICE float4 add4(float4 a, float4 b) { return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }
HB_DEVICE float4 sub4(float4 a, float4 b) { return make_float4(a.x - b.x, a.y - b.y, a.z - b.z, a.w - b.w); }
HB_DEVICE float4 scl4(float s, float4 a) { return make_float4(s * a.x, s * a.y, s * a.z, s * a.w); }

template <int NT>
__global__ void __launch_bounds__(NT, 1) intra_bwd64_kernel(Ptrs p) {
  extern __shared__ float sm[];
  float* q = sm;
  float* k = q + TILE;
  float* G = k + TILE;
  float* dq = G + TILE;    // Linv, later dq
  float* dA = dq + TILE;   // dU, later dN -> dA
  float* T5 = dA + TILE;   // dWt, later Zr | TK
  float* dk = T5 + TILE;   // X, later dk
  float* dG = dk + TILE;   // Y, later dG
  float* T8 = dG + TILE;   // Ut, later Zq | SS
  float* T9 = T8 + TILE;   // Wt, later Zk
  float* dP = T9 + TILE;
  float* T11 = dP + TILE;  // A, later TQ
  float* bet = T11 + TILE;
  float* dbt = bet + C;
  float* red = dbt + C;
  float* Li = dq;
  float* dU = dA;
  float* dWt = T5;
  float* X = dk;
  float* Y = dG;
  float* Ut = T8;
  float* Wt = T9;
  float* Am = T11;
  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const float scale = p.scale;
  PhaseClock pc(p.prof);
  const long long co = chunk_off(p, b, h, n, C * D), po = chunk_off(p, b, h, n, C * C);
  // three load groups, consumed in order: (Linv, dU, dWt) for X and Y,
  // (Ut, Wt) for dN, then (q, k, g, dP, A)
  cp_chunk_tile(Li, p.Linv + po);
  cp_chunk_tile(dU, p.dU + co);
  cp_chunk_tile(dWt, p.dWt + co);
  cp_async_commit();
  cp_chunk_tile(Ut, p.Ut + co);
  cp_chunk_tile(Wt, p.Wt + co);
  cp_async_commit();
  cp_token_rows(p, p.q, b, h, n, q);
  cp_token_rows(p, p.k, b, h, n, k);
  cp_token_rows(p, p.g, b, h, n, G);
  cp_chunk_tile(dP, p.dP + po);
  cp_chunk_tile(Am, p.Am + po);
  cp_async_commit();
  load_beta(p, b, h, n, bet);
  if (threadIdx.x < D) red[threadIdx.x] = 0.f;
  cp_async_wait<2>();
  __syncthreads();
  pc.mark(10);
  // X = Linv^T dU,  Y = Linv^T dWt
  mm<C, D, C, true, false>(X, L, Li, L, dU, L, 1.f, false);
  mm<C, D, C, true, false>(Y, L, Li, L, dWt, L, 1.f, false);
  cp_async_wait<1>();
  __syncthreads();
  pc.mark(11);
  // dN = -(X Ut^T + Y Wt^T)   (same warp tiles in both calls: no barrier needed)
  float* dN = dA;
  mm<C, C, D, false, true>(dN, L, X, L, Ut, L, -1.f, false);
  mm<C, C, D, false, true>(dN, L, Y, L, Wt, L, -1.f, true);
  cp_async_wait<0>();
  __syncthreads();
  // v, dKh and dQg land in the freed dWt / Ut / Wt tiles while dbeta starts
  float* vs = T5;
  float* dKh = T8;
  float* dQg = T9;
  cp_token_rows(p, p.v, b, h, n, vs);
  cp_chunk_tile(dKh, p.dKh + co);
  cp_chunk_tile(dQg, p.dQg + co);
  cp_async_commit();
  cumsum_log2(G);
  for (int i = threadIdx.x; i < C * C; i += blockDim.x) {
    const int t = i / C, s = i % C;
    if (s > t) dP[t * L + s] = 0.f;
  }
  cp_async_wait<0>();
  __syncthreads();
  pc.mark(12);
  // dbeta_t = v_t.X_t + 2 b_t (sum_c K e^G Y + sum_{s<t} dN_ts A_ts);  dv = b X
  for (int t = warp; t < C; t += nw) {
    const int tg = n * C + t;
    const bool ok = tg < p.S;
    float s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      const int c = lane + 32 * cc;
      const int si = t * L + c;
      const float x = X[si];
      s3 += vs[si] * x;   // zero past S
      if (ok) p.dv[tok_off(p, b, tg, h, D) + c] = bet[t] * x;
      s2 += k[si] * exp2_fast(G[si]) * Y[si];
      if (c < t) s1 += dN[si] * Am[si];
    }
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    s3 = warp_sum(s3);
    if (lane == 0) dbt[t] = s3 + 2.f * bet[t] * (s1 + s2);
  }
  __syncthreads();
  pc.mark(13);
  // accumulators: dk = b^2 Y e^G + dKh e^{G_C-G};  dq = scale dQg e^G;
  // dG = b^2 Y K e^G - dKh K e^{G_C-G} + scale dQg Q e^G;  red = sum_t dKh K e^{G_C-G};
  // dA = diag(b^2) dN (strictly lower).  Work item (row t, 4 channels); a
  // thread keeps one channel group (blockDim % 16 == 0).
  {
    const float* GC = G + (C - 1) * L;
    const int c = (threadIdx.x % (D / 4)) * 4;
    const float4 gc = ld4(GC + c);
    float4 racc = f4(0.f);
    for (int i = threadIdx.x; i < C * D / 4; i += blockDim.x) {
      const int t = i / (D / 4);
      const int si = t * L + c;
      const float b2 = bet[t] * bet[t];
      const float4 gt = ld4(G + si);
      const float4 eg = exp2_4(gt, f4(0.f)), eh = exp2_4(gc, gt);
      const float4 y = ld4(Y + si), kk = ld4(k + si), qq = ld4(q + si);
      const float4 dkh = ld4(dKh + si), dqg = ld4(dQg + si);
      const float4 w = mul4(mul4(dkh, kk), eh);
      racc = add4(racc, w);
      const float4 yb = scl4(b2, mul4(y, eg));
      st4(X + si, fma4(dkh, eh, yb));                                          // dk
      st4(Y + si, add4(sub4(mul4(yb, kk), w), scl4(scale, mul4(mul4(dqg, qq), eg))));  // dG
      st4(Li + si, scl4(scale, mul4(dqg, eg)));                                 // dq
      const float4 dn = ld4(dN + si);                                          // dA (C == D)
      st4(dN + si, make_float4(c < t ? b2 * dn.x : 0.f, c + 1 < t ? b2 * dn.y : 0.f,
                               c + 2 < t ? b2 * dn.z : 0.f, c + 3 < t ? b2 * dn.w : 0.f));
    }
    atomicAdd(red + c, racc.x);
    atomicAdd(red + c + 1, racc.y);
    atomicAdd(red + c + 2, racc.z);
    atomicAdd(red + c + 3, racc.w);
  }
  __syncthreads();
  pc.mark(14);
  // off-diagonal column blocks j = 0, 1, 2 through the factorised decays
  float* Zr = T5;              // 16 rows
  float* TK = T5 + BS * L;     // up to 48 rows
  float* Zq = T8;              // up to 48 rows
  float* SS = T8 + 48 * L;     // 16 rows
  float* Zk = T9;              // up to 48 rows
  float* TQ = T11;             // up to 48 rows
  auto offdiag_round = [&](auto jc) {
    constexpr int j = decltype(jc)::value;
    constexpr int r0 = BS * (j + 1), M = C - r0, e = BS * j + BS - 1;
    for (int i = threadIdx.x; i < BS * D / 4; i += blockDim.x) {
      const int s = i / (D / 4), c = (i % (D / 4)) * 4;
      const int si = (BS * j + s) * L + c;
      st4(Zr + s * L + c, mul4(ld4(k + si), exp2_4(ld4(G + e * L + c), ld4(G + si))));
    }
    for (int i = threadIdx.x; i < M * D / 4; i += blockDim.x) {
      const int tt = i / (D / 4), c = (i % (D / 4)) * 4;
      const int si = (r0 + tt) * L + c;
      const float4 lt = exp2_4(ld4(G + si), ld4(G + e * L + c));
      st4(Zq + tt * L + c, scl4(scale, mul4(ld4(q + si), lt)));
      st4(Zk + tt * L + c, mul4(ld4(k + si), lt));
    }
    __syncthreads();
    pc.mark(15 + 3 * j);
    mm<M, D, BS, false, false>(TQ, L, dP + r0 * L + BS * j, L, Zr, L, 1.f, false);
    mm<M, D, BS, false, false>(TK, L, dA + r0 * L + BS * j, L, Zr, L, 1.f, false);
    mm<BS, D, M, true, false>(SS, L, dP + r0 * L + BS * j, L, Zq, L, 1.f, false);
    mm<BS, D, M, true, false>(SS, L, dA + r0 * L + BS * j, L, Zk, L, 1.f, true);
    __syncthreads();
    pc.mark(16 + 3 * j);
    for (int i = threadIdx.x; i < M * D / 4; i += blockDim.x) {
      const int tt = i / (D / 4), c = (i % (D / 4)) * 4;
      const int si = (r0 + tt) * L + c;
      const float4 lt = exp2_4(ld4(G + si), ld4(G + e * L + c));
      const float4 tq = scl4(scale, mul4(lt, ld4(TQ + tt * L + c))), tk = mul4(lt, ld4(TK + tt * L + c));
      st4(dq + si, add4(ld4(dq + si), tq));
      st4(dk + si, add4(ld4(dk + si), tk));
      st4(dG + si, add4(ld4(dG + si), fma4(ld4(q + si), tq, mul4(ld4(k + si), tk))));
    }
    for (int i = threadIdx.x; i < BS * D / 4; i += blockDim.x) {
      const int s = i / (D / 4), c = (i % (D / 4)) * 4;
      const int si = (BS * j + s) * L + c;
      const float4 ss = mul4(exp2_4(ld4(G + e * L + c), ld4(G + si)), ld4(SS + s * L + c));
      st4(dk + si, add4(ld4(dk + si), ss));
      st4(dG + si, sub4(ld4(dG + si), mul4(ld4(k + si), ss)));
    }
    __syncthreads();
    pc.mark(17 + 3 * j);
  };
  offdiag_round(std::integral_constant<int, 0>{});
  offdiag_round(std::integral_constant<int, 1>{});
  offdiag_round(std::integral_constant<int, 2>{});
  // diagonal blocks pair by pair: item (row r, 4 channels) gathers its t-side
  // (s <= r) and its s-side (t >= r) terms, so no two threads write one element
  for (int i = threadIdx.x; i < C * D / 4; i += blockDim.x) {
    const int r = i / (D / 4), c = (i % (D / 4)) * 4;
    const int b0 = r & ~(BS - 1);
    const int si = r * L + c;
    const float4 gr = ld4(G + si), qr = ld4(q + si), kr = ld4(k + si);
    float4 aq = f4(0.f), ak = f4(0.f), ag = f4(0.f);
    for (int s = b0; s <= r; ++s) {
      const float4 ks = mul4(ld4(k + s * L + c), exp2_4(gr, ld4(G + s * L + c)));
      const float w = scale * dP[r * L + s], a = dA[r * L + s];
      aq = fma4(f4(w), ks, aq);
      ak = fma4(f4(a), ks, ak);
      ag = fma4(fma4(f4(w), qr, scl4(a, kr)), ks, ag);
    }
    for (int t = r; t < b0 + BS; ++t) {
      const int ti = t * L + c;
      const float w = scale * dP[t * L + r], a = dA[t * L + r];
      const float4 x = mul4(fma4(f4(w), ld4(q + ti), scl4(a, ld4(k + ti))), exp2_4(ld4(G + ti), gr));
      ak = add4(ak, x);
      ag = sub4(ag, mul4(kr, x));
    }
    st4(dq + si, add4(ld4(dq + si), aq));
    st4(dk + si, add4(ld4(dk + si), ak));
    st4(dG + si, add4(ld4(dG + si), ag));
  }
  __syncthreads();
  pc.mark(24);
  // dG_C = red + dgC e^{G_C} enters every row; dg = reverse cumsum of dG
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float acc = red[c] + p.dgC[chunk_off(p, b, h, n, D) + c] * exp2_fast(G[(C - 1) * L + c]);
#pragma unroll 16
    for (int t = C - 1; t >= 0; --t) {
      acc += dG[t * L + c];
      dG[t * L + c] = acc;
    }
  }
  __syncthreads();
  pc.mark(25);
  for (int i = threadIdx.x; i < C * D / 4; i += blockDim.x) {
    const int r = i / (D / 4), c = (i % (D / 4)) * 4;
    const int t = n * C + r;
    if (t >= p.S) continue;
    const long long o = tok_off(p, b, t, h, D) + c;
    const int si = r * L + c;
    st4(p.dq + o, ld4(dq + si));
    st4(p.dk + o, ld4(dk + si));
    st4(p.dg + o, ld4(dG + si));
  }
  for (int r = threadIdx.x; r < C; r += blockDim.x) {
    const int t = n * C + r;
    if (t < p.S) p.dbeta[((long long)b * p.S + t) * p.H + h] = dbt[r];
  }
  pc.mark(26);
}

}  // namespace kda64

static bool al16_64(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// tcgen05 version of the chunk-parallel backward state products (kda64_tc.cu)
void kda64_products_tc(const float* dU, const float* dout, const float* states, const float* dstates,
                       const float* U, float* dWt, float* dQg, float* dP, float* dKh, float* dgC, int B, int S,
                       int H, int NC);

// The products run on tcgen05 (fp32-accurate 3-pass tf32); HB_KDA64_TC=0
// selects the warp-level (mma.sync) kernel instead.
static bool kda64_use_tc() {
  static const bool on = [] {
    const char* e = getenv("HB_KDA64_TC");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Phase-cycle counters of the chunk-64 intra kernels (nullptr: off).
static unsigned long long* g_kda64_prof = nullptr;

// Sets (a 64-slot int64 CUDA tensor) or clears (None) the phase counters; the
// caller keeps the tensor alive while it is set.
void kda64_set_profile(c10::optional<torch::Tensor> counters) {
  if (!counters.has_value()) {
    g_kda64_prof = nullptr;
    return;
  }
  HB_CHECK(counters->scalar_type() == at::kLong && counters->numel() >= 64 && counters->is_cuda(),
           "kda64_set_profile: 64-slot int64 CUDA tensor");
  g_kda64_prof = reinterpret_cast<unsigned long long*>(counters->data_ptr<int64_t>());
}

static void set_smem64(const void* f, int bytes) {
  HB_CUDA_CHECK(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

// q,k,v,g: [B,S,H,64] fp32; beta [B,S,H]; o [B,S,H,64];
// saved: Wt,Ut,Kh,Qg,U [B,H,NC,64,64], Pm,Linv,Am [B,H,NC,64,64], gC [B,H,NC,64],
// states [B,H,NC,64,64]
void kda_fwd64(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g, torch::Tensor beta,
               double scale, torch::Tensor o, torch::Tensor Wt, torch::Tensor Ut, torch::Tensor Kh,
               torch::Tensor Qg, torch::Tensor Pm, torch::Tensor gC, torch::Tensor states,
               torch::Tensor Linv, torch::Tensor Am, torch::Tensor U) {
  using namespace kda64;
  Ptrs p{};
  p.B = q.size(0);
  p.S = q.size(1);
  p.H = q.size(2);
  HB_CHECK(q.size(3) == D, "kda_fwd64: head dim 64");
  p.NC = (p.S + C - 1) / C;
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
  p.Linv = Linv.data_ptr<float>();
  p.Am = Am.data_ptr<float>();
  p.Usv = U.data_ptr<float>();
  p.scale = (float)scale;
  p.prof = g_kda64_prof;
  HB_CHECK(Pm.size(-1) == C && Linv.size(-1) == C && Am.size(-1) == C, "kda_fwd64: chunk size mismatch");
  for (const void* ptr : {(const void*)p.q, (const void*)p.k, (const void*)p.v, (const void*)p.g,
                          (const void*)p.o, (const void*)p.Wt, (const void*)p.Ut, (const void*)p.Kh,
                          (const void*)p.Qg, (const void*)p.Pm, (const void*)p.states, (const void*)p.Linv,
                          (const void*)p.Am, (const void*)p.Usv, (const void*)p.gC})
    HB_CHECK(al16_64(ptr), "kda_fwd64: 16-byte aligned buffers required");
  const int s1 = fwd_smem(), s2 = state_fwd64_smem(), s3 = out64_smem();
  static bool cfg = false;
  if (!cfg) {
    set_smem64((const void*)intra_fwd64_kernel, s1);
    set_smem64((const void*)state_fwd64_kernel, s2);
    set_smem64((const void*)out64_kernel, s3);
    cfg = true;
  }
  intra_fwd64_kernel<<<dim3(p.NC, p.H, p.B), NTFW, s1, cur_stream()>>>(p);
  HB_CUDA_CHECK(cudaGetLastError());
  state_fwd64_kernel<<<dim3(D / VS, p.H, p.B), 256, s2, cur_stream()>>>(p);
  HB_CUDA_CHECK(cudaGetLastError());
  out64_kernel<<<dim3(p.NC, p.H, p.B), 256, s3, cur_stream()>>>(p);
  HB_CUDA_CHECK(cudaGetLastError());
}

// Backward of kda_fwd64.  Workspace (written here): dstates, dSq [B,H,NC,64,64],
// dU, dUp, dQg, dKh, dWt, dP [B,H,NC,64,64], dgC [B,H,NC,64].
void kda_bwd64(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g, torch::Tensor beta,
               double scale, torch::Tensor dout, torch::Tensor Wt, torch::Tensor Ut, torch::Tensor Kh,
               torch::Tensor Qg, torch::Tensor Pm, torch::Tensor gC, torch::Tensor states,
               torch::Tensor Linv, torch::Tensor Am, torch::Tensor U, torch::Tensor dstates,
               torch::Tensor dU, torch::Tensor dUp, torch::Tensor dSq, torch::Tensor dQg,
               torch::Tensor dKh, torch::Tensor dWt, torch::Tensor dP, torch::Tensor dgC,
               torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor dg, torch::Tensor dbeta) {
  using namespace kda64;
  Ptrs p{};
  p.B = q.size(0);
  p.S = q.size(1);
  p.H = q.size(2);
  HB_CHECK(q.size(3) == D, "kda_bwd64: head dim 64");
  HB_CHECK(dout.is_contiguous(), "kda_bwd64: contiguous dout");
  p.NC = (p.S + C - 1) / C;
  p.q = q.data_ptr<float>();
  p.k = k.data_ptr<float>();
  p.v = v.data_ptr<float>();
  p.g = g.data_ptr<float>();
  p.beta = beta.data_ptr<float>();
  p.dout = dout.data_ptr<float>();
  p.Wt = Wt.data_ptr<float>();
  p.Ut = Ut.data_ptr<float>();
  p.Kh = Kh.data_ptr<float>();
  p.Qg = Qg.data_ptr<float>();
  p.Pm = Pm.data_ptr<float>();
  p.gC = gC.data_ptr<float>();
  p.states = states.data_ptr<float>();
  p.Linv = Linv.data_ptr<float>();
  p.Am = Am.data_ptr<float>();
  p.Usv = U.data_ptr<float>();
  p.dstates = dstates.data_ptr<float>();
  p.dU = dU.data_ptr<float>();
  p.dUp = dUp.data_ptr<float>();
  p.dSq = dSq.data_ptr<float>();
  p.dQg = dQg.data_ptr<float>();
  p.dKh = dKh.data_ptr<float>();
  p.dWt = dWt.data_ptr<float>();
  p.dP = dP.data_ptr<float>();
  p.dgC = dgC.data_ptr<float>();
  p.dq = dq.data_ptr<float>();
  p.dk = dk.data_ptr<float>();
  p.dv = dv.data_ptr<float>();
  p.dg = dg.data_ptr<float>();
  p.dbeta = dbeta.data_ptr<float>();
  p.scale = (float)scale;
  p.prof = g_kda64_prof;
  for (const void* ptr : {(const void*)p.q, (const void*)p.k, (const void*)p.g, (const void*)p.dout,
                          (const void*)p.states, (const void*)p.dstates, (const void*)p.dU, (const void*)p.dUp,
                          (const void*)p.dSq, (const void*)p.dQg, (const void*)p.dKh, (const void*)p.dWt,
                          (const void*)p.dP, (const void*)p.dq, (const void*)p.dk, (const void*)p.dg,
                          (const void*)p.Linv, (const void*)p.Am, (const void*)p.Usv, (const void*)p.gC,
                          (const void*)p.dgC})
    HB_CHECK(al16_64(ptr), "kda_bwd64: 16-byte aligned buffers required");
  const int s0 = bwd_pre64_smem(), s1 = state_bwd64_smem(), s2 = prod_smem(), s3 = bwd_smem();
  static bool cfg = false;
  if (!cfg) {
    set_smem64((const void*)bwd_pre64_kernel, s0);
    set_smem64((const void*)state_bwd64_kernel, s1);
    set_smem64((const void*)state_products64_kernel, s2);
    set_smem64((const void*)intra_bwd64_kernel<512>, s3);
    set_smem64((const void*)intra_bwd64_kernel<1024>, s3);
    cfg = true;
  }
  const dim3 chunks(p.NC, p.H, p.B);
  const bool tc = kda64_use_tc();
  bwd_pre64_kernel<<<chunks, 256, s0, cur_stream()>>>(p);
  HB_CUDA_CHECK(cudaGetLastError());
  state_bwd64_kernel<<<dim3(D / VS, p.H, p.B), 256, s1, cur_stream()>>>(p);
  HB_CUDA_CHECK(cudaGetLastError());
  if (tc) {
    kda64_products_tc(p.dU, p.dout, p.states, p.dstates, p.Usv, p.dWt, p.dQg, p.dP, p.dKh, p.dgC, p.B, p.S,
                      p.H, p.NC);
  } else {
    state_products64_kernel<<<chunks, NTP, s2, cur_stream()>>>(p);
    HB_CUDA_CHECK(cudaGetLastError());
  }
  static const int bwd_threads = [] {
    const char* e = getenv("HB_KDA64_BWD_THREADS");
    return e && atoi(e) == 512 ? 512 : 1024;
  }();
  if (bwd_threads == 512) intra_bwd64_kernel<512><<<chunks, 512, s3, cur_stream()>>>(p);
  else intra_bwd64_kernel<1024><<<chunks, 1024, s3, cur_stream()>>>(p);
  HB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace hb
