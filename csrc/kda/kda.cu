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

namespace hb {
namespace kda {

constexpr int NT = 256;

// Shared-memory matrices use row strides = cols + 4 (a multiple of 4 that is
// 4 mod 32 for the widths used): the tensor-core fragment loads of a row-major
// operand (lanes over 8 rows x 4 columns) then touch 32 distinct banks, the
// transposed ones at most 2-way, and the SIMT loops (lanes over columns) none.
template <int DK>
constexpr int LDK() { return DK + 4; }
template <int C>
constexpr int LDC() { return C + 4; }

// out[m][n] (+)= alpha * sum_k A(m,k) B(k,n);  A(m,k) = a[m*lda+k] (or a[k*lda+m] if TA),
// B(k,n) = b[k*ldb+n] (or b[n*ldb+k] if TB).  Shared-memory operands, fp32 out.
//
// Tensor cores: mma.sync m16n8k8 with tf32 inputs, each fp32 operand split as
// x = hi + lo with hi = x truncated to tf32 (exact) and lo = x - hi (exact in
// fp32; the tensor core reads its top 19 bits), product hi*hi + hi*lo + lo*hi:
// about 2^-19 relative error per product, fp32-level for the recurrence that
// accumulates over the whole sequence.  A warp owns a 16 x 8*NS output tile
// (NS = 2 when that still gives every warp a tile, so one A fragment feeds two
// n-subtiles).
HB_DEVICE void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  hi = __float_as_uint(x) & 0xffffe000u;
  lo = __float_as_uint(x - __uint_as_float(hi));
}
HB_DEVICE void mma_tf32(float* c, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

template <int M, int N, int KD, bool TA, bool TB>
HB_DEVICE void mm(float* out, int ldo, const float* a, int lda, const float* b, int ldb, float alpha,
                  bool acc) {
  static_assert(M % 16 == 0 && N % 8 == 0 && KD % 8 == 0, "mm tile shape");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  constexpr int TM = M / 16;
  constexpr int NS = ((N / 8) % 2 == 0 && TM * (N / 16) >= 8) ? 2 : 1;
  constexpr int TN = N / (8 * NS);
  auto A = [&](int m, int k) { return TA ? a[k * lda + m] : a[m * lda + k]; };
  auto B = [&](int k, int n) { return TB ? b[n * ldb + k] : b[k * ldb + n]; };
  for (int tile = warp; tile < TM * TN; tile += nw) {
    const int m0 = (tile / TN) * 16, n0 = (tile % TN) * 8 * NS;
    float c[NS][4];
#pragma unroll
    for (int j = 0; j < NS; ++j) c[j][0] = c[j][1] = c[j][2] = c[j][3] = 0.f;
#pragma unroll 2
    for (int k0 = 0; k0 < KD; k0 += 8) {
      uint32_t ah[4], al[4];
      split_tf32(A(m0 + g, k0 + t), ah[0], al[0]);
      split_tf32(A(m0 + g + 8, k0 + t), ah[1], al[1]);
      split_tf32(A(m0 + g, k0 + t + 4), ah[2], al[2]);
      split_tf32(A(m0 + g + 8, k0 + t + 4), ah[3], al[3]);
#pragma unroll
      for (int j = 0; j < NS; ++j) {
        uint32_t bh[2], bl[2];
        split_tf32(B(k0 + t, n0 + 8 * j + g), bh[0], bl[0]);
        split_tf32(B(k0 + t + 4, n0 + 8 * j + g), bh[1], bl[1]);
        mma_tf32(c[j], al, bh);
        mma_tf32(c[j], ah, bl);
        mma_tf32(c[j], ah, bh);
      }
    }
#pragma unroll
    for (int j = 0; j < NS; ++j) {
      const int r0 = m0 + g, cc = n0 + 8 * j + 2 * t;
      float* o0 = out + r0 * ldo + cc;
      float* o1 = out + (r0 + 8) * ldo + cc;
      if (acc) {
        o0[0] += alpha * c[j][0];
        o0[1] += alpha * c[j][1];
        o1[0] += alpha * c[j][2];
        o1[1] += alpha * c[j][3];
      } else {
        o0[0] = alpha * c[j][0];
        o0[1] = alpha * c[j][1];
        o1[0] = alpha * c[j][2];
        o1[1] = alpha * c[j][3];
      }
    }
  }
}

struct Ptrs {
  const float *q, *k, *v, *g, *beta, *dout;
  float *Wt, *Ut, *Kh, *Qg, *Pm, *gC, *o, *states, *dstates;
  float *dq, *dk, *dv, *dg, *dbeta;
  int B, S, H, NC;
  float scale;
  const float* init_state;  // optional [B, H, K, V]
  float* final_state;       // optional
};

// global row pointer of token t in [B, S, H, DK]
HB_DEVICE long long tok_off(const Ptrs& p, int b, int t, int h, int DK) {
  return (((long long)b * p.S + t) * p.H + h) * DK;
}
// chunk-intermediate offset [B, H, NC, rows, cols]
HB_DEVICE long long chunk_off(const Ptrs& p, int b, int h, int n, int sz) {
  return ((((long long)b * p.H + h) * p.NC) + n) * sz;
}

// 16-byte shared/global accesses (every row offset used below is a multiple of 4 floats).
HB_DEVICE float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
HB_DEVICE void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }

// Thread count of the intra-chunk kernels: 256 up to head dim 64 (two or more
// blocks per SM), 512 for head dim 128 (one block per SM with 205 KB of tiles).
template <int DK>
constexpr int NTB() { return DK >= 128 ? 512 : 256; }

// Load one chunk's rows of [B, S, H, DK] x (zeros past S) into padded smem.
template <int DK, int C>
HB_DEVICE void load_rows(const Ptrs& p, const float* x, int b, int h, int n, float* dst) {
  constexpr int L = LDK<DK>(), D4 = DK / 4;
  for (int i = threadIdx.x; i < C * D4; i += blockDim.x) {
    const int r = i / D4, c = (i % D4) * 4;
    const int t = n * C + r;
    float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    if (t < p.S) z = ld4(x + tok_off(p, b, t, h, DK) + c);
    st4(dst + r * L + c, z);
  }
}

// In shared memory the cumulative decays are kept as G' = G log2(e), so every
// e^{G_t - G_s} of the chunk kernels is one 2^{G'_t - G'_s} on the MUFU unit
// (PTX ex2.approx), without a separate multiply by log2(e).
constexpr float kLog2e = 1.4426950408889634f;
HB_DEVICE float exp2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// q, k, v, g and beta of one chunk; g is cumulated in place into G
// (registers per column, so the 32 loads of a column are independent).
template <int DK, int C>
HB_DEVICE void load_chunk(const Ptrs& p, int b, int h, int n, float* q, float* k, float* v, float* G,
                          float* bet) {
  constexpr int L = LDK<DK>();
  load_rows<DK, C>(p, p.q, b, h, n, q);
  load_rows<DK, C>(p, p.k, b, h, n, k);
  load_rows<DK, C>(p, p.v, b, h, n, v);
  load_rows<DK, C>(p, p.g, b, h, n, G);
  for (int r = threadIdx.x; r < C; r += blockDim.x) {
    const int t = n * C + r;
    bet[r] = t < p.S ? p.beta[((long long)b * p.S + t) * p.H + h] : 0.f;
  }
  __syncthreads();
  for (int c = threadIdx.x; c < DK; c += blockDim.x) {
    float x[C];
#pragma unroll
    for (int r = 0; r < C; ++r) x[r] = G[r * L + c];
#pragma unroll
    for (int r = 1; r < C; ++r) x[r] += x[r - 1];
#pragma unroll
    for (int r = 0; r < C; ++r) G[r * L + c] = x[r] * kLog2e;  // base-2 log decays
  }
  __syncthreads();
}

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

// x <- (I + N)^{-1} x for one column held in registers (N strictly lower):
// right-looking substitution, each step's updates are independent.
template <int C>
HB_DEVICE void col_solve_lower(float (&x)[C], const float* N) {
  constexpr int LC = LDC<C>();
#pragma unroll
  for (int p = 0; p < C - 1; ++p) {
#pragma unroll
    for (int t = p + 1; t < C; ++t) x[t] = fmaf(-N[t * LC + p], x[p], x[t]);
  }
}
// x <- (I + N)^{-T} x
template <int C>
HB_DEVICE void col_solve_upper_t(float (&x)[C], const float* N) {
  constexpr int LC = LDC<C>();
#pragma unroll
  for (int t = C - 1; t > 0; --t) {
#pragma unroll
    for (int s = 0; s < t; ++s) x[s] = fmaf(-N[t * LC + s], x[t], x[s]);
  }
}

// For each of `ncols` columns: x_t = ld(t, col); solve; st(t, col, x_t).
// Each thread owns whole columns, so dst may alias src.
template <int C, bool UPPER_T, class Ld, class St>
HB_DEVICE void solve_cols(int ncols, const float* N, Ld ld, St st) {
  for (int col = threadIdx.x; col < ncols; col += blockDim.x) {
    float x[C];
#pragma unroll
    for (int t = 0; t < C; ++t) x[t] = ld(t, col);
    if (UPPER_T) col_solve_upper_t<C>(x, N);
    else col_solve_lower<C>(x, N);
#pragma unroll
    for (int t = 0; t < C; ++t) st(t, col, x[t]);
  }
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

// ------------------------------------------------------------------ state fwd
// grid (DK / VS, H, B): value columns [vs*VS, vs*VS+VS) of the state, chunks in
// order.  The next chunk's operands (Wt, Qg, the Ut slice, P, gC) are fetched
// with cp.async into the second half of a double buffer while the current
// chunk computes; Kh (needed last) has one buffer, refilled right after its
// use for the following chunk.
HB_DEVICE void cp_async16(float* smem, const float* gmem, bool valid = true) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(valid ? 16 : 0)
               : "memory");
}
HB_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
HB_DEVICE void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// rows x cols fp32 (cols % 4 == 0) from global (row stride gs) to smem (row stride ls)
template <int ROWS, int COLS>
HB_DEVICE void cp_tile(float* s, int ls, const float* g, long long gs) {
  constexpr int C4 = COLS / 4;
  for (int i = threadIdx.x; i < ROWS * C4; i += blockDim.x) {
    const int r = i / C4, c = (i % C4) * 4;
    cp_async16(s + r * ls + c, g + r * gs + c);
  }
}

template <int DK, int C, int VS>
struct StateFwdSmem {
  static constexpr int L = LDK<DK>(), LC = LDC<C>(), LV = VS + 4;
  static constexpr int BUF = 2 * C * L + C * LV + C * LC + DK;  // Wt, Qg, Ut slice, P, gC
  static constexpr int FLOATS = 2 * DK * LV + 2 * C * LV + C * L + 2 * BUF;
};

template <int DK, int C, int VS>
__global__ void __launch_bounds__(NT) state_fwd_kernel(Ptrs p) {
  using SM = StateFwdSmem<DK, C, VS>;
  constexpr int L = SM::L, LC = SM::LC, LV = SM::LV;
  extern __shared__ float sm[];
  float* S = sm;                 // DK x LV
  float* Tn = S + DK * LV;       // DK x LV
  float* U = Tn + DK * LV;       // C x LV
  float* O = U + C * LV;         // C x LV
  float* Kh = O + C * LV;        // C x L
  float* buf0 = Kh + C * L;      // two operand sets
  const int vs = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int v0 = vs * VS;
  auto set = [&](int n) { return buf0 + (n & 1) * SM::BUF; };
  auto fetch = [&](int n) {
    float* bs = set(n);
    const long long co = chunk_off(p, b, h, n, C * DK);
    cp_tile<C, DK>(bs, L, p.Wt + co, DK);
    cp_tile<C, DK>(bs + C * L, L, p.Qg + co, DK);
    cp_tile<C, VS>(bs + 2 * C * L, LV, p.Ut + co + v0, DK);
    cp_tile<C, C>(bs + 2 * C * L + C * LV, LC, p.Pm + chunk_off(p, b, h, n, C * C), C);
    cp_tile<1, DK>(bs + 2 * C * L + C * LV + C * LC, DK, p.gC + chunk_off(p, b, h, n, DK), DK);
  };
  for (int i = threadIdx.x; i < DK * VS; i += blockDim.x) {
    const int r = i / VS, c = i % VS;
    S[r * LV + c] = p.init_state ? p.init_state[((long long)b * p.H + h) * DK * DK + r * DK + v0 + c] : 0.f;
  }
  fetch(0);
  cp_tile<C, DK>(Kh, L, p.Kh + chunk_off(p, b, h, 0, C * DK), DK);
  cp_async_commit();
  for (int n = 0; n < p.NC; ++n) {
    cp_async_wait_all();
    __syncthreads();
    if (n + 1 < p.NC) {  // the next chunk's operands land during this chunk's math
      fetch(n + 1);
      cp_async_commit();
    }
    const float* bs = set(n);
    const float* Wt = bs;
    const float* Qg = bs + C * L;
    const float* Ut = bs + 2 * C * L;
    const float* P = Ut + C * LV;
    const float* gc = P + C * LC;
    const long long so = chunk_off(p, b, h, n, DK * DK);
    for (int i = threadIdx.x; i < DK * VS / 4; i += blockDim.x) {
      const int r = i / (VS / 4), c = (i % (VS / 4)) * 4;
      st4(p.states + so + r * DK + v0 + c, ld4(S + r * LV + c));
    }
    for (int i = threadIdx.x; i < C * VS; i += blockDim.x) U[(i / VS) * LV + i % VS] = Ut[(i / VS) * LV + i % VS];
    __syncthreads();
    // U = Ut - Wt S ;  O = Qg S
    mm<C, VS, DK, false, false>(U, LV, Wt, L, S, LV, -1.f, true);
    mm<C, VS, DK, false, false>(O, LV, Qg, L, S, LV, 1.f, false);
    __syncthreads();
    // O += P U (P lower triangular);  Tn = Kh^T U
    mm<C, VS, C, false, false>(O, LV, P, LC, U, LV, 1.f, true);
    mm<DK, VS, C, true, false>(Tn, LV, Kh, L, U, LV, 1.f, false);
    __syncthreads();
    if (n + 1 < p.NC) {
      cp_tile<C, DK>(Kh, L, p.Kh + chunk_off(p, b, h, n + 1, C * DK), DK);
      cp_async_commit();
    }
    for (int e = threadIdx.x; e < DK * VS; e += blockDim.x) {
      const int r = e / VS, c = e % VS;
      S[r * LV + c] = gc[r] * S[r * LV + c] + Tn[r * LV + c];
    }
    for (int i = threadIdx.x; i < C * VS / 4; i += blockDim.x) {
      const int r = i / (VS / 4), c = (i % (VS / 4)) * 4;
      const int t = n * C + r;
      if (t < p.S) st4(p.o + tok_off(p, b, t, h, DK) + v0 + c, ld4(O + r * LV + c));
    }
  }
  __syncthreads();
  if (p.final_state)
    for (int i = threadIdx.x; i < DK * VS; i += blockDim.x) {
      const int r = i / VS, c = i % VS;
      p.final_state[((long long)b * p.H + h) * DK * DK + r * DK + v0 + c] = S[r * LV + c];
    }
}

// ------------------------------------------------------------------ state bwd
// dS_prev = gC * dS + Qg^T dO - Wt^T dU,  dU = P^T dO + Kh dS.  dstates[n] = dS at
// the END of chunk n.  grid (DK / VS, H, B) over value-column slices, chunks in
// reverse order, every operand of the next (earlier) chunk prefetched with
// cp.async into the other half of a double buffer.
template <int DK, int C, int VS>
struct StateBwdSmem {
  static constexpr int L = LDK<DK>(), LC = LDC<C>(), LV = VS + 4;
  static constexpr int BUF = 3 * C * L + C * LV + C * LC + DK;  // Kh, Wt, Qg, dO slice, P, gC
  static constexpr int FLOATS = 2 * DK * LV + C * LV + 2 * BUF;
};

template <int DK, int C, int VS>
__global__ void __launch_bounds__(NT) state_bwd_kernel(Ptrs p) {
  using SM = StateBwdSmem<DK, C, VS>;
  constexpr int L = SM::L, LC = SM::LC, LV = SM::LV;
  extern __shared__ float sm[];
  float* dS = sm;                // DK x LV
  float* T2 = dS + DK * LV;      // DK x LV
  float* dU = T2 + DK * LV;      // C x LV
  float* buf0 = dU + C * LV;
  const int vs = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int v0 = vs * VS;
  auto set = [&](int n) { return buf0 + (n & 1) * SM::BUF; };
  auto fetch = [&](int n) {
    float* bs = set(n);
    const long long co = chunk_off(p, b, h, n, C * DK);
    cp_tile<C, DK>(bs, L, p.Kh + co, DK);
    cp_tile<C, DK>(bs + C * L, L, p.Wt + co, DK);
    cp_tile<C, DK>(bs + 2 * C * L, L, p.Qg + co, DK);
    float* dO = bs + 3 * C * L;
    constexpr int V4 = VS / 4;
    for (int i = threadIdx.x; i < C * V4; i += blockDim.x) {
      const int r = i / V4, c = (i % V4) * 4;
      const int t = n * C + r;
      const bool ok = t < p.S;
      cp_async16(dO + r * LV + c, ok ? p.dout + tok_off(p, b, t, h, DK) + v0 + c : p.dout, ok);
    }
    cp_tile<C, C>(dO + C * LV, LC, p.Pm + chunk_off(p, b, h, n, C * C), C);
    cp_tile<1, DK>(dO + C * LV + C * LC, DK, p.gC + chunk_off(p, b, h, n, DK), DK);
  };
  for (int i = threadIdx.x; i < DK * LV; i += blockDim.x) dS[i] = 0.f;
  fetch(p.NC - 1);
  cp_async_commit();
  for (int n = p.NC - 1; n >= 0; --n) {
    cp_async_wait_all();
    __syncthreads();
    if (n > 0) {
      fetch(n - 1);
      cp_async_commit();
    }
    const float* bs = set(n);
    const float* Kh = bs;
    const float* Wt = bs + C * L;
    const float* Qg = bs + 2 * C * L;
    const float* dO = bs + 3 * C * L;
    const float* P = dO + C * LV;
    const float* gc = P + C * LC;
    const long long so = chunk_off(p, b, h, n, DK * DK);
    for (int i = threadIdx.x; i < DK * VS / 4; i += blockDim.x) {
      const int r = i / (VS / 4), c = (i % (VS / 4)) * 4;
      st4(p.dstates + so + r * DK + v0 + c, ld4(dS + r * LV + c));
    }
    // dU = P^T dO + Kh dS ;  T2 = Qg^T dO
    mm<C, VS, C, true, false>(dU, LV, P, LC, dO, LV, 1.f, false);
    mm<DK, VS, C, true, false>(T2, LV, Qg, L, dO, LV, 1.f, false);
    __syncthreads();
    mm<C, VS, DK, false, false>(dU, LV, Kh, L, dS, LV, 1.f, true);
    __syncthreads();
    // T2 -= Wt^T dU
    mm<DK, VS, C, true, false>(T2, LV, Wt, L, dU, LV, -1.f, true);
    __syncthreads();
    for (int e = threadIdx.x; e < DK * VS; e += blockDim.x) {
      const int r = e / VS, c = e % VS;
      dS[r * LV + c] = gc[r] * dS[r * LV + c] + T2[r * LV + c];
    }
  }
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
template <int DK, int C, int VS>
constexpr int state_fwd_smem() { return StateFwdSmem<DK, C, VS>::FLOATS * 4; }
template <int DK, int C, int VS>
constexpr int state_bwd_smem() { return StateBwdSmem<DK, C, VS>::FLOATS * 4; }
template <int DK, int C>
constexpr int intra_bwd_smem() {
  return (10 * C * LDK<DK>() + 2 * PANEL<DK>() * LDK<DK>() + 4 * C * LDC<C>() + 2 * C + 2 * DK) * 4;
}

// ================================================================ front-end
// One warp per token (all heads), two adjacent channels per lane: bf16x2 loads
// of the projection taps, float4 loads of the conv taps, float2 stores.
// raw: [T, 3*HK] bf16 rows (q | k | v projections, row stride ld_raw); conv
// weights [HK, 4] fp32 each; outputs fp32 [T, H, K].
HB_DEVICE float2 ld_bf2(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}
HB_DEVICE float tap(const float4& w, int i) { return i == 0 ? w.x : i == 1 ? w.y : i == 2 ? w.z : w.w; }
HB_DEVICE float rbf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
HB_DEVICE float silu_f(float x) { return x / (1.f + __expf(-x)); }
HB_DEVICE float dsilu_f(float x) {
  const float s = 1.f / (1.f + __expf(-x));
  return s * (1.f + x * (1.f - s));
}
// softplus(y) = max(y, 0) + log1p(exp(-|y|)) never overflows
HB_DEVICE float softplus_f(float y) { return fmaxf(y, 0.f) + log1pf(__expf(-fabsf(y))); }

// Causal 4-tap conv of channels (ch, ch+1) of projection `which` at token t;
// rows[i] is the row of token t - 3 + i (nullptr before the sequence start).
// The result is rounded to the compute dtype (model/kda.py:136, 257-259).
HB_DEVICE float2 conv2(const __nv_bfloat16* const (&rows)[4], int off, const float* w, int ch) {
  const float4 wa = *reinterpret_cast<const float4*>(w + ch * 4);
  const float4 wb = *reinterpret_cast<const float4*>(w + ch * 4 + 4);
  float a0 = 0.f, a1 = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (!rows[i]) continue;
    const float2 x = ld_bf2(rows[i] + off);
    a0 += tap(wa, i) * x.x;
    a1 += tap(wb, i) * x.y;
  }
  return make_float2(rbf(a0), rbf(a1));
}

template <int DK>
__global__ void prep_fwd_kernel(const __nv_bfloat16* __restrict__ raw, long long ld_raw,
                                const float* __restrict__ wq, const float* __restrict__ wk,
                                const float* __restrict__ wv, const float* __restrict__ f,
                                const float* __restrict__ a_log, const float* __restrict__ dt_bias,
                                const float* __restrict__ braw, int gate_mode, int T, int S, int H,
                                float* __restrict__ q, float* __restrict__ k, float* __restrict__ v,
                                float* __restrict__ g, float* __restrict__ beta) {
  constexpr int NP = (DK + 63) / 64;
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  const int HK = H * DK;
  for (long long t = blockIdx.x * (long long)warps + (threadIdx.x >> 5); t < T; t += (long long)gridDim.x * warps) {
    const int pos = t % S;
    const __nv_bfloat16* rows[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) rows[i] = pos - (3 - i) >= 0 ? raw + (t - (3 - i)) * ld_raw : nullptr;
    for (int h = 0; h < H; ++h) {
      float2 qv[NP], kv[NP];
      float ssq = 0.f, ssk = 0.f;
#pragma unroll
      for (int j = 0; j < NP; ++j) {
        const int c = 2 * lane + 64 * j;
        qv[j] = kv[j] = make_float2(0.f, 0.f);
        if (c >= DK) continue;
        const int ch = h * DK + c;
        const float2 cq = conv2(rows, ch, wq, ch), ck = conv2(rows, HK + ch, wk, ch),
                     cv = conv2(rows, 2 * HK + ch, wv, ch);
        qv[j] = make_float2(silu_f(cq.x), silu_f(cq.y));
        kv[j] = make_float2(silu_f(ck.x), silu_f(ck.y));
        ssq += qv[j].x * qv[j].x + qv[j].y * qv[j].y;
        ssk += kv[j].x * kv[j].x + kv[j].y * kv[j].y;
        const long long o = t * HK + ch;
        *reinterpret_cast<float2*>(v + o) = make_float2(silu_f(cv.x), silu_f(cv.y));
        const float2 fz = *reinterpret_cast<const float2*>(f + o);
        const float2 db = *reinterpret_cast<const float2*>(dt_bias + ch);
        const float z0 = fz.x + db.x, z1 = fz.y + db.y;
        float2 gg;
        if (gate_mode == 0) {
          const float A = -__expf(a_log[h]);
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
      if (lane == 0) beta[t * H + h] = 1.f / (1.f + __expf(-braw[t * H + h]));
    }
  }
}

// Backward part 1 (block per head, warp per token): gradients at the conv
// outputs of q/k/v (fp32, [T, 3*HK]), df [T, HK] (bf16: it only feeds the
// f_proj GEMMs), dbraw [T, H]; d dt_bias and
// d a_log of the block's head are summed in each lane's registers over its
// tokens, then reduced through shared memory with one global atomic each.
template <int DK>
__global__ void __launch_bounds__(256, DK >= 128 ? 2 : 3) prep_bwd1_kernel(const __nv_bfloat16* __restrict__ raw, long long ld_raw,
                                 const float* __restrict__ wq, const float* __restrict__ wk,
                                 const float* __restrict__ wv, const float* __restrict__ f,
                                 const float* __restrict__ a_log, const float* __restrict__ dt_bias,
                                 const float* __restrict__ beta, int gate_mode, int T, int S, int H,
                                 const float* __restrict__ dq, const float* __restrict__ dk,
                                 const float* __restrict__ dv, const float* __restrict__ dg,
                                 const float* __restrict__ dbeta, float* __restrict__ dconv,
                                 __nv_bfloat16* __restrict__ df, float* __restrict__ dbraw,
                                 float* __restrict__ d_alog, float* __restrict__ d_dtb) {
  constexpr int NP = (DK + 63) / 64;
  __shared__ float s_dtb[DK + 1];  // this block's head: d dt_bias, then d a_log
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  const int HK = H * DK;
  const int h = blockIdx.y;        // one head per block: the bias gradients sum in registers
  float2 acc_dtb[NP];
#pragma unroll
  for (int j = 0; j < NP; ++j) acc_dtb[j] = make_float2(0.f, 0.f);
  float acc_al = 0.f;
  for (int i = threadIdx.x; i < DK + 1; i += blockDim.x) s_dtb[i] = 0.f;
  __syncthreads();
  for (long long t = blockIdx.x * (long long)warps + (threadIdx.x >> 5); t < T; t += (long long)gridDim.x * warps) {
    const int pos = t % S;
    const __nv_bfloat16* rows[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) rows[i] = pos - (3 - i) >= 0 ? raw + (t - (3 - i)) * ld_raw : nullptr;
    {
      float2 cq[NP], ck[NP], sq[NP], sk[NP], gq[NP], gk[NP];
      float ssq = 0.f, ssk = 0.f, dotq = 0.f, dotk = 0.f, dal = 0.f;
#pragma unroll
      for (int j = 0; j < NP; ++j) {
        const int c = 2 * lane + 64 * j;
        cq[j] = ck[j] = sq[j] = sk[j] = gq[j] = gk[j] = make_float2(0.f, 0.f);
        if (c >= DK) continue;
        const int ch = h * DK + c;
        const long long o = t * HK + ch;
        cq[j] = conv2(rows, ch, wq, ch);
        ck[j] = conv2(rows, HK + ch, wk, ch);
        const float2 cv = conv2(rows, 2 * HK + ch, wv, ch);
        sq[j] = make_float2(silu_f(cq[j].x), silu_f(cq[j].y));
        sk[j] = make_float2(silu_f(ck[j].x), silu_f(ck[j].y));
        ssq += sq[j].x * sq[j].x + sq[j].y * sq[j].y;
        ssk += sk[j].x * sk[j].x + sk[j].y * sk[j].y;
        gq[j] = *reinterpret_cast<const float2*>(dq + o);
        gk[j] = *reinterpret_cast<const float2*>(dk + o);
        dotq += gq[j].x * sq[j].x + gq[j].y * sq[j].y;
        dotk += gk[j].x * sk[j].x + gk[j].y * sk[j].y;
        const float2 gv = *reinterpret_cast<const float2*>(dv + o);
        const long long co = t * 3 * HK + ch;
        *reinterpret_cast<float2*>(dconv + co + 2 * HK) = make_float2(gv.x * dsilu_f(cv.x), gv.y * dsilu_f(cv.y));
        // decay gate
        const float2 fz = *reinterpret_cast<const float2*>(f + o);
        const float2 db = *reinterpret_cast<const float2*>(dt_bias + ch);
        const float2 gg = *reinterpret_cast<const float2*>(dg + o);
        const float z[2] = {fz.x + db.x, fz.y + db.y}, dgv[2] = {gg.x, gg.y};
        float dz[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float sig = 1.f / (1.f + __expf(-z[e]));
          if (gate_mode == 0) {
            const float A = __expf(a_log[h]);
            dz[e] = dgv[e] * (-A) * sig;
            dal += dgv[e] * (-A * softplus_f(z[e]));
          } else {
            dz[e] = dgv[e] * (1.f - sig);
          }
        }
        *reinterpret_cast<__nv_bfloat162*>(df + o) = __floats2bfloat162_rn(dz[0], dz[1]);
        acc_dtb[j].x += dz[0];
        acc_dtb[j].y += dz[1];
      }
      ssq = warp_sum(ssq);
      ssk = warp_sum(ssk);
      dotq = warp_sum(dotq);
      dotk = warp_sum(dotk);
      dal = warp_sum(dal);
      const float nq = sqrtf(ssq + 1e-6f), nk = sqrtf(ssk + 1e-6f);
#pragma unroll
      for (int j = 0; j < NP; ++j) {
        const int c = 2 * lane + 64 * j;
        if (c >= DK) continue;
        const long long co = t * 3 * HK + h * DK + c;
        // y = x / n, n = sqrt(|x|^2 + eps): dx = (dy - y (dy . y)) / n
        const float dq0 = (gq[j].x - sq[j].x / nq * (dotq / nq)) / nq;
        const float dq1 = (gq[j].y - sq[j].y / nq * (dotq / nq)) / nq;
        const float dk0 = (gk[j].x - sk[j].x / nk * (dotk / nk)) / nk;
        const float dk1 = (gk[j].y - sk[j].y / nk * (dotk / nk)) / nk;
        *reinterpret_cast<float2*>(dconv + co) = make_float2(dq0 * dsilu_f(cq[j].x), dq1 * dsilu_f(cq[j].y));
        *reinterpret_cast<float2*>(dconv + co + HK) = make_float2(dk0 * dsilu_f(ck[j].x), dk1 * dsilu_f(ck[j].y));
      }
      acc_al += dal;
      if (lane == 0) {
        const float bt = beta[t * H + h];
        dbraw[t * H + h] = dbeta[t * H + h] * bt * (1.f - bt);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < NP; ++j) {
    const int c = 2 * lane + 64 * j;
    if (c < DK) {
      atomicAdd(s_dtb + c, acc_dtb[j].x);
      atomicAdd(s_dtb + c + 1, acc_dtb[j].y);
    }
  }
  if (lane == 0 && gate_mode == 0) atomicAdd(s_dtb + DK, acc_al);
  __syncthreads();
  for (int i = threadIdx.x; i < DK; i += blockDim.x)
    if (s_dtb[i] != 0.f) atomicAdd(d_dtb + h * DK + i, s_dtb[i]);
  if (threadIdx.x == 0 && s_dtb[DK] != 0.f) atomicAdd(d_alog + h, s_dtb[DK]);
}

// Backward part 2 (thread per channel of the 3*HK conv inputs, a run of tokens):
//   draw[t] = sum_i w[i] dconv[t + 3 - i] (same sequence); dw[i] += dconv[t] raw[t-3+i]
// dconv and raw are held in 4-deep register windows, so each element is loaded once.
__global__ void prep_bwd2_kernel(const __nv_bfloat16* __restrict__ raw, long long ld_raw,
                                 const float* __restrict__ wq, const float* __restrict__ wk,
                                 const float* __restrict__ wv, const float* __restrict__ dconv,
                                 int T, int S, int HK, __nv_bfloat16* __restrict__ draw,
                                 float* __restrict__ dwq, float* __restrict__ dwk, float* __restrict__ dwv) {
  const int C3 = 3 * HK;
  const int ch = blockIdx.x * blockDim.x + threadIdx.x;
  if (ch >= C3) return;
  const int which = ch / HK, cc = ch % HK;
  const float* w = which == 0 ? wq : (which == 1 ? wk : wv);
  float* dw = which == 0 ? dwq : (which == 1 ? dwk : dwv);
  const float4 wt = *reinterpret_cast<const float4*>(w + cc * 4);
  const int tpb = (T + gridDim.y - 1) / gridDim.y;
  const int tb = blockIdx.y * tpb, te = min(T, tb + tpb);
  if (tb >= te) return;
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  const float* dcol = dconv + ch;
  const __nv_bfloat16* rcol = raw + ch;
  auto dc = [&](int t) { return t < T ? dcol[(long long)t * C3] : 0.f; };
  auto rw = [&](int t) { return t >= 0 ? __bfloat162float(rcol[(long long)t * ld_raw]) : 0.f; };
  // windows: d0..d3 = dconv[t..t+3], r1..r3 = raw[t-1..t-3]
  float d0 = dc(tb), d1 = dc(tb + 1), d2 = dc(tb + 2), d3 = dc(tb + 3);
  float r1 = rw(tb - 1), r2 = rw(tb - 2), r3 = rw(tb - 3);
  int pos = tb % S;
  for (int t = tb; t < te; ++t) {
    const float r0 = rw(t);
    const float dn = dc(t + 4);
    float acc = wt.w * d0;
    if (pos + 1 < S) acc += wt.z * d1;
    if (pos + 2 < S) acc += wt.y * d2;
    if (pos + 3 < S) acc += wt.x * d3;
    draw[(long long)t * ld_raw + ch] = __float2bfloat16_rn(acc);
    a3 += d0 * r0;
    if (pos >= 1) a2 += d0 * r1;
    if (pos >= 2) a1 += d0 * r2;
    if (pos >= 3) a0 += d0 * r3;
    d0 = d1;
    d1 = d2;
    d2 = d3;
    d3 = dn;
    r3 = r2;
    r2 = r1;
    r1 = r0;
    if (++pos == S) pos = 0;
  }
  atomicAdd(dw + cc * 4 + 0, a0);
  atomicAdd(dw + cc * 4 + 1, a1);
  atomicAdd(dw + cc * 4 + 2, a2);
  atomicAdd(dw + cc * 4 + 3, a3);
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
  const int grid = (int)std::min<long long>(((long long)T + 7) / 8, num_sms() * 16);
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
                  torch::Tensor dbeta, torch::Tensor dconv, torch::Tensor df, torch::Tensor dbraw,
                  torch::Tensor d_alog, torch::Tensor d_dtb, torch::Tensor draw, torch::Tensor dwq,
                  torch::Tensor dwk, torch::Tensor dwv) {
  const int T = dq.size(0), H = dq.size(1), DKV = dq.size(2);
  HB_CHECK(raw.stride(0) % 2 == 0 && DKV % 2 == 0, "kda_prep: even row stride and head dim");
  HB_CHECK(df.scalar_type() == at::kBFloat16 && df.is_contiguous(), "kda_prep_bwd: df must be contiguous bf16");
  // blocks: (token runs) x (heads); about 8 resident blocks per SM in all
  const int gx = (int)std::max<long long>(
      1, std::min<long long>(((long long)T + 7) / 8, ((long long)num_sms() * 8 + H - 1) / H));
  const dim3 grid(gx, H);
  auto launch = [&](auto dkc) {
    constexpr int DK = decltype(dkc)::value;
    kda::prep_bwd1_kernel<DK><<<grid, 256, 0, cur_stream()>>>(
        (const __nv_bfloat16*)raw.data_ptr(), raw.stride(0), wq.data_ptr<float>(), wk.data_ptr<float>(),
        wv.data_ptr<float>(), f.data_ptr<float>(), a_log.data_ptr<float>(), dt_bias.data_ptr<float>(),
        beta.data_ptr<float>(), (int)gate_mode, T, (int)S, H, dq.data_ptr<float>(), dk.data_ptr<float>(),
        dv.data_ptr<float>(), dg.data_ptr<float>(), dbeta.data_ptr<float>(), dconv.data_ptr<float>(),
        (__nv_bfloat16*)df.data_ptr(), dbraw.data_ptr<float>(), d_alog.data_ptr<float>(), d_dtb.data_ptr<float>());
  };
  if (DKV == 16) launch(std::integral_constant<int, 16>{});
  else if (DKV == 32) launch(std::integral_constant<int, 32>{});
  else if (DKV == 64) launch(std::integral_constant<int, 64>{});
  else if (DKV == 128) launch(std::integral_constant<int, 128>{});
  else HB_CHECK(false, "kda_prep: unsupported head dim");
  HB_CUDA_CHECK(cudaGetLastError());
  const int HK = H * DKV;
  dim3 g2((3 * HK + 255) / 256, std::max(1, std::min(64, T / 64)));
  kda::prep_bwd2_kernel<<<g2, 256, 0, cur_stream()>>>(
      (const __nv_bfloat16*)raw.data_ptr(), raw.stride(0), wq.data_ptr<float>(), wk.data_ptr<float>(),
      wv.data_ptr<float>(), dconv.data_ptr<float>(), T, (int)S, HK, (__nv_bfloat16*)draw.data_ptr(),
      dwq.data_ptr<float>(), dwk.data_ptr<float>(), dwv.data_ptr<float>());
  HB_CUDA_CHECK(cudaGetLastError());
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
    if (!g_dev_ptr[dev]) {
      void* ptr = nullptr;
      if (cudaGetSymbolAddress(&ptr, g_scratch) != cudaSuccess || ptr == nullptr)
        return HB_NOALLOC_CUDA_ERROR;
      g_dev_ptr[dev] = static_cast<float*>(ptr);
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
