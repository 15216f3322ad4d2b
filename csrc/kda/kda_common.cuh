// Chunked gated delta rule (Kimi Delta Attention): device code shared by the
// chunk-32 kernels (kda.cu, all head dims) and the chunk-64 sub-block kernels
// (kda64.cu, head dim 64): the 3xTF32 warp-tile matmul helper, chunk loads,
// base-2 log decays, the triangular column solves and the two sequential
// state recurrences (templated on the chunk size).
#pragma once
#include <cuda_runtime.h>

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
  // chunk-64 path (kda64.cu): forward saves Linv = (I + diag(b^2) A)^{-1} and A
  // ([B, H, NC, C, C]); its backward recurrence writes dU ([B, H, NC, C, K]) and
  // the state-product kernel dQg, dKh, dWt, dP ([B, H, NC, C, K|C]) and dgC
  // ([B, H, NC, K]).
  float *Linv, *Am, *dU, *dQg, *dKh, *dWt, *dP, *dgC;
  // chunk-64 recurrences: U = Ut - Wt S0 per chunk (saved by the forward), and
  // the backward's state-independent parts P^T dO ([.., C, K]) and Qg^T dO ([.., K, K])
  float *Usv, *dUp, *dSq;
  // optional phase-cycle counters of the chunk-64 intra kernels (nullptr: off)
  unsigned long long* prof;
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
// waits until at most N of this thread's committed cp.async groups are pending
template <int N>
HB_DEVICE void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

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

template <int DK, int C, int VS>
constexpr int state_fwd_smem() { return StateFwdSmem<DK, C, VS>::FLOATS * 4; }
template <int DK, int C, int VS>
constexpr int state_bwd_smem() { return StateBwdSmem<DK, C, VS>::FLOATS * 4; }

}  // namespace kda
}  // namespace hb
