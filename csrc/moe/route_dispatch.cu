// MoE router and token dispatch (model/moe.py:37-85, 170-293).
//
// router_fwd   fp32 router logits, sigmoid(+bias) or softmax scores, top-k
//              selection, renormalised weights, and per-sequence aux partials
//              (counts, routing-probability sums, logsumexp^2, entropy).  The
//              logits run on the tcgen05 GEMM: the fp32 weight is split into three
//              bf16 terms (hi + mid + lo) and x (bf16, exact) multiplies all three
//              with fp32 accumulation, which reproduces the fp32 product of the
//              reference (model/moe.py:177-181); a SIMT kernel covers shapes whose
//              rows are not 16-byte aligned.
// router_grads dx and dW of the router GEMM, also as split-bf16 tensor-core GEMMs.
// router_bwd   d(logits) from the gradients of the combine weights, the z-loss
//              and the sequence-wise balance loss.
// moe_plan     stable counting sort of the T*K (token, slot) pairs by expert into a
//              row buffer whose expert segments start at multiples of 128; emits
//              per-expert starts / counts, the grouped-GEMM tile prefix, and the
//              row of every (token, slot).
// moe_gather / moe_scatter_add, moe_combine / moe_combine_bwd  permute and
//              un-permute rows; the pad rows of every expert segment are zero.
#include <torch/extension.h>

#include "../common/host.h"
#include "../common/sm100.cuh"

namespace hb {

namespace {

constexpr int MAXN = 256;  // experts
constexpr int MAXK = 16;   // top-k

// ------------------------------------------------------------------ router fwd
// Block = RT_TOK consecutive tokens.  The router weight W_r [D, N] is staged in
// shared memory in row chunks of DC rows (the whole matrix when it fits) and
// every token's logits are accumulated in a shared [RT_TOK][N] array; one warp
// per token, lane e owns experts e, e+32, ...
constexpr int RT_TOK = 64;
constexpr int RT_SMEM_W = 32 * 1024;   // router-weight chunk staged per block
constexpr int RT_NSEQ = 4;             // sequences a block reduces in shared memory

// Per-token routing from the logits lg (lane e holds experts e, e+32, ...):
// scores, aux partials, top-k and the renormalised combine weights.
template <int EPL>
HB_DEVICE void route_token(int t, float (&lg)[8], const float* __restrict__ bias, int S, int N, int K,
                           int softmax_mode, float scaling, int b_first, float* __restrict__ logits_out,
                           int* __restrict__ topi, float* __restrict__ topw, float* __restrict__ seq_counts,
                           float* __restrict__ seq_probs, float* scnt, float* sprb, float& zsum,
                           float& esum) {
  const int lane = threadIdx.x & 31;
  float sc[8], ef[8];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = lane + 32 * i;
    if (i < EPL && e < N) {
      logits_out[(long long)t * N + e] = lg[i];
      mx = fmaxf(mx, lg[i]);
    }
  }
  mx = warp_max(mx);
  float se = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (i < EPL && lane + 32 * i < N) se += __expf(lg[i] - mx);
  se = warp_sum(se);
  const float lse = mx + __logf(se);
  float ssum = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = lane + 32 * i;
    if (i < EPL && e < N) {
      sc[i] = softmax_mode ? __expf(lg[i] - lse) : 1.f / (1.f + __expf(-lg[i]));
      ef[i] = softmax_mode ? sc[i] : sc[i] + bias[e];
      ssum += sc[i];
    } else {
      sc[i] = 0.f;
      ef[i] = -INFINITY;
    }
  }
  ssum = warp_sum(ssum);
  float ent = 0.f;
  const float inv = 1.f / (ssum + 1e-9f);
  const int b = t / S;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = lane + 32 * i;
    if (i < EPL && e < N) {
      const float pr = sc[i] * inv;
      ent -= pr * __logf(pr + 1e-9f);
      if (b - b_first < RT_NSEQ) atomicAdd(sprb + (b - b_first) * N + e, pr);
      else atomicAdd(seq_probs + (long long)b * N + e, pr);
    }
  }
  ent = warp_sum(ent);
  // top-k by repeated warp argmax (ties -> lowest expert id, like top_k).  A NaN
  // score ranks as -inf, and every round picks an expert not yet taken, so the
  // K ids are always distinct and in [0, N) (they index shared memory and the
  // dispatch), whatever the logits hold.
  float selsum = 0.f;
  float selv[MAXK];
  int seli[MAXK];
  unsigned taken = 0;
  for (int kk = 0; kk < K; ++kk) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = lane + 32 * i;
      const float v = ef[i] != ef[i] ? -INFINITY : ef[i];
      if (i < EPL && e < N && !(taken >> i & 1u) && (v > bv || (v == bv && e < bi))) {
        bv = v;
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (bi >= N) bi = 0;  // unreachable for K <= N; keeps the id in range regardless
    float s_win = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (lane + 32 * i == bi) {
        s_win = sc[i];
        taken |= 1u << i;
      }
    s_win = warp_sum(s_win);
    seli[kk] = bi;
    selv[kk] = s_win;
    selsum += s_win;
  }
  if (lane == 0) {
    const float denom = selsum + 1e-9f;
    for (int kk = 0; kk < K; ++kk) {
      topi[(long long)t * K + kk] = seli[kk];
      topw[(long long)t * K + kk] = selv[kk] / denom * (softmax_mode ? 1.f : scaling);
      if (b - b_first < RT_NSEQ) atomicAdd(scnt + (b - b_first) * N + seli[kk], 1.f);
      else atomicAdd(seq_counts + (long long)b * N + seli[kk], 1.f);
    }
    zsum += lse * lse;
    esum += ent;
  }
}

// Block-level flush of the per-sequence partials and the z / entropy sums.
HB_DEVICE void route_flush(int t_begin, int t_end, int S, int N, int b_first, float* __restrict__ seq_counts,
                           float* __restrict__ seq_probs, const float* scnt, const float* sprb, float zsum,
                           float esum, float* __restrict__ sums) {
  if ((threadIdx.x & 31) == 0) {
    atomicAdd(sums + 0, zsum);
    atomicAdd(sums + 1, esum);
  }
  __syncthreads();
  const int nb = min(RT_NSEQ, (t_end - 1) / S - b_first + 1);
  for (int i = threadIdx.x; i < nb * N; i += blockDim.x) {
    const int bl = i / N, e = i % N;
    const long long gi = (long long)(b_first + bl) * N + e;
    if (scnt[i] != 0.f) atomicAdd(seq_counts + gi, scnt[i]);
    if (sprb[i] != 0.f) atomicAdd(seq_probs + gi, sprb[i]);
  }
}

template <int EPL>
__global__ void router_fwd_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ W,
                                  const float* __restrict__ bias, int T, int S, int D, int N, int K,
                                  int softmax_mode, float scaling, int DC, float* __restrict__ logits_out,
                                  int* __restrict__ topi, float* __restrict__ topw,
                                  float* __restrict__ seq_counts, float* __restrict__ seq_probs,
                                  float* __restrict__ sums /* [0]=sum lse^2, [1]=sum entropy */) {
  extern __shared__ float sh[];
  float* wsh = sh;                      // [DC][N]
  float* acc = sh + DC * N;             // [RT_TOK][N]
  float* scnt = acc + RT_TOK * N;       // [RT_NSEQ][N] per-sequence counts of this block
  float* sprb = scnt + RT_NSEQ * N;     // [RT_NSEQ][N] per-sequence probability sums
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int warps = blockDim.x >> 5;
  // EPL (template): experts per lane, ceil(N / 32)
  const int t_begin = blockIdx.x * RT_TOK;
  const int t_end = min(T, t_begin + RT_TOK);
  const int b_first = t_begin / S;
  for (int i = threadIdx.x; i < RT_TOK * N; i += blockDim.x) acc[i] = 0.f;
  for (int i = threadIdx.x; i < 2 * RT_NSEQ * N; i += blockDim.x) scnt[i] = 0.f;
  for (int d0 = 0; d0 < D; d0 += DC) {
    const int dn = min(DC, D - d0);
    __syncthreads();
    for (int i = threadIdx.x; i < dn * N; i += blockDim.x) wsh[i] = W[(long long)d0 * N + i];
    __syncthreads();
    for (int t = t_begin + warp; t < t_end; t += warps) {
      float a[EPL];
#pragma unroll
      for (int i = 0; i < EPL; ++i) a[i] = 0.f;
      const __nv_bfloat16* xr = x + (long long)t * D + d0;
      const bool full = (N % 32) == 0;
      for (int r0 = 0; r0 < dn; r0 += 32) {
        const float xv_l = (r0 + lane < dn) ? __bfloat162float(xr[r0 + lane]) : 0.f;
        const int rn = min(32, dn - r0);
#pragma unroll 8
        for (int r = 0; r < rn; ++r) {
          const float xv = __shfl_sync(0xffffffffu, xv_l, r);
          const float* wr = wsh + (r0 + r) * N + lane;
#pragma unroll
          for (int i = 0; i < EPL; ++i)
            if (full || lane + 32 * i < N) a[i] += xv * wr[32 * i];
        }
      }
      float* ar = acc + (t - t_begin) * N;
#pragma unroll
      for (int i = 0; i < EPL; ++i)
        if (lane + 32 * i < N) ar[lane + 32 * i] += a[i];
    }
  }
  __syncthreads();
  float zsum = 0.f, esum = 0.f;
  for (int t = t_begin + warp; t < t_end; t += warps) {
    const float* ar = acc + (t - t_begin) * N;
    float lg[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = lane + 32 * i;
      lg[i] = (i < EPL && e < N) ? ar[e] : -INFINITY;
    }
    route_token<EPL>(t, lg, bias, S, N, K, softmax_mode, scaling, b_first, logits_out, topi, topw,
                     seq_counts, seq_probs, scnt, sprb, zsum, esum);
  }
  route_flush(t_begin, t_end, S, N, b_first, seq_counts, seq_probs, scnt, sprb, zsum, esum, sums);
}

// Router on precomputed partial logits: l3 [T, 3N] holds x @ [W_hi | W_mid | W_lo]
// (three bf16 terms of the fp32 router weight, products accumulated in fp32 by
// the tensor-core GEMM); the logits are their sum.  Block = RT_TOK tokens.
template <int EPL>
__global__ void router_select_kernel(const float* __restrict__ l3, const float* __restrict__ bias,
                                     int T, int S, int N, int K, int softmax_mode, float scaling,
                                     float* __restrict__ logits_out, int* __restrict__ topi,
                                     float* __restrict__ topw, float* __restrict__ seq_counts,
                                     float* __restrict__ seq_probs, float* __restrict__ sums) {
  __shared__ float scnt[RT_NSEQ * MAXN];
  __shared__ float sprb[RT_NSEQ * MAXN];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
  const int t_begin = blockIdx.x * RT_TOK;
  const int t_end = min(T, t_begin + RT_TOK);
  const int b_first = t_begin / S;
  for (int i = threadIdx.x; i < RT_NSEQ * N; i += blockDim.x) scnt[i] = sprb[i] = 0.f;
  __syncthreads();
  float zsum = 0.f, esum = 0.f;
  for (int t = t_begin + warp; t < t_end; t += warps) {
    const float* r = l3 + (long long)t * 3 * N;
    float lg[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = lane + 32 * i;
      lg[i] = (i < EPL && e < N) ? (r[e] + r[N + e]) + r[2 * N + e] : -INFINITY;
    }
    route_token<EPL>(t, lg, bias, S, N, K, softmax_mode, scaling, b_first, logits_out, topi, topw,
                     seq_counts, seq_probs, scnt, sprb, zsum, esum);
  }
  route_flush(t_begin, t_end, S, N, b_first, seq_counts, seq_probs, scnt, sprb, zsum, esum, sums);
}

// W [D, N] fp32 -> w3 = [hi | mid | lo] and w3x = [hi | hi | mid], both [D, 3N]
// bf16, with hi = bf16(W), mid = bf16(W - hi), lo = bf16(W - hi - mid).
__global__ void router_split_w_kernel(const float* __restrict__ W, long long n, int N,
                                      __nv_bfloat16* __restrict__ w3, __nv_bfloat16* __restrict__ w3x) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long d = i / N;
    const int e = i % N;
    const float w = W[i];
    const __nv_bfloat16 hi = __float2bfloat16_rn(w);
    const float r = w - __bfloat162float(hi);
    const __nv_bfloat16 mid = __float2bfloat16_rn(r);
    const __nv_bfloat16 lo = __float2bfloat16_rn(r - __bfloat162float(mid));
    __nv_bfloat16* o = w3 + d * 3 * N + e;
    o[0] = hi;
    o[N] = mid;
    o[2 * N] = lo;
    __nv_bfloat16* ox = w3x + d * 3 * N + e;
    ox[0] = hi;
    ox[N] = hi;
    ox[2 * N] = mid;
  }
}

// dl [T, N] fp32 -> a3 [T, 3N] bf16 = [hi | lo | hi]:  a3 @ [hi | hi | mid]^T
// = dl_hi W_hi + dl_lo W_hi + dl_hi W_mid (16-bit-mantissa accurate product).
__global__ void router_split_dl_kernel(const float* __restrict__ dl, long long n, int N,
                                       __nv_bfloat16* __restrict__ a3) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long t = i / N;
    const int e = i % N;
    const float v = dl[i];
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
    __nv_bfloat16* o = a3 + t * 3 * N + e;
    o[0] = hi;
    o[N] = lo;
    o[2 * N] = hi;
  }
}

// ------------------------------------------------------------------ router bwd
// dlogits[t, :] from
//   dtopw [T, K]           gradient of the combine weights
//   coef_z (device scalar) d(total)/d(lse_t) = coef_z * lse_t  (z-loss)
//   bal_coef [B, N]        d(total)/d(probs[t, e]) for the balance loss (per seq)
__global__ void router_bwd_kernel(const float* __restrict__ logits, const int* __restrict__ topi,
                                  const float* __restrict__ dtopw, const float* __restrict__ bal_coef,
                                  int T, int S, int N, int K, int softmax_mode, float scaling,
                                  const float* __restrict__ coef_z_ptr, float* __restrict__ dlogits) {
  const float coef_z = *coef_z_ptr;
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int EPL = (N + 31) / 32;
  for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
    float lg[8], sc[8], ds[8];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = lane + 32 * i;
      lg[i] = (i < EPL && e < N) ? logits[(long long)t * N + e] : -INFINITY;
      mx = fmaxf(mx, lg[i]);
      ds[i] = 0.f;
    }
    mx = warp_max(mx);
    float se = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < EPL && lane + 32 * i < N) se += __expf(lg[i] - mx);
    se = warp_sum(se);
    const float lse = mx + __logf(se);
    float ssum = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = lane + 32 * i;
      sc[i] = (i < EPL && e < N) ? (softmax_mode ? __expf(lg[i] - lse) : 1.f / (1.f + __expf(-lg[i]))) : 0.f;
      ssum += sc[i];
    }
    ssum = warp_sum(ssum);
    const int b = t / S;
    // balance loss through probs = s / (sum s + 1e-9)
    const float Z = ssum + 1e-9f;
    float dp[8];
    float dps = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = lane + 32 * i;
      dp[i] = (i < EPL && e < N) ? bal_coef[(long long)b * N + e] : 0.f;
      dps += dp[i] * sc[i];
    }
    dps = warp_sum(dps) / (Z * Z);
#pragma unroll
    for (int i = 0; i < 8; ++i) ds[i] += dp[i] / Z - dps;
    // combine weights w_k = s_{i_k} / (sum_j s_{i_j} + 1e-9) * scale
    float selsum = 0.f, wdot = 0.f;
    for (int k = 0; k < K; ++k) {
      const int e = topi[(long long)t * K + k];
      float s_e = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (lane + 32 * i == e) s_e = sc[i];
      s_e = warp_sum(s_e);
      selsum += s_e;
      wdot += dtopw[(long long)t * K + k] * s_e;
    }
    const float den = selsum + 1e-9f;
    const float scl = softmax_mode ? 1.f : scaling;
    for (int k = 0; k < K; ++k) {
      const int e = topi[(long long)t * K + k];
      const float dw = dtopw[(long long)t * K + k];
      const float g = scl * (dw / den - wdot / (den * den));
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (lane + 32 * i == e) ds[i] += g;
    }
    // scores -> logits
    float sdot = 0.f;
    if (softmax_mode) {
#pragma unroll
      for (int i = 0; i < 8; ++i) sdot += ds[i] * sc[i];
      sdot = warp_sum(sdot);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = lane + 32 * i;
      if (!(i < EPL && e < N)) continue;
      float dl = softmax_mode ? sc[i] * (ds[i] - sdot) : ds[i] * sc[i] * (1.f - sc[i]);
      // z-loss: d lse / d l_e = softmax_e
      dl += coef_z * lse * __expf(lg[i] - lse);
      dlogits[(long long)t * N + e] = dl;
    }
  }
}

// ------------------------------------------------------------------ router grads
// dx[t, d] (+)= sum_e dl[t, e] * W[d, e].  W is staged expert-major
// (wsh[e][d], d contiguous) so lanes read consecutive addresses; one warp per
// token, lane owns d = lane + 32 j; the token's dl row is held in registers.
__global__ void router_dx_kernel(const float* __restrict__ dl, const float* __restrict__ W,
                                 float* __restrict__ dx, int T, int D, int N, int DCH) {
  extern __shared__ float wsh[];  // [N][DCH]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
  const int tb = blockIdx.x * RT_TOK, te = min(T, tb + RT_TOK);
  const int EPL = (N + 31) / 32;
  {
    const int d0 = blockIdx.y * DCH;
    const int dn = min(DCH, D - d0);
    __syncthreads();
    for (int i = threadIdx.x; i < dn * N; i += blockDim.x) {
      const int d = i / N, e = i % N;
      wsh[e * DCH + d] = W[(long long)(d0 + d) * N + e];
    }
    __syncthreads();
    for (int t = tb + warp; t < te; t += warps) {
      float g[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) g[i] = (i < EPL && lane + 32 * i < N) ? dl[(long long)t * N + lane + 32 * i] : 0.f;
      for (int c0 = 0; c0 < dn; c0 += 128) {
        float a[4] = {0.f, 0.f, 0.f, 0.f};
        for (int e = 0; e < N; ++e) {
          const int gi = e >> 5;
          float src = g[0];
#pragma unroll
          for (int i = 1; i < 8; ++i)
            if (gi == i) src = g[i];
          const float ge = __shfl_sync(0xffffffffu, src, e & 31);
          const float* wr = wsh + e * DCH + c0;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (c0 + lane + 32 * j < dn) a[j] += ge * wr[lane + 32 * j];
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int d = d0 + c0 + lane + 32 * j;
          if (c0 + lane + 32 * j < dn) dx[(long long)t * D + d] += a[j];
        }
      }
    }
  }
}

// dW[d, e] += sum_t x[t, d] * dl[t, e]; block = 128 d x N experts, token split.
__global__ void router_dw_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ dl,
                                 float* __restrict__ dW, int T, int D, int N, int t_per_block) {
  extern __shared__ float sh[];  // xs [32][128], ds [32][N]
  float* xs = sh;
  float* ds = sh + 32 * 128;
  const int d0 = blockIdx.x * 128;
  const int tb = blockIdx.y * t_per_block, te = min(T, tb + t_per_block);
  // each thread: d = d0 + (tid % 128), experts e = tid / 128 + 2*j
  const int dl_ = threadIdx.x % 128;
  const int eo = threadIdx.x / 128;  // 0..1 for 256 threads
  float acc[MAXN / 2];
  const int EPT = (N + 1) / 2;
  for (int j = 0; j < EPT; ++j) acc[j] = 0.f;
  for (int t0 = tb; t0 < te; t0 += 32) {
    __syncthreads();
    for (int i = threadIdx.x; i < 32 * 128; i += blockDim.x) {
      const int r = i / 128, c = i % 128;
      xs[i] = (t0 + r < te && d0 + c < D) ? __bfloat162float(x[(long long)(t0 + r) * D + d0 + c]) : 0.f;
    }
    for (int i = threadIdx.x; i < 32 * N; i += blockDim.x) {
      const int r = i / N, c = i % N;
      ds[i] = (t0 + r < te) ? dl[(long long)(t0 + r) * N + c] : 0.f;
    }
    __syncthreads();
    for (int r = 0; r < 32; ++r) {
      const float xv = xs[r * 128 + dl_];
      for (int j = 0; j < EPT; ++j) {
        const int e = eo + 2 * j;
        if (e < N) acc[j] += xv * ds[r * N + e];
      }
    }
  }
  if (d0 + dl_ < D)
    for (int j = 0; j < EPT; ++j) {
      const int e = eo + 2 * j;
      if (e < N) atomicAdd(dW + (long long)(d0 + dl_) * N + e, acc[j]);
    }
}

// ------------------------------------------------------------------ plan
// A stable counting sort of the T*K slots by expert, in three kernels:
//   plan_hist    block b histograms its PLAN_CH slots -> bh[b][e], counts[e]
//   plan_scan    expert starts (128-aligned segments), GEMM tile prefix
//   plan_assign  block b: its base per expert (start + the earlier blocks'
//                counts), then per warp the rank among equal experts
//                (__match_any_sync), per-warp offsets by a scan over warps;
//                slot i goes to row base + offset + rank (slot order kept)
// Expert ids outside [0, N) are skipped and recorded as kErrBounds.
constexpr int PLAN_CH = 1024;

__global__ void plan_hist_kernel(const int* __restrict__ topi, long long n, int N, int* __restrict__ counts,
                                 int* __restrict__ bh, int* status) {
  __shared__ int h[MAXN];
  for (int i = threadIdx.x; i < N; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const long long lo = (long long)blockIdx.x * PLAN_CH, hi = min(n, lo + PLAN_CH);
  for (long long i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const int e = topi[i];
    if (e >= 0 && e < N) atomicAdd(&h[e], 1);
    else set_error(status, kErrBounds);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    bh[(long long)blockIdx.x * N + i] = h[i];
    if (h[i]) atomicAdd(counts + i, h[i]);
  }
}

// single block: starts (128-aligned), tile prefix for the grouped GEMM.
__global__ void plan_scan_kernel(const int* __restrict__ counts, int N, int align, int tiles_n,
                                 int* __restrict__ starts, int* __restrict__ tile_prefix,
                                 int* __restrict__ padded_counts, int* __restrict__ total_rows) {
  if (threadIdx.x == 0) {
    int s = 0, tp = 0;
    for (int e = 0; e < N; ++e) {
      starts[e] = s;
      tile_prefix[e] = tp;
      const int c = counts[e];
      const int pc = (c + align - 1) / align * align;
      padded_counts[e] = pc;
      s += pc;
      tp += (c + 127) / 128 * tiles_n;
    }
    tile_prefix[N] = tp;
    *total_rows = s;
  }
}

// PLAN_CH threads (32 warps) per block, one slot each.
__global__ void __launch_bounds__(PLAN_CH) plan_assign_kernel(const int* __restrict__ topi, long long n, int N,
                                                                const int* __restrict__ starts,
                                                                const int* __restrict__ bh, int* __restrict__ pos,
                                                                int* __restrict__ row_src) {
  __shared__ int wcnt[PLAN_CH / 32][MAXN];   // per warp and expert: count, then offset
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < (PLAN_CH / 32) * N; i += blockDim.x) wcnt[i / N][i % N] = 0;
  __syncthreads();
  const long long i = (long long)blockIdx.x * PLAN_CH + threadIdx.x;
  int e = i < n ? topi[i] : -1;
  if (e < 0 || e >= N) e = -1;
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  const int rank = __popc(peers & ((1u << lane) - 1));
  if (e >= 0 && rank == 0) wcnt[w][e] = __popc(peers);
  __syncthreads();
  // thread e: base of this block, then the exclusive scan over the warps
  for (int x = threadIdx.x; x < N; x += blockDim.x) {
    int base = starts[x];
    for (int b = 0; b < (int)blockIdx.x; ++b) base += bh[(long long)b * N + x];
    for (int ww = 0; ww < PLAN_CH / 32; ++ww) {
      const int c = wcnt[ww][x];
      wcnt[ww][x] = base;
      base += c;
    }
  }
  __syncthreads();
  if (e >= 0) {
    const int r = wcnt[w][e] + rank;
    pos[i] = r;
    row_src[r] = (int)i;  // slot id = t * K + k
  }
}

// xp[r, :] = x[row_src[r] / K, :] or 0 for pad rows (row_src = -1).  The
// index-consuming kernels below check every data-dependent row index
// (index_ok: out of range -> skipped, kErrBounds in the status word).
__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ x, const int* __restrict__ row_src,
                                   __nv_bfloat16* __restrict__ xp, long long R, int D, int K,
                                   long long n_tok, int* status) {
  const int vec = D / 8;  // uint4 of 8 bf16
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < R * vec;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / vec;
    const int c = i % vec;
    const int src = row_src[r];
    uint4 v = make_uint4(0, 0, 0, 0);
    if (src >= 0 && index_ok(src / K, n_tok, status))
      v = reinterpret_cast<const uint4*>(x + (long long)(src / K) * D)[c];
    reinterpret_cast<uint4*>(xp + r * D)[c] = v;
  }
}

// dx[t, :] += sum_k dxp[pos[t, k], :]   (fp32 accumulate; dxp bf16 or fp32)
HB_DEVICE float2 load2(const __nv_bfloat16* p) {
  const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(p);
  return make_float2(__bfloat162float(v.x), __bfloat162float(v.y));
}
HB_DEVICE float2 load2(const float* p) { return *reinterpret_cast<const float2*>(p); }

template <typename T_>
__global__ void scatter_add_rows_kernel(const T_* __restrict__ dxp, const int* __restrict__ pos,
                                        float* __restrict__ dx, __nv_bfloat16* __restrict__ out_b, int T,
                                        int D, int K, long long R, int* status) {
  const long long total = (long long)T * (D / 2);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long t = i / (D / 2);
    const int c = (i % (D / 2)) * 2;
    float a0 = 0.f, a1 = 0.f;
    for (int k = 0; k < K; ++k) {
      const long long r = pos[t * K + k];
      if (!index_ok(r, R, status)) continue;
      const float2 v = load2(dxp + r * D + c);
      a0 += v.x;
      a1 += v.y;
    }
    if (out_b) {   // final gradient in bf16: dx + the rows, no fp32 write
      const float2 base = *reinterpret_cast<const float2*>(dx + t * D + c);
      *reinterpret_cast<__nv_bfloat162*>(out_b + t * D + c) = __floats2bfloat162_rn(base.x + a0, base.y + a1);
    } else {
      dx[t * D + c] += a0;
      dx[t * D + c + 1] += a1;
    }
  }
}

// out[t, :] += sum_k bf16(w[t,k]) * y[pos[t,k], :]
__global__ void combine_kernel(const __nv_bfloat16* __restrict__ y, const int* __restrict__ pos,
                               const float* __restrict__ w, float* __restrict__ out, int T, int D, int K,
                               long long R, int* status) {
  const long long total = (long long)T * (D / 2);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long t = i / (D / 2);
    const int c = (i % (D / 2)) * 2;
    float a0 = 0.f, a1 = 0.f;
    for (int k = 0; k < K; ++k) {
      const long long r = pos[t * K + k];
      if (!index_ok(r, R, status)) continue;
      const float wk = __bfloat162float(__float2bfloat16_rn(w[t * K + k]));
      const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(y + r * D + c);
      a0 += wk * __bfloat162float(v.x);
      a1 += wk * __bfloat162float(v.y);
    }
    out[t * D + c] += a0;
    out[t * D + c + 1] += a1;
  }
}

// dy[pos[t,k], :] = bf16(w[t,k]) * dout[t, :];  dw[t,k] = <dout[t], y[pos[t,k]]>
// one warp per token.  Pad rows of dy are zeroed by zero_pad_rows.
__global__ void combine_bwd_kernel(const float* __restrict__ dout, const __nv_bfloat16* __restrict__ y,
                                   const int* __restrict__ pos, const float* __restrict__ w,
                                   __nv_bfloat16* __restrict__ dy, float* __restrict__ dw, int T, int D,
                                   int K, long long R, int* status) {
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
    for (int k = 0; k < K; ++k) {
      const long long r = pos[(long long)t * K + k];
      if (!index_ok(r, R, status)) {   // warp-uniform: r is the same for every lane
        if (lane == 0) dw[(long long)t * K + k] = 0.f;
        continue;
      }
      const float wk = __bfloat162float(__float2bfloat16_rn(w[(long long)t * K + k]));
      float dot = 0.f;
      for (int c = lane * 2; c < D; c += 64) {
        const float g0 = dout[(long long)t * D + c], g1 = dout[(long long)t * D + c + 1];
        const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(y + r * D + c);
        dot += g0 * __bfloat162float(v.x) + g1 * __bfloat162float(v.y);
        *reinterpret_cast<__nv_bfloat162*>(dy + r * D + c) = __floats2bfloat162_rn(wk * g0, wk * g1);
      }
      dot = warp_sum(dot);
      if (lane == 0) dw[(long long)t * K + k] = dot;
    }
  }
}

__global__ void zero_pad_rows_kernel(const int* __restrict__ row_src, __nv_bfloat16* __restrict__ a,
                                     long long R, int D) {
  const int vec = D / 8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < R * vec;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / vec;
    if (row_src[r] < 0) reinterpret_cast<uint4*>(a + r * D)[i % vec] = make_uint4(0, 0, 0, 0);
  }
}

int grid_for(long long work, int per_block) {
  long long g = (work + per_block - 1) / per_block;
  long long cap = (long long)num_sms() * 8;
  return (int)std::max(1LL, std::min(g, cap));
}

}  // namespace

// ================================================================ host API
void gemm(torch::Tensor a, torch::Tensor b, torch::Tensor c, bool trans_a, bool trans_b,
          bool accumulate, double alpha, c10::optional<torch::Tensor> alpha_t);

// The tensor-core route needs 16-byte rows for every GEMM operand.
static bool router_tc_ok(const torch::Tensor& x, int N) {
  return N % 8 == 0 && x.size(1) % 8 == 0 && x.stride(1) == 1 && x.stride(0) % 8 == 0;
}

// W [D, N] fp32 -> (w3 = [hi | mid | lo], w3x = [hi | hi | mid]) bf16 [D, 3N].
static std::pair<torch::Tensor, torch::Tensor> router_split_w(const torch::Tensor& W) {
  const int D = W.size(0), N = W.size(1);
  auto opt = W.options().dtype(torch::kBFloat16);
  auto w3 = torch::empty({D, 3 * N}, opt), w3x = torch::empty({D, 3 * N}, opt);
  const long long n = (long long)D * N;
  router_split_w_kernel<<<grid_for(n, 256), 256, 0, cur_stream()>>>(
      W.data_ptr<float>(), n, N, (__nv_bfloat16*)w3.data_ptr(), (__nv_bfloat16*)w3x.data_ptr());
  HB_CUDA_CHECK(cudaGetLastError());
  return {w3, w3x};
}

void router_fwd(torch::Tensor x, torch::Tensor W, torch::Tensor bias, int64_t S, int64_t K,
                bool softmax_mode, double scaling, torch::Tensor logits, torch::Tensor topi,
                torch::Tensor topw, torch::Tensor seq_counts, torch::Tensor seq_probs,
                torch::Tensor sums) {
  check_bf16(x, "x");
  const int T = x.size(0), D = x.size(1), N = W.size(1);
  HB_CHECK(N <= MAXN && K <= MAXK && K <= N, "router: N <= 256, K <= 16");
  HB_CHECK(W.is_contiguous() && W.scalar_type() == torch::kFloat32, "router: fp32 contiguous W");
  if (T == 0) return;
  const int grid = (T + RT_TOK - 1) / RT_TOK;
  const int epl = (N + 31) / 32;
  if (router_tc_ok(x, N)) {
    // fp32-accurate logits on the tensor cores: x @ [hi | mid | lo], summed in the select kernel
    auto w3 = router_split_w(W).first;
    auto l3 = torch::empty({T, 3 * N}, x.options().dtype(torch::kFloat32));
    gemm(x, w3, l3, false, false, false, 1.0, c10::nullopt);
    auto kern = epl == 1 ? router_select_kernel<1> : epl == 2 ? router_select_kernel<2>
              : epl <= 4 ? router_select_kernel<4> : router_select_kernel<8>;
    kern<<<grid, 256, 0, cur_stream()>>>(
        l3.data_ptr<float>(), bias.data_ptr<float>(), T, (int)S, N, (int)K, softmax_mode ? 1 : 0,
        (float)scaling, logits.data_ptr<float>(), topi.data_ptr<int>(), topw.data_ptr<float>(),
        seq_counts.data_ptr<float>(), seq_probs.data_ptr<float>(), sums.data_ptr<float>());
    HB_CUDA_CHECK(cudaGetLastError());
    return;
  }
  const int DC = std::max(32, std::min(D, (int)(RT_SMEM_W / (N * sizeof(float)))) / 32 * 32);
  const size_t smem = (size_t)(DC * N + RT_TOK * N + 2 * RT_NSEQ * N) * sizeof(float);
  auto kern = epl == 1 ? router_fwd_kernel<1> : epl == 2 ? router_fwd_kernel<2>
            : epl <= 4 ? router_fwd_kernel<4> : router_fwd_kernel<8>;
  HB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  kern<<<grid, 256, smem, cur_stream()>>>(
      (const __nv_bfloat16*)x.data_ptr(), W.data_ptr<float>(), bias.data_ptr<float>(), T, (int)S, D,
      N, (int)K, softmax_mode ? 1 : 0, (float)scaling, DC, logits.data_ptr<float>(), topi.data_ptr<int>(),
      topw.data_ptr<float>(), seq_counts.data_ptr<float>(), seq_probs.data_ptr<float>(),
      sums.data_ptr<float>());
  HB_CUDA_CHECK(cudaGetLastError());
}

void router_bwd(torch::Tensor logits, torch::Tensor topi, torch::Tensor dtopw, torch::Tensor bal_coef,
                int64_t S, bool softmax_mode, double scaling, torch::Tensor coef_z, torch::Tensor dlogits) {
  const int T = logits.size(0), N = logits.size(1), K = topi.size(1);
  if (T == 0) return;
  router_bwd_kernel<<<grid_for(T, 8), 256, 0, cur_stream()>>>(
      logits.data_ptr<float>(), topi.data_ptr<int>(), dtopw.data_ptr<float>(),
      bal_coef.data_ptr<float>(), T, (int)S, N, K, softmax_mode ? 1 : 0, (float)scaling,
      coef_z.data_ptr<float>(), dlogits.data_ptr<float>());
  HB_CUDA_CHECK(cudaGetLastError());
}

void router_grads(torch::Tensor x, torch::Tensor W, torch::Tensor dl, torch::Tensor dx, torch::Tensor dW) {
  const int T = x.size(0), D = x.size(1), N = W.size(1);
  if (T == 0) return;
  HB_CHECK(dx.scalar_type() == torch::kFloat32 && dW.scalar_type() == torch::kFloat32 &&
               dl.is_contiguous(), "router_grads: fp32 dx / dW, contiguous dl");
  if (router_tc_ok(x, N) && dx.stride(1) == 1 && dx.stride(0) % 4 == 0 && dW.is_contiguous()) {
    // dx += [dl_hi | dl_lo | dl_hi] @ [W_hi | W_hi | W_mid]^T ;  dW += x^T dl_hi + x^T dl_lo
    auto w3x = router_split_w(W).second;
    auto a3 = torch::empty({T, 3 * N}, x.options());
    const long long n = (long long)T * N;
    router_split_dl_kernel<<<grid_for(n, 256), 256, 0, cur_stream()>>>(dl.data_ptr<float>(), n, N,
                                                                      (__nv_bfloat16*)a3.data_ptr());
    HB_CUDA_CHECK(cudaGetLastError());
    gemm(a3, w3x, dx, false, true, true, 1.0, c10::nullopt);
    gemm(x, a3.narrow(1, 0, N), dW, true, false, true, 1.0, c10::nullopt);
    gemm(x, a3.narrow(1, N, N), dW, true, false, true, 1.0, c10::nullopt);
    return;
  }
  {
    static bool cfg = false;
    if (!cfg) {
      HB_CUDA_CHECK(cudaFuncSetAttribute(router_dx_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, RT_SMEM_W));
      cfg = true;
    }
    const int DCH = std::max(128, std::min(D, (int)(RT_SMEM_W / (N * sizeof(float)))) / 128 * 128);
    const dim3 grid((T + RT_TOK - 1) / RT_TOK, (D + DCH - 1) / DCH);
    router_dx_kernel<<<grid, 256, (size_t)N * DCH * 4, cur_stream()>>>(
        dl.data_ptr<float>(), W.data_ptr<float>(), dx.data_ptr<float>(), T, D, N, DCH);
    HB_CUDA_CHECK(cudaGetLastError());
  }
  {
    const int tpb = 1024;
    dim3 grid((D + 127) / 128, (T + tpb - 1) / tpb);
    const size_t smem = (32 * 128 + 32 * N) * 4;
    router_dw_kernel<<<grid, 256, smem, cur_stream()>>>((const __nv_bfloat16*)x.data_ptr(),
                                                        dl.data_ptr<float>(), dW.data_ptr<float>(), T,
                                                        D, N, tpb);
    HB_CUDA_CHECK(cudaGetLastError());
  }
}

// Returns nothing; fills counts[N], starts[N], tile_prefix[N+1], padded_counts[N],
// total_rows[1], pos[T*K], row_src[R_max] (pre-filled with -1 by the caller).
void moe_plan(torch::Tensor topi, int64_t N, int64_t tiles_n, torch::Tensor counts,
              torch::Tensor starts, torch::Tensor tile_prefix, torch::Tensor padded_counts,
              torch::Tensor total_rows, torch::Tensor pos, torch::Tensor row_src) {
  const long long n = topi.numel();
  const int K = topi.size(-1);
  HB_CHECK(N <= MAXN, "moe_plan: too many experts");
  (void)K;
  counts.zero_();
  if (n == 0) return;
  const int nblk = (int)((n + PLAN_CH - 1) / PLAN_CH);
  auto bh = torch::empty({(long long)nblk * N}, topi.options());
  plan_hist_kernel<<<nblk, 256, 0, cur_stream()>>>(topi.data_ptr<int>(), n, (int)N, counts.data_ptr<int>(),
                                                   bh.data_ptr<int>(), status_ptr());
  plan_scan_kernel<<<1, 32, 0, cur_stream()>>>(counts.data_ptr<int>(), (int)N, 128, (int)tiles_n,
                                               starts.data_ptr<int>(), tile_prefix.data_ptr<int>(),
                                               padded_counts.data_ptr<int>(), total_rows.data_ptr<int>());
  plan_assign_kernel<<<nblk, PLAN_CH, 0, cur_stream()>>>(topi.data_ptr<int>(), n, (int)N, starts.data_ptr<int>(),
                                                         bh.data_ptr<int>(), pos.data_ptr<int>(),
                                                         row_src.data_ptr<int>());
  HB_CUDA_CHECK(cudaGetLastError());
}

void moe_gather(torch::Tensor x, torch::Tensor row_src, torch::Tensor xp, int64_t K) {
  const long long R = xp.size(0);
  const int D = xp.size(1);
  HB_CHECK(D % 8 == 0, "moe_gather: D % 8");
  gather_rows_kernel<<<grid_for(R * D / 8, 256), 256, 0, cur_stream()>>>(
      (const __nv_bfloat16*)x.data_ptr(), row_src.data_ptr<int>(), (__nv_bfloat16*)xp.data_ptr(), R,
      D, (int)K, (long long)x.size(0), status_ptr());
  HB_CUDA_CHECK(cudaGetLastError());
}

// dx += rows of dxp gathered by pos; with out_b the sum goes to out_b (bf16)
// and dx is left as it was.
void moe_scatter_add(torch::Tensor dxp, torch::Tensor pos, torch::Tensor dx, c10::optional<torch::Tensor> out_b) {
  const int T = pos.size(0), K = pos.size(1), D = dx.size(1);
  HB_CHECK(D % 2 == 0 && dx.is_contiguous(), "moe_scatter_add: contiguous dx, even D");
  __nv_bfloat16* ob = nullptr;
  if (out_b.has_value()) {
    HB_CHECK(out_b->scalar_type() == at::kBFloat16 && out_b->is_contiguous() && out_b->numel() == dx.numel(),
             "moe_scatter_add: out_b like dx, bf16");
    ob = (__nv_bfloat16*)out_b->data_ptr();
  }
  if (dxp.scalar_type() == at::kFloat)
    scatter_add_rows_kernel<float><<<grid_for((long long)T * D / 2, 256), 256, 0, cur_stream()>>>(
        dxp.data_ptr<float>(), pos.data_ptr<int>(), dx.data_ptr<float>(), ob, T, D, K, (long long)dxp.size(0),
        status_ptr());
  else
    scatter_add_rows_kernel<__nv_bfloat16><<<grid_for((long long)T * D / 2, 256), 256, 0, cur_stream()>>>(
        (const __nv_bfloat16*)dxp.data_ptr(), pos.data_ptr<int>(), dx.data_ptr<float>(), ob, T, D, K,
        (long long)dxp.size(0), status_ptr());
  HB_CUDA_CHECK(cudaGetLastError());
}

void moe_combine(torch::Tensor y, torch::Tensor pos, torch::Tensor w, torch::Tensor out) {
  const int T = pos.size(0), K = pos.size(1), D = out.size(1);
  combine_kernel<<<grid_for((long long)T * D / 2, 256), 256, 0, cur_stream()>>>(
      (const __nv_bfloat16*)y.data_ptr(), pos.data_ptr<int>(), w.data_ptr<float>(), out.data_ptr<float>(),
      T, D, K, (long long)y.size(0), status_ptr());
  HB_CUDA_CHECK(cudaGetLastError());
}

void moe_combine_bwd(torch::Tensor dout, torch::Tensor y, torch::Tensor pos, torch::Tensor w,
                     torch::Tensor row_src, torch::Tensor dy, torch::Tensor dw) {
  const int T = pos.size(0), K = pos.size(1), D = dout.size(1);
  const long long R = dy.size(0);
  zero_pad_rows_kernel<<<grid_for(R * D / 8, 256), 256, 0, cur_stream()>>>(
      row_src.data_ptr<int>(), (__nv_bfloat16*)dy.data_ptr(), R, D);
  combine_bwd_kernel<<<grid_for(T, 8), 256, 0, cur_stream()>>>(
      dout.data_ptr<float>(), (const __nv_bfloat16*)y.data_ptr(), pos.data_ptr<int>(), w.data_ptr<float>(),
      (__nv_bfloat16*)dy.data_ptr(), dw.data_ptr<float>(), T, D, K, R, status_ptr());
  HB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace hb
