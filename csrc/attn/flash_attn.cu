// Causal / sliding-window GQA flash attention, forward and backward
// (model/attention.py:136-224 semantics: query i sees key j iff j <= i and,
// with a window W > 0, i - j < W; softmax in fp32; scale 1/sqrt(H)).
//
// Tiles of 64 queries x 64 keys, 4 warps (16 rows each), bf16 mma.sync
// m16n8k16 with fp32 accumulation, XOR-swizzled shared memory fed by cp.async
// (double-buffered K/V), online softmax in the exp2 domain.
//   fwd      Q-major; writes O (bf16) and the row log-sum-exp (log2 units)
//   bwd      delta = rowsum(dO * O); a KV-major kernel accumulates dK, dV over
//            all query heads of the KV group (no atomics); a Q-major kernel
//            recomputes P and dS and accumulates dQ (no atomics).
// Tiles that the causal / window mask removes entirely are skipped.
#include <torch/extension.h>

#include <cstdlib>
#include <string>

#include "../common/host.h"
#include "../common/sm100.cuh"

namespace hb {
namespace fa {

constexpr int BR = 64;
constexpr int BC = 64;
constexpr int NT = 128;
constexpr float LOG2E = 1.4426950408889634f;

HB_DEVICE void cp_async16(uint32_t dst, const void* src, bool pred) {
  const int sz = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz));
}
HB_DEVICE void cp_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
HB_DEVICE void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N)); }

HB_DEVICE void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
HB_DEVICE void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
HB_DEVICE void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Swizzled [64 rows][H] bf16 tile: 16-byte chunk c of row r lives at chunk
// c ^ (r & SWZ), SWZ = min(8, chunks per row) - 1.
template <int H>
HB_DEVICE constexpr int swz_mask() { return (H / 8 >= 8 ? 8 : H / 8) - 1; }
template <int H>
HB_DEVICE uint32_t tile_addr(uint32_t base, int r, int col) {
  const int chunk = col >> 3;
  return base + r * (H * 2) + (((chunk ^ (r & swz_mask<H>()))) << 4) + ((col & 7) << 1);
}

// Load a [64][H] tile from global rows (row stride `ld` elements) with cp.async.
template <int H>
HB_DEVICE void load_tile(uint32_t sbase, const __nv_bfloat16* g, long long ld, int rows_valid) {
  constexpr int CH = H / 8;  // 16-byte chunks per row
  for (int i = threadIdx.x; i < 64 * CH; i += NT) {
    const int r = i / CH, c = i % CH;
    const bool ok = r < rows_valid;
    const __nv_bfloat16* src = g + (long long)(ok ? r : 0) * ld + c * 8;
    cp_async16(sbase + r * (H * 2) + ((c ^ (r & swz_mask<H>())) << 4), src, ok);
  }
}

// A fragments (16 x 16 at rows r0.., cols k0..) of a row-major tile: non-trans ldmatrix.
template <int H>
HB_DEVICE void load_a(uint32_t base, int r0, int k0, uint32_t* a) {
  const int lane = threadIdx.x & 31;
  ldsm_x4(tile_addr<H>(base, r0 + (lane & 15), k0 + ((lane >> 4) << 3)), a[0], a[1], a[2], a[3]);
}
// B fragments for two n-tiles (n0.., n0+8..) with k-range k0..k0+15, where the
// smem tile stores rows = n (k contiguous): non-trans ldmatrix.
template <int H>
HB_DEVICE void load_b_nk(uint32_t base, int n0, int k0, uint32_t* b) {
  const int lane = threadIdx.x & 31;
  ldsm_x4(tile_addr<H>(base, n0 + (lane & 7) + ((lane >> 4) << 3), k0 + (((lane >> 3) & 1) << 3)),
          b[0], b[1], b[2], b[3]);
}
// B fragments for two n-tiles when the smem tile stores rows = k (n contiguous): trans ldmatrix.
template <int H>
HB_DEVICE void load_b_kn(uint32_t base, int k0, int n0, uint32_t* b) {
  const int lane = threadIdx.x & 31;
  ldsm_x4_t(tile_addr<H>(base, k0 + (lane & 7) + (((lane >> 3) & 1) << 3), n0 + ((lane >> 4) << 3)),
            b[0], b[1], b[2], b[3]);
}
// A fragments from a tile stored transposed (rows = k, cols = m): trans ldmatrix.
template <int H>
HB_DEVICE void load_a_t(uint32_t base, int m0, int k0, uint32_t* a) {
  const int lane = threadIdx.x & 31;
  // matrices: (m0..7,k0..7) (m8..15,k0..7) (m0..7,k8..15) (m8..15,k8..15)
  const int mat = lane >> 3, rr = lane & 7;
  const int krow = k0 + rr + ((mat >> 1) << 3);
  const int mcol = m0 + ((mat & 1) << 3);
  ldsm_x4_t(tile_addr<H>(base, krow, mcol), a[0], a[1], a[2], a[3]);
}

HB_DEVICE uint32_t pack2(float a, float b) { return pack_bf16x2(a, b); }

struct Params {
  const __nv_bfloat16 *q, *k, *v, *o, *dout;
  __nv_bfloat16 *out, *dq, *dk, *dv;
  float *lse, *delta;
  int B, S, Nq, Nkv, window;
  long long q_row, kv_row;  // row strides (elements) of q/o and k/v: N*H
  float scale;
};

// key range [lo, hi) of keys visible from query rows [q0, q0+64)
HB_DEVICE void kv_range(const Params& p, int q0, int& lo, int& hi) {
  hi = min(p.S, q0 + BR);
  lo = 0;
  if (p.window > 0) lo = max(0, q0 - p.window + 1);
}
// query range [lo, hi) that sees keys [k0, k0+64)
HB_DEVICE void q_range(const Params& p, int k0, int& lo, int& hi) {
  lo = k0;
  hi = p.S;
  if (p.window > 0) hi = min(p.S, k0 + BC - 1 + p.window);
}
HB_DEVICE bool visible(const Params& p, int qi, int kj) {
  return kj <= qi && (p.window <= 0 || qi - kj < p.window) && kj < p.S && qi < p.S;
}

// ============================================================== forward
template <int H>
__global__ void __launch_bounds__(NT) fwd_kernel(Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + 64 * H * 2;
  const uint32_t sV0 = sK0 + 2 * 64 * H * 2;
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Nq / p.Nkv);
  const int q0 = qb * BR;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const __nv_bfloat16* qg = p.q + ((long long)b * p.S + q0) * p.q_row + h * H;
  const __nv_bfloat16* kg = p.k + (long long)b * p.S * p.kv_row + hk * H;
  const __nv_bfloat16* vg = p.v + (long long)b * p.S * p.kv_row + hk * H;
  int lo, hi;
  kv_range(p, q0, lo, hi);
  const int jb0 = lo / BC, jb1 = (hi + BC - 1) / BC;
  load_tile<H>(sQ, qg, p.q_row, p.S - q0);
  cp_commit();
  load_tile<H>(sK0, kg + (long long)jb0 * BC * p.kv_row, p.kv_row, p.S - jb0 * BC);
  load_tile<H>(sV0, vg + (long long)jb0 * BC * p.kv_row, p.kv_row, p.S - jb0 * BC);
  cp_commit();
  cp_wait<1>();
  __syncthreads();
  uint32_t qf[H / 16][4];
#pragma unroll
  for (int kk = 0; kk < H / 16; ++kk) load_a<H>(sQ, warp * 16, kk * 16, qf[kk]);
  float acc[H / 8][4];
#pragma unroll
  for (int i = 0; i < H / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  float m_i[2] = {-INFINITY, -INFINITY}, l_i[2] = {0.f, 0.f};
  const float sl2 = p.scale * LOG2E;
  const int row_a = q0 + warp * 16 + (lane >> 2);
  for (int jb = jb0; jb < jb1; ++jb) {
    const int buf = (jb - jb0) & 1;
    const uint32_t sK = sK0 + buf * 64 * H * 2, sV = sV0 + buf * 64 * H * 2;
    if (jb + 1 < jb1) {
      const int nb = buf ^ 1;
      load_tile<H>(sK0 + nb * 64 * H * 2, kg + (long long)(jb + 1) * BC * p.kv_row, p.kv_row, p.S - (jb + 1) * BC);
      load_tile<H>(sV0 + nb * 64 * H * 2, vg + (long long)(jb + 1) * BC * p.kv_row, p.kv_row, p.S - (jb + 1) * BC);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < H / 16; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bb[4];
        load_b_nk<H>(sK, np * 16, kk * 16, bb);
        mma16816(s[2 * np], qf[kk], bb[0], bb[1]);
        mma16816(s[2 * np + 1], qf[kk], bb[2], bb[3]);
      }
    }
    // mask + scale
    const int k0 = jb * BC;
    const bool need_mask = (k0 + BC > q0) || (p.window > 0) || (k0 + BC > p.S);
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi = row_a + ((e >> 1) << 3);
        const int kj = k0 + n * 8 + ((lane & 3) << 1) + (e & 1);
        float v = s[n][e] * sl2;
        if (need_mask && !visible(p, qi, kj)) v = -INFINITY;
        s[n][e] = v;
      }
    // online softmax (rows r and r+8)
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float mx = m_i[r];
#pragma unroll
      for (int n = 0; n < 8; ++n) mx = fmaxf(mx, fmaxf(s[n][2 * r], s[n][2 * r + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mref = (mx == -INFINITY) ? 0.f : mx;
      const float alpha = exp2f(m_i[r] - mref);
      float rs = 0.f;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        s[n][2 * r] = exp2f(s[n][2 * r] - mref);
        s[n][2 * r + 1] = exp2f(s[n][2 * r + 1] - mref);
        rs += s[n][2 * r] + s[n][2 * r + 1];
      }
      rs += __shfl_xor_sync(0xffffffffu, rs, 1);
      rs += __shfl_xor_sync(0xffffffffu, rs, 2);
      l_i[r] = l_i[r] * alpha + rs;
      m_i[r] = mx;
#pragma unroll
      for (int i = 0; i < H / 8; ++i) {
        acc[i][2 * r] *= alpha;
        acc[i][2 * r + 1] *= alpha;
      }
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4];
      a[0] = pack2(s[2 * kk][0], s[2 * kk][1]);
      a[1] = pack2(s[2 * kk][2], s[2 * kk][3]);
      a[2] = pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = pack2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < H / 16; ++np) {
        uint32_t bb[4];
        load_b_kn<H>(sV, kk * 16, np * 16, bb);
        mma16816(acc[2 * np], a, bb[0], bb[1]);
        mma16816(acc[2 * np + 1], a, bb[2], bb[3]);
      }
    }
    __syncthreads();
  }
  // epilogue
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = row_a + r * 8;
    if (qi >= p.S) continue;
    const float inv = l_i[r] > 0.f ? 1.f / l_i[r] : 0.f;
    __nv_bfloat16* og = p.out + ((long long)b * p.S + qi) * p.q_row + h * H;
#pragma unroll
    for (int i = 0; i < H / 8; ++i) {
      const int c = i * 8 + ((lane & 3) << 1);
      *reinterpret_cast<uint32_t*>(og + c) = pack2(acc[i][2 * r] * inv, acc[i][2 * r + 1] * inv);
    }
    if ((lane & 3) == 0)
      p.lse[((long long)b * p.Nq + h) * p.S + qi] = (l_i[r] > 0.f) ? m_i[r] + log2f(l_i[r]) : INFINITY;
  }
}

// ============================================================== backward: delta
template <int H>
__global__ void delta_kernel(Params p) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const long long rows = (long long)p.B * p.S * p.Nq;
  for (long long r = blockIdx.x * (long long)warps + (threadIdx.x >> 5); r < rows;
       r += (long long)gridDim.x * warps) {
    const long long bs = r / p.Nq;
    const int h = r % p.Nq;
    const __nv_bfloat16* o = p.o + bs * p.q_row + h * H;
    const __nv_bfloat16* d = p.dout + bs * p.q_row + h * H;
    float acc = 0.f;
    for (int c = lane; c < H; c += 32) acc += __bfloat162float(o[c]) * __bfloat162float(d[c]);
    acc = warp_sum(acc);
    if (lane == 0) {
      const long long b = bs / p.S, s = bs % p.S;
      p.delta[(b * p.Nq + h) * p.S + s] = acc;
    }
  }
}

// ============================================================== backward: dK dV
template <int H>
__global__ void __launch_bounds__(NT) bwd_dkdv_kernel(Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sK = smem_u32(smem);
  const uint32_t sV = sK + 64 * H * 2;
  const uint32_t sQ0 = sV + 64 * H * 2;           // 2 buffers
  const uint32_t sD0 = sQ0 + 2 * 64 * H * 2;      // 2 buffers (dO)
  float* sLse = reinterpret_cast<float*>(smem + 6 * 64 * H * 2);  // 2 x 64
  float* sDel = sLse + 128;                                        // 2 x 64
  const int kb = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int k0 = kb * BC;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rep = p.Nq / p.Nkv;
  const __nv_bfloat16* kg = p.k + ((long long)b * p.S + k0) * p.kv_row + hk * H;
  const __nv_bfloat16* vg = p.v + ((long long)b * p.S + k0) * p.kv_row + hk * H;
  load_tile<H>(sK, kg, p.kv_row, p.S - k0);
  load_tile<H>(sV, vg, p.kv_row, p.S - k0);
  cp_commit();
  int qlo, qhi;
  q_range(p, k0, qlo, qhi);
  const int ib0 = qlo / BR, ib1 = (qhi + BR - 1) / BR;
  const int nq = ib1 - ib0;
  const int total = nq * rep;
  auto issue = [&](int it, int buf) {
    const int hq = hk * rep + it / nq;
    const int ib = ib0 + it % nq;
    const int q0 = ib * BR;
    const __nv_bfloat16* qg = p.q + ((long long)b * p.S + q0) * p.q_row + hq * H;
    const __nv_bfloat16* dg = p.dout + ((long long)b * p.S + q0) * p.q_row + hq * H;
    load_tile<H>(sQ0 + buf * 64 * H * 2, qg, p.q_row, p.S - q0);
    load_tile<H>(sD0 + buf * 64 * H * 2, dg, p.q_row, p.S - q0);
    for (int i = threadIdx.x; i < 64; i += NT) {
      const long long idx = ((long long)b * p.Nq + hq) * p.S + q0 + i;
      const bool ok = q0 + i < p.S;
      sLse[buf * 64 + i] = ok ? p.lse[idx] : INFINITY;
      sDel[buf * 64 + i] = ok ? p.delta[idx] : 0.f;
    }
  };
  if (total > 0) issue(0, 0);
  cp_commit();
  cp_wait<1>();
  __syncthreads();
  uint32_t kf[H / 16][4], vf[H / 16][4];
#pragma unroll
  for (int kk = 0; kk < H / 16; ++kk) {
    load_a<H>(sK, warp * 16, kk * 16, kf[kk]);
    load_a<H>(sV, warp * 16, kk * 16, vf[kk]);
  }
  float dk[H / 8][4], dv[H / 8][4];
#pragma unroll
  for (int i = 0; i < H / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;
  const float sl2 = p.scale * LOG2E;
  const int key_a = k0 + warp * 16 + (lane >> 2);
  for (int it = 0; it < total; ++it) {
    const int buf = it & 1;
    __syncthreads();  // previous consumers of buf^1 are done
    if (it + 1 < total) {
      issue(it + 1, buf ^ 1);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const uint32_t sQ = sQ0 + buf * 64 * H * 2, sD = sD0 + buf * 64 * H * 2;
    const float* lse = sLse + buf * 64;
    const float* del = sDel + buf * 64;
    const int q0 = (ib0 + it % nq) * BR;
    // S^T = K Q^T  (16 keys x 64 queries per warp)
    float st[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) st[n][0] = st[n][1] = st[n][2] = st[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < H / 16; ++kk)
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bb[4];
        load_b_nk<H>(sQ, np * 16, kk * 16, bb);
        mma16816(st[2 * np], kf[kk], bb[0], bb[1]);
        mma16816(st[2 * np + 1], kf[kk], bb[2], bb[3]);
      }
    // P^T
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kj = key_a + ((e >> 1) << 3);
        const int ql = n * 8 + ((lane & 3) << 1) + (e & 1);
        const int qi = q0 + ql;
        float pv = exp2f(st[n][e] * sl2 - lse[ql]);
        if (!visible(p, qi, kj)) pv = 0.f;
        st[n][e] = pv;
      }
    // dV += P^T dO
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4];
      a[0] = pack2(st[2 * kk][0], st[2 * kk][1]);
      a[1] = pack2(st[2 * kk][2], st[2 * kk][3]);
      a[2] = pack2(st[2 * kk + 1][0], st[2 * kk + 1][1]);
      a[3] = pack2(st[2 * kk + 1][2], st[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < H / 16; ++np) {
        uint32_t bb[4];
        load_b_kn<H>(sD, kk * 16, np * 16, bb);
        mma16816(dv[2 * np], a, bb[0], bb[1]);
        mma16816(dv[2 * np + 1], a, bb[2], bb[3]);
      }
    }
    // dP^T = V dO^T
    float dpt[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) dpt[n][0] = dpt[n][1] = dpt[n][2] = dpt[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < H / 16; ++kk)
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bb[4];
        load_b_nk<H>(sD, np * 16, kk * 16, bb);
        mma16816(dpt[2 * np], vf[kk], bb[0], bb[1]);
        mma16816(dpt[2 * np + 1], vf[kk], bb[2], bb[3]);
      }
    // dS^T = P^T * (dP^T - delta)
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ql = n * 8 + ((lane & 3) << 1) + (e & 1);
        dpt[n][e] = st[n][e] * (dpt[n][e] - del[ql]);
      }
    // dK += dS^T Q
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4];
      a[0] = pack2(dpt[2 * kk][0], dpt[2 * kk][1]);
      a[1] = pack2(dpt[2 * kk][2], dpt[2 * kk][3]);
      a[2] = pack2(dpt[2 * kk + 1][0], dpt[2 * kk + 1][1]);
      a[3] = pack2(dpt[2 * kk + 1][2], dpt[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < H / 16; ++np) {
        uint32_t bb[4];
        load_b_kn<H>(sQ, kk * 16, np * 16, bb);
        mma16816(dk[2 * np], a, bb[0], bb[1]);
        mma16816(dk[2 * np + 1], a, bb[2], bb[3]);
      }
    }
  }
  // store dK * scale, dV
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int kj = key_a + r * 8;
    if (kj >= p.S) continue;
    __nv_bfloat16* dkg = p.dk + ((long long)b * p.S + kj) * p.kv_row + hk * H;
    __nv_bfloat16* dvg = p.dv + ((long long)b * p.S + kj) * p.kv_row + hk * H;
#pragma unroll
    for (int i = 0; i < H / 8; ++i) {
      const int c = i * 8 + ((lane & 3) << 1);
      *reinterpret_cast<uint32_t*>(dkg + c) = pack2(dk[i][2 * r] * p.scale, dk[i][2 * r + 1] * p.scale);
      *reinterpret_cast<uint32_t*>(dvg + c) = pack2(dv[i][2 * r], dv[i][2 * r + 1]);
    }
  }
}

// ============================================================== backward: dQ
template <int H>
__global__ void __launch_bounds__(NT) bwd_dq_kernel(Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sDo = sQ + 64 * H * 2;
  const uint32_t sK0 = sDo + 64 * H * 2;
  const uint32_t sV0 = sK0 + 2 * 64 * H * 2;
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Nq / p.Nkv);
  const int q0 = qb * BR;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const __nv_bfloat16* qg = p.q + ((long long)b * p.S + q0) * p.q_row + h * H;
  const __nv_bfloat16* dg = p.dout + ((long long)b * p.S + q0) * p.q_row + h * H;
  const __nv_bfloat16* kg = p.k + (long long)b * p.S * p.kv_row + hk * H;
  const __nv_bfloat16* vg = p.v + (long long)b * p.S * p.kv_row + hk * H;
  int lo, hi;
  kv_range(p, q0, lo, hi);
  const int jb0 = lo / BC, jb1 = (hi + BC - 1) / BC;
  load_tile<H>(sQ, qg, p.q_row, p.S - q0);
  load_tile<H>(sDo, dg, p.q_row, p.S - q0);
  cp_commit();
  load_tile<H>(sK0, kg + (long long)jb0 * BC * p.kv_row, p.kv_row, p.S - jb0 * BC);
  load_tile<H>(sV0, vg + (long long)jb0 * BC * p.kv_row, p.kv_row, p.S - jb0 * BC);
  cp_commit();
  cp_wait<1>();
  __syncthreads();
  uint32_t qf[H / 16][4], df[H / 16][4];
#pragma unroll
  for (int kk = 0; kk < H / 16; ++kk) {
    load_a<H>(sQ, warp * 16, kk * 16, qf[kk]);
    load_a<H>(sDo, warp * 16, kk * 16, df[kk]);
  }
  const int row_a = q0 + warp * 16 + (lane >> 2);
  float lse[2], del[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = row_a + r * 8;
    const long long idx = ((long long)b * p.Nq + h) * p.S + qi;
    lse[r] = qi < p.S ? p.lse[idx] : INFINITY;
    del[r] = qi < p.S ? p.delta[idx] : 0.f;
  }
  float dq[H / 8][4];
#pragma unroll
  for (int i = 0; i < H / 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
  const float sl2 = p.scale * LOG2E;
  for (int jb = jb0; jb < jb1; ++jb) {
    const int buf = (jb - jb0) & 1;
    const uint32_t sK = sK0 + buf * 64 * H * 2, sV = sV0 + buf * 64 * H * 2;
    if (jb + 1 < jb1) {
      const int nb = buf ^ 1;
      load_tile<H>(sK0 + nb * 64 * H * 2, kg + (long long)(jb + 1) * BC * p.kv_row, p.kv_row, p.S - (jb + 1) * BC);
      load_tile<H>(sV0 + nb * 64 * H * 2, vg + (long long)(jb + 1) * BC * p.kv_row, p.kv_row, p.S - (jb + 1) * BC);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    float s[8][4], dp[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[n][e] = dp[n][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < H / 16; ++kk)
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bb[4];
        load_b_nk<H>(sK, np * 16, kk * 16, bb);
        mma16816(s[2 * np], qf[kk], bb[0], bb[1]);
        mma16816(s[2 * np + 1], qf[kk], bb[2], bb[3]);
        load_b_nk<H>(sV, np * 16, kk * 16, bb);
        mma16816(dp[2 * np], df[kk], bb[0], bb[1]);
        mma16816(dp[2 * np + 1], df[kk], bb[2], bb[3]);
      }
    const int k0 = jb * BC;
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = e >> 1;
        const int qi = row_a + r * 8;
        const int kj = k0 + n * 8 + ((lane & 3) << 1) + (e & 1);
        float pv = exp2f(s[n][e] * sl2 - lse[r]);
        if (!visible(p, qi, kj)) pv = 0.f;
        s[n][e] = pv * (dp[n][e] - del[r]);  // dS
      }
    // dQ += dS K
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4];
      a[0] = pack2(s[2 * kk][0], s[2 * kk][1]);
      a[1] = pack2(s[2 * kk][2], s[2 * kk][3]);
      a[2] = pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = pack2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < H / 16; ++np) {
        uint32_t bb[4];
        load_b_kn<H>(sK, kk * 16, np * 16, bb);
        mma16816(dq[2 * np], a, bb[0], bb[1]);
        mma16816(dq[2 * np + 1], a, bb[2], bb[3]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = row_a + r * 8;
    if (qi >= p.S) continue;
    __nv_bfloat16* dqg = p.dq + ((long long)b * p.S + qi) * p.q_row + h * H;
#pragma unroll
    for (int i = 0; i < H / 8; ++i) {
      const int c = i * 8 + ((lane & 3) << 1);
      *reinterpret_cast<uint32_t*>(dqg + c) = pack2(dq[i][2 * r] * p.scale, dq[i][2 * r + 1] * p.scale);
    }
  }
}

template <int H>
void set_smem(const void* k, int bytes) {
  HB_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

}  // namespace fa

using fa::Params;

static Params make_params(const torch::Tensor& q, const torch::Tensor& k, int64_t window) {
  Params p{};
  p.B = q.size(0);
  p.S = q.size(1);
  p.Nq = q.size(2);
  p.Nkv = k.size(2);
  p.window = (int)window;
  p.q_row = (long long)q.size(2) * q.size(3);
  p.kv_row = (long long)k.size(2) * k.size(3);
  p.scale = 1.f / std::sqrt((float)q.size(3));
  return p;
}

static void check_qkv(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v) {
  check_bf16(q, "q");
  check_bf16(k, "k");
  check_bf16(v, "v");
  HB_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous(), "attention: contiguous [B,S,N,H]");
  HB_CHECK(q.dim() == 4 && k.dim() == 4 && q.size(3) == k.size(3), "attention: [B,S,N,H]");
  HB_CHECK(q.size(2) % k.size(2) == 0, "attention: Nq must be a multiple of Nkv");
  HB_CHECK(q.size(3) == 32 || q.size(3) == 64 || q.size(3) == 128, "attention: head_dim 32, 64 or 128");
}

// q [B,S,Nq,H], k/v [B,S,Nkv,H] -> out [B,S,Nq,H], lse [B,Nq,S] (log2 units)
void flash_fwd_tc(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor lse,
                  int64_t window);
void flash_bwd_kv_tc(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor dout, torch::Tensor lse,
                     torch::Tensor delta, torch::Tensor dk, torch::Tensor dv, int64_t window);
void flash_bwd_q_tc(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor dout, torch::Tensor lse,
                    torch::Tensor delta, torch::Tensor dq, int64_t window);

// Head dims 64 and 128 run on the tcgen05 kernels (flash_tc.cu: forward, dK /
// dV and dQ of the backward) unless HB_FA_TC=0; head dim 32 and HB_FA_TC=0 on
// the mma.sync kernels of this file.
static bool use_fwd_tc(int H) {
  static const bool on = [] {
    const char* e = std::getenv("HB_FA_TC");
    return !(e && std::string(e) == "0");
  }();
  return on && (H == 64 || H == 128);
}

void flash_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor lse,
               int64_t window) {
  check_qkv(q, k, v);
  if (use_fwd_tc(q.size(3))) {
    flash_fwd_tc(q, k, v, out, lse, window);
    return;
  }
  Params p = make_params(q, k, window);
  p.q = (const __nv_bfloat16*)q.data_ptr();
  p.k = (const __nv_bfloat16*)k.data_ptr();
  p.v = (const __nv_bfloat16*)v.data_ptr();
  p.out = (__nv_bfloat16*)out.data_ptr();
  p.lse = lse.data_ptr<float>();
  dim3 grid((p.S + fa::BR - 1) / fa::BR, p.Nq, p.B);
  const int H = q.size(3);
  const int smem = 5 * 64 * H * 2;
  if (H == 32) {
    static bool c = false;
    if (!c) { fa::set_smem<32>((const void*)fa::fwd_kernel<32>, smem); c = true; }
    fa::fwd_kernel<32><<<grid, fa::NT, smem, cur_stream()>>>(p);
  } else if (H == 64) {
    static bool c = false;
    if (!c) { fa::set_smem<64>((const void*)fa::fwd_kernel<64>, smem); c = true; }
    fa::fwd_kernel<64><<<grid, fa::NT, smem, cur_stream()>>>(p);
  } else {
    static bool c = false;
    if (!c) { fa::set_smem<128>((const void*)fa::fwd_kernel<128>, smem); c = true; }
    fa::fwd_kernel<128><<<grid, fa::NT, smem, cur_stream()>>>(p);
  }
  HB_CUDA_CHECK(cudaGetLastError());
}

void flash_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor dout,
               torch::Tensor lse, torch::Tensor delta, torch::Tensor dq, torch::Tensor dk, torch::Tensor dv,
               int64_t window) {
  check_qkv(q, k, v);
  HB_CHECK(dout.is_contiguous() && out.is_contiguous(), "attention bwd: contiguous O/dO");
  Params p = make_params(q, k, window);
  p.q = (const __nv_bfloat16*)q.data_ptr();
  p.k = (const __nv_bfloat16*)k.data_ptr();
  p.v = (const __nv_bfloat16*)v.data_ptr();
  p.o = (const __nv_bfloat16*)out.data_ptr();
  p.dout = (const __nv_bfloat16*)dout.data_ptr();
  p.dq = (__nv_bfloat16*)dq.data_ptr();
  p.dk = (__nv_bfloat16*)dk.data_ptr();
  p.dv = (__nv_bfloat16*)dv.data_ptr();
  p.lse = lse.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  const int H = q.size(3);
  const long long rows = (long long)p.B * p.S * p.Nq;
  const int dgrid = (int)std::min<long long>((rows + 7) / 8, num_sms() * 16);
  if (H == 32) fa::delta_kernel<32><<<dgrid, 256, 0, cur_stream()>>>(p);
  else if (H == 64) fa::delta_kernel<64><<<dgrid, 256, 0, cur_stream()>>>(p);
  else fa::delta_kernel<128><<<dgrid, 256, 0, cur_stream()>>>(p);
  HB_CUDA_CHECK(cudaGetLastError());
  const int smem_kv = 6 * 64 * H * 2 + 4 * 64 * 4;
  const int smem_q = 6 * 64 * H * 2;
  dim3 gkv((p.S + fa::BC - 1) / fa::BC, p.Nkv, p.B);
  dim3 gq((p.S + fa::BR - 1) / fa::BR, p.Nq, p.B);
  if (H == 32) {
    static bool c = false;
    if (!c) {
      fa::set_smem<32>((const void*)fa::bwd_dkdv_kernel<32>, smem_kv);
      fa::set_smem<32>((const void*)fa::bwd_dq_kernel<32>, smem_q);
      c = true;
    }
    fa::bwd_dkdv_kernel<32><<<gkv, fa::NT, smem_kv, cur_stream()>>>(p);
    fa::bwd_dq_kernel<32><<<gq, fa::NT, smem_q, cur_stream()>>>(p);
  } else if (H == 64) {
    static bool c = false;
    if (!c) {
      fa::set_smem<64>((const void*)fa::bwd_dkdv_kernel<64>, smem_kv);
      fa::set_smem<64>((const void*)fa::bwd_dq_kernel<64>, smem_q);
      c = true;
    }
    if (use_fwd_tc(64)) {   // dK / dV and dQ on tcgen05 (flash_tc.cu)
      flash_bwd_kv_tc(q, k, v, dout, lse, delta, dk, dv, window);
      flash_bwd_q_tc(q, k, v, dout, lse, delta, dq, window);
    } else {
      fa::bwd_dkdv_kernel<64><<<gkv, fa::NT, smem_kv, cur_stream()>>>(p);
      fa::bwd_dq_kernel<64><<<gq, fa::NT, smem_q, cur_stream()>>>(p);
    }
  } else {
    static bool c = false;
    if (!c) {
      fa::set_smem<128>((const void*)fa::bwd_dkdv_kernel<128>, smem_kv);
      fa::set_smem<128>((const void*)fa::bwd_dq_kernel<128>, smem_q);
      c = true;
    }
    if (use_fwd_tc(128)) {
      flash_bwd_kv_tc(q, k, v, dout, lse, delta, dk, dv, window);
      flash_bwd_q_tc(q, k, v, dout, lse, delta, dq, window);
    } else {
      fa::bwd_dkdv_kernel<128><<<gkv, fa::NT, smem_kv, cur_stream()>>>(p);
      fa::bwd_dq_kernel<128><<<gq, fa::NT, smem_q, cur_stream()>>>(p);
    }
  }
  HB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace hb
