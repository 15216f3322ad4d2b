// Chunk-parallel products of the chunk-64 KDA backward on the 5th-generation
// tensor cores (tcgen05 + TMEM), fp32 accurate.
//
// Each CTA handles one chunk (64 tokens of one head) and computes two 64x64
// products that share their B operand, as ONE M = 128 MMA:
//
//     [C_top; C_bot] (128 x 64) = [A_top; A_bot] (128 x 64) . B (64 x 64)
//
//   bwd_pre      A = [P^T ; Qg^T] (MN-major), B = dO  (MN-major)
//                -> dUp = P^T dO,  dSq = Qg^T dO
//   products_u   A = [dU ; dO]    (K-major),  B = S0^T (K-major)
//                -> dWt = -dU S0^T, dQg = dO S0^T
//   products_s   A = [dO ; dS]    (K-major),  B = U^T  (K-major)
//                -> dP = dO U^T,   dKh = (dS U^T)^T;  and dgC = rowsum(dS * S0)
//
// Operands are fp32 [64 x 64] tiles loaded by TMA (two 32-column boxes with
// 128-byte swizzle, the canonical tcgen05 tile layout; rows past the sequence
// read as zeros).  fp32 accuracy with kind::tf32: every operand is split in
// place into hi = x with the low 13 mantissa bits cleared and lo = x - hi (both
// exact), and the product is hi.hi + hi.lo + lo.hi (three MMAs per K step of
// 8), accumulated in fp32 in TMEM.  One elected thread issues the MMAs; the
// four warps read the 128 x 64 accumulator back with tcgen05.ld (warp w owns
// TMEM lanes 32w..32w+31 = output rows) and store it.  Every wait is bounded
// (status word), and TMEM is freed on every path.
#include <torch/extension.h>

#include "../common/host.h"
#include "../common/sm100.cuh"
#include "kda_common.cuh"

namespace hb {
namespace kda64tc {

constexpr int THREADS = 128;
constexpr int ATOM = 8192;                 // one 32-column x 64-row fp32 box (128 B rows)
constexpr int A_BYTES = 4 * ATOM;          // 128 x 64 fp32
constexpr int B_BYTES = 2 * ATOM;          // 64 x 64 fp32
constexpr int SMEM = 2 * (A_BYTES + B_BYTES) + 1024 + 64;  // hi + lo regions, align, barriers
constexpr int TMEM_COLS = 64;

// Instruction descriptor, kind::tf32: D fp32, A / B tf32, M = 128, N = 64.
__host__ __device__ constexpr uint32_t idesc_tf32(bool a_mn, bool b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(64 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

HB_DEVICE void umma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// Where a tile comes from: chunk layout [B, H, NC, 64, 64] (2-D map over rows
// of 64 floats) or token layout [B, S, H * 64] (3-D map; rows past S are zeros).
enum : int { kChunk = 0, kToken = 1 };

struct Args {
  int S, H, NC;
  float* out_top;       // [B, H, NC, 64, 64]
  float* out_bot;
  float alpha_top, alpha_bot;
  int kind_top, kind_bot, kind_b;
  int bot_transposed;   // store C_bot^T
  const float* dS;      // optional: dgC = rowsum(dS * S0) per chunk
  const float* S0;
  float* dgC;           // [B, H, NC, 64]
  int* status;
  unsigned long long budget_ns;
};

HB_DEVICE void load_box(uint32_t dst, const CUtensorMap* m, uint32_t bar, int kind, int col, int c,
                        int n, int h, int b) {
  if (kind == kChunk) tma_load_2d(dst, m, bar, col, c * 64);
  else tma_load_3d(dst, m, bar, h * 64 + col, n * 64, b);
}

// K-major (canonical, 128-byte swizzle) descriptor: rows of 128 B, 8-row groups
// 1024 B apart; a K step of 8 fp32 advances 32 B inside the swizzle atom.
HB_DEVICE uint64_t desc_kmajor(uint32_t base, int rows, int kk) {
  return make_smem_desc(base + (kk >> 2) * rows * 128 + (kk & 3) * 32, 16, 1024);
}
// MN-major: 32-element MN atoms of [64 K rows x 128 B] (8 KB apart); a K step
// of 8 rows advances 1024 B.
HB_DEVICE uint64_t desc_mnmajor(uint32_t base, int kk) { return make_smem_desc(base + kk * 1024, ATOM, 1024); }

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(THREADS, 2)
    pair_product_kernel(const __grid_constant__ CUtensorMap tmTop, const __grid_constant__ CUtensorMap tmBot,
                        const __grid_constant__ CUtensorMap tmB, const Args p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sA = smem_u32(smem);
  const uint32_t sB = sA + A_BYTES;
  const uint32_t sAlo = sB + B_BYTES;
  const uint32_t sBlo = sAlo + A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 2 * (A_BYTES + B_BYTES));
  uint64_t* full = bars;
  uint64_t* done = bars + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  volatile int* go_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  const int n = c % p.NC, h = (c / p.NC) % p.H, b = c / (p.NC * p.H);

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(full), 1);
    mbar_init(smem_u32(done), 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // ---- TMA: A_top, A_bot, B (two 32-column boxes each)
  if (threadIdx.x == 0) {
    mbar_expect_tx(smem_u32(full), A_BYTES + B_BYTES);
    for (int a = 0; a < 2; ++a) {
      // K-major A: [k atom][128 rows]; MN-major A: [m atom][64 k rows]
      const uint32_t top = A_MN ? sA + a * ATOM : sA + a * 2 * ATOM;
      const uint32_t bot = A_MN ? sA + (2 + a) * ATOM : sA + a * 2 * ATOM + ATOM;
      load_box(top, &tmTop, smem_u32(full), p.kind_top, 32 * a, c, n, h, b);
      load_box(bot, &tmBot, smem_u32(full), p.kind_bot, 32 * a, c, n, h, b);
      load_box(sB + a * ATOM, &tmB, smem_u32(full), p.kind_b, 32 * a, c, n, h, b);
    }
  }
  bool ok = mbar_wait(smem_u32(full), 0, p.status, kErrTimeoutProducer, p.budget_ns);
  if (!ok) mbar_wait(smem_u32(full), 0, nullptr, 0, p.budget_ns);  // copies still in flight
  // ---- hi / lo split in place (elementwise: the swizzle does not matter)
  if (ok) {
    float4* hi = reinterpret_cast<float4*>(smem);
    float4* lo = reinterpret_cast<float4*>(smem + A_BYTES + B_BYTES);
    for (int i = threadIdx.x; i < (A_BYTES + B_BYTES) / 16; i += THREADS) {
      float4 x = hi[i];
      float4 hv, lv;
      hv.x = __uint_as_float(__float_as_uint(x.x) & 0xffffe000u);
      hv.y = __uint_as_float(__float_as_uint(x.y) & 0xffffe000u);
      hv.z = __uint_as_float(__float_as_uint(x.z) & 0xffffe000u);
      hv.w = __uint_as_float(__float_as_uint(x.w) & 0xffffe000u);
      lv = make_float4(x.x - hv.x, x.y - hv.y, x.z - hv.z, x.w - hv.w);
      hi[i] = hv;
      lo[i] = lv;
    }
    fence_proxy_async();   // generic-proxy smem writes -> visible to the tensor core
  }
  // one decision for the whole CTA: thread 0's view of its loads and the status
  if (threadIdx.x == 0) *go_flag = (ok && *reinterpret_cast<volatile int*>(p.status) == 0) ? 1 : 0;
  __syncthreads();
  const bool go = *go_flag != 0;
  // ---- MMAs: 8 K steps x (hi.hi + hi.lo + lo.hi)
  if (go && threadIdx.x == 0) {
    tc_fence_after();
    constexpr uint32_t idesc = idesc_tf32(A_MN, B_MN);
    for (int kk = 0; kk < 8; ++kk) {
      const uint64_t ah = A_MN ? desc_mnmajor(sA, kk) : desc_kmajor(sA, 128, kk);
      const uint64_t al = A_MN ? desc_mnmajor(sAlo, kk) : desc_kmajor(sAlo, 128, kk);
      const uint64_t bh = B_MN ? desc_mnmajor(sB, kk) : desc_kmajor(sB, 64, kk);
      const uint64_t bl = B_MN ? desc_mnmajor(sBlo, kk) : desc_kmajor(sBlo, 64, kk);
      umma_tf32(tmem, ah, bh, idesc, kk > 0 ? 1u : 0u);
      umma_tf32(tmem, ah, bl, idesc, 1u);
      umma_tf32(tmem, al, bh, idesc, 1u);
    }
    umma_commit(smem_u32(done));
  }
  ok = go;
  if (go) {
    ok = mbar_wait(smem_u32(done), 0, p.status, kErrTimeoutMma, p.budget_ns);
    if (!ok) mbar_wait(smem_u32(done), 0, nullptr, 0, p.budget_ns);  // MMAs still in flight
  }
  tc_fence_after();
  // ---- epilogue: row r = 32 warp + lane of the 128 x 64 accumulator
  if (ok) {
    const long long co = (long long)c * 64 * 64;
    const int r = 32 * warp + lane;
    const bool top = r < 64;
    const int rr = top ? r : r - 64;
    const float alpha = top ? p.alpha_top : p.alpha_bot;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(tmem + ((uint32_t)(32 * warp) << 16) + 32 * half, v);
      tmem_ld_wait();
      if (top || !p.bot_transposed) {
        float* dst = (top ? p.out_top : p.out_bot) + co + rr * 64 + 32 * half;
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          *reinterpret_cast<float4*>(dst + j) =
              make_float4(alpha * __uint_as_float(v[j]), alpha * __uint_as_float(v[j + 1]),
                          alpha * __uint_as_float(v[j + 2]), alpha * __uint_as_float(v[j + 3]));
      } else {
        // transposed: element (rr, col) goes to [col][rr] (lanes write consecutive rr)
        float* dst = p.out_bot + co + rr;
#pragma unroll
        for (int j = 0; j < 32; ++j) dst[(32 * half + j) * 64] = alpha * __uint_as_float(v[j]);
      }
    }
  }
  // optional dgC[k] = sum_v dS[k][v] S0[k][v] (one warp per row)
  if (p.dgC) {
    const long long co = (long long)c * 64 * 64;
    for (int r = warp; r < 64; r += THREADS / 32) {
      const float* ds = p.dS + co + r * 64;
      const float* s0 = p.S0 + co + r * 64;
      float sv = ds[lane] * s0[lane] + ds[lane + 32] * s0[lane + 32];
      sv = warp_sum(sv);
      if (lane == 0) p.dgC[(long long)c * 64 + r] = sv;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, TMEM_COLS);
}

}  // namespace kda64tc

// ---------------------------------------------------------------- host side
namespace {
CUtensorMap chunk_map(const float* base, long long chunks) {
  uint64_t dims[2] = {64, (uint64_t)chunks * 64};
  uint64_t strides[1] = {64 * 4};
  uint32_t box[2] = {32, 64};
  return make_tmap(base, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}
CUtensorMap token_map(const float* base, int B, int S, int H) {
  uint64_t dims[3] = {(uint64_t)H * 64, (uint64_t)S, (uint64_t)B};
  uint64_t strides[2] = {(uint64_t)H * 64 * 4, (uint64_t)S * H * 64 * 4};
  uint32_t box[3] = {32, 64, 1};
  return make_tmap(base, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <bool A_MN, bool B_MN>
void launch_pair(const CUtensorMap& top, const CUtensorMap& bot, const CUtensorMap& bm,
                 const kda64tc::Args& a, int chunks) {
  auto kern = kda64tc::pair_product_kernel<A_MN, B_MN>;
  static bool cfg = false;
  if (!cfg) {
    HB_CUDA_CHECK(cudaFuncSetAttribute((const void*)kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kda64tc::SMEM));
    cfg = true;
  }
  kern<<<chunks, kda64tc::THREADS, kda64tc::SMEM, cur_stream()>>>(top, bot, bm, a);
  HB_CUDA_CHECK(cudaGetLastError());
}

kda64tc::Args base_args(int S, int H, int NC) {
  kda64tc::Args a{};
  a.S = S;
  a.H = H;
  a.NC = NC;
  a.alpha_top = a.alpha_bot = 1.f;
  a.status = status_ptr();
  a.budget_ns = wait_budget_ns();
  return a;
}
}  // namespace

// dUp = P^T dO, dSq = Qg^T dO for every chunk (tcgen05).
void kda64_bwd_pre_tc(const float* Pm, const float* Qg, const float* dout, float* dUp, float* dSq, int B,
                      int S, int H, int NC) {
  const long long chunks = (long long)B * H * NC;
  auto a = base_args(S, H, NC);
  a.out_top = dUp;
  a.out_bot = dSq;
  a.kind_top = a.kind_bot = kda64tc::kChunk;
  a.kind_b = kda64tc::kToken;
  launch_pair<true, true>(chunk_map(Pm, chunks), chunk_map(Qg, chunks), token_map(dout, B, S, H), a,
                          (int)chunks);
}

// dWt = -dU S0^T, dQg = dO S0^T;  dP = dO U^T, dKh = (dS U^T)^T, dgC (tcgen05).
void kda64_products_tc(const float* dU, const float* dout, const float* states, const float* dstates,
                       const float* U, float* dWt, float* dQg, float* dP, float* dKh, float* dgC, int B, int S,
                       int H, int NC) {
  const long long chunks = (long long)B * H * NC;
  const CUtensorMap mdO = token_map(dout, B, S, H);
  auto a = base_args(S, H, NC);
  a.out_top = dWt;
  a.out_bot = dQg;
  a.alpha_top = -1.f;
  a.kind_top = kda64tc::kChunk;
  a.kind_bot = kda64tc::kToken;
  a.kind_b = kda64tc::kChunk;
  launch_pair<false, false>(chunk_map(dU, chunks), mdO, chunk_map(states, chunks), a, (int)chunks);
  auto a2 = base_args(S, H, NC);
  a2.out_top = dP;
  a2.out_bot = dKh;
  a2.bot_transposed = 1;
  a2.kind_top = kda64tc::kToken;
  a2.kind_bot = kda64tc::kChunk;
  a2.kind_b = kda64tc::kChunk;
  a2.dS = dstates;
  a2.S0 = states;
  a2.dgC = dgC;
  launch_pair<false, false>(mdO, chunk_map(dstates, chunks), chunk_map(U, chunks), a2, (int)chunks);
}

}  // namespace hb

namespace hb {
// Direct entry for tests: the three stacked products of one chunk-64 KDA
// backward on tcgen05, from fp32 chunk-layout / token-layout tensors.
void kda64_tc_products(torch::Tensor Pm, torch::Tensor Qg, torch::Tensor dout, torch::Tensor dU,
                       torch::Tensor states, torch::Tensor dstates, torch::Tensor U, torch::Tensor dUp,
                       torch::Tensor dSq, torch::Tensor dWt, torch::Tensor dQg, torch::Tensor dP,
                       torch::Tensor dKh, torch::Tensor dgC) {
  const int B = dout.size(0), S = dout.size(1), H = dout.size(2);
  const int NC = (S + 63) / 64;
  kda64_bwd_pre_tc(Pm.data_ptr<float>(), Qg.data_ptr<float>(), dout.data_ptr<float>(), dUp.data_ptr<float>(),
                   dSq.data_ptr<float>(), B, S, H, NC);
  kda64_products_tc(dU.data_ptr<float>(), dout.data_ptr<float>(), states.data_ptr<float>(),
                    dstates.data_ptr<float>(), U.data_ptr<float>(), dWt.data_ptr<float>(), dQg.data_ptr<float>(),
                    dP.data_ptr<float>(), dKh.data_ptr<float>(), dgC.data_ptr<float>(), B, S, H, NC);
}
}  // namespace hb
