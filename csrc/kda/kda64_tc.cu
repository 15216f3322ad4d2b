// Chunk-parallel products of the chunk-64 KDA backward on the 5th-generation
// tensor cores (tcgen05 + TMEM), fp32 accurate.
//
// Per chunk (64 tokens of one head) two 64x64 products that share their B
// operand run as ONE M = 128 MMA:
//
//     [C_top; C_bot] (128 x 64) = [A_top; A_bot] (128 x 64) . B (64 x 64)
//
//   products_u   A = [dU ; dO],  B = S0^T  -> dWt = -dU S0^T, dQg = dO S0^T
//   products_s   A = [dO ; dS],  B = U^T   -> dP = dO U^T,   dKh = (dS U^T)^T;
//                                             and dgC = rowsum(dS * S0)
//
// Both contract over the value index, the contiguous one of every tile, so
// all operands are K-major.  (Products over the row index, like P^T dO, would
// need MN-major fp32 operands, which tcgen05 reads only in the 128-byte swizzle
// with 32-byte atoms; those stay on the warp-level kernels.)
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
constexpr int TMEM_COLS = 128;   // two 64-column accumulators

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

// Persistent: each CTA walks chunks c = blockIdx.x, blockIdx.x + gridDim.x, ...
// The next chunk's TMA loads are issued as soon as the current chunk's MMAs
// have retired (the operand tiles are free) and land while the current
// accumulator is read back from TMEM and stored; the accumulator alternates
// between two 64-column TMEM buffers.
__global__ void __launch_bounds__(THREADS, 2)
    pair_product_kernel(const __grid_constant__ CUtensorMap tmTop, const __grid_constant__ CUtensorMap tmBot,
                        const __grid_constant__ CUtensorMap tmB, const Args p, int chunks) {
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
  const uint32_t tmem0 = *tmem_slot;

  auto issue_loads = [&](int c) {
    const int n = c % p.NC, h = (c / p.NC) % p.H, b = c / (p.NC * p.H);
    mbar_expect_tx(smem_u32(full), A_BYTES + B_BYTES);
    for (int a = 0; a < 2; ++a) {
      // K-major A: [k atom][128 rows] (top rows 0-63, bottom rows 64-127)
      const uint32_t top = sA + a * 2 * ATOM;
      const uint32_t bot = top + ATOM;
      load_box(top, &tmTop, smem_u32(full), p.kind_top, 32 * a, c, n, h, b);
      load_box(bot, &tmBot, smem_u32(full), p.kind_bot, 32 * a, c, n, h, b);
      load_box(sB + a * ATOM, &tmB, smem_u32(full), p.kind_b, 32 * a, c, n, h, b);
    }
  };
  if (threadIdx.x == 0 && blockIdx.x < chunks) issue_loads(blockIdx.x);
  bool alive = true;
  int it = 0;
  for (int c = blockIdx.x; c < chunks && alive; c += gridDim.x, ++it) {
    const uint32_t par = it & 1;
    bool ok = mbar_wait(smem_u32(full), par, p.status, kErrTimeoutProducer, p.budget_ns);
    // after a timeout, wait (bounded) for the copies still in flight; if they
    // land the chunk is computed all the same
    if (!ok) ok = mbar_wait(smem_u32(full), par, nullptr, 0, p.budget_ns);
    // ---- hi / lo split in place (elementwise: the swizzle does not matter)
    if (ok) {
      float4* hi = reinterpret_cast<float4*>(smem);
      float4* lo = reinterpret_cast<float4*>(smem + A_BYTES + B_BYTES);
      for (int i = threadIdx.x; i < (A_BYTES + B_BYTES) / 16; i += THREADS) {
        const float4 x = hi[i];
        float4 hv;
        hv.x = __uint_as_float(__float_as_uint(x.x) & 0xffffe000u);
        hv.y = __uint_as_float(__float_as_uint(x.y) & 0xffffe000u);
        hv.z = __uint_as_float(__float_as_uint(x.z) & 0xffffe000u);
        hv.w = __uint_as_float(__float_as_uint(x.w) & 0xffffe000u);
        hi[i] = hv;
        lo[i] = make_float4(x.x - hv.x, x.y - hv.y, x.z - hv.z, x.w - hv.w);
      }
      fence_proxy_async();   // generic-proxy smem writes -> visible to the tensor core
    }
    tc_fence_before();
    // one decision for the whole CTA: thread 0's view of its loads (an error
    // recorded by another kernel does not stop this one: its outputs feed the
    // rest of the step and must be written)
    if (threadIdx.x == 0) *go_flag = ok ? 1 : 0;
    __syncthreads();
    const bool go = *go_flag != 0;
    const uint32_t tmem = tmem0 + 64 * par;
    // ---- MMAs: 8 K steps x (hi.hi + hi.lo + lo.hi), then the next chunk's loads
    if (go && threadIdx.x == 0) {
      tc_fence_after();
      constexpr uint32_t idesc = idesc_tf32(false, false);
      for (int kk = 0; kk < 8; ++kk) {
        const uint64_t ah = desc_kmajor(sA, 128, kk), al = desc_kmajor(sAlo, 128, kk);
        const uint64_t bh = desc_kmajor(sB, 64, kk), bl = desc_kmajor(sBlo, 64, kk);
        umma_tf32(tmem, ah, bh, idesc, kk > 0 ? 1u : 0u);
        umma_tf32(tmem, ah, bl, idesc, 1u);
        umma_tf32(tmem, al, bh, idesc, 1u);
      }
      umma_commit(smem_u32(done));
    }
    ok = go;
    if (go) {
      ok = mbar_wait(smem_u32(done), par, p.status, kErrTimeoutMma, p.budget_ns);
      if (!ok) ok = mbar_wait(smem_u32(done), par, nullptr, 0, p.budget_ns);  // MMAs still in flight
    }
    tc_fence_after();
    if (!ok) alive = false;
    // operands consumed: the next chunk's tiles land during this epilogue
    if (ok && threadIdx.x == 0 && c + gridDim.x < chunks) issue_loads(c + gridDim.x);
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
      // optional dgC[k] = sum_v dS[k][v] S0[k][v]: 8 threads per row, float4 loads
      if (p.dgC) {
        for (int i = threadIdx.x; i < 64 * 8; i += THREADS) {
          const int row = i >> 3, q8 = (i & 7) * 8;
          const float4 a0 = *reinterpret_cast<const float4*>(p.dS + co + row * 64 + q8);
          const float4 a1 = *reinterpret_cast<const float4*>(p.dS + co + row * 64 + q8 + 4);
          const float4 b0 = *reinterpret_cast<const float4*>(p.S0 + co + row * 64 + q8);
          const float4 b1 = *reinterpret_cast<const float4*>(p.S0 + co + row * 64 + q8 + 4);
          float sv = a0.x * b0.x + a0.y * b0.y + a0.z * b0.z + a0.w * b0.w + a1.x * b1.x + a1.y * b1.y +
                     a1.z * b1.z + a1.w * b1.w;
          sv += __shfl_xor_sync(0xffffffffu, sv, 1);
          sv += __shfl_xor_sync(0xffffffffu, sv, 2);
          sv += __shfl_xor_sync(0xffffffffu, sv, 4);
          if ((i & 7) == 0) p.dgC[(long long)c * 64 + row] = sv;
        }
      }
    }
    tc_fence_before();
    __syncthreads();   // TMEM buffer and barrier phases are reused two iterations on
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem0, TMEM_COLS);
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

void launch_pair(const CUtensorMap& top, const CUtensorMap& bot, const CUtensorMap& bm,
                 const kda64tc::Args& a, int chunks) {
  auto kern = kda64tc::pair_product_kernel;
  static bool cfg = false;
  if (!cfg) {
    HB_CUDA_CHECK(cudaFuncSetAttribute((const void*)kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kda64tc::SMEM));
    cfg = true;
  }
  const int grid = std::min(chunks, 2 * num_sms());
  kern<<<grid, kda64tc::THREADS, kda64tc::SMEM, cur_stream()>>>(top, bot, bm, a, chunks);
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
  launch_pair(chunk_map(dU, chunks), mdO, chunk_map(states, chunks), a, (int)chunks);
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
  launch_pair(mdO, chunk_map(dstates, chunks), chunk_map(U, chunks), a2, (int)chunks);
}

}  // namespace hb

namespace hb {
// Direct entry for tests: the stacked products of the chunk-64 KDA backward on
// tcgen05, from fp32 chunk-layout / token-layout tensors.
void kda64_tc_products(torch::Tensor dout, torch::Tensor dU, torch::Tensor states, torch::Tensor dstates,
                       torch::Tensor U, torch::Tensor dWt, torch::Tensor dQg, torch::Tensor dP, torch::Tensor dKh,
                       torch::Tensor dgC) {
  const int B = dout.size(0), S = dout.size(1), H = dout.size(2);
  const int NC = (S + 63) / 64;
  kda64_products_tc(dU.data_ptr<float>(), dout.data_ptr<float>(), states.data_ptr<float>(),
                    dstates.data_ptr<float>(), U.data_ptr<float>(), dWt.data_ptr<float>(), dQg.data_ptr<float>(),
                    dP.data_ptr<float>(), dKh.data_ptr<float>(), dgC.data_ptr<float>(), B, S, H, NC);
}
}  // namespace hb
