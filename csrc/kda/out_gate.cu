// KDA output gate (model/kda.py:361-376), fused:
//   y = RMSNorm_K(o) * o_norm * sigmoid(gl + g_bias)      -> bf16, input of wo
// o [T, H, K] fp32 (the recurrence output), gl [T, H*K] fp32 (low-rank gate
// logits), o_norm [K], g_bias [H*K]; the norm runs over each head's K channels
// with eps 1e-5.  One warp per (token, head) row, blocks per head; the
// backward emits do, dgl and the two parameter gradients (register sums per
// lane, then shared memory, then one atomic per element and block).
#include <torch/extension.h>

#include "../common/host.h"
#include "../common/sm100.cuh"

namespace hb {
namespace {

// sigmoid by the hardware exponential and an approximate divide (2 ulp)
__device__ __forceinline__ float sigm(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

// Block per head (blockIdx.y), warp per token: the head's o_norm and g_bias
// stay in registers, and the backward sums their gradients in registers too.
template <int DK>
__global__ void __launch_bounds__(256) out_gate_fwd_kernel(
    const float* __restrict__ o, const float* __restrict__ gl, const float* __restrict__ w,
    const float* __restrict__ gb, long long T, int H, float eps, __nv_bfloat16* __restrict__ y,
    float* __restrict__ rstd) {
  constexpr int PL = DK / 32;
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5, h = blockIdx.y;
  float wr[PL], br[PL];
#pragma unroll
  for (int j = 0; j < PL; ++j) {
    wr[j] = w[lane + 32 * j];
    br[j] = gb[h * DK + lane + 32 * j];
  }
  for (long long t = blockIdx.x * (long long)warps + (threadIdx.x >> 5); t < T;
       t += (long long)gridDim.x * warps) {
    const long long r = t * H + h;
    const long long base = r * DK;
    float ov[PL], zv[PL], ss = 0.f;
#pragma unroll
    for (int j = 0; j < PL; ++j) {
      ov[j] = o[base + lane + 32 * j];
      zv[j] = gl[base + lane + 32 * j];
      ss += ov[j] * ov[j];
    }
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / DK + eps);
#pragma unroll
    for (int j = 0; j < PL; ++j)
      y[base + lane + 32 * j] = __float2bfloat16_rn(ov[j] * rs * wr[j] * sigm(zv[j] + br[j]));
    if (lane == 0) rstd[r] = rs;
  }
}

template <int DK>
__global__ void __launch_bounds__(256) out_gate_bwd_kernel(
    const __nv_bfloat16* __restrict__ dy, const float* __restrict__ o, const float* __restrict__ gl,
    const float* __restrict__ w, const float* __restrict__ gb, const float* __restrict__ rstd, long long T,
    int H, float* __restrict__ dO, float* __restrict__ dgl, float* __restrict__ dw, float* __restrict__ dgb) {
  constexpr int PL = DK / 32;
  __shared__ float sgb[DK], sw[DK];
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5, h = blockIdx.y;
  for (int i = threadIdx.x; i < DK; i += blockDim.x) sgb[i] = sw[i] = 0.f;
  __syncthreads();
  float wr[PL], br[PL], accw[PL], accb[PL];
#pragma unroll
  for (int j = 0; j < PL; ++j) {
    wr[j] = w[lane + 32 * j];
    br[j] = gb[h * DK + lane + 32 * j];
    accw[j] = accb[j] = 0.f;
  }
  for (long long t = blockIdx.x * (long long)warps + (threadIdx.x >> 5); t < T;
       t += (long long)gridDim.x * warps) {
    const long long r = t * H + h;
    const long long base = r * DK;
    const float rs = rstd[r];
    float n[PL], dn[PL], dot = 0.f;
#pragma unroll
    for (int j = 0; j < PL; ++j) {
      const int c = lane + 32 * j;
      n[j] = o[base + c] * rs;
      const float s = sigm(gl[base + c] + br[j]);
      const float g = __bfloat162float(dy[base + c]);
      const float don = g * s;
      const float dz = g * n[j] * wr[j] * s * (1.f - s);
      dgl[base + c] = dz;
      accb[j] += dz;
      accw[j] += don * n[j];
      dn[j] = don * wr[j];
      dot += dn[j] * n[j];
    }
    dot = warp_sum(dot) * (1.f / DK);
#pragma unroll
    for (int j = 0; j < PL; ++j) dO[base + lane + 32 * j] = rs * (dn[j] - n[j] * dot);
  }
#pragma unroll
  for (int j = 0; j < PL; ++j) {
    atomicAdd(sw + lane + 32 * j, accw[j]);
    atomicAdd(sgb + lane + 32 * j, accb[j]);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < DK; i += blockDim.x) {
    atomicAdd(dw + i, sw[i]);
    atomicAdd(dgb + h * DK + i, sgb[i]);
  }
}

// blocks: (token runs) x (heads), about 8 resident blocks per SM in all
dim3 grid_heads(long long T, int H) {
  const long long gx = std::max(1LL, std::min((T + 7) / 8, ((long long)num_sms() * 8 + H - 1) / H));
  return dim3((unsigned)gx, (unsigned)H);
}

}  // namespace

#define OUT_GATE_DISPATCH(DKV, ...)                              \
  if (DKV == 32) {                                               \
    constexpr int DK = 32;                                       \
    __VA_ARGS__                                                  \
  } else if (DKV == 64) {                                        \
    constexpr int DK = 64;                                       \
    __VA_ARGS__                                                  \
  } else if (DKV == 128) {                                       \
    constexpr int DK = 128;                                      \
    __VA_ARGS__                                                  \
  } else {                                                       \
    HB_CHECK(false, "kda_out_gate: head dim 32, 64 or 128");     \
  }

void kda_out_gate_fwd(torch::Tensor o, torch::Tensor gl, torch::Tensor w, torch::Tensor gb, double eps,
                      torch::Tensor y, torch::Tensor rstd) {
  HB_CHECK(o.is_contiguous() && gl.is_contiguous() && y.is_contiguous(), "kda_out_gate_fwd: contiguous");
  const int H = o.size(-2), DKV = o.size(-1);
  const long long rows = o.numel() / DKV;
  if (rows == 0) return;
  const long long T = rows / H;
  OUT_GATE_DISPATCH(DKV, {
    out_gate_fwd_kernel<DK><<<grid_heads(T, H), 256, 0, cur_stream()>>>(
        o.data_ptr<float>(), gl.data_ptr<float>(), w.data_ptr<float>(), gb.data_ptr<float>(), T, H,
        (float)eps, (__nv_bfloat16*)y.data_ptr(), rstd.data_ptr<float>());
  })
  HB_CUDA_CHECK(cudaGetLastError());
}

void kda_out_gate_bwd(torch::Tensor dy, torch::Tensor o, torch::Tensor gl, torch::Tensor w, torch::Tensor gb,
                      torch::Tensor rstd, torch::Tensor dO, torch::Tensor dgl, torch::Tensor dw,
                      torch::Tensor dgb) {
  check_bf16(dy, "dy");
  HB_CHECK(dy.is_contiguous() && dO.is_contiguous() && dgl.is_contiguous(), "kda_out_gate_bwd: contiguous");
  const int H = o.size(-2), DKV = o.size(-1);
  const long long rows = o.numel() / DKV;
  if (rows == 0) return;
  const long long T = rows / H;
  OUT_GATE_DISPATCH(DKV, {
    out_gate_bwd_kernel<DK><<<grid_heads(T, H), 256, 0, cur_stream()>>>(
        (const __nv_bfloat16*)dy.data_ptr(), o.data_ptr<float>(), gl.data_ptr<float>(), w.data_ptr<float>(),
        gb.data_ptr<float>(), rstd.data_ptr<float>(), T, H, dO.data_ptr<float>(), dgl.data_ptr<float>(),
        dw.data_ptr<float>(), dgb.data_ptr<float>());
  })
  HB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace hb
