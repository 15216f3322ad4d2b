// KDA output gate (model/kda.py:361-376), fused:
//   y = RMSNorm_K(o) * o_norm * sigmoid(gl + g_bias)      -> bf16, input of wo
// o [T, H, K] fp32 (the recurrence output), gl [T, H*K] fp32 (low-rank gate
// logits), o_norm [K], g_bias [H*K]; the norm runs over each head's K channels
// with eps 1e-5.  One warp per (token, head) row; the backward emits do, dgl
// and the two parameter gradients (block partials in shared memory, then one
// atomic per element and block).
#include <torch/extension.h>

#include "../common/host.h"
#include "../common/sm100.cuh"

namespace hb {
namespace {

template <int DK>
__global__ void out_gate_fwd_kernel(const float* __restrict__ o, const float* __restrict__ gl,
                                    const float* __restrict__ w, const float* __restrict__ gb, long long rows,
                                    int H, float eps, __nv_bfloat16* __restrict__ y, float* __restrict__ rstd) {
  constexpr int PL = DK / 32;
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  for (long long r = blockIdx.x * (long long)warps + (threadIdx.x >> 5); r < rows;
       r += (long long)gridDim.x * warps) {
    const int h = r % H;
    const long long base = r * DK;
    float ov[PL], ss = 0.f;
#pragma unroll
    for (int j = 0; j < PL; ++j) {
      ov[j] = o[base + lane + 32 * j];
      ss += ov[j] * ov[j];
    }
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / DK + eps);
#pragma unroll
    for (int j = 0; j < PL; ++j) {
      const int c = lane + 32 * j;
      const float z = gl[base + c] + gb[h * DK + c];
      const float s = 1.f / (1.f + __expf(-z));
      y[base + c] = __float2bfloat16_rn(ov[j] * rs * w[c] * s);
    }
    if (lane == 0) rstd[r] = rs;
  }
}

template <int DK>
__global__ void out_gate_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const float* __restrict__ o,
                                    const float* __restrict__ gl, const float* __restrict__ w,
                                    const float* __restrict__ gb, const float* __restrict__ rstd,
                                    long long rows, int H, float* __restrict__ dO, float* __restrict__ dgl,
                                    float* __restrict__ dw, float* __restrict__ dgb) {
  constexpr int PL = DK / 32;
  extern __shared__ float sh[];  // dgb partial [H*DK], dw partial [DK]
  float* sgb = sh;
  float* sw = sh + H * DK;
  for (int i = threadIdx.x; i < H * DK + DK; i += blockDim.x) sh[i] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  float accw[PL];
#pragma unroll
  for (int j = 0; j < PL; ++j) accw[j] = 0.f;
  for (long long r = blockIdx.x * (long long)warps + (threadIdx.x >> 5); r < rows;
       r += (long long)gridDim.x * warps) {
    const int h = r % H;
    const long long base = r * DK;
    const float rs = rstd[r];
    float n[PL], dn[PL], dot = 0.f;
#pragma unroll
    for (int j = 0; j < PL; ++j) {
      const int c = lane + 32 * j;
      n[j] = o[base + c] * rs;
      const float z = gl[base + c] + gb[h * DK + c];
      const float s = 1.f / (1.f + __expf(-z));
      const float g = __bfloat162float(dy[base + c]);
      const float on = n[j] * w[c];
      const float don = g * s;
      const float dz = g * on * s * (1.f - s);
      dgl[base + c] = dz;
      atomicAdd(sgb + h * DK + c, dz);
      accw[j] += don * n[j];
      dn[j] = don * w[c];
      dot += dn[j] * n[j];
    }
    dot = warp_sum(dot) / DK;
#pragma unroll
    for (int j = 0; j < PL; ++j) dO[base + lane + 32 * j] = rs * (dn[j] - n[j] * dot);
  }
#pragma unroll
  for (int j = 0; j < PL; ++j) atomicAdd(sw + lane + 32 * j, accw[j]);
  __syncthreads();
  for (int i = threadIdx.x; i < H * DK; i += blockDim.x)
    if (sgb[i] != 0.f) atomicAdd(dgb + i, sgb[i]);
  for (int i = threadIdx.x; i < DK; i += blockDim.x) atomicAdd(dw + i, sw[i]);
}

int grid_rows(long long rows) {
  const long long g = (rows + 7) / 8;
  return (int)std::max(1LL, std::min(g, (long long)num_sms() * 8));
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
  OUT_GATE_DISPATCH(DKV, {
    out_gate_fwd_kernel<DK><<<grid_rows(rows), 256, 0, cur_stream()>>>(
        o.data_ptr<float>(), gl.data_ptr<float>(), w.data_ptr<float>(), gb.data_ptr<float>(), rows, H,
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
  const size_t smem = (size_t)(H * DKV + DKV) * 4;
  HB_CHECK(smem <= 200 * 1024, "kda_out_gate_bwd: too many heads");
  OUT_GATE_DISPATCH(DKV, {
    static bool cfg = false;
    if (!cfg) {
      HB_CUDA_CHECK(cudaFuncSetAttribute(out_gate_bwd_kernel<DK>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
      cfg = true;
    }
    out_gate_bwd_kernel<DK><<<grid_rows(rows), 256, smem, cur_stream()>>>(
        (const __nv_bfloat16*)dy.data_ptr(), o.data_ptr<float>(), gl.data_ptr<float>(), w.data_ptr<float>(),
        gb.data_ptr<float>(), rstd.data_ptr<float>(), rows, H, dO.data_ptr<float>(), dgl.data_ptr<float>(),
        dw.data_ptr<float>(), dgb.data_ptr<float>());
  })
  HB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace hb
