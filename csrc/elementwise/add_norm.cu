// Residual add fused with the following RMSNorm (model/transformer.py:80-99):
//   x_new = x + rs * a          (fp32 residual stream, rs = the block's scalar)
//   h     = x_new * rsqrt(mean(x_new^2) + eps) * w      (compute dtype, bf16)
// Backward, per row, with g = dL/dx_new from later layers and dh = dL/dh:
//   dx = g + rstd * (dh*w - n * mean(dh*w*n)),  n = x_new * rstd
//   da = rs * dx,  drs = sum(dx * a),  dw = sum_t dh * n
// One warp per row, 16-byte accesses; the two reductions over rows are block
// partials (shared memory) flushed with one atomic per element and block.
#include <torch/extension.h>

#include "../common/host.h"
#include "../common/sm100.cuh"

namespace hb {
namespace {

constexpr int AN_MAXV = 16;  // float4 per lane: D <= 2048

template <int NV>
__global__ void add_norm_fwd_kernel(const float* __restrict__ x, const float* __restrict__ a,
                                    const float* __restrict__ rs_p, const float* __restrict__ w, int T, int D,
                                    float eps, float* __restrict__ xn, __nv_bfloat16* __restrict__ h,
                                    float* __restrict__ rstd) {
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  const float rs = *rs_p;
  const int D4 = D / 4;
  for (long long r = blockIdx.x * (long long)warps + (threadIdx.x >> 5); r < T; r += (long long)gridDim.x * warps) {
    const float4* xr = reinterpret_cast<const float4*>(x + r * D);
    const float4* ar = reinterpret_cast<const float4*>(a + r * D);
    float4 v[NV];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = lane + 32 * j;
      if (i < D4) {
        const float4 xv = xr[i], av = ar[i];
        v[j] = make_float4(xv.x + rs * av.x, xv.y + rs * av.y, xv.z + rs * av.z, xv.w + rs * av.w);
        ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
      }
    }
    ss = warp_sum(ss);
    const float rr = rsqrtf(ss / D + eps);
    float4* xo = reinterpret_cast<float4*>(xn + r * D);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = lane + 32 * j;
      if (i < D4) {
        xo[i] = v[j];
        const float4 wv = reinterpret_cast<const float4*>(w)[i];
        __nv_bfloat162 p0 = __floats2bfloat162_rn(v[j].x * rr * wv.x, v[j].y * rr * wv.y);
        __nv_bfloat162 p1 = __floats2bfloat162_rn(v[j].z * rr * wv.z, v[j].w * rr * wv.w);
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t*>(&p0);
        pk.y = *reinterpret_cast<uint32_t*>(&p1);
        *reinterpret_cast<uint2*>(h + r * D + 4 * i) = pk;
      }
    }
    if (lane == 0) rstd[r] = rr;
  }
}

// Backward: each warp keeps a private dw row in shared memory (lane-owned
// 16-byte slots, no atomics), a row is read twice (the second read hits L1)
// so no per-row arrays stay in registers.
template <int NV>
__global__ void add_norm_bwd_kernel(const float* __restrict__ g, const __nv_bfloat16* __restrict__ dh,
                                    const float* __restrict__ xn, const float* __restrict__ a,
                                    const float* __restrict__ rs_p, const float* __restrict__ w,
                                    const float* __restrict__ rstd, int T, int D, float* __restrict__ dx,
                                    float* __restrict__ da, float* __restrict__ drs, float* __restrict__ dw) {
  extern __shared__ float sdw[];  // [warps][D]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
  for (int i = threadIdx.x; i < warps * D; i += blockDim.x) sdw[i] = 0.f;
  __syncthreads();
  float4* mydw = reinterpret_cast<float4*>(sdw + warp * D);
  const float rs = *rs_p;
  const int D4 = D / 4;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  auto ld_dh = [&](long long r, int i) {
    const uint2 pk = *reinterpret_cast<const uint2*>(dh + r * D + 4 * i);
    const float2 h01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&pk.x));
    const float2 h23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&pk.y));
    return make_float4(h01.x, h01.y, h23.x, h23.y);
  };
  float drs_acc = 0.f;
  for (long long r = blockIdx.x * (long long)warps + warp; r < T; r += (long long)gridDim.x * warps) {
    const float rr = rstd[r];
    const float4* x4 = reinterpret_cast<const float4*>(xn + r * D);
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = lane + 32 * j;
      if (i < D4) {
        const float4 xv = x4[i], wv = w4[i], hv = ld_dh(r, i);
        const float4 n = make_float4(xv.x * rr, xv.y * rr, xv.z * rr, xv.w * rr);
        dot += hv.x * wv.x * n.x + hv.y * wv.y * n.y + hv.z * wv.z * n.z + hv.w * wv.w * n.w;
        float4 acc = mydw[i];
        acc.x += hv.x * n.x;
        acc.y += hv.y * n.y;
        acc.z += hv.z * n.z;
        acc.w += hv.w * n.w;
        mydw[i] = acc;
      }
    }
    dot = warp_sum(dot) / D;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = lane + 32 * j;
      if (i < D4) {
        const float4 xv = x4[i], wv = w4[i], hv = ld_dh(r, i);
        float4 d = make_float4(rr * (hv.x * wv.x - xv.x * rr * dot), rr * (hv.y * wv.y - xv.y * rr * dot),
                               rr * (hv.z * wv.z - xv.z * rr * dot), rr * (hv.w * wv.w - xv.w * rr * dot));
        if (g) {
          const float4 gv = reinterpret_cast<const float4*>(g + r * D)[i];
          d.x += gv.x;
          d.y += gv.y;
          d.z += gv.z;
          d.w += gv.w;
        }
        reinterpret_cast<float4*>(dx + r * D)[i] = d;
        reinterpret_cast<float4*>(da + r * D)[i] = make_float4(rs * d.x, rs * d.y, rs * d.z, rs * d.w);
        const float4 av = reinterpret_cast<const float4*>(a + r * D)[i];
        drs_acc += d.x * av.x + d.y * av.y + d.z * av.z + d.w * av.w;
      }
    }
  }
  drs_acc = warp_sum(drs_acc);
  if (lane == 0) atomicAdd(drs, drs_acc);
  __syncthreads();
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < warps; ++k) s += sdw[k * D + i];
    atomicAdd(dw + i, s);
  }
}

int grid_rows(long long rows) {
  const long long g = (rows + 7) / 8;
  return (int)std::max(1LL, std::min(g, (long long)num_sms() * 8));
}

}  // namespace

#define AN_DISPATCH(D, ...)                                  \
  {                                                          \
    const int nv_ = (D / 4 + 31) / 32;                       \
    if (nv_ <= 4) {                                          \
      constexpr int NV = 4;                                  \
      __VA_ARGS__                                            \
    } else if (nv_ <= 8) {                                   \
      constexpr int NV = 8;                                  \
      __VA_ARGS__                                            \
    } else {                                                 \
      constexpr int NV = AN_MAXV;                            \
      __VA_ARGS__                                            \
    }                                                        \
  }

void add_norm_fwd(torch::Tensor x, torch::Tensor a, torch::Tensor rs, torch::Tensor w, double eps,
                  torch::Tensor xn, torch::Tensor h, torch::Tensor rstd) {
  const int T = x.size(0), D = x.size(1);
  HB_CHECK(x.is_contiguous() && a.is_contiguous() && xn.is_contiguous() && h.is_contiguous(),
           "add_norm_fwd: contiguous operands");
  HB_CHECK(D % 4 == 0 && D <= 4 * 32 * AN_MAXV, "add_norm: D % 4 == 0 and D <= 2048");
  check_bf16(h, "h");
  if (T == 0) return;
  AN_DISPATCH(D, {
    add_norm_fwd_kernel<NV><<<grid_rows(T), 256, 0, cur_stream()>>>(
        x.data_ptr<float>(), a.data_ptr<float>(), rs.data_ptr<float>(), w.data_ptr<float>(), T, D,
        (float)eps, xn.data_ptr<float>(), (__nv_bfloat16*)h.data_ptr(), rstd.data_ptr<float>());
  })
  HB_CUDA_CHECK(cudaGetLastError());
}

void add_norm_bwd(c10::optional<torch::Tensor> g, torch::Tensor dh, torch::Tensor xn, torch::Tensor a,
                  torch::Tensor rs, torch::Tensor w, torch::Tensor rstd, torch::Tensor dx, torch::Tensor da,
                  torch::Tensor drs, torch::Tensor dw) {
  const int T = xn.size(0), D = xn.size(1);
  check_bf16(dh, "dh");
  HB_CHECK(dh.is_contiguous() && dx.is_contiguous() && da.is_contiguous(), "add_norm_bwd: contiguous");
  if (g.has_value()) HB_CHECK(g->is_contiguous() && g->scalar_type() == torch::kFloat32, "add_norm_bwd: g");
  if (T == 0) return;
  HB_CHECK(D % 4 == 0 && D <= 4 * 32 * AN_MAXV, "add_norm: D % 4 == 0 and D <= 2048");
  AN_DISPATCH(D, {
    if (D * 4 * 8 > 48 * 1024) {
      HB_CUDA_CHECK(cudaFuncSetAttribute(add_norm_bwd_kernel<NV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         D * 4 * 8));
    }
    add_norm_bwd_kernel<NV><<<grid_rows(T), 256, (size_t)D * 4 * 8, cur_stream()>>>(
        g.has_value() ? g->data_ptr<float>() : nullptr, (const __nv_bfloat16*)dh.data_ptr(),
        xn.data_ptr<float>(), a.data_ptr<float>(), rs.data_ptr<float>(), w.data_ptr<float>(),
        rstd.data_ptr<float>(), T, D, dx.data_ptr<float>(), da.data_ptr<float>(), drs.data_ptr<float>(),
        dw.data_ptr<float>());
  })
  HB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace hb
