// Memory-bound kernels of the transformer block: RMSNorm (fwd/bwd), RoPE
// (fwd/bwd), SwiGLU activation (fwd/bwd), token embedding (fwd/bwd).
//
// RMSNorm (model/transformer.py:14-24): y = x * rsqrt(mean(x^2) + eps) * w in
// fp32, cast to the output dtype.  One warp per row; rows are processed by a
// persistent grid so the weight-gradient partial sums of a warp are reduced
// in registers before one atomic per column.
#include <torch/extension.h>

#include "../common/host.h"
#include "../common/sm100.cuh"

namespace hb {

namespace {

template <typename T>
HB_DEVICE float to_f(T v);
template <>
HB_DEVICE float to_f<float>(float v) { return v; }
template <>
HB_DEVICE float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
HB_DEVICE T from_f(float v);
template <>
HB_DEVICE float from_f<float>(float v) { return v; }
template <>
HB_DEVICE __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

constexpr int NORM_MAX_PER_LANE = 64;  // backward keeps D/32 column partials per lane: D <= 2048

// ---------------------------------------------------------------- RMSNorm
// x: [T, D] fp32; w: [D] fp32; y: [T, D] (OutT); rstd: [T] fp32.
template <typename OutT>
__global__ void rmsnorm_fwd_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                   OutT* __restrict__ y, float* __restrict__ rstd, int T, int D,
                                   float eps) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < T; row += gridDim.x * warps) {
    const float* xr = x + (long long)row * D;
    float ss = 0.f;
    for (int c = lane * 4; c < D; c += 128) {
      float4 v = *reinterpret_cast<const float4*>(xr + c);
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / D + eps);
    if (lane == 0 && rstd) rstd[row] = r;
    OutT* yr = y + (long long)row * D;
    for (int c = lane * 4; c < D; c += 128) {
      float4 v = *reinterpret_cast<const float4*>(xr + c);
      float4 ww = *reinterpret_cast<const float4*>(w + c);
      yr[c + 0] = from_f<OutT>(v.x * r * ww.x);
      yr[c + 1] = from_f<OutT>(v.y * r * ww.y);
      yr[c + 2] = from_f<OutT>(v.z * r * ww.z);
      yr[c + 3] = from_f<OutT>(v.w * r * ww.w);
    }
  }
}

// dy: [T, D] (InT); dx: [T, D] fp32 (written, or added when accumulate);
// dw: [D] fp32 accumulated with one atomic per column per warp.
template <typename InT>
__global__ void rmsnorm_bwd_kernel(const InT* __restrict__ dy, const float* __restrict__ x,
                                   const float* __restrict__ w, const float* __restrict__ rstd,
                                   float* __restrict__ dx, float* __restrict__ dw, int T, int D,
                                   bool accumulate) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  float dwacc[NORM_MAX_PER_LANE];
#pragma unroll
  for (int i = 0; i < NORM_MAX_PER_LANE; ++i) dwacc[i] = 0.f;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < T; row += gridDim.x * warps) {
    const float* xr = x + (long long)row * D;
    const InT* dyr = dy + (long long)row * D;
    const float r = rstd[row];
    // dot = sum(dy * w * xhat)
    float dot = 0.f;
    int i = 0;
    for (int c = lane; c < D; c += 32, ++i) {
      const float xh = xr[c] * r;
      const float g = to_f<InT>(dyr[c]);
      dot += g * w[c] * xh;
      dwacc[i] += g * xh;
    }
    dot = warp_sum(dot) / D;
    float* dxr = dx + (long long)row * D;
    for (int c = lane; c < D; c += 32) {
      const float xh = xr[c] * r;
      const float g = to_f<InT>(dyr[c]);
      const float v = r * (g * w[c] - xh * dot);
      dxr[c] = accumulate ? dxr[c] + v : v;
    }
  }
  int i = 0;
  for (int c = lane; c < D; c += 32, ++i) atomicAdd(dw + c, dwacc[i]);
}

// ---------------------------------------------------------------- RoPE
// q: [T, Nh, H] bf16 (in place), positions implicit (t % S) or explicit.
// cos/sin: [Smax, H] bf16 tables (rotate-half layout).  inverse=true applies
// the transpose rotation (backward).
__global__ void rope_kernel(__nv_bfloat16* __restrict__ q, int T, int Nh, int H, int S,
                            const __nv_bfloat16* __restrict__ cosT,
                            const __nv_bfloat16* __restrict__ sinT,
                            const long long* __restrict__ positions, bool inverse) {
  const int half = H / 2;
  const long long total = (long long)T * Nh * half;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int j = idx % half;
    const long long th = idx / half;  // t * Nh + h
    const long long t = th / Nh;
    const long long pos = positions ? positions[t] : (t % S);
    __nv_bfloat16* base = q + th * H;
    const float x1 = __bfloat162float(base[j]);
    const float x2 = __bfloat162float(base[j + half]);
    const float c1 = __bfloat162float(cosT[pos * H + j]);
    const float c2 = __bfloat162float(cosT[pos * H + j + half]);
    const float s1 = __bfloat162float(sinT[pos * H + j]);
    const float s2 = __bfloat162float(sinT[pos * H + j + half]);
    float y1, y2;
    if (!inverse) {
      // y = x*c + rotate_half(x)*s, rotate_half(x) = [-x2, x1]
      y1 = x1 * c1 - x2 * s1;
      y2 = x2 * c2 + x1 * s2;
    } else {
      // dx_j = dy_j c_j + dy_{j+h} s_{j+h};  dx_{j+h} = dy_{j+h} c_{j+h} - dy_j s_j
      y1 = x1 * c1 + x2 * s2;
      y2 = x2 * c2 - x1 * s1;
    }
    base[j] = __float2bfloat16_rn(y1);
    base[j + half] = __float2bfloat16_rn(y2);
  }
}

// ---------------------------------------------------------------- SwiGLU
// gu: [R, 2F] bf16 rows with ld_gu; h = silu(g) * u -> [R, F] bf16.
// rows with row_src[r] < 0 (MoE pad rows) are written as zeros.
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ h,
                                  long long R, int F, const int* __restrict__ row_src) {
  const long long total = R * (F / 2);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / (F / 2);
    const int c = (i % (F / 2)) * 2;
    if (row_src && row_src[r] < 0) {
      *reinterpret_cast<__nv_bfloat162*>(h + r * F + c) = __floats2bfloat162_rn(0.f, 0.f);
      continue;
    }
    const __nv_bfloat162 g2 = *reinterpret_cast<const __nv_bfloat162*>(gu + r * 2 * F + c);
    const __nv_bfloat162 u2 = *reinterpret_cast<const __nv_bfloat162*>(gu + r * 2 * F + F + c);
    const float g0 = __bfloat162float(g2.x), g1 = __bfloat162float(g2.y);
    // silu in the compute dtype, then the product (moe.py:23-29 rounds silu(g) to bf16)
    const float s0 = __bfloat162float(__float2bfloat16_rn(__fdividef(g0, 1.f + __expf(-g0))));
    const float s1 = __bfloat162float(__float2bfloat16_rn(__fdividef(g1, 1.f + __expf(-g1))));
    __nv_bfloat162 o = __floats2bfloat162_rn(s0 * __bfloat162float(u2.x), s1 * __bfloat162float(u2.y));
    *reinterpret_cast<__nv_bfloat162*>(h + r * F + c) = o;
  }
}

// dh: [R, F]; gu: [R, 2F] -> dgu: [R, 2F] bf16.
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dh, const __nv_bfloat16* __restrict__ gu,
                                  __nv_bfloat16* __restrict__ dgu, long long R, int F,
                                  const int* __restrict__ row_src) {
  const long long total = R * F;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / F;
    const int c = i % F;
    if (row_src && row_src[r] < 0) {
      dgu[r * 2 * F + c] = __float2bfloat16_rn(0.f);
      dgu[r * 2 * F + F + c] = __float2bfloat16_rn(0.f);
      continue;
    }
    const float g = __bfloat162float(gu[r * 2 * F + c]);
    const float u = __bfloat162float(gu[r * 2 * F + F + c]);
    const float d = __bfloat162float(dh[r * F + c]);
    const float sg = __fdividef(1.f, 1.f + __expf(-g));
    const float silu = g * sg;
    const float dsilu = sg * (1.f + g * (1.f - sg));
    dgu[r * 2 * F + c] = __float2bfloat16_rn(d * u * dsilu);
    dgu[r * 2 * F + F + c] = __float2bfloat16_rn(d * silu);
  }
}

// ---------------------------------------------------------------- embedding
// x[t, :] = float(wte[tok[t], :]);  wte bf16 or fp32.
template <typename WT>
__global__ void embed_fwd_kernel(const long long* __restrict__ tok, const WT* __restrict__ wte,
                                 float* __restrict__ x, int T, int D, int V, int* status) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
    long long id = tok[t];
    if (id < 0 || id >= V) {
      if (lane == 0) set_error(status, kErrBounds);
      id = 0;
    }
    for (int c = lane; c < D; c += 32) x[(long long)t * D + c] = to_f<WT>(wte[id * D + c]);
  }
}

// dwte[tok[t], :] += dx[t, :]
__global__ void embed_bwd_kernel(const long long* __restrict__ tok, const float* __restrict__ dx,
                                 float* __restrict__ dwte, int T, int D, int V) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
    const long long id = tok[t];
    if (id < 0 || id >= V) continue;
    for (int c = lane; c < D; c += 32) atomicAdd(dwte + id * D + c, dx[(long long)t * D + c]);
  }
}

int grid_for(long long work, int per_block) {
  long long g = (work + per_block - 1) / per_block;
  long long cap = (long long)num_sms() * 8;
  return (int)std::max(1LL, std::min(g, cap));
}

}  // namespace

// ============================================================== host API
void rmsnorm_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor y, torch::Tensor rstd, double eps) {
  HB_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous(), "rmsnorm: x must be contiguous fp32");
  const int D = x.size(-1);
  const int T = x.numel() / D;
  HB_CHECK(D % 4 == 0, "rmsnorm: D must be a multiple of 4");
  const int grid = grid_for(T, 8);
  if (y.scalar_type() == at::kBFloat16)
    rmsnorm_fwd_kernel<__nv_bfloat16><<<grid, 256, 0, cur_stream()>>>(
        x.data_ptr<float>(), w.data_ptr<float>(), (__nv_bfloat16*)y.data_ptr(),
        rstd.data_ptr<float>(), T, D, (float)eps);
  else
    rmsnorm_fwd_kernel<float><<<grid, 256, 0, cur_stream()>>>(
        x.data_ptr<float>(), w.data_ptr<float>(), y.data_ptr<float>(), rstd.data_ptr<float>(), T,
        D, (float)eps);
  HB_CUDA_CHECK(cudaGetLastError());
}

void rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd,
                 torch::Tensor dx, torch::Tensor dw, bool accumulate) {
  const int D = x.size(-1);
  const int T = x.numel() / D;
  HB_CHECK(D <= 32 * NORM_MAX_PER_LANE, "rmsnorm_bwd: D too large");
  HB_CHECK(dy.is_contiguous() && dx.is_contiguous(), "rmsnorm_bwd: contiguous tensors required");
  const int grid = std::min(grid_for(T, 8), num_sms() * 2);
  if (dy.scalar_type() == at::kBFloat16)
    rmsnorm_bwd_kernel<__nv_bfloat16><<<grid, 256, 0, cur_stream()>>>(
        (const __nv_bfloat16*)dy.data_ptr(), x.data_ptr<float>(), w.data_ptr<float>(),
        rstd.data_ptr<float>(), dx.data_ptr<float>(), dw.data_ptr<float>(), T, D, accumulate);
  else
    rmsnorm_bwd_kernel<float><<<grid, 256, 0, cur_stream()>>>(
        dy.data_ptr<float>(), x.data_ptr<float>(), w.data_ptr<float>(), rstd.data_ptr<float>(),
        dx.data_ptr<float>(), dw.data_ptr<float>(), T, D, accumulate);
  HB_CUDA_CHECK(cudaGetLastError());
}

void rope_apply(torch::Tensor q, torch::Tensor cos, torch::Tensor sin, int64_t seq_len,
                c10::optional<torch::Tensor> positions, bool inverse) {
  check_bf16(q, "q");
  HB_CHECK(q.is_contiguous() && q.dim() == 3, "rope: q must be contiguous [T, N, H]");
  const int T = q.size(0), N = q.size(1), H = q.size(2);
  const long long work = (long long)T * N * (H / 2);
  const long long* pos = positions.has_value() ? reinterpret_cast<long long*>(positions->data_ptr<int64_t>()) : nullptr;
  rope_kernel<<<grid_for(work, 256), 256, 0, cur_stream()>>>(
      (__nv_bfloat16*)q.data_ptr(), T, N, H, (int)seq_len, (const __nv_bfloat16*)cos.data_ptr(),
      (const __nv_bfloat16*)sin.data_ptr(), pos, inverse);
  HB_CUDA_CHECK(cudaGetLastError());
}

void swiglu_fwd(torch::Tensor gu, torch::Tensor h, c10::optional<torch::Tensor> row_src) {
  const long long R = gu.size(0);
  const int F = gu.size(1) / 2;
  HB_CHECK(F % 2 == 0 && gu.is_contiguous() && h.is_contiguous(), "swiglu_fwd: bad layout");
  if (R == 0) return;
  swiglu_fwd_kernel<<<grid_for(R * F / 2, 256), 256, 0, cur_stream()>>>(
      (const __nv_bfloat16*)gu.data_ptr(), (__nv_bfloat16*)h.data_ptr(), R, F,
      row_src.has_value() ? row_src->data_ptr<int>() : nullptr);
  HB_CUDA_CHECK(cudaGetLastError());
}

void swiglu_bwd(torch::Tensor dh, torch::Tensor gu, torch::Tensor dgu,
                c10::optional<torch::Tensor> row_src) {
  const long long R = gu.size(0);
  const int F = gu.size(1) / 2;
  if (R == 0) return;
  swiglu_bwd_kernel<<<grid_for(R * F, 256), 256, 0, cur_stream()>>>(
      (const __nv_bfloat16*)dh.data_ptr(), (const __nv_bfloat16*)gu.data_ptr(),
      (__nv_bfloat16*)dgu.data_ptr(), R, F, row_src.has_value() ? row_src->data_ptr<int>() : nullptr);
  HB_CUDA_CHECK(cudaGetLastError());
}

void embed_fwd(torch::Tensor tok, torch::Tensor wte, torch::Tensor x) {
  const int T = tok.numel(), V = wte.size(0), D = wte.size(1);
  HB_CHECK(tok.scalar_type() == at::kLong, "embed: tokens must be int64");
  const int grid = grid_for(T, 8);
  if (wte.scalar_type() == at::kBFloat16)
    embed_fwd_kernel<__nv_bfloat16><<<grid, 256, 0, cur_stream()>>>(
        reinterpret_cast<long long*>(tok.data_ptr<int64_t>()), (const __nv_bfloat16*)wte.data_ptr(), x.data_ptr<float>(), T, D,
        V, status_ptr());
  else
    embed_fwd_kernel<float><<<grid, 256, 0, cur_stream()>>>(
        reinterpret_cast<long long*>(tok.data_ptr<int64_t>()), wte.data_ptr<float>(), x.data_ptr<float>(), T, D, V,
        status_ptr());
  HB_CUDA_CHECK(cudaGetLastError());
}

void embed_bwd(torch::Tensor tok, torch::Tensor dx, torch::Tensor dwte) {
  const int T = tok.numel(), V = dwte.size(0), D = dwte.size(1);
  embed_bwd_kernel<<<grid_for(T, 8), 256, 0, cur_stream()>>>(
      reinterpret_cast<long long*>(tok.data_ptr<int64_t>()), dx.data_ptr<float>(), dwte.data_ptr<float>(), T, D, V);
  HB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace hb
