// Cross-entropy over a chunk of logits and the fused optimizer update.
//
// CE (train.py:191-196): per row, loss = logsumexp(z) - z[target]; the kernel
// also writes the row's gradient (softmax(z) - onehot(target)) * scale in bf16
// so the head's backward GEMMs read it directly; the [T, V] logits of a whole
// batch are never resident (the caller walks token chunks).
//
// Optimizer (optimizer.py:126-155): one pass over the flat fp32 shard reads
// grad, master and moments, applies the global-norm clip coefficient (a device
// scalar, so no host sync), Lion or AdamW with lr-scaled decoupled decay, and
// writes master, moments and the compute-dtype working copy.
#include <torch/extension.h>

#include "../common/host.h"
#include "../common/sm100.cuh"

namespace hb {

namespace {

__device__ __forceinline__ float block_reduce_sum(float v, float* sh) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) sh[w] = v;
  __syncthreads();
  float r = (threadIdx.x < (blockDim.x >> 5)) ? sh[threadIdx.x] : 0.f;
  if (w == 0) r = warp_sum(r);
  if (threadIdx.x == 0) sh[0] = r;
  __syncthreads();
  float out = sh[0];
  __syncthreads();
  return out;
}

__device__ __forceinline__ float block_reduce_max(float v, float* sh) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) sh[w] = v;
  __syncthreads();
  float r = (threadIdx.x < (blockDim.x >> 5)) ? sh[threadIdx.x] : -INFINITY;
  if (w == 0) r = warp_max(r);
  if (threadIdx.x == 0) sh[0] = r;
  __syncthreads();
  float out = sh[0];
  __syncthreads();
  return out;
}

// logits: [T, V] fp32; targets: [T] int64; valid: [T] fp32 or null;
// loss_sum: scalar fp32 accumulated; dlogits: [T, V] bf16 = (p - onehot) * scale * valid.
__global__ void ce_fwd_bwd_kernel(const float* __restrict__ logits, const long long* __restrict__ tgt,
                                  const float* __restrict__ valid, float* __restrict__ loss_sum,
                                  __nv_bfloat16* __restrict__ dlogits, int T, int V, float scale,
                                  int* status) {
  __shared__ float sh[32];
  for (int row = blockIdx.x; row < T; row += gridDim.x) {
    const float* z = logits + (long long)row * V;
    float m = -INFINITY;
    for (int c = threadIdx.x * 4; c < V; c += blockDim.x * 4) {
      float4 v = *reinterpret_cast<const float4*>(z + c);
      m = fmaxf(m, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
    }
    m = block_reduce_max(m, sh);
    float s = 0.f;
    for (int c = threadIdx.x * 4; c < V; c += blockDim.x * 4) {
      float4 v = *reinterpret_cast<const float4*>(z + c);
      s += __expf(v.x - m) + __expf(v.y - m) + __expf(v.z - m) + __expf(v.w - m);
    }
    s = block_reduce_sum(s, sh);
    const float lse = m + __logf(s);
    long long t = tgt[row];
    float vw = valid ? valid[row] : 1.f;
    if (!index_ok(t, V, status)) {   // a label outside the vocabulary: row skipped
      t = -4;
      vw = 0.f;
    }
    if (threadIdx.x == 0 && t >= 0) atomicAdd(loss_sum, (lse - z[t]) * vw);
    const float inv = 1.f / s;
    const float g = scale * vw;
    __nv_bfloat16* d = dlogits + (long long)row * V;
    for (int c = threadIdx.x * 4; c < V; c += blockDim.x * 4) {
      float4 v = *reinterpret_cast<const float4*>(z + c);
      float p0 = __expf(v.x - m) * inv, p1 = __expf(v.y - m) * inv;
      float p2 = __expf(v.z - m) * inv, p3 = __expf(v.w - m) * inv;
      if (c == (t & ~3LL)) {
        const int o = t & 3;
        if (o == 0) p0 -= 1.f;
        if (o == 1) p1 -= 1.f;
        if (o == 2) p2 -= 1.f;
        if (o == 3) p3 -= 1.f;
      }
      uint2 w;
      w.x = pack_bf16x2(p0 * g, p1 * g);
      w.y = pack_bf16x2(p2 * g, p3 * g);
      *reinterpret_cast<uint2*>(d + c) = w;
    }
  }
}

// Sum of squares over several flat fp32 buffers -> out (fp32 scalar, atomics).
__global__ void sumsq_kernel(const float* __restrict__ a, long long n, float* out) {
  __shared__ float sh[32];
  float s = 0.f;
  for (long long i = (blockIdx.x * (long long)blockDim.x + threadIdx.x) * 4; i < n;
       i += (long long)gridDim.x * blockDim.x * 4) {
    if (i + 3 < n) {
      float4 v = *reinterpret_cast<const float4*>(a + i);
      s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    } else {
      for (long long j = i; j < n; ++j) s += a[j] * a[j];
    }
  }
  s = block_reduce_sum(s, sh);
  if (threadIdx.x == 0) atomicAdd(out, s);
}

// mode 0 = AdamW, 1 = Lion.  coef_ptr: device scalar clip multiplier.
template <typename WorkT, typename MT>
__global__ void fused_update_kernel(float* __restrict__ p, const float* __restrict__ g,
                                    MT* __restrict__ m, float* __restrict__ v,
                                    const float* __restrict__ decay, WorkT* __restrict__ work,
                                    long long n, int mode, float lr, float wd, float b1, float b2,
                                    float eps, float bc1, float bc2,
                                    const float* __restrict__ coef_ptr) {
  const float coef = *coef_ptr;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float gg = g[i] * coef;
    float pv = p[i];
    const float dec = decay[i];
    if (mode == 0) {
      const float mm = b1 * (float)m[i] + (1.f - b1) * gg;
      const float vv = b2 * v[i] + (1.f - b2) * gg * gg;
      m[i] = (MT)mm;
      v[i] = vv;
      const float upd = (mm / bc1) / (sqrtf(vv / bc2) + eps);
      pv = pv - lr * upd - lr * wd * pv * dec;
    } else {
      const float mf = (float)m[i];
      const float c = (1.f - b1) * gg + b1 * mf;
      const float u = (c > 0.f) ? 1.f : ((c < 0.f) ? -1.f : 0.f);
      m[i] = (MT)(b2 * mf + (1.f - b2) * gg);
      pv = pv - lr * u - lr * wd * pv * dec;
    }
    p[i] = pv;
    work[i] = (WorkT)pv;
  }
}

int grid_for(long long work, int per_block) {
  long long g = (work + per_block - 1) / per_block;
  long long cap = (long long)num_sms() * 8;
  return (int)std::max(1LL, std::min(g, cap));
}

}  // namespace

void ce_fwd_bwd(torch::Tensor logits, torch::Tensor tgt, c10::optional<torch::Tensor> valid,
                torch::Tensor loss_sum, torch::Tensor dlogits, double scale) {
  HB_CHECK(logits.scalar_type() == at::kFloat && logits.is_contiguous(), "ce: fp32 logits");
  const int T = logits.size(0), V = logits.size(1);
  HB_CHECK(V % 4 == 0, "ce: vocab must be a multiple of 4");
  if (T == 0) return;
  const float* vp = valid.has_value() ? valid->data_ptr<float>() : nullptr;
  const int grid = std::min(T, num_sms() * 4);
  ce_fwd_bwd_kernel<<<grid, 512, 0, cur_stream()>>>(
      logits.data_ptr<float>(), reinterpret_cast<long long*>(tgt.data_ptr<int64_t>()), vp, loss_sum.data_ptr<float>(),
      (__nv_bfloat16*)dlogits.data_ptr(), T, V, (float)scale, status_ptr());
  HB_CUDA_CHECK(cudaGetLastError());
}

void sumsq(torch::Tensor a, torch::Tensor out) {
  HB_CHECK(a.scalar_type() == at::kFloat && a.is_contiguous(), "sumsq: contiguous fp32");
  const long long n = a.numel();
  if (n == 0) return;
  HB_CHECK((reinterpret_cast<uintptr_t>(a.data_ptr()) & 15) == 0, "sumsq: 16-byte aligned input");
  sumsq_kernel<<<grid_for(n / 4 + 1, 256), 256, 0, cur_stream()>>>(a.data_ptr<float>(), n,
                                                                     out.data_ptr<float>());
  HB_CUDA_CHECK(cudaGetLastError());
}

void fused_update(torch::Tensor p, torch::Tensor g, torch::Tensor m, c10::optional<torch::Tensor> v,
                  torch::Tensor decay, torch::Tensor work, int64_t mode, double lr, double wd,
                  double b1, double b2, double eps, int64_t step, torch::Tensor coef) {
  const long long n = p.numel();
  if (n == 0) return;
  const float bc1 = mode == 0 ? (float)(1.0 - std::pow(b1, (double)step)) : 1.f;
  const float bc2 = mode == 0 ? (float)(1.0 - std::pow(b2, (double)step)) : 1.f;
  float* vp = v.has_value() ? v->data_ptr<float>() : nullptr;
  HB_CHECK(mode == 1 || vp != nullptr, "AdamW needs the second moment");
  const int grid = grid_for(n, 256);
  auto launch = [&](auto* wptr, auto* mptr) {
    using W = std::remove_pointer_t<decltype(wptr)>;
    using M = std::remove_pointer_t<decltype(mptr)>;
    fused_update_kernel<W, M><<<grid, 256, 0, cur_stream()>>>(
        p.data_ptr<float>(), g.data_ptr<float>(), mptr, vp, decay.data_ptr<float>(), wptr, n,
        (int)mode, (float)lr, (float)wd, (float)b1, (float)b2, (float)eps, bc1, bc2,
        coef.data_ptr<float>());
  };
  const bool wb = work.scalar_type() == at::kBFloat16;
  const bool mb = m.scalar_type() == at::kBFloat16;
  if (wb && mb) launch((__nv_bfloat16*)work.data_ptr(), (__nv_bfloat16*)m.data_ptr());
  else if (wb) launch((__nv_bfloat16*)work.data_ptr(), m.data_ptr<float>());
  else if (mb) launch(work.data_ptr<float>(), (__nv_bfloat16*)m.data_ptr());
  else launch(work.data_ptr<float>(), m.data_ptr<float>());
  HB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace hb
