// Fused data-parallel gradient / weight exchange over NVLink peer memory.
//
// The gradient and working-weight buffers of every rank live in symmetric
// memory, so each rank holds the device addresses of its peers' buffers.
//   p2p_barrier          every rank stores `epoch` into slot [my_rank] of each
//                        peer's signal pad (release, system scope) and waits,
//                        bounded, until all slots of its own pad reach `epoch`
//   p2p_reduce_scatter   grad[lo:hi] = scale * sum_r peer_grad_r[lo:hi]
//                        (peer loads over NVLink, fp32), plus sum of squares
//   p2p_update_bcast     Lion / AdamW on the shard; the new working value is
//                        stored into the working copy of EVERY rank (peer
//                        stores), which replaces the parameter all-gather
// Plain ld/st to peer addresses only: no TMA, no multicast.  A wait that runs
// out of budget records kErrTimeoutPeer in the status word and returns; the
// reduce-scatter and update kernels read the status word first and do nothing
// (no peer load or store) once any earlier kernel recorded an error, so a rank
// whose peers stopped never reads gradients that may not be final.
#include <torch/extension.h>

#include "../common/host.h"
#include "../common/sm100.cuh"

namespace hb {
namespace {

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void barrier_kernel(const long long* __restrict__ pads, int rank, int world, unsigned epoch,
                               int* status, unsigned long long budget_ns) {
  const int r = threadIdx.x;
  __threadfence_system();
  if (r < world) {
    unsigned* peer = reinterpret_cast<unsigned*>(pads[r]);
    st_release_sys(peer + rank, epoch);
  }
  __syncthreads();
  if (r < world) {
    const unsigned* mine = reinterpret_cast<const unsigned*>(pads[rank]);
    const uint64_t t0 = globaltimer();
    while ((int)(ld_acquire_sys(mine + r) - epoch) < 0) {
      if (globaltimer() - t0 > budget_ns) {
        set_error(status, kErrTimeoutPeer);
        break;
      }
    }
  }
  __syncthreads();
  __threadfence_system();
}

__device__ __forceinline__ float block_sum(float v) {
  __shared__ float sh[32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) sh[w] = v;
  __syncthreads();
  v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
  if (w == 0) v = warp_sum(v);
  return v;
}

// out[i] = scale * sum_r peers[r][off + i]  (float4 vectorised); sumsq += out^2
__global__ void reduce_scatter_kernel(const long long* __restrict__ peers, int world, long long off,
                                      long long n, float* __restrict__ out, float scale,
                                      float* __restrict__ sumsq, const int* __restrict__ status) {
  if (*reinterpret_cast<const volatile int*>(status) != 0) return;
  float ss = 0.f;
  const long long n4 = n / 4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < world; ++r) {
      const float4 v = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(peers[r]) + off)[i];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    acc.x *= scale;
    acc.y *= scale;
    acc.z *= scale;
    acc.w *= scale;
    reinterpret_cast<float4*>(out)[i] = acc;
    ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
  }
  for (long long i = n4 * 4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    float a = 0.f;
    for (int r = 0; r < world; ++r) a += reinterpret_cast<const float*>(peers[r])[off + i];
    a *= scale;
    out[i] = a;
    ss += a * a;
  }
  ss = block_sum(ss);
  if (threadIdx.x == 0) atomicAdd(sumsq, ss);
}

// Optimizer step on the shard; the working value goes to every rank.
template <typename WorkT, typename MT>
__global__ void update_bcast_kernel(float* __restrict__ p, const float* __restrict__ g, MT* __restrict__ m,
                                    float* __restrict__ v, const float* __restrict__ decay,
                                    const long long* __restrict__ work_peers, int world, long long off,
                                    long long n, int mode, float lr, float wd, float b1, float b2,
                                    float eps, float bc1, float bc2, const float* __restrict__ coef_ptr,
                                    const int* __restrict__ status) {
  if (*reinterpret_cast<const volatile int*>(status) != 0) return;
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
      pv = pv - lr * ((mm / bc1) / (sqrtf(vv / bc2) + eps)) - lr * wd * pv * dec;
    } else {
      const float mf = (float)m[i];
      const float c = (1.f - b1) * gg + b1 * mf;
      const float u = (c > 0.f) ? 1.f : ((c < 0.f) ? -1.f : 0.f);
      m[i] = (MT)(b2 * mf + (1.f - b2) * gg);
      pv = pv - lr * u - lr * wd * pv * dec;
    }
    p[i] = pv;
    const WorkT wv = (WorkT)pv;
    for (int r = 0; r < world; ++r) reinterpret_cast<WorkT*>(work_peers[r])[off + i] = wv;
  }
}

int grid_for(long long work, int per_block) {
  long long gsz = (work + per_block - 1) / per_block;
  return (int)std::max(1LL, std::min(gsz, (long long)num_sms() * 8));
}

}  // namespace

void p2p_barrier(torch::Tensor pads, int64_t rank, int64_t world, int64_t epoch) {
  HB_CHECK(world <= 1024, "p2p_barrier: world too large");
  barrier_kernel<<<1, 1024 >= world ? (int)((world + 31) / 32 * 32) : 1024, 0, cur_stream()>>>(
      reinterpret_cast<const long long*>(pads.data_ptr<int64_t>()), (int)rank, (int)world,
      (unsigned)epoch, status_ptr(), peer_wait_budget_ns());
  HB_CUDA_CHECK(cudaGetLastError());
}

void p2p_reduce_scatter(torch::Tensor peers, int64_t world, int64_t off, int64_t n, torch::Tensor out,
                        double scale, torch::Tensor sumsq) {
  HB_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous(), "p2p_reduce_scatter: fp32 out");
  HB_CHECK(off % 4 == 0, "p2p_reduce_scatter: offset must be 16-byte aligned");
  if (n == 0) return;
  reduce_scatter_kernel<<<grid_for(n / 4 + 1, 256), 256, 0, cur_stream()>>>(
      reinterpret_cast<const long long*>(peers.data_ptr<int64_t>()), (int)world, off, n,
      out.data_ptr<float>(), (float)scale, sumsq.data_ptr<float>(), status_ptr());
  HB_CUDA_CHECK(cudaGetLastError());
}

void p2p_update_bcast(torch::Tensor p, torch::Tensor g, torch::Tensor m, c10::optional<torch::Tensor> v,
                      torch::Tensor decay, torch::Tensor work_peers, int64_t world, int64_t off,
                      bool work_bf16, int64_t mode, double lr, double wd, double b1, double b2, double eps,
                      int64_t step, torch::Tensor coef) {
  const long long n = p.numel();
  if (n == 0) return;
  const float bc1 = mode == 0 ? (float)(1.0 - std::pow(b1, (double)step)) : 1.f;
  const float bc2 = mode == 0 ? (float)(1.0 - std::pow(b2, (double)step)) : 1.f;
  float* vp = v.has_value() ? v->data_ptr<float>() : nullptr;
  const long long* wp = reinterpret_cast<const long long*>(work_peers.data_ptr<int64_t>());
  const int grid = grid_for(n, 256);
  auto launch = [&](auto wtag, auto* mptr) {
    using W = decltype(wtag);
    using M = std::remove_pointer_t<decltype(mptr)>;
    update_bcast_kernel<W, M><<<grid, 256, 0, cur_stream()>>>(
        p.data_ptr<float>(), g.data_ptr<float>(), mptr, vp, decay.data_ptr<float>(), wp, (int)world, off,
        n, (int)mode, (float)lr, (float)wd, (float)b1, (float)b2, (float)eps, bc1, bc2,
        coef.data_ptr<float>(), status_ptr());
  };
  const bool mb = m.scalar_type() == at::kBFloat16;
  if (work_bf16 && mb) launch(__nv_bfloat16(), (__nv_bfloat16*)m.data_ptr());
  else if (work_bf16) launch(__nv_bfloat16(), m.data_ptr<float>());
  else if (mb) launch(float(), (__nv_bfloat16*)m.data_ptr());
  else launch(float(), m.data_ptr<float>());
  HB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace hb
