// Expert-parallel MoE transport over NVLink peer memory (fused dispatch /
// return), capacity-factor layout.
//
// Ranks r = 0..E-1 each own Nl = N / E experts (global expert e lives on rank
// e / Nl as local expert e % Nl).  Every rank owns, in symmetric memory,
//   recv [Nl][E][cap][D]   rows sent TO its experts, block (le, src)
//   ret  [N][cap][D]       expert outputs returned to it, block e (global)
// A source's (token, slot) routed to expert e keeps its rank i inside that
// expert's token-ordered list (the local stable plan); i >= cap is dropped.
//   ep_scatter     row (x[t], or w_tk * dout[t] in the backward, with the dot
//                  <dout[t], ret[e][i]> for the weight gradient) -> peer recv
//   ep_zero_pads   rows [kept_e, cap) of every block this source owns on each
//                  peer are zeroed and kept_e is written to the peer's counts
//   ep_return      rows [0, cnt) of every (le, src) block -> peer src's ret
//   ep_combine     out[t] += sum_k bf16(w_tk) * ret[e][i]   (kept slots)
//   ep_gather_add  dx[t] += sum_k ret[e][i]                  (kept slots)
// All peer traffic is plain loads/stores (no TMA, no multicast); phases are
// separated by the bounded device barrier of comm/p2p.cu.
#include <torch/extension.h>

#include "../common/host.h"
#include "../common/sm100.cuh"

namespace hb {
namespace {

int grid_for(long long work, int per_block) {
  long long g = (work + per_block - 1) / per_block;
  return (int)std::max(1LL, std::min(g, (long long)num_sms() * 16));
}

// slot -> (global expert, rank within the expert's list); -1 when dropped.
// An expert id outside [0, n_exp) (it would pick a peer pointer and a row
// from outside the tables) drops the slot.
__device__ __forceinline__ int slot_rank(const int* pos, const int* starts, const int* topi, long long s,
                                         int cap, int n_exp, int& e) {
  e = topi[s];
  if (e < 0 || e >= n_exp) return -1;
  const int i = pos[s] - starts[e];
  return i >= 0 && i < cap ? i : -1;
}

// one warp per slot
__global__ void scatter_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ dout,
                               const float* __restrict__ w, const __nv_bfloat16* __restrict__ ret,
                               float* __restrict__ dw, const int* __restrict__ topi,
                               const int* __restrict__ pos, const int* __restrict__ starts,
                               const long long* __restrict__ peers, int T, int K, int D, int me, int E,
                               int Nl, int cap, int backward) {
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  for (long long s = blockIdx.x * (long long)warps + (threadIdx.x >> 5); s < (long long)T * K;
       s += (long long)gridDim.x * warps) {
    int e;
    const int i = slot_rank(pos, starts, topi, s, cap, E * Nl, e);
    const long long t = s / K;
    if (i < 0) {
      if (backward && lane == 0) dw[s] = 0.f;
      continue;
    }
    const int dest = e / Nl, le = e % Nl;
    __nv_bfloat16* drow = reinterpret_cast<__nv_bfloat16*>(peers[dest]) +
                          (((long long)le * E + me) * cap + i) * D;
    if (!backward) {
      const uint4* src = reinterpret_cast<const uint4*>(x + t * D);
      for (int c = lane; c < D / 8; c += 32) reinterpret_cast<uint4*>(drow)[c] = src[c];
    } else {
      const float wk = __bfloat162float(__float2bfloat16_rn(w[s]));
      const __nv_bfloat16* yrow = ret + ((long long)e * cap + i) * D;
      float dot = 0.f;
      for (int c = lane * 2; c < D; c += 64) {
        const float g0 = dout[t * D + c], g1 = dout[t * D + c + 1];
        const __nv_bfloat162 yv = *reinterpret_cast<const __nv_bfloat162*>(yrow + c);
        dot += g0 * __bfloat162float(yv.x) + g1 * __bfloat162float(yv.y);
        *reinterpret_cast<__nv_bfloat162*>(drow + c) = __floats2bfloat162_rn(wk * g0, wk * g1);
      }
      dot = warp_sum(dot);
      if (lane == 0) dw[s] = dot;
    }
  }
}

// blocks: one per global expert e; zero rows [kept, cap) of block (le, me) on
// the owner, and publish kept to the owner's counts [Nl][E].
__global__ void zero_pads_kernel(const int* __restrict__ counts, const long long* __restrict__ peers,
                                 const long long* __restrict__ count_peers, int D, int me, int E, int Nl,
                                 int cap) {
  const int e = blockIdx.x;
  const int dest = e / Nl, le = e % Nl;
  const int kept = min(counts[e], cap);
  __nv_bfloat16* base = reinterpret_cast<__nv_bfloat16*>(peers[dest]) + ((long long)le * E + me) * cap * D;
  const long long n = (long long)(cap - kept) * D / 8;
  uint4* p = reinterpret_cast<uint4*>(base + (long long)kept * D);
  for (long long j = threadIdx.x; j < n; j += blockDim.x) p[j] = make_uint4(0, 0, 0, 0);
  if (threadIdx.x == 0 && count_peers)
    reinterpret_cast<int*>(count_peers[dest])[le * E + me] = kept;
}

// rows of block (le, src), i < cnt[le][src], -> peer src's ret[(me*Nl+le)][i]
__global__ void return_kernel(const __nv_bfloat16* __restrict__ rows, const int* __restrict__ cnt,
                              const long long* __restrict__ peers, int D, int me, int E, int Nl, int cap) {
  const int blk = blockIdx.y;  // le * E + src
  const int le = blk / E, src = blk % E;
  const int n = cnt[blk];
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(peers[src]) + ((long long)(me * Nl + le) * cap) * D;
  const __nv_bfloat16* s0 = rows + (long long)blk * cap * D;
  for (int i = blockIdx.x * warps + (threadIdx.x >> 5); i < n; i += gridDim.x * warps) {
    const uint4* sr = reinterpret_cast<const uint4*>(s0 + (long long)i * D);
    uint4* dr = reinterpret_cast<uint4*>(dst + (long long)i * D);
    for (int c = lane; c < D / 8; c += 32) dr[c] = sr[c];
  }
}

// out[t] += sum_k (w? bf16(w_tk) : 1) * ret[e][i]   over kept slots.
// One warp per token: lanes 0..K-1 resolve the token's K (expert, row) pairs
// once, the pairs are broadcast into registers, then each lane streams two
// columns at a time (K <= MK).
constexpr int EP_MAXK = 16;
template <int MK>
__global__ void combine_kernel(const __nv_bfloat16* __restrict__ ret, const float* __restrict__ w,
                               const int* __restrict__ topi, const int* __restrict__ pos,
                               const int* __restrict__ starts, float* __restrict__ out, int T, int K, int D,
                               int cap, int n_exp) {
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  for (long long t = blockIdx.x * (long long)warps + (threadIdx.x >> 5); t < T;
       t += (long long)gridDim.x * warps) {
    int my_row = -1;
    float my_w = 0.f;
    if (lane < K) {
      int e;
      const int i = slot_rank(pos, starts, topi, t * K + lane, cap, n_exp, e);
      if (i >= 0) {
        my_row = e * cap + i;
        my_w = w ? __bfloat162float(__float2bfloat16_rn(w[t * K + lane])) : 1.f;
      }
    }
    int rows[MK];
    float wk[MK];
#pragma unroll
    for (int k = 0; k < MK; ++k) {
      rows[k] = __shfl_sync(0xffffffffu, my_row, k);
      wk[k] = __shfl_sync(0xffffffffu, my_w, k);
    }
    for (int c = lane * 2; c < D; c += 64) {
      float a0 = 0.f, a1 = 0.f;
#pragma unroll
      for (int k = 0; k < MK; ++k) {
        if (k < K && rows[k] >= 0) {
          const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(ret + (long long)rows[k] * D + c);
          a0 += wk[k] * __bfloat162float(v.x);
          a1 += wk[k] * __bfloat162float(v.y);
        }
      }
      float2* o = reinterpret_cast<float2*>(out + t * D + c);
      const float2 prev = *o;
      *o = make_float2(prev.x + a0, prev.y + a1);
    }
  }
}

}  // namespace

void ep_scatter(torch::Tensor x, c10::optional<torch::Tensor> dout, c10::optional<torch::Tensor> w,
                c10::optional<torch::Tensor> ret, c10::optional<torch::Tensor> dw, torch::Tensor topi,
                torch::Tensor pos, torch::Tensor starts, torch::Tensor peers, int64_t me, int64_t E,
                int64_t Nl, int64_t cap, bool backward) {
  const int T = topi.size(0), K = topi.size(1), D = x.size(1);
  HB_CHECK(D % 8 == 0, "ep_scatter: D % 8");
  scatter_kernel<<<grid_for((long long)T * K, 8), 256, 0, cur_stream()>>>(
      (const __nv_bfloat16*)x.data_ptr(), dout.has_value() ? dout->data_ptr<float>() : nullptr,
      w.has_value() ? w->data_ptr<float>() : nullptr,
      ret.has_value() ? (const __nv_bfloat16*)ret->data_ptr() : nullptr,
      dw.has_value() ? dw->data_ptr<float>() : nullptr, topi.data_ptr<int>(), pos.data_ptr<int>(),
      starts.data_ptr<int>(), reinterpret_cast<const long long*>(peers.data_ptr<int64_t>()), T, K, D,
      (int)me, (int)E, (int)Nl, (int)cap, backward ? 1 : 0);
  HB_CUDA_CHECK(cudaGetLastError());
}

void ep_zero_pads(torch::Tensor counts, torch::Tensor peers, c10::optional<torch::Tensor> count_peers,
                  int64_t D, int64_t me, int64_t E, int64_t Nl, int64_t cap) {
  const int N = counts.numel();
  zero_pads_kernel<<<N, 256, 0, cur_stream()>>>(
      counts.data_ptr<int>(), reinterpret_cast<const long long*>(peers.data_ptr<int64_t>()),
      count_peers.has_value() ? reinterpret_cast<const long long*>(count_peers->data_ptr<int64_t>()) : nullptr,
      (int)D, (int)me, (int)E, (int)Nl, (int)cap);
  HB_CUDA_CHECK(cudaGetLastError());
}

void ep_return(torch::Tensor rows, torch::Tensor cnt, torch::Tensor peers, int64_t me, int64_t E, int64_t Nl,
               int64_t cap) {
  const int D = rows.size(-1);
  dim3 grid(std::max(1, (int)std::min<long long>(64, (cap + 7) / 8)), (int)(Nl * E));
  return_kernel<<<grid, 256, 0, cur_stream()>>>((const __nv_bfloat16*)rows.data_ptr(), cnt.data_ptr<int>(),
                                                reinterpret_cast<const long long*>(peers.data_ptr<int64_t>()),
                                                D, (int)me, (int)E, (int)Nl, (int)cap);
  HB_CUDA_CHECK(cudaGetLastError());
}

void ep_combine(torch::Tensor ret, c10::optional<torch::Tensor> w, torch::Tensor topi, torch::Tensor pos,
                torch::Tensor starts, torch::Tensor out, int64_t cap) {
  const int T = topi.size(0), K = topi.size(1), D = out.size(1);
  HB_CHECK(K <= EP_MAXK && D % 2 == 0 && out.is_contiguous(), "ep_combine: K <= 16, even D, contiguous out");
  HB_CHECK((long long)starts.numel() * cap < (1LL << 31), "ep_combine: row index range");
  auto kern = K <= 8 ? combine_kernel<8> : combine_kernel<EP_MAXK>;
  kern<<<grid_for(T, 8), 256, 0, cur_stream()>>>(
      (const __nv_bfloat16*)ret.data_ptr(), w.has_value() ? w->data_ptr<float>() : nullptr,
      topi.data_ptr<int>(), pos.data_ptr<int>(), starts.data_ptr<int>(), out.data_ptr<float>(), T, K, D,
      (int)cap, (int)starts.numel());
  HB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace hb
