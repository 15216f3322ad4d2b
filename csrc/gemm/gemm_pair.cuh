// tcgen05 GEMM over CTA pairs (cta_group::2) for sm_100a:
//
//   C[M,N] (+)= A[M,K] * B[K,N]      pair tile 256 x 256, k-block 64
//
// A cluster of two CTAs shares one 256 x 256 tile: CTA r loads A rows
// [m0 + 128 r, +128) and B columns [n0 + 128 r, +128) of each k-block into its
// own shared memory; the leader (rank 0) issues tcgen05.mma.cta_group::2,
// which reads both CTAs' halves, and each CTA's TMEM holds its 128 accumulator
// rows x 256 columns.  Per SM this halves the B traffic of the 1-CTA kernel
// (48 KB -> 32 KB per k-block for the same math), which is what the 128 x 256
// tile was bound by.
//
// Synchronisation (no multicast anywhere):
//   full[s]   leader-only barrier: the leader expects both CTAs' bytes, both
//             CTAs' TMA loads complete on it (.cta_group::2 loads)
//   empty[s]  per CTA; the leader's MMA commit arrives on its own and, via the
//             mapa address, on the peer's
//   tfull[a]  per CTA; same double commit after a tile's last MMA
//   tempty[a] leader-only, 256 arrivals: both CTAs' epilogue threads
// Every wait is bounded (status word); the teardown is a cluster barrier so
// neither CTA leaves while the other may still signal it.
#pragma once
#include "gemm_kernel.cuh"

namespace hb {

// warp 0: TMA producer, warp 1: MMA issuer (leader CTA), warps 2..9: epilogue
// (two warps per TMEM lane quadrant, alternate 32-column chunks)
constexpr int PAIR_THREADS = 64 + 32 * GEMM_EPI_WARPS;
// K split into segments, each with its own K-major B (DENSE, !B_MN only):
// C = sum_s A[:, k_s .. k_s+1) B_s^T, one write of C.  nseg 0 = one B (tmB).
constexpr int KSEG_MAX = 6;
struct alignas(64) KSegMaps {
  CUtensorMap seg[KSEG_MAX];
  int seg_k[KSEG_MAX + 1];   // K start of each segment (multiples of 64), then K
  int nseg;
};

constexpr int PAIR_BM = 256;   // rows per pair tile (128 per CTA)
constexpr int PAIR_BN = 256;   // columns per pair tile (B: 128 per CTA)
constexpr int PAIR_A_BYTES = 128 * GEMM_BK * 2;
constexpr int PAIR_B_BYTES = 128 * GEMM_BK * 2;
constexpr int PAIR_STAGE_BYTES = PAIR_A_BYTES + PAIR_B_BYTES;
constexpr int PAIR_STAGES = 6;
constexpr int PAIR_TMEM_COLS = 2 * PAIR_BN;
constexpr int PAIR_SMEM = PAIR_STAGES * PAIR_STAGE_BYTES + 1024 + 256;

template <int MODE>
__device__ __forceinline__ bool get_pair_tile(const GemmArgs& a, int t, TileInfo& ti) {
  if (MODE == DENSE) {
    if (t >= a.num_tiles) return false;
    const int split = t % a.k_splits;
    const int tile = t / a.k_splits;
    const int mb = tile / a.tiles_n, nb = tile - mb * a.tiles_n;
    ti.m0 = mb * PAIR_BM;
    ti.n0 = nb * PAIR_BN;
    const int total_k = (a.K + GEMM_BK - 1) / GEMM_BK;
    const int per = (total_k + a.k_splits - 1) / a.k_splits;
    const int kb0 = split * per;
    ti.k0 = kb0 * GEMM_BK;
    ti.k_iters = max(0, min(per, total_k - kb0));
    ti.group = 0;
    ti.m_limit = a.M;
    return true;
  } else {  // GROUPED_K
    if (t >= a.num_tiles) return false;
    const int per = a.tiles_m * a.tiles_n;
    const int g = t / per;
    const int local = t - g * per;
    const int mb = local / a.tiles_n, nb = local - mb * a.tiles_n;
    ti.m0 = mb * PAIR_BM;
    ti.n0 = nb * PAIR_BN;
    ti.k0 = __ldg(a.grp_start + g);
    ti.k_iters = (__ldg(a.grp_count + g) + GEMM_BK - 1) / GEMM_BK;
    ti.group = g;
    ti.m_limit = a.M;
    return true;
  }
}

template <bool A_MN, bool B_MN, int MODE, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PAIR_THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const GemmArgs args, const __grid_constant__ KSegMaps ks) {
  static_assert(MODE == DENSE || MODE == GROUPED_K, "pair kernel: dense or grouped-K");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* bar_area = smem + PAIR_STAGES * PAIR_STAGE_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(bar_area);
  uint64_t* empty_bar = full_bar + PAIR_STAGES;
  uint64_t* tfull_bar = empty_bar + PAIR_STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x / 2, npairs = gridDim.x / 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < PAIR_STAGES; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&tfull_bar[i]), 1);
      mbar_init(smem_u32(&tempty_bar[i]), 2 * 32 * GEMM_EPI_WARPS);  // both CTAs' epilogue threads
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), PAIR_TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before either signals the other
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = pair; ok; t += npairs) {
        TileInfo ti;
        if (!get_pair_tile<MODE>(args, t, ti)) break;
        const int mr = ti.m0 + 128 * (int)rank;   // this CTA's A rows
        const int nr = ti.n0 + 128 * (int)rank;   // this CTA's B columns
        for (int kb = 0; kb < ti.k_iters; ++kb) {
          if (!mbar_wait(smem_u32(&empty_bar[stage]), phase ^ 1, args.status, kErrTimeoutProducer,
                         args.budget_ns)) {
            ok = false;
            break;
          }
          const uint32_t fb_local = smem_u32(&full_bar[stage]);
          const uint32_t fb = mapa_shared(fb_local, 0);
          if (leader) mbar_expect_tx(fb_local, 2 * PAIR_STAGE_BYTES);
          const uint32_t sa = smem_u32(smem + stage * PAIR_STAGE_BYTES);
          const uint32_t sb = sa + PAIR_A_BYTES;
          const int kc = ti.k0 + kb * GEMM_BK;
          if (!A_MN) {
            tma_load_2d_pair(sa, &tmA, fb, kc, mr);
          } else {
            tma_load_2d_pair(sa, &tmA, fb, mr, kc);
            tma_load_2d_pair(sa + 8192, &tmA, fb, mr + 64, kc);
          }
          if (!B_MN) {
            if (ks.nseg > 0) {
              int sg = 0;
              while (sg + 1 < ks.nseg && kc >= ks.seg_k[sg + 1]) ++sg;
              tma_load_2d_pair(sb, &ks.seg[sg], fb, kc - ks.seg_k[sg], nr);
            } else {
              tma_load_2d_pair(sb, &tmB, fb, kc, nr);
            }
          } else {
            tma_load_2d_pair(sb, &tmB, fb, nr, kc);
            tma_load_2d_pair(sb + 8192, &tmB, fb, nr + 64, kc);
          }
          if (++stage == PAIR_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (leader && elect_one()) {
      constexpr uint32_t idesc = make_idesc_bf16(PAIR_BM, PAIR_BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = pair; ok; t += npairs) {
        TileInfo ti;
        if (!get_pair_tile<MODE>(args, t, ti)) break;
        if (!mbar_wait(smem_u32(&tempty_bar[acc]), acc_phase ^ 1, args.status, kErrTimeoutMma,
                       args.budget_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * PAIR_BN;
        for (int kb = 0; kb < ti.k_iters; ++kb) {
          if (!mbar_wait(smem_u32(&full_bar[stage]), phase, args.status, kErrTimeoutMma, args.budget_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * PAIR_STAGE_BYTES);
          const uint32_t sb = sa + PAIR_A_BYTES;
#pragma unroll
          for (int kk = 0; kk < GEMM_BK / 16; ++kk) {
            const uint64_t ad = !A_MN ? make_smem_desc(sa + kk * 32, 16, 1024) : make_smem_desc(sa + kk * 2048, 8192, 1024);
            const uint64_t bd = !B_MN ? make_smem_desc(sb + kk * 32, 16, 1024) : make_smem_desc(sb + kk * 2048, 8192, 1024);
            umma_f16_pair(d_tmem, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          const uint32_t eb = smem_u32(&empty_bar[stage]);
          umma_commit_pair(eb);
          umma_commit_pair(mapa_shared(eb, 1));
          if (++stage == PAIR_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        const uint32_t tb = smem_u32(&tfull_bar[acc]);
        umma_commit_pair(tb);
        umma_commit_pair(mapa_shared(tb, 1));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const float alpha = args.alpha_ptr ? *args.alpha_ptr : args.alpha;
    const int row_in_tile = quad * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = pair;; t += npairs) {
      TileInfo ti;
      if (!get_pair_tile<MODE>(args, t, ti)) break;
      if (!mbar_wait(smem_u32(&tfull_bar[acc]), acc_phase, args.status, kErrTimeoutEpilogue, args.budget_ns))
        break;
      tc_fence_after();
      const int m = ti.m0 + 128 * (int)rank + row_in_tile;
      const bool row_ok = m < ti.m_limit;
      const bool has_k = ti.k_iters > 0;
      char* cbase = reinterpret_cast<char*>(args.C);
      if (MODE == GROUPED_K) cbase += (long long)ti.group * args.c_group_stride * (EPI == EPI_BF16 ? 2 : 4);
#pragma unroll 1
      for (int c = half; c < PAIR_BN / 32; c += 2) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * PAIR_BN + c * 32, r);
        tmem_ld_wait();
        const int n = ti.n0 + c * 32;
        if (!row_ok || n >= args.N) continue;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = has_k ? __uint_as_float(r[j]) * alpha : 0.f;
        const bool full = (n + 32 <= args.N);
        if (EPI == EPI_BF16) {
          __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(cbase) + (long long)m * args.ldc + n;
          if (full) {
            uint4* o4 = reinterpret_cast<uint4*>(out);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 w;
              w.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
              w.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
              w.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
              w.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
              o4[q] = w;
            }
          } else {
            for (int j = 0; j < 32 && n + j < args.N; ++j) out[j] = __float2bfloat16_rn(v[j]);
          }
        } else {
          float* out = reinterpret_cast<float*>(cbase) + (long long)m * args.ldc + n;
          if (MODE == DENSE && args.k_splits > 1) {
            if (has_k) {
              if (full) {
#pragma unroll
                for (int q = 0; q < 8; ++q)
                  atomicAdd(reinterpret_cast<float4*>(out) + q,
                            make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]));
              } else {
                for (int j = 0; j < 32 && n + j < args.N; ++j) atomicAdd(out + j, v[j]);
              }
            }
          } else if (full) {
            float4* o4 = reinterpret_cast<float4*>(out);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              float4 w = make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
              if (EPI == EPI_F32_ACC) {
                const float4 o = o4[q];
                w.x += o.x;
                w.y += o.y;
                w.z += o.z;
                w.w += o.w;
              }
              o4[q] = w;
            }
          } else {
            for (int j = 0; j < 32 && n + j < args.N; ++j) out[j] = (EPI == EPI_F32_ACC ? out[j] : 0.f) + v[j];
          }
        }
      }
      tc_fence_before();
      const uint32_t teb = smem_u32(&tempty_bar[acc]);
      if (leader) mbar_arrive(teb);
      else mbar_arrive_remote(mapa_shared(teb, 0));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no signal to either CTA is still in flight
  if (warp == 1) tmem_dealloc_pair(tmem_base, PAIR_TMEM_COLS);
}

template <bool A_MN, bool B_MN, int MODE, int EPI>
void gemm_pair_launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& args, int grid,
                      const KSegMaps* ks = nullptr) {
  auto kern = gemm_pair_kernel<A_MN, B_MN, MODE, EPI>;
  static bool configured = false;
  if (!configured) {
    HB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PAIR_SMEM));
    configured = true;
  }
  static const KSegMaps none{};
  kern<<<grid, PAIR_THREADS, PAIR_SMEM, cur_stream()>>>(ta, tb, args, ks ? *ks : none);
  HB_CUDA_CHECK(cudaGetLastError());
}

void gemm_dispatch_pair(int mode, bool a_mn, bool b_mn, int epi, const CUtensorMap& ta, const CUtensorMap& tb,
                        const GemmArgs& args, int grid, const KSegMaps* ks = nullptr);

}  // namespace hb
