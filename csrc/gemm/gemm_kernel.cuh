// tcgen05 GEMM for sm_100a: bf16 operands, fp32 TMEM accumulators.
//
//   C[M,N] (+)= A[M,K] * B[K,N]
//
// Persistent kernel, one CTA per SM, 6 warps with fixed roles:
//   warp 0      TMA producer (one elected lane) filling a STAGES-deep smem ring
//   warp 1      TMEM allocator + MMA issuer (one elected lane, tcgen05.mma)
//   warps 2..5  epilogue: tcgen05.ld of the 128xBN fp32 tile, convert, store
// Two TMEM accumulators (2*BN columns) let the epilogue of tile i overlap the
// main loop of tile i+1.
//
// Operand majorness is a template choice so that all three products of a
// linear layer run without transposes:
//   forward  y  = x  @ W     A K-major (x [M,K]),  B MN-major (W [K,N])
//   grad-in  dx = dy @ W^T   A K-major (dy [M,N]), B K-major  (W read as [N,K])
//   grad-W   dW = x^T @ dy   A MN-major (x [K,M]), B MN-major (dy [K,N])
//
// Modes
//   DENSE      one problem
//   GROUPED_M  MoE expert GEMMs: rows of A/C are partitioned into groups whose
//              starts are multiples of 128 (the dispatch pads each expert's
//              segment), each group multiplies its own B[g]; tile counts per
//              group come from a device prefix array so no host sync is needed
//   GROUPED_K  MoE expert weight gradients: the contraction runs over each
//              group's (padded) row segment, C[g] = A_g^T B_g
#pragma once
#include <torch/extension.h>

#include "../common/host.h"
#include "../common/sm100.cuh"

namespace hb {

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
// warp 0: TMA producer, warp 1: MMA issuer, warps 2..9: epilogue.  Two
// epilogue warps share each TMEM lane quadrant (alternate 32-column chunks),
// so twice the loads and stores are in flight per SM as with one warp each.
constexpr int GEMM_EPI_WARPS = 8;
constexpr int GEMM_THREADS = 64 + 32 * GEMM_EPI_WARPS;

enum GemmMode { DENSE = 0, GROUPED_M = 1, GROUPED_K = 2 };
// EPI_SWIGLU_BWD (grouped-over-M only): the accumulator is dh = dY W_down^T
// for the rows of a SwiGLU; the epilogue reads g, u from args.aux ([R, 2F]
// bf16, the forward's gate | up) and writes dgu = [dh u silu'(g) | dh silu(g)]
// (bf16, ldc = 2F); the pad rows of each expert's 128-row segment get zeros.
// EPI_SWIGLU_FWD (grouped-over-M, MN-major B, BN 256 only): virtual N = 2F;
// tile j loads columns [128 j, 128 j + 128) of W_gate (tmB) and of W_up
// (GatherMaps::b_hi), so TMEM holds g and u of the same 128 columns; the
// epilogue writes h = bf16(silu(g)) * u to C ([R, F]) and g | u (bf16) to
// args.c2 ([R, 2F]); pad rows of each expert segment get h = 0.
enum GemmEpi { EPI_BF16 = 0, EPI_F32 = 1, EPI_F32_ACC = 2, EPI_SWIGLU_BWD = 3, EPI_SWIGLU_FWD = 4 };

struct GemmArgs {
  int M, N, K;
  int tiles_m, tiles_n;
  int num_tiles;                // DENSE / GROUPED_K; GROUPED_M reads grp_tile_start[G]
  int k_splits;                 // DENSE: split the K loop over CTAs (fp32 atomic epilogue)
  int num_groups;
  const int* grp_start;         // GROUPED_M: row start; GROUPED_K: k start
  const int* grp_count;         // rows / k per group
  const int* grp_tile_start;    // GROUPED_M: prefix of tiles per group [G+1]
  void* C;
  long long ldc;
  long long c_group_stride;     // GROUPED_K: elements between C[g] and C[g+1]
  float alpha;
  const float* alpha_ptr;       // optional device scalar; overrides alpha
  const void* aux;              // EPI_SWIGLU_BWD: gate | up of the forward
  void* c2;                     // EPI_SWIGLU_FWD: g | u output
  long long ldc2;
  int k_split_b;                // GROUPED_M, K-major B: K at or past this comes from
                                // GatherMaps::b_hi (at k - k_split_b); 0 = one B
  int* status;
  unsigned long long budget_ns;
};

// Fused all-gather of the B operand (FSDP expert weights), GROUPED_M only.
// B[g] lives on rank g / groups_per_rank (its shard of groups); every B tile
// (group, k-block, n-block) is fetched ONCE per GPU (over NVLink unless this
// GPU owns it): the first CTA that needs it claims flags[tile] (0 -> 1), TMA-loads it
// from the owner's memory into its smem stage (plain TMA load, no multicast),
// feeds it to the MMA and TMA-stores the same stage into the local gathered
// copy, then publishes flags[tile] = 2.  Every other CTA waits (bounded) for
// 2 and loads the tile from the local copy.  The claimant never waits on
// anyone, so the scheme cannot deadlock.
constexpr int GATHER_MAX_PEERS = 8;
struct alignas(64) GatherMaps {
  CUtensorMap peer[GATHER_MAX_PEERS];  // rank r's shard of B: [groups_per_rank, K, N]
  CUtensorMap local;                   // gathered copy on this GPU: [G, K, N]
  const __nv_bfloat16* src[GATHER_MAX_PEERS];  // the same shards as plain pointers
  __nv_bfloat16* dst;                  // the gathered copy
  int* flags;                          // [G][tiles_n][k_blocks]
  int rank, world, groups_per_rank;
  // Not part of the gather: the second K-major B of a K-concatenated grouped
  // GEMM, C = A[:, :Ks] B[g]^T + A[:, Ks:] B_hi[g]^T (GemmArgs::k_split_b = Ks).
  CUtensorMap b_hi;
};

// Copy-ahead of the gathered B tiles by two extra warps (the last two warps
// of the gathered variant), concurrent with the producer, MMA and epilogue.  CTA i takes tiles
// i, i + grid, ... in the order the tile schedule needs them, claims each with
// the same flag protocol as the producer (so a tile is copied exactly once)
// and moves it with 16-byte peer loads / local stores.  Groups without rows
// are skipped.
constexpr int GATHER_COPY_THREADS = 64;  // two extra warps in the gathered variant

template <int BN>
__device__ void gather_copy_ahead(const GemmArgs& args, const GatherMaps& gm) {
  constexpr int CT = GATHER_COPY_THREADS;
  constexpr int PER = 16;                        // 16-byte pieces in flight per thread
  constexpr int ROUNDS = GEMM_BK * BN / 8 / CT / PER;
  static_assert(ROUNDS * PER * CT * 8 == GEMM_BK * BN, "copy split");
  __shared__ int s_claim[2];
  const int tid = threadIdx.x - (GEMM_THREADS);  // 0..CT-1
  const int K = args.K, N = args.N, TN = args.tiles_n;
  const int KB = (K + GEMM_BK - 1) / GEMM_BK;
  const long long total = (long long)args.num_groups * KB * TN;
  int it = 0;
  for (long long c = blockIdx.x; c < total; c += gridDim.x) {
    const int nb = c % TN;
    const int kb = (c / TN) % KB;
    const int g = c / ((long long)TN * KB);
    if (__ldg(args.grp_count + g) == 0) continue;
    int* flag = gm.flags + ((long long)g * TN + nb) * KB + kb;
    // claim broadcast through alternating slots: one barrier per tile
    if (tid == 0) s_claim[it & 1] = ld_acquire_gpu(flag) == 0 && atomicCAS(flag, 0, 1) == 0;
    asm volatile("bar.sync 1, %0;" ::"n"(CT) : "memory");
    const bool won = s_claim[it & 1];
    ++it;
    if (!won) continue;
    const int owner = g / gm.groups_per_rank;
    const int k0 = kb * GEMM_BK, n0 = nb * BN;
    const int rows = min(GEMM_BK, K - k0), cols = min(BN, N - n0);
    const __nv_bfloat16* src = gm.src[owner] + ((long long)(g - owner * gm.groups_per_rank) * K + k0) * N + n0;
    __nv_bfloat16* dst = gm.dst + ((long long)g * K + k0) * N + n0;
    const int c8 = cols / 8;  // N % 8 == 0: 16-byte pieces
    const int n8 = rows * c8;
#pragma unroll 1
    for (int rd = 0; rd < ROUNDS; ++rd) {
      uint4 v[PER];
#pragma unroll
      for (int j = 0; j < PER; ++j) {  // every load of the round in flight before the stores
        const int i = tid + CT * (rd * PER + j);
        if (i < n8) {
          const int r = i / c8, q = i - r * c8;
          v[j] = *reinterpret_cast<const uint4*>(src + (long long)r * N + 8 * q);
        }
      }
#pragma unroll
      for (int j = 0; j < PER; ++j) {
        const int i = tid + CT * (rd * PER + j);
        if (i < n8) {
          const int r = i / c8, q = i - r * c8;
          *reinterpret_cast<uint4*>(dst + (long long)r * N + 8 * q) = v[j];
        }
      }
    }
    __threadfence();
    fence_proxy_async_global();
    asm volatile("bar.sync 1, %0;" ::"n"(CT) : "memory");
    if (tid == 0) st_release_gpu(flag, 2);
  }
}

template <int BN>
struct GemmCfg {
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;
  static constexpr int B_BYTES = BN * GEMM_BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN == 256) ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int TMEM_COLS = (2 * BN <= 32) ? 32 : 2 * BN;  // power of two
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

struct TileInfo {
  int m0, n0, k0, k_iters, group, m_limit;
};

template <int MODE, int BN>
__device__ __forceinline__ bool get_tile(const GemmArgs& a, int t, TileInfo& ti) {
  if (MODE == DENSE) {
    if (t >= a.num_tiles) return false;
    const int split = t % a.k_splits;
    const int tile = t / a.k_splits;
    int mb = tile / a.tiles_n, nb = tile - mb * a.tiles_n;
    ti.m0 = mb * GEMM_BM;
    ti.n0 = nb * BN;
    const int total_k = (a.K + GEMM_BK - 1) / GEMM_BK;
    const int per = (total_k + a.k_splits - 1) / a.k_splits;
    const int kb0 = split * per;
    ti.k0 = kb0 * GEMM_BK;
    ti.k_iters = max(0, min(per, total_k - kb0));
    ti.group = 0;
    ti.m_limit = a.M;
    return true;
  } else if (MODE == GROUPED_M) {
    const int total = __ldg(a.grp_tile_start + a.num_groups);
    if (t >= total) return false;
    int g = 0;
    // groups are few (<= 256): linear scan over the prefix array
    while (g + 1 < a.num_groups && __ldg(a.grp_tile_start + g + 1) <= t) ++g;
    int local = t - __ldg(a.grp_tile_start + g);
    int mb = local / a.tiles_n, nb = local - mb * a.tiles_n;
    int start = __ldg(a.grp_start + g);
    ti.m0 = start + mb * GEMM_BM;
    ti.n0 = nb * BN;
    ti.k0 = 0;
    ti.k_iters = (a.K + GEMM_BK - 1) / GEMM_BK;
    ti.group = g;
    ti.m_limit = start + __ldg(a.grp_count + g);
    return true;
  } else {
    if (t >= a.num_tiles) return false;
    const int per = a.tiles_m * a.tiles_n;
    int g = t / per;
    int local = t - g * per;
    int mb = local / a.tiles_n, nb = local - mb * a.tiles_n;
    ti.m0 = mb * GEMM_BM;
    ti.n0 = nb * BN;
    ti.k0 = __ldg(a.grp_start + g);
    ti.k_iters = (__ldg(a.grp_count + g) + GEMM_BK - 1) / GEMM_BK;
    ti.group = g;
    ti.m_limit = a.M;
    return true;
  }
}

// EPI_SWIGLU_FWD: one row, 32 columns (n .. n+31, F a multiple of 128).  g and u
// are rounded to bf16 as stored, silu(g) is rounded to bf16, then h = silu * u
// (the rounding of the standalone SwiGLU kernel).
HB_DEVICE void swiglu_fwd_store(const GemmArgs& args, int m, int n, bool row_ok, bool has_k, float alpha,
                                const uint32_t (&rg)[32], const uint32_t (&ru)[32]) {
  const int F = args.N / 2;
  uint4* h4 = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(args.C) + (long long)m * args.ldc + n);
  if (!row_ok) {
#pragma unroll
    for (int q = 0; q < 4; ++q) h4[q] = make_uint4(0u, 0u, 0u, 0u);
    return;
  }
  __nv_bfloat16* gp = reinterpret_cast<__nv_bfloat16*>(args.c2) + (long long)m * args.ldc2 + n;
  uint4* g4 = reinterpret_cast<uint4*>(gp);
  uint4* u4 = reinterpret_cast<uint4*>(gp + F);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 wh, wg, wu;
    uint32_t* ph = reinterpret_cast<uint32_t*>(&wh);
    uint32_t* pg = reinterpret_cast<uint32_t*>(&wg);
    uint32_t* pu = reinterpret_cast<uint32_t*>(&wu);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int j = q * 8 + 2 * e;
      const float g0 = has_k ? __uint_as_float(rg[j]) * alpha : 0.f;
      const float g1 = has_k ? __uint_as_float(rg[j + 1]) * alpha : 0.f;
      const float u0 = has_k ? __uint_as_float(ru[j]) * alpha : 0.f;
      const float u1 = has_k ? __uint_as_float(ru[j + 1]) * alpha : 0.f;
      pg[e] = pack_bf16x2(g0, g1);
      pu[e] = pack_bf16x2(u0, u1);
      const float gr0 = __uint_as_float(pg[e] << 16), gr1 = __uint_as_float(pg[e] & 0xffff0000u);
      const float ur0 = __uint_as_float(pu[e] << 16), ur1 = __uint_as_float(pu[e] & 0xffff0000u);
      const float s0 = __bfloat162float(__float2bfloat16_rn(__fdividef(gr0, 1.f + __expf(-gr0))));
      const float s1 = __bfloat162float(__float2bfloat16_rn(__fdividef(gr1, 1.f + __expf(-gr1))));
      ph[e] = pack_bf16x2(s0 * ur0, s1 * ur1);
    }
    h4[q] = wh;
    g4[q] = wg;
    u4[q] = wu;
  }
}

// EPI_SWIGLU_BWD: one thread's 32 columns of the forward's g and u (bf16).
// They do not depend on the accumulator, so the epilogue loads a tile's first
// chunk before it waits for the MMAs and each next chunk while it computes the
// current one; everything stays in registers (constant indices only).
struct SwigluAux {
  uint4 g[4], u[4];
};

HB_DEVICE void swiglu_aux_load(const GemmArgs& args, long long m, bool row_ok, int n, SwigluAux& a) {
  const int F = args.N;
  if (!row_ok || n >= F) return;
  const __nv_bfloat16* gp = reinterpret_cast<const __nv_bfloat16*>(args.aux) + m * args.ldc + n;
  const __nv_bfloat16* up = gp + F;
  if (n + 32 <= F && (F % 8) == 0) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      a.g[q] = reinterpret_cast<const uint4*>(gp)[q];
      a.u[q] = reinterpret_cast<const uint4*>(up)[q];
    }
  } else {
    const int cnt = F - n;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t wg[4], wu[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = q * 8 + 2 * e;
        const uint32_t g0 = j < cnt ? __bfloat16_as_ushort(gp[j]) : 0u;
        const uint32_t g1 = j + 1 < cnt ? __bfloat16_as_ushort(gp[j + 1]) : 0u;
        const uint32_t u0 = j < cnt ? __bfloat16_as_ushort(up[j]) : 0u;
        const uint32_t u1 = j + 1 < cnt ? __bfloat16_as_ushort(up[j + 1]) : 0u;
        wg[e] = g0 | (g1 << 16);
        wu[e] = u0 | (u1 << 16);
      }
      a.g[q] = make_uint4(wg[0], wg[1], wg[2], wg[3]);
      a.u[q] = make_uint4(wu[0], wu[1], wu[2], wu[3]);
    }
  }
}

// dgu = [dh u silu'(g) | dh silu(g)] for one 32-column chunk (pad rows: zeros)
HB_DEVICE void swiglu_bwd_chunk(const GemmArgs& args, char* cbase, long long m, bool row_ok, int n,
                                bool has_k, float alpha, const uint32_t (&r)[32], const SwigluAux& a) {
  const int F = args.N;
  if (n >= F) return;
  __nv_bfloat16* dg = reinterpret_cast<__nv_bfloat16*>(cbase) + m * args.ldc + n;
  __nv_bfloat16* du = dg + F;
  const bool vec = n + 32 <= F && (F % 8) == 0;
  uint4 og[4], ou[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t gw[4] = {a.g[q].x, a.g[q].y, a.g[q].z, a.g[q].w};
    const uint32_t uw[4] = {a.u[q].x, a.u[q].y, a.u[q].z, a.u[q].w};
    uint32_t pg[4], pu[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float vg[2], vu[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int j = q * 8 + 2 * e + h;
        // dh is rounded to bf16 first, as when it is stored between kernels
        const float d = __bfloat162float(__float2bfloat16_rn(has_k ? __uint_as_float(r[j]) * alpha : 0.f));
        const float g = __uint_as_float(h ? (gw[e] & 0xffff0000u) : (gw[e] << 16));
        const float u = __uint_as_float(h ? (uw[e] & 0xffff0000u) : (uw[e] << 16));
        // approximate divide (2 ulp; 1 / inf = 0 keeps the limit): the results are rounded to bf16
        const float sg = __fdividef(1.f, 1.f + __expf(-g));
        const float silu = g * sg;
        const float dsilu = sg * (1.f + g * (1.f - sg));
        vg[h] = row_ok ? d * u * dsilu : 0.f;
        vu[h] = row_ok ? d * silu : 0.f;
      }
      pg[e] = pack_bf16x2(vg[0], vg[1]);
      pu[e] = pack_bf16x2(vu[0], vu[1]);
    }
    og[q] = make_uint4(pg[0], pg[1], pg[2], pg[3]);
    ou[q] = make_uint4(pu[0], pu[1], pu[2], pu[3]);
  }
  if (vec) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      reinterpret_cast<uint4*>(dg)[q] = og[q];
      reinterpret_cast<uint4*>(du)[q] = ou[q];
    }
  } else {
    const int cnt = F - n;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t gw[4] = {og[q].x, og[q].y, og[q].z, og[q].w};
      const uint32_t uw[4] = {ou[q].x, ou[q].y, ou[q].z, ou[q].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = q * 8 + 2 * e;
        if (j < cnt) {
          dg[j] = __ushort_as_bfloat16((unsigned short)(gw[e] & 0xffffu));
          du[j] = __ushort_as_bfloat16((unsigned short)(uw[e] & 0xffffu));
        }
        if (j + 1 < cnt) {
          dg[j + 1] = __ushort_as_bfloat16((unsigned short)(gw[e] >> 16));
          du[j + 1] = __ushort_as_bfloat16((unsigned short)(uw[e] >> 16));
        }
      }
    }
  }
}

template <int BN, bool A_MN, bool B_MN, int MODE, int EPI, bool GATHER = false>
__global__ void __launch_bounds__(GATHER ? GEMM_THREADS + GATHER_COPY_THREADS : GEMM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmArgs args, const __grid_constant__ GatherMaps gm) {
  static_assert(!GATHER || (MODE == GROUPED_M && B_MN), "gathered B: grouped-M, MN-major B");
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* bar_area = smem + STAGES * Cfg::STAGE_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(bar_area);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&tfull_bar[i]), 1);
      mbar_init(smem_u32(&tempty_bar[i]), 32 * GEMM_EPI_WARPS);
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok; t += gridDim.x) {
        TileInfo ti;
        if (!get_tile<MODE, BN>(args, t, ti)) break;
        // gathered B: one parallel read of the tile column's flags; when all
        // are published the k-loop loads from the local copy without checks
        int* fcol = nullptr;
        bool col_ready = false;
        if (GATHER) {
          fcol = gm.flags + ((long long)ti.group * args.tiles_n + ti.n0 / BN) * ti.k_iters;
          int nr = 0;
#pragma unroll 8
          for (int kb = 0; kb < ti.k_iters; ++kb) nr += ld_relaxed_gpu(fcol + kb) == 2;
          col_ready = nr == ti.k_iters;
          if (col_ready) {
            fence_acquire_gpu();
            fence_proxy_async_global();
          }
        }
        for (int kb = 0; kb < ti.k_iters; ++kb) {
          if (!mbar_wait(smem_u32(&empty_bar[stage]), phase ^ 1, args.status, kErrTimeoutProducer,
                         args.budget_ns)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&full_bar[stage]);
          mbar_expect_tx(fb, Cfg::STAGE_BYTES);
          const uint32_t sa = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t sb = sa + Cfg::A_BYTES;
          const int kc = ti.k0 + kb * GEMM_BK;
          if (!A_MN) {
            tma_load_2d(sa, &tmA, fb, kc, ti.m0);
          } else {
#pragma unroll
            for (int i = 0; i < GEMM_BM / 64; ++i) tma_load_2d(sa + i * 8192, &tmA, fb, ti.m0 + 64 * i, kc);
          }
          if (GATHER) {
            // own experts go through the same claim / copy path (a local copy),
            // so the gathered buffer is complete for the backward
            const int g = ti.group;
            const int owner = g / gm.groups_per_rank;
            if (col_ready) {
#pragma unroll
              for (int i = 0; i < BN / 64; ++i) tma_load_3d(sb + i * 8192, &gm.local, fb, ti.n0 + 64 * i, kc, g);
            } else {
              int* flag = fcol + kb;
              const bool won = ld_acquire_gpu(flag) == 0 && atomicCAS(flag, 0, 1) == 0;
              if (won) {
#pragma unroll
                for (int i = 0; i < BN / 64; ++i)
                  tma_load_3d(sb + i * 8192, &gm.peer[owner], fb, ti.n0 + 64 * i, kc,
                              g - owner * gm.groups_per_rank);
                // the stage also feeds the MMA; wait for it here and copy it out
                if (!mbar_wait(fb, phase, args.status, kErrTimeoutProducer, args.budget_ns)) {
                  ok = false;
                  break;
                }
#pragma unroll
                for (int i = 0; i < BN / 64; ++i) tma_store_3d(&gm.local, sb + i * 8192, ti.n0 + 64 * i, kc, g);
                bulk_commit_group();
                bulk_wait_group_0();
                fence_proxy_async_global();
                st_release_gpu(flag, 2);
              } else {
                const uint64_t t0 = globaltimer();
                while (ld_acquire_gpu(flag) != 2) {
                  if (globaltimer() - t0 > args.budget_ns) {
                    set_error(args.status, kErrTimeoutPeer);
                    ok = false;
                    break;
                  }
                }
                if (!ok) break;
                fence_proxy_async_global();
#pragma unroll
                for (int i = 0; i < BN / 64; ++i) tma_load_3d(sb + i * 8192, &gm.local, fb, ti.n0 + 64 * i, kc, g);
              }
            }
          } else if (MODE == GROUPED_M) {
            if (!B_MN) {
              if (args.k_split_b > 0 && kc >= args.k_split_b)
                tma_load_3d(sb, &gm.b_hi, fb, kc - args.k_split_b, ti.n0, ti.group);
              else
                tma_load_3d(sb, &tmB, fb, kc, ti.n0, ti.group);
            } else if (EPI == EPI_SWIGLU_FWD) {
              // first half of the tile from W_gate, second half from W_up
#pragma unroll
              for (int i = 0; i < BN / 64; ++i)
                tma_load_3d(sb + i * 8192, i < BN / 128 ? &tmB : &gm.b_hi, fb,
                            ti.n0 / 2 + 64 * (i % (BN / 128)), kc, ti.group);
            } else {
#pragma unroll
              for (int i = 0; i < BN / 64; ++i) tma_load_3d(sb + i * 8192, &tmB, fb, ti.n0 + 64 * i, kc, ti.group);
            }
          } else {
            if (!B_MN) {
              tma_load_2d(sb, &tmB, fb, kc, ti.n0);
            } else {
#pragma unroll
              for (int i = 0; i < BN / 64; ++i) tma_load_2d(sb + i * 8192, &tmB, fb, ti.n0 + 64 * i, kc);
            }
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc = make_idesc_bf16(GEMM_BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok; t += gridDim.x) {
        TileInfo ti;
        if (!get_tile<MODE, BN>(args, t, ti)) break;
        if (!mbar_wait(smem_u32(&tempty_bar[acc]), acc_phase ^ 1, args.status, kErrTimeoutMma,
                       args.budget_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < ti.k_iters; ++kb) {
          if (!mbar_wait(smem_u32(&full_bar[stage]), phase, args.status, kErrTimeoutMma,
                         args.budget_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t sb = sa + Cfg::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < GEMM_BK / 16; ++kk) {
            uint64_t ad, bd;
            if (!A_MN)
              ad = make_smem_desc(sa + kk * 32, 16, 1024);
            else
              ad = make_smem_desc(sa + kk * 2048, 8192, 1024);
            if (!B_MN)
              bd = make_smem_desc(sb + kk * 32, 16, 1024);
            else
              bd = make_smem_desc(sb + kk * 2048, 8192, 1024);
            umma_f16(d_tmem, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(smem_u32(&empty_bar[stage]));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(smem_u32(&tfull_bar[acc]));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
  } else if (GATHER && warp >= GEMM_THREADS / 32) {
    // ------------------------------------------------------------ copy warps
    gather_copy_ahead<BN>(args, gm);
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;  // TMEM lane quadrant accessible to this warp
    const int half = (warp - 2) >> 2;  // which of the two warps of this quadrant
    const float alpha = args.alpha_ptr ? *args.alpha_ptr : args.alpha;
    const int row_in_tile = quad * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x;; t += gridDim.x) {
      TileInfo ti;
      if (!get_tile<MODE, BN>(args, t, ti)) break;
      SwigluAux aux[2];   // EPI_SWIGLU_BWD: chunk buffers (first one loaded before the wait)
      if constexpr (EPI == EPI_SWIGLU_BWD)
        swiglu_aux_load(args, ti.m0 + row_in_tile, ti.m0 + row_in_tile < ti.m_limit, ti.n0 + half * 32, aux[0]);
      if (!mbar_wait(smem_u32(&tfull_bar[acc]), acc_phase, args.status, kErrTimeoutEpilogue,
                     args.budget_ns))
        break;
      tc_fence_after();
      const int m = ti.m0 + row_in_tile;
      const bool row_ok = m < ti.m_limit;
      const bool has_k = ti.k_iters > 0;
      char* cbase = reinterpret_cast<char*>(args.C);
      if (MODE == GROUPED_K) cbase += (long long)ti.group * args.c_group_stride * (EPI == EPI_BF16 ? 2 : 4);
      if constexpr (EPI == EPI_SWIGLU_FWD) {
        const int F = args.N / 2;
#pragma unroll 1
        for (int c = half; c < BN / 64; c += 2) {
          uint32_t rg[32], ru[32];
          const uint32_t tb = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN;
          tmem_ld_32x32b_x32(tb + c * 32, rg);
          tmem_ld_32x32b_x32(tb + BN / 2 + c * 32, ru);
          tmem_ld_wait();
          const int n = ti.n0 / 2 + c * 32;
          if (n < F) swiglu_fwd_store(args, m, n, row_ok, has_k, alpha, rg, ru);
        }
      }
      if constexpr (EPI == EPI_SWIGLU_BWD) {
        // chunk j = columns (half + 2 j) * 32: TMEM read, next chunk's g | u
        // loads in flight, then this chunk's arithmetic and stores
#pragma unroll
        for (int j = 0; j < BN / 64; ++j) {
          const int c = half + 2 * j;
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN + c * 32, r);
          if (j + 1 < BN / 64) swiglu_aux_load(args, m, row_ok, ti.n0 + (c + 2) * 32, aux[(j + 1) & 1]);
          tmem_ld_wait();
          swiglu_bwd_chunk(args, cbase, m, row_ok, ti.n0 + c * 32, has_k, alpha, r, aux[j & 1]);
        }
      }
#pragma unroll 1
      for (int c = half; c < (EPI == EPI_SWIGLU_FWD || EPI == EPI_SWIGLU_BWD ? 0 : BN / 32); c += 2) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN + c * 32, r);
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
            // split-K: partial products meet in global memory
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
                float4 o = o4[q];
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
      mbar_arrive(smem_u32(&tempty_bar[acc]));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
}


template <int BN, bool A_MN, bool B_MN, int MODE, int EPI, bool GATHER = false>
void gemm_launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& args, int grid,
                 const GatherMaps* gm = nullptr) {
  using Cfg = GemmCfg<BN>;
  auto kern = gemm_tc_kernel<BN, A_MN, B_MN, MODE, EPI, GATHER>;
  static bool configured = false;  // one static per instantiation
  if (!configured) {
    HB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    configured = true;
  }
  static const GatherMaps none{};
  kern<<<grid, GATHER ? GEMM_THREADS + GATHER_COPY_THREADS : GEMM_THREADS, Cfg::SMEM, cur_stream()>>>(
      ta, tb, args, gm ? *gm : none);
  HB_CUDA_CHECK(cudaGetLastError());
}

// Dispatchers, each defined in its own translation unit.
void gemm_dispatch_dense_ak(int bn, bool b_mn, int epi, const CUtensorMap& ta, const CUtensorMap& tb,
                            const GemmArgs& args, int grid);
void gemm_dispatch_dense_amn(int bn, bool b_mn, int epi, const CUtensorMap& ta, const CUtensorMap& tb,
                             const GemmArgs& args, int grid);
void gemm_dispatch_grouped(int mode, int bn, bool a_mn, bool b_mn, int epi, const CUtensorMap& ta,
                           const CUtensorMap& tb, const GemmArgs& args, int grid,
                           const GatherMaps* gm = nullptr);
void gemm_dispatch_gather(int bn, const CUtensorMap& ta, const GemmArgs& args, const GatherMaps& gm, int grid);

}  // namespace hb
