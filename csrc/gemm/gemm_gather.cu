// Fused FSDP all-gather + grouped GEMM (MoE expert weights sharded by expert
// over the data-parallel ranks):
//   c[rows of g] = a[rows of g] @ B[g],   B[g] read from rank g / groups_per_rank
// The remote tiles cross NVLink once per GPU and land in `gathered` ([G, K, N],
// the local copy the backward reads): the epilogue warps of every CTA copy
// them ahead at kernel start (peer loads), the TMA producers claim any tile
// still uncopied when they reach it (TMA load from the owner); see GatherMaps
// in gemm_kernel.cuh.
#include "gemm_kernel.cuh"

namespace hb {

void gemm_dispatch_gather(int bn, const CUtensorMap& ta, const GemmArgs& args, const GatherMaps& gm, int grid) {
  if (bn == 256) {
    gemm_launch<256, false, true, GROUPED_M, EPI_BF16, true>(ta, ta, args, grid, &gm);
  } else {
    gemm_launch<128, false, true, GROUPED_M, EPI_BF16, true>(ta, ta, args, grid, &gm);
  }
}

namespace {
int pick_bn_g(int n) { return n >= 256 ? 256 : 128; }
}  // namespace

// a: [R, K] bf16 (expert-sorted rows, 128-aligned segments); peer_ptrs[r]: device
// address of rank r's shard [groups_per_rank, K, N] (bf16, contiguous; the local
// rank's entry is this GPU's own shard); gathered: [G, K, N] bf16 on this GPU;
// flags: int32 [G * ceil(K/64) * ceil(N/BN)], zeroed here before the launch;
// c: [R, N] bf16.
void grouped_gemm_m_gather(torch::Tensor a, std::vector<int64_t> peer_ptrs, int64_t rank,
                           int64_t groups_per_rank, torch::Tensor gathered, torch::Tensor flags,
                           torch::Tensor c, torch::Tensor grp_start, torch::Tensor grp_count,
                           torch::Tensor grp_tile_start) {
  check_bf16(a, "a");
  check_bf16(gathered, "gathered");
  check_bf16(c, "c");
  const int world = (int)peer_ptrs.size();
  HB_CHECK(world >= 1 && world <= GATHER_MAX_PEERS, "grouped_gemm_m_gather: 1..8 ranks");
  HB_CHECK(gathered.dim() == 3 && gathered.is_contiguous(), "gathered must be contiguous [G, K, N]");
  const int G = gathered.size(0), K = gathered.size(1), N = gathered.size(2);
  HB_CHECK(G == groups_per_rank * world, "grouped_gemm_m_gather: G != groups_per_rank * world");
  HB_CHECK(a.size(1) == K && c.size(1) == N && c.size(0) == a.size(0) && c.stride(1) == 1,
           "grouped_gemm_m_gather: bad shapes");
  HB_CHECK(N % 8 == 0 && K % 8 == 0, "grouped_gemm_m_gather: 16-byte rows");
  const int R = a.size(0);
  if (R == 0) return;
  const c10::cuda::CUDAGuard guard(a.device());
  const int BN = pick_bn_g(N);
  const int tiles_n = (N + BN - 1) / BN;
  const int kblocks = (K + GEMM_BK - 1) / GEMM_BK;
  HB_CHECK(flags.scalar_type() == torch::kInt32 && flags.numel() >= (long long)G * kblocks * tiles_n,
           "grouped_gemm_m_gather: flags too small");
  HB_CUDA_CHECK(cudaMemsetAsync(flags.data_ptr(), 0, (size_t)G * kblocks * tiles_n * 4, cur_stream()));
  GatherMaps gm{};
  for (int r = 0; r < world; ++r) {
    HB_CHECK(peer_ptrs[r] % 16 == 0, "grouped_gemm_m_gather: peer shard not 16-byte aligned");
    gm.peer[r] = tmap_bf16_3d(reinterpret_cast<const void*>(peer_ptrs[r]), groups_per_rank, K, N, N,
                              (uint64_t)K * N, 64, 64);
  }
  gm.local = tmap_bf16_3d(gathered.data_ptr(), G, K, N, N, (uint64_t)K * N, 64, 64);
  for (int r = 0; r < world; ++r) gm.src[r] = reinterpret_cast<const __nv_bfloat16*>(peer_ptrs[r]);
  gm.dst = reinterpret_cast<__nv_bfloat16*>(gathered.data_ptr());
  gm.flags = flags.data_ptr<int>();
  gm.rank = (int)rank;
  gm.world = world;
  gm.groups_per_rank = (int)groups_per_rank;
  CUtensorMap ta = tmap_bf16_2d(a.data_ptr(), R, K, a.stride(0), 64, GEMM_BM);
  GemmArgs args{};
  args.C = c.data_ptr();
  args.ldc = c.stride(0);
  args.alpha = 1.f;
  args.alpha_ptr = nullptr;
  args.status = status_ptr();
  args.budget_ns = wait_budget_ns();
  args.k_splits = 1;
  args.M = R;
  args.N = N;
  args.K = K;
  args.tiles_n = tiles_n;
  args.num_groups = G;
  args.grp_start = grp_start.data_ptr<int>();
  args.grp_count = grp_count.data_ptr<int>();
  args.grp_tile_start = grp_tile_start.data_ptr<int>();
  const int max_tiles = ((R + GEMM_BM - 1) / GEMM_BM) * tiles_n;
  const int grid = std::max(1, std::min(max_tiles, num_sms()));
  gemm_dispatch_gather(BN, ta, args, gm, grid);
}

}  // namespace hb
