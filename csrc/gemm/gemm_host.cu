// Host entry points of the tcgen05 GEMM: operand checks, TMA descriptors,
// tile counts, and dispatch to the instantiation units.
#include <cstdlib>
#include <string>
#include <vector>

#include "gemm_kernel.cuh"
#include "gemm_pair.cuh"

namespace hb {

namespace {

// CTA-pair kernel selection: HB_GEMM_PAIR=0 disables it, =force uses it for
// every supported shape (tests), default uses it when the 256 x 256 pair tiles
// fill at least one wave of SM pairs.
int pair_mode() {
  static int m = [] {
    const char* e = std::getenv("HB_GEMM_PAIR");
    if (e && std::string(e) == "0") return 0;
    if (e && std::string(e) == "force") return 2;
    return 1;
  }();
  return m;
}
bool use_pair(long long pair_tiles) {
  const int pm = pair_mode();
  return pm == 2 || (pm == 1 && pair_tiles >= num_sms() / 2);
}


int pick_bn(int N) { return N >= 256 ? 256 : 128; }

int epi_of(const torch::Tensor& c, bool accumulate) {
  if (c.scalar_type() == at::kBFloat16) {
    HB_CHECK(!accumulate, "accumulate requires an fp32 output");
    return EPI_BF16;
  }
  HB_CHECK(c.scalar_type() == at::kFloat, "output must be bf16 or fp32");
  return accumulate ? EPI_F32_ACC : EPI_F32;
}

GemmArgs base_args(const torch::Tensor& c, double alpha,
                   const c10::optional<torch::Tensor>& alpha_t = c10::nullopt) {
  GemmArgs a{};
  a.k_splits = 1;
  a.C = c.data_ptr();
  a.ldc = c.stride(-2);
  a.alpha = (float)alpha;
  if (alpha_t.has_value()) {
    HB_CHECK(alpha_t->scalar_type() == at::kFloat && alpha_t->numel() == 1 && alpha_t->is_cuda(),
             "alpha tensor must be a CUDA fp32 scalar");
    a.alpha_ptr = alpha_t->data_ptr<float>();
  }
  a.status = status_ptr();
  a.budget_ns = wait_budget_ns();
  return a;
}

}  // namespace

// c[M,N] (+)= op(a) @ op(b);  a is [M,K] (or [K,M] when trans_a); b is [K,N]
// (or [N,K] when trans_b).  All operands row-major with unit column stride.
void gemm(torch::Tensor a, torch::Tensor b, torch::Tensor c, bool trans_a, bool trans_b,
          bool accumulate, double alpha, c10::optional<torch::Tensor> alpha_t) {
  check_bf16(a, "a");
  check_bf16(b, "b");
  HB_CHECK(a.dim() == 2 && b.dim() == 2 && c.dim() == 2, "gemm expects 2-D tensors");
  HB_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && c.stride(1) == 1, "unit column stride required");
  const int M = trans_a ? a.size(1) : a.size(0);
  const int K = trans_a ? a.size(0) : a.size(1);
  const int N = trans_b ? b.size(0) : b.size(1);
  HB_CHECK((trans_b ? b.size(1) : b.size(0)) == K, "gemm: inner dimensions differ");
  HB_CHECK(c.size(0) == M && c.size(1) == N, "gemm: bad output shape");
  if (M == 0 || N == 0) return;
  const c10::cuda::CUDAGuard guard(a.device());
  const int BN = pick_bn(N);
  // A operand
  CUtensorMap ta = trans_a ? tmap_bf16_2d(a.data_ptr(), K, M, a.stride(0), 64, 64)
                           : tmap_bf16_2d(a.data_ptr(), M, K, a.stride(0), 64, GEMM_BM);
  CUtensorMap tb = trans_b ? tmap_bf16_2d(b.data_ptr(), N, K, b.stride(0), 64, BN)
                           : tmap_bf16_2d(b.data_ptr(), K, N, b.stride(0), 64, 64);
  GemmArgs args = base_args(c, alpha, alpha_t);
  args.M = M;
  args.N = N;
  args.K = K;
  args.tiles_m = (M + GEMM_BM - 1) / GEMM_BM;
  args.tiles_n = (N + BN - 1) / BN;
  args.num_tiles = args.tiles_m * args.tiles_n;
  if (K == 0) {
    HB_CHECK(false, "gemm with K == 0 is not supported");
  }
  const int epi = epi_of(c, accumulate);
  if (M >= 128 && N >= 256 && !(trans_a && trans_b)) {
    const long long ptiles = (long long)((M + PAIR_BM - 1) / PAIR_BM) * ((N + PAIR_BN - 1) / PAIR_BN);
    if (use_pair(ptiles)) {
      GemmArgs pa = args;
      pa.tiles_m = (M + PAIR_BM - 1) / PAIR_BM;
      pa.tiles_n = (N + PAIR_BN - 1) / PAIR_BN;
      pa.num_tiles = pa.tiles_m * pa.tiles_n;
      pa.k_splits = 1;
      CUtensorMap tbp = trans_b ? tmap_bf16_2d(b.data_ptr(), N, K, b.stride(0), 64, 128) : tb;
      const int grid = 2 * std::min(pa.num_tiles, num_sms() / 2);
      gemm_dispatch_pair(DENSE, trans_a, !trans_b, epi, ta, tbp, pa, grid);
      return;
    }
  }
  // Split the K loop when the output has too few tiles to fill the GPU
  // (weight gradients: small [in, out] output, K = tokens).  fp32 outputs only.
  args.k_splits = 1;
  const int sms = num_sms();
  const int kblocks = (K + GEMM_BK - 1) / GEMM_BK;
  if (epi != EPI_BF16 && args.num_tiles * 2 <= sms && kblocks >= 16) {
    int s = std::min(sms / args.num_tiles, kblocks / 8);
    s = std::max(1, std::min(s, 32));
    if (s > 1) {
      if (epi == EPI_F32) c.zero_();  // partials are added atomically
      args.k_splits = s;
      args.num_tiles *= s;
    }
  }
  const int grid = std::min(args.num_tiles, sms);
  if (trans_a)
    gemm_dispatch_dense_amn(BN, !trans_b, epi, ta, tb, args, grid);
  else
    gemm_dispatch_dense_ak(BN, !trans_b, epi, ta, tb, args, grid);
}

// c (+)= sum_s a[:, k_s : k_s + K_s] @ b_s^T for K-major b_s [N, K_s]: the
// input gradient of several projections whose output gradients sit side by
// side in a.  One CTA-pair launch (a K-segmented B) where the pair path
// applies, else one accumulating GEMM per segment.
void gemm_kseg(torch::Tensor a, std::vector<torch::Tensor> bs, torch::Tensor c, bool accumulate) {
  check_bf16(a, "a");
  HB_CHECK(!bs.empty() && (int)bs.size() <= KSEG_MAX, "gemm_kseg: 1..6 segments");
  HB_CHECK(a.dim() == 2 && a.stride(1) == 1 && c.dim() == 2 && c.stride(1) == 1, "gemm_kseg: 2-D, unit column stride");
  const int M = a.size(0), N = c.size(1);
  int K = 0;
  bool aligned = true;
  for (auto& b : bs) {
    check_bf16(b, "b");
    HB_CHECK(b.dim() == 2 && b.stride(1) == 1 && b.size(0) == N, "gemm_kseg: each b must be [N, K_s]");
    aligned = aligned && b.size(1) % GEMM_BK == 0;
    K += b.size(1);
  }
  HB_CHECK(a.size(1) == K && c.size(0) == M, "gemm_kseg: shapes differ");
  if (M == 0 || N == 0) return;
  const c10::cuda::CUDAGuard guard(a.device());
  const int epi = epi_of(c, accumulate);
  const long long ptiles = (long long)((M + PAIR_BM - 1) / PAIR_BM) * ((N + PAIR_BN - 1) / PAIR_BN);
  if (aligned && M >= 128 && N >= 256 && use_pair(ptiles)) {
    KSegMaps ks{};
    int k0 = 0;
    for (size_t i = 0; i < bs.size(); ++i) {
      ks.seg[i] = tmap_bf16_2d(bs[i].data_ptr(), N, bs[i].size(1), bs[i].stride(0), 64, 128);
      ks.seg_k[i] = k0;
      k0 += bs[i].size(1);
    }
    ks.seg_k[bs.size()] = k0;
    ks.nseg = (int)bs.size();
    CUtensorMap ta = tmap_bf16_2d(a.data_ptr(), M, K, a.stride(0), 64, GEMM_BM);
    GemmArgs pa = base_args(c, 1.0);
    pa.M = M;
    pa.N = N;
    pa.K = K;
    pa.tiles_m = (M + PAIR_BM - 1) / PAIR_BM;
    pa.tiles_n = (N + PAIR_BN - 1) / PAIR_BN;
    pa.num_tiles = pa.tiles_m * pa.tiles_n;
    const int grid = 2 * std::min(pa.num_tiles, num_sms() / 2);
    gemm_dispatch_pair(DENSE, false, false, epi, ta, ks.seg[0], pa, grid, &ks);
    return;
  }
  int k0 = 0;
  for (size_t i = 0; i < bs.size(); ++i) {
    const int ks_ = bs[i].size(1);
    gemm(a.narrow(1, k0, ks_), bs[i], c, false, true, accumulate || i > 0, 1.0, c10::nullopt);
    k0 += ks_;
  }
}

// Grouped over M (MoE forward / input-gradient):
//   c[rows of g] = a[rows of g] @ op(b[g])
// a: [R, K] bf16;  b: [G, K, N] (trans_b false) or [G, N, K] (trans_b true);
// grp_start/grp_count: int32 [G] (starts multiples of 128);
// grp_tile_start: int32 [G+1] prefix of ceil(count/128)*tiles_n (device).
void grouped_gemm_m(torch::Tensor a, torch::Tensor b, torch::Tensor c, torch::Tensor grp_start,
                    torch::Tensor grp_count, torch::Tensor grp_tile_start, bool trans_b,
                    bool accumulate) {
  check_bf16(a, "a");
  check_bf16(b, "b");
  HB_CHECK(b.dim() == 3 && b.is_contiguous(), "b must be contiguous [G, *, *]");
  const int G = b.size(0);
  const int R = a.size(0), K = a.size(1);
  const int N = trans_b ? b.size(1) : b.size(2);
  HB_CHECK((trans_b ? b.size(2) : b.size(1)) == K, "grouped_gemm_m: inner dims differ");
  HB_CHECK(c.size(0) == R && c.size(1) == N && c.stride(1) == 1, "grouped_gemm_m: bad output");
  HB_CHECK(grp_start.numel() == G && grp_count.numel() == G && grp_tile_start.numel() == G + 1,
           "grouped_gemm_m: bad group arrays");
  if (R == 0) return;
  const c10::cuda::CUDAGuard guard(a.device());
  const int BN = pick_bn(N);
  CUtensorMap ta = tmap_bf16_2d(a.data_ptr(), R, K, a.stride(0), 64, GEMM_BM);
  CUtensorMap tb = trans_b ? tmap_bf16_3d(b.data_ptr(), G, N, K, K, (uint64_t)N * K, 64, BN)
                           : tmap_bf16_3d(b.data_ptr(), G, K, N, N, (uint64_t)K * N, 64, 64);
  GemmArgs args = base_args(c, 1.0);
  args.M = R;
  args.N = N;
  args.K = K;
  args.tiles_n = (N + BN - 1) / BN;
  args.num_groups = G;
  args.grp_start = grp_start.data_ptr<int>();
  args.grp_count = grp_count.data_ptr<int>();
  args.grp_tile_start = grp_tile_start.data_ptr<int>();
  const int max_tiles = ((R + GEMM_BM - 1) / GEMM_BM) * args.tiles_n;
  const int grid = std::max(1, std::min(max_tiles, num_sms()));
  const int epi = epi_of(c, accumulate);
  gemm_dispatch_grouped(GROUPED_M, BN, false, !trans_b, epi, ta, tb, args, grid);
}

// Grouped over M with the SwiGLU backward in the epilogue (MoE backward):
//   dh[rows of g] = a[rows of g] @ b[g]^T   (a [R, D] = dY, b [G, F, D] = W_down)
//   dgu = [dh * u * silu'(g) | dh * silu(g)]   from gu = [g | u] ([R, 2F] bf16)
// dh never reaches memory; pad rows of each expert segment get zeros.
void grouped_gemm_m_swiglu_bwd(torch::Tensor a, torch::Tensor b, torch::Tensor gu, torch::Tensor dgu,
                               torch::Tensor grp_start, torch::Tensor grp_count, torch::Tensor grp_tile_start) {
  check_bf16(a, "a");
  check_bf16(b, "b");
  check_bf16(gu, "gu");
  check_bf16(dgu, "dgu");
  HB_CHECK(b.dim() == 3 && b.is_contiguous(), "b must be contiguous [G, F, D]");
  const int G = b.size(0);
  const int R = a.size(0), K = a.size(1);
  const int F = b.size(1);
  HB_CHECK(b.size(2) == K, "grouped_gemm_m_swiglu_bwd: inner dims differ");
  HB_CHECK(gu.is_contiguous() && dgu.is_contiguous() && gu.size(0) == R && gu.size(1) == 2 * F &&
               dgu.size(0) == R && dgu.size(1) == 2 * F,
           "grouped_gemm_m_swiglu_bwd: gu / dgu must be contiguous [R, 2F]");
  HB_CHECK(grp_start.numel() == G && grp_count.numel() == G && grp_tile_start.numel() == G + 1,
           "grouped_gemm_m_swiglu_bwd: bad group arrays");
  if (R == 0) return;
  const c10::cuda::CUDAGuard guard(a.device());
  const int BN = pick_bn(F);
  CUtensorMap ta = tmap_bf16_2d(a.data_ptr(), R, K, a.stride(0), 64, GEMM_BM);
  CUtensorMap tb = tmap_bf16_3d(b.data_ptr(), G, F, K, K, (uint64_t)F * K, 64, BN);
  GemmArgs args = base_args(dgu, 1.0);
  args.ldc = 2LL * F;
  args.aux = gu.data_ptr();
  args.M = R;
  args.N = F;
  args.K = K;
  args.tiles_n = (F + BN - 1) / BN;
  args.num_groups = G;
  args.grp_start = grp_start.data_ptr<int>();
  args.grp_count = grp_count.data_ptr<int>();
  args.grp_tile_start = grp_tile_start.data_ptr<int>();
  const int max_tiles = ((R + GEMM_BM - 1) / GEMM_BM) * args.tiles_n;
  const int grid = std::max(1, std::min(max_tiles, num_sms()));
  gemm_dispatch_grouped(GROUPED_M, BN, false, false, EPI_SWIGLU_BWD, ta, tb, args, grid);
}

// Grouped over M with the SwiGLU in the epilogue (MoE expert forward):
//   g = a @ b1[g], u = a @ b2[g]  (a [R, K], b1 / b2 [G, K, F] MN-major)
//   gu = [g | u] (bf16, kept for the backward), h = bf16(silu(g)) * u
// grp_tile_start counts tiles of the virtual width 2F in 256-column tiles.
void grouped_gemm_m_swiglu_fwd(torch::Tensor a, torch::Tensor b1, torch::Tensor b2, torch::Tensor h,
                               torch::Tensor gu, torch::Tensor grp_start, torch::Tensor grp_count,
                               torch::Tensor grp_tile_start) {
  check_bf16(a, "a");
  check_bf16(b1, "b1");
  check_bf16(b2, "b2");
  check_bf16(h, "h");
  check_bf16(gu, "gu");
  HB_CHECK(b1.dim() == 3 && b1.is_contiguous() && b2.is_contiguous() && b1.sizes() == b2.sizes(),
           "grouped_gemm_m_swiglu_fwd: b1 / b2 must be contiguous [G, K, F] of one shape");
  const int G = b1.size(0), K = b1.size(1), F = b1.size(2);
  const int R = a.size(0);
  HB_CHECK(a.size(1) == K && a.stride(1) == 1, "grouped_gemm_m_swiglu_fwd: a must be [R, K]");
  HB_CHECK(F % 128 == 0, "grouped_gemm_m_swiglu_fwd: F must be a multiple of 128");
  HB_CHECK(h.is_contiguous() && h.size(0) == R && h.size(1) == F, "grouped_gemm_m_swiglu_fwd: h must be [R, F]");
  HB_CHECK(gu.is_contiguous() && gu.size(0) == R && gu.size(1) == 2 * F,
           "grouped_gemm_m_swiglu_fwd: gu must be [R, 2F]");
  HB_CHECK(grp_start.numel() == G && grp_count.numel() == G && grp_tile_start.numel() == G + 1,
           "grouped_gemm_m_swiglu_fwd: bad group arrays");
  if (R == 0) return;
  const c10::cuda::CUDAGuard guard(a.device());
  constexpr int BN = 256;
  CUtensorMap ta = tmap_bf16_2d(a.data_ptr(), R, K, a.stride(0), 64, GEMM_BM);
  CUtensorMap tb = tmap_bf16_3d(b1.data_ptr(), G, K, F, F, (uint64_t)K * F, 64, 64);
  GatherMaps gm{};
  gm.b_hi = tmap_bf16_3d(b2.data_ptr(), G, K, F, F, (uint64_t)K * F, 64, 64);
  GemmArgs args = base_args(h, 1.0);
  args.c2 = gu.data_ptr();
  args.ldc2 = 2LL * F;
  args.M = R;
  args.N = 2 * F;
  args.K = K;
  args.tiles_n = 2 * F / BN;
  args.num_groups = G;
  args.grp_start = grp_start.data_ptr<int>();
  args.grp_count = grp_count.data_ptr<int>();
  args.grp_tile_start = grp_tile_start.data_ptr<int>();
  const int max_tiles = ((R + GEMM_BM - 1) / GEMM_BM) * args.tiles_n;
  const int grid = std::max(1, std::min(max_tiles, num_sms()));
  gemm_dispatch_grouped(GROUPED_M, BN, false, true, EPI_SWIGLU_FWD, ta, tb, args, grid, &gm);
}

// Grouped over M with two K-major B operands concatenated along K (MoE
// input gradient through the SwiGLU's gate and up projections, one GEMM):
//   c[rows of g] = a[rows of g, :K1] @ b1[g]^T + a[rows of g, K1:] @ b2[g]^T
// a [R, 2 K1] (dg | du), b1 / b2 [G, N, K1] (W_gate, W_up), c [R, N] bf16 or fp32
// (written once, no second accumulating pass).
void grouped_gemm_m_cat2(torch::Tensor a, torch::Tensor b1, torch::Tensor b2, torch::Tensor c,
                         torch::Tensor grp_start, torch::Tensor grp_count, torch::Tensor grp_tile_start) {
  check_bf16(a, "a");
  check_bf16(b1, "b1");
  check_bf16(b2, "b2");
  HB_CHECK(b1.dim() == 3 && b1.is_contiguous() && b2.is_contiguous() && b1.sizes() == b2.sizes(),
           "grouped_gemm_m_cat2: b1 / b2 must be contiguous [G, N, K1] of one shape");
  const int G = b1.size(0), N = b1.size(1), K1 = b1.size(2);
  const int R = a.size(0);
  HB_CHECK(a.size(1) == 2 * K1 && a.stride(1) == 1, "grouped_gemm_m_cat2: a must be [R, 2 K1]");
  HB_CHECK(K1 % GEMM_BK == 0, "grouped_gemm_m_cat2: K1 must be a multiple of 64");
  HB_CHECK(c.size(0) == R && c.size(1) == N && c.stride(1) == 1, "grouped_gemm_m_cat2: bad output");
  HB_CHECK(grp_start.numel() == G && grp_count.numel() == G && grp_tile_start.numel() == G + 1,
           "grouped_gemm_m_cat2: bad group arrays");
  if (R == 0) return;
  const c10::cuda::CUDAGuard guard(a.device());
  const int BN = pick_bn(N);
  CUtensorMap ta = tmap_bf16_2d(a.data_ptr(), R, 2 * K1, a.stride(0), 64, GEMM_BM);
  CUtensorMap tb = tmap_bf16_3d(b1.data_ptr(), G, N, K1, K1, (uint64_t)N * K1, 64, BN);
  GatherMaps gm{};
  gm.b_hi = tmap_bf16_3d(b2.data_ptr(), G, N, K1, K1, (uint64_t)N * K1, 64, BN);
  GemmArgs args = base_args(c, 1.0);
  args.M = R;
  args.N = N;
  args.K = 2 * K1;
  args.k_split_b = K1;
  args.tiles_n = (N + BN - 1) / BN;
  args.num_groups = G;
  args.grp_start = grp_start.data_ptr<int>();
  args.grp_count = grp_count.data_ptr<int>();
  args.grp_tile_start = grp_tile_start.data_ptr<int>();
  const int max_tiles = ((R + GEMM_BM - 1) / GEMM_BM) * args.tiles_n;
  const int grid = std::max(1, std::min(max_tiles, num_sms()));
  gemm_dispatch_grouped(GROUPED_M, BN, false, false, epi_of(c, false), ta, tb, args, grid, &gm);
}

// Grouped over K (MoE weight gradients):  c[g] (+)= a_g^T @ b_g
// a: [R, M] bf16 rows of group g at [start, start+count);  b: [R, N] bf16;
// c: [G, M, N] fp32 (or bf16 without accumulate); counts multiples of 64.
void grouped_gemm_k(torch::Tensor a, torch::Tensor b, torch::Tensor c, torch::Tensor grp_start,
                    torch::Tensor grp_count, bool accumulate) {
  check_bf16(a, "a");
  check_bf16(b, "b");
  HB_CHECK(c.dim() == 3 && c.is_contiguous(), "c must be contiguous [G, M, N]");
  const int G = c.size(0), M = c.size(1), N = c.size(2);
  const int R = a.size(0);
  HB_CHECK(a.size(1) == M && b.size(0) == R && b.size(1) == N, "grouped_gemm_k: bad shapes");
  if (G == 0) return;
  const c10::cuda::CUDAGuard guard(a.device());
  const int BN = pick_bn(N);
  CUtensorMap ta = tmap_bf16_2d(a.data_ptr(), R, M, a.stride(0), 64, 64);
  CUtensorMap tb = tmap_bf16_2d(b.data_ptr(), R, N, b.stride(0), 64, 64);
  GemmArgs args = base_args(c, 1.0);
  args.ldc = N;
  args.c_group_stride = (long long)M * N;
  args.M = M;
  args.N = N;
  args.K = R;
  args.tiles_m = (M + GEMM_BM - 1) / GEMM_BM;
  args.tiles_n = (N + BN - 1) / BN;
  args.num_tiles = G * args.tiles_m * args.tiles_n;
  args.num_groups = G;
  args.grp_start = grp_start.data_ptr<int>();
  args.grp_count = grp_count.data_ptr<int>();
  const int epi = epi_of(c, accumulate);
  if (M >= 128 && N >= 256 && epi != EPI_BF16) {
    const long long ptiles = (long long)G * ((M + PAIR_BM - 1) / PAIR_BM) * ((N + PAIR_BN - 1) / PAIR_BN);
    if (use_pair(ptiles)) {
      GemmArgs pa = args;
      pa.tiles_m = (M + PAIR_BM - 1) / PAIR_BM;
      pa.tiles_n = (N + PAIR_BN - 1) / PAIR_BN;
      pa.num_tiles = G * pa.tiles_m * pa.tiles_n;
      const int grid = 2 * std::min(pa.num_tiles, num_sms() / 2);
      gemm_dispatch_pair(GROUPED_K, true, true, epi, ta, tb, pa, grid);
      return;
    }
  }
  const int grid = std::min(args.num_tiles, num_sms());
  gemm_dispatch_grouped(GROUPED_K, BN, true, true, epi, ta, tb, args, grid);
}

}  // namespace hb
