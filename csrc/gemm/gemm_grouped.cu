// Instantiations of the grouped (MoE) tcgen05 GEMMs.
#include "gemm_kernel.cuh"

namespace hb {

void gemm_dispatch_grouped(int mode, int bn, bool a_mn, bool b_mn, int epi, const CUtensorMap& ta,
                           const CUtensorMap& tb, const GemmArgs& args, int grid, const GatherMaps* gm) {
#define HB_G(MD, BNV, AM, BMN, E)                                      \
  if (mode == MD && bn == BNV && a_mn == AM && b_mn == BMN && epi == E) { \
    gemm_launch<BNV, AM, BMN, MD, E>(ta, tb, args, grid, gm);           \
    return;                                                            \
  }
  HB_G(GROUPED_M, 256, false, true, EPI_BF16) HB_G(GROUPED_M, 256, false, true, EPI_F32)
  HB_G(GROUPED_M, 256, false, false, EPI_F32_ACC) HB_G(GROUPED_M, 128, false, false, EPI_F32_ACC)
  HB_G(GROUPED_M, 256, false, false, EPI_BF16) HB_G(GROUPED_M, 256, false, false, EPI_F32)
  HB_G(GROUPED_M, 128, false, true, EPI_BF16) HB_G(GROUPED_M, 128, false, true, EPI_F32)
  HB_G(GROUPED_M, 128, false, false, EPI_BF16) HB_G(GROUPED_M, 128, false, false, EPI_F32)
  HB_G(GROUPED_M, 256, false, true, EPI_SWIGLU_FWD)
  HB_G(GROUPED_M, 256, false, false, EPI_SWIGLU_BWD) HB_G(GROUPED_M, 128, false, false, EPI_SWIGLU_BWD)
  HB_G(GROUPED_K, 256, true, true, EPI_F32) HB_G(GROUPED_K, 256, true, true, EPI_F32_ACC)
  HB_G(GROUPED_K, 256, true, true, EPI_BF16)
  HB_G(GROUPED_K, 128, true, true, EPI_F32) HB_G(GROUPED_K, 128, true, true, EPI_F32_ACC)
  HB_G(GROUPED_K, 128, true, true, EPI_BF16)
#undef HB_G
  HB_CHECK(false, "unsupported grouped gemm variant");
}

}  // namespace hb
