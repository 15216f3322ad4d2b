// Instantiations of the dense tcgen05 GEMM with a K-major A operand.
#include "gemm_kernel.cuh"

namespace hb {

void gemm_dispatch_dense_ak(int bn, bool b_mn, int epi, const CUtensorMap& ta, const CUtensorMap& tb,
                            const GemmArgs& args, int grid) {
#define HB_G(BNV, BMN, E)                                              \
  if (bn == BNV && b_mn == BMN && epi == E) {                          \
    gemm_launch<BNV, false, BMN, DENSE, E>(ta, tb, args, grid);         \
    return;                                                            \
  }
  HB_G(256, true, EPI_BF16) HB_G(256, true, EPI_F32) HB_G(256, true, EPI_F32_ACC)
  HB_G(256, false, EPI_BF16) HB_G(256, false, EPI_F32) HB_G(256, false, EPI_F32_ACC)
  HB_G(128, true, EPI_BF16) HB_G(128, true, EPI_F32) HB_G(128, true, EPI_F32_ACC)
  HB_G(128, false, EPI_BF16) HB_G(128, false, EPI_F32) HB_G(128, false, EPI_F32_ACC)
#undef HB_G
  HB_CHECK(false, "unsupported dense gemm variant");
}

}  // namespace hb
