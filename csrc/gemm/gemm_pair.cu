// Instantiations of the CTA-pair tcgen05 GEMM (dense and grouped-over-K).
#include "gemm_pair.cuh"

namespace hb {

void gemm_dispatch_pair(int mode, bool a_mn, bool b_mn, int epi, const CUtensorMap& ta, const CUtensorMap& tb,
                        const GemmArgs& args, int grid, const KSegMaps* ks) {
#define HB_P(MD, AM, BMN, E)                                         \
  if (mode == MD && a_mn == AM && b_mn == BMN && epi == E) {         \
    gemm_pair_launch<AM, BMN, MD, E>(ta, tb, args, grid, ks);        \
    return;                                                          \
  }
  HB_P(DENSE, false, true, EPI_BF16) HB_P(DENSE, false, true, EPI_F32) HB_P(DENSE, false, true, EPI_F32_ACC)
  HB_P(DENSE, false, false, EPI_BF16) HB_P(DENSE, false, false, EPI_F32) HB_P(DENSE, false, false, EPI_F32_ACC)
  HB_P(DENSE, true, true, EPI_BF16) HB_P(DENSE, true, true, EPI_F32) HB_P(DENSE, true, true, EPI_F32_ACC)
  HB_P(GROUPED_K, true, true, EPI_F32) HB_P(GROUPED_K, true, true, EPI_F32_ACC)
#undef HB_P
  HB_CHECK(false, "unsupported pair gemm variant");
}

}  // namespace hb
