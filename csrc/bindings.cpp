// Python bindings of the hanuman_b200 native extension (module `_C`).
#include <torch/extension.h>

#include "common/host.h"

namespace hb {
void set_wait_budget_ns(uint64_t ns);
// gemm
void gemm(torch::Tensor a, torch::Tensor b, torch::Tensor c, bool trans_a, bool trans_b,
          bool accumulate, double alpha);
void grouped_gemm_m(torch::Tensor a, torch::Tensor b, torch::Tensor c, torch::Tensor grp_start,
                    torch::Tensor grp_count, torch::Tensor grp_tile_start, bool trans_b);
void grouped_gemm_k(torch::Tensor a, torch::Tensor b, torch::Tensor c, torch::Tensor grp_start,
                    torch::Tensor grp_count, bool accumulate);
}  // namespace hb

static int64_t read_status() {
  int v = 0;
  HB_CUDA_CHECK(cudaMemcpy(&v, hb::status_ptr(), sizeof(int), cudaMemcpyDeviceToHost));
  return v;
}
static void clear_status() { HB_CUDA_CHECK(cudaMemset(hb::status_ptr(), 0, sizeof(int))); }

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "hanuman_b200 sm_100a kernels";
  m.def("num_sms", &hb::num_sms);
  m.def("read_status", &read_status, "read the device status word (0 = ok)");
  m.def("clear_status", &clear_status);
  m.def("set_wait_budget_ns", &hb::set_wait_budget_ns);
  m.def("gemm", &hb::gemm, "c (+)= op(a) @ op(b) on tcgen05");
  m.def("grouped_gemm_m", &hb::grouped_gemm_m);
  m.def("grouped_gemm_k", &hb::grouped_gemm_k);
}
