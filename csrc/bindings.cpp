// Python bindings of the hanuman_b200 native extension (module `_C`).
#include <torch/extension.h>

#include "common/host.h"

namespace hb {
void set_wait_budget_ns(uint64_t ns);
void set_peer_wait_budget_ns(uint64_t ns);
// gemm
void gemm(torch::Tensor a, torch::Tensor b, torch::Tensor c, bool trans_a, bool trans_b,
          bool accumulate, double alpha, c10::optional<torch::Tensor> alpha_t);
void grouped_gemm_m(torch::Tensor a, torch::Tensor b, torch::Tensor c, torch::Tensor grp_start,
                    torch::Tensor grp_count, torch::Tensor grp_tile_start, bool trans_b,
                    bool accumulate);
void grouped_gemm_k(torch::Tensor a, torch::Tensor b, torch::Tensor c, torch::Tensor grp_start,
                    torch::Tensor grp_count, bool accumulate);
void grouped_gemm_m_swiglu_bwd(torch::Tensor a, torch::Tensor b, torch::Tensor gu, torch::Tensor dgu,
                               torch::Tensor grp_start, torch::Tensor grp_count, torch::Tensor grp_tile_start);
void gemm_kseg(torch::Tensor a, std::vector<torch::Tensor> bs, torch::Tensor c, bool accumulate);
void grouped_gemm_m_swiglu_fwd(torch::Tensor a, torch::Tensor b1, torch::Tensor b2, torch::Tensor h,
                               torch::Tensor gu, torch::Tensor grp_start, torch::Tensor grp_count,
                               torch::Tensor grp_tile_start);
void grouped_gemm_m_cat2(torch::Tensor a, torch::Tensor b1, torch::Tensor b2, torch::Tensor c,
                         torch::Tensor grp_start, torch::Tensor grp_count, torch::Tensor grp_tile_start);
void grouped_gemm_m_gather(torch::Tensor a, std::vector<int64_t> peer_ptrs, int64_t rank,
                           int64_t groups_per_rank, torch::Tensor gathered, torch::Tensor flags,
                           torch::Tensor c, torch::Tensor grp_start, torch::Tensor grp_count,
                           torch::Tensor grp_tile_start);
// elementwise
void rmsnorm_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor y, torch::Tensor rstd, double eps);
void rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd,
                 torch::Tensor dx, torch::Tensor dw, bool accumulate);
void rope_apply(torch::Tensor q, torch::Tensor cos, torch::Tensor sin, int64_t seq_len,
                c10::optional<torch::Tensor> positions, bool inverse);
void swiglu_fwd(torch::Tensor gu, torch::Tensor h, c10::optional<torch::Tensor> row_src);
void swiglu_bwd(torch::Tensor dh, torch::Tensor gu, torch::Tensor dgu, c10::optional<torch::Tensor> row_src);
void embed_fwd(torch::Tensor tok, torch::Tensor wte, torch::Tensor x);
void embed_bwd(torch::Tensor tok, torch::Tensor dx, torch::Tensor dwte);
void ce_fwd_bwd(torch::Tensor logits, torch::Tensor tgt, c10::optional<torch::Tensor> valid,
                torch::Tensor loss_sum, torch::Tensor dlogits, double scale);
void sumsq(torch::Tensor a, torch::Tensor out);
void fused_update(torch::Tensor p, torch::Tensor g, torch::Tensor m, c10::optional<torch::Tensor> v,
                  torch::Tensor decay, torch::Tensor work, int64_t mode, double lr, double wd,
                  double b1, double b2, double eps, int64_t step, torch::Tensor coef);
void add_norm_fwd(torch::Tensor x, torch::Tensor a, torch::Tensor rs, torch::Tensor w, double eps,
                  torch::Tensor xn, torch::Tensor h, torch::Tensor rstd);
void add_norm_bwd(c10::optional<torch::Tensor> g, torch::Tensor dh, torch::Tensor xn, torch::Tensor a,
                  torch::Tensor rs, torch::Tensor w, torch::Tensor rstd, torch::Tensor dx, torch::Tensor da,
                  torch::Tensor drs, torch::Tensor dw);
// moe
void router_fwd(torch::Tensor x, torch::Tensor W, torch::Tensor bias, int64_t S, int64_t K,
                bool softmax_mode, double scaling, torch::Tensor logits, torch::Tensor topi,
                torch::Tensor topw, torch::Tensor seq_counts, torch::Tensor seq_probs,
                torch::Tensor sums);
void router_bwd(torch::Tensor logits, torch::Tensor topi, torch::Tensor dtopw, torch::Tensor bal_coef,
                int64_t S, bool softmax_mode, double scaling, torch::Tensor coef_z, torch::Tensor dlogits);
void router_grads(torch::Tensor x, torch::Tensor W, torch::Tensor dl, torch::Tensor dx, torch::Tensor dW);
void moe_plan(torch::Tensor topi, int64_t N, int64_t tiles_n, torch::Tensor counts,
              torch::Tensor starts, torch::Tensor tile_prefix, torch::Tensor padded_counts,
              torch::Tensor total_rows, torch::Tensor pos, torch::Tensor row_src);
void moe_gather(torch::Tensor x, torch::Tensor row_src, torch::Tensor xp, int64_t K);
void moe_scatter_add(torch::Tensor dxp, torch::Tensor pos, torch::Tensor dx, c10::optional<torch::Tensor> out_b);
void moe_combine(torch::Tensor y, torch::Tensor pos, torch::Tensor w, torch::Tensor out);
void moe_combine_bwd(torch::Tensor dout, torch::Tensor y, torch::Tensor pos, torch::Tensor w,
                     torch::Tensor row_src, torch::Tensor dy, torch::Tensor dw);
// attention
void flash_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor lse,
               int64_t window);
void flash_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor dout,
               torch::Tensor lse, torch::Tensor delta, torch::Tensor dq, torch::Tensor dk, torch::Tensor dv,
               int64_t window);
// kda
void kda_out_gate_fwd(torch::Tensor o, torch::Tensor gl, torch::Tensor w, torch::Tensor gb, double eps,
                      torch::Tensor y, torch::Tensor rstd);
void kda_out_gate_bwd(torch::Tensor dy, torch::Tensor o, torch::Tensor gl, torch::Tensor w, torch::Tensor gb,
                      torch::Tensor rstd, torch::Tensor dO, torch::Tensor dgl, torch::Tensor dw,
                      torch::Tensor dgb);
int64_t kda_chunk_size(int64_t dk);
void kda_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g, torch::Tensor beta,
             double scale, torch::Tensor o, torch::Tensor Wt, torch::Tensor Ut, torch::Tensor Kh,
             torch::Tensor Qg, torch::Tensor Pm, torch::Tensor gC, torch::Tensor states,
             c10::optional<torch::Tensor> init_state, c10::optional<torch::Tensor> final_state);
void kda_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g, torch::Tensor beta,
             double scale, torch::Tensor dout, torch::Tensor Wt, torch::Tensor Kh, torch::Tensor Qg,
             torch::Tensor Pm, torch::Tensor gC, torch::Tensor states, torch::Tensor dstates,
             torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor dg, torch::Tensor dbeta);
void kda_fwd64(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g, torch::Tensor beta,
               double scale, torch::Tensor o, torch::Tensor Wt, torch::Tensor Ut, torch::Tensor Kh,
               torch::Tensor Qg, torch::Tensor Pm, torch::Tensor gC, torch::Tensor states,
               torch::Tensor Linv, torch::Tensor Am, torch::Tensor U);
void kda_bwd64(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g, torch::Tensor beta,
               double scale, torch::Tensor dout, torch::Tensor Wt, torch::Tensor Ut, torch::Tensor Kh,
               torch::Tensor Qg, torch::Tensor Pm, torch::Tensor gC, torch::Tensor states,
               torch::Tensor Linv, torch::Tensor Am, torch::Tensor U, torch::Tensor dstates,
               torch::Tensor dU, torch::Tensor dUp, torch::Tensor dSq, torch::Tensor dQg,
               torch::Tensor dKh, torch::Tensor dWt, torch::Tensor dP, torch::Tensor dgC,
               torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor dg, torch::Tensor dbeta);
void kda64_set_profile(c10::optional<torch::Tensor> counters);
void kda64_tc_products(torch::Tensor dout, torch::Tensor dU, torch::Tensor states, torch::Tensor dstates,
                       torch::Tensor U, torch::Tensor dWt, torch::Tensor dQg, torch::Tensor dP, torch::Tensor dKh,
                       torch::Tensor dgC);
void kda_prep_fwd(torch::Tensor raw, torch::Tensor wq, torch::Tensor wk, torch::Tensor wv, torch::Tensor f,
                  torch::Tensor a_log, torch::Tensor dt_bias, torch::Tensor braw, int64_t gate_mode,
                  int64_t S, torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g,
                  torch::Tensor beta);
void kda_prep_bwd(torch::Tensor raw, torch::Tensor wq, torch::Tensor wk, torch::Tensor wv, torch::Tensor f,
                  torch::Tensor a_log, torch::Tensor dt_bias, torch::Tensor beta, int64_t gate_mode,
                  int64_t S, torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor dg,
                  torch::Tensor dbeta, torch::Tensor df, torch::Tensor dbraw,
                  torch::Tensor d_alog, torch::Tensor d_dtb, torch::Tensor draw, torch::Tensor dwq,
                  torch::Tensor dwk, torch::Tensor dwv);
// comm
void p2p_barrier(torch::Tensor pads, int64_t rank, int64_t world, int64_t epoch);
void p2p_reduce_scatter(torch::Tensor peers, int64_t world, int64_t off, int64_t n, torch::Tensor out,
                        double scale, torch::Tensor sumsq);
void p2p_update_bcast(torch::Tensor p, torch::Tensor g, torch::Tensor m, c10::optional<torch::Tensor> v,
                      torch::Tensor decay, torch::Tensor work_peers, int64_t world, int64_t off,
                      bool work_bf16, int64_t mode, double lr, double wd, double b1, double b2, double eps,
                      int64_t step, torch::Tensor coef);
// expert parallel
void ep_scatter(torch::Tensor x, c10::optional<torch::Tensor> dout, c10::optional<torch::Tensor> w,
                c10::optional<torch::Tensor> ret, c10::optional<torch::Tensor> dw, torch::Tensor topi,
                torch::Tensor pos, torch::Tensor starts, torch::Tensor peers, int64_t me, int64_t E,
                int64_t Nl, int64_t cap, bool backward);
void ep_zero_pads(torch::Tensor counts, torch::Tensor peers, c10::optional<torch::Tensor> count_peers,
                  int64_t D, int64_t me, int64_t E, int64_t Nl, int64_t cap);
void ep_return(torch::Tensor rows, torch::Tensor cnt, torch::Tensor peers, int64_t me, int64_t E, int64_t Nl,
               int64_t cap);
void ep_combine(torch::Tensor ret, c10::optional<torch::Tensor> w, torch::Tensor topi, torch::Tensor pos,
                torch::Tensor starts, torch::Tensor out, int64_t cap);
}  // namespace hb

static int64_t read_status() {
  int v = 0;
  HB_CUDA_CHECK(cudaMemcpy(&v, hb::status_ptr(), sizeof(int), cudaMemcpyDeviceToHost));
  return v;
}
static void clear_status() { HB_CUDA_CHECK(cudaMemset(hb::status_ptr(), 0, sizeof(int))); }

// The status word of the current device as a one-element int32 CUDA tensor
// (a view: it lives as long as the process), for asynchronous copies.
static torch::Tensor status_view() {
  int dev = 0;
  HB_CUDA_CHECK(cudaGetDevice(&dev));
  return torch::from_blob(hb::status_ptr(), {1},
                          torch::TensorOptions().dtype(torch::kInt32).device(torch::kCUDA, dev));
}

// FSDP gather through the copy engines: out[r * shard_bytes ...] = bytes at
// srcs[r] (every rank's shard, peer addresses included), one cudaMemcpyAsync
// per rank on the current stream; no SM runs the copy, so it overlaps compute.
static void copy_engine_gather(std::vector<int64_t> srcs, int64_t shard_bytes, torch::Tensor out) {
  HB_CHECK(out.is_contiguous() && (int64_t)out.numel() * out.element_size() == shard_bytes * (int64_t)srcs.size(),
           "copy_engine_gather: contiguous output of world * shard bytes");
  char* dst = reinterpret_cast<char*>(out.data_ptr());
  const cudaStream_t st = hb::cur_stream();
  for (size_t r = 0; r < srcs.size(); ++r)
    HB_CUDA_CHECK(cudaMemcpyAsync(dst + r * shard_bytes, reinterpret_cast<const void*>(srcs[r]), shard_bytes,
                                  cudaMemcpyDeviceToDevice, st));
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "hanuman_b200 sm_100a kernels";
  m.def("num_sms", &hb::num_sms);
  m.def("read_status", &read_status, "read the device status word (0 = ok)");
  m.def("clear_status", &clear_status);
  m.def("status_view", &status_view, "the device status word as an int32 tensor view");
  m.def("copy_engine_gather", &copy_engine_gather);
  m.def("set_wait_budget_ns", &hb::set_wait_budget_ns);
  m.def("set_peer_wait_budget_ns", &hb::set_peer_wait_budget_ns);
  m.def("gemm", &hb::gemm, "c (+)= op(a) @ op(b) on tcgen05", py::arg("a"), py::arg("b"),
        py::arg("c"), py::arg("trans_a"), py::arg("trans_b"), py::arg("accumulate"),
        py::arg("alpha") = 1.0, py::arg("alpha_t") = py::none());
  m.def("grouped_gemm_m", &hb::grouped_gemm_m, py::arg("a"), py::arg("b"), py::arg("c"),
        py::arg("grp_start"), py::arg("grp_count"), py::arg("grp_tile_start"), py::arg("trans_b"),
        py::arg("accumulate") = false);
  m.def("grouped_gemm_k", &hb::grouped_gemm_k);
  m.def("grouped_gemm_m_gather", &hb::grouped_gemm_m_gather);
  m.def("grouped_gemm_m_swiglu_bwd", &hb::grouped_gemm_m_swiglu_bwd);
  m.def("grouped_gemm_m_cat2", &hb::grouped_gemm_m_cat2);
  m.def("gemm_kseg", &hb::gemm_kseg);
  m.def("grouped_gemm_m_swiglu_fwd", &hb::grouped_gemm_m_swiglu_fwd);
  m.def("rmsnorm_fwd", &hb::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &hb::rmsnorm_bwd);
  m.def("rope_apply", &hb::rope_apply);
  m.def("swiglu_fwd", &hb::swiglu_fwd, py::arg("gu"), py::arg("h"), py::arg("row_src") = py::none());
  m.def("swiglu_bwd", &hb::swiglu_bwd, py::arg("dh"), py::arg("gu"), py::arg("dgu"),
        py::arg("row_src") = py::none());
  m.def("embed_fwd", &hb::embed_fwd);
  m.def("embed_bwd", &hb::embed_bwd);
  m.def("ce_fwd_bwd", &hb::ce_fwd_bwd);
  m.def("sumsq", &hb::sumsq);
  m.def("fused_update", &hb::fused_update);
  m.def("add_norm_fwd", &hb::add_norm_fwd);
  m.def("add_norm_bwd", &hb::add_norm_bwd);
  m.def("kda_out_gate_fwd", &hb::kda_out_gate_fwd);
  m.def("kda_out_gate_bwd", &hb::kda_out_gate_bwd);
  m.def("router_fwd", &hb::router_fwd);
  m.def("router_bwd", &hb::router_bwd);
  m.def("router_grads", &hb::router_grads);
  m.def("moe_plan", &hb::moe_plan);
  m.def("moe_gather", &hb::moe_gather);
  m.def("moe_scatter_add", &hb::moe_scatter_add, py::arg("dxp"), py::arg("pos"), py::arg("dx"),
        py::arg("out_b") = py::none());
  m.def("moe_combine", &hb::moe_combine);
  m.def("moe_combine_bwd", &hb::moe_combine_bwd);
  m.def("flash_fwd", &hb::flash_fwd);
  m.def("flash_bwd", &hb::flash_bwd);
  m.def("kda_chunk_size", &hb::kda_chunk_size);
  m.def("kda_fwd", &hb::kda_fwd);
  m.def("kda_bwd", &hb::kda_bwd);
  m.def("kda_fwd64", &hb::kda_fwd64);
  m.def("kda_bwd64", &hb::kda_bwd64);
  m.def("kda64_set_profile", &hb::kda64_set_profile);
  m.def("kda64_tc_products", &hb::kda64_tc_products);
  m.def("kda_prep_fwd", &hb::kda_prep_fwd);
  m.def("kda_prep_bwd", &hb::kda_prep_bwd);
  m.def("p2p_barrier", &hb::p2p_barrier);
  m.def("p2p_reduce_scatter", &hb::p2p_reduce_scatter);
  m.def("p2p_update_bcast", &hb::p2p_update_bcast);
  m.def("ep_scatter", &hb::ep_scatter);
  m.def("ep_zero_pads", &hb::ep_zero_pads);
  m.def("ep_return", &hb::ep_return);
  m.def("ep_combine", &hb::ep_combine);
}
