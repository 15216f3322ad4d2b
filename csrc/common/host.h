// Host-side helpers shared by every extension source: TMA descriptor
// encoding through the driver entry point, the per-device status word that
// kernels write on a bounded-wait timeout, SM count and stream access.
#pragma once
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <cstdint>
#include <string>

namespace hb {

#define HB_CHECK(cond, msg)                                              \
  do {                                                                   \
    if (!(cond)) {                                                       \
      throw std::runtime_error(std::string("hanuman_b200: ") + (msg));   \
    }                                                                    \
  } while (0)

#define HB_CUDA_CHECK(expr)                                                          \
  do {                                                                               \
    cudaError_t _e = (expr);                                                         \
    if (_e != cudaSuccess)                                                           \
      throw std::runtime_error(std::string("hanuman_b200 CUDA error: ") +           \
                               cudaGetErrorString(_e) + " at " + __FILE__ + ":" +    \
                               std::to_string(__LINE__));                            \
  } while (0)

inline cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

int num_sms();
int* status_ptr();  // device status word of the current device (zeroed at creation)
uint64_t wait_budget_ns();       // budget of a bounded wait on work of this GPU
// Budget of a wait on another rank (device barrier on peer signal pads): ranks
// can drift apart by seconds (first steps: lazy module loading, descriptor
// creation), so it is much larger than the on-device budget.
uint64_t peer_wait_budget_ns();

// 2-D / 3-D bf16 (or other) tiled tensor maps with 128-byte swizzle.
// dims/strides are innermost-first; strides in bytes for dims 1..rank-1.
CUtensorMap make_tmap(const void* base, CUtensorMapDataType dtype, int rank,
                      const uint64_t* dims, const uint64_t* strides_bytes,
                      const uint32_t* box, CUtensorMapSwizzle swz);

// Row-major 2-D bf16 matrix [rows, cols] with row stride `ld` (elements);
// box = {box_cols, box_rows}.
CUtensorMap tmap_bf16_2d(const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                         uint32_t box_cols, uint32_t box_rows);
// [groups, rows, cols] row-major bf16, contiguous groups of rows*ld elements.
CUtensorMap tmap_bf16_3d(const void* base, uint64_t groups, uint64_t rows, uint64_t cols,
                         uint64_t ld, uint64_t group_stride, uint32_t box_cols,
                         uint32_t box_rows);

inline void check_bf16(const torch::Tensor& t, const char* name) {
  HB_CHECK(t.is_cuda(), std::string(name) + " must be a CUDA tensor");
  HB_CHECK(t.scalar_type() == at::kBFloat16, std::string(name) + " must be bfloat16");
}

}  // namespace hb
