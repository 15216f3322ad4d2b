// Host helpers: status word, SM count, TMA descriptor encoding.
#include "host.h"

#include <mutex>
#include <vector>

namespace hb {

namespace {
std::mutex g_mu;
std::vector<int*> g_status;  // per device
std::vector<int> g_sms;
uint64_t g_budget_ns = 4000000000ull;         // 4 s per bounded wait on this GPU
uint64_t g_peer_budget_ns = 120000000000ull;  // 120 s for a wait on another rank

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;

EncodeTiledFn encoder() {
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    HB_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
    HB_CHECK(fn != nullptr && q == cudaDriverEntryPointSuccess,
             "cuTensorMapEncodeTiled not available from the driver");
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
  return g_encode;
}
}  // namespace

int num_sms() {
  int dev;
  HB_CUDA_CHECK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_mu);
  if ((int)g_sms.size() <= dev) g_sms.resize(dev + 1, 0);
  if (!g_sms[dev]) HB_CUDA_CHECK(cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev));
  return g_sms[dev];
}

int* status_ptr() {
  int dev;
  HB_CUDA_CHECK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_mu);
  if ((int)g_status.size() <= dev) g_status.resize(dev + 1, nullptr);
  if (!g_status[dev]) {
    HB_CUDA_CHECK(cudaMalloc(&g_status[dev], 64));
    HB_CUDA_CHECK(cudaMemset(g_status[dev], 0, 64));
  }
  return g_status[dev];
}

uint64_t wait_budget_ns() { return g_budget_ns; }
void set_wait_budget_ns(uint64_t ns) { g_budget_ns = ns; }
uint64_t peer_wait_budget_ns() { return g_peer_budget_ns; }
void set_peer_wait_budget_ns(uint64_t ns) { g_peer_budget_ns = ns; }

CUtensorMap make_tmap(const void* base, CUtensorMapDataType dtype, int rank,
                      const uint64_t* dims, const uint64_t* strides_bytes,
                      const uint32_t* box, CUtensorMapSwizzle swz) {
  HB_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base address must be 16-byte aligned");
  for (int i = 0; i < rank - 1; ++i)
    HB_CHECK(strides_bytes[i] % 16 == 0, "TMA strides must be multiples of 16 bytes");
  CUtensorMap m;
  cuuint64_t gd[5];
  cuuint64_t gs[4];
  cuuint32_t bd[5];
  cuuint32_t es[5];
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bd[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) gs[i] = strides_bytes[i];
  CUresult r = encoder()(&m, dtype, rank, const_cast<void*>(base), gd, gs, bd, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  HB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
  return m;
}

CUtensorMap tmap_bf16_2d(const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                         uint32_t box_cols, uint32_t box_rows) {
  uint64_t dims[2] = {cols, rows};
  uint64_t strides[1] = {ld * 2};
  uint32_t box[2] = {box_cols, box_rows};
  return make_tmap(base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B);
}

CUtensorMap tmap_bf16_3d(const void* base, uint64_t groups, uint64_t rows, uint64_t cols,
                         uint64_t ld, uint64_t group_stride, uint32_t box_cols,
                         uint32_t box_rows) {
  uint64_t dims[3] = {cols, rows, groups};
  uint64_t strides[2] = {ld * 2, group_stride * 2};
  uint32_t box[3] = {box_cols, box_rows, 1};
  return make_tmap(base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace hb
