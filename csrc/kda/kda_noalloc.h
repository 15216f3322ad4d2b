// Allocation-free forward of the chunked gated delta rule (KDA core).
//
// This entry point has no counterpart in the reference (theorionic/hanuman):
// it is an addition for callers that cannot call cudaMalloc themselves, such as
// code that runs while a CUDA graph is being captured, host runtimes that own a
// fixed device-memory pool, and plugins loaded into a process whose allocator
// they must not touch.
//
//   o = KDA(q, k, v, g, beta)   all fp32, q/k/v/g/o [B, S, H, DK], beta [B, S, H]
//
// The caller passes device pointers to the inputs and the output and a stream;
// q, k, v, g and o must be 16-byte aligned (HB_NOALLOC_BAD_SHAPE otherwise).
// Head dims 16, 32 and 64 are accepted; any other DK (the allocating entry
// point also takes 128) returns HB_NOALLOC_BAD_HEAD_DIM.
// The chunk intermediates live in a file-scope __device__ array of 64 MiB
// (16 Mi floats) that every GPU which loads the library holds until the
// process exits; inputs needing more (B * H * ceil(S / 32) * (4*32*DK + 32*32 +
// DK + DK*DK) floats) are rejected with HB_NOALLOC_TOO_LARGE and nothing is
// launched.  No cudaMalloc, cudaFree or allocating library routine is called.
//
// The first call on a device looks the array's device address up with
// cudaGetSymbolAddress (with that device current) and caches it together with
// the device's current CUDA context; make that first call before any stream
// capture begins.  A later call that finds a different current context (after
// cudaDeviceReset, for instance) looks the address up again, so that call too
// must come before any capture.  All calls share the one array:
// calls whose kernels overlap on the GPU (different streams, or concurrent host
// threads) race on it and must be serialised by the caller.  Every scratch
// region is fully written before it is read, so no clearing is needed between
// calls.  Returns HB_NOALLOC_OK (0) on success.
#pragma once
#include <cuda_runtime.h>

#define HB_NOALLOC_OK 0
#define HB_NOALLOC_BAD_HEAD_DIM 1
#define HB_NOALLOC_BAD_SHAPE 2
#define HB_NOALLOC_TOO_LARGE 3
#define HB_NOALLOC_CUDA_ERROR 4

#ifdef __cplusplus
extern "C" {
#endif
int hb_kda_fwd_noalloc(const float* q, const float* k, const float* v, const float* g,
                       const float* beta, float* o, int B, int S, int H, int DK, float scale,
                       cudaStream_t stream);
#ifdef __cplusplus
}
#endif
