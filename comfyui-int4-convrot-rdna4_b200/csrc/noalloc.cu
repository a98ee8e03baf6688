// No-allocation form of the fused W4A4 linear, for callers that cannot
// allocate device memory (no cudaMalloc, no allocator of their own).
//
// ck_convrot_w4a4_linear needs a workspace for the quantized activations (the
// packed codes [M, K/2] and the row scales [M]). This entry takes the same
// arguments minus the workspace and uses a static device array instead:
// kNoAllocScratchBytes of __device__ memory, which the CUDA runtime places
// when it loads this file's module. Nothing here calls cudaMalloc, cudaFree or
// a library call that allocates.
//
// Rules for the caller:
//   - sizes: linear_workspace_bytes(M, K) must not exceed kNoAllocScratchBytes
//     (checked before any CUDA call; -1 and a message otherwise);
//   - nothing in the scratch needs initial contents: the quantizer writes every
//     byte the GEMM reads, on every call;
//   - one scratch per device, shared by every call on that device: two calls
//     that can run at the same time (different streams or host threads without
//     ordering between them) race on it. Calls issued on one stream are
//     ordered and safe;
//   - the first call on a device looks up the scratch address
//     (cudaGetSymbolAddress with that device current), which loads this module;
//     make that first call before any stream capture. Later calls only launch
//     kernels and can be captured.
// This file is its own translation unit so its module (and the scratch with
// it) is loaded only by programs that call this entry.
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <mutex>

#include "linear_api.cuh"

#define CONVROT_API extern "C" __attribute__((visibility("default")))

namespace convrot {

constexpr size_t kNoAllocScratchBytes = static_cast<size_t>(128) << 20;   // 128 MiB per device
constexpr int kNoAllocMaxDevices = 64;

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[kNoAllocMaxDevices];

// Device address of the scratch on the current device (looked up once per device).
int noalloc_scratch(unsigned char** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return static_cast<int>(e);
    if (dev < 0 || dev >= kNoAllocMaxDevices) return fail("device ordinal beyond the no-alloc scratch table (64)");
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_ptr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return static_cast<int>(e);
        g_noalloc_ptr[dev] = p;
    }
    *out = static_cast<unsigned char*>(g_noalloc_ptr[dev]);
    return 0;
}

}  // namespace convrot

using namespace convrot;

CONVROT_API int ck_convrot_w4a4_linear_noalloc(const void* x, int in_dtype, const void* Wp, const void* wscale,
                                               const void* bias, int bias_dtype, void* out, int out_dtype,
                                               int M, int N, int K, int G, void* stream) {
    if (int rc = check_linear_args(x, in_dtype, Wp, wscale, bias_dtype, out, out_dtype, M, N, K, G)) return rc;
    if (M == 0 || N == 0) return 0;
    if (linear_workspace_bytes(M, K) > kNoAllocScratchBytes)
        return fail("M x K too large for the 128 MiB static scratch of ck_convrot_w4a4_linear_noalloc "
                    "(needs ck_convrot_w4a4_linear_workspace_size(M, K) <= 134217728); "
                    "use ck_convrot_w4a4_linear with a workspace, or split the rows");
    unsigned char* scratch = nullptr;
    if (int rc = noalloc_scratch(&scratch)) return rc;
    return run_linear(x, in_dtype, Wp, static_cast<const float*>(wscale), BiasRef{bias, bias_dtype}, out,
                      out_dtype, M, N, K, G, scratch, static_cast<cudaStream_t>(stream));
}
