// No-allocation form of the fused W4A4 linear, for callers that cannot
// allocate device memory: code that runs where a cudaMalloc is not allowed or
// not wanted (a host framework that owns all device memory through its own
// arena and hands out only input and output buffers, a plugin ABI that passes
// plain pointers and no allocator, a process that must not grow its footprint
// after start-up).
//
// ck_convrot_w4a4_linear needs a workspace for the quantized activations (the
// packed codes [M, K/2] and the row scales [M]). This entry takes the same
// arguments minus the workspace and uses a static device array instead:
// kNoAllocScratchBytes of __device__ memory, which the CUDA runtime places
// when it loads this file's module. Nothing here calls cudaMalloc, cudaFree or
// a library call that allocates.
//
// Rules for the caller:
//   - sizes: packed_linear_workspace_bytes(M, K) (the packed codes and row
//     scales; this entry always quantizes to packed codes) must not exceed
//     kNoAllocScratchBytes
//     (checked before any CUDA call; -1 and a message otherwise);
//   - nothing in the scratch needs initial contents: the quantizer writes every
//     byte the GEMM reads, on every call, so the previous call's leftovers are
//     never read;
//   - one scratch per device, shared by every call on that device: two calls
//     that can run at the same time (different streams or host threads without
//     ordering between them) race on it. Calls issued on one stream are
//     ordered and safe;
//   - the first call on a device (and the first call after the device's
//     primary context was reset) looks up the scratch address with
//     cudaGetSymbolAddress, with that device current; make that first call
//     before any stream capture.
// Where the array lives: with lazy module loading (CUDA_MODULE_LOADING=LAZY,
// the default since CUDA 12.2) the module, and with it the 128 MiB, is placed
// on a device by the first call there, so programs that never call this entry
// do not pay for it. With CUDA_MODULE_LOADING=EAGER every module of the
// library is loaded when a context is created, so every process that loads
// libconvrot_b200.so holds the 128 MiB on every device it uses, until exit.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <mutex>

#include "linear_api.cuh"

#define CONVROT_API extern "C" __attribute__((visibility("default")))

namespace convrot {

constexpr size_t kNoAllocScratchBytes = static_cast<size_t>(128) << 20;   // 128 MiB per device
constexpr int kNoAllocMaxDevices = 64;

// The scratch. In host code this name is only a stand-in for the symbol, not a
// device address: the kernels get the address that cudaGetSymbolAddress
// returns for the current device (noalloc_scratch below).
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[kNoAllocMaxDevices];
CUcontext g_noalloc_ctx[kNoAllocMaxDevices];   // context the address above belongs to

// cuCtxGetCurrent through the runtime's driver entry point (no link against
// libcuda); null when the driver does not provide it.
PFN_cuCtxGetCurrent_v4000 ctx_get_current_fn() {
    static PFN_cuCtxGetCurrent_v4000 fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
        return static_cast<PFN_cuCtxGetCurrent_v4000>(nullptr);
    }();
    return fn;
}

CUcontext current_context() {
    CUcontext ctx = nullptr;
    if (auto fn = ctx_get_current_fn()) {
        if (fn(&ctx) != CUDA_SUCCESS) ctx = nullptr;
    }
    return ctx;
}

// Device address of the scratch on the current device. Looked up once per
// device with that device current, and again when the current context is not
// the one the cached address was taken in (the primary context was reset and
// the module reloaded, possibly at another address).
int noalloc_scratch(unsigned char** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return static_cast<int>(e);
    if (dev < 0 || dev >= kNoAllocMaxDevices) return fail("device ordinal beyond the no-alloc scratch table (64)");
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    CUcontext ctx = current_context();
    if (g_noalloc_ptr[dev] == nullptr || ctx == nullptr || ctx != g_noalloc_ctx[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return static_cast<int>(e);
        g_noalloc_ptr[dev] = p;
        g_noalloc_ctx[dev] = current_context();   // the lookup made the primary context current
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
    if (packed_linear_workspace_bytes(M, K) > kNoAllocScratchBytes)
        return fail("M x K too large for the 128 MiB static scratch of ck_convrot_w4a4_linear_noalloc "
                    "(needs align256(M * K / 2) + align256(4 * M) <= 134217728); "
                    "use ck_convrot_w4a4_linear with a workspace, or split the rows");
    unsigned char* scratch = nullptr;
    if (int rc = noalloc_scratch(&scratch)) return rc;
    return run_linear(x, in_dtype, Wp, static_cast<const float*>(wscale), BiasRef{bias, bias_dtype}, out,
                      out_dtype, M, N, K, G, scratch, static_cast<cudaStream_t>(stream), false);
}
