// Pieces of the fused W4A4 linear shared by its two C entries
// (convrot_b200.cu: caller workspace; noalloc.cu: static scratch).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>

namespace convrot {

// Bias vector [N] in its own dtype (0 = f32, 1 = bf16, 2 = f16, the activation
// codes of the C-ABI) or absent. Widening to fp32 is exact, so reading bf16/f16
// here gives the same sums as adding a bias converted to fp32 beforehand.
struct BiasRef {
    const void* ptr;
    int kind;
    __device__ __forceinline__ float at(int n) const {
        if (kind == 1) return __bfloat162float(static_cast<const __nv_bfloat16*>(ptr)[n]);
        if (kind == 2) return __half2float(static_cast<const __half*>(ptr)[n]);
        return static_cast<const float*>(ptr)[n];
    }
};

// Extra output destinations of the pair GEMM's direct-store epilogue (the
// column-split linear): every output row chunk goes to ptr[0 .. count) at
// row * ldo + col0 + column instead of to `out` at row * N + column. Pointers
// may be other GPUs' memory (peer mappings); count == 0: the plain output.
struct PeerOut {
    void* ptr[8];
    int count;
    int ldo;
    int col0;
};

// Records `msg` for ck_convrot_last_error() and returns -1.
int fail(const char* msg);

// Shape, dtype and pointer checks of the fused linear (no CUDA call).
int check_linear_args(const void* x, int in_dtype, const void* Wp, const void* wscale, int bias_dtype,
                      const void* out, int out_dtype, int M, int N, int K, int G);

// Bytes of scratch the fused linear uses for M rows of K (one int8 per code
// from the A8 form's row count on, packed codes below it).
size_t linear_workspace_bytes(int M, int K);

// Bytes of scratch of the packed-code form alone (allow_a8 = false below).
size_t packed_linear_workspace_bytes(int M, int K);

// Quantizer then GEMM/GEMV on `stream`, scratch at `workspace` (256-byte aligned,
// linear_workspace_bytes or, without allow_a8, packed_linear_workspace_bytes).
// allow_a8: many bf16 rows may take the A8 form (same output bits).
int run_linear(const void* x, int in_dtype, const void* Wp, const float* ws, BiasRef bias, void* out,
               int out_dtype, int M, int N, int K, int G, unsigned char* workspace, cudaStream_t stream,
               bool allow_a8);

}  // namespace convrot
