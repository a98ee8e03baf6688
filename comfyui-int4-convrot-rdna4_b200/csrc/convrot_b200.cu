// ConvRot W4A4 linear path for NVIDIA B200 (sm_100a).
//
// The kernels and the C-ABI that the Python host layer (ctypes) binds:
//
//  (1) convrot_quant_kernel: blockwise regular-Hadamard rotation of an
//      activation row, row-wise absmax int4 quantization and nibble packing.
//      Same contract as the reference's fused quantizer
//      (_int4/int4_gemm.hip:348-408), with the quantizer arithmetic of its
//      eager path (_int4/eager.py:112-120) so codes and scales match eager.
//
//  (2) int4_gemm_pair_kernel (gemm_pair.cuh): packed-int4 x packed-int4 GEMM
//      on the 5th-generation tensor cores, CTA pairs (cta_group::2). Every
//      packed byte is split into its high nibble (b & 0xF0) and its low nibble
//      moved up (b << 4), both int8 values 16*code; tcgen05.mma.kind::i8 on the
//      two halves accumulates 256 * sum_k x_k w_k exactly in int32 TMEM. The
//      epilogue shifts the accumulator back (exact), applies
//      ((D * xs[m]) * ws[n]) + bias[n] in fp32 (_int4/int4_gemm.hip:152-169)
//      and stores bf16 or fp32.
//
//  (3) int4_gemv_kernel: the same product for M <= 4 on CUDA cores (__dp4a),
//      streaming the weights through shared memory at HBM rate.
//
// The reference exports (_int4/int4_gemm.hip:627-741) are mirrored with the
// same names, argument order and return codes: 0 on success, -1 when a shape
// or pointer precondition fails (no launch happens), otherwise the CUDA error.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "sm100_ptx.cuh"
#include "linear_api.cuh"

#define CONVROT_API extern "C" __attribute__((visibility("default")))

namespace convrot {

// Device-side status word: a kernel that gives up on a bounded wait records
// where (a nonzero code) and returns. Read and cleared by ck_convrot_device_status.
__device__ int g_device_status;

enum : int {
    kStatusOk = 0,
    kStatusTimeoutProducer = 1,
    kStatusTimeoutMma = 2,
    kStatusTimeoutExpand = 3,
    kStatusTimeoutEpilogue = 4,
    kStatusTimeoutSelfTest = 5,
    kStatusTimeoutPeer = 6,
};

__device__ __forceinline__ void record_status(int code) { atomicCAS(&g_device_status, 0, code); }

// ===========================================================================
// (1) Fused rotation + quantization + packing
// ===========================================================================

template <typename T> struct Act;
template <> struct Act<__nv_bfloat16> {
    static constexpr int kCode = 1;
    __device__ static float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
    __device__ static __nv_bfloat16 from_f32(float v) { return __float2bfloat16_rn(v); }
    __device__ static float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
    // torch clamps a bf16 tensor at bf16(1e-10).
    __device__ static float floor_value() { return __uint_as_float(0x2EDC0000u); }
};
template <> struct Act<__half> {
    static constexpr int kCode = 2;
    __device__ static float to_f32(__half v) { return __half2float(v); }
    __device__ static __half from_f32(float v) { return __float2half_rn(v); }
    __device__ static float round(float v) { return __half2float(__float2half_rn(v)); }
    __device__ static float floor_value() { return 0.0f; }           // 1e-10 underflows in fp16
};
template <> struct Act<float> {
    static constexpr int kCode = 0;
    __device__ static float to_f32(float v) { return v; }
    __device__ static float from_f32(float v) { return v; }
    __device__ static float round(float v) { return v; }
    __device__ static float floor_value() { return 1e-10f; }
};

// Regular Hadamard H4 = J - 2R (ones, minus twice the anti-diagonal):
// out_i = (v0+v1)+(v2+v3) - 2*v_(3-i), each output rounded once.
__device__ __forceinline__ void h4(float& v0, float& v1, float& v2, float& v3) {
    const float s = __fadd_rn(__fadd_rn(v0, v1), __fadd_rn(v2, v3));
    const float o0 = __fmaf_rn(-2.0f, v3, s);
    const float o1 = __fmaf_rn(-2.0f, v2, s);
    const float o2 = __fmaf_rn(-2.0f, v1, s);
    const float o3 = __fmaf_rn(-2.0f, v0, s);
    v0 = o0; v1 = o1; v2 = o2; v3 = o3;
}

// H16 = H4 (x) H4 on v[16] indexed 4*hi + lo: first along lo, then along hi.
__device__ __forceinline__ void h16(float (&v)[16]) {
    #pragma unroll
    for (int hi = 0; hi < 4; ++hi) h4(v[4 * hi], v[4 * hi + 1], v[4 * hi + 2], v[4 * hi + 3]);
    #pragma unroll
    for (int lo = 0; lo < 4; ++lo) h4(v[lo], v[lo + 4], v[lo + 8], v[lo + 12]);
}

__device__ __forceinline__ void h4_low_digit(float (&v)[16]) {
    #pragma unroll
    for (int hi = 0; hi < 4; ++hi) h4(v[4 * hi], v[4 * hi + 1], v[4 * hi + 2], v[4 * hi + 3]);
}

template <typename T>
__device__ __forceinline__ void load16(const T* p, float (&v)[16]) {
    if constexpr (sizeof(T) == 2) {
        const uint4* q = reinterpret_cast<const uint4*>(p);
        uint4 a = q[0], b = q[1];
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        #pragma unroll
        for (int i = 0; i < 8; ++i) {
            T lo, hi;
            uint16_t l16 = static_cast<uint16_t>(w[i] & 0xFFFF), h16v = static_cast<uint16_t>(w[i] >> 16);
            memcpy(&lo, &l16, 2);
            memcpy(&hi, &h16v, 2);
            v[2 * i] = Act<T>::to_f32(lo);
            v[2 * i + 1] = Act<T>::to_f32(hi);
        }
    } else {
        const float4* q = reinterpret_cast<const float4*>(p);
        #pragma unroll
        for (int i = 0; i < 4; ++i) {
            float4 a = q[i];
            v[4 * i] = a.x; v[4 * i + 1] = a.y; v[4 * i + 2] = a.z; v[4 * i + 3] = a.w;
        }
    }
}

constexpr int kQuantThreads = 256;
constexpr int kTrStride = 20;                        // floats per transposed row (16 + pad, 16 B aligned)
constexpr int kTransposeFloats = 16 * 16 * kTrStride; // 16 half-warps x 16 x 20

// 16x16 transpose of 4-bit codes held by the 16 lanes of a half-warp. On entry
// lane b holds column b of a tile, nibble a (bits 4a..4a+3 of the 64-bit word
// {lo, hi}) = element (a, b); on exit lane t holds row t, nibble b = element
// (t, b) -- which, read as 8 little-endian bytes, is the packed int4 row
// (column 2c in the low nibble of byte c). Four butterfly exchanges with the
// lane at distance 8, 4, 2, 1, each swapping the half of the word whose
// nibble-index bit differs from the lane's bit.
__device__ __forceinline__ void transpose_nibbles16(uint32_t& lo, uint32_t& hi, int j, unsigned hmask) {
    // distance 8: nibbles 8..15 are the high word
    {
        const bool up = j & 8;
        const uint32_t got = __shfl_xor_sync(hmask, up ? lo : hi, 8);
        if (up) lo = got; else hi = got;
    }
    // distance 4: nibbles with bit 2 set are the upper 16 bits of each word
    {
        const bool up = j & 4;
        const uint32_t send = up ? __byte_perm(lo, hi, 0x5410) : __byte_perm(lo, hi, 0x7632);
        const uint32_t got = __shfl_xor_sync(hmask, send, 4);
        if (up) { lo = __byte_perm(lo, got, 0x3254); hi = __byte_perm(hi, got, 0x3276); }
        else    { lo = __byte_perm(lo, got, 0x5410); hi = __byte_perm(hi, got, 0x7610); }
    }
    // distance 2: nibbles with bit 1 set are the odd bytes of each word
    {
        const bool up = j & 2;
        const uint32_t send = up ? __byte_perm(lo, hi, 0x6420) : __byte_perm(lo, hi, 0x7531);
        const uint32_t got = __shfl_xor_sync(hmask, send, 2);
        if (up) { lo = __byte_perm(lo, got, 0x3514); hi = __byte_perm(hi, got, 0x3716); }
        else    { lo = __byte_perm(lo, got, 0x5240); hi = __byte_perm(hi, got, 0x7260); }
    }
    // distance 1: nibbles with bit 0 set are the high nibbles of each byte
    {
        const bool up = j & 1;
        const uint32_t send = up ? ((lo & 0x0F0F0F0Fu) | ((hi & 0x0F0F0F0Fu) << 4))
                                 : (((lo >> 4) & 0x0F0F0F0Fu) | (hi & 0xF0F0F0F0u));
        const uint32_t got = __shfl_xor_sync(hmask, send, 1);
        if (up) { lo = (lo & 0xF0F0F0F0u) | (got & 0x0F0F0F0Fu); hi = (hi & 0xF0F0F0F0u) | ((got >> 4) & 0x0F0F0F0Fu); }
        else    { lo = (lo & 0x0F0F0F0Fu) | ((got & 0x0F0F0F0Fu) << 4); hi = (hi & 0x0F0F0F0Fu) | (got & 0xF0F0F0F0u); }
    }
}

// ---- paired fp32 arithmetic (sm_100 f32x2): one instruction for two independent lanes of work
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

// h4 on two tiles at once (same arithmetic as h4(), per component).
__device__ __forceinline__ void h4x2(float2& v0, float2& v1, float2& v2, float2& v3) {
    const float2 m2 = make_float2(-2.0f, -2.0f);
    const float2 s = add2(add2(v0, v1), add2(v2, v3));
    const float2 o0 = fma2(m2, v3, s), o1 = fma2(m2, v2, s), o2 = fma2(m2, v1, s), o3 = fma2(m2, v0, s);
    v0 = o0; v1 = o1; v2 = o2; v3 = o3;
}
__device__ __forceinline__ void h16x2(float2 (&v)[16]) {
    #pragma unroll
    for (int hi = 0; hi < 4; ++hi) h4x2(v[4 * hi], v[4 * hi + 1], v[4 * hi + 2], v[4 * hi + 3]);
    #pragma unroll
    for (int lo = 0; lo < 4; ++lo) h4x2(v[lo], v[lo + 4], v[lo + 8], v[lo + 12]);
}
__device__ __forceinline__ void h4_low_digit_x2(float2 (&v)[16]) {
    #pragma unroll
    for (int hi = 0; hi < 4; ++hi) h4x2(v[4 * hi], v[4 * hi + 1], v[4 * hi + 2], v[4 * hi + 3]);
}

// Rounded rotated values of two tiles, as kept until the row scale is known:
// 16-bit dtypes packed two per register (tile 2p in the low half), f32 as is.
template <typename T> struct PairStore {
    using type = uint32_t;
    __device__ static type pack(float2 v) {
        if constexpr (Act<T>::kCode == 1) {
            __nv_bfloat162 b = __floats2bfloat162_rn(v.x, v.y);
            uint32_t u; memcpy(&u, &b, 4); return u;
        } else {
            __half2 h = __floats2half2_rn(v.x, v.y);
            uint32_t u; memcpy(&u, &h, 4); return u;
        }
    }
    __device__ static float2 unpack(type u) {
        if constexpr (Act<T>::kCode == 1) {
            return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xFFFF0000u));
        } else {
            __half2 h; memcpy(&h, &u, 4); return __half22float2(h);
        }
    }
};
template <> struct PairStore<float> {
    using type = float2;
    __device__ static type pack(float2 v) { return v; }
    __device__ static float2 unpack(type v) { return v; }
};

// 4-bit two's-complement code of y (a value of the activation dtype) divided
// by the row scale, with the eager quantizer's roundings (generic path).
template <typename T>
__device__ __forceinline__ uint32_t quant_nibble(float y, float s) {
    float qf = rintf(Act<T>::round(__fdiv_rn(y, s)));
    qf = fminf(fmaxf(qf, -7.0f), 7.0f);
    return static_cast<uint32_t>(static_cast<int>(qf)) & 0xFu;
}

// bf16 codes of two values: t = bf16(fp32(y * fp32(1/s))), which equals
// bf16(fp32(y / s)) for bf16 y and s; |t| <= 7 * (1 + 2^-8) < 7.5, so no clamp
// is needed; adding 1.5 * 2^23 rounds t half-to-even to an integer held in the
// low mantissa bits, whose low nibble is the two's-complement code.
__device__ __forceinline__ void quant_pair_bf16(float2 y, float2 rcp, uint32_t& n0, uint32_t& n1) {
    const float2 t = mul2(y, rcp);
    __nv_bfloat162 b = __floats2bfloat162_rn(t.x, t.y);
    uint32_t u; memcpy(&u, &b, 4);
    const float2 tb = make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xFFFF0000u));
    const float2 r = add2(tb, make_float2(12582912.0f, 12582912.0f));
    n0 = __float_as_uint(r.x) & 0xFu;
    n1 = __float_as_uint(r.y) & 0xFu;
}

// Persistent: block b handles the row groups b, b + gridDim.x, ... of
// `rows_per_block` rows each. A group's rows are contiguous in memory and
// arrive by one bulk copy into a double-buffered shared-memory slab, issued
// two groups ahead, so HBM streams while the block computes.
// Within a group, half-warp h owns tiles h, h+16, ... (at most MAXT, MAXT
// even). A tile is 256 consecutive elements of a row seen as a 16x16 matrix
// (i = 16a + b); lane j of the half-warp takes row a = j. Tiles are processed
// in pairs so every butterfly step is one paired-fp32 instruction. Rotation:
// H16 along b in registers, a padded shared-memory transpose (lane j now
// holds column b = j), then H16 (G=256) or H4 on the low digit of a (G=64),
// scale 1/sqrt(G), round to the activation dtype. After the row absmax
// (shared atomics) the codes are formed in registers and put back in row
// order with transpose_nibbles16. G == 16 needs no transform along a and
// G == 1 (pre-rotated input) none at all: those keep lane j on row a = j.
template <typename T, int G, int MAXT>
__global__ void __launch_bounds__(kQuantThreads)
convrot_quant_kernel(const T* __restrict__ x, int8_t* __restrict__ qout, float* __restrict__ scaleout,
                     int M, int K, int rows_per_block) {
    static_assert(MAXT % 2 == 0, "tiles are processed in pairs");
    constexpr int NP = MAXT / 2;
    constexpr bool kColumnLayout = (G == 64 || G == 256);
    extern __shared__ __align__(16) unsigned char qsmem[];
    float* tr = reinterpret_cast<float*>(qsmem);                               // transpose scratch
    uint32_t* rowmax = reinterpret_cast<uint32_t*>(tr + kTransposeFloats);     // [rows_per_block]
    float* row_scale = reinterpret_cast<float*>(rowmax + rows_per_block);      // [rows_per_block]
    float* row_rcp = row_scale + rows_per_block;                                // [rows_per_block]
    uint64_t* full = reinterpret_cast<uint64_t*>(
        qsmem + ((static_cast<size_t>(kTransposeFloats + 3 * rows_per_block) * 4 + 15) & ~static_cast<size_t>(15)));
    const size_t slab_elems = static_cast<size_t>(rows_per_block) * K;
    T* slab = reinterpret_cast<T*>(reinterpret_cast<unsigned char*>(full) + 16 + 112);   // 128 B in
    // slab[0 .. slab_elems) and slab[slab_elems .. 2 * slab_elems): the two buffers

    const int tid = threadIdx.x;
    const int groups = (M + rows_per_block - 1) / rows_per_block;
    auto issue = [&](int g, int b) {
        const int r0 = g * rows_per_block;
        const int nr = min(rows_per_block, M - r0);
        const uint32_t bytes = static_cast<uint32_t>(static_cast<size_t>(nr) * K * sizeof(T));
        mbar_arrive_expect_tx(&full[b], bytes);
        bulk_load(slab + b * slab_elems, x + static_cast<size_t>(r0) * K, bytes, &full[b]);
    };
    if (tid == 0) {
        mbar_init(&full[0], 1);
        mbar_init(&full[1], 1);
        fence_mbar_init();
    }
    for (int r = tid; r < rows_per_block; r += kQuantThreads) rowmax[r] = 0u;
    __syncthreads();
    griddep_wait();                   // x may be the previous kernel's output
    griddep_launch_dependents();
    if (tid == 0) {
        if (blockIdx.x < groups) issue(blockIdx.x, 0);
        if (blockIdx.x + gridDim.x < groups) issue(blockIdx.x + gridDim.x, 1);
    }

    const int hw = tid >> 4;          // half-warp 0..15
    const int j = tid & 15;           // lane within the half-warp
    const unsigned hmask = 0xFFFFu << (16 * ((tid & 31) >> 4));
    const int ntile = (K + 255) >> 8;
    float* my_tr = tr + hw * (16 * kTrStride);

    int trow[MAXT], tkb[MAXT];
    #pragma unroll
    for (int i = 0; i < MAXT; ++i) {
        const int g = hw + 16 * i;
        trow[i] = g / ntile;
        tkb[i] = (g - trow[i] * ntile) * 256;
    }

    int it = 0;
    for (int grp = blockIdx.x; grp < groups; grp += gridDim.x, ++it) {
        const int buf = it & 1;
        const int row0 = grp * rows_per_block;
        const int nrows = min(rows_per_block, M - row0);
        const int my_tiles = max(0, (nrows * ntile - hw + 15) >> 4);   // tiles of this half-warp (<= MAXT)
        auto row_valid = [&](int i) { return i < my_tiles && 16 * j < K - tkb[i]; };
        if (!mbar_wait_bounded(&full[buf], (it >> 1) & 1)) { record_status(kStatusTimeoutExpand); break; }
        const T* src = slab + buf * slab_elems;

        // ---- this lane's rows of its tiles, from the slab
        float2 v[NP][16];
        #pragma unroll
        for (int p = 0; p < NP; ++p) {
            float a0[16], a1[16];
            #pragma unroll
            for (int e = 0; e < 16; ++e) { a0[e] = 0.0f; a1[e] = 0.0f; }
            if (row_valid(2 * p)) load16<T>(src + static_cast<size_t>(trow[2 * p]) * K + tkb[2 * p] + 16 * j, a0);
            if (row_valid(2 * p + 1))
                load16<T>(src + static_cast<size_t>(trow[2 * p + 1]) * K + tkb[2 * p + 1] + 16 * j, a1);
            #pragma unroll
            for (int e = 0; e < 16; ++e) v[p][e] = make_float2(a0[e], a1[e]);
        }
        __syncthreads();                  // slab buffer consumed: refill it two groups ahead
        if (tid == 0 && grp + 2 * static_cast<int>(gridDim.x) < groups) issue(grp + 2 * gridDim.x, buf);

        // ---- rotate and round in place, two tiles per pass; row absmax through shared atomics
        #pragma unroll
        for (int p = 0; p < NP; ++p) {
            if (2 * p >= my_tiles) break;
            if constexpr (G != 1) h16x2(v[p]);                    // along b
            if constexpr (kColumnLayout) {
                #pragma unroll
                for (int h = 0; h < 2; ++h) {
                    #pragma unroll
                    for (int b = 0; b < 16; ++b) my_tr[b * kTrStride + j] = h ? v[p][b].y : v[p][b].x;
                    __syncwarp(hmask);
                    #pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float4 c = *reinterpret_cast<const float4*>(my_tr + j * kTrStride + 4 * q);
                        if (h) { v[p][4 * q].y = c.x; v[p][4 * q + 1].y = c.y; v[p][4 * q + 2].y = c.z; v[p][4 * q + 3].y = c.w; }
                        else   { v[p][4 * q].x = c.x; v[p][4 * q + 1].x = c.y; v[p][4 * q + 2].x = c.z; v[p][4 * q + 3].x = c.w; }
                    }
                    __syncwarp(hmask);
                }
                if constexpr (G == 256) h16x2(v[p]);              // along a
                else h4_low_digit_x2(v[p]);                       // along a0 (groups of 4 rows)
            }
            float m0 = 0.0f, m1 = 0.0f;
            constexpr float kNorm = (G == 256) ? 0.0625f : (G == 64) ? 0.125f : (G == 16) ? 0.25f : 1.0f;
            #pragma unroll
            for (int e = 0; e < 16; ++e) {
                float2 sc = v[p][e];
                if constexpr (G != 1) sc = mul2(sc, make_float2(kNorm, kNorm));
                v[p][e] = make_float2(Act<T>::round(sc.x), Act<T>::round(sc.y));
                m0 = fmaxf(m0, fabsf(v[p][e].x));
                m1 = fmaxf(m1, fabsf(v[p][e].y));
            }
            #pragma unroll
            for (int off = 8; off > 0; off >>= 1) {
                m0 = fmaxf(m0, __shfl_xor_sync(hmask, m0, off));
                m1 = fmaxf(m1, __shfl_xor_sync(hmask, m1, off));
            }
            if (j == 0) {
                atomicMax(&rowmax[trow[2 * p]], __float_as_uint(m0));
                if (2 * p + 1 < my_tiles) atomicMax(&rowmax[trow[2 * p + 1]], __float_as_uint(m1));
            }
        }
        __syncthreads();

        for (int r = tid; r < nrows; r += kQuantThreads) {
            const float amax = fmaxf(__uint_as_float(rowmax[r]), Act<T>::floor_value());
            const float s = Act<T>::round(__fdiv_rn(amax, 7.0f));
            row_scale[r] = s;
            row_rcp[r] = __frcp_rn(s);
            scaleout[row0 + r] = s;
            rowmax[r] = 0u;               // ready for the next group
        }
        __syncthreads();

        // ---- codes, back in row order, 8 output bytes per lane and tile
        #pragma unroll
        for (int p = 0; p < NP; ++p) {
            if (2 * p >= my_tiles) break;
            const int r0 = trow[2 * p];
            const int r1 = (2 * p + 1 < my_tiles) ? trow[2 * p + 1] : r0;
            uint32_t lo0 = 0u, hi0 = 0u, lo1 = 0u, hi1 = 0u;
            if constexpr (Act<T>::kCode == 1) {
                const float2 rcp = make_float2(row_rcp[r0], row_rcp[r1]);
                #pragma unroll
                for (int e = 0; e < 16; ++e) {
                    uint32_t n0, n1;
                    quant_pair_bf16(v[p][e], rcp, n0, n1);
                    if (e < 8) { lo0 |= n0 << (4 * e); lo1 |= n1 << (4 * e); }
                    else       { hi0 |= n0 << (4 * (e - 8)); hi1 |= n1 << (4 * (e - 8)); }
                }
            } else {
                const float s0 = row_scale[r0], s1 = row_scale[r1];
                #pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const uint32_t n0 = quant_nibble<T>(v[p][e].x, s0), n1 = quant_nibble<T>(v[p][e].y, s1);
                    if (e < 8) { lo0 |= n0 << (4 * e); lo1 |= n1 << (4 * e); }
                    else       { hi0 |= n0 << (4 * (e - 8)); hi1 |= n1 << (4 * (e - 8)); }
                }
            }
            if constexpr (kColumnLayout) {
                transpose_nibbles16(lo0, hi0, j, hmask);
                transpose_nibbles16(lo1, hi1, j, hmask);
            }
            #pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int i = 2 * p + h;
                if (row_valid(i)) {
                    uint2* dst = reinterpret_cast<uint2*>(qout + static_cast<size_t>(row0 + trow[i]) * (K >> 1) +
                                                          (tkb[i] >> 1) + 8 * j);
                    *dst = h ? make_uint2(lo1, hi1) : make_uint2(lo0, hi0);
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// (1b) bf16 rows, G in {64, 256}, K % 256 == 0: two threads per tile
// ---------------------------------------------------------------------------
//
// A round is R whole rows (R * K/256 tiles, at most 192) brought into shared
// memory by one bulk copy, double buffered two rounds ahead. Lane l of a warp
// takes half h = l / 16 of tile t = l % 16 (of the warp's 16 tiles): rows
// a = 8h .. 8h+7 of the 16 x 16 tile, i.e. a1 in {2h, 2h+1}, all a0 and b.
// Its 128 values sit in fp32 pairs V[p][e] = {row with a1 = 2h, row with
// a1 = 2h+1} at chunk p = (a0, bh) and column e of the chunk, so the H4 steps
// along b0, b1 and a0 are paired-fp32 instructions in registers, and the step
// along a1 exchanges the pairs with lane l ^ 16 (the tile's other half).
// Shared-memory reads are conflict-free because lane t reads its chunk
// c ^ (t & 7) into slot c: the XOR relabels digits b1 (by 2) and a0, and
// H4 = J - 2R with S = (v0+v1)+(v2+v3) is unchanged under such a relabelling
// (the sums only commute), so every slot ends up holding the rotated values of
// the chunk it was loaded from; the stores undo the relabelling.
// After rounding to bf16 (kept packed), the row absmax goes through shared
// atomics (one per thread, three arrays so one barrier per round suffices).
// Codes: t = bf16(y * fl(1/s)) as in the generic path, then bf16(t + 192) is
// 192 + rint(t) exactly (unit spacing in [128, 256), ties to even), whose low
// mantissa nibble is the two's-complement code.

#ifndef CONVROT_Q5_MAX_THREADS
#define CONVROT_Q5_MAX_THREADS 384
#endif
constexpr int kQ5MaxThreads = CONVROT_Q5_MAX_THREADS;
constexpr int kQ5MaxTiles = kQ5MaxThreads / 2;           // tiles per round, at most
#ifndef CONVROT_Q5_ROUND_TILES
#define CONVROT_Q5_ROUND_TILES 48
#endif
constexpr int kQ5RoundTiles = CONVROT_Q5_ROUND_TILES;    // target tiles per round (several blocks per SM)
constexpr int kQ5RowmaxOffset = 16;
constexpr int kQ5SlabOffset = 2432;                      // 16 + 3 * 192 * 4, to 128 B
// shared memory of a block of `threads` threads: two slabs of threads / 2 tiles
constexpr int q5_smem_bytes(int threads) { return kQ5SlabOffset + 2 * (threads / 2) * 512; }

__device__ __forceinline__ uint32_t bf16x2_bits(float lo, float hi) {
    __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
    uint32_t u;
    memcpy(&u, &b, 4);
    return u;
}

// max(|a|, |b|) per bf16 half, sign bits unspecified
__device__ __forceinline__ uint32_t bf16x2_absmax(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ uint32_t bf16x2_add(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// BITS = 4: int4 codes (scale = absmax / 7), packed [M, K/2], or with UNPACKED one
// sign-extended int8 per code [M, K] (the operand form of the int8 tensor-core
// GEMM); BITS = 8: int8 codes [M, K] (scale = absmax / 127, the W8A8 tier,
// _int4/int8_eager.py:22-27).
#ifndef CONVROT_Q5_MIN_BLOCKS
#define CONVROT_Q5_MIN_BLOCKS 1
#endif
// LNMOD: the rows are first normalised and modulated as the producer of x
// before a Flux block's QKV or MLP-up projection does,
//   y = bf16(bf16(bf16(1 + scale[k]) * xn) + shift[k]),  xn = bf16((x - mean) * rstd),
// LayerNorm without affine over the row (biased variance, eps), all in fp32 in a
// fixed order: lane l of a warp sums elements l, l + 32, ... of the row (from
// the slab in shared memory), then an xor butterfly over the 32 lane sums;
// mean = sum / K; the squared deviations (x - mean)^2 (two roundings) likewise;
// rstd = 1 / sqrt(var + eps), each step rounded. y then goes through the
// rotation and the quantizer as x would; the normalised tensor never touches HBM.
struct LnModArgs {
    const __nv_bfloat16* scale;     // [K] or nullptr (scale 0)
    const __nv_bfloat16* shift;     // [K] or nullptr (shift 0)
    float eps;
};
constexpr int kQ5LnMaxK = 6144;     // the staged modulation vectors share the block's shared memory
// extra shared memory of the LNMOD form: row statistics [rows][mean, rstd] and
// the staged bf16(1 + scale) and shift vectors
constexpr int q5_lnmod_bytes(int K) { return kQ5MaxTiles * 16 + 4 * K; }

// p[0] + p[1] + ... + p[n-1] left to right (n >= 1); the loads of eight
// partials are issued before their additions.
__device__ __forceinline__ float q5_ordered_sum(const float* p, int n) {
    float acc = p[0];
    int i = 1;
    for (; i + 8 <= n; i += 8) {
        float v[8];
        #pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = p[i + j];
        #pragma unroll
        for (int j = 0; j < 8; ++j) acc = __fadd_rn(acc, v[j]);
    }
    for (; i < n; ++i) acc = __fadd_rn(acc, p[i]);
    return acc;
}

// Sum of a thread's 128 bf16 values in the slab (its 16 chunks of 8, read in
// slot order, chunk s ^ kx in slot s) -- or, with sq, of (v - mean)^2 (two
// roundings each): a binary tree over the 8 values of each chunk, then over
// slots 0..7 and 8..15 apart, then their sum. Under the XOR relabelling the
// aligned pairs, quads and octets of slots are those of the chunks, so the
// value is the one of the same tree in memory order.
__device__ __forceinline__ float q5_slab_tree_sum(const unsigned char* src, int kx, bool sq, float mean) {
    float c[16];
    #pragma unroll
    for (int s = 0; s < 16; ++s) {
        const uint4 raw = *reinterpret_cast<const uint4*>(src + 16 * (s ^ kx));
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
        float v[8];
        #pragma unroll
        for (int i = 0; i < 4; ++i) {
            v[2 * i] = __uint_as_float(w[i] << 16);
            v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        }
        if (sq) {
            #pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float d = __fsub_rn(v[e], mean);
                v[e] = __fmul_rn(d, d);
            }
        }
        c[s] = __fadd_rn(__fadd_rn(__fadd_rn(v[0], v[1]), __fadd_rn(v[2], v[3])),
                         __fadd_rn(__fadd_rn(v[4], v[5]), __fadd_rn(v[6], v[7])));
    }
    #pragma unroll
    for (int w = 8; w > 0; w >>= 1)
        #pragma unroll
        for (int s = 0; s < w; ++s) c[s] = __fadd_rn(c[2 * s], c[2 * s + 1]);
    return c[0];
}

template <int G, int BITS, bool UNPACKED = false, bool LNMOD = false>
__global__ void __launch_bounds__(kQ5MaxThreads, CONVROT_Q5_MIN_BLOCKS)
convrot_quant_bf16_kernel(const __nv_bfloat16* __restrict__ x, int8_t* __restrict__ qout,
                          float* __restrict__ scaleout, int M, int K, int rows_per_round, LnModArgs lnmod) {
    static_assert(G == 64 || G == 256, "two-digit tiles only");
    static_assert(BITS == 4 || BITS == 8, "int4 or int8 codes");
    static_assert(!UNPACKED || BITS == 4, "int8 codes are never packed");
    extern __shared__ __align__(128) unsigned char q5smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(q5smem);
    uint32_t* rowmax = reinterpret_cast<uint32_t*>(q5smem + kQ5RowmaxOffset);   // [3][kQ5MaxTiles]
    unsigned char* slab = q5smem + kQ5SlabOffset;
    const int slab_bytes = static_cast<int>(blockDim.x) * 256;   // blockDim / 2 tiles of 512 B

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int t = lane & 15, h = lane >> 4;
    const int kx = t & 7;                              // chunk relabelling of this lane
    const int tile = (tid >> 5) * 16 + t;              // tile of the round, in slab order
    const int ntile = K >> 8;
    const int my_row = tile / ntile;                   // row of the round
    const int tile_in_row = tile - my_row * ntile;
    const int rounds = (M + rows_per_round - 1) / rows_per_round;
    const size_t round_elems = static_cast<size_t>(rows_per_round) * K;

    auto issue = [&](int rd, int b) {
        const int nr = min(rows_per_round, M - rd * rows_per_round);
        const uint32_t bytes = static_cast<uint32_t>(static_cast<size_t>(nr) * K * 2);
        mbar_arrive_expect_tx(&full[b], bytes);
        bulk_load(slab + b * slab_bytes, x + static_cast<size_t>(rd) * round_elems, bytes, &full[b]);
    };
    if (tid == 0) {
        mbar_init(&full[0], 1);
        mbar_init(&full[1], 1);
        fence_mbar_init();
    }
    for (int i = tid; i < 3 * kQ5MaxTiles; i += blockDim.x) rowmax[i] = 0u;
    __syncthreads();
    griddep_wait();                                    // x may be the previous kernel's output
    griddep_launch_dependents();
    if (tid == 0) {
        if (blockIdx.x < rounds) issue(blockIdx.x, 0);
        if (blockIdx.x + gridDim.x < rounds) issue(blockIdx.x + gridDim.x, 1);
    }
    // LNMOD shared memory after the two slabs: the threads' partial sums (two
    // arrays: sums, squared deviations), bf16(1 + scale)[K], shift[K]
    float* ln_part = reinterpret_cast<float*>(slab + 2 * slab_bytes);
    float* ln_part2 = ln_part + 2 * kQ5MaxTiles;
    __nv_bfloat16* ln_s1 = reinterpret_cast<__nv_bfloat16*>(ln_part2 + 2 * kQ5MaxTiles);
    __nv_bfloat16* ln_sh = ln_s1 + K;
    if constexpr (LNMOD) {
        // eight columns per step, all loads of a thread issued before their use
        const bool vec = !(reinterpret_cast<uintptr_t>(lnmod.scale) & 15u) && !(reinterpret_cast<uintptr_t>(lnmod.shift) & 15u);
        #pragma unroll 4
        for (int c = tid; c < K / 8; c += blockDim.x) {
            uint32_t sw[4] = {0u, 0u, 0u, 0u}, hw[4] = {0u, 0u, 0u, 0u};
            if (vec) {
                if (lnmod.scale != nullptr) {
                    const uint4 v = __ldg(reinterpret_cast<const uint4*>(lnmod.scale) + c);
                    sw[0] = v.x; sw[1] = v.y; sw[2] = v.z; sw[3] = v.w;
                }
                if (lnmod.shift != nullptr) {
                    const uint4 v = __ldg(reinterpret_cast<const uint4*>(lnmod.shift) + c);
                    hw[0] = v.x; hw[1] = v.y; hw[2] = v.z; hw[3] = v.w;
                }
            } else {
                #pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t lo_s = lnmod.scale ? __bfloat16_as_ushort(lnmod.scale[8 * c + 2 * i]) : 0u;
                    const uint32_t hi_s = lnmod.scale ? __bfloat16_as_ushort(lnmod.scale[8 * c + 2 * i + 1]) : 0u;
                    const uint32_t lo_h = lnmod.shift ? __bfloat16_as_ushort(lnmod.shift[8 * c + 2 * i]) : 0u;
                    const uint32_t hi_h = lnmod.shift ? __bfloat16_as_ushort(lnmod.shift[8 * c + 2 * i + 1]) : 0u;
                    sw[i] = lo_s | (hi_s << 16);
                    hw[i] = lo_h | (hi_h << 16);
                }
            }
            uint32_t s1[4];
            #pragma unroll
            for (int i = 0; i < 4; ++i)
                s1[i] = bf16x2_bits(__fadd_rn(1.0f, __uint_as_float(sw[i] << 16)),
                                    __fadd_rn(1.0f, __uint_as_float(sw[i] & 0xFFFF0000u)));
            reinterpret_cast<uint4*>(ln_s1)[c] = make_uint4(s1[0], s1[1], s1[2], s1[3]);
            reinterpret_cast<uint4*>(ln_sh)[c] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        }
        __syncthreads();
    }

    int it = 0;
    for (int rd = blockIdx.x; rd < rounds; rd += gridDim.x, ++it) {
        const int buf = it & 1;
        const int row0 = rd * rows_per_round;
        const int nrows = min(rows_per_round, M - row0);
        const bool active = my_row < nrows;
        uint32_t* rmax = rowmax + (it % 3) * kQ5MaxTiles;
        // one thread waits for the slab; the others sleep at the block barrier
        // (no issue slots spent polling) and see the copy through it
        const bool ok = !__syncthreads_or(tid == 0 && !mbar_wait_bounded(&full[buf], (it >> 1) & 1));

        uint32_t packed[8][8];                         // rounded rotated values, bf16 pairs
        // a tile's two halves are lanes l and l ^ 16: both in or both out
        const unsigned mask = __ballot_sync(0xFFFFFFFFu, active && ok);
        float ln_mean = 0.0f, ln_rstd = 0.0f;
        if constexpr (LNMOD) {
            // row statistics: every thread reduces its own 128 values of the slab
            // (binary trees over the 8 values of a chunk and over the 16 chunks,
            // read in the lane's XOR order: a tree over aligned pairs, quads, ...
            // has the same value in either order, the sums only commute), then adds
            // its row's 2 K / 256 partials in order; the variance likewise
            const bool live = active && ok;
            const unsigned char* lsrc = slab + buf * slab_bytes + tile * 512 + h * 256;
            const int seg = 2 * tile + h;
            const int seg0 = 2 * (my_row * ntile);
            const int nseg = 2 * ntile;
            ln_part[seg] = live ? q5_slab_tree_sum(lsrc, kx, false, 0.0f) : 0.0f;
            __syncthreads();
            if (live) ln_mean = __fdiv_rn(q5_ordered_sum(ln_part + seg0, nseg), static_cast<float>(K));
            ln_part2[seg] = live ? q5_slab_tree_sum(lsrc, kx, true, ln_mean) : 0.0f;
            __syncthreads();
            if (live) {
                const float var = __fdiv_rn(q5_ordered_sum(ln_part2 + seg0, nseg), static_cast<float>(K));
                ln_rstd = __frcp_rn(__fsqrt_rn(__fadd_rn(var, lnmod.eps)));
            }
        }
        float2 V[8][8];
        if (active && ok) {
            const unsigned char* src = slab + buf * slab_bytes + tile * 512 + h * 256;
            #pragma unroll
            for (int s = 0; s < 16; ++s) {
                const uint4 raw = *reinterpret_cast<const uint4*>(src + 16 * (s ^ kx));
                uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
                if constexpr (LNMOD) {
                    // y = bf16(bf16(bf16(1 + scale) * bf16((x - mean) * rstd)) + shift);
                    // columns tile_in_row * 256 + h * 128 + 8 (s ^ kx) + 0..7
                    const int col = tile_in_row * 256 + h * 128 + 8 * (s ^ kx);
                    const uint4 s1v = *reinterpret_cast<const uint4*>(ln_s1 + col);
                    const uint4 shv = *reinterpret_cast<const uint4*>(ln_sh + col);
                    const uint32_t s1w[4] = {s1v.x, s1v.y, s1v.z, s1v.w};
                    const uint32_t shw[4] = {shv.x, shv.y, shv.z, shv.w};
                    // paired fp32 (x - mean = x + (-mean) exactly); every product goes
                    // through a bf16 rounding before any sum, so nothing can contract
                    const float2 nm = make_float2(-ln_mean, -ln_mean), rs = make_float2(ln_rstd, ln_rstd);
                    auto unpack = [](uint32_t b) {
                        return make_float2(__uint_as_float(b << 16), __uint_as_float(b & 0xFFFF0000u));
                    };
                    #pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float2 xn = fmul2_rn(fadd2_rn(unpack(w[i]), nm), rs);
                        const float2 t2 = fmul2_rn(unpack(s1w[i]), unpack(bf16x2_bits(xn.x, xn.y)));
                        const float2 y = fadd2_rn(unpack(bf16x2_bits(t2.x, t2.y)), unpack(shw[i]));
                        w[i] = bf16x2_bits(y.x, y.y);
                    }
                }
                #pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float lo = __uint_as_float(w[i] << 16), hi = __uint_as_float(w[i] & 0xFFFF0000u);
                    if (s < 8) { V[s][2 * i].x = lo; V[s][2 * i + 1].x = hi; }
                    else       { V[s - 8][2 * i].y = lo; V[s - 8][2 * i + 1].y = hi; }
                }
            }
            // along b0 (columns within a chunk)
            #pragma unroll
            for (int p = 0; p < 8; ++p) {
                h4x2(V[p][0], V[p][1], V[p][2], V[p][3]);
                h4x2(V[p][4], V[p][5], V[p][6], V[p][7]);
            }
            // along b1 = 2 bh + (e >> 2)
            #pragma unroll
            for (int p = 0; p < 8; p += 2)
                #pragma unroll
                for (int e = 0; e < 4; ++e) h4x2(V[p][e], V[p][e + 4], V[p + 1][e], V[p + 1][e + 4]);
            // along a0 (p = 2 a0 + bh)
            #pragma unroll
            for (int bh = 0; bh < 2; ++bh)
                #pragma unroll
                for (int e = 0; e < 8; ++e) h4x2(V[bh][e], V[bh + 2][e], V[bh + 4][e], V[bh + 6][e]);
            if constexpr (G == 256) {
                // along a1, with the other half of the tile (lane ^ 16). Lane h
                // holds {v_2h, v_2h+1}; the lanes swap their pair sums, so both
                // form S = (v0+v1)+(v2+v3) (sums commute), and lane h computes
                // out_{3-2h} = fma(-2, v_2h, S) and out_{2-2h} = fma(-2, v_2h+1, S)
                // from its own values: it ends up holding the rows a1 = 2h', 2h'+1
                // of the other half h' = 1 - h, which is where it stores them.
                #pragma unroll
                for (int p = 0; p < 8; ++p) {
                    #pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const float2 v = V[p][e];
                        const float own = __fadd_rn(v.x, v.y);
                        const float s = __fadd_rn(own, __shfl_xor_sync(mask, own, 16));
                        float2 o = fma2(make_float2(-2.0f, -2.0f), v, make_float2(s, s));
                        o = mul2(o, make_float2(0.0625f, 0.0625f));
                        packed[p][e] = bf16x2_bits(o.y, o.x);   // {row 2h', row 2h' + 1}
                    }
                }
            } else {
                #pragma unroll
                for (int p = 0; p < 8; ++p)
                    #pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const float2 o = mul2(V[p][e], make_float2(0.125f, 0.125f));
                        packed[p][e] = bf16x2_bits(o.x, o.y);
                    }
            }
            uint32_t m = 0u;
            #pragma unroll
            for (int p = 0; p < 8; ++p)
                #pragma unroll
                for (int e = 0; e < 8; ++e) m = bf16x2_absmax(m, packed[p][e]);
            const uint32_t amax_bits = max((m & 0x7FFFu) << 16, m & 0x7FFF0000u);
            atomicMax(&rmax[my_row], amax_bits);
        }
        if (__syncthreads_or(!ok)) { if (tid == 0) record_status(kStatusTimeoutExpand); break; }
        // the slab buffer is consumed: refill it two rounds ahead; clear the
        // row-max array of round it + 2 (last read before this barrier)
        if (tid == 0 && rd + 2 * static_cast<int>(gridDim.x) < rounds) issue(rd + 2 * gridDim.x, buf);
        for (int i = tid; i < rows_per_round; i += blockDim.x) rowmax[((it + 2) % 3) * kQ5MaxTiles + i] = 0u;

        if (active) {
            constexpr float kQMax = BITS == 4 ? 7.0f : 127.0f;
            const float amax = fmaxf(__uint_as_float(rmax[my_row]), Act<__nv_bfloat16>::floor_value());
            const float sc = Act<__nv_bfloat16>::round(__fdiv_rn(amax, kQMax));
            const float rcp = __frcp_rn(sc);
            if (h == 0 && tile_in_row == 0) scaleout[row0 + my_row] = sc;
            const float2 rcp2 = make_float2(rcp, rcp);
            const bool swap_b = kx & 1;                     // slot bh 0 holds columns 8..15
            const int hs = G == 256 ? h ^ 1 : h;            // half of the tile whose rows this lane holds
            if constexpr (BITS == 4 && !UNPACKED) {
                const uint32_t magic = 0x43404340u;        // bf16 pair {192, 192}
                uint32_t words[8][2];                       // per chunk: {a1 = 2h row, a1 = 2h+1 row}
                #pragma unroll
                for (int p = 0; p < 8; ++p) {
                    uint32_t tb[4];
                    #pragma unroll
                    for (int jj = 0; jj < 4; ++jj) {
                        uint32_t c[2];
                        #pragma unroll
                        for (int u = 0; u < 2; ++u) {
                            const uint32_t y = packed[p][2 * jj + u];
                            const float2 q = mul2(make_float2(__uint_as_float(y << 16), __uint_as_float(y & 0xFFFF0000u)), rcp2);
                            c[u] = bf16x2_add(bf16x2_bits(q.x, q.y), magic) & 0x000F000Fu;
                        }
                        tb[jj] = c[0] | (c[1] << 4);            // byte 0: row 2h pair, byte 2: row 2h+1 pair
                    }
                    const uint32_t w01 = __byte_perm(tb[0], tb[1], 0x6240);
                    const uint32_t w23 = __byte_perm(tb[2], tb[3], 0x6240);
                    words[p][0] = __byte_perm(w01, w23, 0x5410);
                    words[p][1] = __byte_perm(w01, w23, 0x7632);
                }
                int8_t* dst = qout + static_cast<size_t>(row0 + my_row) * (K >> 1) + tile_in_row * 128 + hs * 64;
                #pragma unroll
                for (int a0s = 0; a0s < 4; ++a0s) {
                    const int a0n = a0s ^ (kx >> 1);
                    #pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const uint32_t w0 = words[2 * a0s][u], w1 = words[2 * a0s + 1][u];
                        *reinterpret_cast<uint2*>(dst + (a0n + 4 * u) * 8) = swap_b ? make_uint2(w1, w0) : make_uint2(w0, w1);
                    }
                }
            } else if constexpr (BITS == 4) {
                // unpacked int4: the packed path's magic add of 192 gives bf16 bits
                // 0x4340 + q, whose low byte is 0x40 + q; subtracting 0x40 per 16-bit
                // half leaves q sign-extended in the low byte -- so the codes are those
                // of the packed path for every input -- then one int8 per column.
                const uint32_t magic = 0x43404340u;
                int8_t* dst = qout + static_cast<size_t>(row0 + my_row) * K + tile_in_row * 256 + hs * 128;
                #pragma unroll
                for (int a0s = 0; a0s < 4; ++a0s) {
                    uint32_t rw[2][4];                          // [a1 row][16 columns as 4 words], slot order
                    #pragma unroll
                    for (int bh = 0; bh < 2; ++bh) {
                        const int p = 2 * a0s + bh;
                        uint32_t pr[4];                         // columns 2jj, 2jj+1: row 2h' in bytes 0-1, row 2h'+1 in 2-3
                        #pragma unroll
                        for (int jj = 0; jj < 4; ++jj) {
                            uint32_t c[2];
                            #pragma unroll
                            for (int u = 0; u < 2; ++u) {
                                const uint32_t y = packed[p][2 * jj + u];
                                const float2 q = mul2(make_float2(__uint_as_float(y << 16), __uint_as_float(y & 0xFFFF0000u)), rcp2);
                                c[u] = bf16x2_add(bf16x2_bits(q.x, q.y), magic) - 0x00400040u;
                            }
                            pr[jj] = __byte_perm(c[0], c[1], 0x6240);
                        }
                        rw[0][2 * bh] = __byte_perm(pr[0], pr[1], 0x5410);
                        rw[1][2 * bh] = __byte_perm(pr[0], pr[1], 0x7632);
                        rw[0][2 * bh + 1] = __byte_perm(pr[2], pr[3], 0x5410);
                        rw[1][2 * bh + 1] = __byte_perm(pr[2], pr[3], 0x7632);
                    }
                    const int a0n = a0s ^ (kx >> 1);
                    #pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        *reinterpret_cast<uint4*>(dst + (a0n + 4 * u) * 16) =
                            swap_b ? make_uint4(rw[u][2], rw[u][3], rw[u][0], rw[u][1])
                                   : make_uint4(rw[u][0], rw[u][1], rw[u][2], rw[u][3]);
                    }
                }
            } else {
                // int8: t = bf16(y * fl(1/s)) as above; rint(t) by adding 1.5 * 2^23
                // in fp32 (exact for |t| < 2^22, ties to even), whose low bits hold
                // the integer; clamp to +-127; one int8 per column, rows in order.
                constexpr int kQI = 127;
                int8_t* dst = qout + static_cast<size_t>(row0 + my_row) * K + tile_in_row * 256 + hs * 128;
                #pragma unroll
                for (int a0s = 0; a0s < 4; ++a0s) {
                    uint32_t rw[2][4];                          // [a1 row][16 columns as 4 words], slot order
                    #pragma unroll
                    for (int bh = 0; bh < 2; ++bh) {
                        const int p = 2 * a0s + bh;
                        int cv[2][8];
                        #pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const uint32_t y = packed[p][e];
                            const float2 q = mul2(make_float2(__uint_as_float(y << 16), __uint_as_float(y & 0xFFFF0000u)), rcp2);
                            const uint32_t tb = bf16x2_bits(q.x, q.y);
                            const float2 r = add2(make_float2(__uint_as_float(tb << 16), __uint_as_float(tb & 0xFFFF0000u)),
                                                  make_float2(12582912.0f, 12582912.0f));
                            cv[0][e] = min(kQI, max(-kQI, static_cast<int>(__float_as_uint(r.x) - 0x4B400000u)));
                            cv[1][e] = min(kQI, max(-kQI, static_cast<int>(__float_as_uint(r.y) - 0x4B400000u)));
                        }
                        #pragma unroll
                        for (int u = 0; u < 2; ++u) {
                            rw[u][2 * bh] = __byte_perm(__byte_perm(cv[u][0], cv[u][1], 0x0040),
                                                        __byte_perm(cv[u][2], cv[u][3], 0x0040), 0x5410);
                            rw[u][2 * bh + 1] = __byte_perm(__byte_perm(cv[u][4], cv[u][5], 0x0040),
                                                            __byte_perm(cv[u][6], cv[u][7], 0x0040), 0x5410);
                        }
                    }
                    const int a0n = a0s ^ (kx >> 1);
                    #pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        *reinterpret_cast<uint4*>(dst + (a0n + 4 * u) * 16) =
                            swap_b ? make_uint4(rw[u][2], rw[u][3], rw[u][0], rw[u][1])
                                   : make_uint4(rw[u][0], rw[u][1], rw[u][2], rw[u][3]);
                    }
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// (1c) packed int4 -> one sign-extended int8 per code (column order kept)
// ---------------------------------------------------------------------------
// The operand form of the int8 tensor-core GEMM: with both operands unpacked,
// sum_k x_k w_k is the int8 product over the same K, so the int4 layer runs on
// the int8 pipeline with the exact same accumulators. HBM bound, run once per
// weight tensor.
__global__ void __launch_bounds__(256)
int4_unpack_kernel(const uint4* __restrict__ packed, uint4* __restrict__ codes, size_t n16) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n16;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const uint4 v = packed[i];
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t o[8];
        #pragma unroll
        for (int e = 0; e < 4; ++e) {
            // nibble n in [0, 15] -> n - 16 * (n >= 8): per byte (n ^ 8) - 8
            const uint32_t lo = __vsub4((w[e] & 0x0F0F0F0Fu) ^ 0x08080808u, 0x08080808u);
            const uint32_t hi = __vsub4(((w[e] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u, 0x08080808u);
            o[2 * e] = __byte_perm(lo, hi, 0x5140);        // column 2j, 2j+1 of bytes 0, 1
            o[2 * e + 1] = __byte_perm(lo, hi, 0x7362);    // of bytes 2, 3
        }
        codes[2 * i] = make_uint4(o[0], o[1], o[2], o[3]);
        codes[2 * i + 1] = make_uint4(o[4], o[5], o[6], o[7]);
    }
}

// Output forms of the GEMM kernels: fp32, bf16, fp32 accumulate into `out`
// (split-K export), raw int32 accumulators.
enum : int { kOutF32 = 0, kOutBF16 = 1, kOutF32Accumulate = 2, kOutS32 = 3 };


}  // namespace convrot

#include "gemm_pair.cuh"
#include "gemm_a8t.cuh"
#include "lora_down.cuh"

namespace convrot {

// ===========================================================================
// (3) Few-token GEMV on CUDA cores (M <= 4): weight streaming at HBM rate
// ===========================================================================
//
// For a handful of tokens the product is bound by reading the packed weights
// once. One block per SM owns a contiguous range of weight rows. A producer
// lane streams them through a ring of shared-memory stages; a stage holds one
// K slice of 2 * RW consecutive rows -- one bulk copy when a row is a single
// slice (rows are contiguous), else one copy per row. RW (rows per warp) is 4,
// 2 or 1 as rows get longer, so that a stage stays near 12-16 KB: the 2 * RW
// rows of a stage belong to a pair of consumer warps, RW rows each, 32 / RW
// lanes per row. A warp keeps its int32 accumulators across the slices of its
// rows and reduces over each row's lanes with log2(32 / RW) shuffles.
// Each warp pair owns its own ring slots, so the slot a pair waits on was last
// filled for (and consumed by) that same pair: an mbarrier parity wait never
// has to tell phase k - 1 from phase k + 1. Row groups go to the pairs round
// robin and the producer fills slice j of every pair's group before slice
// j + 1, which is the order the pairs consume them in. The producer starts
// streaming before the activations are staged.
// A packed word is split like in the tensor-core path -- (w & 0xF0F0F0F0) and
// ((w << 4) & 0xF0F0F0F0) hold 16 * code as int8 -- and __dp4a of matching
// halves accumulates 256 * sum(x * w) exactly in int32; the activation halves
// are split once into shared memory. The epilogue is the GEMM's:
// ((float(D) * xs[m]) * ws[n]) + bias[n], one rounding.

constexpr int kGemvConsumers = 16;                         // consumer warps
constexpr int kGemvThreads = (kGemvConsumers + 1) * 32;   // + one producer warp
constexpr int kGemvIters = 16;                             // 16-byte steps per lane per slice
// packed bytes of one row per stage with RW rows per warp (32 / RW lanes per row)
__host__ __device__ constexpr int gemv_slice_max(int rw) { return kGemvIters * 16 * (32 / rw); }
constexpr int kGemvMaxStages = 64;
constexpr int kGemvBarrierBytes = 2 * kGemvMaxStages * 8;
constexpr int kGemvSmemBytes = 227 * 1024;

template <int MT, int RW, int OUT>
__global__ void __launch_bounds__(kGemvThreads, 1)
int4_gemv_kernel(const uint8_t* __restrict__ Xp, const uint8_t* __restrict__ Wp,
                 const float* __restrict__ xscale, const float* __restrict__ wscale,
                 BiasRef bias, void* __restrict__ out, int M, int N, int K,
                 int slice, int nslices, int pairs, int slots_per_pair, int ring_off, int rows_per_block) {
    constexpr int kLanes = 32 / RW;                           // lanes per row
    constexpr int kStageRows = 2 * RW;                        // a stage feeds two warps
    extern __shared__ __align__(128) unsigned char gv_smem[];
    const int kb = K >> 1;                                    // packed bytes per row
    const int chunks = kb >> 4;                               // 16-byte chunks per row
    const int stage_bytes = kStageRows * slice;
    const int stages = pairs * slots_per_pair;
    uint64_t* full = reinterpret_cast<uint64_t*>(gv_smem);
    uint64_t* empty = full + stages;
    uint4* xs_sh = reinterpret_cast<uint4*>(gv_smem + kGemvBarrierBytes);   // [MT][high, low][chunks]
    unsigned char* ring = gv_smem + ring_off;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row_begin = blockIdx.x * rows_per_block;
    const int row_end = min(N, row_begin + rows_per_block);
    const int groups = (row_end - row_begin + kStageRows - 1) / kStageRows;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 2);
        }
        fence_mbar_init();
    }
    if (warp == kGemvConsumers && lane == 0 && row_begin < row_end) {
        // the block's first weight bytes into L2 while the previous kernel may
        // still run (a hint: safe whatever it wrote)
        const size_t span = static_cast<size_t>(row_end - row_begin) * kb;
        const uint32_t bytes = static_cast<uint32_t>(min(span, static_cast<size_t>(stages) * stage_bytes));
        bulk_prefetch_l2(Wp + static_cast<size_t>(row_begin) * kb, bytes);
    }
    __syncthreads();
    griddep_wait();                   // activations, scales and bias may be the previous kernel's output
    griddep_launch_dependents();

    if (warp == kGemvConsumers) {
        if (lane == 0) {
            // ---------------- producer: round r gives row group r * pairs + q to
            // pair q; within a round, slice j of every group before slice j + 1
            int k = 0;                                        // slot index within each pair's slots
            uint32_t ph = 0;
            for (int r0g = 0; r0g < groups; r0g += pairs) {
                const int in_round = min(pairs, groups - r0g);
                for (int j = 0; j < nslices; ++j) {
                    const int off = j * slice;
                    const int len = min(slice, kb - off);
                    for (int q = 0; q < in_round; ++q) {
                        const int s = q * slots_per_pair + k;
                        if (!mbar_wait_bounded(&empty[s], ph ^ 1)) { record_status(kStatusTimeoutProducer); return; }
                        const int r0 = row_begin + (r0g + q) * kStageRows;
                        const int nr = min(kStageRows, row_end - r0);
                        unsigned char* dst = ring + static_cast<size_t>(s) * stage_bytes;
                        const uint8_t* src = Wp + static_cast<size_t>(r0) * kb + off;
                        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(nr * len));
                        if (nslices == 1) {
                            bulk_load(dst, src, static_cast<uint32_t>(nr * len), &full[s]);
                        } else {
                            for (int r = 0; r < nr; ++r)
                                bulk_load(dst + r * slice, src + static_cast<size_t>(r) * kb,
                                          static_cast<uint32_t>(len), &full[s]);
                        }
                    }
                    if (++k == slots_per_pair) { k = 0; ph ^= 1u; }
                }
            }
        }
        return;
    }

    // ---------------- consumers
    for (int i = threadIdx.x; i < MT * chunks; i += kGemvConsumers * 32) {
        const int m = i / chunks, c = i - m * chunks;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (m < M) v = __ldg(reinterpret_cast<const uint4*>(Xp + static_cast<size_t>(m) * kb) + c);
        xs_sh[(2 * m) * chunks + c] = make_uint4(v.x & 0xF0F0F0F0u, v.y & 0xF0F0F0F0u,
                                                 v.z & 0xF0F0F0F0u, v.w & 0xF0F0F0F0u);
        xs_sh[(2 * m + 1) * chunks + c] = make_uint4((v.x << 4) & 0xF0F0F0F0u, (v.y << 4) & 0xF0F0F0F0u,
                                                     (v.z << 4) & 0xF0F0F0F0u, (v.w << 4) & 0xF0F0F0F0u);
    }
    named_barrier_sync(1, kGemvConsumers * 32);

    // warp w takes rows [RW (w & 1), RW (w & 1) + RW) of row groups q, q + pairs, ... (q = w / 2)
    const int q = warp >> 1;
    if (q >= pairs) return;
    const int kp = lane % kLanes;                             // lane within the row's lanes
    const int row_in_stage = (warp & 1) * RW + lane / kLanes;
    const float xsv = (OUT != kOutS32 && kp < MT && kp < M) ? xscale[kp] : 0.0f;
    int k = 0;
    uint32_t ph = 0;
    for (int g = q; g < groups; g += pairs) {
        const int n = row_begin + g * kStageRows + row_in_stage;
        const bool live = n < row_end;
        const bool writer = live && kp < MT && kp < M;        // lane kp writes token kp of its row
        const size_t o = static_cast<size_t>(kp) * N + n;
        // epilogue factors are requested before the stage waits, so their
        // latency overlaps the weight copy
        float wsv = 0.0f, addend = 0.0f;
        if constexpr (OUT != kOutS32) {
            if (live) {
                wsv = wscale[n];
                if constexpr (OUT == kOutF32Accumulate) {
                    if (writer) addend = reinterpret_cast<const float*>(out)[o];
                } else {
                    if (bias.ptr != nullptr) addend = bias.at(n);
                }
            }
        }
        int acc4[MT][4];                                      // four independent dp4a chains per token
        #pragma unroll
        for (int m = 0; m < MT; ++m)
            #pragma unroll
            for (int e = 0; e < 4; ++e) acc4[m][e] = 0;
        bool ok = true;
        for (int j = 0, off = 0; j < nslices; ++j, off += slice) {
            const int s = q * slots_per_pair + k;
            if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(&full[s], ph))) {
                if (lane == 0) record_status(kStatusTimeoutExpand);
                ok = false;
                break;
            }
            if (live) {
                const int nc = min(slice, kb - off) >> 4;
                const uint4* wrow = reinterpret_cast<const uint4*>(ring + static_cast<size_t>(s) * stage_bytes +
                                                                   static_cast<size_t>(row_in_stage) * slice) + kp;
                const uint4* xrow = xs_sh + (off >> 4) + kp;
                #pragma unroll
                for (int i = 0; i < kGemvIters; ++i) {
                    if (kLanes * i < nc) {                    // uniform per row; ragged lanes read zero weights
                        uint4 wv = make_uint4(0u, 0u, 0u, 0u);
                        if (kp + kLanes * i < nc) wv = wrow[kLanes * i];
                        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
                        int wh[4], wl[4];
                        #pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            wh[e] = static_cast<int>(ww[e] & 0xF0F0F0F0u);
                            wl[e] = static_cast<int>((ww[e] << 4) & 0xF0F0F0F0u);
                        }
                        #pragma unroll
                        for (int m = 0; m < MT; ++m) {
                            const uint4 xh = xrow[(2 * m) * chunks + kLanes * i];
                            const uint4 xl = xrow[(2 * m + 1) * chunks + kLanes * i];
                            const int xhw[4] = {static_cast<int>(xh.x), static_cast<int>(xh.y),
                                                static_cast<int>(xh.z), static_cast<int>(xh.w)};
                            const int xlw[4] = {static_cast<int>(xl.x), static_cast<int>(xl.y),
                                                static_cast<int>(xl.z), static_cast<int>(xl.w)};
                            #pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                acc4[m][e] = __dp4a(wh[e], xhw[e], acc4[m][e]);
                                acc4[m][e] = __dp4a(wl[e], xlw[e], acc4[m][e]);
                            }
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);            // this warp's rows of the slice are read
            if (++k == slots_per_pair) { k = 0; ph ^= 1u; }
        }
        if (!ok) break;
        int d = 0;
        #pragma unroll
        for (int m = 0; m < MT; ++m) {
            int a = (acc4[m][0] + acc4[m][1]) + (acc4[m][2] + acc4[m][3]);
            #pragma unroll
            for (int sh = 1; sh < kLanes; sh <<= 1) a += __shfl_xor_sync(0xFFFFFFFFu, a, sh);
            if (m == kp) d = a >> 8;
        }
        if (writer) {
            if constexpr (OUT == kOutS32) {
                reinterpret_cast<int32_t*>(out)[o] = d;
            } else {
                const float v = __fmul_rn(__fmul_rn(static_cast<float>(d), xsv), wsv);
                const float y = __fadd_rn(addend, v);
                if constexpr (OUT == kOutBF16) reinterpret_cast<__nv_bfloat16*>(out)[o] = __float2bfloat16_rn(y);
                else reinterpret_cast<float*>(out)[o] = y;
            }
        }
    }
}

// ===========================================================================
// Host side
// ===========================================================================

thread_local char g_last_error[256] = "";

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 2) return 148;
    return n;
}


// Launch with programmatic stream serialization: the kernel may start its
// prologue while the previous kernel in the stream drains; every kernel of this
// library calls griddep_wait() before touching memory another kernel wrote.
template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...);
}

int fail(const char* msg) {
    snprintf(g_last_error, sizeof(g_last_error), "%s", msg);
    return -1;
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// Packed int4 matrix [rows, K/2] bytes, box [box_rows, 128 B], 128-byte swizzle.
bool make_packed_tmap(CUtensorMap* map, const void* base, int rows, int K, int box_rows) {
    constexpr int box_bytes = kPairBKP;
    auto enc = get_encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K / 2), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K / 2)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_bytes), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <typename KernelT>
cudaError_t ensure_smem(KernelT kernel, int bytes) {
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

// bf16 output [M, N] for TMA stores of 128-row x 64-column boxes (128 B swizzle).
bool make_out_tmap(CUtensorMap* map, void* out, int M, int N) {
    auto enc = get_encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(N) * 2};
    const cuuint32_t box[2] = {64, 128};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, out, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// fp16 matrix [rows, cols] (row-major) read in boxes of 64 columns x box_rows, 128 B swizzle.
bool make_f16_tmap(CUtensorMap* map, const void* base, int rows, int cols, int box_rows) {
    auto enc = get_encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
    const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct LoraArgs {
    const void* t = nullptr;      // fp16 [M, rank]
    const void* b = nullptr;      // fp16 [N, rank]
    int rank = 0;
    float scale = 0.0f;
};

template <int BN, bool SWAP, int OUT, bool STAGED, bool LORA, bool I8 = false, bool A8 = false>
int launch_pair_impl(const void* Xp, const void* Wp, const float* xs, const float* ws, BiasRef bias,
                     void* out, int M, int N, int K, const LoraArgs& lora, cudaStream_t stream,
                     const PeerOut& peers = PeerOut{}) {
    using Cfg = PairCfg<BN, STAGED, SWAP, LORA, I8, A8>;
    const void* a_ptr = SWAP ? Wp : Xp;
    const void* b_ptr = SWAP ? Xp : Wp;
    const int rows_a = SWAP ? N : M;
    const int rows_b = SWAP ? M : N;
    CUtensorMap ta, tb, to, tlt, tlb;
    memset(&to, 0, sizeof(to));
    memset(&tlt, 0, sizeof(tlt));
    memset(&tlb, 0, sizeof(tlb));
    // (the packed-int4 map of 2K codes is the int8 map of K values: K bytes a row)
    // (A8: int8 activation codes, K bytes a row; the expanders read the packed
    // weights through plain loads, so they need no map)
    const int kcodes = I8 ? 2 * K : K;
    if (A8) memset(&tb, 0, sizeof(tb));
    const bool maps_ok = A8 ? make_packed_tmap(&ta, a_ptr, rows_a, 2 * K, 128)
                            : make_packed_tmap(&ta, a_ptr, rows_a, kcodes, 128) &&
                                  make_packed_tmap(&tb, b_ptr, rows_b, kcodes, BN / 2);
    if (!maps_ok)
        return fail("cuTensorMapEncodeTiled failed (pointer not 16-byte aligned or driver entry point missing)");
    if (STAGED && !make_out_tmap(&to, out, M, N))
        return fail("cuTensorMapEncodeTiled failed for the output");
    if (LORA && (!make_f16_tmap(&tlt, lora.t, M, lora.rank, 128) ||
                 !make_f16_tmap(&tlb, lora.b, N, lora.rank, BN / 2)))
        return fail("cuTensorMapEncodeTiled failed for the LoRA operands");
    auto kernel = int4_gemm_pair_kernel<BN, SWAP, OUT, STAGED, LORA, I8, A8>;
    cudaError_t e = ensure_smem(kernel, Cfg::kSmemBytes);
    if (e != cudaSuccess) return static_cast<int>(e);
    const int tiles_a = (rows_a + 255) / 256;
    const int tiles_b = (rows_b + BN - 1) / BN;
    const long num_tiles = static_cast<long>(tiles_a) * tiles_b;
    if (num_tiles > 0x7FFFFFFF) return fail("too many output tiles");
    const int clusters = static_cast<int>(num_tiles < sm_count() / 2 ? num_tiles : sm_count() / 2);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * clusters, 1, 1);
    cfg.blockDim = dim3(kPairThreads, 1, 1);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    e = cudaLaunchKernelEx(&cfg, kernel, ta, tb, to, tlt, tlb, xs, ws, bias, out, M, N, K, tiles_a,
                           static_cast<int>(num_tiles), lora.scale, b_ptr, peers);
    if (e != cudaSuccess) return static_cast<int>(e);
    return static_cast<int>(cudaGetLastError());
}

template <int BN, bool SWAP, int OUT, bool LORA = false>
int launch_pair(const void* Xp, const void* Wp, const float* xs, const float* ws, BiasRef bias,
                void* out, int M, int N, int K, cudaStream_t stream, const LoraArgs& lora = LoraArgs()) {
    if constexpr (OUT == kOutBF16 && !SWAP) {
        // The staged bf16 tile (64 KB at BN = 256) costs the k-stage ring one
        // slot (3 instead of 4). Short rows drain a tile every few stages and
        // gain more from TMA stores; long rows (24+ stages per tile) gain more
        // from the deeper ring.
        const bool long_rows = BN == 256 && K >= 6144;
        if ((N % 8) == 0 && aligned16(out) && !long_rows)
            return launch_pair_impl<BN, SWAP, OUT, true, LORA>(Xp, Wp, xs, ws, bias, out, M, N, K, lora, stream);
    }
    return launch_pair_impl<BN, SWAP, OUT, false, LORA>(Xp, Wp, xs, ws, bias, out, M, N, K, lora, stream);
}

struct GemvPlan {
    int rw, slice, nslices, pairs, slots_per_pair, ring_off;
    size_t smem;
    bool ok;
};

// Shared-memory plan of the few-token path for K: rows per warp by row length
// (a stage of 2 * RW rows stays within 16 KB), split activation halves, then as
// many ring stages as fit, shared out among up to eight consumer warp pairs
// with at least two slots per pair.
template <int MT>
GemvPlan gemv_plan(int K) {
    GemvPlan p{};
    const int kb = K / 2;
    p.rw = kb <= gemv_slice_max(4) ? 4 : kb <= gemv_slice_max(2) ? 2 : 1;
    const int smax = gemv_slice_max(p.rw);
    p.nslices = (kb + smax - 1) / smax;
    p.slice = ((kb + p.nslices - 1) / p.nslices + 15) & ~15;
    // 512 spare bytes after the activations: ragged lanes of the last step
    // read up to 31 chunks past the end of a token's codes
    p.ring_off = (kGemvBarrierBytes + MT * 2 * kb + 512 + 127) & ~127;
    const int stage_bytes = 2 * p.rw * p.slice;
    int stages = (kGemvSmemBytes - p.ring_off) / stage_bytes;
    if (stages > kGemvMaxStages) stages = kGemvMaxStages;
    // every consumer pair double-buffers at least: as many pairs as that allows
    p.pairs = stages / 2 < kGemvConsumers / 2 ? stages / 2 : kGemvConsumers / 2;
    p.slots_per_pair = p.pairs > 0 ? stages / p.pairs : 0;
    p.ok = p.pairs >= 1;
    p.smem = static_cast<size_t>(p.ring_off) + static_cast<size_t>(p.ok ? p.pairs * p.slots_per_pair : 0) * stage_bytes;
    return p;
}

template <int MT, int RW, int OUT>
int launch_gemv_rw(const void* Xp, const void* Wp, const float* xs, const float* ws, BiasRef bias,
                   void* out, int M, int N, int K, const GemvPlan& p, cudaStream_t stream) {
    auto kernel = int4_gemv_kernel<MT, RW, OUT>;
    cudaError_t e = ensure_smem(kernel, static_cast<int>(p.smem));
    if (e != cudaSuccess) return static_cast<int>(e);
    // contiguous row ranges of equal length, one block per SM
    int blocks = sm_count();
    const int rows_per_block = (N + blocks - 1) / blocks;
    blocks = (N + rows_per_block - 1) / rows_per_block;
    e = launch_pdl(kernel, dim3(blocks), dim3(kGemvThreads), p.smem, stream, static_cast<const uint8_t*>(Xp),
                   static_cast<const uint8_t*>(Wp), xs, ws, bias, out, M, N, K, p.slice, p.nslices, p.pairs,
                   p.slots_per_pair, p.ring_off, rows_per_block);
    return static_cast<int>(e);
}

template <int MT, int OUT>
int launch_gemv(const void* Xp, const void* Wp, const float* xs, const float* ws, BiasRef bias,
                void* out, int M, int N, int K, cudaStream_t stream) {
    const GemvPlan p = gemv_plan<MT>(K);
    if (!p.ok) return fail("K too large for the few-token path");
    if ((reinterpret_cast<uintptr_t>(Wp) & 15u) || (reinterpret_cast<uintptr_t>(Xp) & 15u))
        return fail("packed operands must be 16-byte aligned");
    if (p.rw == 4) return launch_gemv_rw<MT, 4, OUT>(Xp, Wp, xs, ws, bias, out, M, N, K, p, stream);
    if (p.rw == 2) return launch_gemv_rw<MT, 2, OUT>(Xp, Wp, xs, ws, bias, out, M, N, K, p, stream);
    return launch_gemv_rw<MT, 1, OUT>(Xp, Wp, xs, ws, bias, out, M, N, K, p, stream);
}

template <int OUT>
int dispatch_gemm(const void* Xp, const void* Wp, const float* xs, const float* ws, BiasRef bias,
                  void* out, int M, int N, int K, cudaStream_t stream) {
    // a few tokens: stream the weights on CUDA cores
    if (M == 1 && gemv_plan<1>(K).ok) return launch_gemv<1, OUT>(Xp, Wp, xs, ws, bias, out, M, N, K, stream);
    if (M <= 2 && gemv_plan<2>(K).ok) return launch_gemv<2, OUT>(Xp, Wp, xs, ws, bias, out, M, N, K, stream);
    if (M <= 4 && gemv_plan<4>(K).ok) return launch_gemv<4, OUT>(Xp, Wp, xs, ws, bias, out, M, N, K, stream);
    if (M <= 32) return launch_pair<32, true, OUT>(Xp, Wp, xs, ws, bias, out, M, N, K, stream);
    if (M <= 64) return launch_pair<64, true, OUT>(Xp, Wp, xs, ws, bias, out, M, N, K, stream);
    if (M <= 128) return launch_pair<128, true, OUT>(Xp, Wp, xs, ws, bias, out, M, N, K, stream);
    // 256x256 pair tiles unless that leaves more than half of the CTA pairs idle
    const long tiles256 = static_cast<long>((M + 255) / 256) * ((N + 255) / 256);
    if (2 * tiles256 < sm_count() / 2)
        return launch_pair<128, false, OUT>(Xp, Wp, xs, ws, bias, out, M, N, K, stream);
    return launch_pair<256, false, OUT>(Xp, Wp, xs, ws, bias, out, M, N, K, stream);
}

// W8A8 tier: int8 X [M, K] and W [N, K] on CTA pairs (no swapped or few-token
// forms: small M pays for a partly empty 256-row tile).
template <int OUT>
int dispatch_gemm_i8(const void* X, const void* W, const float* xs, const float* ws, BiasRef bias,
                     void* out, int M, int N, int K, cudaStream_t stream) {
    const long tiles256 = static_cast<long>((M + 255) / 256) * ((N + 255) / 256);
    if (2 * tiles256 < sm_count() / 2)
        return launch_pair_impl<128, false, OUT, false, false, true>(X, W, xs, ws, bias, out, M, N, K, LoraArgs(), stream);
    if constexpr (OUT == kOutBF16) {
        if ((N % 8) == 0 && aligned16(out) && K < 3072)    // under 24 stages a tile: staged stores
            return launch_pair_impl<256, false, OUT, true, false, true>(X, W, xs, ws, bias, out, M, N, K, LoraArgs(), stream);
    }
    return launch_pair_impl<256, false, OUT, false, false, true>(X, W, xs, ws, bias, out, M, N, K, LoraArgs(), stream);
}

// Packed int4 weights [rows, K/2] in boxes of 128 rows x 64 bytes (128 codes), 64-byte swizzle.
bool make_w64_tmap(CUtensorMap* map, const void* base, int rows, int K) {
    auto enc = get_encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K / 2), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K / 2)};
    const cuuint32_t box[2] = {64, 128};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// bf16 output [M, N] for TMA stores of 32-token x 32-column boxes (64 B rows, 64 B swizzle).
bool make_out_box32_tmap(CUtensorMap* map, void* out, int M, int N) {
    auto enc = get_encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(N) * 2};
    const cuuint32_t box[2] = {32, 32};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, out, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
               CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The A8T form (weights as the TMEM operand): 256 weight rows x BN tokens per CTA pair.
template <int BN, int OUT, bool STAGED>
int launch_a8t_impl(const void* X8, const void* Wp, const float* xs, const float* ws, BiasRef bias, void* out,
                    int M, int N, int K, cudaStream_t stream) {
    using Cfg = A8tCfg<BN, STAGED>;
    CUtensorMap tx, tw, to;
    memset(&to, 0, sizeof(to));
    if (!make_packed_tmap(&tx, X8, M, 2 * K, BN / 2) || !make_w64_tmap(&tw, Wp, N, K))
        return fail("cuTensorMapEncodeTiled failed (pointer not 16-byte aligned or driver entry point missing)");
    if (STAGED && !make_out_box32_tmap(&to, out, M, N)) return fail("cuTensorMapEncodeTiled failed for the output");
    auto kernel = int4_gemm_a8t_kernel<BN, OUT, STAGED>;
    cudaError_t e = ensure_smem(kernel, Cfg::kSmemBytes);
    if (e != cudaSuccess) return static_cast<int>(e);
    const int tiles_w = (N + 255) / 256;
    const long num_tiles = static_cast<long>(tiles_w) * ((M + BN - 1) / BN);
    if (num_tiles > 0x7FFFFFFF) return fail("too many output tiles");
    const int clusters = static_cast<int>(num_tiles < sm_count() / 2 ? num_tiles : sm_count() / 2);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * clusters, 1, 1);
    cfg.blockDim = dim3(kPairThreads, 1, 1);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    e = cudaLaunchKernelEx(&cfg, kernel, tx, tw, to, xs, ws, bias, out, M, N, K, tiles_w,
                           static_cast<int>(num_tiles), Wp);
    if (e != cudaSuccess) return static_cast<int>(e);
    return static_cast<int>(cudaGetLastError());
}

template <int BN, int OUT>
int launch_a8t(const void* X8, const void* Wp, const float* xs, const float* ws, BiasRef bias, void* out,
               int M, int N, int K, cudaStream_t stream) {
    if constexpr (OUT == kOutBF16) {
        if (N % 8 == 0 && aligned16(out))
            return launch_a8t_impl<BN, OUT, true>(X8, Wp, xs, ws, bias, out, M, N, K, stream);
    }
    return launch_a8t_impl<BN, OUT, false>(X8, Wp, xs, ws, bias, out, M, N, K, stream);
}

#ifndef CONVROT_A8T_BN
#define CONVROT_A8T_BN 256
#endif

// int4 layers on int8 activation codes and packed weights (the A8 form): 256 x 256
// pair tiles, or 256 x 128 when 256-column tiles leave most CTA pairs idle; with
// a LoRA side path the same rule (256-column LoRA tiles hold one accumulator pair).
template <int OUT>
int dispatch_gemm_a8(const void* X8, const void* Wp, const float* xs, const float* ws, BiasRef bias,
                     void* out, int M, int N, int K, const LoraArgs& lora, cudaStream_t stream) {
    const long tiles256 = static_cast<long>((M + 255) / 256) * ((N + 255) / 256);
    if (lora.rank > 0) {
        if (2 * tiles256 >= sm_count())
            return launch_pair_impl<256, false, OUT, false, true, false, true>(X8, Wp, xs, ws, bias, out, M, N, K,
                                                                               lora, stream);
        return launch_pair_impl<128, false, OUT, false, true, false, true>(X8, Wp, xs, ws, bias, out, M, N, K,
                                                                           lora, stream);
    }
    if (CONVROT_A8T_BN > 0) {
        const long tiles_t = static_cast<long>((N + 255) / 256) * ((M + CONVROT_A8T_BN - 1) / CONVROT_A8T_BN);
        if (2 * tiles_t >= sm_count()) {
            // wave quantization: the share of CTA-pair slots the tiles fill; 192-token
            // tiles when they fill the last wave much better (e.g. 2304 x 3072: 108
            // tiles of 256 for 74 pairs fill 73 %, 144 tiles of 192 fill 97 %)
            const long pairs = sm_count() / 2;
            const long tiles_192 = static_cast<long>((N + 255) / 256) * ((M + 191) / 192);
            auto fill = [&](long t) { return static_cast<double>(t) / static_cast<double>(((t + pairs - 1) / pairs) * pairs); };
            if (CONVROT_A8T_BN == 256 && fill(tiles_192) >= fill(tiles_t) + 0.15)
                return launch_a8t<192, OUT>(X8, Wp, xs, ws, bias, out, M, N, K, stream);
            return launch_a8t<(CONVROT_A8T_BN > 0 ? CONVROT_A8T_BN : 192), OUT>(X8, Wp, xs, ws, bias, out, M, N, K,
                                                                               stream);
        }
    }
    if (2 * tiles256 >= sm_count() / 2)
        return launch_pair_impl<256, false, OUT, false, false, false, true>(X8, Wp, xs, ws, bias, out, M, N, K,
                                                                            lora, stream);
    return launch_pair_impl<128, false, OUT, false, false, false, true>(X8, Wp, xs, ws, bias, out, M, N, K,
                                                                        lora, stream);
}

int check_gemm_args(const void* Xp, const void* Wp, int M, int N, int K) {
    if (M < 0 || N < 0 || K <= 0) return fail("M, N must be >= 0 and K > 0");
    if (K % 32 != 0) return fail("K must be a multiple of 32");
    if (K > 65536) return fail("K must be <= 65536 (int32 accumulator headroom)");
    if (M > 0 && N > 0 && (!Xp || !Wp)) return fail("null operand pointer");
    if (!aligned16(Xp) || !aligned16(Wp)) return fail("packed operands must be 16-byte aligned");
    return 0;
}

template <typename T, int G>
int launch_quant_t(const void* x, void* q, void* s, int M, int K, cudaStream_t stream) {
    const int ntile = (K + 255) / 256;
    // at most MAXT tiles per half-warp: 16 half-warps x MAXT tiles per row group
    const bool big = ntile > 64;
    const int maxt = big ? 16 : 4;
    int rows = (16 * maxt) / ntile;
    rows = rows < 1 ? 1 : rows;
    if (rows > M) rows = M;
    if (static_cast<long>(rows) * ntile > 16L * maxt) return fail("row too long for the quantizer");
    const size_t head = ((static_cast<size_t>(kTransposeFloats) + 3 * rows) * 4 + 15) & ~static_cast<size_t>(15);
    const size_t bytes = head + 128 + 2 * static_cast<size_t>(rows) * K * sizeof(T);
    if (bytes > 227 * 1024) return fail("row too long for the quantizer's shared-memory slabs");
    auto kernel = big ? convrot_quant_kernel<T, G, 16> : convrot_quant_kernel<T, G, 4>;
    cudaError_t e = ensure_smem(kernel, static_cast<int>(bytes));
    if (e != cudaSuccess) return static_cast<int>(e);
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kQuantThreads, bytes);
    if (e != cudaSuccess) return static_cast<int>(e);
    const int groups = (M + rows - 1) / rows;
    const int resident = sm_count() * (per_sm > 0 ? per_sm : 1);
    const int grid = groups < resident ? groups : resident;
    e = launch_pdl(kernel, dim3(grid), dim3(kQuantThreads), bytes, stream, static_cast<const T*>(x),
                   static_cast<int8_t*>(q), static_cast<float*>(s), M, K, rows);
    return static_cast<int>(e);
}

// bf16 rows of whole 256-column tiles, G in {64, 256}: the two-threads-per-tile kernel.
template <int G, int BITS, bool UNPACKED = false, bool LNMOD = false>
int launch_quant_bf16_tiles(const void* x, void* q, void* s, int M, int K, cudaStream_t stream,
                            LnModArgs lnmod = LnModArgs{nullptr, nullptr, 0.0f}) {
    const int ntile = K / 256;
    // Rounds of about kQ5RoundTiles tiles let several blocks share an SM (their
    // phases drift apart, which mixes the FMA-heavy rotation with the ALU-heavy
    // packing and the shared-memory loads); longer rows take one row per round.
    int rows = kQ5RoundTiles / ntile;
    if (rows < 1) rows = 1;
    const int full_tiles = (rows * ntile + 15) / 16 * 16;
    const int blocks_per_sm = full_tiles <= kQ5MaxTiles / 2 ? kQ5MaxTiles / full_tiles : 1;
    const int slots = blocks_per_sm * sm_count();
    const int per_block = (M + slots - 1) / slots;
    if (rows > per_block) rows = per_block;            // small M: spread the rows over the SMs
    if (rows < 1) rows = 1;
    const int tiles = (rows * ntile + 15) / 16 * 16;
    const int smem = q5_smem_bytes(2 * tiles) + (LNMOD ? q5_lnmod_bytes(K) : 0);
    auto kernel = convrot_quant_bf16_kernel<G, BITS, UNPACKED, LNMOD>;
    cudaError_t e = ensure_smem(kernel, q5_smem_bytes(kQ5MaxThreads) + (LNMOD ? q5_lnmod_bytes(kQ5LnMaxK) : 0));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 static_cast<int>(cudaSharedmemCarveoutMaxShared));
    if (e != cudaSuccess) return static_cast<int>(e);
    const int rounds = (M + rows - 1) / rows;
    const int grid = rounds < slots ? rounds : slots;
    e = launch_pdl(kernel, dim3(grid), dim3(2 * tiles), static_cast<size_t>(smem), stream,
                   static_cast<const __nv_bfloat16*>(x), static_cast<int8_t*>(q), static_cast<float*>(s), M, K, rows,
                   lnmod);
    return static_cast<int>(e);
}

template <int G>
int launch_quant_g(const void* x, int in_dtype, void* q, void* s, int M, int K, cudaStream_t stream) {
    if constexpr (G == 64 || G == 256) {
        if (in_dtype == 1 && K % 256 == 0 && K / 256 <= kQ5MaxTiles)
            return launch_quant_bf16_tiles<G, 4>(x, q, s, M, K, stream);
    }
    switch (in_dtype) {
        case 0: return launch_quant_t<float, G>(x, q, s, M, K, stream);
        case 1: return launch_quant_t<__nv_bfloat16, G>(x, q, s, M, K, stream);
        case 2: return launch_quant_t<__half, G>(x, q, s, M, K, stream);
        default: return fail("in_dtype must be 0 (f32), 1 (bf16) or 2 (f16)");
    }
}

int check_quant_args(const void* x, int in_dtype, const void* q, const void* s, int M, int K) {
    if (M < 0 || K <= 0) return fail("M must be >= 0 and K > 0");
    if (K % 16 != 0) return fail("K must be a multiple of 16");
    if (in_dtype < 0 || in_dtype > 2) return fail("in_dtype must be 0 (f32), 1 (bf16) or 2 (f16)");
    if (M > 0 && (!x || !q || !s)) return fail("null pointer");
    if (!aligned16(x) || (reinterpret_cast<uintptr_t>(q) & 7u)) return fail("x must be 16-byte and qout 8-byte aligned");
    return 0;
}

int check_linear_args(const void* x, int in_dtype, const void* Wp, const void* wscale, int bias_dtype,
                      const void* out, int out_dtype, int M, int N, int K, int G) {
    if (!(G == 16 || G == 64 || G == 256)) return fail("G must be 16, 64 or 256");
    if (K <= 0 || K % G != 0) return fail("K must be divisible by G");
    if (int rc = check_gemm_args(x, Wp, M, N, K)) return rc;
    if (in_dtype < 0 || in_dtype > 2) return fail("in_dtype must be 0 (f32), 1 (bf16) or 2 (f16)");
    if (out_dtype != 0 && out_dtype != 1) return fail("out_dtype must be 0 (f32) or 1 (bf16)");
    if (bias_dtype < 0 || bias_dtype > 2) return fail("bias_dtype must be 0 (f32), 1 (bf16) or 2 (f16)");
    if (M > 0 && N > 0 && (!wscale || !out)) return fail("null scale or output pointer");
    return 0;
}

// Workspace of the packed-code linear: activation codes [M, K/2], then the
// row scales [M] f32, each from a 256-byte boundary.
size_t packed_linear_workspace_bytes(int M, int K) {
    const size_t codes = (static_cast<size_t>(M) * static_cast<size_t>(K / 2) + 255) & ~static_cast<size_t>(255);
    return codes + ((static_cast<size_t>(M) * 4 + 255) & ~static_cast<size_t>(255));
}

// Rows from which the fused linear takes the A8 form (int8 activation codes,
// packed weights): the tensor-core pipeline without activation expansion.
constexpr int kA8MinRows = 129;

bool a8_eligible(int in_dtype, int M, int K, int G) {
    return in_dtype == 1 && (G == 64 || G == 256) && K % 256 == 0 && K / 256 <= kQ5MaxTiles && M >= kA8MinRows;
}

// Workspace of ck_convrot_w4a4_linear: one int8 per code when the call may take
// the A8 form (M >= kA8MinRows; the size cannot depend on the dtype, which the
// size query does not see), else packed codes.
size_t linear_workspace_bytes(int M, int K) {
    if (M < kA8MinRows) return packed_linear_workspace_bytes(M, K);
    const size_t codes = (static_cast<size_t>(M) * static_cast<size_t>(K) + 255) & ~static_cast<size_t>(255);
    return codes + ((static_cast<size_t>(M) * 4 + 255) & ~static_cast<size_t>(255));
}

// Rotate + quantize x into the workspace, then the int4 GEMM (or GEMV) with the
// bias read in its own dtype. The second launch is a programmatic dependent of
// the first, so its prologue and weight prefetch overlap the quantizer. With
// allow_a8 and many bf16 rows the codes are written one per byte and the A8
// GEMM expands only the packed weights (the same accumulators and output bits).
int run_linear(const void* x, int in_dtype, const void* Wp, const float* ws, BiasRef bias, void* out,
               int out_dtype, int M, int N, int K, int G, unsigned char* workspace, cudaStream_t stream,
               bool allow_a8) {
    if (allow_a8 && a8_eligible(in_dtype, M, K, G)) {
        unsigned char* q = workspace;
        float* xs = reinterpret_cast<float*>(q + ((static_cast<size_t>(M) * K + 255) & ~static_cast<size_t>(255)));
        int rc = G == 256 ? launch_quant_bf16_tiles<256, 4, true>(x, q, xs, M, K, stream)
                          : launch_quant_bf16_tiles<64, 4, true>(x, q, xs, M, K, stream);
        if (rc != 0) return rc;
        if (out_dtype == 1) return dispatch_gemm_a8<kOutBF16>(q, Wp, xs, ws, bias, out, M, N, K, LoraArgs(), stream);
        return dispatch_gemm_a8<kOutF32>(q, Wp, xs, ws, bias, out, M, N, K, LoraArgs(), stream);
    }
    void* q = workspace;
    float* xs = reinterpret_cast<float*>(workspace + ((static_cast<size_t>(M) * (K / 2) + 255) & ~static_cast<size_t>(255)));
    int rc = G == 256 ? launch_quant_g<256>(x, in_dtype, q, xs, M, K, stream)
           : G == 64  ? launch_quant_g<64>(x, in_dtype, q, xs, M, K, stream)
                      : launch_quant_g<16>(x, in_dtype, q, xs, M, K, stream);
    if (rc != 0) return rc;
    if (out_dtype == 1) return dispatch_gemm<kOutBF16>(q, Wp, xs, ws, bias, out, M, N, K, stream);
    return dispatch_gemm<kOutF32>(q, Wp, xs, ws, bias, out, M, N, K, stream);
}

// Dynamic-LoRA down projection (lora_down.cuh): one 128-row tile per CTA, K split
// over a cluster of up to 8 CTAs when the tiles alone would leave most SMs idle.
template <bool kConvert>
int launch_lora_down(const void* x, const void* down, void* t, int M, int K, int R, cudaStream_t stream) {
    CUtensorMap tx, ta;
    // the x map only moves 2-byte elements (no conversion in the copy), so bf16 x
    // uses the fp16 map; out-of-bounds elements are zero bits in either type
    if (!make_f16_tmap(&tx, x, M, K, kLdRows) || !make_f16_tmap(&ta, down, R, K, kLdN))
        return fail("cuTensorMapEncodeTiled failed (pointer not 16-byte aligned or driver entry point missing)");
    auto kernel = lora_down_kernel<kConvert>;
    cudaError_t e = ensure_smem(kernel, kLdSmemBytes);
    if (e != cudaSuccess) return static_cast<int>(e);
    const int m_tiles = (M + kLdRows - 1) / kLdRows;
    const int num_kt = (K + kLdBK - 1) / kLdBK;
    int ksplit = 1;
    if (m_tiles < sm_count()) {
        ksplit = sm_count() / m_tiles;
        if (ksplit > 8) ksplit = 8;
        if (ksplit > num_kt) ksplit = num_kt;
        if (ksplit < 1) ksplit = 1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kLdThreads, 1, 1);
    cfg.dynamicSmemBytes = kLdSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // clusters of ksplit CTAs only fit where a GPC has ksplit free SMs: split less
    // until every tile's cluster is resident at once (a second wave doubles the time)
    for (; ksplit > 1; --ksplit) {
        attr[0].val.clusterDim.x = static_cast<unsigned>(ksplit);
        cfg.gridDim = dim3(static_cast<unsigned>(m_tiles) * static_cast<unsigned>(ksplit), 1, 1);
        int active = 0;
        if (cudaOccupancyMaxActiveClusters(&active, kernel, &cfg) != cudaSuccess) {
            (void)cudaGetLastError();
            continue;
        }
        if (active >= m_tiles) break;
    }
    attr[0].val.clusterDim.x = static_cast<unsigned>(ksplit);
    cfg.gridDim = dim3(static_cast<unsigned>(m_tiles) * static_cast<unsigned>(ksplit), 1, 1);
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    e = cudaLaunchKernelEx(&cfg, kernel, tx, ta, static_cast<__half*>(t), M, K, R, ksplit);
    if (e != cudaSuccess) return static_cast<int>(e);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace convrot

using namespace convrot;

// ---------------------------------------------------------------------------
// C-ABI (declared in include/convrot_b200.h)
// ---------------------------------------------------------------------------

CONVROT_API const char* ck_convrot_last_error(void) { return g_last_error; }

CONVROT_API int ck_convrot_quant_int4(const void* x, int in_dtype, void* qout, void* scaleout,
                                      int M, int K, int G, void* stream) {
    if (!(G == 16 || G == 64 || G == 256)) return fail("G must be 16, 64 or 256");
    if (K % G != 0) return fail("K must be divisible by G");
    if (int rc = check_quant_args(x, in_dtype, qout, scaleout, M, K)) return rc;
    if (M == 0) return 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (G == 256) return launch_quant_g<256>(x, in_dtype, qout, scaleout, M, K, s);
    if (G == 64) return launch_quant_g<64>(x, in_dtype, qout, scaleout, M, K, s);
    return launch_quant_g<16>(x, in_dtype, qout, scaleout, M, K, s);
}

CONVROT_API int ck_int4_quant_rowwise(const void* x, int in_dtype, void* qout, void* scaleout,
                                      int M, int K, void* stream) {
    if (int rc = check_quant_args(x, in_dtype, qout, scaleout, M, K)) return rc;
    if (M == 0) return 0;
    return launch_quant_g<1>(x, in_dtype, qout, scaleout, M, K, static_cast<cudaStream_t>(stream));
}

CONVROT_API int ck_int4_convrot_gemm(const void* Xp, const void* Wp, const void* xscale, const void* wscale,
                                     const void* bias, void* out, int M, int N, int K, int out_dtype,
                                     void* stream) {
    if (int rc = check_gemm_args(Xp, Wp, M, N, K)) return rc;
    if (out_dtype != 0 && out_dtype != 1) return fail("out_dtype must be 0 (f32) or 1 (bf16)");
    if (M == 0 || N == 0) return 0;
    if (!xscale || !wscale || !out) return fail("null scale or output pointer");
    const float* xs = static_cast<const float*>(xscale);
    const float* ws = static_cast<const float*>(wscale);
    const BiasRef b{bias, 0};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (out_dtype == 1) return dispatch_gemm<kOutBF16>(Xp, Wp, xs, ws, b, out, M, N, K, s);
    return dispatch_gemm<kOutF32>(Xp, Wp, xs, ws, b, out, M, N, K, s);
}

CONVROT_API size_t ck_convrot_w4a4_linear_workspace_size(int M, int K) {
    if (M <= 0 || K <= 0) return 0;
    return linear_workspace_bytes(M, K);
}

CONVROT_API int ck_convrot_w4a4_linear(const void* x, int in_dtype, const void* Wp, const void* wscale,
                                       const void* bias, int bias_dtype, void* out, int out_dtype,
                                       int M, int N, int K, int G, void* workspace, size_t workspace_bytes,
                                       void* stream) {
    if (int rc = check_linear_args(x, in_dtype, Wp, wscale, bias_dtype, out, out_dtype, M, N, K, G)) return rc;
    if (M == 0 || N == 0) return 0;
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255u)) return fail("workspace must be 256-byte aligned");
    if (workspace_bytes < linear_workspace_bytes(M, K))
        return fail("workspace smaller than ck_convrot_w4a4_linear_workspace_size(M, K)");
    return run_linear(x, in_dtype, Wp, static_cast<const float*>(wscale), BiasRef{bias, bias_dtype}, out,
                      out_dtype, M, N, K, G, static_cast<unsigned char*>(workspace),
                      static_cast<cudaStream_t>(stream), true);
}

CONVROT_API int ck_int4_convrot_gemm_lora(const void* Xp, const void* Wp, const void* xscale, const void* wscale,
                                          const void* bias, int bias_dtype, void* out, int M, int N, int K,
                                          int out_dtype, const void* lora_t, const void* lora_b, int rank,
                                          float lora_scale, void* stream) {
    if (int rc = check_gemm_args(Xp, Wp, M, N, K)) return rc;
    if (out_dtype != 0 && out_dtype != 1) return fail("out_dtype must be 0 (f32) or 1 (bf16)");
    if (bias_dtype < 0 || bias_dtype > 2) return fail("bias_dtype must be 0 (f32), 1 (bf16) or 2 (f16)");
    if (rank < 8 || rank > 64 || rank % 8 != 0) return fail("LoRA rank must be a multiple of 8 in [8, 64]");
    if (M == 0 || N == 0) return 0;
    if (!xscale || !wscale || !out || !lora_t || !lora_b) return fail("null pointer");
    if (!aligned16(lora_t) || !aligned16(lora_b)) return fail("LoRA operands must be 16-byte aligned");
    LoraArgs lora;
    lora.t = lora_t;
    lora.b = lora_b;
    lora.rank = rank;
    lora.scale = lora_scale;
    const float* xs = static_cast<const float*>(xscale);
    const float* ws = static_cast<const float*>(wscale);
    const BiasRef b{bias, bias_dtype};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // 256 x 128 pair tiles leave TMEM room for the fp32 LoRA accumulator
    if (out_dtype == 1) return launch_pair<128, false, kOutBF16, true>(Xp, Wp, xs, ws, b, out, M, N, K, s, lora);
    return launch_pair<128, false, kOutF32, true>(Xp, Wp, xs, ws, b, out, M, N, K, s, lora);
}

CONVROT_API int ck_int4_convrot_gemm_splitk(const void* Xp, const void* Wp, const void* xscale,
                                            const void* wscale, void* accum, int M, int N, int K,
                                            int nsplit, void* stream) {
    if (int rc = check_gemm_args(Xp, Wp, M, N, K)) return rc;
    if (nsplit < 1) return fail("nsplit must be >= 1");
    if (M == 0 || N == 0) return 0;
    if (!xscale || !wscale || !accum) return fail("null scale or accumulator pointer");
    return dispatch_gemm<kOutF32Accumulate>(Xp, Wp, static_cast<const float*>(xscale),
                                            static_cast<const float*>(wscale), BiasRef{nullptr, 0}, accum, M, N, K,
                                            static_cast<cudaStream_t>(stream));
}

CONVROT_API int ck_int4_gemm_s32(const void* Xp, const void* Wp, void* acc, int M, int N, int K, void* stream) {
    if (int rc = check_gemm_args(Xp, Wp, M, N, K)) return rc;
    if (M == 0 || N == 0) return 0;
    if (!acc) return fail("null accumulator pointer");
    return dispatch_gemm<kOutS32>(Xp, Wp, nullptr, nullptr, BiasRef{nullptr, 0}, acc, M, N, K,
                                  static_cast<cudaStream_t>(stream));
}

CONVROT_API int ck_convrot_quant_int8(const void* x, int in_dtype, void* qout, void* scaleout,
                                      int M, int K, int G, void* stream) {
    if (!(G == 16 || G == 64 || G == 256)) return fail("G must be 16, 64 or 256");
    if (K <= 0 || K % G != 0) return fail("K must be divisible by G");
    if (int rc = check_quant_args(x, in_dtype, qout, scaleout, M, K)) return rc;
    if (in_dtype != 1 || (G != 64 && G != 256) || K % 256 != 0 || K / 256 > kQ5MaxTiles)
        return fail("the int8 quantizer takes bf16 rows of whole 256-column tiles with G = 64 or 256");
    if (reinterpret_cast<uintptr_t>(qout) & 15u) return fail("qout must be 16-byte aligned");
    if (M == 0) return 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (G == 256) return launch_quant_bf16_tiles<256, 8>(x, qout, scaleout, M, K, s);
    return launch_quant_bf16_tiles<64, 8>(x, qout, scaleout, M, K, s);
}

int check_gemm_i8_args(const void* X, const void* W, int M, int N, int K) {
    if (M < 0 || N < 0 || K <= 0) return fail("M, N must be >= 0 and K > 0");
    if (K % 16 != 0) return fail("K must be a multiple of 16");
    if (M > 0 && N > 0 && (!X || !W)) return fail("null operand pointer");
    if (!aligned16(X) || !aligned16(W)) return fail("int8 operands must be 16-byte aligned");
    return 0;
}

CONVROT_API int ck_int8_convrot_gemm_lora(const void* X, const void* W, const void* xscale, const void* wscale,
                                          const void* bias, int bias_dtype, void* out, int M, int N, int K,
                                          int out_dtype, const void* lora_t, const void* lora_b, int rank,
                                          float lora_scale, void* stream) {
    if (int rc = check_gemm_i8_args(X, W, M, N, K)) return rc;
    if (out_dtype != 0 && out_dtype != 1) return fail("out_dtype must be 0 (f32) or 1 (bf16)");
    if (bias_dtype < 0 || bias_dtype > 2) return fail("bias_dtype must be 0 (f32), 1 (bf16) or 2 (f16)");
    if (rank < 8 || rank > 64 || rank % 8 != 0) return fail("LoRA rank must be a multiple of 8 in [8, 64]");
    if (M == 0 || N == 0) return 0;
    if (!xscale || !wscale || !out || !lora_t || !lora_b) return fail("null pointer");
    if (!aligned16(lora_t) || !aligned16(lora_b)) return fail("LoRA operands must be 16-byte aligned");
    LoraArgs lora;
    lora.t = lora_t;
    lora.b = lora_b;
    lora.rank = rank;
    lora.scale = lora_scale;
    const float* xs = static_cast<const float*>(xscale);
    const float* ws = static_cast<const float*>(wscale);
    const BiasRef b{bias, bias_dtype};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // 256 x 256 pair tiles (one int32 + fp32 accumulator pair fills TMEM) halve the
    // operand bytes per MMA of 256 x 128 tiles (two buffers, epilogue overlapped);
    // the latter only when 256-column tiles leave most CTA pairs idle
    const long tiles256 = static_cast<long>((M + 255) / 256) * ((N + 255) / 256);
    const bool wide = 2 * tiles256 >= sm_count();
    if (out_dtype == 1) {
        if (wide)
            return launch_pair_impl<256, false, kOutBF16, false, true, true>(X, W, xs, ws, b, out, M, N, K, lora, s);
        if ((N % 8) == 0 && aligned16(out) && K < 3072)
            return launch_pair_impl<128, false, kOutBF16, true, true, true>(X, W, xs, ws, b, out, M, N, K, lora, s);
        return launch_pair_impl<128, false, kOutBF16, false, true, true>(X, W, xs, ws, b, out, M, N, K, lora, s);
    }
    if (wide)
        return launch_pair_impl<256, false, kOutF32, false, true, true>(X, W, xs, ws, b, out, M, N, K, lora, s);
    return launch_pair_impl<128, false, kOutF32, false, true, true>(X, W, xs, ws, b, out, M, N, K, lora, s);
}

CONVROT_API int ck_int8_convrot_gemm(const void* X, const void* W, const void* xscale, const void* wscale,
                                     const void* bias, void* out, int M, int N, int K, int out_dtype,
                                     void* stream) {
    if (int rc = check_gemm_i8_args(X, W, M, N, K)) return rc;
    if (out_dtype != 0 && out_dtype != 1) return fail("out_dtype must be 0 (f32) or 1 (bf16)");
    if (M == 0 || N == 0) return 0;
    if (!xscale || !wscale || !out) return fail("null scale or output pointer");
    const float* xs = static_cast<const float*>(xscale);
    const float* ws = static_cast<const float*>(wscale);
    const BiasRef b{bias, 0};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (out_dtype == 1) return dispatch_gemm_i8<kOutBF16>(X, W, xs, ws, b, out, M, N, K, s);
    return dispatch_gemm_i8<kOutF32>(X, W, xs, ws, b, out, M, N, K, s);
}

CONVROT_API int ck_int8_gemm_s32(const void* X, const void* W, void* acc, int M, int N, int K, void* stream) {
    if (int rc = check_gemm_i8_args(X, W, M, N, K)) return rc;
    if (M == 0 || N == 0) return 0;
    if (!acc) return fail("null accumulator pointer");
    return dispatch_gemm_i8<kOutS32>(X, W, nullptr, nullptr, BiasRef{nullptr, 0}, acc, M, N, K,
                                     static_cast<cudaStream_t>(stream));
}

CONVROT_API int ck_int4_convrot_gemm_a8(const void* X8, const void* Wp, const void* xscale, const void* wscale,
                                        const void* bias, int bias_dtype, void* out, int M, int N, int K,
                                        int out_dtype, const void* lora_t, const void* lora_b, int rank,
                                        float lora_scale, void* stream) {
    if (M < 0 || N < 0 || K <= 0 || K % 128 != 0 || K > 65536)
        return fail("M, N must be >= 0 and K a multiple of 128 in [128, 65536]");
    if (out_dtype != 0 && out_dtype != 1 && out_dtype != 3) return fail("out_dtype must be 0 (f32), 1 (bf16) or 3 (s32)");
    if (bias_dtype < 0 || bias_dtype > 2) return fail("bias_dtype must be 0 (f32), 1 (bf16) or 2 (f16)");
    const bool with_lora = lora_t != nullptr || lora_b != nullptr;
    if (with_lora && (rank < 8 || rank > 64 || rank % 8 != 0)) return fail("LoRA rank must be a multiple of 8 in [8, 64]");
    if (with_lora && out_dtype == 3) return fail("the int32 accumulator output has no LoRA side path");
    if (M == 0 || N == 0) return 0;
    if (!X8 || !Wp || !out) return fail("null operand or output pointer");
    if (out_dtype != 3 && (!xscale || !wscale)) return fail("null scale pointer");
    if (!aligned16(X8) || !aligned16(Wp)) return fail("operands must be 16-byte aligned");
    if (with_lora && (!lora_t || !lora_b || !aligned16(lora_t) || !aligned16(lora_b)))
        return fail("LoRA operands must be non-null and 16-byte aligned");
    LoraArgs lora;
    if (with_lora) {
        lora.t = lora_t;
        lora.b = lora_b;
        lora.rank = rank;
        lora.scale = lora_scale;
    }
    const float* xs = static_cast<const float*>(xscale);
    const float* ws = static_cast<const float*>(wscale);
    const BiasRef b{bias, bias_dtype};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (out_dtype == 1) return dispatch_gemm_a8<kOutBF16>(X8, Wp, xs, ws, b, out, M, N, K, lora, s);
    if (out_dtype == 0) return dispatch_gemm_a8<kOutF32>(X8, Wp, xs, ws, b, out, M, N, K, lora, s);
    return dispatch_gemm_a8<kOutS32>(X8, Wp, nullptr, nullptr, BiasRef{nullptr, 0}, out, M, N, K, lora, s);
}

CONVROT_API int ck_lora_down(const void* x, int in_dtype, const void* down, void* t, int M, int K, int R,
                             void* stream) {
    if (M < 0 || K <= 0 || K % 8 != 0) return fail("M must be >= 0 and K a positive multiple of 8");
    if (R < 8 || R > 64 || R % 8 != 0) return fail("rank R must be a multiple of 8 in [8, 64]");
    if (in_dtype != 1 && in_dtype != 2) return fail("in_dtype must be 1 (bf16) or 2 (f16)");
    if (M == 0) return 0;
    if (!x || !down || !t) return fail("null operand or output pointer");
    if (!aligned16(x) || !aligned16(down) || !aligned16(t)) return fail("operands must be 16-byte aligned");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return in_dtype == 1 ? launch_lora_down<true>(x, down, t, M, K, R, s)
                         : launch_lora_down<false>(x, down, t, M, K, R, s);
}

CONVROT_API int ck_int4_unpack(const void* packed, void* codes, long long rows, int K, void* stream) {
    if (rows < 0 || K <= 0 || K % 32 != 0) return fail("rows must be >= 0 and K a positive multiple of 32");
    if (rows == 0) return 0;
    if (!packed || !codes) return fail("null pointer");
    if (!aligned16(packed) || !aligned16(codes)) return fail("packed and codes must be 16-byte aligned");
    const size_t n16 = static_cast<size_t>(rows) * static_cast<size_t>(K / 2) / 16;
    const int grid = static_cast<int>(n16 / 256 + 1 < static_cast<size_t>(4 * sm_count()) ? n16 / 256 + 1 : 4 * sm_count());
    int4_unpack_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(packed), static_cast<uint4*>(codes), n16);
    return static_cast<int>(cudaGetLastError());
}

namespace convrot {

int check_unpacked_linear_args(const void* x, int in_dtype, int M, int K, int G) {
    if (in_dtype != 1 || (G != 64 && G != 256) || K <= 0 || K % 256 != 0 || K / 256 > kQ5MaxTiles)
        return fail("the unpacked-code path takes bf16 rows of whole 256-column tiles with G = 64 or 256");
    if (M < 0) return fail("M must be >= 0");
    if (M > 0 && !x) return fail("null pointer");
    if (!aligned16(x)) return fail("x must be 16-byte aligned");
    return 0;
}

size_t unpacked_linear_workspace_bytes(int M, int K) {
    const size_t codes = (static_cast<size_t>(M) * static_cast<size_t>(K) + 255) & ~static_cast<size_t>(255);
    return codes + ((static_cast<size_t>(M) * 4 + 255) & ~static_cast<size_t>(255));
}

}  // namespace convrot

CONVROT_API int ck_convrot_quant_int4_unpacked(const void* x, int in_dtype, void* qout, void* scaleout,
                                               int M, int K, int G, void* stream) {
    if (int rc = check_unpacked_linear_args(x, in_dtype, M, K, G)) return rc;
    if (M == 0) return 0;
    if (!qout || !scaleout) return fail("null pointer");
    if (reinterpret_cast<uintptr_t>(qout) & 15u) return fail("qout must be 16-byte aligned");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (G == 256) return launch_quant_bf16_tiles<256, 4, true>(x, qout, scaleout, M, K, s);
    return launch_quant_bf16_tiles<64, 4, true>(x, qout, scaleout, M, K, s);
}

CONVROT_API size_t ck_convrot_w4a4_linear_unpacked_workspace_size(int M, int K) {
    if (M <= 0 || K <= 0) return 0;
    return unpacked_linear_workspace_bytes(M, K);
}

CONVROT_API int ck_convrot_w4a4_linear_unpacked(const void* x, int in_dtype, const void* Wcodes, const void* wscale,
                                                const void* bias, int bias_dtype, void* out, int out_dtype,
                                                int M, int N, int K, int G, void* workspace,
                                                size_t workspace_bytes, void* stream) {
    if (int rc = check_unpacked_linear_args(x, in_dtype, M, K, G)) return rc;
    if (int rc = check_gemm_i8_args(x, Wcodes, M, N, K)) return rc;
    if (out_dtype != 0 && out_dtype != 1) return fail("out_dtype must be 0 (f32) or 1 (bf16)");
    if (bias_dtype < 0 || bias_dtype > 2) return fail("bias_dtype must be 0 (f32), 1 (bf16) or 2 (f16)");
    if (M == 0 || N == 0) return 0;
    if (!wscale || !out) return fail("null scale or output pointer");
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255u)) return fail("workspace must be 256-byte aligned");
    if (workspace_bytes < unpacked_linear_workspace_bytes(M, K))
        return fail("workspace smaller than ck_convrot_w4a4_linear_unpacked_workspace_size(M, K)");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned char* q = static_cast<unsigned char*>(workspace);
    float* xs = reinterpret_cast<float*>(q + ((static_cast<size_t>(M) * K + 255) & ~static_cast<size_t>(255)));
    int rc = G == 256 ? launch_quant_bf16_tiles<256, 4, true>(x, q, xs, M, K, s)
                      : launch_quant_bf16_tiles<64, 4, true>(x, q, xs, M, K, s);
    if (rc != 0) return rc;
    const BiasRef b{bias, bias_dtype};
    const float* ws = static_cast<const float*>(wscale);
    if (out_dtype == 1) return dispatch_gemm_i8<kOutBF16>(q, Wcodes, xs, ws, b, out, M, N, K, s);
    return dispatch_gemm_i8<kOutF32>(q, Wcodes, xs, ws, b, out, M, N, K, s);
}

// A wait that nothing ends: one thread waits on a fresh mbarrier that no one
// arrives on, gives up after limit_ns, records kStatusTimeoutSelfTest and
// returns -- the path every pipeline wait takes when a partner never shows up.
__global__ void selftest_wait_timeout_kernel(unsigned long long limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    fence_mbar_init();
    if (!mbar_wait_bounded(&bar, 0, limit_ns)) record_status(kStatusTimeoutSelfTest);
}

CONVROT_API int ck_convrot_selftest_wait_timeout(long long limit_ns, void* stream) {
    if (limit_ns <= 0 || limit_ns > 100000000LL) return fail("limit_ns must be in (0, 1e8]");
    selftest_wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<unsigned long long>(limit_ns));
    return static_cast<int>(cudaGetLastError());
}

CONVROT_API int ck_convrot_device_status(void* stream, int* status) {
    if (!status) return fail("null status pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int host = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(&host, g_device_status, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return static_cast<int>(e);
    *status = host;
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_device_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    return static_cast<int>(e);
}

// ---------------------------------------------------------------------------
// Column-split linear over peer memory (no reference counterpart: the
// reference runs on one device). Each rank's GEMM stores its column block into
// every rank's [M, ldo] output through peer mappings (CUDA IPC, plain stores
// over NVLink, no multicast), then a flag barrier tells each rank that every
// peer's block has landed in its own output.
// ---------------------------------------------------------------------------

namespace convrot {

struct PeerFlags {
    unsigned* ptr[8];       // rank p's flag words (this process's mapping); slot q = written by rank q
};

// One warp: thread p signals rank p (slot `rank` of its flags) with this call's
// epoch, then waits, bounded, for rank p's signal in its own slot p. The epoch
// is a per-process device counter, so the kernel can be replayed from a graph.
__global__ void peer_barrier_kernel(PeerFlags f, int nranks, int rank, unsigned* counter,
                                    unsigned long long limit_ns) {
    const int p = threadIdx.x;
    unsigned epoch = 0u;
    if (p == 0) {
        epoch = *counter + 1u;
        *counter = epoch;
    }
    epoch = __shfl_sync(0xFFFFFFFFu, epoch, 0);
    if (p >= nranks) return;
    __threadfence_system();                           // the stores of the kernels before this one
    asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(f.ptr[p] + rank), "r"(epoch) : "memory");
    const unsigned* mine = f.ptr[rank] + p;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        unsigned v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
        if (static_cast<int>(v - epoch) >= 0) break;
        if (globaltimer_ns() - t0 > limit_ns) {
            record_status(kStatusTimeoutPeer);
            break;
        }
        __nanosleep(64);
    }
}

}  // namespace convrot

CONVROT_API int ck_peer_buffer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
    if (!ptr || !ipc_handle || bytes == 0) return fail("null pointer or zero size");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return static_cast<int>(e);
    e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return static_cast<int>(e);
    }
    *ptr = p;
    return 0;
}

CONVROT_API int ck_peer_buffer_open(const void* ipc_handle, void** ptr) {
    if (!ptr || !ipc_handle) return fail("null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    return static_cast<int>(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

CONVROT_API int ck_peer_buffer_close(void* ptr) {
    return ptr ? static_cast<int>(cudaIpcCloseMemHandle(ptr)) : 0;
}

CONVROT_API int ck_peer_buffer_free(void* ptr) {
    return ptr ? static_cast<int>(cudaFree(ptr)) : 0;
}

CONVROT_API int ck_peer_barrier(void* const* flags, int nranks, int rank, void* counter, long long timeout_ns,
                                void* stream) {
    if (nranks < 1 || nranks > 8 || rank < 0 || rank >= nranks) return fail("nranks in [1, 8], 0 <= rank < nranks");
    if (!flags || !counter) return fail("null flag or counter pointer");
    if (timeout_ns <= 0 || timeout_ns > 60000000000LL) return fail("timeout_ns must be in (0, 6e10]");
    PeerFlags f{};
    for (int p = 0; p < nranks; ++p) {
        if (!flags[p] || (reinterpret_cast<uintptr_t>(flags[p]) & 3u)) return fail("flag pointers must be 4-byte aligned");
        f.ptr[p] = static_cast<unsigned*>(flags[p]);
    }
    peer_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
        f, nranks, rank, static_cast<unsigned*>(counter), static_cast<unsigned long long>(timeout_ns));
    return static_cast<int>(cudaGetLastError());
}

CONVROT_API int ck_int4_convrot_gemm_a8_peers(const void* X8, const void* Wp, const void* xscale, const void* wscale,
                                              const void* bias, int bias_dtype, void* const* outs, int nouts,
                                              int ldo, int col0, int M, int N, int K, int out_dtype,
                                              const void* lora_t, const void* lora_b, int rank,
                                              float lora_scale, void* stream) {
    if (M < 0 || N < 0 || K <= 0 || K % 128 != 0 || K > 65536)
        return fail("M, N must be >= 0 and K a multiple of 128 in [128, 65536]");
    if (out_dtype != 0 && out_dtype != 1) return fail("out_dtype must be 0 (f32) or 1 (bf16)");
    if (bias_dtype < 0 || bias_dtype > 2) return fail("bias_dtype must be 0 (f32), 1 (bf16) or 2 (f16)");
    if (nouts < 1 || nouts > 8 || !outs) return fail("1 to 8 output pointers");
    if (col0 < 0 || ldo < col0 + N || ldo % 8 != 0 || col0 % 8 != 0)
        return fail("need 0 <= col0, col0 + N <= ldo, ldo and col0 multiples of 8");
    const bool with_lora = lora_t != nullptr || lora_b != nullptr;
    if (with_lora && (rank < 8 || rank > 64 || rank % 8 != 0)) return fail("LoRA rank must be a multiple of 8 in [8, 64]");
    if (M == 0 || N == 0) return 0;
    if (!X8 || !Wp || !xscale || !wscale) return fail("null operand or scale pointer");
    if (!aligned16(X8) || !aligned16(Wp)) return fail("operands must be 16-byte aligned");
    if (with_lora && (!lora_t || !lora_b || !aligned16(lora_t) || !aligned16(lora_b)))
        return fail("LoRA operands must be non-null and 16-byte aligned");
    PeerOut peers{};
    for (int d = 0; d < nouts; ++d) {
        if (!outs[d] || !aligned16(outs[d])) return fail("output pointers must be non-null and 16-byte aligned");
        peers.ptr[d] = outs[d];
    }
    peers.count = nouts;
    peers.ldo = ldo;
    peers.col0 = col0;
    LoraArgs lora;
    if (with_lora) {
        lora.t = lora_t;
        lora.b = lora_b;
        lora.rank = rank;
        lora.scale = lora_scale;
    }
    const float* xs = static_cast<const float*>(xscale);
    const float* ws = static_cast<const float*>(wscale);
    const BiasRef b{bias, bias_dtype};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // the direct-store A8 pair kernel: 256 x 256 tiles when they fill the CTA pairs
    const bool wide = 2L * ((M + 255) / 256) * ((N + 255) / 256) >= sm_count();
    if (out_dtype == 1) {
        if (with_lora)
            return wide ? launch_pair_impl<256, false, kOutBF16, false, true, false, true>(X8, Wp, xs, ws, b, nullptr, M, N, K, lora, s, peers)
                        : launch_pair_impl<128, false, kOutBF16, false, true, false, true>(X8, Wp, xs, ws, b, nullptr, M, N, K, lora, s, peers);
        return wide ? launch_pair_impl<256, false, kOutBF16, false, false, false, true>(X8, Wp, xs, ws, b, nullptr, M, N, K, lora, s, peers)
                    : launch_pair_impl<128, false, kOutBF16, false, false, false, true>(X8, Wp, xs, ws, b, nullptr, M, N, K, lora, s, peers);
    }
    if (with_lora)
        return wide ? launch_pair_impl<256, false, kOutF32, false, true, false, true>(X8, Wp, xs, ws, b, nullptr, M, N, K, lora, s, peers)
                    : launch_pair_impl<128, false, kOutF32, false, true, false, true>(X8, Wp, xs, ws, b, nullptr, M, N, K, lora, s, peers);
    return wide ? launch_pair_impl<256, false, kOutF32, false, false, false, true>(X8, Wp, xs, ws, b, nullptr, M, N, K, lora, s, peers)
                : launch_pair_impl<128, false, kOutF32, false, false, false, true>(X8, Wp, xs, ws, b, nullptr, M, N, K, lora, s, peers);
}

CONVROT_API int ck_peer_copy_columns(void* const* dsts, int ndst, const void* src, long long pitch_bytes,
                                     long long offset_bytes, long long width_bytes, long long rows, void* stream) {
    if (ndst < 0 || ndst > 8 || (ndst > 0 && !dsts) || !src) return fail("0 to 8 destinations and a source");
    if (pitch_bytes <= 0 || width_bytes <= 0 || offset_bytes < 0 || offset_bytes + width_bytes > pitch_bytes || rows < 0)
        return fail("need 0 <= offset, offset + width <= pitch, rows >= 0");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const unsigned char* from = static_cast<const unsigned char*>(src) + offset_bytes;
    for (int d = 0; d < ndst; ++d) {
        if (!dsts[d]) return fail("null destination");
        cudaError_t e = cudaMemcpy2DAsync(static_cast<unsigned char*>(dsts[d]) + offset_bytes,
                                          static_cast<size_t>(pitch_bytes), from, static_cast<size_t>(pitch_bytes),
                                          static_cast<size_t>(width_bytes), static_cast<size_t>(rows),
                                          cudaMemcpyDefault, s);
        if (e != cudaSuccess) return static_cast<int>(e);
    }
    return 0;
}

// ---------------------------------------------------------------------------
// Rotation fused into the producer of x: LayerNorm + modulation, then rotate +
// quantize, in one pass over x (no reference counterpart: the reference
// quantizes the activation the model's own LayerNorm/modulation kernels wrote).
// ---------------------------------------------------------------------------

namespace convrot {

int check_lnmod_args(const void* x, const void* mod_scale, const void* mod_shift, float eps, int M, int K, int G) {
    if (M < 0 || K <= 0) return fail("M must be >= 0 and K > 0");
    if (!(G == 64 || G == 256)) return fail("G must be 64 or 256 for the fused LayerNorm form");
    if (K % 256 != 0 || K > kQ5LnMaxK) return fail("K must be a multiple of 256 and at most 6144");
    if (!(eps >= 0.0f)) return fail("eps must be >= 0");
    if (M > 0 && !x) return fail("null activation pointer");
    if (!aligned16(x) || (reinterpret_cast<uintptr_t>(mod_scale) & 1u) || (reinterpret_cast<uintptr_t>(mod_shift) & 1u))
        return fail("x must be 16-byte aligned, the modulation vectors 2-byte aligned");
    return 0;
}

template <bool UNPACKED>
int launch_quant_lnmod(const void* x, const LnModArgs& ln, void* q, void* s, int M, int K, int G, cudaStream_t stream) {
    return G == 256 ? launch_quant_bf16_tiles<256, 4, UNPACKED, true>(x, q, s, M, K, stream, ln)
                    : launch_quant_bf16_tiles<64, 4, UNPACKED, true>(x, q, s, M, K, stream, ln);
}

}  // namespace convrot

CONVROT_API int ck_convrot_quant_int4_lnmod(const void* x, const void* mod_scale, const void* mod_shift, float eps,
                                            void* qout, void* scaleout, int M, int K, int G, int unpacked,
                                            void* stream) {
    if (int rc = check_lnmod_args(x, mod_scale, mod_shift, eps, M, K, G)) return rc;
    if (M == 0) return 0;
    if (!qout || !scaleout || (reinterpret_cast<uintptr_t>(qout) & 7u)) return fail("qout (8-byte aligned) and scaleout needed");
    const LnModArgs ln{static_cast<const __nv_bfloat16*>(mod_scale), static_cast<const __nv_bfloat16*>(mod_shift), eps};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return unpacked ? launch_quant_lnmod<true>(x, ln, qout, scaleout, M, K, G, s)
                    : launch_quant_lnmod<false>(x, ln, qout, scaleout, M, K, G, s);
}

CONVROT_API int ck_convrot_w4a4_linear_lnmod(const void* x, const void* mod_scale, const void* mod_shift, float eps,
                                             const void* Wp, const void* wscale, const void* bias, int bias_dtype,
                                             void* out, int out_dtype, int M, int N, int K, int G, void* workspace,
                                             size_t workspace_bytes, void* stream) {
    if (int rc = check_lnmod_args(x, mod_scale, mod_shift, eps, M, K, G)) return rc;
    if (int rc = check_linear_args(x, 1, Wp, wscale, bias_dtype, out, out_dtype, M, N, K, G)) return rc;
    if (M == 0 || N == 0) return 0;
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255u)) return fail("workspace must be 256-byte aligned");
    if (workspace_bytes < linear_workspace_bytes(M, K))
        return fail("workspace smaller than ck_convrot_w4a4_linear_workspace_size(M, K)");
    const LnModArgs ln{static_cast<const __nv_bfloat16*>(mod_scale), static_cast<const __nv_bfloat16*>(mod_shift), eps};
    const float* ws = static_cast<const float*>(wscale);
    const BiasRef b{bias, bias_dtype};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned char* q = static_cast<unsigned char*>(workspace);
    if (a8_eligible(1, M, K, G)) {
        float* xs = reinterpret_cast<float*>(q + ((static_cast<size_t>(M) * K + 255) & ~static_cast<size_t>(255)));
        if (int rc = launch_quant_lnmod<true>(x, ln, q, xs, M, K, G, s)) return rc;
        if (out_dtype == 1) return dispatch_gemm_a8<kOutBF16>(q, Wp, xs, ws, b, out, M, N, K, LoraArgs(), s);
        return dispatch_gemm_a8<kOutF32>(q, Wp, xs, ws, b, out, M, N, K, LoraArgs(), s);
    }
    float* xs = reinterpret_cast<float*>(q + ((static_cast<size_t>(M) * (K / 2) + 255) & ~static_cast<size_t>(255)));
    if (int rc = launch_quant_lnmod<false>(x, ln, q, xs, M, K, G, s)) return rc;
    if (out_dtype == 1) return dispatch_gemm<kOutBF16>(q, Wp, xs, ws, b, out, M, N, K, s);
    return dispatch_gemm<kOutF32>(q, Wp, xs, ws, b, out, M, N, K, s);
}
