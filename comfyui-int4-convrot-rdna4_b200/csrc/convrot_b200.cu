// ConvRot W4A4 linear path for NVIDIA B200 (sm_100a).
//
// Two kernels and the C-ABI that the Python host layer (ctypes) binds:
//
//  (1) convrot_quant_kernel: blockwise regular-Hadamard rotation of an
//      activation row, row-wise absmax int4 quantization and nibble packing.
//      Same contract as the reference's fused quantizer
//      (_int4/int4_gemm.hip:348-408), with the quantizer arithmetic of its
//      eager path (_int4/eager.py:112-120) so codes and scales match eager.
//
//  (2) int4_gemm_kernel: packed-int4 x packed-int4 GEMM on the 5th-generation
//      tensor cores. TMA brings packed [rows x 64 B] tiles into shared memory;
//      expander warps split every byte into its high nibble (b & 0xF0) and its
//      low nibble moved up (b << 4), both as int8 values 16*code; one thread
//      issues tcgen05.mma.kind::i8 on the two halves into one int32 TMEM
//      accumulator, which therefore holds 256 * sum_k x_k w_k exactly. The
//      epilogue reads TMEM, shifts the accumulator back (exact), applies
//      ((D * xs[m]) * ws[n]) + bias[n] in fp32 (_int4/int4_gemm.hip:152-169)
//      and stores bf16 or fp32.
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
        uint4 a = __ldg(q), b = __ldg(q + 1);
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
            float4 a = __ldg(q + i);
            v[4 * i] = a.x; v[4 * i + 1] = a.y; v[4 * i + 2] = a.z; v[4 * i + 3] = a.w;
        }
    }
}

constexpr int kQuantThreads = 256;
constexpr int kTransposeFloats = 16 * 16 * 17;   // 16 half-warps x 16 x 17 (padded)

// One block handles `rows_per_block` rows. Phase 1: each half-warp rotates
// 256-element tiles (a 16x16 matrix, element i = 16a + b): H16 along b in
// registers, a padded shared-memory transpose, then H_{G/16} along a; the
// result is rounded to the activation dtype, kept in a shared row buffer and
// folded into the row absmax. Phase 2: per-row scale. Phase 3: quantize and
// pack 16 elements per step into 8 output bytes.
// G == 1 skips the rotation (the input is already rotated).
template <typename T, int G>
__global__ void __launch_bounds__(kQuantThreads)
convrot_quant_kernel(const T* __restrict__ x, int8_t* __restrict__ qout, float* __restrict__ scaleout,
                     int M, int K, int rows_per_block) {
    extern __shared__ __align__(16) unsigned char qsmem[];
    float* tr = reinterpret_cast<float*>(qsmem);                               // transpose scratch
    uint32_t* rowmax = reinterpret_cast<uint32_t*>(tr + kTransposeFloats);     // [rows_per_block]
    float* row_scale = reinterpret_cast<float*>(rowmax + rows_per_block);      // [rows_per_block]
    float* row_rcp = row_scale + rows_per_block;                                // [rows_per_block]
    T* rowbuf = reinterpret_cast<T*>(qsmem + (((kTransposeFloats + 3 * rows_per_block) * 4 + 15) & ~15));

    const int row0 = blockIdx.x * rows_per_block;
    const int nrows = min(rows_per_block, M - row0);
    const int tid = threadIdx.x;
    for (int r = tid; r < nrows; r += kQuantThreads) rowmax[r] = 0u;
    __syncthreads();

    const int hw = tid >> 4;          // half-warp 0..15
    const int j = tid & 15;           // lane within the half-warp
    const unsigned hmask = 0xFFFFu << (16 * ((tid & 31) >> 4));
    const int ntile = (K + 255) >> 8;
    float* my_tr = tr + hw * (16 * 17);

    for (int t = hw; t < nrows * ntile; t += 16) {
        const int r = t / ntile;
        const int tile = t - r * ntile;
        const int kbase = tile * 256;
        const int valid_rows = min(16, (K - kbase) >> 4);      // rows a of this tile inside K
        const T* src = x + static_cast<size_t>(row0 + r) * K + kbase;
        T* dst = rowbuf + static_cast<size_t>(r) * K + kbase;
        float v[16];
        if (j < valid_rows) load16<T>(src + 16 * j, v);
        else {
            #pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0.0f;
        }
        float m = 0.0f;
        if constexpr (G == 1) {
            if (j < valid_rows) {
                #pragma unroll
                for (int b = 0; b < 16; ++b) {
                    m = fmaxf(m, fabsf(v[b]));
                    dst[16 * j + b] = Act<T>::from_f32(v[b]);
                }
            }
        } else {
            h16(v);                                      // along b
            #pragma unroll
            for (int b = 0; b < 16; ++b) my_tr[j * 17 + b] = v[b];
            __syncwarp(hmask);
            float w[16];
            #pragma unroll
            for (int a = 0; a < 16; ++a) w[a] = my_tr[a * 17 + j];
            __syncwarp(hmask);
            if constexpr (G == 256) h16(w);              // along a
            else if constexpr (G == 64) h4_low_digit(w); // along a0 only (groups of 4 rows)
            constexpr float kNorm = (G == 256) ? 0.0625f : (G == 64) ? 0.125f : 0.25f;
            #pragma unroll
            for (int a = 0; a < 16; ++a) {
                if (a < valid_rows) {
                    const float y = Act<T>::round(__fmul_rn(w[a], kNorm));
                    m = fmaxf(m, fabsf(y));
                    dst[16 * a + j] = Act<T>::from_f32(y);
                }
            }
        }
        #pragma unroll
        for (int off = 8; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(hmask, m, off));
        if (j == 0) atomicMax(&rowmax[r], __float_as_uint(m));
    }
    __syncthreads();

    for (int r = tid; r < nrows; r += kQuantThreads) {
        const float amax = fmaxf(__uint_as_float(rowmax[r]), Act<T>::floor_value());
        const float s = Act<T>::round(__fdiv_rn(amax, 7.0f));
        row_scale[r] = s;
        row_rcp[r] = __frcp_rn(s);
        scaleout[row0 + r] = s;
    }
    __syncthreads();

    const int steps_per_row = K >> 4;
    for (int c = tid; c < nrows * steps_per_row; c += kQuantThreads) {
        const int r = c / steps_per_row;
        const int k0 = (c - r * steps_per_row) << 4;
        const T* src = rowbuf + static_cast<size_t>(r) * K + k0;
        const float s = row_scale[r];
        const float rcp = row_rcp[r];
        uint32_t packed[2] = {0u, 0u};
        #pragma unroll
        for (int i = 0; i < 16; ++i) {
            const float y = Act<T>::to_f32(src[i]);
            float tq;
            if constexpr (Act<T>::kCode == 1) {
                // For bf16 y and s, bf16(fp32(y * fp32(1/s))) == bf16(fp32(y / s)).
                tq = Act<T>::round(__fmul_rn(y, rcp));
            } else {
                tq = Act<T>::round(__fdiv_rn(y, s));
            }
            float qf = rintf(tq);
            qf = fminf(fmaxf(qf, -7.0f), 7.0f);
            const uint32_t nib = static_cast<uint32_t>(static_cast<int>(qf)) & 0xFu;
            packed[i >> 3] |= nib << (4 * (i & 7));
        }
        uint2* out = reinterpret_cast<uint2*>(qout + static_cast<size_t>(row0 + r) * (K >> 1) + (k0 >> 1));
        *out = make_uint2(packed[0], packed[1]);
    }
}

// ===========================================================================
// (2) int4 x int4 GEMM on tcgen05 (kind::i8, int32 accumulators in TMEM)
// ===========================================================================

constexpr int kBM = 128;                 // MMA M (accumulator lanes)
constexpr int kBKP = 64;                 // packed bytes of K per stage (128 codes)
constexpr int kSwizzle64 = 4;            // tcgen05 descriptor code for 64-byte swizzle
constexpr int kExpWarps = 8;             // expander / epilogue warps
constexpr int kGemmThreads = (4 + kExpWarps) * 32;

enum : int { kOutF32 = 0, kOutBF16 = 1, kOutF32Accumulate = 2, kOutS32 = 3 };

template <int BN>
struct GemmCfg {
    static constexpr int kStageBytes = 2 * (kBM + BN) * kBKP;        // packed/high + low halves
    static constexpr int kStages = (BN == 256) ? 4 : 6;
    static constexpr int kHalfBytes = (kBM + BN) * kBKP;               // one half (A then B)
    static constexpr int kTxBytes = (kBM + BN) * kBKP;                 // TMA bytes per stage
    static constexpr int kBarOffset = kStages * kStageBytes;
    // barriers: full, expanded, empty per stage + accumulator-ready
    static constexpr int kNumBars = 3 * kStages + 1;
    static constexpr int kMiscOffset = kBarOffset + kNumBars * 8;
    // tmem slot (16 B) + ws/bias tiles
    static constexpr int kWsOffset = kMiscOffset + 16;
    static constexpr int kBiasOffset = kWsOffset + BN * 4;
    static constexpr int kSmemBytes = kBiasOffset + BN * 4 + 1024;    // + alignment slack
    static constexpr uint32_t kIdesc = idesc_i8(kBM, BN);
};

template <int BN, int OUT>
__global__ void __launch_bounds__(kGemmThreads, 1)
int4_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                 const float* __restrict__ xscale, const float* __restrict__ wscale,
                 const float* __restrict__ bias, void* __restrict__ out, int M, int N, int K) {
    using Cfg = GemmCfg<BN>;
    extern __shared__ __align__(1024) unsigned char gsmem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(gsmem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOffset);
    uint64_t* full_bar = bars;
    uint64_t* exp_bar = bars + Cfg::kStages;
    uint64_t* empty_bar = bars + 2 * Cfg::kStages;
    uint64_t* accum_bar = bars + 3 * Cfg::kStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::kMiscOffset);
    float* ws_tile = reinterpret_cast<float*>(smem + Cfg::kWsOffset);
    float* bias_tile = reinterpret_cast<float*>(smem + Cfg::kBiasOffset);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN;
    const int m0 = blockIdx.y * kBM;
    const int num_kt = ((K >> 1) + kBKP - 1) / kBKP;

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::kStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&exp_bar[s], kExpWarps * 32);
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(accum_bar, 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmap_x);
        tma_prefetch_desc(&tmap_w);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, BN);
        tmem_relinquish();
    }
    if (warp >= 4 && OUT != kOutS32) {
        for (int c = threadIdx.x - 128; c < BN; c += kExpWarps * 32) {
            const int n = n0 + c;
            ws_tile[c] = (n < N) ? wscale[n] : 0.0f;
            bias_tile[c] = (bias != nullptr && n < N) ? bias[n] : 0.0f;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer
            for (int kt = 0; kt < num_kt; ++kt) {
                const int s = kt % Cfg::kStages;
                const uint32_t ph = (kt / Cfg::kStages) & 1;
                if (!mbar_wait_bounded(&empty_bar[s], ph ^ 1)) { record_status(kStatusTimeoutProducer); break; }
                unsigned char* st = smem + s * Cfg::kStageBytes;
                mbar_arrive_expect_tx(&full_bar[s], Cfg::kTxBytes);
                tma_load_2d(st, &tmap_x, &full_bar[s], kt * kBKP, m0);
                tma_load_2d(st + kBM * kBKP, &tmap_w, &full_bar[s], kt * kBKP, n0);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer
            for (int kt = 0; kt < num_kt; ++kt) {
                const int s = kt % Cfg::kStages;
                const uint32_t ph = (kt / Cfg::kStages) & 1;
                if (!mbar_wait_bounded(&exp_bar[s], ph)) { record_status(kStatusTimeoutMma); break; }
                tc_fence_after();
                const uint32_t hi_base = smem_u32(smem + s * Cfg::kStageBytes);
                const uint32_t lo_base = hi_base + Cfg::kHalfBytes;
                #pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const uint32_t a_base = half == 0 ? hi_base : lo_base;
                    const uint32_t b_base = a_base + kBM * kBKP;
                    #pragma unroll
                    for (int ks = 0; ks < kBKP / 32; ++ks) {
                        const uint64_t ad = smem_desc_kmajor(a_base + ks * 32, 8 * kBKP, kSwizzle64);
                        const uint64_t bd = smem_desc_kmajor(b_base + ks * 32, 8 * kBKP, kSwizzle64);
                        mma_i8_ss(tmem_base, ad, bd, Cfg::kIdesc, (kt | half | ks) != 0);
                    }
                }
                mma_commit(&empty_bar[s]);
            }
            mma_commit(accum_bar);
        }
    } else if (warp >= 4) {
        // ---------------- expanders: packed byte -> (b & 0xF0, b << 4), 16 B at a time
        const int et = threadIdx.x - 128;
        bool ok = true;
        for (int kt = 0; kt < num_kt; ++kt) {
            const int s = kt % Cfg::kStages;
            const uint32_t ph = (kt / Cfg::kStages) & 1;
            if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(&full_bar[s], ph))) {
                record_status(kStatusTimeoutExpand);
                ok = false;
                break;
            }
            uint4* hi = reinterpret_cast<uint4*>(smem + s * Cfg::kStageBytes);
            uint4* lo = reinterpret_cast<uint4*>(smem + s * Cfg::kStageBytes + Cfg::kHalfBytes);
            #pragma unroll 2
            for (int c = et; c < Cfg::kHalfBytes / 16; c += kExpWarps * 32) {
                const uint4 v = hi[c];
                uint4 h, l;
                h.x = v.x & 0xF0F0F0F0u; l.x = (v.x << 4) & 0xF0F0F0F0u;
                h.y = v.y & 0xF0F0F0F0u; l.y = (v.y << 4) & 0xF0F0F0F0u;
                h.z = v.z & 0xF0F0F0F0u; l.z = (v.z << 4) & 0xF0F0F0F0u;
                h.w = v.w & 0xF0F0F0F0u; l.w = (v.w << 4) & 0xF0F0F0F0u;
                hi[c] = h;
                lo[c] = l;
            }
            fence_proxy_async_smem();
            mbar_arrive(&exp_bar[s]);
        }

        // ---------------- epilogue: TMEM -> registers -> global
        // Warp-uniform outcome: the TMEM loads below are warp-collective.
        ok = __all_sync(0xFFFFFFFFu, ok && mbar_wait_bounded(accum_bar, 0));
        if (!ok && lane == 0) record_status(kStatusTimeoutEpilogue);
        tc_fence_after();
        const int quarter = warp & 3;
        const int col_half = (warp - 4) >> 2;
        const int row = m0 + quarter * 32 + lane;
        const float xs = (ok && row < M && OUT != kOutS32) ? xscale[row] : 0.0f;
        #pragma unroll 1
        for (int cc = 0; cc < BN / 64; ++cc) {
            const int col0 = col_half * (BN / 2) + cc * 32;
            uint32_t r[32];
            __syncwarp();                                // tcgen05.ld is warp-collective
            tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + col0, r);
            tmem_ld_wait();
            if (!ok || row >= M) continue;
            const int n = n0 + col0;
            const size_t obase = static_cast<size_t>(row) * N + n;
            const bool full = (n + 32 <= N);
            if constexpr (OUT == kOutS32) {
                int32_t* o = reinterpret_cast<int32_t*>(out) + obase;
                #pragma unroll
                for (int i = 0; i < 32; ++i)
                    if (full || n + i < N) o[i] = static_cast<int32_t>(r[i]) >> 8;
            } else {
                float v[32];
                #pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float d = static_cast<float>(static_cast<int32_t>(r[i]) >> 8);
                    v[i] = __fmul_rn(__fmul_rn(d, xs), ws_tile[col0 + i]);
                }
                if constexpr (OUT == kOutBF16) {
                    #pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = __fadd_rn(v[i], bias_tile[col0 + i]);
                    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out) + obase;
                    if (full && (N & 7) == 0) {
                        #pragma unroll
                        for (int i = 0; i < 32; i += 8) {
                            uint4 pk;
                            __nv_bfloat162 p0 = __floats2bfloat162_rn(v[i], v[i + 1]);
                            __nv_bfloat162 p1 = __floats2bfloat162_rn(v[i + 2], v[i + 3]);
                            __nv_bfloat162 p2 = __floats2bfloat162_rn(v[i + 4], v[i + 5]);
                            __nv_bfloat162 p3 = __floats2bfloat162_rn(v[i + 6], v[i + 7]);
                            memcpy(&pk.x, &p0, 4); memcpy(&pk.y, &p1, 4);
                            memcpy(&pk.z, &p2, 4); memcpy(&pk.w, &p3, 4);
                            *reinterpret_cast<uint4*>(o + i) = pk;
                        }
                    } else {
                        #pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (n + i < N) o[i] = __float2bfloat16_rn(v[i]);
                    }
                } else if constexpr (OUT == kOutF32) {
                    #pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = __fadd_rn(v[i], bias_tile[col0 + i]);
                    float* o = reinterpret_cast<float*>(out) + obase;
                    if (full && (N & 3) == 0) {
                        #pragma unroll
                        for (int i = 0; i < 32; i += 4)
                            *reinterpret_cast<float4*>(o + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
                    } else {
                        #pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (n + i < N) o[i] = v[i];
                    }
                } else {  // kOutF32Accumulate: out += ((D * xs) * ws), no bias
                    float* o = reinterpret_cast<float*>(out) + obase;
                    #pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (full || n + i < N) o[i] = __fadd_rn(o[i], v[i]);
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, BN);
    }
}

}  // namespace convrot

#include "gemm_pair.cuh"

namespace convrot {

// ===========================================================================
// Host side
// ===========================================================================

thread_local char g_last_error[256] = "";

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

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

// Packed int4 matrix [rows, K/2] bytes, box [box_rows, box_bytes]; 64- or
// 128-byte swizzle to match box_bytes.
bool make_packed_tmap(CUtensorMap* map, const void* base, int rows, int K, int box_rows, int box_bytes = kBKP) {
    auto enc = get_encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K / 2), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K / 2)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_bytes), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE,
                     box_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <typename KernelT>
cudaError_t ensure_smem(KernelT kernel, int bytes) {
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

template <int BN, int OUT>
int launch_gemm(const void* Xp, const void* Wp, const float* xs, const float* ws, const float* bias,
                void* out, int M, int N, int K, cudaStream_t stream) {
    CUtensorMap tx, tw;
    if (!make_packed_tmap(&tx, Xp, M, K, kBM) || !make_packed_tmap(&tw, Wp, N, K, BN))
        return fail("cuTensorMapEncodeTiled failed (pointer not 16-byte aligned or driver entry point missing)");
    auto kernel = int4_gemm_kernel<BN, OUT>;
    cudaError_t e = ensure_smem(kernel, GemmCfg<BN>::kSmemBytes);
    if (e != cudaSuccess) return static_cast<int>(e);
    dim3 grid((N + BN - 1) / BN, (M + kBM - 1) / kBM);
    kernel<<<grid, kGemmThreads, GemmCfg<BN>::kSmemBytes, stream>>>(tx, tw, xs, ws, bias, out, M, N, K);
    return static_cast<int>(cudaGetLastError());
}

int sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 2) return 148;
    return n;
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

template <int BN, bool SWAP, int OUT, bool STAGED>
int launch_pair_impl(const void* Xp, const void* Wp, const float* xs, const float* ws, const float* bias,
                     void* out, int M, int N, int K, cudaStream_t stream) {
    using Cfg = PairCfg<BN, STAGED>;
    const void* a_ptr = SWAP ? Wp : Xp;
    const void* b_ptr = SWAP ? Xp : Wp;
    const int rows_a = SWAP ? N : M;
    const int rows_b = SWAP ? M : N;
    CUtensorMap ta, tb, to;
    memset(&to, 0, sizeof(to));
    if (!make_packed_tmap(&ta, a_ptr, rows_a, K, 128, kPairBKP) ||
        !make_packed_tmap(&tb, b_ptr, rows_b, K, BN / 2, kPairBKP))
        return fail("cuTensorMapEncodeTiled failed (pointer not 16-byte aligned or driver entry point missing)");
    if (STAGED && !make_out_tmap(&to, out, M, N))
        return fail("cuTensorMapEncodeTiled failed for the output");
    auto kernel = int4_gemm_pair_kernel<BN, SWAP, OUT, STAGED>;
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
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kernel, ta, tb, to, xs, ws, bias, out, M, N, K, tiles_a,
                           static_cast<int>(num_tiles));
    if (e != cudaSuccess) return static_cast<int>(e);
    return static_cast<int>(cudaGetLastError());
}

template <int BN, bool SWAP, int OUT>
int launch_pair(const void* Xp, const void* Wp, const float* xs, const float* ws, const float* bias,
                void* out, int M, int N, int K, cudaStream_t stream) {
    if constexpr (OUT == kOutBF16 && !SWAP) {
        if ((N % 8) == 0 && aligned16(out))
            return launch_pair_impl<BN, SWAP, OUT, true>(Xp, Wp, xs, ws, bias, out, M, N, K, stream);
    }
    return launch_pair_impl<BN, SWAP, OUT, false>(Xp, Wp, xs, ws, bias, out, M, N, K, stream);
}

bool force_single_cta_kernel() {
    static const bool force = [] {
        const char* v = getenv("CONVROT_GEMM_SINGLE_CTA");
        return v != nullptr && v[0] == '1';
    }();
    return force;
}

template <int OUT>
int dispatch_gemm(const void* Xp, const void* Wp, const float* xs, const float* ws, const float* bias,
                  void* out, int M, int N, int K, cudaStream_t stream) {
    if (force_single_cta_kernel()) {
        const long tiles256 = static_cast<long>((M + kBM - 1) / kBM) * ((N + 255) / 256);
        if (N > 128 && tiles256 >= 148)
            return launch_gemm<256, OUT>(Xp, Wp, xs, ws, bias, out, M, N, K, stream);
        return launch_gemm<128, OUT>(Xp, Wp, xs, ws, bias, out, M, N, K, stream);
    }
    if (M <= 32) return launch_pair<32, true, OUT>(Xp, Wp, xs, ws, bias, out, M, N, K, stream);
    if (M <= 64) return launch_pair<64, true, OUT>(Xp, Wp, xs, ws, bias, out, M, N, K, stream);
    if (M <= 128) return launch_pair<128, true, OUT>(Xp, Wp, xs, ws, bias, out, M, N, K, stream);
    return launch_pair<256, false, OUT>(Xp, Wp, xs, ws, bias, out, M, N, K, stream);
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
    int rows = 48 / ntile;
    rows = rows < 1 ? 1 : (rows > 64 ? 64 : rows);
    if (rows > M) rows = M;
    const size_t head = ((kTransposeFloats + 3 * rows) * 4 + 15) & ~static_cast<size_t>(15);
    const size_t bytes = head + static_cast<size_t>(rows) * K * sizeof(T);
    if (bytes > 227 * 1024) return fail("row too long for the shared-memory row buffer");
    auto kernel = convrot_quant_kernel<T, G>;
    cudaError_t e = ensure_smem(kernel, static_cast<int>(bytes));
    if (e != cudaSuccess) return static_cast<int>(e);
    const int grid = (M + rows - 1) / rows;
    kernel<<<grid, kQuantThreads, bytes, stream>>>(static_cast<const T*>(x), static_cast<int8_t*>(q),
                                                  static_cast<float*>(s), M, K, rows);
    return static_cast<int>(cudaGetLastError());
}

template <int G>
int launch_quant_g(const void* x, int in_dtype, void* q, void* s, int M, int K, cudaStream_t stream) {
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
    const float* b = static_cast<const float*>(bias);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (out_dtype == 1) return dispatch_gemm<kOutBF16>(Xp, Wp, xs, ws, b, out, M, N, K, s);
    return dispatch_gemm<kOutF32>(Xp, Wp, xs, ws, b, out, M, N, K, s);
}

CONVROT_API int ck_int4_convrot_gemm_splitk(const void* Xp, const void* Wp, const void* xscale,
                                            const void* wscale, void* accum, int M, int N, int K,
                                            int nsplit, void* stream) {
    if (int rc = check_gemm_args(Xp, Wp, M, N, K)) return rc;
    if (nsplit < 1) return fail("nsplit must be >= 1");
    if (M == 0 || N == 0) return 0;
    if (!xscale || !wscale || !accum) return fail("null scale or accumulator pointer");
    return dispatch_gemm<kOutF32Accumulate>(Xp, Wp, static_cast<const float*>(xscale),
                                            static_cast<const float*>(wscale), nullptr, accum, M, N, K,
                                            static_cast<cudaStream_t>(stream));
}

CONVROT_API int ck_int4_gemm_s32(const void* Xp, const void* Wp, void* acc, int M, int N, int K, void* stream) {
    if (int rc = check_gemm_args(Xp, Wp, M, N, K)) return rc;
    if (M == 0 || N == 0) return 0;
    if (!acc) return fail("null accumulator pointer");
    return dispatch_gemm<kOutS32>(Xp, Wp, nullptr, nullptr, nullptr, acc, M, N, K,
                                  static_cast<cudaStream_t>(stream));
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
