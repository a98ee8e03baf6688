// Dynamic-LoRA down projection T = fp16(x) . A^T on the tensor cores.
//
// T [M, R] fp16 (R <= 64, the stacked adapter rank padded to a multiple of 8),
// x [M, K] bf16 or fp16, A [R, K] fp16 (the adapters' down matrices, the dtype
// the node prepares them in: int4_ops.py:165-167). Each product term is
// fp16(x) * A in exact fp32 (tcgen05.mma kind::f16, fp32 accumulator) and T is
// rounded to fp16 once, as an fp16 matmul with fp32 accumulation does.
//
// The kernel is bound by reading x once from HBM (2 M K bytes); the MMA work
// (2 M K 64 flops) is a few percent of the tensor-core rate. Per CTA: one
// 128-row M tile and a contiguous range of 64-column K stages.
//   w0      TMA producer (one lane): x tile [128 x 64] and A tile [64 x 64],
//           128-byte swizzle; rows of A beyond R and of x beyond M arrive as
//           zeros (out-of-bounds fill)
//   w1      TMEM allocation (64 columns) and the MMA issuer (one elected lane):
//           four M=128 N=64 K=16 MMAs a stage
//   w2..w5  bf16 x: convert each landed x tile to fp16 in place (same element
//           size, so the swizzled position of every element is unchanged);
//           then the epilogue (TMEM lanes 32 * (warp % 4) ..)
// Grids with few M tiles split K over a cluster of up to 8 CTAs: each CTA
// leaves its fp32 partial in its own shared memory and CTA 0 of the cluster
// sums the partials in rank order (deterministic) through distributed shared
// memory before the single fp16 rounding.
#pragma once

namespace convrot {

constexpr int kLdRows = 128;                 // x rows per tile (TMEM lanes)
constexpr int kLdBK = 64;                    // K columns per stage (one 128-byte swizzle row)
constexpr int kLdN = 64;                     // MMA N: maximum rank
constexpr int kLdXBytes = kLdRows * kLdBK * 2;
constexpr int kLdABytes = kLdN * kLdBK * 2;
constexpr int kLdStageBytes = kLdXBytes + kLdABytes;
constexpr int kLdStages = 8;
constexpr int kLdThreads = 192;
constexpr int kLdRedBytes = kLdRows * kLdN * 4;     // fp32 partial of a split-K CTA
constexpr int kLdBarOffset = kLdStages * kLdStageBytes;
constexpr int kLdSmemBytes = kLdBarOffset + (3 * kLdStages + 1) * 8 + 16 + 1024;
static_assert(kLdRedBytes <= kLdBarOffset, "the split-K partial reuses the operand ring");
static_assert(kLdSmemBytes <= 227 * 1024, "shared memory budget");

// Two bf16 (low half first) -> two fp16, each widened exactly and rounded to
// nearest even: the result of a bf16 -> fp16 cast.
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t u) {
    const __half2 h = __floats2half2_rn(__uint_as_float(u << 16), __uint_as_float(u & 0xFFFF0000u));
    uint32_t r;
    memcpy(&r, &h, 4);
    return r;
}

// Eight fp32 (bit patterns) -> eight fp16, round to nearest even, as one 16-byte word.
__device__ __forceinline__ uint4 pack_f16x8(const uint32_t* f) {
    uint32_t w[4];
    #pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 h = __floats2half2_rn(__uint_as_float(f[2 * i]), __uint_as_float(f[2 * i + 1]));
        memcpy(&w[i], &h, 4);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

template <bool kConvert>
__global__ void __launch_bounds__(kLdThreads, 1)
lora_down_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_a,
                 __half* __restrict__ t_out, int M, int K, int R, int ksplit) {
    extern __shared__ __align__(1024) unsigned char ld_smem_raw[];
    unsigned char* smem = ld_smem_raw + ((1024u - (smem_u32(ld_smem_raw) & 1023u)) & 1023u);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kLdBarOffset);
    uint64_t* full_bar = bars;                        // TMA landed
    uint64_t* conv_bar = full_bar + kLdStages;        // x tile converted to fp16
    uint64_t* empty_bar = conv_bar + kLdStages;       // MMAs done with the slot
    uint64_t* acc_bar = empty_bar + kLdStages;        // accumulator complete
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_bar + 1);
    float* red = reinterpret_cast<float*>(smem);      // split-K partial, after the last MMA

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int kpart = static_cast<int>(blockIdx.x) % ksplit;
    const int mtile = static_cast<int>(blockIdx.x) / ksplit;
    const int num_kt = (K + kLdBK - 1) / kLdBK;
    const int kt0 = static_cast<int>((static_cast<long>(num_kt) * kpart) / ksplit);
    const int kt1 = static_cast<int>((static_cast<long>(num_kt) * (kpart + 1)) / ksplit);
    const int nkt = kt1 - kt0;                        // >= 1: the host keeps ksplit <= num_kt
    const int m0 = mtile * kLdRows;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kLdStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&conv_bar[s], 4);
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(acc_bar, 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmap_x);
        tma_prefetch_desc(&tmap_a);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kLdN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    griddep_wait();                                   // x may be the previous kernel's output
    griddep_launch_dependents();
    const uint32_t tmem_acc = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- producer
            for (int i = 0; i < nkt; ++i) {
                const int s = i % kLdStages;
                if (!mbar_wait_bounded(&empty_bar[s], ((i / kLdStages) & 1) ^ 1)) {
                    record_status(kStatusTimeoutProducer);
                    break;
                }
                unsigned char* st = smem + s * kLdStageBytes;
                mbar_arrive_expect_tx(&full_bar[s], kLdStageBytes);
                tma_load_2d(st, &tmap_x, &full_bar[s], (kt0 + i) * kLdBK, m0);
                tma_load_2d(st + kLdXBytes, &tmap_a, &full_bar[s], (kt0 + i) * kLdBK, 0);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer: D[128 x 64] += x[128 x 64] . A[64 x 64]^T per stage
        constexpr uint32_t kIdesc = idesc_f16(kLdRows, kLdN);
        for (int i = 0; i < nkt; ++i) {
            const int s = i % kLdStages;
            uint64_t* ready = kConvert ? &conv_bar[s] : &full_bar[s];
            if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(ready, (i / kLdStages) & 1))) {
                if (lane == 0) record_status(kStatusTimeoutMma);
                break;
            }
            tc_fence_after();
            const uint32_t st = smem_u32(smem + s * kLdStageBytes);
            const uint64_t ad = smem_desc_kmajor(st, 8 * 128, kSwizzle128);
            const uint64_t bd = smem_desc_kmajor(st + kLdXBytes, 8 * 128, kSwizzle128);
            if (elect_one()) {
                #pragma unroll
                for (int j = 0; j < kLdBK / 16; ++j)          // 32-byte K steps: +2 in the address field
                    mma_f16kind_ss(tmem_acc, ad + 2 * j, bd + 2 * j, kIdesc, (i | j) != 0);
                mma_commit(&empty_bar[s]);
            }
            __syncwarp();
        }
        if (elect_one()) mma_commit(acc_bar);
        __syncwarp();
    } else {
        const int ct = threadIdx.x - 64;                    // 0..127
        if constexpr (kConvert) {
            // ---------------- bf16 -> fp16 in place (round to nearest even, as a cast does)
            for (int i = 0; i < nkt; ++i) {
                const int s = i % kLdStages;
                if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(&full_bar[s], (i / kLdStages) & 1))) {
                    if (lane == 0) record_status(kStatusTimeoutExpand);
                    break;
                }
                uint4* xt = reinterpret_cast<uint4*>(smem + s * kLdStageBytes);
                #pragma unroll
                for (int c = 0; c < kLdXBytes / 16 / 128; ++c) {
                    uint4 v = xt[ct + 128 * c];
                    v.x = bf16x2_to_f16x2(v.x);
                    v.y = bf16x2_to_f16x2(v.y);
                    v.z = bf16x2_to_f16x2(v.z);
                    v.w = bf16x2_to_f16x2(v.w);
                    xt[ct + 128 * c] = v;
                }
                fence_proxy_async_smem();                   // generic writes before the MMA reads them
                __syncwarp();
                if (lane == 0) mbar_arrive(&conv_bar[s]);
            }
        }
        // ---------------- epilogue: TMEM lane r = row m0 + r of the tile
        const int q = warp & 3;
        const int r = q * 32 + lane;
        if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(acc_bar, 0)) && lane == 0)
            record_status(kStatusTimeoutEpilogue);
        tc_fence_after();
        uint32_t a0[32], a1[32];
        const uint32_t taddr = tmem_acc + (static_cast<uint32_t>(q * 32) << 16);
        tmem_ld_32x32b_x32(taddr, a0);
        tmem_ld_32x32b_x32(taddr + 32, a1);
        tmem_ld_wait_regs(a0);
        tmem_ld_wait_regs(a1);
        if (ksplit == 1) {
            const int m = m0 + r;
            if (m < M) {
                uint4* row = reinterpret_cast<uint4*>(t_out + static_cast<size_t>(m) * R);
                #pragma unroll
                for (int c = 0; c < kLdN / 8; ++c) {
                    if (c < R / 8) {
                        const uint32_t* src = c < 4 ? a0 + 8 * c : a1 + 8 * (c - 4);
                        row[c] = pack_f16x8(src);
                    }
                }
            }
        } else {
            // fp32 partial into this CTA's shared memory (the ring is idle: every
            // load was consumed before the accumulator completed); 16-byte chunks
            // XOR-swizzled by row so a warp's stores spread over the banks
            float4* rrow = reinterpret_cast<float4*>(red + r * kLdN);
            #pragma unroll
            for (int c = 0; c < kLdN / 4; ++c) {
                const uint32_t* src = c < 8 ? a0 + 4 * c : a1 + 4 * (c - 8);
                rrow[c ^ (r & 15)] = make_float4(__uint_as_float(src[0]), __uint_as_float(src[1]),
                                                 __uint_as_float(src[2]), __uint_as_float(src[3]));
            }
        }
    }

    if (ksplit > 1) {
        __syncwarp();
        cluster_sync();                                    // every partial written
        if (kpart == 0 && warp >= 2) {
            const int r = (warp & 3) * 32 + lane;
            const int m = m0 + r;
            if (m < M) {
                const uint32_t rrow = smem_u32(red + r * kLdN);
                uint4* row = reinterpret_cast<uint4*>(t_out + static_cast<size_t>(m) * R);
                #pragma unroll 1
                for (int c = 0; c < R / 8; ++c) {
                    float4 lo = make_float4(0.f, 0.f, 0.f, 0.f), hi = lo;
                    for (int p = 0; p < ksplit; ++p) {       // rank order: a fixed summation order
                        const float4 u = ld_shared_cluster_f4(mapa_shared(rrow + (((2 * c) ^ (r & 15)) << 4), p));
                        const float4 v = ld_shared_cluster_f4(mapa_shared(rrow + (((2 * c + 1) ^ (r & 15)) << 4), p));
                        if (p == 0) { lo = u; hi = v; continue; }
                        lo = make_float4(lo.x + u.x, lo.y + u.y, lo.z + u.z, lo.w + u.w);
                        hi = make_float4(hi.x + v.x, hi.y + v.y, hi.z + v.z, hi.w + v.w);
                    }
                    const uint32_t f[8] = {__float_as_uint(lo.x), __float_as_uint(lo.y), __float_as_uint(lo.z),
                                           __float_as_uint(lo.w), __float_as_uint(hi.x), __float_as_uint(hi.y),
                                           __float_as_uint(hi.z), __float_as_uint(hi.w)};
                    row[c] = pack_f16x8(f);
                }
            }
        }
        __syncwarp();
        cluster_sync();                                    // no CTA leaves while CTA 0 reads its partial
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_acc, kLdN);
    }
}

}  // namespace convrot
