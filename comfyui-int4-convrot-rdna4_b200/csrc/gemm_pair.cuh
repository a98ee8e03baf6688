// int4 x int4 GEMM on CTA pairs (tcgen05.mma.cta_group::2.kind::i8, A from TMEM).
//
// Included by convrot_b200.cu. Operand roles:
//   A: 256 rows per CTA pair (128 per CTA), expanded by warps straight into
//      tensor memory (tcgen05.st) -- no shared-memory round trip;
//   B: BN rows per pair, BN/2 in each CTA's shared memory, expanded in place
//      (high nibbles) plus a second buffer (low nibbles);
//   D: int32 [128 lanes x BN columns] in each CTA's TMEM.
// Normally A = activations (rows m) and B = weights (rows n). With SWAP the
// weights are A and the activations B, which keeps the big operand off shared
// memory when M is small (weight-bound layers).
//
// Byte split: a packed byte b holds codes (lo, hi). (b & 0xF0) is the int8
// value 16*hi and (b << 4) & 0xF0 is 16*lo, so the MMA over both halves sums
// 256 * (lo_x*lo_w + hi_x*hi_w): the accumulator is 256 * D exactly
// (|256 * D| <= 256 * 64 * 65536 < 2^31).
//
// Warp roles (12 warps, both CTAs alike):
//   w0        TMA producer (one lane): packed A and B-half tiles per k-stage
//   w1        TMEM allocation; in the even CTA, one lane issues the MMAs
//   w2, w3    odd CTA only: forward "stage expanded" to the even CTA, one
//             cluster-scope release per stage, alternating stages
//   w4..w7    A expanders (row = 32*(w%4) + lane), then epilogue
//   w8..w11   B expanders, then epilogue
//
// Stage hand-off: expander warps arrive with CTA-scope release on a local
// barrier (the MMA's own barrier in the even CTA, a forwarding barrier in the
// odd one). A cluster-scope release costs a memory-barrier round trip, so the
// odd CTA pays it once per stage in a forwarding warp, off the expanders' path;
// two forwarding warps keep two of them in flight.
#pragma once

namespace convrot {

constexpr int kPairThreads = 12 * 32;
constexpr uint32_t kTmemCols = 512;

template <int BN>
struct PairCfg {
    static constexpr int kBHalf = BN / 2;
    static constexpr int kABytes = 128 * kBKP;
    static constexpr int kBBytes = kBHalf * kBKP;
    static constexpr int kStageBytes = kABytes + 2 * kBBytes;
    static constexpr int kTmemStageCols = 2 * kBKP / 4;          // hi + lo bytes of a row, 4 per column
    static constexpr int kStagesByTmem = (static_cast<int>(kTmemCols) - BN) / kTmemStageCols;
    static constexpr int kStagesBySmem = (192 * 1024) / kStageBytes;
    static constexpr int kStages0 = kStagesByTmem < kStagesBySmem ? kStagesByTmem : kStagesBySmem;
    static constexpr int kStages = kStages0 < 16 ? kStages0 : 16;
    static constexpr int kBarOffset = kStages * kStageBytes;
    static constexpr int kNumBars = 4 * kStages + 1;
    static constexpr int kMiscOffset = kBarOffset + kNumBars * 8;
    static constexpr int kColScaleOffset = kMiscOffset + 16;
    static constexpr int kColBiasOffset = kColScaleOffset + BN * 4;
    static constexpr int kSmemBytes = kColBiasOffset + BN * 4 + 1024;
    static constexpr uint32_t kIdesc = idesc_i8(256, BN);
    static constexpr int kLocalArrivals = 8;                       // expander warps per CTA
    static constexpr int kReadyCount = kLocalArrivals + 1;         // + the odd CTA's forwarder
    static_assert(BN >= 32 && BN <= 256 && BN % 32 == 0, "pair MMA N must be a multiple of 32 in [32, 256]");
    static_assert(kStages >= 2, "pipeline needs at least two stages");
};

// Dequantize and store 32 consecutive outputs of one output row (non-swapped
// layout). v[] holds ((D * xs) * ws) already; bias is added here.
template <int OUT>
__device__ __forceinline__ void store_row32(void* out, size_t obase, int n, int N, float (&v)[32],
                                            const float* bias_cols) {
    const bool full = (n + 32 <= N);
    if constexpr (OUT == kOutBF16) {
        #pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __fadd_rn(v[i], bias_cols[i]);
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
        for (int i = 0; i < 32; ++i) v[i] = __fadd_rn(v[i], bias_cols[i]);
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
    } else if constexpr (OUT == kOutF32Accumulate) {
        float* o = reinterpret_cast<float*>(out) + obase;
        #pragma unroll
        for (int i = 0; i < 32; ++i)
            if (full || n + i < N) o[i] = __fadd_rn(o[i], v[i]);
    }
}

template <int BN, bool SWAP, int OUT>
__global__ void __launch_bounds__(kPairThreads, 1)
int4_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                      const float* __restrict__ xscale, const float* __restrict__ wscale,
                      const float* __restrict__ bias, void* __restrict__ out, int M, int N, int K) {
    using Cfg = PairCfg<BN>;
    extern __shared__ __align__(1024) unsigned char psmem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(psmem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOffset);
    uint64_t* full_bar = bars;
    uint64_t* ready_bar = bars + Cfg::kStages;
    uint64_t* empty_bar = bars + 2 * Cfg::kStages;
    uint64_t* fwd_bar = bars + 3 * Cfg::kStages;
    uint64_t* accum_bar = bars + 4 * Cfg::kStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::kMiscOffset);
    float* col_scale = reinterpret_cast<float*>(smem + Cfg::kColScaleOffset);
    float* col_bias = reinterpret_cast<float*>(smem + Cfg::kColBiasOffset);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t cta = cluster_ctarank();
    const int a_row0 = (blockIdx.x >> 1) * 256 + static_cast<int>(cta) * 128;
    const int b_tile0 = blockIdx.y * BN;
    const int b_row0 = b_tile0 + static_cast<int>(cta) * Cfg::kBHalf;
    const int num_kt = ((K >> 1) + kBKP - 1) / kBKP;
    const int rows_b = SWAP ? M : N;

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::kStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&ready_bar[s], Cfg::kReadyCount);
            mbar_init(&empty_bar[s], 1);
            mbar_init(&fwd_bar[s], Cfg::kLocalArrivals);
        }
        mbar_init(accum_bar, 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmap_a);
        tma_prefetch_desc(&tmap_b);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, kTmemCols);
        tmem_relinquish_pair();
    }
    if (warp >= 4 && OUT != kOutS32) {
        // per-column factors of the output tile: B rows are output columns (n)
        // normally, tokens (m) when swapped
        for (int c = threadIdx.x - 128; c < BN; c += 256) {
            const int r = b_tile0 + c;
            if constexpr (SWAP) {
                col_scale[c] = (r < rows_b) ? xscale[r] : 0.0f;
                col_bias[c] = 0.0f;
            } else {
                col_scale[c] = (r < rows_b) ? wscale[r] : 0.0f;
                col_bias[c] = (bias != nullptr && r < rows_b) ? bias[r] : 0.0f;
            }
        }
    }
    tc_fence_before();
    cluster_sync();                       // peer barriers initialised before any remote arrive
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t tmem_a0 = tmem_base + BN;  // A stages follow the accumulator columns

    if (warp == 0) {
        if (lane == 0) {
            for (int kt = 0; kt < num_kt; ++kt) {
                const int s = kt % Cfg::kStages;
                const uint32_t ph = (kt / Cfg::kStages) & 1;
                if (!mbar_wait_bounded<true>(&empty_bar[s], ph ^ 1)) { record_status(kStatusTimeoutProducer); break; }
                unsigned char* st = smem + s * Cfg::kStageBytes;
                mbar_arrive_expect_tx(&full_bar[s], Cfg::kABytes + Cfg::kBBytes);
                tma_load_2d(st, &tmap_a, &full_bar[s], kt * kBKP, a_row0);
                tma_load_2d(st + Cfg::kABytes, &tmap_b, &full_bar[s], kt * kBKP, b_row0);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && cta == 0) {
            for (int kt = 0; kt < num_kt; ++kt) {
                const int s = kt % Cfg::kStages;
                const uint32_t ph = (kt / Cfg::kStages) & 1;
                if (!mbar_wait_bounded<true>(&ready_bar[s], ph)) { record_status(kStatusTimeoutMma); break; }
                tc_fence_after();
                const uint32_t b_hi = smem_u32(smem + s * Cfg::kStageBytes + Cfg::kABytes);
                #pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t b_addr = b_hi + (j >> 1) * Cfg::kBBytes + (j & 1) * 32;
                    const uint64_t bd = smem_desc_kmajor(b_addr, 8 * kBKP, kSwizzle64);
                    mma_i8_ts_pair(tmem_base, tmem_a0 + s * Cfg::kTmemStageCols + j * 8, bd, Cfg::kIdesc,
                                   (kt | j) != 0);
                }
                mma_commit_pair_multicast(&empty_bar[s], 0x3);
            }
            mma_commit_pair_multicast(accum_bar, 0x3);
        }
    } else if (warp < 4) {
        if (cta == 1 && lane == 0) {
            // ---------------- forwarders (odd CTA): local expansion done -> even CTA's MMA barrier
            const uint32_t ready_leader0 = mapa_shared(smem_u32(&ready_bar[0]), 0);
            for (int kt = warp - 2; kt < num_kt; kt += 2) {
                const int s = kt % Cfg::kStages;
                const uint32_t ph = (kt / Cfg::kStages) & 1;
                if (!mbar_wait_bounded(&fwd_bar[s], ph)) { record_status(kStatusTimeoutExpand); break; }
                mbar_arrive_cluster(ready_leader0 + s * 8);
            }
        }
    } else {
        // expansion done for stage s: local arrive (CTA-scope release)
        uint64_t* done_bar = (cta == 0) ? ready_bar : fwd_bar;
        const int quarter = warp & 3;
        bool ok = true;
        if (warp < 8) {
            // ---------------- A expanders: one row per thread, into TMEM
            const int r = quarter * 32 + lane;
            const uint32_t swz = static_cast<uint32_t>((r >> 1) & 3);
            for (int kt = 0; kt < num_kt; ++kt) {
                const int s = kt % Cfg::kStages;
                const uint32_t ph = (kt / Cfg::kStages) & 1;
                if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(&full_bar[s], ph))) {
                    record_status(kStatusTimeoutExpand); ok = false; break;
                }
                const unsigned char* row = smem + s * Cfg::kStageBytes + r * kBKP;
                uint32_t w[32];
                #pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint4 v = *reinterpret_cast<const uint4*>(row + ((c ^ swz) << 4));
                    const uint32_t p[4] = {v.x, v.y, v.z, v.w};
                    #pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        w[4 * c + e] = p[e] & 0xF0F0F0F0u;
                        w[16 + 4 * c + e] = (p[e] << 4) & 0xF0F0F0F0u;
                    }
                }
                __syncwarp();
                tmem_st_32x32b_x32(tmem_a0 + (static_cast<uint32_t>(quarter * 32) << 16) + s * Cfg::kTmemStageCols, w);
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&done_bar[s]);
            }
        } else {
            // ---------------- B expanders: in place (high) + second buffer (low)
            const int et = threadIdx.x - 256;
            for (int kt = 0; kt < num_kt; ++kt) {
                const int s = kt % Cfg::kStages;
                const uint32_t ph = (kt / Cfg::kStages) & 1;
                if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(&full_bar[s], ph))) {
                    record_status(kStatusTimeoutExpand); ok = false; break;
                }
                uint4* hi = reinterpret_cast<uint4*>(smem + s * Cfg::kStageBytes + Cfg::kABytes);
                uint4* lo = reinterpret_cast<uint4*>(smem + s * Cfg::kStageBytes + Cfg::kABytes + Cfg::kBBytes);
                #pragma unroll
                for (int c = et; c < Cfg::kBBytes / 16; c += 128) {
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
                __syncwarp();
                if (lane == 0) mbar_arrive(&done_bar[s]);
            }
        }

        // ---------------- epilogue: this CTA's 128 accumulator lanes x BN columns
        ok = __all_sync(0xFFFFFFFFu, ok && mbar_wait_bounded<true>(accum_bar, 0));
        if (!ok && lane == 0) record_status(kStatusTimeoutEpilogue);
        tc_fence_after();
        constexpr bool kSplitCols = BN >= 64;
        constexpr int kColsPerWarp = kSplitCols ? BN / 2 : BN;
        const int col_half = (warp - 4) >> 2;
        if (kSplitCols || col_half == 0) {
            const int a = a_row0 + quarter * 32 + lane;          // A row of this lane
            const bool lane_ok = ok && a < (SWAP ? N : M);
            float lane_scale = 0.0f, lane_bias = 0.0f;
            if (lane_ok && OUT != kOutS32) {
                if constexpr (SWAP) {
                    lane_scale = wscale[a];
                    lane_bias = bias != nullptr ? bias[a] : 0.0f;
                } else {
                    lane_scale = xscale[a];
                }
            }
            #pragma unroll 1
            for (int cc = 0; cc < kColsPerWarp / 32; ++cc) {
                const int col0 = col_half * kColsPerWarp + cc * 32;
                uint32_t r[32];
                __syncwarp();
                tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + col0, r);
                tmem_ld_wait();
                if (!lane_ok) continue;
                const int b = b_tile0 + col0;                       // first B row of this chunk
                if constexpr (OUT == kOutS32) {
                    #pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const int32_t d = static_cast<int32_t>(r[i]) >> 8;
                        if constexpr (SWAP) {
                            if (b + i < M) reinterpret_cast<int32_t*>(out)[static_cast<size_t>(b + i) * N + a] = d;
                        } else {
                            if (b + i < N) reinterpret_cast<int32_t*>(out)[static_cast<size_t>(a) * N + b + i] = d;
                        }
                    }
                } else if constexpr (SWAP) {
                    #pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        if (b + i >= M) break;
                        const float d = static_cast<float>(static_cast<int32_t>(r[i]) >> 8);
                        const float v = __fmul_rn(__fmul_rn(d, col_scale[col0 + i]), lane_scale);
                        const size_t o = static_cast<size_t>(b + i) * N + a;
                        if constexpr (OUT == kOutBF16)
                            reinterpret_cast<__nv_bfloat16*>(out)[o] = __float2bfloat16_rn(__fadd_rn(v, lane_bias));
                        else if constexpr (OUT == kOutF32)
                            reinterpret_cast<float*>(out)[o] = __fadd_rn(v, lane_bias);
                        else
                            reinterpret_cast<float*>(out)[o] = __fadd_rn(reinterpret_cast<float*>(out)[o], v);
                    }
                } else {
                    float v[32];
                    #pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const float d = static_cast<float>(static_cast<int32_t>(r[i]) >> 8);
                        v[i] = __fmul_rn(__fmul_rn(d, lane_scale), col_scale[col0 + i]);
                    }
                    store_row32<OUT>(out, static_cast<size_t>(a) * N + b, b, N, v, col_bias + col0);
                }
            }
        }
    }

    tc_fence_before();
    cluster_sync();                       // no CTA leaves while its pair may still touch its TMEM
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, kTmemCols);
    }
}

}  // namespace convrot
