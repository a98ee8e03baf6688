// A8T form of the int4 GEMM: packed int4 weights as the MMA's A operand in
// tensor memory, int8 activation codes as the B operand in shared memory
// (tcgen05.mma.cta_group::2.kind::i8, A from TMEM), persistent over output tiles.
//
// Included by convrot_b200.cu after gemm_pair.cuh (shares its constants).
//
// Why this orientation: with both operands in shared memory (the A8 form) every
// k-stage writes and reads the activation tile and the expanded weight tile
// there, and shared-memory bandwidth bounds the MMA rate. Here only the
// activation codes and the packed weight bytes (half the expanded size) pass
// through shared memory; the expanded weights go from registers into TMEM
// (tcgen05.st), which the MMA reads directly.
//
// Per CTA pair and tile: 256 weight rows (128 per CTA, one per TMEM lane) x BN
// tokens (BN/2 per CTA); D[n, m] int32 in TMEM lanes n, columns m. Each k-stage
// covers 128 codes of K: 64 packed bytes a weight row (TMA, 64-byte swizzle)
// and 128 code bytes a token row (TMA pair load, 128-byte swizzle). A packed
// byte b (codes lo, hi) expands to the int8 pair (16*lo, 16*hi) in K order, so
// the accumulator is 16 * D (|16 * D| <= 16 * 56 * 65536 < 2^31).
//
// Warp roles (16 warps, both CTAs alike):
//   w0        activation producer (one lane): code tiles, pair loads completing
//             on the even CTA's barrier
//   w1        TMEM allocation; in the even CTA the MMA issuer (one elected lane)
//   w2        packed-weight producer (one lane): this CTA's 128 weight rows
//   w3        L2 prefetch of the first tile's weight rows
//   w4..w11   expanders: two groups of four warps take k-stages in turn; the
//             thread of TMEM lane r expands weight row r (64 packed bytes ->
//             32 TMEM columns)
//   w12..w15  epilogue (TMEM lanes 32*(w%4) ..): dequantize, add bias; bf16
//             output goes through per-warp [32 tokens x 32 weight rows] boxes in
//             shared memory (written transposed by stmatrix) and TMA stores
//             (STAGED), other outputs are stored directly
//
// The epilogue converts D = acc / 16 to float by the magic-number method
// (bits of 1.5 * 2^23 plus D, minus 1.5 * 2^23), exact for |D| < 2^22, which
// int4 codes guarantee for K <= 65536 (|D| <= 56 K).
#pragma once

namespace convrot {

#ifndef CONVROT_A8T_PSTAGES
#define CONVROT_A8T_PSTAGES 8
#endif

template <int BN, bool STAGED>
struct A8tCfg {
    static constexpr int kXHalf = BN / 2;                      // token rows per CTA and tile
    static constexpr int kXBytes = kXHalf * kPairBKP;          // activation stage: 128 codes of K a row
    static constexpr int kWRows = 128;                         // weight rows per CTA and tile
    static constexpr int kWRowBytes = 64;                      // packed bytes of a weight row per stage
    static constexpr int kWBytes = kWRows * kWRowBytes;        // packed-weight stage
    static constexpr int kPStages = CONVROT_A8T_PSTAGES;
    static constexpr int kGroups = 2;                          // expander groups (k-stages in turn)
    static constexpr int kGroupWarps = 4;                      // one warp per 32 TMEM lanes
    static constexpr int kStageCols = kPairBKP / 4;            // TMEM columns of an expanded stage
    // accumulators: two buffers when the expanded-weight ring still gets four stages
    static constexpr int kAccBufs = (2 * BN + 4 * kStageCols <= static_cast<int>(kTmemCols)) ? 2 : 1;
    static constexpr int kTmemFree = static_cast<int>(kTmemCols) - kAccBufs * BN;
    static constexpr int kTmemStages = kTmemFree / kStageCols >= 8 ? 8 : kTmemFree / kStageCols;
    static constexpr int kPRingBytes = kPStages * kWBytes;
    static constexpr int kBoxBytes = 32 * 32 * 2;                  // one staged bf16 output box (2 KB)
    static constexpr int kStagingBytes = STAGED ? 4 * 2 * kBoxBytes : 0;   // two boxes per epilogue warp
    static constexpr int kFixedBytes = 2048 + 2 * 2 * BN * 4 + 1024 + kStagingBytes;
    static constexpr int kStagesBySmem = (227 * 1024 - kFixedBytes - kPRingBytes) / kXBytes;
    static constexpr int kStages = kStagesBySmem < 16 ? kStagesBySmem : 16;
    static constexpr int kPOffset = kStages * kXBytes;
    static constexpr int kStagingOffset = kPOffset + kPRingBytes;
    static constexpr int kBarOffset = kStagingOffset + kStagingBytes;
    static constexpr int kNumBars = 2 * kStages + 2 * kPStages + 2 * kTmemStages + 4;
    static constexpr int kMiscOffset = kBarOffset + kNumBars * 8;
    static constexpr int kColOffset = kMiscOffset + 16;
    static constexpr int kSmemBytes = kColOffset + 2 * BN * 4 + 1024;
    static constexpr uint32_t kIdesc = idesc_i8(256, BN);
    static constexpr int kAccShift = 4;
    static_assert(BN == 128 || BN == 192 || BN == 256, "token tile: 128, 192 or 256");
    static_assert(kXBytes % 1024 == 0, "activation stages stay 1024-byte aligned (128 B swizzle atoms)");
    static_assert(kTmemStages >= 2 && kTmemStages % kGroups == 0,
                  "every TMEM stage is always taken by the same expander group");
    static_assert(kPStages % kGroups == 0, "every packed slot is always taken by the same expander group");
    static_assert(kStages >= 2, "activation ring needs two stages");
    static_assert((BN / 32) % 2 == 0, "the epilogue drains two 32-column chunks per wait");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

// D = acc / 16 as a float, exactly, for |D| < 2^22 (see the header).
__device__ __forceinline__ float a8t_acc_to_float(uint32_t acc) {
    return __fsub_rn(__int_as_float((static_cast<int32_t>(acc) >> 4) + 0x4B400000), 12582912.0f);
}

template <int BN, int OUT, bool STAGED>
__global__ void __launch_bounds__(kPairThreads, 1)
int4_gemm_a8t_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                     const __grid_constant__ CUtensorMap tmap_out,
                     const float* __restrict__ xscale, const float* __restrict__ wscale, BiasRef bias,
                     void* __restrict__ out, int M, int N, int K, int tiles_w, int num_tiles,
                     const void* __restrict__ wraw) {
    using Cfg = A8tCfg<BN, STAGED>;
    static_assert(!STAGED || OUT == kOutBF16, "staged stores are for bf16 output");
    extern __shared__ __align__(1024) unsigned char a8t_smem_raw[];
    // 1024-byte aligned by pointer arithmetic on the shared array itself, so the
    // compiler keeps the shared address space (ld.shared / st.shared, not generic
    // accesses) for everything addressed from here
    unsigned char* smem = a8t_smem_raw + ((1024u - (smem_u32(a8t_smem_raw) & 1023u)) & 1023u);
    unsigned char* xring = smem;
    unsigned char* pring = smem + Cfg::kPOffset;
    unsigned char* staging = smem + Cfg::kStagingOffset;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOffset);
    uint64_t* full_bar = bars;                                  // even CTA: both activation halves landed
    uint64_t* empty_bar = full_bar + Cfg::kStages;              // MMAs done with the activation slot
    uint64_t* pfull_bar = empty_bar + Cfg::kStages;             // this CTA's packed weights landed
    uint64_t* pempty_bar = pfull_bar + Cfg::kPStages;           // the expanders have read the packed slot
    uint64_t* ready_bar = pempty_bar + Cfg::kPStages;           // even CTA: both CTAs' weights are in TMEM
    uint64_t* tfree_bar = ready_bar + Cfg::kTmemStages;         // MMAs done with the TMEM stage
    uint64_t* acc_full_bar = tfree_bar + Cfg::kTmemStages;      // [2]
    uint64_t* acc_empty_bar = acc_full_bar + 2;                 // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::kMiscOffset);
    float* col_factors = reinterpret_cast<float*>(smem + Cfg::kColOffset);   // [2][BN] token scales

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t cta = cluster_ctarank();
    const int cluster_id = blockIdx.x >> 1;
    const int num_clusters = gridDim.x >> 1;
    const int num_kt = K / kPairBKP;
    const int my_tiles = (num_tiles - cluster_id + num_clusters - 1) / num_clusters;
    const int total_it = my_tiles * num_kt;

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::kStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int p = 0; p < Cfg::kPStages; ++p) {
            mbar_init(&pfull_bar[p], 1);
            mbar_init(&pempty_bar[p], Cfg::kGroupWarps);
        }
        for (int t = 0; t < Cfg::kTmemStages; ++t) {
            mbar_init(&ready_bar[t], 2 * Cfg::kGroupWarps);     // both CTAs' expander warps
            mbar_init(&tfree_bar[t], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full_bar[b], 1);
            mbar_init(&acc_empty_bar[b], 2);                    // one epilogue arrival from each CTA
        }
        fence_mbar_init();
        tma_prefetch_desc(&tmap_x);
        tma_prefetch_desc(&tmap_w);
        if constexpr (STAGED) tma_prefetch_desc(&tmap_out);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();                       // peer barriers initialised before any remote arrive
    tc_fence_after();
    if (warp == 3 && lane == 0 && cluster_id < num_tiles) {
        // an L2 hint, safe whatever the previous kernel writes: this CTA's weight rows of
        // its first tile (one contiguous block of packed bytes) start streaming while the
        // previous kernel (the quantizer) still runs
        const int w_row0 = (cluster_id % tiles_w) * 256 + static_cast<int>(cta) * Cfg::kWRows;
        const int rows = N - w_row0 < Cfg::kWRows ? N - w_row0 : Cfg::kWRows;
        if (rows > 0)
            bulk_prefetch_l2(static_cast<const unsigned char*>(wraw) + static_cast<size_t>(w_row0) * (K >> 1),
                             static_cast<uint32_t>(rows) * static_cast<uint32_t>(K >> 1));
    }
    // every operand, scale and output may belong to the previous kernel
    griddep_wait();
    griddep_launch_dependents();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t tmem_a0 = tmem_base + Cfg::kAccBufs * BN;    // expanded-weight stages follow the accumulators

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- activation producer
            int it = 0;
            bool ok = true;
            for (int t = cluster_id; t < num_tiles && ok; t += num_clusters) {
                const int x_row0 = (t / tiles_w) * BN + static_cast<int>(cta) * Cfg::kXHalf;
                for (int kt = 0; kt < num_kt; ++kt, ++it) {
                    const int s = it % Cfg::kStages;
                    if (!mbar_wait_bounded<true>(&empty_bar[s], ((it / Cfg::kStages) & 1) ^ 1)) {
                        record_status(kStatusTimeoutProducer); ok = false; break;
                    }
                    const uint32_t full_leader = mapa_shared(smem_u32(&full_bar[s]), 0);
                    if (cta == 0) mbar_arrive_expect_tx(&full_bar[s], 2 * Cfg::kXBytes);
                    tma_load_2d_pair(xring + s * Cfg::kXBytes, &tmap_x, full_leader, kt * kPairBKP, x_row0);
                }
            }
        }
    } else if (warp == 1) {
        if (cta == 0) {
            // ---------------- MMA issuer (even CTA): the whole warp runs the loop,
            // one elected lane issues
            int it = 0;
            bool ok = true;
            for (int lt = 0; lt < my_tiles && ok; ++lt) {
                const int abuf = lt % Cfg::kAccBufs, ause = lt / Cfg::kAccBufs;
                if (ause > 0 && !__all_sync(0xFFFFFFFFu, mbar_wait_bounded(&acc_empty_bar[abuf], (ause - 1) & 1))) {
                    if (lane == 0) record_status(kStatusTimeoutMma);
                    break;
                }
                const uint32_t acc_tmem = tmem_base + abuf * BN;
                tc_fence_after();
                for (int kt = 0; kt < num_kt; ++kt, ++it) {
                    const int s = it % Cfg::kStages;
                    if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(&full_bar[s], (it / Cfg::kStages) & 1))) {
                        if (lane == 0) record_status(kStatusTimeoutMma);
                        ok = false;
                        break;
                    }
                    const int ts = it % Cfg::kTmemStages;
                    if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded<true>(&ready_bar[ts], (it / Cfg::kTmemStages) & 1))) {
                        if (lane == 0) record_status(kStatusTimeoutMma);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    // K-major, 128 B swizzle: the j-th 32-byte K step is +2 in the address field;
                    // in TMEM it is 8 columns
                    const uint64_t db = smem_desc_kmajor(smem_u32(xring + s * Cfg::kXBytes), 8 * kPairBKP,
                                                         kSwizzle128);
                    if (elect_one()) {
                        #pragma unroll
                        for (int j = 0; j < kPairBKP / 32; ++j)
                            mma_i8_ts_pair(acc_tmem, tmem_a0 + ts * Cfg::kStageCols + j * 8, db + 2 * j, Cfg::kIdesc,
                                           (kt | j) != 0);
                        mma_commit_pair_multicast(&empty_bar[s], 0x3);
                        mma_commit_pair_multicast(&tfree_bar[ts], 0x3);
                    }
                    __syncwarp();
                }
                if (ok && elect_one()) mma_commit_pair_multicast(&acc_full_bar[abuf], 0x3);
                __syncwarp();
            }
        }
    } else if (warp == 2) {
        if (lane == 0) {
            // ---------------- packed-weight producer (this CTA's 128 rows)
            int it = 0;
            bool ok = true;
            for (int t = cluster_id; t < num_tiles && ok; t += num_clusters) {
                const int w_row0 = (t % tiles_w) * 256 + static_cast<int>(cta) * Cfg::kWRows;
                for (int kt = 0; kt < num_kt; ++kt, ++it) {
                    const int p = it % Cfg::kPStages;
                    if (!mbar_wait_bounded(&pempty_bar[p], ((it / Cfg::kPStages) & 1) ^ 1)) {
                        record_status(kStatusTimeoutProducer); ok = false; break;
                    }
                    mbar_arrive_expect_tx(&pfull_bar[p], Cfg::kWBytes);
                    tma_load_2d(pring + p * Cfg::kWBytes, &tmap_w, &pfull_bar[p], kt * Cfg::kWRowBytes, w_row0);
                }
            }
        }
    } else if (warp == 3) {
        // (its L2 prefetch ran before the wait for the previous kernel)
    } else if (warp < 12) {
        // ---------------- expanders: weight row r of the slot -> TMEM lane r
        const int group = (warp - 4) / Cfg::kGroupWarps;
        const int quarter = warp & 3;                           // TMEM lanes 32*quarter .. (warp % 4 rule)
        const int r = quarter * 32 + lane;
        const uint32_t sw = static_cast<uint32_t>((r >> 1) & 3);   // 64 B swizzle: chunk ^= (row / 2) % 4
        const uint32_t ready_leader0 = mapa_shared(smem_u32(ready_bar), 0);
        const uint32_t lane_field = static_cast<uint32_t>(quarter * 32) << 16;
        for (int it = group; it < total_it; it += Cfg::kGroups) {
            const int p = it % Cfg::kPStages;
            if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(&pfull_bar[p], (it / Cfg::kPStages) & 1))) {
                record_status(kStatusTimeoutExpand); break;
            }
            const unsigned char* row = pring + p * Cfg::kWBytes + r * Cfg::kWRowBytes;
            uint4 v[4];
            #pragma unroll
            for (int c = 0; c < 4; ++c) v[c] = *reinterpret_cast<const uint4*>(row + ((c ^ sw) << 4));
            __syncwarp();
            if (lane == 0) mbar_arrive(&pempty_bar[p]);
            uint32_t o[32];
            #pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint32_t w[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
                #pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const uint32_t lo = (w[e] << 4) & 0xF0F0F0F0u, hi = w[e] & 0xF0F0F0F0u;
                    o[8 * c + 2 * e] = __byte_perm(lo, hi, 0x5140);          // codes 8i .. 8i+3
                    o[8 * c + 2 * e + 1] = __byte_perm(lo, hi, 0x7362);      // codes 8i+4 .. 8i+7
                }
            }
            // expanded in registers first: after the stage frees only the store remains
            const int ts = it % Cfg::kTmemStages;
            if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded<true>(&tfree_bar[ts], ((it / Cfg::kTmemStages) & 1) ^ 1))) {
                record_status(kStatusTimeoutExpand); break;
            }
            tc_fence_after();
            tmem_st_32x32b_x32(tmem_a0 + lane_field + ts * Cfg::kStageCols, o);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                // the odd CTA's warps arrive on the even CTA's barrier (CTA-scope release:
                // the TMEM stores are complete after tcgen05.wait::st)
                if (cta == 1) mbar_arrive_remote_cta(ready_leader0 + ts * 8);
                else mbar_arrive(&ready_bar[ts]);
            }
        }
    } else {
        // ---------------- epilogue: TMEM lanes = this CTA's 128 weight rows, columns = BN tokens
        const int quarter = warp & 3;
        const int et = threadIdx.x - 384;                       // 0..127
        const int r = quarter * 32 + lane;
        const uint32_t acc_empty_leader0 = mapa_shared(smem_u32(acc_empty_bar), 0);
        // STAGED: this warp's two [32 tokens][32 weight rows] bf16 boxes (64 B rows,
        // 64 B swizzle), used in turn
        const uint32_t boxes = smem_u32(staging + quarter * 2 * Cfg::kBoxBytes);
        int box_seq = 0;
        for (int lt = 0; lt < my_tiles; ++lt) {
            const int t = cluster_id + lt * num_clusters;
            const int w_base = (t % tiles_w) * 256 + static_cast<int>(cta) * Cfg::kWRows;
            const int x0 = (t / tiles_w) * BN;                          // first token m of the tile
            float* cscale = col_factors + (lt & 1) * BN;
            if constexpr (OUT != kOutS32) {
                for (int c = et; c < BN; c += kEpiThreads) cscale[c] = (x0 + c < M) ? xscale[x0 + c] : 0.0f;
            }
            const int abuf = lt % Cfg::kAccBufs, ause = lt / Cfg::kAccBufs;
            // accumulator drained: hand TMEM back to the MMA issuer
            auto release = [&]() {
                tc_fence_before();
                named_barrier_sync(kEpiBarrier, kEpiThreads);
                if (et == 0) {
                    if (cta == 0) mbar_arrive(&acc_empty_bar[abuf]);
                    else mbar_arrive_cluster(acc_empty_leader0 + abuf * 8);
                }
            };
            if constexpr (STAGED) {
                // 16x256b loads: thread t holds weight rows n = 16h + 8nh + t/4 (h: which
                // 16-lane half of this warp's 32, nh: register pair) at token pairs
                // 8j + 2(t%4), +1 -- the fragment layout of a transposing stmatrix, which
                // writes each token's 8 consecutive weight rows as one 16-byte row
                const int tq = lane >> 2, tr = lane & 3;
                float2 ws2[2][2], b2[2][2];
                #pragma unroll
                for (int h = 0; h < 2; ++h) {
                    #pragma unroll
                    for (int nh = 0; nh < 2; ++nh) {
                        const int n = w_base + quarter * 32 + 16 * h + 8 * nh + tq;
                        const float wsv = n < N ? wscale[n] : 0.0f;
                        const float bv = (n < N && bias.ptr != nullptr) ? bias.at(n) : 0.0f;
                        ws2[h][nh] = make_float2(wsv, wsv);
                        b2[h][nh] = make_float2(bv, bv);
                    }
                }
                named_barrier_sync(kEpiBarrier, kEpiThreads);
                if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded<true>(&acc_full_bar[abuf], ause & 1))) {
                    if (lane == 0) record_status(kStatusTimeoutEpilogue);
                    break;
                }
                tc_fence_after();
                const uint32_t tb0 = tmem_base + abuf * BN + (static_cast<uint32_t>(quarter * 32) << 16);
                const uint32_t tb1 = tb0 + (16u << 16);
                const float2 mg = make_float2(-12582912.0f, -12582912.0f);
                auto emit = [&](const uint32_t (&acc)[32], int c) {
                    const int m0 = x0 + c * 32;
                    const uint32_t box = boxes + (box_seq & 1) * Cfg::kBoxBytes;
                    if (lane == 0) bulk_wait_group_read1();             // the box's previous store has read it
                    __syncwarp();
                    #pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        uint32_t pk[8];                                 // matrix 2j + nh
                        #pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float2 xs2 = *reinterpret_cast<const float2*>(cscale + c * 32 + 8 * j + 2 * tr);
                            #pragma unroll
                            for (int nh = 0; nh < 2; ++nh) {
                                const uint32_t a0 = acc[16 * h + 4 * j + 2 * nh], a1 = acc[16 * h + 4 * j + 2 * nh + 1];
                                const float2 raw = make_float2(
                                    __int_as_float((static_cast<int32_t>(a0) >> 4) + 0x4B400000),
                                    __int_as_float((static_cast<int32_t>(a1) >> 4) + 0x4B400000));
                                // packed products, scalar bias adds: a packed add after the
                                // packed products gave other last bits than the scalar
                                // sequence on rounding ties (as if contracted into an fma)
                                const float2 pm = fmul2_rn(fmul2_rn(fadd2_rn(raw, mg), xs2), ws2[h][nh]);
                                const float2 v = make_float2(__fadd_rn(pm.x, b2[h][nh].x), __fadd_rn(pm.y, b2[h][nh].y));
                                const __nv_bfloat162 p2 = __floats2bfloat162_rn(v.x, v.y);
                                uint32_t u;
                                memcpy(&u, &p2, 4);
                                pk[2 * j + nh] = u;
                            }
                        }
                        #pragma unroll
                        for (int sx = 0; sx < 2; ++sx) {
                            // matrix 4 sx + lane / 8: token row 8 j + lane % 8, weight rows 16h + 8nh ..
                            const int mi = 4 * sx + (lane >> 3);
                            const int mrow = 8 * (mi >> 1) + (lane & 7);
                            const int chunk = 2 * h + (mi & 1);
                            const uint32_t addr = box + mrow * 64 + ((chunk ^ ((mrow >> 1) & 3)) << 4);
                            stmatrix_x4_trans(addr, pk[4 * sx], pk[4 * sx + 1], pk[4 * sx + 2], pk[4 * sx + 3]);
                        }
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0 && w_base + quarter * 32 < N && m0 < M) {
                        tma_store_2d(&tmap_out, staging + (box - smem_u32(staging)), w_base + quarter * 32, m0);
                        bulk_commit_group();
                    }
                    ++box_seq;
                };
                // TMEM loads one chunk ahead of the stores; the buffer goes back to the
                // MMA issuer as soon as its last chunk is in registers
                uint32_t ra[32], rb[32];
                __syncwarp();
                tmem_ld_16x256b_x4(tb0, ra);
                tmem_ld_16x256b_x4(tb1, ra + 16);
                tmem_ld_wait_regs(ra);
                #pragma unroll 1
                for (int c = 0; c < BN / 32; c += 2) {
                    tmem_ld_16x256b_x4(tb0 + (c + 1) * 32, rb);
                    tmem_ld_16x256b_x4(tb1 + (c + 1) * 32, rb + 16);
                    emit(ra, c);
                    tmem_ld_wait_regs(rb);
                    const bool more = c + 2 < BN / 32;
                    if (more) {
                        tmem_ld_16x256b_x4(tb0 + (c + 2) * 32, ra);
                        tmem_ld_16x256b_x4(tb1 + (c + 2) * 32, ra + 16);
                    } else {
                        release();
                    }
                    emit(rb, c + 1);
                    if (more) tmem_ld_wait_regs(ra);
                }
            } else {
                // direct stores: one weight row (TMEM lane) per thread, 32 tokens per load
                const int a = w_base + r;
                const bool lane_ok = a < N;
                float lane_scale = 0.0f, lane_bias = 0.0f;
                if (lane_ok && OUT != kOutS32) {
                    lane_scale = wscale[a];
                    lane_bias = bias.ptr != nullptr ? bias.at(a) : 0.0f;
                }
                named_barrier_sync(kEpiBarrier, kEpiThreads);
                if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded<true>(&acc_full_bar[abuf], ause & 1))) {
                    if (lane == 0) record_status(kStatusTimeoutEpilogue);
                    break;
                }
                tc_fence_after();
                const uint32_t tbase = tmem_base + abuf * BN + (static_cast<uint32_t>(quarter * 32) << 16);
                auto emit = [&](const uint32_t (&acc)[32], int c) {
                    if (!lane_ok) return;
                    const int m0 = x0 + c * 32;
                    #pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        if (m0 + i >= M) continue;
                        const size_t oi = static_cast<size_t>(m0 + i) * N + a;
                        if constexpr (OUT == kOutS32) {
                            reinterpret_cast<int32_t*>(out)[oi] = static_cast<int32_t>(acc[i]) >> Cfg::kAccShift;
                        } else {
                            const float v = __fadd_rn(
                                __fmul_rn(__fmul_rn(a8t_acc_to_float(acc[i]), cscale[c * 32 + i]), lane_scale),
                                lane_bias);
                            if constexpr (OUT == kOutBF16)
                                reinterpret_cast<__nv_bfloat16*>(out)[oi] = __float2bfloat16_rn(v);
                            else
                                reinterpret_cast<float*>(out)[oi] = v;
                        }
                    }
                };
                uint32_t ra[32], rb[32];
                __syncwarp();
                tmem_ld_32x32b_x32(tbase, ra);
                tmem_ld_wait_regs(ra);
                #pragma unroll 1
                for (int c = 0; c < BN / 32; c += 2) {
                    tmem_ld_32x32b_x32(tbase + (c + 1) * 32, rb);
                    emit(ra, c);
                    tmem_ld_wait_regs(rb);
                    const bool more = c + 2 < BN / 32;
                    if (more) tmem_ld_32x32b_x32(tbase + (c + 2) * 32, ra);
                    else release();
                    emit(rb, c + 1);
                    if (more) tmem_ld_wait_regs(ra);
                }
            }
        }
        if constexpr (STAGED) {
            if (lane == 0) bulk_wait_group0();
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
