// int4 x int4 GEMM on CTA pairs (tcgen05.mma.cta_group::2.kind::i8, A from TMEM),
// persistent over output tiles.
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
// Each cluster walks the tiles t = cluster, cluster + clusters, ...; the
// k-stage ring and all barrier phases run on across tiles, so the loads and
// expansion of tile i+1 overlap the epilogue of tile i. The epilogue drains
// the accumulator (into a swizzled shared-memory tile that a TMA store writes
// out, for bf16 output), then hands TMEM back to the MMA issuer.
//
// Warp roles (16 warps, both CTAs alike):
//   w0        TMA producer (one lane): packed A and B-half tiles per k-stage
//   w1        TMEM allocation; in the even CTA, one lane issues the MMAs
//   w2, w3    odd CTA only: forward "stage expanded" to the even CTA, one
//             cluster-scope release per stage, alternating stages
//   w4..w7    A expanders (row = 32*(w%4) + lane)
//   w8..w11   B expanders
//   w12..w15  epilogue (TMEM lanes 32*(w%4) ..)
//
// A8 form (int8 activation codes, packed int4 weights): the activations come
// from the quantizer as one sign-extended int8 per code and go by TMA
// (cta_group::2) straight into shared memory, like the W8A8 tier; only the
// weights stay packed in HBM. Expander warps load them (64 bytes of K per row
// and stage) straight into registers, a stage ahead, and write each byte b as
// the int8 pair (16*lo, 16*hi) in column order into a weight slot (128 B
// swizzle); the accumulator is 16 * D. Shared-memory bandwidth bounds these
// pipelines, so the packed bytes never pass through shared memory.
//
// Stage hand-off: expander warps arrive with CTA-scope release on a local
// barrier (the MMA's own barrier in the even CTA, a forwarding barrier in the
// odd one). A cluster-scope release costs a memory-barrier round trip, so the
// odd CTA pays it once per stage in a forwarding warp, off the expanders' path;
// two forwarding warps keep two of them in flight.
#pragma once

namespace convrot {

// A8 weight-slot ring depth and expander groups (stages taken in turn; the
// depth must be a multiple of the groups).
#ifndef CONVROT_A8_BSTAGES
#define CONVROT_A8_BSTAGES 4
#endif
#ifndef CONVROT_A8_GROUPS
#define CONVROT_A8_GROUPS 4
#endif

constexpr int kPairThreads = 16 * 32;
constexpr uint32_t kTmemCols = 512;
constexpr int kPairBKP = 128;            // packed bytes of K per stage (256 codes), one 128 B swizzle row
constexpr int kSwizzle128 = 2;           // tcgen05 descriptor code for 128-byte swizzle
constexpr int kEpiThreads = 128;         // four epilogue warps
constexpr uint32_t kEpiBarrier = 1;      // named barrier id of the epilogue warps

// I8: the W8A8 tier -- plain int8 operands, no nibble expansion: both operands
// go by TMA (cta_group::2, completing on the even CTA's barrier) straight into
// shared memory and the MMAs read them there.
// A8: int4 layers with int8 activation codes (one per byte) and packed int4
// weights expanded in shared memory (see the header).
template <int BN, bool STAGED, bool SWAP, bool LORA = false, bool I8 = false, bool A8 = false>
struct PairCfg {
    static constexpr int kBHalf = BN / 2;
    static constexpr bool kASmem = I8 || A8;                       // A by TMA into shared memory (MMA SS)
    // A8: packed weight ring (64 bytes of K a row per stage: 128 codes)
    static constexpr int kPackedRowBytes = 64;                     // packed bytes of a weight row per stage
    static constexpr int kPackedChunks = A8 ? kBHalf * kPackedRowBytes / 16 : 0;   // 16-byte chunks per stage
    static constexpr int kA8ExpWarps = 8;                          // warps 4..11
    // the expander warps form groups that take whole stages in turn, so several
    // stages are expanded at once (each group's wait/expand/fence/arrive chain
    // then only has to keep up with every kA8Groups-th stage)
    static constexpr int kA8Groups = CONVROT_A8_GROUPS;
    static constexpr int kA8GroupWarps = kA8ExpWarps / kA8Groups;
    // A8 rings: activation tiles (the operand ring, kStages deep, A only) and
    // expanded weight half-tiles (kBStages deep).
    static constexpr int kBStages = A8 ? (LORA && BN > 128 ? 4 : CONVROT_A8_BSTAGES) : 0;
    static constexpr int kBRing = A8 ? kBStages : 1;               // kBStages as a divisor (A8 code only)
    // A8: the odd CTA's expander warps arrive on the even CTA's barrier themselves
    static constexpr bool kA8Direct = A8;
    // int8 form with 256 x 128 tiles (few tiles: small M or N): two 128-byte K
    // sub-tiles per stage, 8 MMAs per barrier wait and commit; a stage is
    // [A sub 0 | A sub 1 | B sub 0 | B sub 1]. (256-column tiles keep one: their
    // 64 KB double stages would leave a 3-deep ring.)
    static constexpr int kSubK = (I8 && !STAGED && !LORA && BN <= 128) ? 2 : 1;
    static constexpr int kStageK = kSubK * kPairBKP;               // operand bytes of K per stage
    static constexpr int kABytes = 128 * kPairBKP;                 // one sub-tile
    static constexpr int kBBytes = kBHalf * kPairBKP;
    static constexpr int kStageBytes = I8 ? kSubK * (kABytes + kBBytes) : A8 ? kABytes : kABytes + 2 * kBBytes;
    static constexpr int kTmemStageCols = 2 * kPairBKP / 4;      // hi + lo bytes of a row, 4 per column
    static constexpr int kMmasPerStage = (I8 ? kSubK : A8 ? 1 : 2) * kPairBKP / 32;   // K = 32 bytes per MMA
    // int4 halves accumulate 256 * D, A8's 16x-scaled weights 16 * D
    static constexpr int kAccShift = I8 ? 0 : A8 ? 4 : 8;
    // bf16 output tile staged for the TMA store: 128 rows x BN cols, 64-col boxes
    static constexpr int kStagingBytes = STAGED ? 128 * BN * 2 : 0;
    // 227 KB per block, minus alignment slack, barriers and the staging tile
    // Dynamic-LoRA operands per tile: T rows (x A^T, fp16, 64 per 128 B row) and
    // this CTA's half of the LoRA up-projection rows
    static constexpr int kLoraTBytes = LORA ? 128 * 128 : 0;
    static constexpr int kLoraBBytes = LORA ? kBHalf * 128 : 0;
    static constexpr int kSmemForStages = 227 * 1024 - 2048 - 4 * BN * 4 - kStagingBytes - kLoraTBytes - kLoraBBytes
                                          - kBStages * kBBytes;
    // TMA ring (shared memory) and expanded-A ring (TMEM slots) are sized
    // independently: the loads may run further ahead than TMEM allows.
    static constexpr int kAccCols = LORA ? 2 * BN : BN;          // int32 accumulator (+ fp32 LoRA accumulator)
    // Accumulator buffers: with two, the next tile's MMAs run while the epilogue
    // drains the previous tile (the int8 tier has no A operand in TMEM, so both fit).
    // (256-column LoRA tiles need all 512 columns for one int32 + fp32 pair: one buffer)
    static constexpr int kAccBufs = (kASmem && !(LORA && BN > 128)) ? 2 : 1;
    static constexpr int kTmemStages0 =
        kASmem ? 16 : (static_cast<int>(kTmemCols) - kAccCols * kAccBufs) / kTmemStageCols;
    static constexpr int kStagesBySmem = kSmemForStages / kStageBytes;
    static constexpr int kStagesCapped = kStagesBySmem < 16 ? kStagesBySmem : 16;
    // Swapped tiles: the three expander groups take TMA stages in turn, and TMA
    // copies may land out of order, so each ring slot must always belong to
    // the same group (which has then seen the slot's previous phase complete
    // before waiting on the next: a parity wait cannot tell phase k - 1 from
    // phase k + 1). The forwarders and the other waiters see stages complete
    // in order, so they need no such rounding.
    static constexpr int kStages = SWAP ? kStagesCapped - kStagesCapped % 3 : kStagesCapped;
    static constexpr int kTmemStages = kTmemStages0 < kStages ? kTmemStages0 : kStages;
    static constexpr int kBexpOffset = kStages * kStageBytes;
    static constexpr int kStagingOffset = kBexpOffset + kBStages * kBBytes;
    static constexpr int kLoraOffset = kStagingOffset + kStagingBytes;
    static constexpr int kBarOffset = kLoraOffset + kLoraTBytes + kLoraBBytes;
    // ready / forward barriers: one per weight slot in A8, per operand stage otherwise
    static constexpr int kReadyStages = A8 ? kBStages : kStages;
    static constexpr int kNumBars = 2 * kStages + 2 * kReadyStages + kTmemStages + 6 + kBStages;
    static constexpr int kMiscOffset = kBarOffset + kNumBars * 8;
    // per-tile column factors (scale, bias) x 2 tiles in flight
    static constexpr int kColOffset = kMiscOffset + 16;
    static constexpr int kSmemBytes = kColOffset + 2 * 2 * BN * 4 + 1024;
    static constexpr uint32_t kIdesc = idesc_i8(256, BN);
    static constexpr uint32_t kIdescLora = idesc_f16(256, BN);    // fp16 T and B, fp32 accumulator
    // swapped (weight-bound) tiles: three groups of four warps take turns on
    // whole stages (A and B), otherwise four A and four B expander warps
    static constexpr int kExpGroups = SWAP ? 3 : 1;
    static constexpr int kLocalArrivals = SWAP ? 4 : A8 ? kA8GroupWarps : 8;   // expander warps per CTA and stage
    // + the odd CTA's forwarder (A8: each odd expander warp)
    static constexpr int kReadyCount = kA8Direct ? 2 * kLocalArrivals : kLocalArrivals + 1;
    static_assert(BN >= 32 && BN <= 256 && BN % 32 == 0, "pair MMA N must be a multiple of 32 in [32, 256]");
    static_assert(kStages >= 2 && kTmemStages >= 2, "pipeline needs at least two stages");
    static_assert(!SWAP || (kExpGroups == 3 && kStages % 3 == 0), "swapped tiles: ring slots owned by one group");
    static_assert(!I8 || !SWAP, "the int8 form uses non-swapped tiles");
    static_assert(!A8 || (!I8 && !SWAP && !STAGED), "A8: non-swapped tiles, direct stores");
    static_assert(!A8 || kPackedChunks % (kA8GroupWarps * 32) == 0, "A8: whole chunks per expander thread");
    static_assert(!A8 || kBStages % kA8Groups == 0,
                  "A8: every weight / packed slot is always taken by the same expander group");
    static_assert(!LORA || kAccBufs * kAccCols <= static_cast<int>(kTmemCols), "accumulators fit TMEM");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

// Dequantize and store 32 consecutive outputs of one output row directly to
// global memory. v[] holds ((D * xs) * ws) already; bias is added here.
template <int OUT>
__device__ __forceinline__ void store_row32(void* out, size_t obase, int n, int N, float (&v)[32],
                                            const float* bias_cols) {
    const bool full = (n + 32 <= N);
    #define BIAS_AT(i) (bias_cols != nullptr ? bias_cols[i] : 0.0f)
    if constexpr (OUT == kOutBF16) {
        __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out) + obase;
        if (full && (reinterpret_cast<uintptr_t>(o) & 15u) == 0) {
            #pragma unroll
            for (int i = 0; i < 32; i += 8) {
                uint32_t w[4];
                #pragma unroll
                for (int e = 0; e < 4; ++e) {
                    __nv_bfloat162 b2 = __floats2bfloat162_rn(__fadd_rn(v[i + 2 * e], BIAS_AT(i + 2 * e)),
                                                              __fadd_rn(v[i + 2 * e + 1], BIAS_AT(i + 2 * e + 1)));
                    memcpy(&w[e], &b2, 4);
                }
                *reinterpret_cast<uint4*>(o + i) = make_uint4(w[0], w[1], w[2], w[3]);
            }
        } else {
            #pragma unroll
            for (int i = 0; i < 32; ++i)
                if (full || n + i < N) o[i] = __float2bfloat16_rn(__fadd_rn(v[i], BIAS_AT(i)));
        }
    } else if constexpr (OUT == kOutF32) {
        float* o = reinterpret_cast<float*>(out) + obase;
        if (full && (N & 3) == 0) {
            #pragma unroll
            for (int i = 0; i < 32; i += 4)
                *reinterpret_cast<float4*>(o + i) = make_float4(
                    __fadd_rn(v[i], BIAS_AT(i)), __fadd_rn(v[i + 1], BIAS_AT(i + 1)),
                    __fadd_rn(v[i + 2], BIAS_AT(i + 2)), __fadd_rn(v[i + 3], BIAS_AT(i + 3)));
        } else {
            #pragma unroll
            for (int i = 0; i < 32; ++i)
                if (n + i < N) o[i] = __fadd_rn(v[i], BIAS_AT(i));
        }
    } else if constexpr (OUT == kOutF32Accumulate) {
        float* o = reinterpret_cast<float*>(out) + obase;
        #pragma unroll
        for (int i = 0; i < 32; ++i)
            if (full || n + i < N) o[i] = __fadd_rn(o[i], v[i]);
    }
    #undef BIAS_AT
}

// STAGED (bf16, not swapped, N % 8 == 0): output goes through a shared-memory
// tile and TMA stores (tmap_out); otherwise the epilogue stores directly.
// LORA (not swapped): a rank <= 64 side path out += lora_scale * T[m, :] . B[n, :]
// (T = x A^T precomputed, both fp16) on the tensor cores into a second, fp32
// accumulator, added in the epilogue before the single output rounding.
template <int BN, bool SWAP, int OUT, bool STAGED, bool LORA = false, bool I8 = false, bool A8 = false>
__global__ void __launch_bounds__(kPairThreads, 1)
int4_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                      const __grid_constant__ CUtensorMap tmap_out,
                      const __grid_constant__ CUtensorMap tmap_lt, const __grid_constant__ CUtensorMap tmap_lb,
                      const float* __restrict__ xscale, const float* __restrict__ wscale,
                      BiasRef bias, void* __restrict__ out, int M, int N, int K,
                      int tiles_a, int num_tiles, float lora_scale, const void* __restrict__ wraw,
                      const __grid_constant__ PeerOut peers) {
    using Cfg = PairCfg<BN, STAGED, SWAP, LORA, I8, A8>;
    static_assert(!LORA || !SWAP, "the LoRA side path is fused into non-swapped tiles");
    static_assert(!STAGED || (OUT == kOutBF16 && !SWAP), "staged epilogue is for bf16, non-swapped tiles");
    extern __shared__ __align__(1024) unsigned char psmem_raw[];
    // 1024-byte aligned by pointer arithmetic on the shared array itself, so the
    // compiler keeps the shared address space (ld.shared / st.shared, not generic
    // accesses) for everything addressed from here
    unsigned char* smem = psmem_raw + ((1024u - (smem_u32(psmem_raw) & 1023u)) & 1023u);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOffset);
    uint64_t* full_bar = bars;
    uint64_t* empty_bar = bars + Cfg::kStages;
    uint64_t* ready_bar = bars + 2 * Cfg::kStages;               // [kReadyStages]
    uint64_t* fwd_bar = ready_bar + Cfg::kReadyStages;           // [kReadyStages]
    uint64_t* tmem_free_bar = fwd_bar + Cfg::kReadyStages;       // [kTmemStages]
    uint64_t* acc_full_bar = tmem_free_bar + Cfg::kTmemStages;   // [2] per accumulator buffer
    uint64_t* acc_empty_bar = acc_full_bar + 2;                  // [2]
    uint64_t* lora_full_bar = acc_full_bar + 4;                  // even CTA: both CTAs' LoRA tiles landed
    uint64_t* lora_empty_bar = acc_full_bar + 5;                 // LoRA MMAs of the previous tile done
    uint64_t* bempty_bar = acc_full_bar + 6;                     // A8: MMAs done with a weight slot [kBStages]
    unsigned char* bexp_ring = smem + Cfg::kBexpOffset;
    constexpr int kReadyStages = Cfg::kReadyStages;
    unsigned char* lora_t = smem + Cfg::kLoraOffset;
    unsigned char* lora_b = lora_t + Cfg::kLoraTBytes;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::kMiscOffset);
    unsigned char* staging = smem + Cfg::kStagingOffset;
    float* col_factors = reinterpret_cast<float*>(smem + Cfg::kColOffset);   // [2][scale BN | bias BN]

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t cta = cluster_ctarank();
    const int cluster_id = blockIdx.x >> 1;
    const int num_clusters = gridDim.x >> 1;
    const int row_bytes = Cfg::kASmem ? K : (K >> 1);              // A operand bytes per row
    const int num_kt = (row_bytes + Cfg::kStageK - 1) / Cfg::kStageK;
    const int rows_a = SWAP ? N : M;
    // tiles of this cluster, and k-stage iterations over all of them
    const int my_tiles = (num_tiles - cluster_id + num_clusters - 1) / num_clusters;
    const int total_it = my_tiles * num_kt;

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::kStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int s = 0; s < kReadyStages; ++s) {
            mbar_init(&ready_bar[s], Cfg::kReadyCount);
            mbar_init(&fwd_bar[s], Cfg::kLocalArrivals);
        }
        for (int t = 0; t < Cfg::kTmemStages; ++t) mbar_init(&tmem_free_bar[t], 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full_bar[b], 1);
            mbar_init(&acc_empty_bar[b], 2);  // one epilogue arrival from each CTA
        }
        mbar_init(lora_full_bar, 1);
        mbar_init(lora_empty_bar, 1);
        for (int b = 0; b < Cfg::kBStages; ++b) mbar_init(&bempty_bar[b], 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmap_a);
        if constexpr (!A8) tma_prefetch_desc(&tmap_b);           // (A8 reads its weights without a map)
        if constexpr (STAGED) tma_prefetch_desc(&tmap_out);
        if constexpr (LORA) { tma_prefetch_desc(&tmap_lt); tma_prefetch_desc(&tmap_lb); }
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, kTmemCols);
        tmem_relinquish_pair();
    }
    // The weight boxes of this CTA's first tile are pulled into L2 (a hint:
    // safe whatever the previous kernel wrote). The nibble-expanding forms do it
    // here, while the previous kernel may still be running.
    auto prefetch_first_weights = [&]() {
        if (cluster_id >= num_tiles) return;
        const int t = cluster_id;
        if constexpr (SWAP) {
            const int w_row0 = (t % tiles_a) * 256 + static_cast<int>(cta) * 128;
            for (int x = 0; x < num_kt * Cfg::kStageK; x += kPairBKP) tma_prefetch_l2_2d(&tmap_a, x, w_row0);
        } else if constexpr (A8) {
            // this CTA's weight rows are one contiguous block of packed bytes
            const int w_row0 = (t / tiles_a) * BN + static_cast<int>(cta) * Cfg::kBHalf;
            const int rows = N - w_row0 < Cfg::kBHalf ? N - w_row0 : Cfg::kBHalf;
            if (rows > 0)
                bulk_prefetch_l2(static_cast<const unsigned char*>(wraw) + static_cast<size_t>(w_row0) * (K >> 1),
                                 static_cast<uint32_t>(rows) * static_cast<uint32_t>(K >> 1));
        } else {
            const int w_row0 = (t / tiles_a) * BN + static_cast<int>(cta) * Cfg::kBHalf;
            for (int x = 0; x < num_kt * Cfg::kStageK; x += kPairBKP) tma_prefetch_l2_2d(&tmap_b, x, w_row0);
        }
    };
    if (!Cfg::kASmem && warp == 0 && lane == 0) prefetch_first_weights();
    tc_fence_before();
    cluster_sync();                       // peer barriers initialised before any remote arrive
    tc_fence_after();
    // int8 and A8 forms: warp 3 has no role, so it pulls the weight boxes of this CTA's
    // first tile into L2 ahead of the ring, after the sync (one prefetch per
    // k-stage; issued before the sync they held every warp back). The A8 form's
    // single contiguous prefetch goes before the wait for the previous kernel.
    if (A8 && warp == 3 && lane == 0) prefetch_first_weights();
    // every operand, scale and output may belong to the previous kernel
    griddep_wait();
    griddep_launch_dependents();
    if (Cfg::kASmem && !A8 && warp == 3 && lane == 0) prefetch_first_weights();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t tmem_a0 = tmem_base + Cfg::kAccCols * Cfg::kAccBufs;  // A stages follow the accumulators
    // fp32 LoRA accumulator (LORA only): the second half of each accumulator buffer
    auto tmem_lora = [&](int abuf) -> uint32_t { return tmem_base + abuf * Cfg::kAccCols + BN; };

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer
            int it = 0;
            bool ok = true;
            int lt = 0;
            for (int t = cluster_id; t < num_tiles && ok; t += num_clusters, ++lt) {
                const int a_row0 = (t % tiles_a) * 256 + static_cast<int>(cta) * 128;
                const int b_row0 = (t / tiles_a) * BN + static_cast<int>(cta) * Cfg::kBHalf;
                if constexpr (LORA) {
                    if (!mbar_wait_bounded<true>(lora_empty_bar, (lt & 1) ^ 1)) {
                        record_status(kStatusTimeoutProducer); ok = false; break;
                    }
                    const uint32_t lora_full_leader = mapa_shared(smem_u32(lora_full_bar), 0);
                    if (cta == 0) mbar_arrive_expect_tx(lora_full_bar, 2 * (Cfg::kLoraTBytes + Cfg::kLoraBBytes));
                    tma_load_2d_pair(lora_t, &tmap_lt, lora_full_leader, 0, a_row0);
                    tma_load_2d_pair(lora_b, &tmap_lb, lora_full_leader, 0, b_row0);
                }
                for (int kt = 0; kt < num_kt; ++kt, ++it) {
                    const int s = it % Cfg::kStages;
                    const uint32_t ph = (it / Cfg::kStages) & 1;
                    if (!mbar_wait_bounded<true>(&empty_bar[s], ph ^ 1)) {
                        record_status(kStatusTimeoutProducer); ok = false; break;
                    }
                    unsigned char* st = smem + s * Cfg::kStageBytes;
                    if constexpr (A8) {
                        // int8 activation codes into the operand slot, both CTAs
                        // completing on the even CTA's barrier (the packed weights have a
                        // producer of their own, warp 2)
                        const uint32_t full_leader = mapa_shared(smem_u32(&full_bar[s]), 0);
                        if (cta == 0) mbar_arrive_expect_tx(&full_bar[s], 2 * Cfg::kABytes);
                        tma_load_2d_pair(st, &tmap_a, full_leader, kt * kPairBKP, a_row0);
                    } else if constexpr (I8) {
                        // both CTAs' tiles complete on the even CTA's barrier
                        const uint32_t full_leader = mapa_shared(smem_u32(&full_bar[s]), 0);
                        if (cta == 0) mbar_arrive_expect_tx(&full_bar[s], 2 * Cfg::kStageBytes);
                        #pragma unroll
                        for (int sub = 0; sub < Cfg::kSubK; ++sub) {
                            const int x = kt * Cfg::kStageK + sub * kPairBKP;
                            tma_load_2d_pair(st + sub * Cfg::kABytes, &tmap_a, full_leader, x, a_row0);
                            tma_load_2d_pair(st + Cfg::kSubK * Cfg::kABytes + sub * Cfg::kBBytes, &tmap_b,
                                             full_leader, x, b_row0);
                        }
                    } else {
                        mbar_arrive_expect_tx(&full_bar[s], Cfg::kABytes + Cfg::kBBytes);
                        tma_load_2d(st, &tmap_a, &full_bar[s], kt * kPairBKP, a_row0);
                        tma_load_2d(st + Cfg::kABytes, &tmap_b, &full_bar[s], kt * kPairBKP, b_row0);
                    }
                }
            }
        }
    } else if (warp == 1 && Cfg::kASmem) {
        if (cta == 0) {
            // ---------------- MMA issuer (even CTA), int8 form: the whole warp runs
            // the loop, so the stage index, barrier phase and operand descriptors
            // are warp-uniform values, and one elected lane issues the MMAs
            int it = 0;
            bool ok = true;
            for (int lt = 0; lt < my_tiles && ok; ++lt) {
                const int abuf = lt % Cfg::kAccBufs, ause = lt / Cfg::kAccBufs;
                if (ause > 0 && !__all_sync(0xFFFFFFFFu, mbar_wait_bounded(&acc_empty_bar[abuf], (ause - 1) & 1))) {
                    if (lane == 0) record_status(kStatusTimeoutMma);
                    break;
                }
                const uint32_t acc_tmem = tmem_base + abuf * Cfg::kAccCols;
                tc_fence_after();
                if constexpr (LORA) {
                    // the side path T . B^T on fp16 MMAs into this buffer's fp32 half, ahead
                    // of the K loop: its operand slot is then free for the next tile's
                    // side path early, and the producer does not stall between tiles
                    if (ok && !__all_sync(0xFFFFFFFFu, mbar_wait_bounded(lora_full_bar, lt & 1))) {
                        if (lane == 0) record_status(kStatusTimeoutMma);
                        ok = false;
                    }
                    if (ok) {
                        tc_fence_after();
                        const uint64_t dt = smem_desc_kmajor(smem_u32(lora_t), 1024, kSwizzle128);
                        const uint64_t dl = smem_desc_kmajor(smem_u32(lora_b), 1024, kSwizzle128);
                        if (elect_one()) {
                            #pragma unroll
                            for (int j = 0; j < 4; ++j)    // rank 64 = four K = 16 bf16 steps of a 128 B row
                                mma_f16kind_ss_pair(tmem_lora(abuf), dt + 2 * j, dl + 2 * j, Cfg::kIdescLora, j != 0);
                            mma_commit_pair_multicast(lora_empty_bar, 0x3);
                        }
                        __syncwarp();
                    }
                }
                for (int kt = 0; kt < num_kt && ok; ++kt, ++it) {
                    const int s = it % Cfg::kStages;
                    const uint32_t ph = (it / Cfg::kStages) & 1;
                    if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(&full_bar[s], ph))) {
                        if (lane == 0) record_status(kStatusTimeoutMma);
                        ok = false;
                        break;
                    }
                    // A8: the weight half-tiles of both CTAs expanded into weight slot sb
                    // (cluster scope: the odd CTA's half arrives from its forwarder)
                    const int sb = A8 ? it % Cfg::kBRing : 0;
                    if (A8 && !__all_sync(0xFFFFFFFFu,
                                          mbar_wait_bounded<true>(&ready_bar[sb], (it / Cfg::kBRing) & 1))) {
                        if (lane == 0) record_status(kStatusTimeoutMma);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + s * Cfg::kStageBytes);
                    const uint32_t b_addr = A8 ? smem_u32(bexp_ring + sb * Cfg::kBBytes)
                                               : a_addr + Cfg::kSubK * Cfg::kABytes;
                    // K-major, 128 B swizzle: the j-th 32-byte K step of a sub-tile is +2
                    // in the address field
                    uint64_t da[Cfg::kSubK], db[Cfg::kSubK];
                    #pragma unroll
                    for (int sub = 0; sub < Cfg::kSubK; ++sub) {
                        da[sub] = smem_desc_kmajor(a_addr + sub * Cfg::kABytes, 8 * kPairBKP, kSwizzle128);
                        db[sub] = smem_desc_kmajor(b_addr + sub * Cfg::kBBytes, 8 * kPairBKP, kSwizzle128);
                    }
                    if (elect_one()) {
                        #pragma unroll
                        for (int j = 0; j < Cfg::kMmasPerStage; ++j)
                            mma_i8_ss_pair(acc_tmem, da[j >> 2] + 2 * (j & 3), db[j >> 2] + 2 * (j & 3),
                                           Cfg::kIdesc, (kt | j) != 0);
                        mma_commit_pair_multicast(&empty_bar[s], 0x3);
                        if constexpr (A8) mma_commit_pair_multicast(&bempty_bar[sb], 0x3);
                    }
                    __syncwarp();
                }
                if (ok && elect_one()) mma_commit_pair_multicast(&acc_full_bar[abuf], 0x3);
                __syncwarp();
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && cta == 0) {
            // ---------------- MMA issuer (even CTA)
            int it = 0;
            bool ok = true;
            constexpr int kHalfSteps = Cfg::kMmasPerStage / 2;
            for (int lt = 0; lt < my_tiles && ok; ++lt) {
                const int abuf = lt % Cfg::kAccBufs, ause = lt / Cfg::kAccBufs;
                if (ause > 0 && !mbar_wait_bounded<true>(&acc_empty_bar[abuf], (ause - 1) & 1)) {
                    record_status(kStatusTimeoutMma); break;
                }
                const uint32_t acc_tmem = tmem_base + abuf * Cfg::kAccCols;
                tc_fence_after();
                if constexpr (LORA) {
                    if (ok && !mbar_wait_bounded<true>(lora_full_bar, lt & 1)) {
                        record_status(kStatusTimeoutMma); ok = false;
                    }
                    if (ok) {                              // side path first (see the int8 issuer)
                        tc_fence_after();
                        const uint32_t t_addr = smem_u32(lora_t), b_addr = smem_u32(lora_b);
                        #pragma unroll
                        for (int j = 0; j < 4; ++j)        // rank 64 = four K = 16 bf16 steps of a 128 B row
                            mma_f16kind_ss_pair(tmem_lora(abuf), smem_desc_kmajor(t_addr + 32 * j, 1024, kSwizzle128),
                                             smem_desc_kmajor(b_addr + 32 * j, 1024, kSwizzle128),
                                             Cfg::kIdescLora, j != 0);
                        mma_commit_pair_multicast(lora_empty_bar, 0x3);
                    }
                }
                for (int kt = 0; kt < num_kt && ok; ++kt, ++it) {
                    const int s = it % Cfg::kStages;
                    const uint32_t ph = (it / Cfg::kStages) & 1;
                    if (!mbar_wait_bounded<true>(&ready_bar[s], ph)) {
                        record_status(kStatusTimeoutMma); ok = false; break;
                    }
                    tc_fence_after();
                    const uint32_t b_hi = smem_u32(smem + s * Cfg::kStageBytes + Cfg::kABytes);
                    const int ts = it % Cfg::kTmemStages;
                    #pragma unroll
                    for (int j = 0; j < Cfg::kMmasPerStage; ++j) {
                        const uint32_t b_addr = b_hi + (j / kHalfSteps) * Cfg::kBBytes + (j % kHalfSteps) * 32;
                        const uint64_t bd = smem_desc_kmajor(b_addr, 8 * kPairBKP, kSwizzle128);
                        mma_i8_ts_pair(acc_tmem, tmem_a0 + ts * Cfg::kTmemStageCols + j * 8, bd, Cfg::kIdesc,
                                       (kt | j) != 0);
                    }
                    mma_commit_pair_multicast(&empty_bar[s], 0x3);
                    mma_commit_pair_multicast(&tmem_free_bar[ts], 0x3);
                }
                if (ok) mma_commit_pair_multicast(&acc_full_bar[abuf], 0x3);
            }
        }
    } else if (warp < 4) {
        if (!I8 && !Cfg::kA8Direct && cta == 1 && lane == 0) {
            // ---------------- forwarders (odd CTA): local expansion done -> even CTA's MMA barrier
            const uint32_t ready_leader0 = mapa_shared(smem_u32(&ready_bar[0]), 0);
            for (int it = warp - 2; it < total_it; it += 2) {
                const int s = it % kReadyStages;
                const uint32_t ph = (it / kReadyStages) & 1;
                if (!mbar_wait_bounded(&fwd_bar[s], ph)) { record_status(kStatusTimeoutExpand); break; }
                mbar_arrive_cluster(ready_leader0 + s * 8);
            }
        }
    } else if (A8 && warp < 4 + Cfg::kA8ExpWarps) {
        // ---------------- A8 weight expanders (warps 4..11): packed bytes from global
        // memory into registers one group-stage ahead, then int8 pairs (16*lo, 16*hi)
        // in column order, 128 B swizzled, into the weight slot
        const uint32_t ready_leader0 = mapa_shared(smem_u32(ready_bar), 0);
        const int group = (warp - 4) / Cfg::kA8GroupWarps;
        const int et = ((warp - 4) % Cfg::kA8GroupWarps) * 32 + lane;
        constexpr int kStride = Cfg::kA8GroupWarps * 32;
        constexpr int kPer = A8 ? Cfg::kPackedChunks / kStride : 1;   // chunks per thread and stage
        const unsigned char* wbytes = static_cast<const unsigned char*>(wraw);
        const size_t wrow_bytes = static_cast<size_t>(K >> 1);
        // chunk f of a stage: weight row f / 4, packed bytes 16 (f % 4) .. + 15 of its 64
        auto load_stage = [&](int it, uint4 (&v)[kPer]) {
            const int tp = cluster_id + (it / num_kt) * num_clusters;
            const int w_row0 = (tp / tiles_a) * BN + static_cast<int>(cta) * Cfg::kBHalf;
            const size_t col = static_cast<size_t>(it % num_kt) * Cfg::kPackedRowBytes;
            #pragma unroll
            for (int j = 0; j < kPer; ++j) {
                const int f = et + j * kStride;
                const int n = w_row0 + (f >> 2);
                v[j] = n < N ? __ldg(reinterpret_cast<const uint4*>(wbytes + static_cast<size_t>(n) * wrow_bytes +
                                                                    col + (f & 3) * 16))
                             : make_uint4(0u, 0u, 0u, 0u);
            }
        };
        uint4 nxt[kPer];
        if (group < total_it) load_stage(group, nxt);
        for (int it = group; it < total_it; it += Cfg::kA8Groups) {
            const int s = it % Cfg::kBRing;
            uint4 cur[kPer];
            #pragma unroll
            for (int j = 0; j < kPer; ++j) cur[j] = nxt[j];
            if (it + Cfg::kA8Groups < total_it) load_stage(it + Cfg::kA8Groups, nxt);
            // the weight slot's previous MMAs are done with it
            if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded<true>(&bempty_bar[s], ((it / Cfg::kBRing) & 1) ^ 1))) {
                record_status(kStatusTimeoutExpand); break;
            }
            unsigned char* dst = bexp_ring + s * Cfg::kBBytes;
            #pragma unroll
            for (int j = 0; j < kPer; ++j) {
                const int f = et + j * kStride;
                const int row = f >> 2, c = f & 3, sw = row & 7;
                const uint32_t w[4] = {cur[j].x, cur[j].y, cur[j].z, cur[j].w};
                uint32_t o[8];
                #pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const uint32_t lo = (w[e] << 4) & 0xF0F0F0F0u, hi = w[e] & 0xF0F0F0F0u;
                    o[2 * e] = __byte_perm(lo, hi, 0x5140);          // codes 8e .. 8e+3
                    o[2 * e + 1] = __byte_perm(lo, hi, 0x7362);      // codes 8e+4 .. 8e+7
                }
                unsigned char* drow = dst + row * kPairBKP;
                *reinterpret_cast<uint4*>(drow + (((2 * c) ^ sw) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
                *reinterpret_cast<uint4*>(drow + (((2 * c + 1) ^ sw) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                // the odd CTA's warps arrive on the even CTA's barrier: CTA-scope release
                // after the proxy fence (a cluster-scope release costs thousands of cycles
                // here and throttled the ring)
                if (cta == 1) mbar_arrive_remote_cta(ready_leader0 + s * 8);
                else mbar_arrive(&ready_bar[s]);
            }
        }
    } else if (!I8 && !A8 && (warp < 12 || SWAP)) {
        // expansion done for stage s: local arrive (CTA-scope release)
        uint64_t* done_bar = (cta == 0) ? ready_bar : fwd_bar;
        const int quarter = warp & 3;
        // A rows into TMEM: one row (128 packed bytes) per thread
        auto expand_a = [&](int s, int ts) {
            const int r = quarter * 32 + lane;
            const uint32_t swz = static_cast<uint32_t>(r & 7);   // 128 B swizzle: chunk ^= row % 8
            const unsigned char* row = smem + s * Cfg::kStageBytes + r * kPairBKP;
            uint32_t hi[32], lo[32];
            #pragma unroll
            for (int c = 0; c < 8; ++c) {
                const uint4 v = *reinterpret_cast<const uint4*>(row + ((c ^ swz) << 4));
                const uint32_t p[4] = {v.x, v.y, v.z, v.w};
                #pragma unroll
                for (int e = 0; e < 4; ++e) {
                    hi[4 * c + e] = p[e] & 0xF0F0F0F0u;
                    lo[4 * c + e] = (p[e] << 4) & 0xF0F0F0F0u;
                }
            }
            const uint32_t ta = tmem_a0 + (static_cast<uint32_t>(quarter * 32) << 16) + ts * Cfg::kTmemStageCols;
            __syncwarp();
            tmem_st_32x32b_x32(ta, hi);
            tmem_st_32x32b_x32(ta + 32, lo);
            tmem_st_wait();
            tc_fence_before();
        };
        // B half tile: in place (high) + second buffer (low), by `nthr` threads
        auto expand_b = [&](int s, int et, int nthr) {
            uint4* hi = reinterpret_cast<uint4*>(smem + s * Cfg::kStageBytes + Cfg::kABytes);
            uint4* lo = reinterpret_cast<uint4*>(smem + s * Cfg::kStageBytes + Cfg::kABytes + Cfg::kBBytes);
            for (int c = et; c < Cfg::kBBytes / 16; c += nthr) {
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
        };
        if constexpr (SWAP) {
            // ---------------- three groups of four warps, whole stages in turn
            const int group = (warp - 4) >> 2;
            const int et = (warp & 3) * 32 + lane;
            for (int it = group; it < total_it; it += Cfg::kExpGroups) {
                const int s = it % Cfg::kStages;
                const uint32_t ph = (it / Cfg::kStages) & 1;
                if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(&full_bar[s], ph))) {
                    record_status(kStatusTimeoutExpand); break;
                }
                const int ts = it % Cfg::kTmemStages;
                if (!__all_sync(0xFFFFFFFFu,
                                mbar_wait_bounded<true>(&tmem_free_bar[ts], ((it / Cfg::kTmemStages) & 1) ^ 1))) {
                    record_status(kStatusTimeoutExpand); break;
                }
                tc_fence_after();
                expand_a(s, ts);
                expand_b(s, et, 128);
                __syncwarp();
                if (lane == 0) mbar_arrive(&done_bar[s]);
            }
        } else if (warp < 8) {
            // ---------------- A expanders
            for (int it = 0; it < total_it; ++it) {
                const int s = it % Cfg::kStages;
                const uint32_t ph = (it / Cfg::kStages) & 1;
                if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(&full_bar[s], ph))) {
                    record_status(kStatusTimeoutExpand); break;
                }
                const int ts = it % Cfg::kTmemStages;
                if (!__all_sync(0xFFFFFFFFu,
                                mbar_wait_bounded<true>(&tmem_free_bar[ts], ((it / Cfg::kTmemStages) & 1) ^ 1))) {
                    record_status(kStatusTimeoutExpand); break;
                }
                tc_fence_after();
                expand_a(s, ts);
                __syncwarp();
                if (lane == 0) mbar_arrive(&done_bar[s]);
            }
        } else {
            // ---------------- B expanders
            for (int it = 0; it < total_it; ++it) {
                const int s = it % Cfg::kStages;
                const uint32_t ph = (it / Cfg::kStages) & 1;
                if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(&full_bar[s], ph))) {
                    record_status(kStatusTimeoutExpand); break;
                }
                expand_b(s, threadIdx.x - 256, 128);
                __syncwarp();
                if (lane == 0) mbar_arrive(&done_bar[s]);
            }
        }
    }
    if (warp >= 12) {
        // (with SWAP these warps also took their turns as expanders above)
        // ---------------- epilogue: this CTA's 128 accumulator lanes x BN columns, per tile
        const int quarter = warp & 3;
        const int et = threadIdx.x - 384;                       // 0..127
        const int r = quarter * 32 + lane;                      // row within the CTA tile
        const uint32_t acc_empty_leader0 = mapa_shared(smem_u32(acc_empty_bar), 0);
        for (int lt = 0; lt < my_tiles; ++lt) {
            const int t = cluster_id + lt * num_clusters;
            const int a_row0 = (t % tiles_a) * 256 + static_cast<int>(cta) * 128;
            const int b_tile0 = (t / tiles_a) * BN;
            const int a = a_row0 + r;                                // A row of this lane
            const bool lane_ok = a < rows_a;
            // Per-tile factors, fetched while the tile's MMAs still run: the lane's
            // row factor in a register, the BN column factors into shared memory
            // (read back as warp-wide broadcasts).
            float lane_scale = 0.0f, lane_bias = 0.0f;
            if (lane_ok && OUT != kOutS32) {
                if constexpr (SWAP) {
                    lane_scale = wscale[a];
                    lane_bias = bias.ptr != nullptr ? bias.at(a) : 0.0f;
                } else {
                    lane_scale = xscale[a];
                }
            }
            float* cscale = col_factors + (lt & 1) * (2 * BN);
            float* cbias = cscale + BN;
            if constexpr (OUT != kOutS32) {
                for (int c = et; c < BN; c += kEpiThreads) {
                    const int n = b_tile0 + c;
                    if constexpr (SWAP) {
                        cscale[c] = (n < M) ? xscale[n] : 0.0f;
                        cbias[c] = 0.0f;
                    } else {
                        cscale[c] = (n < N) ? wscale[n] : 0.0f;
                        cbias[c] = (bias.ptr != nullptr && n < N) ? bias.at(n) : 0.0f;
                    }
                }
            }
            if constexpr (STAGED) {
                // the previous tile's TMA stores must have read the staging tile
                if (et == 0) bulk_wait_group_read0();
            }
            named_barrier_sync(kEpiBarrier, kEpiThreads);
            const int abuf = lt % Cfg::kAccBufs, ause = lt / Cfg::kAccBufs;
            if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded<true>(&acc_full_bar[abuf], ause & 1))) {
                if (lane == 0) record_status(kStatusTimeoutEpilogue);
                break;
            }
            tc_fence_after();
            // two 32-column TMEM loads in flight per wait (int32 + fp32 chunk with LORA)
            constexpr int kChunks = LORA ? 1 : 2;
            #pragma unroll 1
            for (int cc = 0; cc < BN / 32; cc += kChunks) {
                uint32_t acc2[kChunks][32];
                uint32_t lora2[kChunks][32];
                __syncwarp();
                const uint32_t taddr = tmem_base + abuf * Cfg::kAccCols + (static_cast<uint32_t>(quarter * 32) << 16) + cc * 32;
                tmem_ld_32x32b_x32(taddr, acc2[0]);
                if constexpr (LORA) {
                    tmem_ld_32x32b_x32(tmem_lora(abuf) + (static_cast<uint32_t>(quarter * 32) << 16) + cc * 32, lora2[0]);
                } else {
                    tmem_ld_32x32b_x32(taddr + 32, acc2[kChunks - 1]);
                }
                tmem_ld_wait();
                #pragma unroll
                for (int h = 0; h < kChunks; ++h) {
                    uint32_t (&acc)[32] = acc2[h];
                    const int col0 = (cc + h) * 32;
                    const int b = b_tile0 + col0;                    // first B row of this chunk
                    if constexpr (OUT == kOutS32) {
                        if (!lane_ok) continue;
                        #pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            const int32_t d = static_cast<int32_t>(acc[i]) >> Cfg::kAccShift;
                            if constexpr (SWAP) {
                                if (b + i < M) reinterpret_cast<int32_t*>(out)[static_cast<size_t>(b + i) * N + a] = d;
                            } else {
                                if (b + i < N) reinterpret_cast<int32_t*>(out)[static_cast<size_t>(a) * N + b + i] = d;
                            }
                        }
                    } else if constexpr (SWAP) {
                        if (!lane_ok) continue;
                        #pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            if (b + i >= M) break;
                            const float d = static_cast<float>(static_cast<int32_t>(acc[i]) >> Cfg::kAccShift);
                            const float v = __fmul_rn(__fmul_rn(d, cscale[col0 + i]), lane_scale);
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
                            const float d = static_cast<float>(static_cast<int32_t>(acc[i]) >> Cfg::kAccShift);
                            v[i] = __fmul_rn(__fmul_rn(d, lane_scale), cscale[col0 + i]);
                        }
                        if constexpr (LORA) {
                            // ((D xs) ws + bias) + scale * L: bias is added here, not at the store
                            #pragma unroll
                            for (int i = 0; i < 32; ++i)
                                v[i] = __fadd_rn(__fadd_rn(v[i], cbias[col0 + i]),
                                                 __fmul_rn(__uint_as_float(lora2[h][i]), lora_scale));
                        }
                        // with LORA the bias is already in v
                        const float* vbias = LORA ? nullptr : cbias + col0;
                        auto bias_of = [&](int i) -> float {
                            if constexpr (LORA) return 0.0f; else return cbias[col0 + i];
                        };
                        if constexpr (STAGED) {
                            // 32 bf16 = four 16-byte chunks of a 64-column, 128 B-swizzled box
                            unsigned char* box = staging + (col0 >> 6) * (128 * 128);
                            const int c0 = (col0 & 63) >> 3;
                            #pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                uint4 pk;
                                float w[8];
                                #pragma unroll
                                for (int e = 0; e < 8; ++e)
                                    w[e] = LORA ? v[8 * q + e] : __fadd_rn(v[8 * q + e], bias_of(8 * q + e));
                                __nv_bfloat162 p0 = __floats2bfloat162_rn(w[0], w[1]);
                                __nv_bfloat162 p1 = __floats2bfloat162_rn(w[2], w[3]);
                                __nv_bfloat162 p2 = __floats2bfloat162_rn(w[4], w[5]);
                                __nv_bfloat162 p3 = __floats2bfloat162_rn(w[6], w[7]);
                                memcpy(&pk.x, &p0, 4); memcpy(&pk.y, &p1, 4);
                                memcpy(&pk.z, &p2, 4); memcpy(&pk.w, &p3, 4);
                                *reinterpret_cast<uint4*>(box + r * 128 + (((c0 + q) ^ (r & 7)) << 4)) = pk;
                            }
                        } else {
                            if (!lane_ok) continue;
                            if (peers.count == 0) {
                                store_row32<OUT>(out, static_cast<size_t>(a) * N + b, b, N, v, vbias);
                            } else {
                                // column block of a wider [M, ldo] output on every rank
                                const size_t o = static_cast<size_t>(a) * peers.ldo + peers.col0 + b;
                                #pragma unroll 1
                                for (int d = 0; d < peers.count; ++d) store_row32<OUT>(peers.ptr[d], o, b, N, v, vbias);
                            }
                        }
                    }
                }
            }
            // accumulator drained: hand TMEM back to the MMA issuer
            tc_fence_before();
            if constexpr (STAGED) fence_proxy_async_smem();
            named_barrier_sync(kEpiBarrier, kEpiThreads);
            if (et == 0) {
                if (cta == 0) mbar_arrive(&acc_empty_bar[abuf]);
                else mbar_arrive_cluster(acc_empty_leader0 + abuf * 8);
                if constexpr (STAGED) {
                    for (int bx = 0; bx < BN / 64; ++bx) {
                        if (b_tile0 + bx * 64 < N && a_row0 < M)
                            tma_store_2d(&tmap_out, staging + bx * (128 * 128), b_tile0 + bx * 64, a_row0);
                    }
                    bulk_commit_group();
                }
            }
        }
        if constexpr (STAGED) {
            if (et == 0) bulk_wait_group0();
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
