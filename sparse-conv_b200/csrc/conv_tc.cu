// tcgen05 / TMEM implicit-GEMM submanifold convolution for sm_100a (fp16 / bf16 in,
// fp32 accumulate). Replaces the reference's Triton kernel (implicit_gemm.py:8-57), which
// runs 32x32x16 tiles over every one of the V*ceil(Ci/16) K-steps and reloads the neighbour
// index column per step.
//
// A tile is 128 consecutive entries of the voxel order produced by the map build, so its rows
// share most of their offset masks; the OR of the 128 masks selects the offsets the tile needs.
// The work of a CTA is a stream of steps, one per (tile, active offset v, K chunk of <= 64
// channels). One CTA = NG + 6 warps (NG = 4 or 8 gatherers) with fixed roles, synchronised
// only through mbarriers:
//   warp 0    scheduler: per tile, loads its rows (order) and mask words, ORs them, and splits
//             the active offsets into contexts of <= 16; for each context it loads the 16 x 128
//             neighbour indices (only where a row's mask bit is set; -1 elsewhere) into one of
//             three context buffers by cp.async and hands the buffer over;
//   warps 1..NG gatherers: warp g owns tile rows (128/NG)g .. and runs its own cp.async pipeline:
//             per step, groups of KC/8 lanes copy whole feature rows (16 B per lane, zero-fill
//             for a missing neighbour) into the A stage, straight into the 32/64/128-byte
//             swizzled K-major layout; a step is signalled on the stage's "full" mbarrier once
//             its copies have landed (cp.async.wait_group, proxy fence, arrive), D-1 steps
//             behind the issue, so several steps per warp are in flight; warp 1 lane 0 also
//             loads W[:, v, kc] into the B stage by TMA (bytes counted on the same mbarrier);
//   warp NG+1 MMA: one thread waits for a full stage (rows and weights), issues KC/16
//             tcgen05.mma (M=128, N=Co, K=16) into the tile's TMEM accumulator, and commits to
//             the stage's "empty" mbarrier (and, after a tile's last step, to the accumulator's);
//   warps NG+2..NG+5 epilogue: TMEM lanes 32*(w%4).. -> registers, + bias, one rounding, one
//             16-byte store per 8 outputs; two accumulators alternate so the next tile's MMAs
//             run while a tile is written out.
// Gatherers never wait on the scheduler while holding landed-but-unsignalled steps (they
// flush first), so no wait depends on itself. Every wait is bounded (2 s by default, a kernel
// argument); a timeout sets an abort flag that ends every role, raises
// SPCONV_STATUS_WAIT_TIMEOUT, and the CTA waits (bounded) for its copies, weight loads, MMAs
// and accumulator commits before it frees TMEM and exits.
#include <cuda.h>
#include <mutex>

#include "common.cuh"
#include "conv_internal.h"

namespace spconv {

constexpr int kTileM = 128;
// Index contexts the scheduler keeps loading before it publishes the oldest (see the
// scheduler): 1 publishes each context when the next one has been issued.
#ifndef SPCONV_TC_SCHED_PEND
#define SPCONV_TC_SCHED_PEND 1
#endif
// Channels per K step (the A row width: 64 bf16 = one 128-byte swizzle row).
#ifndef SPCONV_TC_MAX_KC
#define SPCONV_TC_MAX_KC 64
#endif
#ifndef SPCONV_TC_ROWS_MAX_KC
#define SPCONV_TC_ROWS_MAX_KC 32
#endif
#ifndef SPCONV_TC_CHUNK
#define SPCONV_TC_CHUNK 16
#endif
#ifndef SPCONV_TC_2CTA_BUDGET_KB
#define SPCONV_TC_2CTA_BUDGET_KB 110
#endif
constexpr int kChunk = SPCONV_TC_CHUNK;   // active offsets per context (a power of two <= 16)
constexpr int kNPitch = kChunk + 1; // words per row in a context buffer (conflict-free both ways)
constexpr int kRowWindow = 32;      // words per staged index row: a 128-byte aligned window
constexpr int kRowsMaxV = 28;       // V for which a voxel's whole index row fits one window
constexpr int kActMax = 32;         // active offsets per context buffer
// Index-context buffers (how far the scheduler may run ahead of the gatherers), by launch
// shape. Measured on B200, conv alone on cached maps: one CTA per SM, 3 -> 4 -> 5 buffers took
// the indoor conv (C=64) from 843 to 810 to 792 us (wide5, C=128: 851 -> 840 us); a sixth
// would cost a pipeline stage. Two CTAs per SM (cube, C=32): 4 buffers 32.1 -> 31.1 us, 5 lose
// occupancy (38 us).
#ifndef SPCONV_TC_CTX_BUFS_1CTA
#define SPCONV_TC_CTX_BUFS_1CTA 5
#endif
// Stages (A + B tile) up to this many bytes run two CTAs per SM, larger ones one. Random
// 128-byte row gathers by cp.async reach about twice the rate with two CTAs per SM as with one
// at the same warp count (B200, indoor index stream: 4.7-5.0 TB/s with one CTA of 4, 8 or 16
// warps, 8.4-8.9 TB/s with two), so C = 64 stages (24 KB: 3 stages, 4 index contexts) run two
// CTAs: indoor conv 793 -> 605 us.
#ifndef SPCONV_TC_2CTA_MAX_STAGE
#define SPCONV_TC_2CTA_MAX_STAGE (24 * 1024)
#endif
#ifndef SPCONV_TC_CTX_BUFS_2CTA
#define SPCONV_TC_CTX_BUFS_2CTA 4
#endif
constexpr int kTileRing = 4;        // tiles whose rows the epilogue may still need
constexpr int kMaxMaskWords = 4;    // offset masks are used for V <= 128 (else all offsets run)
constexpr int kMaxStages = 8;
// Warp roles for NG gatherer warps: scheduler 0, gatherers 1..NG, MMA NG+1, epilogue NG+2..NG+5.
constexpr int kWarpSched = 0, kWarpGather = 1;
template <int NG> struct TcRoles {
    static constexpr int kWarpMma = NG + 1, kWarpEpi = NG + 2;
    static constexpr int kWarps = NG + 6, kThreads = kWarps * 32;
    static constexpr int kRowsPerWarp = kTileM / NG;
};
constexpr uint32_t kInfoFirst = 1u << 30, kInfoLast = 1u << 31, kInfoEnd = 0x3fffffffu;
constexpr int kCtxFirst = 1, kCtxLast = 2, kCtxRows = 4, kCtxEnd = 8;
// Tiles with more active offsets than this stage whole index rows (when V <= kRowsMaxV): one
// 128-byte window per voxel costs about what a context of 5..8 offsets does.
constexpr int kRowsMinAct = 9;
// Split tiles (SPLIT kernels): of the first kSplitMaxTiles tiles taken (the heaviest: the voxel
// order sorts voxels by neighbour count), those with more than kSplitMinAct active offsets run
// as two work items, each over one half of the tile's offsets, on different CTAs.
constexpr int kSplitMinAct = 16;
constexpr int kSplitMaxTiles = 256;
constexpr int kTileEnd = -2;        // tile-ring info of the epilogue's end marker

template <int CI, int CO>
struct TcCfg {
    static constexpr int KC = CI > SPCONV_TC_MAX_KC ? SPCONV_TC_MAX_KC : CI;   // channels per K step
    static constexpr int NKC = CI / KC;
    static constexpr int kRowBytes = KC * 2;               // = swizzle width (32, 64, 128)
    static constexpr int kLanesPerRow = kRowBytes / 16;    // = rows per lane in a gather warp
    static constexpr int kABytes = kTileM * kRowBytes;
    static constexpr int kBBytes = CO * kRowBytes;
    static constexpr int kStageBytes = kABytes + kBBytes;
    // Whole-row staging pays where the gatherers are fast relative to the index loads (rows of
    // at most 64 bytes); wider rows keep the smaller per-offset buffers and one more stage.
    static constexpr bool kRows = CI <= SPCONV_TC_ROWS_MAX_KC;
    static constexpr bool kTwoCtas = kABytes + kBBytes <= SPCONV_TC_2CTA_MAX_STAGE;   // two CTAs per SM
    static constexpr int kCtxBufs = kTwoCtas ? SPCONV_TC_CTX_BUFS_2CTA : SPCONV_TC_CTX_BUFS_1CTA;
    // mbarriers: full[8] empty[8] cfull[ctx] cempty[ctx] afull[2] aempty[2] tfull[ring] tempty[ring]
    static constexpr int kNumBars = 16 + 2 * kCtxBufs + 4 + 2 * kTileRing;
    static constexpr int kBufWords = kTileM * (kRows ? kRowWindow : kNPitch);   // one context buffer
    static constexpr int kNBytes = kCtxBufs * kBufWords * 4;
    static_assert(kRowWindow >= kNPitch, "context buffer");
    static constexpr int kSchedBytes = kTileM + kCtxBufs * kTileM;           // active list, row shifts
    static constexpr int kFixedBytes = kNBytes + kSchedBytes + kCtxBufs * kActMax * 4 + kCtxBufs * 16 +
                                       kTileRing * kTileM * 4 + kTileRing * 4 + kMaxStages * 4 + kNumBars * 8 + 16;
    // Small stages: about 110 KB per CTA (two CTAs per SM); large: one CTA per SM.
    static constexpr int kBudget = kTwoCtas ? SPCONV_TC_2CTA_BUDGET_KB * 1024 : 219 * 1024;
    static constexpr int kMinBlocks = kTwoCtas ? 2 : 1;   // registers for two CTAs
    static constexpr int kStagesFit = (kBudget - kFixedBytes - 1024) / kStageBytes;
    static constexpr int kStages = kStagesFit > kMaxStages ? kMaxStages : (kStagesFit < 3 ? 3 : kStagesFit);
    static constexpr int kDepth = kStages - 1;             // cp.async groups in flight per gatherer
    // shared memory layout (offsets from a 1024-byte aligned base)
    static constexpr int kOffA = 0;
    static constexpr int kOffB = kOffA + kStages * kABytes;
    static constexpr int kOffN = kOffB + kStages * kBBytes;
    static constexpr int kOffTact = kOffN + kNBytes;
    static constexpr int kOffMis = kOffTact + kTileM;
    static constexpr int kOffAct = kOffMis + kCtxBufs * kTileM;
    static constexpr int kOffCInfo = kOffAct + kCtxBufs * kActMax * 4;
    static constexpr int kOffTRow = kOffCInfo + kCtxBufs * 16;
    static constexpr int kOffTInfo = kOffTRow + kTileRing * kTileM * 4;
    static constexpr int kOffInfo = kOffTInfo + kTileRing * 4;
    static constexpr int kOffBar = kOffInfo + kMaxStages * 4;
    static constexpr int kOffMisc = kOffBar + kNumBars * 8;
    static constexpr int kSmemBytes = kOffMisc + 16 + 1024;  // + alignment slack
    static constexpr int kTmemCols = 2 * CO < 32 ? 32 : 2 * CO;   // two accumulators
    static constexpr int kMaxCtasByTmem = 512 / kTmemCols;
    static_assert(kSmemBytes <= 227 * 1024, "shared memory");
    static_assert(kABytes % 1024 == 0 && kBBytes % (8 * kRowBytes) == 0, "swizzle atom alignment");
    static_assert(kDepth >= 2 && kDepth < kStages, "gather pipeline depth");
};

template <int N>
__device__ __forceinline__ void cp_async_wait_upto(int pending) {
    // wait until at most `pending` groups are outstanding (at most N: waiting for more is safe)
    if (pending >= N) { cp_async_wait<N>(); return; }
    if constexpr (N > 0) cp_async_wait_upto<N - 1>(pending);
}

template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}

__device__ __forceinline__ uint32_t full_mask_word(int w, int V) {
    const int lo = w * 32;
    return (V - lo >= 32) ? 0xffffffffu : ((1u << (V - lo)) - 1u);
}

__device__ __forceinline__ uint32_t sel4(uint32_t a, uint32_t b, uint32_t c, uint32_t d, int w) {
    return w == 0 ? a : (w == 1 ? b : (w == 2 ? c : d));
}

template <int CI, int CO, typename T, bool FLIP, int NG, bool SPLIT>
__global__ void __launch_bounds__(TcRoles<NG>::kThreads, TcCfg<CI, CO>::kMinBlocks)
conv_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const T *__restrict__ feats,
               const T *__restrict__ bias, const int32_t *__restrict__ nbr,
               const uint32_t *__restrict__ masks, const int32_t *__restrict__ order,
               T *__restrict__ out, int64_t M, int V, int MW, int MWS, int num_tiles, int row_mode,
               int32_t *status, uint64_t wait_ns, int split_tiles, float *__restrict__ partials,
               int *__restrict__ split_cnt) {
    using Cfg = TcCfg<CI, CO>;
    using Roles = TcRoles<NG>;
    constexpr int S = Cfg::kStages, KC = Cfg::KC, NKC = Cfg::NKC, RB = Cfg::kRowBytes;
    constexpr int LPR = Cfg::kLanesPerRow, D = Cfg::kDepth, kCtxBufs = Cfg::kCtxBufs;
    constexpr int kWarpMma = Roles::kWarpMma, kWarpEpi = Roles::kWarpEpi, RPW = Roles::kRowsPerWarp;
    // rows per lane: each warp instruction moves 32 / LPR whole rows, NQ instructions per step
    constexpr int NQ = RPW * LPR / 32;
    static_assert(NQ >= 1 && NQ * 32 == RPW * LPR && (NQ & (NQ - 1)) == 0, "gatherer row split");
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const uint32_t sA = smem_u32(base + Cfg::kOffA), sB = smem_u32(base + Cfg::kOffB);
    int32_t *s_n = reinterpret_cast<int32_t *>(base + Cfg::kOffN);        // [ctx][kBufWords]: rows at pitch kNPitch or kRowWindow
    uint8_t *s_mis = base + Cfg::kOffMis;                                 // [ctx][row]: word rotation of the staged row
    uint8_t *s_tact = base + Cfg::kOffTact;                               // scheduler: tile's active offsets
    int32_t *s_act = reinterpret_cast<int32_t *>(base + Cfg::kOffAct);    // [ctx][i] -> v
    int4 *s_cinfo = reinterpret_cast<int4 *>(base + Cfg::kOffCInfo);      // [ctx] {k, cnt, flags}
    int32_t *s_trow = reinterpret_cast<int32_t *>(base + Cfg::kOffTRow);  // [tile % ring][row]
    int32_t *s_tinfo = reinterpret_cast<int32_t *>(base + Cfg::kOffTInfo); // [tile % ring]: split slot*2+half, -1, end
    uint32_t *s_info = reinterpret_cast<uint32_t *>(base + Cfg::kOffInfo);
    uint64_t *bar = reinterpret_cast<uint64_t *>(base + Cfg::kOffBar);
    uint64_t *full = bar, *empty = bar + 8, *cfull = bar + 16, *cempty = cfull + kCtxBufs;
    uint64_t *afull = cempty + kCtxBufs, *aempty = afull + 2, *tfull = aempty + 2, *tempty = tfull + kTileRing;
    uint32_t *s_tmem = reinterpret_cast<uint32_t *>(base + Cfg::kOffMisc);
    volatile int *s_abort = reinterpret_cast<volatile int *>(base + Cfg::kOffMisc + 4);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&full[s]), NG + 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int c = 0; c < kCtxBufs; ++c) {
            mbar_init(smem_u32(&cfull[c]), 1);
            mbar_init(smem_u32(&cempty[c]), NG);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&afull[b]), 1);
            mbar_init(smem_u32(&aempty[b]), 4);
        }
        for (int t = 0; t < kTileRing; ++t) {
            mbar_init(smem_u32(&tfull[t]), 1);
            mbar_init(smem_u32(&tempty[t]), 4);
        }
        *s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == kWarpMma) {
        tmem_alloc(smem_u32(s_tmem), Cfg::kTmemCols);
        tmem_relinquish();
    }
    if (warp == kWarpGather && lane == 0) tma_prefetch_desc(&tmap_w);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;
    grid_dependency_wait();                  // the map build's order, masks and map

    // Tiles are taken from the end of the voxel order first: voxels with the most neighbours
    // sort last, so the tiles with the most active offsets start earliest. CTA c takes work
    // items c + kG (k >= 1) after a first item G-1-c: the CTAs that get one item fewer (the last
    // round is partial) take the heaviest first items. Item i is the tile of rank i (rank 0 =
    // the last 128 voxels of the order); with SPLIT, the first split_tiles ranks have two items
    // each (2r: the first half of the tile's active offsets, 2r+1: the second half), which run
    // on different CTAs when the tile has more than kSplitMinAct active offsets.
    const int G = gridDim.x;
    const int R = SPLIT ? split_tiles : 0;
    const int n_items = num_tiles + R;
    const int nt = (int)blockIdx.x < n_items ? (n_items - 1 - (int)blockIdx.x) / G + 1 : 0;
    auto tile_id = [&](int k) { return k == 0 ? G - 1 - (int)blockIdx.x : (int)blockIdx.x + k * G; };
    auto item_rank = [&](int item) { return item < 2 * R ? item >> 1 : item - R; };
    auto item_half = [&](int item) { return item < 2 * R ? (item & 1) : -1; };
    const bool use_masks = MWS > 0;
    auto wait = [&](uint64_t *b, uint32_t parity) -> bool {
        return mbar_wait_or_abort(smem_u32(b), parity, s_abort, wait_ns);
    };

    if (warp == kWarpSched) {
        // ------------------------------------------------------------------ scheduler
        // Lane l handles rows 4l..4l+3 of each tile. Rows are loaded three tiles ahead and
        // mask words two tiles ahead, so their latency hides behind the tiles in between.
        auto load_rows = [&](int k, int32_t (&r)[4]) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                r[j] = -1;
                if (k < nt) {
                    const int64_t p = (int64_t)(num_tiles - 1 - item_rank(tile_id(k))) * kTileM + 4 * lane + j;
                    if (p < M) r[j] = order ? __ldg(order + p) : (int32_t)p;
                }
            }
        };
        auto load_masks = [&](int32_t (&r)[4], uint32_t (&m)[4][kMaxMaskWords]) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if ((uint32_t)r[j] >= (uint32_t)M) r[j] = -1;   // order entries outside the table are ignored
#pragma unroll
                for (int w = 0; w < kMaxMaskWords; ++w)
                    m[j][w] = (w < MWS && r[j] >= 0) ? __ldg(masks + (int64_t)r[j] * MW + w) : 0u;
            }
        };
        int32_t rA[4], rB[4], rC[4];
        uint32_t mA[4][kMaxMaskWords], mB[4][kMaxMaskWords];
        load_rows(0, rA);
        load_rows(1, rB);
        load_rows(2, rC);
        load_masks(rA, mA);
        load_masks(rB, mB);
        int g = 0;                           // contexts handed out
        // Context buffers whose index loads are in flight, oldest first. After each new context
        // the oldest is published once at most kPend groups remain outstanding, so up to
        // kPend + 1 contexts load at once. kPend < kCtxBufs: a buffer the scheduler waits to
        // reuse was published at least one context earlier, and (kTileRing = 4 > kPend) the
        // tile whose ring slot it waits for has every context published.
        constexpr int kPend = SPCONV_TC_SCHED_PEND < kCtxBufs ? SPCONV_TC_SCHED_PEND : kCtxBufs - 1;
        static_assert(kPend >= 1 && kPend < kTileRing, "scheduler look-ahead");
        // Contexts gp .. g-1 are issued and not yet published (buffer = context % kCtxBufs).
        int gp = 0;
        bool ok = true;
        auto publish_oldest = [&]() {
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&cfull[gp % kCtxBufs]));
            ++gp;
        };
        auto push_pending = [&]() {          // context g's cp.async group is committed
            if (g + 1 - gp > kPend) {
                cp_async_wait<kPend>();
                publish_oldest();
            }
        };
        auto publish_all = [&]() {           // after the last context (g = contexts issued)
            cp_async_wait<0>();
            while (gp < g) publish_oldest();
        };
        int kt = 0;                          // tiles (non-empty items) handed to the MMA and epilogue
        for (int k = 0; k < nt && ok; ++k) {
            uint32_t tm[kMaxMaskWords];
            int nact = 0;
#pragma unroll
            for (int w = 0; w < kMaxMaskWords; ++w) {
                uint32_t m = 0u;
                if (w < MWS) {
                    m = __reduce_or_sync(0xffffffffu, mA[0][w] | mA[1][w] | mA[2][w] | mA[3][w]) &
                        full_mask_word(w, V);
                }
                tm[w] = m;
                nact += __popc(m);
            }
            if (!use_masks) nact = V;
            const bool fake = nact == 0;     // no offset: one step of zeros gives the bias rows
            // This item's share of the tile's active offsets: [lo, hi).
            int lo = 0, hi = nact, tinfo = -1;
            bool skip = false;
            if (SPLIT) {
                const int item = tile_id(k), half = item_half(item);
                if (half >= 0) {
                    if (nact > kSplitMinAct) {
                        const int h = (nact + 1) >> 1;
                        if (half == 0) hi = h;
                        else lo = h;
                        tinfo = item_rank(item) * 2 + half;
                    } else if (half == 1) {
                        skip = true;         // a light tile runs whole as its first item
                    }
                }
            }
            if (!skip) {
            int left = fake ? 1 : hi - lo;

            const int t = kt % kTileRing;
            if (kt >= kTileRing && !wait(&tempty[t], (uint32_t)(((kt / kTileRing) - 1) & 1))) { ok = false; break; }
            *reinterpret_cast<int4 *>(&s_trow[t * kTileM + 4 * lane]) = make_int4(rA[0], rA[1], rA[2], rA[3]);
            if (lane == 0) s_tinfo[t] = tinfo;
            {
                int base_v = 0;
#pragma unroll
                for (int w = 0; w < kMaxMaskWords; ++w) {
                    if (w < MWS) {
                        // active offsets in ascending order: lane b writes bit b of this word
                        // (FLIP: offset V-1-u for mask bit u, so the list is reversed)
                        if ((tm[w] >> lane) & 1u) {
                            const int pos = base_v + __popc(tm[w] & ((1u << lane) - 1u));
                            if (FLIP) s_tact[nact - 1 - pos] = (uint8_t)(V - 1 - (w * 32 + lane));
                            else s_tact[pos] = (uint8_t)(w * 32 + lane);
                        }
                        base_v += __popc(tm[w]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&tfull[t]));

            int c0 = lo;                     // first active offset of the next context
            bool first = true;
            if (Cfg::kRows && row_mode && hi - lo >= kRowsMinAct) {
                // One context per tile: stage every voxel's whole index row (V <= 28 words) as a
                // 128-byte aligned window, 8 lanes per row, 16 bytes per lane. Chunk c of row r
                // lands in slot (c + rot) % 8, rot = (r + r/8) % 8, so word j of the row sits at
                // (j + shift + 4 rot) % 32 with shift = the row's offset in its window; that
                // rotation is kept per row. Rows without a voxel hold -1 throughout.
                const int cb = g % kCtxBufs;
                if (g >= kCtxBufs && !wait(&cempty[cb], (uint32_t)(((g / kCtxBufs) - 1) & 1))) { ok = false; break; }
                const int cnt = left;
                if (lane < cnt) s_act[cb * kActMax + lane] = fake ? 0 : (use_masks ? (int)s_tact[lo + lane] : lo + lane);
                const char *nb = reinterpret_cast<const char *>(nbr);
                const int64_t nbytes = M * (int64_t)V * 4;
                const int c = lane & 7, rs = lane >> 3;
#pragma unroll 4
                for (int it = 0; it < kTileM / 4; ++it) {
                    const int r = 4 * it + rs;
                    const int32_t row = s_trow[t * kTileM + r];
                    int32_t *wrow = &s_n[(cb * kTileM + r) * kRowWindow];
                    if (row < 0 || fake) {
                        if (c == 0) s_mis[cb * kTileM + r] = 0;
                        *reinterpret_cast<int4 *>(wrow + 4 * c) = make_int4(-1, -1, -1, -1);
                        continue;
                    }
                    const int rot = (r + (r >> 3)) & 7;
                    const int64_t a0 = (int64_t)row * V * 4;
                    const int64_t ws = a0 & ~(int64_t)15;
                    const int shift = (int)(a0 - ws) >> 2;
                    if (c == 0) s_mis[cb * kTileM + r] = (uint8_t)((shift + 4 * rot) & 31);
                    if (c < (shift * 4 + V * 4 + 15) >> 4) {
                        const int64_t so = ws + 16 * c;
                        const uint32_t dst = smem_u32(wrow + ((c + rot) & 7) * 4);
                        if (so + 16 <= nbytes) {
                            cp_async_16(dst, nb + so, 16u);
                        } else {                 // the map's last bytes: word by word, in bounds
                            for (int q = 0; q < 4; ++q)
                                if (so + 4 * q + 4 <= nbytes) cp_async_4(dst + 4 * q, nb + so + 4 * q);
                        }
                    }
                }
                cp_async_commit();
                left = 0;
                if (lane == 0) s_cinfo[cb] = make_int4(kt, cnt, kCtxFirst | kCtxLast | kCtxRows, 0);
                push_pending();
                ++g;
            }
            while (left > 0) {
                const int cnt = left < kChunk ? left : kChunk;
                const int cb = g % kCtxBufs;
                if (g >= kCtxBufs && !wait(&cempty[cb], (uint32_t)(((g / kCtxBufs) - 1) & 1))) { ok = false; break; }
                // P = cnt rounded up to a power of two lanes share one voxel's index row: lane l
                // loads offset slot i = l % P of rows (32/P)*kk + l/P, so one warp instruction
                // touches the index rows of 32/P voxels rather than 32.
                const int lp = cnt > 1 ? 32 - __clz(cnt - 1) : 0;        // log2(P)
                const int i = lane & ((1 << lp) - 1);
                int v = 0;
                if (!fake && i < cnt) v = use_masks ? (int)s_tact[c0 + i] : c0 + i;
                if (lane < cnt) s_act[cb * kActMax + lane] = v;
                int32_t *dn = &s_n[cb * Cfg::kBufWords + i];
                // A row's map entry is -1 where its mask bit is clear, so no per-row mask test is
                // needed: the lanes of one row fetch the same cache line(s) either way.
                const int32_t *nv = nbr + (FLIP ? V - 1 - v : v);
                auto load_index = [&](int r) {
                    const int32_t row = s_trow[t * kTileM + r];
                    int32_t *d = dn + r * kNPitch;
                    if (row >= 0 && !fake) cp_async_4(smem_u32(d), nv + (int64_t)row * V);
                    else *d = -1;
                };
                if (i < cnt) {
                    if (lp == 4) {                                       // full contexts: fixed trip count
#pragma unroll 8
                        for (int kk = 0; kk < kTileM / 2; ++kk) load_index(2 * kk + (lane >> 4));
                    } else {
                        const int rpi = 32 >> lp;                        // rows per warp instruction
#pragma unroll 4
                        for (int r = lane >> lp; r < kTileM; r += rpi) load_index(r);
                    }
                }
                cp_async_commit();
                c0 += cnt;
                left -= cnt;
                if (lane == 0) s_cinfo[cb] = make_int4(kt, cnt, (first ? kCtxFirst : 0) | (left == 0 ? kCtxLast : 0), 0);
                first = false;
                push_pending();
                ++g;
            }
            if (!ok) break;
            ++kt;
            }                                // !skip
            // next item: rows of k+3 and masks of k+2 start loading now
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                rA[j] = rB[j];
                rB[j] = rC[j];
#pragma unroll
                for (int q = 0; q < kMaxMaskWords; ++q) mA[j][q] = mB[j][q];
            }
            load_masks(rB, mB);
            load_rows(k + 3, rC);
        }
        publish_all();
        if (SPLIT && ok) {                   // end marker for the epilogue (item count varies)
            const int t = kt % kTileRing;
            if (kt < kTileRing || wait(&tempty[t], (uint32_t)(((kt / kTileRing) - 1) & 1))) {
                if (lane == 0) s_tinfo[t] = kTileEnd;
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&tfull[t]));
            } else {
                ok = false;
            }
        }
        if (ok) {                            // end marker for the gatherers and the MMA
            const int cb = g % kCtxBufs;
            if (g < kCtxBufs || wait(&cempty[cb], (uint32_t)(((g / kCtxBufs) - 1) & 1))) {
                if (lane == 0) s_cinfo[cb] = make_int4(0, 0, kCtxEnd, 0);
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&cfull[cb]));
            }
        }
        cp_async_wait_all();
    } else if (warp >= kWarpGather && warp < kWarpGather + NG) {
        // ------------------------------------------------------------------ gatherers
        // Warp g owns tile rows RPW*g .. RPW*g + RPW - 1. Lane L copies chunk L % LPR of rows
        // RPW*g + (L / LPR) * NQ + q, q < NQ: each warp instruction moves 32 / LPR whole rows,
        // and a lane's NQ neighbour indices are consecutive in the context buffer.
        const int gw = warp - kWarpGather;
        const bool b_loader = gw == 0 && lane == 0;
        const int chunk = lane % LPR;
        const int row0 = RPW * gw + (lane / LPR) * NQ;       // first of this lane's rows
        uint32_t dst[NQ];
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
            const int r = row0 + q;
            dst[q] = (uint32_t)(r * RB + ((chunk ^ ((r * RB >> 7) & (LPR - 1))) << 4));
        }
        int g = 0, step = 0, sig = 0;       // contexts consumed, steps issued, steps signalled
        bool ok = true;
        auto signal_one = [&]() {            // the oldest unsignalled step has landed
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&full[sig % S]));
            ++sig;
        };
        auto flush = [&]() {
            cp_async_wait<0>();
            while (sig < step) signal_one();
        };
        for (;;) {
            const int cb = g % kCtxBufs;
            const uint32_t cpar = (uint32_t)((g / kCtxBufs) & 1);
            if (!mbar_test(smem_u32(&cfull[cb]), cpar)) flush();   // never wait on the scheduler with steps unsignalled
            if (!wait(&cfull[cb], cpar)) { ok = false; break; }
            const int4 ci = s_cinfo[cb];
            if (ci.z & kCtxEnd) break;
            const int k = ci.x, cnt = ci.y;
            const bool cfirst = (ci.z & kCtxFirst) != 0, clast = (ci.z & kCtxLast) != 0;
            const bool crows = (ci.z & kCtxRows) != 0;
            // row mode: the rotations of this lane's NQ rows, one byte each
            uint32_t rotw[(NQ + 3) / 4];
            if (Cfg::kRows && crows) {
                if constexpr (NQ >= 4) {
#pragma unroll
                    for (int w = 0; w < NQ / 4; ++w)
                        rotw[w] = reinterpret_cast<const uint32_t *>(s_mis + cb * kTileM + row0)[w];
                } else if constexpr (NQ == 2) {
                    rotw[0] = *reinterpret_cast<const uint16_t *>(s_mis + cb * kTileM + row0);
                } else {
                    rotw[0] = s_mis[cb * kTileM + row0];
                }
            }
            const int32_t *rowp = &s_n[(cb * kTileM + row0) * kRowWindow];
            for (int i = 0; i < cnt && ok; ++i) {
                const int v = s_act[cb * kActMax + i];
                int32_t n[NQ];
                if (Cfg::kRows && crows) {
                    const int vc = FLIP ? V - 1 - v : v;      // the map column of offset v
#pragma unroll
                    for (int q = 0; q < NQ; ++q)
                        n[q] = rowp[q * kRowWindow + ((vc + (int)(rotw[q >> 2] >> (8 * (q & 3)))) & 31)];
                } else {
                    const int32_t *np = &s_n[cb * Cfg::kBufWords + row0 * kNPitch + i];
#pragma unroll
                    for (int q = 0; q < NQ; ++q) n[q] = np[q * kNPitch];
                }
#pragma unroll
                for (int kc = 0; kc < NKC; ++kc) {
                    const int s = step % S, u = step / S;
                    if (u > 0 && !wait(&empty[s], (uint32_t)((u - 1) & 1))) { ok = false; break; }
                    if (b_loader) {
                        s_info[s] = (uint32_t)k | ((cfirst && i == 0 && kc == 0) ? kInfoFirst : 0u) |
                                    ((clast && i == cnt - 1 && kc == NKC - 1) ? kInfoLast : 0u);
                        mbar_arrive_expect_tx(smem_u32(&full[s]), (uint32_t)Cfg::kBBytes);
                        tma_load_2d(sB + s * Cfg::kBBytes, &tmap_w, v * CI + kc * KC, 0, smem_u32(&full[s]));
                    }
                    const uint32_t a_st = sA + s * Cfg::kABytes;
                    const T *src = feats + kc * KC + chunk * 8;
#pragma unroll
                    for (int q = 0; q < NQ; ++q) {
                        // rows outside the feature table (and missing neighbours) read as zeros
                        const bool have = (uint32_t)n[q] < (uint32_t)M;
                        cp_async_16(a_st + dst[q], src + (int64_t)(have ? n[q] : 0) * CI, have ? 16u : 0u);
                    }
                    cp_async_commit();
                    ++step;
                    if (step - sig > D - 1) {   // keep D-1 steps in flight; the oldest has landed
                        cp_async_wait<D - 1>();
                        signal_one();
                    }
                }
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&cempty[cb]));
            ++g;
        }
        if (ok) {
            flush();
            // end marker: one more "step" carrying no data
            const int s = step % S, u = step / S;
            if (u == 0 || wait(&empty[s], (uint32_t)((u - 1) & 1))) {
                if (b_loader) {
                    s_info[s] = kInfoEnd;
                    mbar_arrive(smem_u32(&full[s]));
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&full[s]));
            }
        }
        cp_async_wait_all();
        if (!ok && b_loader) {
            // wait (bounded) for the weight loads of the last step issued on each stage: the
            // stage's phase completes once its bytes have landed, unless a gatherer that gave
            // up never arrives on it; then kTmaDrainNs bounds the wait
            for (int q = 1; q <= S && q <= step; ++q) {
                const int st = step - q;
                mbar_wait_bounded(smem_u32(&full[st % S]), (uint32_t)((st / S) & 1), kTmaDrainNs);
            }
        }
    } else if (warp == kWarpMma) {
        // ------------------------------------------------------------------ MMA
        if (lane == 0) {
            const uint32_t idesc = instr_desc_f16(dtype_traits<T>::mma_format, kTileM, CO);
            int step = 0;
            int acc0 = 0, acc1 = 0;          // commits made to afull[0], afull[1]
            for (;;) {
                const int s = step % S, u = step / S;
                if (!wait(&full[s], (uint32_t)(u & 1))) break;
                const uint32_t info = s_info[s];
                if (info == kInfoEnd) break;
                const int k = (int)(info & 0x3fffffffu);
                const bool first = (info & kInfoFirst) != 0u, last = (info & kInfoLast) != 0u;
                const int b = k & 1, ua = k >> 1;
                if (first && ua > 0 && !wait(&aempty[b], (uint32_t)((ua - 1) & 1))) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(b * CO);
#pragma unroll
                for (int kk = 0; kk < KC / 16; ++kk) {
                    const uint64_t ad = smem_desc_kmajor_swizzled(sA + s * Cfg::kABytes + kk * 32, RB);
                    const uint64_t bd = smem_desc_kmajor_swizzled(sB + s * Cfg::kBBytes + kk * 32, RB);
                    tc_mma_f16(d, ad, bd, idesc, (!first || kk > 0) ? 1u : 0u);
                }
                tc_commit(smem_u32(&empty[s]));
                if (last) {
                    tc_commit(smem_u32(&afull[b]));
                    if (b) ++acc1; else ++acc0;
                }
                ++step;
            }
            if (*s_abort && step > 0) {      // wait (bounded) for the MMAs issued so far
                const int st = step - 1;
                mbar_wait_bounded(smem_u32(&empty[st % S]), (uint32_t)((st / S) & 1));
                // and for the accumulator commits, whose arrivals must not outlive the CTA
                if (acc0 > 0) mbar_wait_bounded(smem_u32(&afull[0]), (uint32_t)((acc0 - 1) & 1));
                if (acc1 > 0) mbar_wait_bounded(smem_u32(&afull[1]), (uint32_t)((acc1 - 1) & 1));
            }
        }
    } else if (warp >= kWarpEpi) {
        // ------------------------------------------------------------------ epilogue
        constexpr int kCols = CO < 32 ? CO : 32;      // columns per TMEM load batch
        const int quad = warp & 3;
        for (int k = 0; SPLIT || k < nt; ++k) {
            const int b = k & 1, t = k % kTileRing;
            int tinfo = -1;
            if (SPLIT) {     // items without work publish no tile: the scheduler marks the end
                if (!wait(&tfull[t], (uint32_t)((k / kTileRing) & 1))) break;
                tinfo = s_tinfo[t];
                if (tinfo == kTileEnd) break;
                if (!wait(&afull[b], (uint32_t)((k >> 1) & 1))) break;
            } else {
                if (!wait(&afull[b], (uint32_t)((k >> 1) & 1))) break;
                if (!wait(&tfull[t], (uint32_t)((k / kTileRing) & 1))) break;
            }
            tc_fence_after();
            const int32_t row = s_trow[t * kTileM + quad * 32 + lane];
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&tempty[t]));
            const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(b * CO);
            T *orow = out + (int64_t)(row < 0 ? 0 : row) * CO;
            // Writes accumulator columns [c0, c0 + kCols) of this lane's row (+ `add`, + bias).
            auto write_out = [&](int c0, const uint32_t (&acc)[kCols], const float *add) {
#pragma unroll
                for (int m = 0; m < kCols / 8; ++m) {
                    float f[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        f[q] = __uint_as_float(acc[m * 8 + q]);
                        if (add) f[q] += __ldcg(add + c0 + m * 8 + q);
                        if (bias) f[q] += dtype_traits<T>::to_f(bias[c0 + m * 8 + q]);
                    }
                    uint4 p;
                    p.x = pack2<T>(f[0], f[1]);
                    p.y = pack2<T>(f[2], f[3]);
                    p.z = pack2<T>(f[4], f[5]);
                    p.w = pack2<T>(f[6], f[7]);
                    *reinterpret_cast<uint4 *>(orow + c0 + m * 8) = p;
                }
            };
            if (!SPLIT || tinfo < 0) {
#pragma unroll
                for (int c0 = 0; c0 < CO; c0 += kCols) {
                    uint32_t acc[kCols];
#pragma unroll
                    for (int m = 0; m < kCols / 8; ++m) tmem_ld8(taddr + c0 + m * 8, &acc[m * 8]);
                    tc_wait_ld();
                    if (row >= 0) write_out(c0, acc, nullptr);
                }
            } else {
                // Half of a split tile: publish this half's fp32 partial rows, then count the
                // halves done (per tile and lane quadrant); the second to finish adds the other
                // half's partial (fp32 addition of two terms commutes, so the result does not
                // depend on which half finishes last) and writes the output rows.
                const int slot = tinfo >> 1, half = tinfo & 1;
                const int64_t prow = (int64_t)quad * 32 + lane;
                float *mine = partials + ((int64_t)(slot * 2 + half) * kTileM + prow) * CO;
                const float *other = partials + ((int64_t)(slot * 2 + (half ^ 1)) * kTileM + prow) * CO;
#pragma unroll
                for (int c0 = 0; c0 < CO; c0 += kCols) {
                    uint32_t acc[kCols];
#pragma unroll
                    for (int m = 0; m < kCols / 8; ++m) tmem_ld8(taddr + c0 + m * 8, &acc[m * 8]);
                    tc_wait_ld();
                    if (row >= 0) {
#pragma unroll
                        for (int m = 0; m < kCols / 4; ++m)
                            __stcg(reinterpret_cast<float4 *>(mine + c0) + m,
                                   make_float4(__uint_as_float(acc[4 * m]), __uint_as_float(acc[4 * m + 1]),
                                               __uint_as_float(acc[4 * m + 2]), __uint_as_float(acc[4 * m + 3])));
                    }
                }
                __threadfence();
                __syncwarp();
                int done = 0;
                if (lane == 0) done = atomicAdd(split_cnt + slot * 4 + quad, 1);
                done = __shfl_sync(0xffffffffu, done, 0);
                if (done == 1) {
                    __threadfence();
#pragma unroll
                    for (int c0 = 0; c0 < CO; c0 += kCols) {
                        uint32_t acc[kCols];
#pragma unroll
                        for (int m = 0; m < kCols / 8; ++m) tmem_ld8(taddr + c0 + m * 8, &acc[m * 8]);
                        tc_wait_ld();
                        if (row >= 0) write_out(c0, acc, other);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&aempty[b]));
        }
    }

    __syncwarp();
    if (*s_abort && tid == 0) raise_status(status, SPCONV_STATUS_WAIT_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kWarpMma) tmem_dealloc(tmem, Cfg::kTmemCols);
}

// ---------------------------------------------------------------------------------------
// Host side: weight tensor map and launch.
// ---------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn tensor_map_encoder() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 2-D row-major tensor of 16-bit elements: `cols` x `rows`, rows `row_stride` bytes apart;
// box = box_cols x box_rows; swizzle width = box_cols * 2 bytes.
static bool make_tmap_2d(CUtensorMap *map, const void *ptr, uint64_t cols, uint64_t rows,
                         uint64_t row_stride, uint32_t box_cols, uint32_t box_rows) {
    EncodeTiledFn enc = tensor_map_encoder();
    if (!enc) {
        set_error("tcgen05 conv: cuTensorMapEncodeTiled is not available from the driver");
        return false;
    }
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {row_stride};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const uint32_t wbytes = box_cols * 2;
    const CUtensorMapSwizzle sw = wbytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : (wbytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(ptr), dims, strides,
                           box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("tcgen05 conv: tensor map encoding failed (CUresult %d)", (int)r);
        return false;
    }
    return true;
}

// Gatherer warps: four, whether a CTA has an SM to itself (large stages) or two CTAs share
// one. Measured on B200 with the conv alone on cached maps: eight gatherer warps took the
// indoor conv (C=64) from 875 to 901 us and sixteen to 1,015 us; wide3 / wide5 (C=128) were
// unchanged with eight and 10-15 % slower with sixteen. More warps issuing cp.async do not
// raise the gather rate, so it is not one warp's dependent chain that bounds it.
#ifndef SPCONV_TC_GATHER_WARPS_1CTA
#define SPCONV_TC_GATHER_WARPS_1CTA 4
#endif
#ifndef SPCONV_TC_GATHER_WARPS_2CTA
#define SPCONV_TC_GATHER_WARPS_2CTA 4
#endif

// The weight's tensor map, encoded once per (device, address, shape): eager calls reuse it.
// A map holds only the address, sizes, strides and box, so a later tensor at the same address
// with the same shape is described by the same map.
struct TmapKey {
    int dev;
    const void *ptr;
    uint64_t cols, rows;
    uint32_t box_cols;
    bool operator==(const TmapKey &o) const {
        return dev == o.dev && ptr == o.ptr && cols == o.cols && rows == o.rows && box_cols == o.box_cols;
    }
};

static bool weight_tmap(CUtensorMap *map, int dev, const void *ptr, uint64_t cols, uint64_t rows,
                        uint32_t box_cols, uint32_t box_rows) {
    constexpr int kEntries = 32;
    static std::mutex mu;
    static TmapKey keys[kEntries];
    static CUtensorMap maps[kEntries];
    static int used = 0, next = 0;
    const TmapKey key{dev, ptr, cols, rows, box_cols};
    {
        std::lock_guard<std::mutex> lk(mu);
        for (int i = 0; i < used; ++i)
            if (keys[i] == key) {
                *map = maps[i];
                return true;
            }
    }
    if (!make_tmap_2d(map, ptr, cols, rows, cols * 2, box_cols, box_rows)) return false;
    std::lock_guard<std::mutex> lk(mu);
    const int i = used < kEntries ? used++ : (next++ % kEntries);
    keys[i] = key;
    maps[i] = *map;
    return true;
}

template <int CI, int CO, typename T, bool FLIP, bool SPLIT>
static int launch_tc_k(const ConvArgs &a) {
    using Cfg = TcCfg<CI, CO>;
    constexpr int NG = Cfg::kMinBlocks >= 2 ? SPCONV_TC_GATHER_WARPS_2CTA : SPCONV_TC_GATHER_WARPS_1CTA;
    constexpr int kThreads = TcRoles<NG>::kThreads;
    auto kern = conv_tc_kernel<CI, CO, T, FLIP, NG, SPLIT>;
    const int MWS = (a.masks && a.MW <= kMaxMaskWords) ? a.MW : 0;
    // Shared memory is padded so that no more CTAs fit on an SM than its 512 TMEM columns
    // serve (228 KB of shared memory per SM, 1 KB reserved per CTA): tcgen05.alloc never waits.
    constexpr int kSmemForTmem = (228 * 1024) / (Cfg::kMaxCtasByTmem + 1);
    constexpr int smem = Cfg::kSmemBytes > kSmemForTmem ? Cfg::kSmemBytes : kSmemForTmem;
    // Kernel attributes belong to the device's context: set once per device, under a lock
    // so that concurrent host threads see them complete.
    static std::mutex attr_mu;
    static bool attr_done[64] = {false};
    static int occ_cache[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    std::unique_lock<std::mutex> attr_lock(attr_mu);
    if (!attr_done[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return check_launch("conv_tc: set max dynamic shared memory");
        if (cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared) != cudaSuccess)
            return check_launch("conv_tc: set shared memory carveout");
        int occ = occupancy_per_sm((const void *)kern, kThreads, smem);
        if (occ > Cfg::kMaxCtasByTmem) occ = Cfg::kMaxCtasByTmem;
        occ_cache[dev] = occ < 1 ? 1 : occ;
        attr_done[dev] = true;
    }
    const int occ_dev = occ_cache[dev];
    attr_lock.unlock();
    CUtensorMap tw;
    if (!weight_tmap(&tw, dev, a.weight, (uint64_t)a.V * CI, (uint64_t)CO, Cfg::KC, CO))
        return SPCONV_ERR_CUDA;
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int num_tiles = (int)((a.M + kTileM - 1) / kTileM);
    int split_tiles = 0;
    float *partials = nullptr;
    int *split_cnt = nullptr;
    if (SPLIT) {
        split_tiles = num_tiles < kSplitMaxTiles ? num_tiles : kSplitMaxTiles;
        split_cnt = reinterpret_cast<int *>(a.split_ws);
        partials = reinterpret_cast<float *>(reinterpret_cast<char *>(a.split_ws) + split_counter_bytes());
        if (cudaMemsetAsync(split_cnt, 0, (size_t)split_tiles * 4 * sizeof(int), a.stream) != cudaSuccess)
            return check_launch("conv_tc: split counter memset");
    }
    int grid = sms * occ_dev;
    if (grid > num_tiles + split_tiles) grid = num_tiles + split_tiles;
    if (grid < 1) grid = 1;
    // Whole index rows are staged when one fits a 128-byte window and the map is 16-byte aligned.
    const int row_mode = (a.V <= kRowsMaxV && ((uintptr_t)a.nbr & 15u) == 0) ? 1 : 0;
    const cudaError_t le = launch_pdl(kern, dim3(grid), dim3(kThreads), (size_t)smem, a.stream, tw,
                                      (const T *)a.feats, (const T *)a.bias, a.nbr, a.masks, a.order, (T *)a.out,
                                      a.M, a.V, a.MW, MWS, num_tiles, row_mode, a.status, wait_limit_ns(),
                                      split_tiles, partials, split_cnt);
    if (le != cudaSuccess) return check_launch("conv_tc_kernel launch");
    return check_launch("conv_tc_kernel");
}

template <int CI, int CO, typename T>
static int launch_tc(const ConvArgs &a) {
    if (a.flip) return launch_tc_k<CI, CO, T, true, false>(a);
    if (a.split_ws) return launch_tc_k<CI, CO, T, false, true>(a);
    return launch_tc_k<CI, CO, T, false, false>(a);
}

int64_t split_counter_bytes() { return ((int64_t)kSplitMaxTiles * 4 * 4 + 255) & ~int64_t(255); }

int64_t conv_split_workspace_bytes(int64_t M, int Co) {
    const int64_t tiles = (M + kTileM - 1) / kTileM;
    const int64_t r = tiles < kSplitMaxTiles ? tiles : kSplitMaxTiles;
    return split_counter_bytes() + r * 2 * kTileM * (int64_t)Co * 4;
}

bool tc_supported(int dtype, int Ci, int Co, int V) {
    if (dtype != SPCONV_F16 && dtype != SPCONV_BF16) return false;
    auto ok = [](int c) { return c == 16 || c == 32 || c == 64 || c == 128; };
    return ok(Ci) && ok(Co) && V >= 1 && V <= 1024;
}

template <typename T>
static int dispatch_tc_t(const ConvArgs &a) {
#define SPCONV_TC_CO(CI)                                     \
    switch (a.Co) {                                          \
        case 16: return launch_tc<CI, 16, T>(a);             \
        case 32: return launch_tc<CI, 32, T>(a);             \
        case 64: return launch_tc<CI, 64, T>(a);             \
        case 128: return launch_tc<CI, 128, T>(a);           \
        default: break;                                      \
    }
    switch (a.Ci) {
        case 16: SPCONV_TC_CO(16) break;
        case 32: SPCONV_TC_CO(32) break;
        case 64: SPCONV_TC_CO(64) break;
        case 128: SPCONV_TC_CO(128) break;
        default: break;
    }
#undef SPCONV_TC_CO
    set_error("tcgen05 conv: unsupported channels Ci=%d Co=%d", a.Ci, a.Co);
    return SPCONV_ERR_UNSUPPORTED;
}

int launch_conv_tc(const ConvArgs &a) {
    if (!tc_supported(a.dtype, a.Ci, a.Co, a.V)) {
        set_error("tcgen05 conv: unsupported dtype/channels (dtype=%d Ci=%d Co=%d V=%d)", a.dtype, a.Ci, a.Co, a.V);
        return SPCONV_ERR_UNSUPPORTED;
    }
    if (a.dtype == SPCONV_F16) return dispatch_tc_t<__half>(a);
    return dispatch_tc_t<__nv_bfloat16>(a);
}

}  // namespace spconv
