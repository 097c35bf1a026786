// Weight gradient of the submanifold conv on the 5th-generation tensor cores (tcgen05 / TMEM),
// for 16-bit features with Ci = Co = 64:
//
//   grad_W[co, v, ci] = sum_i grad_out[i, co] * feats[nbr[i, v], ci]
//
// (the reference's EXPLICIT_GEMM weight gradient, ops/submanifold_conv3d.py:129-143). Per
// 128-voxel tile of the voxel order the voxels are the K dimension. Offsets are taken in fixed
// pairs (2p, 2p + 1): one MMA (M = 128, N = 64, K = 16) multiplies A = [feats rows at offset
// 2p ; feats rows at offset 2p + 1]^T (M = the two offsets' 64 input channels, MN-major: each
// gathered 128-byte feature row is one K row of A) by B = grad_out rows of the tile^T (N = 64
// output channels, MN-major), so no half of the M = 128 datapath is idle while both offsets
// are active. Each pair accumulates in its own 64 TMEM columns across all the tiles a CTA
// takes: eight pairs (16 offsets, a "group") fill the 512 columns. When one offset of a pair
// has no neighbour in a tile, its half of A is described by a resident block of zeros instead
// of being gathered.
//
// One CTA per SM, 10 warps with fixed roles, synchronised by mbarriers only:
//   warp 0    scheduler: per work item (tile, group) loads the tile's rows (voxel order), ORs
//             their offset masks and, by 4-byte cp.async, loads the map entries of the item's
//             active offsets into one of two index contexts;
//   warps 1-4 gatherers: warp g owns rows 32g .. 32g + 31; per item the grad_out rows into
//             one of two B buffers, then per active pair the feature rows of its active
//             offsets into an A stage (128-byte swizzled rows, zero fill for missing
//             neighbours); each copy group is signalled once it has landed (wait_group, proxy
//             fence, arrive), a few groups behind its issue;
//   warp 5    MMA: one thread issues 8 MMAs per pair and commits stages and B buffers back;
//   warps 6-9 epilogue: when a CTA's run of items in one group ends, reads each pair's
//             accumulator (lanes 0-63: offset 2p, lanes 64-127: offset 2p + 1) and adds it to
//             the fp32 gradient with coalesced atomics.
// Work items are (group, tile) pairs, group-major; CTA c takes items c, c + G, ... (the CTAs walk
// the tiles side by side, so their gathers share the L2), skipping tiles with no neighbour at
// any of the group's offsets (the OR of the tile's offset masks).
// Every wait is bounded (the conv kernels' limit); a timeout raises SPCONV_STATUS_WAIT_TIMEOUT,
// and the CTA waits (bounded) for its own copies and MMAs before it frees TMEM and exits.
#include <mutex>

#include "common.cuh"
#include "conv_internal.h"

namespace spconv {

constexpr int kWtTile = 128;
constexpr int kWtPairs = 8;                    // offset pairs per group
constexpr int kWtGroupOffsets = 2 * kWtPairs;  // 16 offsets per group
constexpr int kWtCols = kWtGroupOffsets + 1;   // context columns: 16 offsets + the row itself
constexpr int kWtCtx = 2;                      // index context buffers
constexpr int kWtStages = 4;                   // A stages (one offset pair each)
constexpr int kWtDepth = kWtStages - 1;        // copy groups in flight per gatherer warp
constexpr int kWtThreads = 320;
constexpr int kWtMaxGroups = 64;
constexpr int kWtHalf = kWtTile * 128;         // 16 KB: 128 rows of 64 16-bit channels
// Shared memory (from a 1024-byte aligned base): zero block, A stages, zero block, two B
// buffers, index contexts, small state.
constexpr int kWtOffZ0 = 0;
constexpr int kWtOffA = kWtOffZ0 + kWtHalf;
constexpr int kWtOffZ1 = kWtOffA + kWtStages * 2 * kWtHalf;
constexpr int kWtOffB = kWtOffZ1 + kWtHalf;
constexpr int kWtOffCtx = kWtOffB + 2 * kWtHalf;
constexpr int kWtOffCInfo = kWtOffCtx + kWtCtx * kWtTile * kWtCols * 4;   // int4 per context
constexpr int kWtOffSInfo = kWtOffCInfo + kWtCtx * 16;                    // uint32 per A stage
constexpr int kWtOffGInfo = kWtOffSInfo + kWtStages * 4;                  // uint32 per B buffer
constexpr int kWtOffSeg = kWtOffGInfo + 2 * 4;                            // int2 per segment slot
constexpr int kWtOffPend = kWtOffSeg + 2 * 8;                             // gatherer signal rings
constexpr int kWtPendRing = 8;
constexpr int kWtOffCnt = kWtOffPend + 4 * kWtPendRing * 4;               // group item offsets
constexpr int kWtNumBars = 2 * kWtStages + 2 * 2 + 2 * kWtCtx + 2;
constexpr int kWtOffBar = (kWtOffCnt + (kWtMaxGroups + 1) * 4 + 7) & ~7;
constexpr int kWtOffMisc = kWtOffBar + kWtNumBars * 8;
constexpr int kWtSmem = kWtOffMisc + 16 + 1024;
static_assert(kWtSmem <= 227 * 1024, "wgrad shared memory");
static_assert(kWtPendRing > kWtDepth + 1, "gatherer signal ring");
// stage / B-buffer info words
constexpr uint32_t kWtEnd = 0xffffffffu;
constexpr uint32_t kWtSegFirst = 1u << 30, kWtSegLast = 1u << 29;

// Shared-memory descriptor of an MN-major operand with the 128-byte swizzle: 8 K rows of 64
// 16-bit elements (one 128-byte row per K index, 16-byte chunks XOR-ed with the row within
// its 8-row group) form a 1024-byte atom; `sbo` = byte distance between atoms adjacent in K,
// `lbo` = byte distance between the 64-element blocks adjacent in M/N.
__device__ __forceinline__ uint64_t smem_desc_mn_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

template <typename T>
__global__ void __launch_bounds__(kWtThreads, 1)
wgrad_tc_kernel(const T *__restrict__ feats, const T *__restrict__ gout, const int32_t *__restrict__ nbr,
                const int32_t *__restrict__ order, const uint32_t *__restrict__ masks, int64_t M, int V, int MW,
                int num_tiles, int groups, float *__restrict__ gw, int32_t *status, uint64_t wait_ns) {
    constexpr int CI = 64, CO = 64;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const uint32_t sZ0 = smem_u32(base + kWtOffZ0), sA = smem_u32(base + kWtOffA);
    const uint32_t sZ1 = smem_u32(base + kWtOffZ1), sB = smem_u32(base + kWtOffB);
    int32_t *s_ctx = reinterpret_cast<int32_t *>(base + kWtOffCtx);      // [ctx][row][kWtCols]
    int4 *s_cinfo = reinterpret_cast<int4 *>(base + kWtOffCInfo);         // {item, group, pairs | halves << 8, flags}
    uint32_t *s_sinfo = reinterpret_cast<uint32_t *>(base + kWtOffSInfo); // A stage: pair | halves << 8
    uint32_t *s_ginfo = reinterpret_cast<uint32_t *>(base + kWtOffGInfo); // B buffer: item flags
    int2 *s_seg = reinterpret_cast<int2 *>(base + kWtOffSeg);             // segment: {group or -1, seen pairs}
    uint32_t *s_pend = reinterpret_cast<uint32_t *>(base + kWtOffPend);   // [gatherer][ring] barrier addresses
    uint64_t *bar = reinterpret_cast<uint64_t *>(base + kWtOffBar);
    uint64_t *full = bar, *empty = bar + kWtStages, *gfull = empty + kWtStages, *gempty = gfull + 2;
    uint64_t *cfull = gempty + 2, *cempty = cfull + kWtCtx, *accfull = cempty + kWtCtx, *accempty = accfull + 1;
    uint32_t *s_tmem = reinterpret_cast<uint32_t *>(base + kWtOffMisc);
    volatile int *s_abort = reinterpret_cast<volatile int *>(base + kWtOffMisc + 4);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // zero blocks
    {
        uint4 *z0 = reinterpret_cast<uint4 *>(base + kWtOffZ0), *z1 = reinterpret_cast<uint4 *>(base + kWtOffZ1);
        for (int j = tid; j < kWtHalf / 16; j += kWtThreads) {
            z0[j] = make_uint4(0u, 0u, 0u, 0u);
            z1[j] = make_uint4(0u, 0u, 0u, 0u);
        }
    }
    if (tid == 0) {
        for (int s = 0; s < kWtStages; ++s) {
            mbar_init(smem_u32(&full[s]), 4);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&gfull[b]), 4);
            mbar_init(smem_u32(&gempty[b]), 1);
        }
        for (int c = 0; c < kWtCtx; ++c) {
            mbar_init(smem_u32(&cfull[c]), 1);
            mbar_init(smem_u32(&cempty[c]), 4);
        }
        mbar_init(smem_u32(accfull), 1);
        mbar_init(smem_u32(accempty), 4);
        *s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 5) {
        tmem_alloc(smem_u32(s_tmem), 512);
        tmem_relinquish();
    }
    fence_proxy_async_smem();                // the zero blocks, read by the MMAs
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;
    // Work items k = g * num_tiles + t, taken by CTA c as k = c, c + G, ...: the CTAs walk the
    // tiles of the voxel order side by side (their gathers share the L2), group after group.
    const int64_t n_items = (int64_t)groups * num_tiles;
    const int G = gridDim.x;
    auto wait = [&](uint64_t *b, uint32_t parity) -> bool {
        return mbar_wait_or_abort(smem_u32(b), parity, s_abort, wait_ns);
    };

    if (warp == 0) {
        // ------------------------------------------------------------------ scheduler
        int pend = -1;
        bool ok = true;
        auto publish = [&](bool all) {
            if (pend < 0) return;
            if (all) cp_async_wait<0>();
            else cp_async_wait<1>();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&cfull[pend]));
            pend = -1;
        };
        int kc = 0, g_last = -1;
        for (int64_t k = blockIdx.x; k < n_items && ok; k += G) {
            const int g = (int)(k / num_tiles), t = (int)(k - (int64_t)g * num_tiles);
            const int v0 = g * kWtGroupOffsets;
            int32_t rows[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int64_t pos = (int64_t)t * kWtTile + lane + 32 * j;
                int32_t row = -1;
                if (pos < M) {
                    row = order ? __ldg(order + pos) : (int32_t)pos;
                    if ((uint32_t)row >= (uint32_t)M) row = -1;
                }
                rows[j] = row;
            }
            // the tile's active offsets in this group: its rows' mask bits v0 .. v0 + 15 (all
            // of the group's offsets when no masks are given)
            uint32_t hm = 0;
            const uint32_t valid = (V - v0 >= 32) ? 0xffffu : (((1u << (V - v0)) - 1u) & 0xffffu);
            if (masks) {
                const int w0 = v0 >> 5, sh = v0 & 31;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (rows[j] < 0) continue;
                    const uint32_t *mr = masks + (int64_t)rows[j] * MW;
                    uint64_t m = __ldg(mr + w0);
                    if (sh > 16 && w0 + 1 < MW) m |= (uint64_t)__ldg(mr + w0 + 1) << 32;
                    hm |= (uint32_t)(m >> sh);
                }
                hm = __reduce_or_sync(0xffffffffu, hm) & valid;
            } else {
                hm = __any_sync(0xffffffffu, rows[0] >= 0) ? valid : 0u;
            }
            if (hm == 0u) continue;                               // nothing of this group here
            uint32_t pm = 0;
#pragma unroll
            for (int p = 0; p < kWtPairs; ++p)
                if ((hm >> (2 * p)) & 3u) pm |= 1u << p;
            const int cb = kc % kWtCtx;
            if (kc >= kWtCtx && !wait(&cempty[cb], (uint32_t)(((kc / kWtCtx) - 1) & 1))) { ok = false; break; }
            int32_t *ctx = s_ctx + cb * kWtTile * kWtCols;
#pragma unroll
            for (int j = 0; j < 4; ++j) ctx[(lane + 32 * j) * kWtCols + kWtGroupOffsets] = rows[j];
            for (int j = 0; j < kWtGroupOffsets; ++j) {
                if (!((hm >> j) & 1u)) continue;
                const int32_t *col = nbr + (v0 + j);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int r = lane + 32 * q;
                    int32_t *d = ctx + r * kWtCols + j;
                    if (rows[q] >= 0) cp_async_4(smem_u32(d), col + (int64_t)rows[q] * V);
                    else *d = -1;
                }
            }
            cp_async_commit();
            if (lane == 0) {
                s_cinfo[cb] = make_int4((int)(k & 0x7fffffff), g, (int)(pm | (hm << 8)), g != g_last ? (int)kWtSegFirst : 0);
                // the previous context closes its segment when the group changes here
                if (pend >= 0 && g != g_last) s_cinfo[pend].w |= (int)kWtSegLast;
            }
            g_last = g;
            publish(false);
            pend = cb;
            ++kc;
        }
        if (lane == 0 && pend >= 0) s_cinfo[pend].w |= (int)kWtSegLast;   // the last context closes its segment
        __syncwarp();
        publish(true);
        if (ok) {                            // end marker
            const int cb = kc % kWtCtx;
            if (kc < kWtCtx || wait(&cempty[cb], (uint32_t)(((kc / kWtCtx) - 1) & 1))) {
                if (lane == 0) s_cinfo[cb] = make_int4(-1, -1, 0, 0);
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&cfull[cb]));
            }
        }
        cp_async_wait_all();
    } else if (warp >= 1 && warp <= 4) {
        // ------------------------------------------------------------------ gatherers
        const int gw = warp - 1;
        const bool leader = gw == 0 && lane == 0;
        const int chunk = lane & 7;
        const int row0 = 32 * gw + (lane >> 3) * 8;          // this lane's 8 rows
        uint32_t dst[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const int r = row0 + q;
            dst[q] = (uint32_t)(r * 128 + ((chunk ^ (r & 7)) << 4));
        }
        uint32_t *ring = s_pend + gw * kWtPendRing;
        int kc = 0, step = 0, sig = 0, st = 0;                // contexts, copy groups issued / signalled, A steps
        bool ok = true;
        auto signal_one = [&]() {
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(ring[sig % kWtPendRing]);
            ++sig;
        };
        auto flush = [&]() {
            cp_async_wait<0>();
            while (sig < step) signal_one();
        };
        auto issued = [&](uint32_t barrier) {                 // a copy group was committed
            if (lane == 0) ring[step % kWtPendRing] = barrier;
            __syncwarp();
            ++step;
            if (step - sig > kWtDepth - 1) {
                cp_async_wait<kWtDepth - 1>();
                signal_one();
            }
        };
        auto gather = [&](uint32_t dst_base, const int32_t *ctx, int col, const T *src) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const int32_t n = ctx[(row0 + q) * kWtCols + col];
                const bool have = (uint32_t)n < (uint32_t)M;
                cp_async_16(dst_base + dst[q], src + (int64_t)(have ? n : 0) * 64 + chunk * 8, have ? 16u : 0u);
            }
        };
        for (;;) {
            const int cb = kc % kWtCtx;
            const uint32_t cpar = (uint32_t)((kc / kWtCtx) & 1);
            if (!mbar_test(smem_u32(&cfull[cb]), cpar)) flush();
            if (!wait(&cfull[cb], cpar)) { ok = false; break; }
            const int4 ci = s_cinfo[cb];
            const int32_t *ctx = s_ctx + cb * kWtTile * kWtCols;
            const int gb = kc & 1;
            if (ci.x < 0) {                                   // end: one B-buffer signal carrying kWtEnd
                flush();
                if (kc < 2 || wait(&gempty[gb], (uint32_t)(((kc >> 1) - 1) & 1))) {
                    if (leader) s_ginfo[gb] = kWtEnd;
                    __syncwarp();
                    if (lane == 0) mbar_arrive(smem_u32(&gfull[gb]));
                }
                break;
            }
            const uint32_t pm = (uint32_t)ci.z & 0xffu, hm = (uint32_t)ci.z >> 8;
            // grad_out rows of the tile into B buffer gb
            if (kc >= 2 && !wait(&gempty[gb], (uint32_t)(((kc >> 1) - 1) & 1))) { ok = false; break; }
            if (leader) s_ginfo[gb] = (uint32_t)ci.w | ((uint32_t)ci.y << 16) | pm;
            gather(sB + gb * kWtHalf, ctx, kWtGroupOffsets, gout);
            cp_async_commit();
            issued(smem_u32(&gfull[gb]));
            // feature rows of each active pair into an A stage
            for (uint32_t m = pm; m && ok; m &= m - 1) {
                const int p = __ffs(m) - 1;
                const int s = st % kWtStages, u = st / kWtStages;
                if (u > 0 && !wait(&empty[s], (uint32_t)((u - 1) & 1))) { ok = false; break; }
                const uint32_t halves = (hm >> (2 * p)) & 3u;
                if (leader) s_sinfo[s] = (uint32_t)p | (halves << 8);
                const uint32_t a_st = sA + s * 2 * kWtHalf;
#pragma unroll
                for (int h = 0; h < 2; ++h)
                    if ((halves >> h) & 1u) gather(a_st + h * kWtHalf, ctx, 2 * p + h, feats);
                cp_async_commit();                            // one copy group per pair
                issued(smem_u32(&full[s]));
                ++st;
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&cempty[cb]));
            ++kc;
        }
        if (ok) flush();
        cp_async_wait_all();
    } else if (warp == 5) {
        // ------------------------------------------------------------------ MMA
        if (lane == 0) {
            const uint32_t idesc = instr_desc_f16(dtype_traits<T>::mma_format, kWtTile, CO) | (1u << 15) | (1u << 16);
            int it = 0, st = 0, seg = 0;
            uint32_t seen = 0;
            bool ok = true;
            for (;;) {
                const int gb = it & 1;
                if (!wait(&gfull[gb], (uint32_t)((it >> 1) & 1))) { ok = false; break; }
                const uint32_t info = s_ginfo[gb];
                if (info == kWtEnd) break;
                const uint32_t pm = info & 0xffu;
                const int g = (int)((info >> 16) & 0x3fu);
                if ((info & kWtSegFirst) && seg > 0) {
                    // the epilogue has read the previous segment's accumulators
                    if (!wait(accempty, (uint32_t)((seg - 1) & 1))) { ok = false; break; }
                    seen = 0;
                }
                tc_fence_after();
                const uint32_t b_base = sB + gb * kWtHalf;
                for (uint32_t m = pm; m; m &= m - 1) {
                    const int s = st % kWtStages, u = st / kWtStages;
                    if (!wait(&full[s], (uint32_t)(u & 1))) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t si = s_sinfo[s];
                    const int p = (int)(si & 0xffu);
                    const uint32_t halves = si >> 8;
                    const uint32_t a_st = sA + s * 2 * kWtHalf;
                    // rows 0-63 of A: offset 2p (or zeros), rows 64-127: offset 2p+1 (or zeros)
                    uint32_t a0, lbo;
                    if (halves == 3u) { a0 = a_st; lbo = kWtHalf; }
                    else if (halves == 1u) { a0 = a_st; lbo = sZ1 - a_st; }
                    else { a0 = sZ0; lbo = a_st + kWtHalf - sZ0; }
                    const uint32_t d = tmem + (uint32_t)(p * CI);
                    const bool first = !((seen >> p) & 1u);
#pragma unroll
                    for (int kk = 0; kk < kWtTile / 16; ++kk) {
                        const uint64_t ad = smem_desc_mn_sw128(a0 + kk * 2048, lbo, 1024);
                        const uint64_t bd = smem_desc_mn_sw128(b_base + kk * 2048, kWtHalf, 1024);
                        tc_mma_f16(d, ad, bd, idesc, (first && kk == 0) ? 0u : 1u);
                    }
                    seen |= 1u << p;
                    tc_commit(smem_u32(&empty[s]));
                    ++st;
                }
                if (!ok) break;
                tc_commit(smem_u32(&gempty[gb]));
                if (info & kWtSegLast) {
                    s_seg[seg & 1] = make_int2(g, (int)seen);
                    __threadfence_block();
                    tc_commit(smem_u32(accfull));
                    ++seg;
                }
                ++it;
            }
            if (ok) {
                // end marker for the epilogue, once it has read the last segment
                if (seg == 0 || wait(accempty, (uint32_t)((seg - 1) & 1))) {
                    s_seg[seg & 1] = make_int2(-1, 0);
                    mbar_arrive(smem_u32(accfull));
                }
            } else if (st > 0) {
                const int sl = st - 1;
                mbar_wait_bounded(smem_u32(&empty[sl % kWtStages]), (uint32_t)((sl / kWtStages) & 1));
                if (seg > 0) mbar_wait_bounded(smem_u32(accfull), (uint32_t)((seg - 1) & 1));
            }
        }
    } else {
        // ------------------------------------------------------------------ epilogue
        const int quad = warp & 3;
        const int half = quad >> 1;                            // lanes 0-63: offset 2p, 64-127: 2p+1
        const int ci = (quad & 1) * 32 + lane;
        for (int seg = 0;; ++seg) {
            if (!wait(accfull, (uint32_t)(seg & 1))) break;
            tc_fence_after();
            const int2 sg = s_seg[seg & 1];
            if (sg.x < 0) break;
            const uint32_t seen = (uint32_t)sg.y;
            for (int p = 0; p < kWtPairs; ++p) {
                if (!((seen >> p) & 1u)) continue;
                const int v = sg.x * kWtGroupOffsets + 2 * p + half;
                float *g = gw + (int64_t)v * CI + ci;                 // + co * V * CI
#pragma unroll
                for (int c = 0; c < CO / 16; ++c) {
                    uint32_t acc[16];
                    tmem_ld16(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(p * CI + c * 16), acc);
                    tc_wait_ld();
                    if (v < V) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const float x = __uint_as_float(acc[j]);
                            if (x != 0.f) atomicAdd(g + (int64_t)(c * 16 + j) * V * CI, x);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(accempty));
        }
    }

    __syncwarp();
    if (*s_abort && tid == 0) raise_status(status, SPCONV_STATUS_WAIT_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 5) tmem_dealloc(tmem, 512);
}

bool wgrad_tc_supported(int dtype, int Ci, int Co, int V) {
    return (dtype == SPCONV_F16 || dtype == SPCONV_BF16) && Ci == 64 && Co == 64 && V >= 1 &&
           (V + kWtGroupOffsets - 1) / kWtGroupOffsets <= kWtMaxGroups;
}

int launch_wgrad_tc(int dtype, const void *feats, const void *gout, const int32_t *nbr, const int32_t *order,
                    const uint32_t *masks, int64_t M, int V, float *gw, int32_t *status, cudaStream_t stream) {
    const int groups = (V + kWtGroupOffsets - 1) / kWtGroupOffsets;
    const int num_tiles = (int)((M + kWtTile - 1) / kWtTile);
    const int MW = (V + 31) / 32;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    {
        static std::mutex mu;
        static bool done[64] = {false};
        std::lock_guard<std::mutex> lk(mu);
        const int d = dev >= 0 && dev < 64 ? dev : 0;
        if (!done[d]) {
            if (cudaFuncSetAttribute(wgrad_tc_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, kWtSmem) != cudaSuccess ||
                cudaFuncSetAttribute(wgrad_tc_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, kWtSmem) != cudaSuccess)
                return check_launch("wgrad_tc: set max dynamic shared memory");
            done[d] = true;
        }
    }
    const int grid = sms;                   // one CTA per SM (all 512 TMEM columns)
    if (dtype == SPCONV_F16)
        wgrad_tc_kernel<__half><<<grid, kWtThreads, kWtSmem, stream>>>(
            (const __half *)feats, (const __half *)gout, nbr, order, masks, M, V, MW, num_tiles, groups, gw,
            status, wait_limit_ns());
    else
        wgrad_tc_kernel<__nv_bfloat16><<<grid, kWtThreads, kWtSmem, stream>>>(
            (const __nv_bfloat16 *)feats, (const __nv_bfloat16 *)gout, nbr, order, masks, M, V, MW, num_tiles,
            groups, gw, status, wait_limit_ns());
    return check_launch("wgrad_tc_kernel");
}

}  // namespace spconv
