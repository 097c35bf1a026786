// Backward of the submanifold conv (the reference's EXPLICIT_GEMM backward, ops:105-150, whose
// autograd wrapper cannot run, ops:186-206):
//
//   grad_feats[j]     = sum_{(i,v): nbr[i,v] = j} grad_out[i] @ W[:, v, :]
//   grad_W[co, v, ci] = sum_i grad_out[i, co] * feats[nbr[i,v], ci]
//   grad_bias[co]     = sum_i grad_out[i, co]
//
// The input gradient is a forward conv over the transposed map nbr_t[j, v] = i (the i with
// nbr[i, v] = j; unique for a valid map) with the weight's channel axes swapped, so it runs on
// the forward kernels; spconv_transpose_neighbor_map builds nbr_t and its offset masks. For
// odd kernel sizes nbr_t[j, v] = nbr[j, V-1-v], the reference's flip (ops:123-126); for even
// sizes the flip is not the transpose (offsets are not symmetric) and this is the exact one.
//
// The weight gradient is a reduction over voxels per offset. wgrad_mma_kernel (16-bit
// features, 16/32/64/128 channels on both sides): one CTA per (group of offsets, run of tiles
// of the voxel order); per 128-voxel tile the grad_out rows are gathered once for the group
// and each offset's neighbour feature rows beside them, by cp.async into padded shared-memory
// rows in the order they sit in HBM (voxel-major), read by ldmatrix.trans straight into
// mma.sync fragments (A = grad_out^T, B = feats^T, K = voxels). Tiles whose voxels have no
// neighbour at any of the group's offsets are skipped. Fp32 accumulators are added to the
// fp32 gradient once per CTA. wgrad_simt_kernel covers fp32 and other channel counts.
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "conv_internal.h"

namespace spconv {

// ---------------------------------------------------------------------------------------
// Transposed map
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
transpose_map_kernel(const int32_t *__restrict__ nbr, int64_t M, int V, int32_t *nbr_t) {
    const int64_t MV = M * (int64_t)V;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < MV;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int32_t j = __ldg(nbr + e);
        if ((uint32_t)j < (uint32_t)M) {
            const int64_t i = e / V;
            // at most one i per (j, v) in a map of distinct coordinates; atomicMax keeps the
            // result deterministic if the caller's coordinates repeat
            atomicMax(nbr_t + (int64_t)j * V + (e - i * V), (int32_t)i);
        }
    }
}

__global__ void __launch_bounds__(256)
map_masks_kernel(const int32_t *__restrict__ nbr, int64_t M, int V, int MW, uint32_t *__restrict__ masks) {
    const int64_t total = M * (int64_t)MW;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = e / MW;
        const int w = (int)(e - j * MW);
        const int v1 = min(V, 32 * w + 32);
        uint32_t bits = 0;
        for (int v = 32 * w; v < v1; ++v)
            if (__ldg(nbr + j * V + v) >= 0) bits |= 1u << (v & 31);
        masks[e] = bits;
    }
}

// ---------------------------------------------------------------------------------------
// Weight gradient on tensor cores (mma.sync m16n8k16, fp32 accumulation)
// ---------------------------------------------------------------------------------------
constexpr int kWgTile = 128;                 // voxels per tile (the K extent of one pass)

template <typename T> struct mma_kind;
template <> struct mma_kind<__half> {
    static __device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
        asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
                     "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
                     : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};
template <> struct mma_kind<__nv_bfloat16> {
    static __device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
        asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
                     "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
                     : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}

// Offsets per group: the grad_out tile is gathered once for OG offsets; warp w owns offset
// w / (CO/16) of the group and output rows 16 (w % (CO/16)) .. +15 (all CI columns), so a CTA
// has OG * CO / 16 warps (<= 16). Two pipeline stages of (grad_out tile + OG feature tiles)
// fit in ~220 KB of shared memory; shapes left with fewer than four warps run on the CUDA cores.
template <typename T, int CO, int CI>
struct WgCfg {
    static constexpr int GP = CO + 8, FP = CI + 8;        // padded row pitch (elements): conflict-free ldmatrix
    static constexpr int kGBytes = kWgTile * GP * 2;
    static constexpr int kFBytes = kWgTile * FP * 2;
    static constexpr int kOgWarps = (CI >= 128 ? 128 : 256) / CO;   // 16 warps (8 with 64 accumulators a thread)
    // small rows: ~55 KB a stage (two CTAs per SM hide the index latency); else ~110 KB
    static constexpr int kStageBudget = (CO <= 32 && CI <= 32 ? 55 : 110) * 1024;
    static constexpr int kOgSmem = (kStageBudget - kGBytes - 4 * kWgTile) / (kFBytes + 4 * kWgTile);
    static constexpr int OG = kOgWarps < kOgSmem ? kOgWarps : kOgSmem;
    static constexpr int kWarps = OG * CO / 16;
    static constexpr int kThreads = kWarps * 32;
    static constexpr int kStageBytes = kGBytes + OG * kFBytes + kWgTile * 4 * (1 + OG);
    static constexpr int kSmem = 2 * kStageBytes + 1024 * 4;             // + group counts
    static constexpr bool kSupported = kWarps >= 4;
};

constexpr int kWgMaxGroups = 1024;

// Offset masks OR-ed over each 128-voxel tile of the voxel order: union[t][w], MW words.
__global__ void __launch_bounds__(kWgTile)
tile_union_kernel(const uint32_t *__restrict__ masks, const int32_t *__restrict__ nbr,
                  const int32_t *__restrict__ order, int64_t M, int V, int MW, uint32_t *__restrict__ uni) {
    __shared__ uint32_t s_or[kWgTile / 32][32];
    const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t p = (int64_t)t * kWgTile + tid;
    int32_t row = -1;
    if (p < M) {
        row = order ? __ldg(order + p) : (int32_t)p;
        if ((uint32_t)row >= (uint32_t)M) row = -1;
    }
    for (int w = 0; w < MW; ++w) {
        uint32_t m = 0;
        if (row >= 0) {
            if (masks) {
                m = __ldg(masks + (int64_t)row * MW + w);
            } else {
                const int v1 = min(V, 32 * w + 32);
                for (int v = 32 * w; v < v1; ++v)
                    if ((uint32_t)__ldg(nbr + (int64_t)row * V + v) < (uint32_t)M) m |= 1u << (v & 31);
            }
        }
        m = __reduce_or_sync(0xffffffffu, m);
        if (lane == 0) s_or[warp][w & 31] = m;
        __syncthreads();
        if (tid == 0) uni[(int64_t)t * MW + w] = s_or[0][w & 31] | s_or[1][w & 31] | s_or[2][w & 31] | s_or[3][w & 31];
        __syncthreads();
    }
}

// One block per offset group: the tiles with a neighbour at any of the group's offsets, in
// tile order, as list[g][0 .. cnt[g]).
__global__ void __launch_bounds__(512)
group_tiles_kernel(const uint32_t *__restrict__ uni, int num_tiles, int MW, int V, int OG,
                   int32_t *__restrict__ list, int32_t *__restrict__ cnt) {
    __shared__ uint32_t s_warp[16];
    const int g = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int lo = g * OG, hi = min(V, lo + OG);
    int base = 0;
    for (int t0 = 0; t0 < num_tiles; t0 += 512) {
        const int t = t0 + tid;
        bool act = false;
        if (t < num_tiles) {
            for (int v = lo; v < hi; ++v)
                if ((__ldg(uni + (int64_t)t * MW + (v >> 5)) >> (v & 31)) & 1u) { act = true; break; }
        }
        const uint32_t bal = __ballot_sync(0xffffffffu, act);
        if (lane == 0) s_warp[warp] = __popc(bal);
        __syncthreads();
        int off = 0, tot = 0;
        for (int w = 0; w < 16; ++w) { const int c = s_warp[w]; off += w < warp ? c : 0; tot += c; }
        if (act) list[(int64_t)g * num_tiles + base + off + __popc(bal & ((1u << lane) - 1u))] = t;
        base += tot;
        __syncthreads();
    }
    if (tid == 0) cnt[g] = base;
}

template <typename T, int CO, int CI>
__global__ void __launch_bounds__(WgCfg<T, CO, CI>::kThreads)
wgrad_mma_kernel(const T *__restrict__ feats, const T *__restrict__ gout,
                 const int32_t *__restrict__ nbr, const int32_t *__restrict__ order,
                 const int32_t *__restrict__ list, const int32_t *__restrict__ cnt,
                 const uint32_t *__restrict__ uni, int MW,
                 int64_t M, int V, int num_tiles, int groups, float *__restrict__ gw) {
    using Cfg = WgCfg<T, CO, CI>;
    static_assert(Cfg::kSupported && Cfg::kThreads >= kWgTile && Cfg::kThreads <= 512, "thread count");
    constexpr int OG = Cfg::OG, NT = Cfg::kThreads, GP = Cfg::GP, FP = Cfg::FP;
    constexpr int kNT = CI / 8;                           // n8 tiles per warp
    constexpr int kMB = CO / 16;                          // m16 blocks per offset
    extern __shared__ __align__(16) uint8_t wg_smem[];
    int32_t *s_cnt = reinterpret_cast<int32_t *>(wg_smem + 2 * Cfg::kStageBytes);   // [groups]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wo = warp / kMB, m0 = (warp % kMB) * 16;    // this warp's offset in the group, rows
    auto g_base = [&](int s) { return smem_u32(wg_smem) + (uint32_t)(s * Cfg::kStageBytes); };
    auto f_base = [&](int s) { return g_base(s) + (uint32_t)Cfg::kGBytes; };
    auto s_row = [&](int s) { return reinterpret_cast<int32_t *>(wg_smem + s * Cfg::kStageBytes + Cfg::kGBytes + OG * Cfg::kFBytes); };

    // this CTA's share of the flattened (group, active tile) list, in group order
    int total = 0;
    for (int g = tid; g < groups; g += NT) s_cnt[g] = cnt[g];
    __syncthreads();
    for (int g = 0; g < groups; ++g) total += s_cnt[g];
    const int per = (total + (int)gridDim.x - 1) / (int)gridDim.x;
    const int f0 = min(total, (int)blockIdx.x * per), f1 = min(total, f0 + per);
    int wg = 0, wk = f0;                                  // cursor: group, index inside the group
    while (wg < groups && wk >= s_cnt[wg]) { wk -= s_cnt[wg]; ++wg; }
    int left = f1 - f0;
    auto next = [&](int &g, int &t) {                     // next work tile, g = -1 at the end
        if (left <= 0) { g = -1; t = 0; return; }
        while (wk >= s_cnt[wg]) { wk = 0; ++wg; }
        g = wg;
        t = __ldg(list + (int64_t)wg * num_tiles + wk);
        ++wk;
        --left;
    };

    // offsets of group g that some voxel of tile t has (bit o = offset g*OG + o)
    auto active = [&](int g, int t) -> uint32_t {
        if (g < 0) return 0u;
        const int v0 = g * OG, ng = min(OG, V - v0);
        const uint32_t *u = uni + (int64_t)t * MW;
        const int w0 = v0 >> 5, sh = v0 & 31;
        uint64_t bits = __ldg(u + w0);
        if (w0 + 1 < MW) bits |= (uint64_t)__ldg(u + w0 + 1) << 32;
        return (uint32_t)(bits >> sh) & ((1u << ng) - 1u);
    };
    // tile row r's voxel and its neighbours at the group's active offsets (threads r < 128)
    int32_t row = -1, jn[OG];
    uint32_t act_next = 0;
    auto load_idx = [&](int g, int t) {
        row = -1;
#pragma unroll
        for (int o = 0; o < OG; ++o) jn[o] = -1;
        act_next = active(g, t);
        if (g < 0 || tid >= kWgTile) return;
        const int64_t p = (int64_t)t * kWgTile + tid;
        if (p >= M) return;
        const int32_t rr = order ? __ldg(order + p) : (int32_t)p;
        if ((uint32_t)rr >= (uint32_t)M) return;
        row = rr;
        const int v0 = g * OG, ng = min(OG, V - v0);
        const int32_t *nr = nbr + (int64_t)rr * V + v0;
#pragma unroll
        for (int o = 0; o < OG; ++o) {
            if (o < ng && ((act_next >> o) & 1u)) {
                const int32_t jj = __ldg(nr + o);
                jn[o] = (uint32_t)jj < (uint32_t)M ? jj : -1;
            }
        }
    };
    auto store_idx = [&](int s) {
        if (tid < kWgTile) {
            int32_t *sr = s_row(s);
            sr[tid] = row;
#pragma unroll
            for (int o = 0; o < OG; ++o) sr[(1 + o) * kWgTile + tid] = jn[o];
        }
    };
    auto gather = [&](int s, int g, uint32_t act) {       // after a barrier that published stage s's indices
        const int32_t *sr = s_row(s);
        const int ng = __popc(act);                       // feature tiles only for the active offsets
        constexpr int kGC = CO / 8, kFC = CI / 8;
        const uint32_t gb = g_base(s), fb = f_base(s);
        for (int e = tid; e < kWgTile * kGC; e += NT) {
            const int r = e / kGC, c = e - r * kGC;
            const int32_t rr = sr[r];
            cp_async_16(gb + (uint32_t)((r * GP + c * 8) * 2), gout + (int64_t)(rr >= 0 ? rr : 0) * CO + c * 8,
                        rr >= 0 ? 16u : 0u);
        }
        for (int e = tid; e < ng * kWgTile * kFC; e += NT) {
            const int c = e % kFC, r = (e / kFC) % kWgTile, k = e / (kFC * kWgTile);
            uint32_t m = act;                             // the k-th active offset of the group
            for (int i = 0; i < k; ++i) m &= m - 1u;
            const int o = __ffs(m) - 1;
            const int32_t jj = sr[(1 + o) * kWgTile + r];
            cp_async_16(fb + (uint32_t)(k * Cfg::kFBytes + (r * FP + c * 8) * 2),
                        feats + (int64_t)(jj >= 0 ? jj : 0) * CI + c * 8, jj >= 0 ? 16u : 0u);
        }
    };

    float acc[kNT][4];
#pragma unroll
    for (int n = 0; n < kNT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
    int cur_g = -1;
    auto flush = [&]() {
        if (cur_g < 0) return;
        const int ng = min(OG, V - cur_g * OG);
        if (wo < ng) {
            // acc[n]: (co = m0 + g, ci = 8n + 2c, +1) and (co = m0 + g + 8, same ci)
            const int gr = lane >> 2, c = lane & 3, v = cur_g * OG + wo;
#pragma unroll
            for (int n = 0; n < kNT; ++n) {
                const int ci = n * 8 + 2 * c;
                float *w0 = gw + ((int64_t)(m0 + gr) * V + v) * CI + ci;
                float *w1 = gw + ((int64_t)(m0 + gr + 8) * V + v) * CI + ci;
                if (acc[n][0] != 0.f) atomicAdd(w0, acc[n][0]);
                if (acc[n][1] != 0.f) atomicAdd(w0 + 1, acc[n][1]);
                if (acc[n][2] != 0.f) atomicAdd(w1, acc[n][2]);
                if (acc[n][3] != 0.f) atomicAdd(w1 + 1, acc[n][3]);
            }
        }
#pragma unroll
        for (int n = 0; n < kNT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
    };

    // two-stage pipeline: tile k+1's rows are in flight while tile k is multiplied, and tile
    // k+2's indices load meanwhile
    int gA, tA, gB, tB, gC, tC;
    next(gA, tA);
    next(gB, tB);
    load_idx(gA, tA);
    uint32_t aA = act_next;
    store_idx(0);
    __syncthreads();
    if (gA >= 0) gather(0, gA, aA);
    cp_async_commit();
    load_idx(gB, tB);
    uint32_t aB = act_next;
    for (int k = 0; gA >= 0; ++k) {
        const int s = k & 1;
        store_idx(s ^ 1);                                 // tile k+1's indices
        __syncthreads();                                  // published; stage s^1 is free
        if (gB >= 0) gather(s ^ 1, gB, aB);
        cp_async_commit();
        next(gC, tC);
        load_idx(gC, tC);                                 // tile k+2's indices load meanwhile
        const uint32_t aC = act_next;
        cp_async_wait<1>();                               // tile k's rows have landed
        __syncthreads();
        if (gA != cur_g) { flush(); cur_g = gA; }
        if ((aA >> wo) & 1u) {                            // this warp's offset is active in the tile
            const int slot = __popc(aA & ((1u << wo) - 1u));      // its feature tile among the active ones
            const uint32_t gb = g_base(s), fb = f_base(s) + (uint32_t)(slot * Cfg::kFBytes);
            const int q = lane >> 3, rr = lane & 7;
#pragma unroll 2
            for (int k0 = 0; k0 < kWgTile; k0 += 16) {
                // A = grad_out^T (m = co, k = voxel) from G[k][m]: matrices (k0|k0+8) x (m0|m0+8)
                uint32_t a[4];
                ldmatrix_x4_trans(a, gb + (uint32_t)(((k0 + rr + (q >> 1) * 8) * GP + m0 + (q & 1) * 8) * 2));
#pragma unroll
                for (int n = 0; n < kNT; n += 2) {
                    // B^T = feats (n = ci, k = voxel) from F[k][n]: two n8 tiles per ldmatrix.x4
                    uint32_t b[4];
                    ldmatrix_x4_trans(b, fb + (uint32_t)(((k0 + rr + (q & 1) * 8) * FP + n * 8 + (q >> 1) * 8) * 2));
                    mma_kind<T>::mma(acc[n], a, b[0], b[1]);
                    mma_kind<T>::mma(acc[n + 1], a, b[2], b[3]);
                }
            }
        }
        gA = gB; tA = tB; aA = aB;
        gB = gC; tB = tC; aB = aC;
    }
    cp_async_wait<0>();
    flush();
}

// ---------------------------------------------------------------------------------------
// Weight gradient on CUDA cores (any dtype and channel counts)
// ---------------------------------------------------------------------------------------
constexpr int kWsVox = 32;                   // voxels staged per batch
constexpr int kWsThreads = 256;
constexpr int kWsOut = 16;                   // outputs per thread per pass

template <typename T>
__global__ void __launch_bounds__(kWsThreads)
wgrad_simt_kernel(const T *__restrict__ feats, const T *__restrict__ gout,
                  const int32_t *__restrict__ nbr, int64_t M, int V, int Ci, int Co,
                  int64_t vox_per_cta, float *__restrict__ gw) {
    extern __shared__ float ws_smem[];
    float *Gs = ws_smem;                                  // [kWsVox][Co]
    float *Fs = ws_smem + kWsVox * Co;                    // [kWsVox][Ci]
    __shared__ int32_t s_row[kWsThreads], s_nbr[kWsThreads];
    __shared__ int s_wcnt[kWsThreads / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int v = blockIdx.y;
    const int64_t i0 = (int64_t)blockIdx.x * vox_per_cta;
    const int64_t i1 = min(M, i0 + vox_per_cta);
    const int nout = Co * Ci;
    for (int o0 = 0; o0 < nout; o0 += kWsThreads * kWsOut) {
        float acc[kWsOut];
#pragma unroll
        for (int k = 0; k < kWsOut; ++k) acc[k] = 0.f;
        for (int64_t b = i0; b < i1; b += kWsThreads) {
            // the voxels of this batch that have a neighbour at offset v, compacted in order
            int32_t jn = -1;
            if (b + tid < i1) {
                jn = __ldg(nbr + (b + tid) * V + v);
                if ((uint32_t)jn >= (uint32_t)M) jn = -1;
            }
            const uint32_t bal = __ballot_sync(0xffffffffu, jn >= 0);
            if (lane == 0) s_wcnt[warp] = __popc(bal);
            __syncthreads();
            int off = 0, n = 0;
#pragma unroll
            for (int w = 0; w < kWsThreads / 32; ++w) {
                const int c = s_wcnt[w];
                off += w < warp ? c : 0;
                n += c;
            }
            if (jn >= 0) {
                const int slot = off + __popc(bal & ((1u << lane) - 1u));
                s_row[slot] = (int32_t)(b + tid);
                s_nbr[slot] = jn;
            }
            __syncthreads();
            for (int s0 = 0; s0 < n; s0 += kWsVox) {
                const int ns = min(kWsVox, n - s0);
                for (int e = tid; e < ns * Co; e += kWsThreads) {
                    const int sv = e / Co, co = e - sv * Co;
                    Gs[sv * Co + co] = dtype_traits<T>::to_f(__ldg(gout + (int64_t)s_row[s0 + sv] * Co + co));
                }
                for (int e = tid; e < ns * Ci; e += kWsThreads) {
                    const int sv = e / Ci, ci = e - sv * Ci;
                    Fs[sv * Ci + ci] = dtype_traits<T>::to_f(__ldg(feats + (int64_t)s_nbr[s0 + sv] * Ci + ci));
                }
                __syncthreads();
#pragma unroll
                for (int k = 0; k < kWsOut; ++k) {
                    const int o = o0 + k * kWsThreads + tid;
                    if (o < nout) {
                        const int co = o / Ci, ci = o - co * Ci;
                        float a = acc[k];
                        for (int sv = 0; sv < ns; ++sv) a = fmaf(Gs[sv * Co + co], Fs[sv * Ci + ci], a);
                        acc[k] = a;
                    }
                }
                __syncthreads();
            }
        }
#pragma unroll
        for (int k = 0; k < kWsOut; ++k) {
            const int o = o0 + k * kWsThreads + tid;
            if (o < nout && acc[k] != 0.f) {
                const int co = o / Ci, ci = o - co * Ci;
                atomicAdd(gw + ((int64_t)co * V + v) * Ci + ci, acc[k]);
            }
        }
    }
}

// grad_bias[co] = sum_i grad_out[i, co]
template <typename T>
__global__ void __launch_bounds__(256)
bias_grad_kernel(const T *__restrict__ gout, int64_t M, int Co, int64_t rows_per_cta, float *__restrict__ gb) {
    const int64_t r0 = (int64_t)blockIdx.x * rows_per_cta;
    const int64_t r1 = min(M, r0 + rows_per_cta);
    for (int co = threadIdx.x; co < Co; co += blockDim.x) {
        float a = 0.f;
        for (int64_t r = r0; r < r1; ++r) a += dtype_traits<T>::to_f(__ldg(gout + r * Co + co));
        if (a != 0.f) atomicAdd(gb + co, a);
    }
}

// Scratch of the weight gradient: tile unions [num_tiles][MW], group lists [V][num_tiles],
// group counts [V].
static int64_t wgrad_scratch_bytes(int64_t M, int V) {
    const int64_t nt = (M + kWgTile - 1) / kWgTile;
    const int64_t MW = (V + 31) / 32;
    return 4 * (nt * MW + (int64_t)V * nt + V) + 256;
}

template <typename T, int CO, int CI>
static int launch_wgrad_mma(const void *feats, const void *gout, const int32_t *nbr, const uint32_t *masks,
                            const int32_t *order, int64_t M, int V, float *gw, void *scratch, cudaStream_t stream) {
    using Cfg = WgCfg<T, CO, CI>;
    auto kern = wgrad_mma_kernel<T, CO, CI>;
    // Kernel attributes and occupancy belong to the device: computed once per device, under a
    // lock so that concurrent host threads see them complete.
    static std::mutex attr_mu;
    static bool attr_done[64] = {false};
    static int occ_cache[64] = {0};
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    int occ_dev = 1;
    {
        std::lock_guard<std::mutex> lock(attr_mu);
        if (!attr_done[dev]) {
            if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem) != cudaSuccess)
                return check_launch("wgrad: set max dynamic shared memory");
            int occ = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, Cfg::kThreads, Cfg::kSmem) != cudaSuccess || occ < 1)
                occ = 1;
            occ_cache[dev] = occ;
            attr_done[dev] = true;
        }
        occ_dev = occ_cache[dev];
    }
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int num_tiles = (int)((M + kWgTile - 1) / kWgTile);
    const int groups = (V + Cfg::OG - 1) / Cfg::OG;
    const int MW = (V + 31) / 32;
    uint32_t *uni = (uint32_t *)scratch;
    int32_t *list = (int32_t *)(uni + (int64_t)num_tiles * MW);
    int32_t *cnt = list + (int64_t)V * num_tiles;
    tile_union_kernel<<<num_tiles, kWgTile, 0, stream>>>(MW <= 4 ? masks : nullptr, nbr, order, M, V, MW, uni);
    if (int rc = check_launch("tile_union_kernel")) return rc;
    group_tiles_kernel<<<groups, 512, 0, stream>>>(uni, num_tiles, MW, V, Cfg::OG, list, cnt);
    if (int rc = check_launch("group_tiles_kernel")) return rc;
    kern<<<sms * occ_dev, Cfg::kThreads, Cfg::kSmem, stream>>>(
        (const T *)feats, (const T *)gout, nbr, order, list, cnt, uni, MW, M, V, num_tiles, groups, gw);
    return check_launch("wgrad_mma_kernel");
}

#ifndef SPCONV_WGRAD_TC
#define SPCONV_WGRAD_TC 1
#endif

template <typename T>
static int launch_wgrad_t(const void *feats, const void *gout, const int32_t *nbr, const uint32_t *masks,
                          const int32_t *order, int64_t M, int V, int Ci, int Co, float *gw, float *gb,
                          void *scratch, int32_t *status, cudaStream_t stream) {
    int rc = SPCONV_OK;
    bool done = false;
    if constexpr (!std::is_same<T, float>::value) {
        const int dtype = std::is_same<T, __half>::value ? SPCONV_F16 : SPCONV_BF16;
        // the tcgen05 kernel (wgrad_tc.cu) for the shapes it covers; it needs no scratch
        if (SPCONV_WGRAD_TC && wgrad_tc_supported(dtype, Ci, Co, V) && ((uintptr_t)feats & 15u) == 0 &&
            ((uintptr_t)gout & 15u) == 0) {
            rc = launch_wgrad_tc(dtype, feats, gout, nbr, order, masks, M, V, gw, status, stream);
            done = true;
        }
    }
    if constexpr (!std::is_same<T, float>::value) {
        static_assert(kWgMaxGroups >= 1024, "group counts of any kernel volume fit in shared memory");
        if (!done && ((uintptr_t)feats & 15u) == 0 && ((uintptr_t)gout & 15u) == 0 && scratch) {
#define SPCONV_WG(CO_, CI_)                                                                  \
            if constexpr (WgCfg<T, CO_, CI_>::kSupported) {                                  \
                if (!done && Co == CO_ && Ci == CI_) {                                       \
                    rc = launch_wgrad_mma<T, CO_, CI_>(feats, gout, nbr, masks, order, M, V, gw, scratch, stream); \
                    done = true;                                                             \
                }                                                                            \
            }
            SPCONV_WG(16, 16) SPCONV_WG(16, 32) SPCONV_WG(16, 64) SPCONV_WG(16, 128)
            SPCONV_WG(32, 16) SPCONV_WG(32, 32) SPCONV_WG(32, 64) SPCONV_WG(32, 128)
            SPCONV_WG(64, 16) SPCONV_WG(64, 32) SPCONV_WG(64, 64) SPCONV_WG(64, 128)
            SPCONV_WG(128, 16) SPCONV_WG(128, 32) SPCONV_WG(128, 64) SPCONV_WG(128, 128)
#undef SPCONV_WG
        }
    }
    if (!done) {
        const int64_t per = 4096;
        const int64_t gx = (M + per - 1) / per;
        const int smem = kWsVox * (Ci + Co) * (int)sizeof(float);
        if (smem > 48 * 1024 &&
            cudaFuncSetAttribute(wgrad_simt_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return check_launch("wgrad: set max dynamic shared memory");
        wgrad_simt_kernel<T><<<dim3((unsigned)gx, V), kWsThreads, smem, stream>>>(
            (const T *)feats, (const T *)gout, nbr, M, V, Ci, Co, per, gw);
        rc = check_launch("wgrad_simt_kernel");
    }
    if (rc != SPCONV_OK || gb == nullptr) return rc;
    const int64_t rows = 2048;
    bias_grad_kernel<T><<<(unsigned)((M + rows - 1) / rows), 256, 0, stream>>>((const T *)gout, M, Co, rows, gb);
    return check_launch("bias_grad_kernel");
}

}  // namespace spconv

using namespace spconv;

extern "C" int spconv_transpose_neighbor_map(const int32_t *nbr, int64_t M, int V, int32_t *nbr_t,
                                             uint32_t *masks_t, int32_t *status, void *stream) {
    (void)status;
    SPCONV_REQUIRE(M >= 0 && M <= 0x7fffffffLL, SPCONV_ERR_ARG, "num_coords %lld out of range", (long long)M);
    SPCONV_REQUIRE(V > 0 && V <= 1024, SPCONV_ERR_ARG, "kernel volume %d out of range [1, 1024]", V);
    if (M == 0) return SPCONV_OK;
    SPCONV_REQUIRE(nbr && nbr_t, SPCONV_ERR_ARG, "null pointer argument");
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemsetAsync(nbr_t, 0xff, (size_t)M * V * sizeof(int32_t), s) != cudaSuccess)
        return check_launch("transposed map memset");
    const int64_t MV = M * (int64_t)V;
    int64_t blocks = (MV + 255) / 256;
    if (blocks > 148LL * 32) blocks = 148LL * 32;
    transpose_map_kernel<<<(unsigned)blocks, 256, 0, s>>>(nbr, M, V, nbr_t);
    if (int rc = check_launch("transpose_map_kernel")) return rc;
    if (masks_t) {
        const int MW = spconv_mask_words(V);
        int64_t mb = (M * MW + 255) / 256;
        if (mb > 148LL * 32) mb = 148LL * 32;
        map_masks_kernel<<<(unsigned)mb, 256, 0, s>>>(nbr_t, M, V, MW, masks_t);
        if (int rc = check_launch("map_masks_kernel")) return rc;
    }
    return SPCONV_OK;
}

extern "C" int64_t spconv_weight_grad_workspace_bytes(int64_t num_coords, int kernel_volume) {
    if (num_coords < 0 || kernel_volume <= 0 || kernel_volume > 1024) return -1;
    return wgrad_scratch_bytes(num_coords, kernel_volume);
}

extern "C" int spconv_submanifold_conv_weight_grad(
    const void *feats, const void *grad_out, int dtype, int64_t M, int Ci, int Co, int V,
    const int32_t *nbr, const uint32_t *masks, const int32_t *order, float *grad_weight, float *grad_bias,
    void *workspace, int64_t workspace_bytes, int32_t *status, void *stream) {
    SPCONV_REQUIRE(M >= 0 && M <= 0x7fffffffLL, SPCONV_ERR_ARG, "num_coords %lld out of range", (long long)M);
    SPCONV_REQUIRE(Ci > 0 && Co > 0, SPCONV_ERR_ARG, "channels must be positive (Ci=%d Co=%d)", Ci, Co);
    SPCONV_REQUIRE(V > 0 && V <= 1024, SPCONV_ERR_ARG, "kernel volume %d out of range [1, 1024]", V);
    SPCONV_REQUIRE(dtype == SPCONV_F32 || dtype == SPCONV_F16 || dtype == SPCONV_BF16,
                   SPCONV_ERR_ARG, "unsupported dtype code %d", dtype);
    SPCONV_REQUIRE(grad_weight, SPCONV_ERR_ARG, "null grad_weight");
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemsetAsync(grad_weight, 0, (size_t)Co * V * Ci * sizeof(float), s) != cudaSuccess)
        return check_launch("grad_weight memset");
    if (grad_bias && cudaMemsetAsync(grad_bias, 0, (size_t)Co * sizeof(float), s) != cudaSuccess)
        return check_launch("grad_bias memset");
    if (M == 0) return SPCONV_OK;
    SPCONV_REQUIRE(feats && grad_out && nbr, SPCONV_ERR_ARG, "null pointer argument");
    SPCONV_REQUIRE(workspace == nullptr || ((uintptr_t)workspace & 15u) == 0, SPCONV_ERR_ARG,
                   "workspace must be 16-byte aligned");
    void *scratch = (workspace && workspace_bytes >= wgrad_scratch_bytes(M, V)) ? workspace : nullptr;
    switch (dtype) {
        case SPCONV_F32:
            return launch_wgrad_t<float>(feats, grad_out, nbr, masks, order, M, V, Ci, Co, grad_weight, grad_bias, scratch, status, s);
        case SPCONV_F16:
            return launch_wgrad_t<__half>(feats, grad_out, nbr, masks, order, M, V, Ci, Co, grad_weight, grad_bias, scratch, status, s);
        default:
            return launch_wgrad_t<__nv_bfloat16>(feats, grad_out, nbr, masks, order, M, V, Ci, Co, grad_weight, grad_bias, scratch, status, s);
    }
}
