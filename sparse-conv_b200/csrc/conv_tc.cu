// tcgen05 / TMEM implicit-GEMM submanifold convolution for sm_100a (fp16 / bf16 in,
// fp32 accumulate). Replaces the reference's Triton kernel (implicit_gemm.py:8-57), which
// runs 32x32x16 tiles over every one of the V*ceil(Ci/16) K-steps and reloads the
// neighbour index column per step.
//
// Structure (one CTA = 4 warps = 128 threads, persistent over 128-row tiles):
//   * a tile is 128 consecutive entries of the voxel order produced by the map build, so
//     rows of a tile share most of their offset masks; the OR of the tile's masks selects
//     the offsets the tile needs (every offset absent from all 128 rows is skipped);
//   * for each active offset v, thread t gathers feature row nbr[row_t, v] (zero-filled by
//     cp.async when missing) into the A stage and the CTA loads W[:, v, :] into the B
//     stage, both K-major in the no-swizzle core-matrix layout (8 rows x 16 bytes);
//   * one thread issues Ci/16 tcgen05.mma (M=128, N=Co, K=16) accumulating into TMEM and
//     commits to the stage's mbarrier, so the next offset's gather overlaps the MMAs;
//   * epilogue: tcgen05.ld of each warp's 32 TMEM lanes, + bias, one rounding to the
//     output dtype, and a single store of each output row (no atomics).
// Every mbarrier wait is bounded; on timeout the CTA raises SPCONV_STATUS_WAIT_TIMEOUT,
// waits (bounded) for its last MMAs, frees its TMEM and exits.
#include "common.cuh"
#include "conv_internal.h"

namespace spconv {

constexpr int kTcThreads = 128;
constexpr int kTileM = 128;
constexpr int kMaskPrefetchWords = 4;      // next-tile mask words held in registers (V <= 128)

template <int CI, int CO>
struct TcCfg {
    static constexpr int kABytes = kTileM * CI * 2;
    static constexpr int kBBytes = CO * CI * 2;
    // Gathers run kAhead = kStages - 2 offsets ahead of the MMA: a refilled stage was last
    // read by the MMA two offsets back, so its completion is off the critical path.
    // Small stages: five (three ahead); mid-size: four; Ci = Co = 128: three (one ahead).
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kStages = kStageBytes <= 8 * 1024 ? 6 : (kStageBytes <= 16 * 1024 ? 5 : (kStageBytes <= 32 * 1024 ? 4 : 3));
    static constexpr int kAhead = kStages - 2;
    static constexpr int kTmemCols = CO < 32 ? 32 : CO;
    static constexpr int kAuxBytes = 256;
    static constexpr int kSmemBytes = kStages * (kABytes + kBBytes) + kAuxBytes + 128;
    static constexpr int kMaxCtasByTmem = 512 / kTmemCols;
};

template <int N>
__device__ __forceinline__ void cp_async_wait_upto(int pending) {
    // wait until at most `pending` (<= N) groups are outstanding
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

template <int CI, int CO, typename T>
__global__ void __launch_bounds__(kTcThreads)
conv_tc_kernel(const T *__restrict__ feats, const T *__restrict__ weight,
               const T *__restrict__ bias, const int32_t *__restrict__ nbr,
               const uint32_t *__restrict__ masks, const int32_t *__restrict__ order,
               T *__restrict__ out, int64_t M, int V, int MW, int num_tiles, int32_t *status) {
    using Cfg = TcCfg<CI, CO>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 127) & ~(uintptr_t)127);
    uint8_t *sA = base;
    uint8_t *sB = base + Cfg::kStages * Cfg::kABytes;
    uint8_t *aux = sB + Cfg::kStages * Cfg::kBBytes;
    uint64_t *mbar = reinterpret_cast<uint64_t *>(aux);               // [Cfg::kStages]
    uint32_t *s_tmem = reinterpret_cast<uint32_t *>(aux + 64);
    uint32_t *s_maskw = reinterpret_cast<uint32_t *>(aux + 128);      // [<= 32]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < Cfg::kStages; ++s) mbar_init(smem_u32(&mbar[s]), 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(s_tmem), Cfg::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;
    const uint32_t idesc = instr_desc_f16(dtype_traits<T>::mma_format, kTileM, CO);
    const uint32_t a_stage0 = smem_u32(sA), b_stage0 = smem_u32(sB);

    uint32_t it = 0;          // stage uses issued by this CTA so far
    bool ok = true;
    // Tiles are taken from the end of the voxel order first: voxels with the most neighbours
    // sort last, and their tiles (the most active offsets) then start earliest.
    const int G = gridDim.x;
    const int my_tiles = (int)blockIdx.x < num_tiles ? (num_tiles - 1 - (int)blockIdx.x) / G + 1 : 0;
    auto row_of = [&](int k) -> int32_t {
        const int tile = num_tiles - 1 - ((int)blockIdx.x + k * G);
        const int64_t r = (int64_t)tile * kTileM + tid;
        int32_t rr = -1;
        if (r < M) rr = order ? __ldg(order + r) : (int32_t)r;
        return rr >= M ? -1 : rr;                 // an order entry outside the table is ignored
    };
    auto mask_word = [&](int32_t rr, int w) -> uint32_t {
        if (rr < 0) return 0u;
        return masks ? __ldg(masks + (int64_t)rr * MW + w) : full_mask_word(w, V);
    };
    // Row and mask words of the next tile are loaded while the current tile runs.
    int32_t row_next = my_tiles > 0 ? row_of(0) : -1;
    uint32_t mk_next[kMaskPrefetchWords];
#pragma unroll
    for (int w = 0; w < kMaskPrefetchWords; ++w) mk_next[w] = w < MW ? mask_word(row_next, w) : 0u;

    for (int k = 0; k < my_tiles; ++k) {
        const int32_t row = row_next;
        uint32_t mk[kMaskPrefetchWords];
#pragma unroll
        for (int w = 0; w < kMaskPrefetchWords; ++w) mk[w] = mk_next[w];
        if (k + 1 < my_tiles) row_next = row_of(k + 1);

        __syncthreads();                          // previous tile done with s_maskw and TMEM
        if (tid < MW) s_maskw[tid] = 0u;
        __syncthreads();
        for (int w = 0; w < MW; ++w) {
            uint32_t m = 0;
            if (MW <= kMaskPrefetchWords) {
#pragma unroll
                for (int q = 0; q < kMaskPrefetchWords; ++q) if (q == w) m = mk[q];
            } else {
                m = mask_word(row, w);
            }
            m = __reduce_or_sync(0xffffffffu, m) & full_mask_word(w, V);
            if (lane == 0 && m) atomicOr(&s_maskw[w], m);
        }
        __syncthreads();

        // Active offsets are consumed in ascending v. Gathers run kAhead offsets ahead of the
        // MMA, so several are in flight per thread while the tensor core works.
        const int32_t *nrow = nbr + (int64_t)(row < 0 ? 0 : row) * V;
        int nact = 0;
        for (int w = 0; w < MW; ++w) nact += __popc(s_maskw[w]);
        int iw = 0;                                 // issue-side cursor over the mask words
        uint32_t im = s_maskw[0];
        const uint32_t it0 = it;
        auto issue = [&](int jj) {
            while (im == 0u && ++iw < MW) im = s_maskw[iw];
            const int v = iw * 32 + __ffs(im) - 1;
            im &= im - 1u;
            const uint32_t slot = it0 + (uint32_t)jj;
            const int s = (int)(slot % Cfg::kStages);
            const uint32_t use = slot / Cfg::kStages;
            if (use > 0 && !mbar_wait_bounded(smem_u32(&mbar[s]), (use - 1u) & 1u)) ok = false;
            int32_t n = row >= 0 ? __ldg(nrow + v) : -1;
            if (n >= M) n = -1;                   // rows outside the feature table read as missing
            const T *src = feats + (int64_t)(n < 0 ? 0 : n) * CI;
            const uint32_t a_st = a_stage0 + s * Cfg::kABytes;
            const uint32_t b_st = b_stage0 + s * Cfg::kBBytes;
#pragma unroll
            for (int c = 0; c < CI / 8; ++c)
                cp_async_16(a_st + (uint32_t)(c * kTileM + tid) * 16u, src + c * 8, n < 0 ? 0u : 16u);
#pragma unroll
            for (int q = tid; q < CO * (CI / 8); q += kTcThreads) {
                const int co = q % CO, c = q / CO;
                cp_async_16(b_st + (uint32_t)(c * CO + co) * 16u,
                            weight + ((int64_t)co * V + v) * CI + c * 8, 16u);
            }
            cp_async_commit();
        };
        int issued = 0;
        while (issued < nact && issued < Cfg::kAhead) issue(issued++);
        int j = 0;
        for (; j < nact; ++j) {
            if (issued < nact) issue(issued++);
            cp_async_wait_upto<Cfg::kAhead>(issued - j - 1);   // offset j's group has landed
            fence_proxy_async_smem();
            if (!__syncthreads_and(ok)) { ok = false; break; }
            const int s = (int)((it0 + (uint32_t)j) % Cfg::kStages);
            if (tid == 0) {
                tc_fence_after();
                const uint32_t a_st = a_stage0 + s * Cfg::kABytes;
                const uint32_t b_st = b_stage0 + s * Cfg::kBBytes;
#pragma unroll
                for (int kk = 0; kk < CI / 16; ++kk) {
                    const uint64_t ad = smem_desc_kmajor_noswizzle(a_st + kk * 2 * (kTileM * 16), kTileM * 16, 128);
                    const uint64_t bd = smem_desc_kmajor_noswizzle(b_st + kk * 2 * (CO * 16), CO * 16, 128);
                    tc_mma_f16(tmem, ad, bd, idesc, (j | kk) != 0 ? 1u : 0u);
                }
                tc_commit(smem_u32(&mbar[s]));
            }
        }
        it = it0 + (uint32_t)j;
        if (!ok) {
            cp_async_wait<0>();
            break;
        }
        // The next tile's mask words (its row load has landed by now).
#pragma unroll
        for (int w = 0; w < kMaskPrefetchWords; ++w)
            mk_next[w] = (k + 1 < my_tiles && w < MW && MW <= kMaskPrefetchWords) ? mask_word(row_next, w) : 0u;
        if (j > 0) {
            const uint32_t last = it - 1u;
            if (!mbar_wait_bounded(smem_u32(&mbar[last % Cfg::kStages]), (last / Cfg::kStages) & 1u)) ok = false;
        }
        if (!__syncthreads_and(ok)) { ok = false; break; }
        tc_fence_after();

        // Epilogue: TMEM lanes 32*warp .. 32*warp+31 hold this warp's 32 rows.
        const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
        T *orow = out + (int64_t)(row < 0 ? 0 : row) * CO;
#pragma unroll
        for (int cc = 0; cc < CO / 16; ++cc) {
            uint32_t acc[16];
            if (j > 0) {
                tmem_ld16(taddr + cc * 16, acc);
                tc_wait_ld();
            } else {
#pragma unroll
                for (int e = 0; e < 16; ++e) acc[e] = 0u;
            }
            if (row >= 0) {
                float f[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    f[e] = __uint_as_float(acc[e]);
                    if (bias) f[e] += dtype_traits<T>::to_f(bias[cc * 16 + e]);
                }
                uint4 p0, p1;
                p0.x = pack2<T>(f[0], f[1]);   p0.y = pack2<T>(f[2], f[3]);
                p0.z = pack2<T>(f[4], f[5]);   p0.w = pack2<T>(f[6], f[7]);
                p1.x = pack2<T>(f[8], f[9]);   p1.y = pack2<T>(f[10], f[11]);
                p1.z = pack2<T>(f[12], f[13]); p1.w = pack2<T>(f[14], f[15]);
                uint4 *dst = reinterpret_cast<uint4 *>(orow + cc * 16);
                dst[0] = p0;
                dst[1] = p1;
            }
        }
        tc_fence_before();
    }

    if (!ok) {
        if (tid == 0) {
            raise_status(status, SPCONV_STATUS_WAIT_TIMEOUT);
            if (it > 0) {
                const uint32_t last = it - 1u;
                mbar_wait_bounded(smem_u32(&mbar[last % Cfg::kStages]), (last / Cfg::kStages) & 1u);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, Cfg::kTmemCols);
}

template <int CI, int CO, typename T>
static int launch_tc(const ConvArgs &a) {
    using Cfg = TcCfg<CI, CO>;
    auto kern = conv_tc_kernel<CI, CO, T>;
    // Shared memory is padded so that no more CTAs fit on an SM than its 512 TMEM columns
    // serve (228 KB of shared memory per SM, 1 KB reserved per CTA): tcgen05.alloc never waits.
    constexpr int kSmemForTmem = (228 * 1024) / (Cfg::kMaxCtasByTmem + 1);
    constexpr int smem = Cfg::kSmemBytes > kSmemForTmem ? Cfg::kSmemBytes : kSmemForTmem;
    static bool attr_done[64] = {false};
    static int occ_cache[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!attr_done[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return check_launch("conv_tc: set max dynamic shared memory");
        // Without a carveout preference the occupancy query (and the launch) may assume a
        // small shared-memory carveout and allow a single CTA per SM.
        if (cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared) != cudaSuccess)
            return check_launch("conv_tc: set shared memory carveout");
        int occ = occupancy_per_sm((const void *)kern, kTcThreads, smem);
        if (occ > Cfg::kMaxCtasByTmem) occ = Cfg::kMaxCtasByTmem;
        occ_cache[dev] = occ;
        attr_done[dev] = true;
    }
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int occ = occ_cache[dev];
    const int num_tiles = (int)((a.M + kTileM - 1) / kTileM);
    int grid = sms * occ;
    if (grid > num_tiles) grid = num_tiles;
    if (grid < 1) grid = 1;
    kern<<<grid, kTcThreads, smem, a.stream>>>(
        (const T *)a.feats, (const T *)a.weight, (const T *)a.bias, a.nbr, a.masks, a.order,
        (T *)a.out, a.M, a.V, a.MW, num_tiles, a.status);
    return check_launch("conv_tc_kernel");
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
