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
// features, 64 or 128 channels on both sides): one CTA per (offset, run of tiles of the voxel
// order), 128 voxels per tile gathered by cp.async into padded shared-memory rows in the
// order they sit in HBM (voxel-major), and read by ldmatrix.trans straight into mma.sync
// fragments (A = grad_out^T, B = feats^T, K = voxels); tiles whose 128 voxels have no
// neighbour at that offset are skipped. Fp32 accumulators are added to the fp32 gradient
// once per CTA. wgrad_simt_kernel covers the other dtypes and channel counts.
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

// CO / 16 warps; warp w owns output rows 16w..16w+15 (co) and every column (ci).
template <typename T, int CO, int CI>
__global__ void __launch_bounds__(CO * 2)
wgrad_mma_kernel(const T *__restrict__ feats, const T *__restrict__ gout,
                 const int32_t *__restrict__ nbr, const int32_t *__restrict__ order,
                 int64_t M, int V, int num_tiles, int tiles_per_cta, float *__restrict__ gw) {
    constexpr int kThreads = CO * 2, kWarps = CO / 16;
    constexpr int GP = CO + 8, FP = CI + 8;               // padded row pitch (elements): conflict-free ldmatrix
    constexpr int kNT = CI / 8;                           // n8 tiles per warp
    extern __shared__ __align__(16) uint8_t wg_smem[];
    T *Gs = reinterpret_cast<T *>(wg_smem);               // [kWgTile][GP]
    T *Fs = Gs + kWgTile * GP;                            // [kWgTile][FP]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int v = blockIdx.y;
    const int t0 = blockIdx.x * tiles_per_cta;
    const int t1 = min(num_tiles, t0 + tiles_per_cta);

    float acc[kNT][4];
#pragma unroll
    for (int n = 0; n < kNT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;

    const uint32_t g_base = smem_u32(Gs), f_base = smem_u32(Fs);
    for (int t = t0; t < t1; ++t) {
        // thread r < 128 owns tile row r: its voxel and that voxel's neighbour at offset v
        static_assert(kThreads >= kWgTile, "one tile row per thread");
        int32_t row = -1, j = -1;
        if (tid < kWgTile) {
            const int64_t p = (int64_t)t * kWgTile + tid;
            if (p < M) {
                row = order ? __ldg(order + p) : (int32_t)p;
                if ((uint32_t)row < (uint32_t)M) {
                    j = __ldg(nbr + (int64_t)row * V + v);
                    if ((uint32_t)j >= (uint32_t)M) j = -1;
                } else {
                    row = -1;
                }
            }
        }
        if (!__syncthreads_or(j >= 0)) continue;          // no voxel of the tile has this neighbour
        // gather: row r's grad_out into Gs[r], its neighbour's feats into Fs[r] (zeros if none)
        if (tid < kWgTile) {
            const int r = tid;
            const bool have = j >= 0;
            const T *gsrc = gout + (int64_t)(have ? row : 0) * CO;
            const T *fsrc = feats + (int64_t)(have ? j : 0) * CI;
#pragma unroll
            for (int c = 0; c < CO / 8; ++c)
                cp_async_16(g_base + (uint32_t)((r * GP + c * 8) * 2), gsrc + c * 8, have ? 16u : 0u);
#pragma unroll
            for (int c = 0; c < CI / 8; ++c)
                cp_async_16(f_base + (uint32_t)((r * FP + c * 8) * 2), fsrc + c * 8, have ? 16u : 0u);
        }
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
        const int m0 = warp * 16;
#pragma unroll 2
        for (int k0 = 0; k0 < kWgTile; k0 += 16) {
            // A = grad_out^T (m = co, k = voxel) from Gs[k][m]: matrices (k0|k0+8) x (m0|m0+8)
            uint32_t a[4];
            {
                const int q = lane >> 3, rr = lane & 7;
                const int kk = k0 + rr + (q >> 1) * 8, mm = m0 + (q & 1) * 8;
                ldmatrix_x4_trans(a, g_base + (uint32_t)((kk * GP + mm) * 2));
            }
#pragma unroll
            for (int n = 0; n < kNT; n += 2) {
                // B^T = feats (n = ci, k = voxel) from Fs[k][n]: two n8 tiles per ldmatrix.x4
                uint32_t b[4];
                const int q = lane >> 3, rr = lane & 7;
                const int kk = k0 + rr + (q & 1) * 8, nn = n * 8 + (q >> 1) * 8;
                ldmatrix_x4_trans(b, f_base + (uint32_t)((kk * FP + nn) * 2));
                mma_kind<T>::mma(acc[n], a, b[0], b[1]);
                mma_kind<T>::mma(acc[n + 1], a, b[2], b[3]);
            }
        }
        __syncthreads();                                  // Gs/Fs are rewritten by the next tile
    }
    // acc[n]: (co = m0 + g, ci = 8n + 2c, +1) and (co = m0 + g + 8, same ci)
    const int g = lane >> 2, c = lane & 3, m0 = warp * 16;
#pragma unroll
    for (int n = 0; n < kNT; ++n) {
        const int ci = n * 8 + 2 * c;
        float *w0 = gw + ((int64_t)(m0 + g) * V + v) * CI + ci;
        float *w1 = gw + ((int64_t)(m0 + g + 8) * V + v) * CI + ci;
        if (acc[n][0] != 0.f) atomicAdd(w0, acc[n][0]);
        if (acc[n][1] != 0.f) atomicAdd(w0 + 1, acc[n][1]);
        if (acc[n][2] != 0.f) atomicAdd(w1, acc[n][2]);
        if (acc[n][3] != 0.f) atomicAdd(w1 + 1, acc[n][3]);
    }
    (void)kWarps;
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
    __shared__ int32_t s_row[kWsVox], s_nbr[kWsVox];
    __shared__ int s_cnt;
    const int tid = threadIdx.x;
    const int v = blockIdx.y;
    const int64_t i0 = (int64_t)blockIdx.x * vox_per_cta;
    const int64_t i1 = min(M, i0 + vox_per_cta);
    const int nout = Co * Ci;
    for (int o0 = 0; o0 < nout; o0 += kWsThreads * kWsOut) {
        float acc[kWsOut];
#pragma unroll
        for (int k = 0; k < kWsOut; ++k) acc[k] = 0.f;
        for (int64_t b = i0; b < i1; b += kWsVox) {
            // compact the batch's voxels that have a neighbour at offset v
            if (tid == 0) s_cnt = 0;
            __syncthreads();
            if (tid < kWsVox && b + tid < i1) {
                const int32_t jn = __ldg(nbr + (b + tid) * V + v);
                if ((uint32_t)jn < (uint32_t)M) {
                    const int slot = atomicAdd(&s_cnt, 1);
                    s_row[slot] = (int32_t)(b + tid);
                    s_nbr[slot] = jn;
                }
            }
            __syncthreads();
            const int n = s_cnt;
            if (n == 0) continue;                         // uniform: s_cnt read after the barrier
            for (int e = tid; e < n * Co; e += kWsThreads) {
                const int s = e / Co, co = e - s * Co;
                Gs[s * Co + co] = dtype_traits<T>::to_f(__ldg(gout + (int64_t)s_row[s] * Co + co));
            }
            for (int e = tid; e < n * Ci; e += kWsThreads) {
                const int s = e / Ci, ci = e - s * Ci;
                Fs[s * Ci + ci] = dtype_traits<T>::to_f(__ldg(feats + (int64_t)s_nbr[s] * Ci + ci));
            }
            __syncthreads();
#pragma unroll
            for (int k = 0; k < kWsOut; ++k) {
                const int o = o0 + k * kWsThreads + tid;
                if (o < nout) {
                    const int co = o / Ci, ci = o - co * Ci;
                    float a = acc[k];
                    for (int s = 0; s < n; ++s) a = fmaf(Gs[s * Co + co], Fs[s * Ci + ci], a);
                    acc[k] = a;
                }
            }
            __syncthreads();
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

template <typename T, int CO, int CI>
static int launch_wgrad_mma(const void *feats, const void *gout, const int32_t *nbr, const int32_t *order,
                            int64_t M, int V, float *gw, cudaStream_t stream) {
    auto kern = wgrad_mma_kernel<T, CO, CI>;
    const int smem = kWgTile * ((CO + 8) + (CI + 8)) * (int)sizeof(T);
    static bool attr_done[64] = {false};
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!attr_done[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return check_launch("wgrad: set max dynamic shared memory");
        attr_done[dev] = true;
    }
    const int num_tiles = (int)((M + kWgTile - 1) / kWgTile);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // about eight CTAs per SM over all offsets; each CTA adds its accumulators once
    int64_t want = (int64_t)sms * 8 / V;
    if (want < 1) want = 1;
    int tiles_per_cta = (int)((num_tiles + want - 1) / want);
    if (tiles_per_cta < 1) tiles_per_cta = 1;
    const int gx = (num_tiles + tiles_per_cta - 1) / tiles_per_cta;
    kern<<<dim3(gx, V), CO * 2, smem, stream>>>((const T *)feats, (const T *)gout, nbr, order, M, V,
                                               num_tiles, tiles_per_cta, gw);
    return check_launch("wgrad_mma_kernel");
}

template <typename T>
static int launch_wgrad_t(const void *feats, const void *gout, const int32_t *nbr, const int32_t *order,
                          int64_t M, int V, int Ci, int Co, float *gw, float *gb, cudaStream_t stream) {
    int rc = SPCONV_OK;
    bool done = false;
    if constexpr (!std::is_same<T, float>::value) {
        if (((uintptr_t)feats & 15u) == 0 && ((uintptr_t)gout & 15u) == 0) {
#define SPCONV_WG(CO_, CI_)                                                                  \
            if (!done && Co == CO_ && Ci == CI_) {                                           \
                rc = launch_wgrad_mma<T, CO_, CI_>(feats, gout, nbr, order, M, V, gw, stream); \
                done = true;                                                                 \
            }
            SPCONV_WG(64, 64) SPCONV_WG(64, 128) SPCONV_WG(128, 64) SPCONV_WG(128, 128)
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

extern "C" int spconv_submanifold_conv_weight_grad(
    const void *feats, const void *grad_out, int dtype, int64_t M, int Ci, int Co, int V,
    const int32_t *nbr, const int32_t *order, float *grad_weight, float *grad_bias,
    int32_t *status, void *stream) {
    (void)status;
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
    switch (dtype) {
        case SPCONV_F32: return launch_wgrad_t<float>(feats, grad_out, nbr, order, M, V, Ci, Co, grad_weight, grad_bias, s);
        case SPCONV_F16: return launch_wgrad_t<__half>(feats, grad_out, nbr, order, M, V, Ci, Co, grad_weight, grad_bias, s);
        default: return launch_wgrad_t<__nv_bfloat16>(feats, grad_out, nbr, order, M, V, Ci, Co, grad_weight, grad_bias, s);
    }
}
