// Conv entry points and the CUDA-core (SIMT) submanifold-conv kernel.
//
// The SIMT kernel covers what the tcgen05 kernel does not: fp32 features (computed with
// fp32 FMAs, not TF32, so results stay within 1e-4 of a float64 evaluation) and channel
// counts outside {16, 32, 64, 128}:
//   out[i, co] = bias[co] + sum_v sum_ci feats[nbr[i,v], ci] * weight[co, v, ci]
// accumulated in fp32 (offsets ascending, then channels ascending) and rounded once.
//
// A block computes a tile of 64 consecutive entries of the voxel order x 32 output channels.
// It ORs the tile's offset masks and walks only the offsets some row of the tile has; per
// offset it gathers the 64 neighbour rows into shared memory in chunks of 32 input channels
// (missing neighbours as zeros), stages W[co0 .. co0+31, v, chunk], and each thread
// accumulates 2 rows x 4 output channels with fp32 FMAs.
#include "common.cuh"
#include "conv_internal.h"

namespace spconv {

constexpr int kSimtBM = 64, kSimtBN = 32, kSimtBK = 32, kSimtThreads = 256, kSimtMaxMW = 32;

template <typename T>
__global__ void __launch_bounds__(kSimtThreads)
conv_simt_kernel(const T *__restrict__ feats, const T *__restrict__ weight,
                 const T *__restrict__ bias, const int32_t *__restrict__ nbr,
                 const uint32_t *__restrict__ masks, const int32_t *__restrict__ order,
                 int64_t M, int Ci, int Co, int V, int MW, int MWS, int flip, T *__restrict__ out) {
    __shared__ float sA[kSimtBK][kSimtBM + 1];                  // [channel][row]
    __shared__ __align__(16) float sB[kSimtBK][kSimtBN + 4];    // [channel][output channel]
    __shared__ int32_t s_row[kSimtBM], s_nb[kSimtBM];
    __shared__ uint32_t s_or[kSimtMaxMW];
    const int tid = threadIdx.x;
    const int64_t p0 = (int64_t)blockIdx.x * kSimtBM;
    const int co0 = blockIdx.y * kSimtBN;
    if (tid < kSimtBM) {
        const int64_t p = p0 + tid;
        int32_t r = -1;
        if (p < M) {
            r = order ? __ldg(order + p) : (int32_t)p;
            if ((uint32_t)r >= (uint32_t)M) r = -1;            // order entries outside the table are ignored
        }
        s_row[tid] = r;
    }
    if (tid < kSimtMaxMW) s_or[tid] = 0u;
    __syncthreads();
    if (MWS > 0 && tid < kSimtBM && s_row[tid] >= 0)
        for (int w = 0; w < MWS; ++w) atomicOr(&s_or[w], __ldg(masks + (int64_t)s_row[tid] * MW + w));
    __syncthreads();
    const int tr = tid >> 3, tc = tid & 7;                      // rows 2tr, 2tr+1; channels 4tc .. 4tc+3
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    for (int v = 0; v < V; ++v) {
        const int col = flip ? V - 1 - v : v;                   // the map column read for offset v
        if (MWS > 0 && !((s_or[col >> 5] >> (col & 31)) & 1u)) continue;   // no row of the tile has it
        if (tid < kSimtBM) {
            const int32_t r = s_row[tid];
            int32_t n = -1;
            if (r >= 0) {
                n = __ldg(nbr + (int64_t)r * V + col);
                if ((uint32_t)n >= (uint32_t)M) n = -1;         // rows outside the feature table read as missing
            }
            s_nb[tid] = n;
        }
        __syncthreads();
        for (int kc = 0; kc < Ci; kc += kSimtBK) {
            for (int e = tid; e < kSimtBM * kSimtBK; e += kSimtThreads) {
                const int r = e / kSimtBK, k = e - r * kSimtBK;
                const int32_t n = s_nb[r];
                float x = 0.f;
                if (n >= 0 && kc + k < Ci) x = dtype_traits<T>::to_f(__ldg(feats + (int64_t)n * Ci + kc + k));
                sA[k][r] = x;
            }
            for (int e = tid; e < kSimtBN * kSimtBK; e += kSimtThreads) {
                const int k = e / kSimtBN, c = e - k * kSimtBN;
                float x = 0.f;
                if (co0 + c < Co && kc + k < Ci)
                    x = dtype_traits<T>::to_f(__ldg(weight + ((int64_t)(co0 + c) * V + v) * Ci + kc + k));
                sB[k][c] = x;
            }
            __syncthreads();
            const int kmax = Ci - kc < kSimtBK ? Ci - kc : kSimtBK;
            for (int k = 0; k < kmax; ++k) {
                const float a0 = sA[k][2 * tr], a1 = sA[k][2 * tr + 1];
                const float4 b = *reinterpret_cast<const float4 *>(&sB[k][4 * tc]);
                acc[0][0] = fmaf(a0, b.x, acc[0][0]);
                acc[0][1] = fmaf(a0, b.y, acc[0][1]);
                acc[0][2] = fmaf(a0, b.z, acc[0][2]);
                acc[0][3] = fmaf(a0, b.w, acc[0][3]);
                acc[1][0] = fmaf(a1, b.x, acc[1][0]);
                acc[1][1] = fmaf(a1, b.y, acc[1][1]);
                acc[1][2] = fmaf(a1, b.z, acc[1][2]);
                acc[1][3] = fmaf(a1, b.w, acc[1][3]);
            }
            __syncthreads();
        }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int32_t r = s_row[2 * tr + i];
        if (r < 0) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int co = co0 + 4 * tc + j;
            if (co >= Co) continue;
            float f = acc[i][j];
            if (bias) f += dtype_traits<T>::to_f(__ldg(bias + co));
            out[(int64_t)r * Co + co] = dtype_traits<T>::from_f(f);
        }
    }
}

int occupancy_per_sm(const void *kern, int threads, int smem_dynamic) {
    cudaFuncAttributes fa{};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaFuncGetAttributes(&fa, kern) != cudaSuccess) {
        cudaGetLastError();
        return 1;
    }
    int smem_sm = 0, reserved = 0, regs_sm = 0, thr_sm = 0, blk_sm = 0;
    cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev);
    cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&thr_sm, cudaDevAttrMaxThreadsPerMultiProcessor, dev);
    cudaDeviceGetAttribute(&blk_sm, cudaDevAttrMaxBlocksPerMultiprocessor, dev);
    const int warps = (threads + 31) / 32;
    const int regs_warp = ((fa.numRegs * 32 + 255) / 256) * 256;      // 256-register granularity
    int occ = blk_sm > 0 ? blk_sm : 32;
    const int per_cta_smem = smem_dynamic + (int)fa.sharedSizeBytes + reserved;
    if (per_cta_smem > 0 && smem_sm / per_cta_smem < occ) occ = smem_sm / per_cta_smem;
    if (regs_warp > 0 && regs_sm / (regs_warp * warps) < occ) occ = regs_sm / (regs_warp * warps);
    if (thr_sm / threads < occ) occ = thr_sm / threads;
    return occ < 1 ? 1 : occ;
}

int launch_conv_simt(const ConvArgs &a) {
    const int64_t tiles = (a.M + kSimtBM - 1) / kSimtBM;
    SPCONV_REQUIRE(tiles <= 0x7fffffffLL, SPCONV_ERR_ARG, "too many rows for the SIMT conv");
    const dim3 grid((unsigned)tiles, (unsigned)((a.Co + kSimtBN - 1) / kSimtBN));
    const int MWS = (a.masks && a.MW <= kSimtMaxMW) ? a.MW : 0;
    switch (a.dtype) {
        case SPCONV_F32:
            conv_simt_kernel<float><<<grid, kSimtThreads, 0, a.stream>>>(
                (const float *)a.feats, (const float *)a.weight, (const float *)a.bias, a.nbr, a.masks, a.order,
                a.M, a.Ci, a.Co, a.V, a.MW, MWS, a.flip, (float *)a.out);
            break;
        case SPCONV_F16:
            conv_simt_kernel<__half><<<grid, kSimtThreads, 0, a.stream>>>(
                (const __half *)a.feats, (const __half *)a.weight, (const __half *)a.bias, a.nbr, a.masks, a.order,
                a.M, a.Ci, a.Co, a.V, a.MW, MWS, a.flip, (__half *)a.out);
            break;
        case SPCONV_BF16:
            conv_simt_kernel<__nv_bfloat16><<<grid, kSimtThreads, 0, a.stream>>>(
                (const __nv_bfloat16 *)a.feats, (const __nv_bfloat16 *)a.weight,
                (const __nv_bfloat16 *)a.bias, a.nbr, a.masks, a.order, a.M, a.Ci, a.Co, a.V, a.MW, MWS, a.flip,
                (__nv_bfloat16 *)a.out);
            break;
        default:
            set_error("unsupported dtype code %d", a.dtype);
            return SPCONV_ERR_ARG;
    }
    return check_launch("conv_simt_kernel");
}

}  // namespace spconv

using namespace spconv;

static int launch_conv(const ConvArgs &a, int kernel_choice);

extern "C" int spconv_submanifold_conv_forward_ex(
    const void *feats, int dtype, int64_t M, int Ci,
    const void *weight, const void *bias, int Co, int V,
    const int32_t *nbr, const uint32_t *masks, const int32_t *order,
    void *out, int32_t *status, void *stream, int kernel_choice) {
    SPCONV_REQUIRE(M >= 0 && M <= 0x7fffffffLL, SPCONV_ERR_ARG, "num_coords %lld out of range", (long long)M);
    SPCONV_REQUIRE(Ci > 0 && Co > 0, SPCONV_ERR_ARG, "channels must be positive (Ci=%d Co=%d)", Ci, Co);
    SPCONV_REQUIRE(V > 0 && V <= 1024, SPCONV_ERR_ARG, "kernel volume %d out of range [1, 1024]", V);
    SPCONV_REQUIRE(dtype == SPCONV_F32 || dtype == SPCONV_F16 || dtype == SPCONV_BF16,
                   SPCONV_ERR_ARG, "unsupported dtype code %d", dtype);
    SPCONV_REQUIRE(kernel_choice >= SPCONV_KERNEL_AUTO && kernel_choice <= SPCONV_KERNEL_TCGEN05,
                   SPCONV_ERR_ARG, "unknown kernel choice %d", kernel_choice);
    if (M == 0) return SPCONV_OK;
    SPCONV_REQUIRE(feats && weight && nbr && out, SPCONV_ERR_ARG, "null pointer argument");
    ConvArgs a{feats, dtype, M, Ci, weight, bias, Co, V, spconv_mask_words(V), nbr, masks, order,
               out, status, (cudaStream_t)stream};
    stage_mark(SPCONV_STAGE_CONV, 0, a.stream);
    const int rc = launch_conv(a, kernel_choice);
    if (rc == SPCONV_OK) stage_mark(SPCONV_STAGE_CONV, 1, a.stream);
    return rc;
}

static int launch_conv(const ConvArgs &a, int kernel_choice) {
    const int dtype = a.dtype, Ci = a.Ci, Co = a.Co, V = a.V;
    const void *feats = a.feats, *weight = a.weight, *out = a.out;
    const bool tc = tc_supported(dtype, Ci, Co, V);
    if (kernel_choice == SPCONV_KERNEL_TCGEN05) {
        if (!tc) {
            set_error("tcgen05 conv does not cover dtype=%d Ci=%d Co=%d", dtype, Ci, Co);
            return SPCONV_ERR_UNSUPPORTED;
        }
        SPCONV_REQUIRE(((uintptr_t)feats & 15u) == 0 && ((uintptr_t)weight & 15u) == 0 &&
                       ((uintptr_t)out & 15u) == 0, SPCONV_ERR_ARG,
                       "tcgen05 conv needs 16-byte aligned feats/weight/out");
        return launch_conv_tc(a);
    }
    if (kernel_choice == SPCONV_KERNEL_AUTO && tc && ((uintptr_t)feats & 15u) == 0 &&
        ((uintptr_t)weight & 15u) == 0 && ((uintptr_t)out & 15u) == 0)
        return launch_conv_tc(a);
    return launch_conv_simt(a);
}

extern "C" int64_t spconv_conv_splitk_workspace_bytes(int64_t num_coords, int Co) {
    if (num_coords < 0 || Co <= 0) return -1;
    return conv_split_workspace_bytes(num_coords, Co);
}

extern "C" int spconv_submanifold_conv_forward_splitk(
    const void *feats, int dtype, int64_t M, int Ci,
    const void *weight, const void *bias, int Co, int V,
    const int32_t *nbr, const uint32_t *masks, const int32_t *order,
    void *workspace, int64_t workspace_bytes,
    void *out, int32_t *status, void *stream) {
    SPCONV_REQUIRE(M >= 0 && M <= 0x7fffffffLL, SPCONV_ERR_ARG, "num_coords %lld out of range", (long long)M);
    SPCONV_REQUIRE(Ci > 0 && Co > 0, SPCONV_ERR_ARG, "channels must be positive (Ci=%d Co=%d)", Ci, Co);
    SPCONV_REQUIRE(V > 0 && V <= 1024, SPCONV_ERR_ARG, "kernel volume %d out of range [1, 1024]", V);
    SPCONV_REQUIRE(dtype == SPCONV_F32 || dtype == SPCONV_F16 || dtype == SPCONV_BF16,
                   SPCONV_ERR_ARG, "unsupported dtype code %d", dtype);
    if (M == 0) return SPCONV_OK;
    SPCONV_REQUIRE(feats && weight && nbr && out, SPCONV_ERR_ARG, "null pointer argument");
    ConvArgs a{feats, dtype, M, Ci, weight, bias, Co, V, spconv_mask_words(V), nbr, masks, order,
               out, status, (cudaStream_t)stream};
    const bool tc = tc_supported(dtype, Ci, Co, V) && ((uintptr_t)feats & 15u) == 0 &&
                    ((uintptr_t)weight & 15u) == 0 && ((uintptr_t)out & 15u) == 0;
    stage_mark(SPCONV_STAGE_CONV, 0, a.stream);
    int rc;
    if (tc) {
        const int64_t need = conv_split_workspace_bytes(M, Co);
        SPCONV_REQUIRE(workspace && ((uintptr_t)workspace & 255u) == 0 && workspace_bytes >= need, SPCONV_ERR_ARG,
                       "split-K workspace must be 256-byte aligned and hold %lld bytes (got %lld)",
                       (long long)need, (long long)workspace_bytes);
        a.split_ws = workspace;
        rc = launch_conv_tc(a);
    } else {
        rc = launch_conv(a, SPCONV_KERNEL_AUTO);   // no tensor-core kernel: nothing to split
    }
    if (rc == SPCONV_OK) stage_mark(SPCONV_STAGE_CONV, 1, a.stream);
    return rc;
}

extern "C" int spconv_submanifold_conv_backward_input(
    const void *grad_out, int dtype, int64_t M, int Co, const void *weight_t, int Ci, int V,
    const int32_t *nbr, const uint32_t *masks, const int32_t *order,
    const int32_t *nbr_t, const uint32_t *masks_t, void *grad_in, int32_t *status, void *stream) {
    SPCONV_REQUIRE(M >= 0 && M <= 0x7fffffffLL, SPCONV_ERR_ARG, "num_coords %lld out of range", (long long)M);
    SPCONV_REQUIRE(Ci > 0 && Co > 0, SPCONV_ERR_ARG, "channels must be positive (Ci=%d Co=%d)", Ci, Co);
    SPCONV_REQUIRE(V > 0 && V <= 1024, SPCONV_ERR_ARG, "kernel volume %d out of range [1, 1024]", V);
    SPCONV_REQUIRE(dtype == SPCONV_F32 || dtype == SPCONV_F16 || dtype == SPCONV_BF16,
                   SPCONV_ERR_ARG, "unsupported dtype code %d", dtype);
    if (M == 0) return SPCONV_OK;
    // Odd V <=> every kernel side odd <=> offsets symmetric: the transpose is the flip.
    const bool flip = (V & 1) != 0;
    SPCONV_REQUIRE(grad_out && weight_t && grad_in && (flip ? nbr != nullptr : nbr_t != nullptr), SPCONV_ERR_ARG,
                   "null pointer argument (even kernel volumes need the transposed map)");
    ConvArgs a{grad_out, dtype, M, Co, weight_t, nullptr, Ci, V, spconv_mask_words(V),
               flip ? nbr : nbr_t, flip ? masks : masks_t, order, grad_in, status, (cudaStream_t)stream};
    a.flip = flip ? 1 : 0;
    stage_mark(SPCONV_STAGE_CONV, 0, a.stream);
    const int rc = launch_conv(a, SPCONV_KERNEL_AUTO);
    if (rc == SPCONV_OK) stage_mark(SPCONV_STAGE_CONV, 1, a.stream);
    return rc;
}

extern "C" int spconv_submanifold_conv_forward(
    const void *feats, int dtype, int64_t M, int Ci,
    const void *weight, const void *bias, int Co, int V,
    const int32_t *nbr, const uint32_t *masks, const int32_t *order,
    void *out, int32_t *status, void *stream) {
    return spconv_submanifold_conv_forward_ex(feats, dtype, M, Ci, weight, bias, Co, V, nbr, masks,
                                              order, out, status, stream, SPCONV_KERNEL_AUTO);
}
