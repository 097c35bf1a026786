// Dense <-> sparse conversion (SparseConvTensor.from_dense / .dense, core.py:52-77).
//
// from_dense: a voxel of a channels-last dense [B, W, H, D, C] tensor is active iff any of its
// C values is non-zero (NaN counts as non-zero, -0 as zero: the test is x != 0, as in
// torch's to_sparse). Three launches: dense_count_kernel flags the voxels of each 1024-voxel
// block and counts them; dense_scan_kernel turns the block counts into offsets and the total;
// the caller reads the total, allocates, and dense_compact_kernel writes the active voxels'
// (b, x, y, z) and features in grid order, which is (b, x, y, z)-sorted. Each pass reads the
// dense tensor once (16-byte loads when a voxel's C values are 16-byte aligned).
// dense: one thread per (voxel, channel) scatters features into a zeroed dense tensor, in
// channels-last or channels-first layout.
#include "common.cuh"

namespace spconv {

constexpr int kCvtThreads = 256;
constexpr int kCvtPerThread = 4;
constexpr int kCvtBlockVox = kCvtThreads * kCvtPerThread;     // voxels per count block

// Is any of voxel e's C values non-zero?
template <typename T>
__device__ __forceinline__ bool voxel_active(const T *__restrict__ x, int64_t e, int C, bool vec16) {
    const T *p = x + e * (int64_t)C;
    if (vec16) {
        const uint4 *q = reinterpret_cast<const uint4 *>(p);
        constexpr int kPer = 16 / sizeof(T);
        for (int c = 0; c < C / kPer; ++c) {
            const uint4 u = __ldg(q + c);
            const T *t = reinterpret_cast<const T *>(&u);
#pragma unroll
            for (int k = 0; k < kPer; ++k)
                if (dtype_traits<T>::to_f(t[k]) != 0.0f) return true;
        }
        return false;
    }
    for (int c = 0; c < C; ++c)
        if (dtype_traits<T>::to_f(__ldg(p + c)) != 0.0f) return true;
    return false;
}

template <typename T>
__global__ void __launch_bounds__(kCvtThreads)
dense_count_kernel(const T *__restrict__ x, int64_t nvox, int C, bool vec16, uint32_t *__restrict__ counts) {
    __shared__ uint32_t s_warp[kCvtThreads / 32];
    const int64_t base = (int64_t)blockIdx.x * kCvtBlockVox;
    uint32_t n = 0;
#pragma unroll
    for (int k = 0; k < kCvtPerThread; ++k) {
        const int64_t e = base + (int64_t)k * kCvtThreads + threadIdx.x;
        if (e < nvox && voxel_active(x, e, C, vec16)) ++n;
    }
    n = __reduce_add_sync(0xffffffffu, n);
    if ((threadIdx.x & 31) == 0) s_warp[threadIdx.x >> 5] = n;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t t = 0;
        for (int w = 0; w < kCvtThreads / 32; ++w) t += s_warp[w];
        counts[blockIdx.x] = t;
    }
}

// Exclusive scan of nblocks counts in place (one block); total into *total.
__global__ void __launch_bounds__(1024)
dense_scan_kernel(uint32_t *__restrict__ counts, int64_t nblocks, int64_t *__restrict__ total) {
    __shared__ uint64_t s_warp[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t per = (nblocks + 1023) / 1024;
    const int64_t b0 = (int64_t)tid * per, b1 = min(nblocks, b0 + per);
    uint64_t sum = 0;
    for (int64_t b = b0; b < b1; ++b) sum += counts[b];
    uint64_t incl = sum;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const uint64_t v = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += v;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    uint64_t run = incl - sum;
    for (int w = 0; w < warp; ++w) run += s_warp[w];
    for (int64_t b = b0; b < b1; ++b) {
        const uint32_t c = counts[b];
        counts[b] = (uint32_t)run;
        run += c;
    }
    if (tid == 1023) *total = (int64_t)run;
}

template <typename T>
__global__ void __launch_bounds__(kCvtThreads)
dense_compact_kernel(const T *__restrict__ x, int64_t nvox, int C, bool vec16, int W, int H, int D,
                     const uint32_t *__restrict__ offsets, int64_t M, int32_t *__restrict__ indices,
                     T *__restrict__ feats) {
    __shared__ uint32_t s_warp[kCvtThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t base = (int64_t)blockIdx.x * kCvtBlockVox;
    uint32_t run = offsets[blockIdx.x];
    // voxels k*256 .. k*256+255 of the block, in grid order: warps' counts in warp order
#pragma unroll 1
    for (int k = 0; k < kCvtPerThread; ++k) {
        const int64_t e = base + (int64_t)k * kCvtThreads + threadIdx.x;
        const bool act = e < nvox && voxel_active(x, e, C, vec16);
        const uint32_t bal = __ballot_sync(0xffffffffu, act);
        if (lane == 0) s_warp[warp] = __popc(bal);
        __syncthreads();
        uint32_t off = 0, tot = 0;
#pragma unroll
        for (int w = 0; w < kCvtThreads / 32; ++w) { const uint32_t c = s_warp[w]; off += w < warp ? c : 0u; tot += c; }
        if (act) {
            const int64_t r = (int64_t)run + off + __popc(bal & ((1u << lane) - 1u));
            if (r < M) {
                int64_t q = e;
                const int z = (int)(q % D); q /= D;
                const int y = (int)(q % H); q /= H;
                const int xx = (int)(q % W); q /= W;
                *reinterpret_cast<int4 *>(indices + 4 * r) = make_int4((int)q, xx, y, z);
                const T *src = x + e * (int64_t)C;
                T *dst = feats + r * (int64_t)C;
                for (int c = 0; c < C; ++c) dst[c] = src[c];
            }
        }
        run += tot;
        __syncthreads();                                  // s_warp is rewritten next
    }
}

template <typename T>
__global__ void __launch_bounds__(256)
sparse_to_dense_kernel(const T *__restrict__ feats, const int32_t *__restrict__ indices, int64_t M, int C,
                       int B, int W, int H, int D, bool channels_first, T *__restrict__ out, int32_t *status) {
    const int64_t total = M * (int64_t)C;
    const int64_t S = (int64_t)W * H * D;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = idx / C;
        const int c = (int)(idx - i * C);
        const int4 p = *reinterpret_cast<const int4 *>(indices + 4 * i);
        if ((uint32_t)p.x >= (uint32_t)B || (uint32_t)p.y >= (uint32_t)W || (uint32_t)p.z >= (uint32_t)H ||
            (uint32_t)p.w >= (uint32_t)D) {
            if (c == 0) raise_status(status, SPCONV_STATUS_COORD_RANGE);
            continue;
        }
        const int64_t cell = ((int64_t)p.y * H + p.z) * D + p.w;
        const int64_t o = channels_first ? (((int64_t)p.x * C + c) * S + cell) : (((int64_t)p.x * S + cell) * C + c);
        out[o] = feats[idx];
    }
}

template <typename T>
static int from_dense_t(const void *dense, int64_t nvox, int C, int W, int H, int D, void *workspace,
                        int32_t *indices, void *feats, int64_t capacity, int64_t *total, int phase,
                        cudaStream_t s) {
    const int64_t nblocks = (nvox + kCvtBlockVox - 1) / kCvtBlockVox;
    uint32_t *counts = (uint32_t *)workspace;
    const bool vec16 = ((C * sizeof(T)) % 16 == 0) && (((uintptr_t)dense & 15u) == 0);
    if (phase == 0) {
        dense_count_kernel<T><<<(unsigned)nblocks, kCvtThreads, 0, s>>>((const T *)dense, nvox, C, vec16, counts);
        if (int rc = check_launch("dense_count_kernel")) return rc;
        dense_scan_kernel<<<1, 1024, 0, s>>>(counts, nblocks, total);
        return check_launch("dense_scan_kernel");
    }
    dense_compact_kernel<T><<<(unsigned)nblocks, kCvtThreads, 0, s>>>((const T *)dense, nvox, C, vec16, W, H, D,
                                                                   counts, capacity, indices, (T *)feats);
    return check_launch("dense_compact_kernel");
}

}  // namespace spconv

using namespace spconv;

extern "C" int64_t spconv_from_dense_workspace_bytes(int batch, int W, int H, int D) {
    const long double nv = (long double)batch * W * H * D;
    if (batch <= 0 || W <= 0 || H <= 0 || D <= 0 || nv > 9.0e18L) return -1;
    const int64_t nblocks = ((int64_t)nv + kCvtBlockVox - 1) / kCvtBlockVox;
    return ((nblocks * 4 + 255) / 256) * 256 + 256;
}

extern "C" int spconv_from_dense(const void *dense, int dtype, int batch, int W, int H, int D, int C,
                                 void *workspace, int64_t workspace_bytes, int64_t *count,
                                 int32_t *indices, void *feats, int64_t capacity, int phase, void *stream) {
    SPCONV_REQUIRE(dtype == SPCONV_F32 || dtype == SPCONV_F16 || dtype == SPCONV_BF16, SPCONV_ERR_ARG,
                   "unsupported dtype code %d", dtype);
    SPCONV_REQUIRE(C > 0, SPCONV_ERR_ARG, "channels must be positive (C=%d)", C);
    const int64_t need = spconv_from_dense_workspace_bytes(batch, W, H, D);
    SPCONV_REQUIRE(need > 0 && workspace && workspace_bytes >= need, SPCONV_ERR_ARG,
                   "workspace missing or too small (%lld < %lld bytes)", (long long)workspace_bytes, (long long)need);
    SPCONV_REQUIRE(phase == 0 || phase == 1, SPCONV_ERR_ARG, "phase must be 0 (count) or 1 (write)");
    SPCONV_REQUIRE(dense && count, SPCONV_ERR_ARG, "null pointer argument");
    SPCONV_REQUIRE(phase == 0 || capacity == 0 || (indices && feats && ((uintptr_t)indices & 15u) == 0),
                   SPCONV_ERR_ARG, "indices must be 16-byte aligned, feats non-null");
    const int64_t nvox = (int64_t)batch * W * H * D;
    cudaStream_t s = (cudaStream_t)stream;
    if (phase == 1 && capacity == 0) return SPCONV_OK;
    switch (dtype) {
        case SPCONV_F32: return from_dense_t<float>(dense, nvox, C, W, H, D, workspace, indices, feats, capacity, count, phase, s);
        case SPCONV_F16: return from_dense_t<__half>(dense, nvox, C, W, H, D, workspace, indices, feats, capacity, count, phase, s);
        default: return from_dense_t<__nv_bfloat16>(dense, nvox, C, W, H, D, workspace, indices, feats, capacity, count, phase, s);
    }
}

extern "C" int spconv_to_dense(const void *feats, int dtype, const int32_t *indices, int64_t M, int C,
                               int batch, int W, int H, int D, int channels_first, void *out,
                               int32_t *status, void *stream) {
    SPCONV_REQUIRE(dtype == SPCONV_F32 || dtype == SPCONV_F16 || dtype == SPCONV_BF16, SPCONV_ERR_ARG,
                   "unsupported dtype code %d", dtype);
    SPCONV_REQUIRE(M >= 0 && C > 0 && batch > 0 && W > 0 && H > 0 && D > 0, SPCONV_ERR_ARG,
                   "bad sizes (M=%lld C=%d N=%d W=%d H=%d D=%d)", (long long)M, C, batch, W, H, D);
    SPCONV_REQUIRE(out, SPCONV_ERR_ARG, "null output");
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t bytes = (int64_t)batch * W * H * D * C * (dtype == SPCONV_F32 ? 4 : 2);
    if (cudaMemsetAsync(out, 0, (size_t)bytes, s) != cudaSuccess) return check_launch("dense memset");
    if (M == 0) return SPCONV_OK;
    SPCONV_REQUIRE(feats && indices && ((uintptr_t)indices & 15u) == 0, SPCONV_ERR_ARG,
                   "feats / 16-byte aligned indices required");
    int64_t blocks = (M * C + 255) / 256;
    if (blocks > 148LL * 64) blocks = 148LL * 64;
    const bool cf = channels_first != 0;
    switch (dtype) {
        case SPCONV_F32:
            sparse_to_dense_kernel<float><<<(unsigned)blocks, 256, 0, s>>>((const float *)feats, indices, M, C, batch, W, H, D, cf, (float *)out, status);
            break;
        case SPCONV_F16:
            sparse_to_dense_kernel<__half><<<(unsigned)blocks, 256, 0, s>>>((const __half *)feats, indices, M, C, batch, W, H, D, cf, (__half *)out, status);
            break;
        default:
            sparse_to_dense_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, s>>>((const __nv_bfloat16 *)feats, indices, M, C, batch, W, H, D, cf, (__nv_bfloat16 *)out, status);
    }
    return check_launch("sparse_to_dense_kernel");
}
