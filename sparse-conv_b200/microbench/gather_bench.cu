// Microbenchmark (not part of the library): random row-gather throughput into shared memory
// on sm_100a, the measurement behind the conv kernel's choice of warp-local cp.async gathers.
//  mode 0: TMA tile::gather4, P producer warps (elected lane issues its share), 1 consumer
//  mode 1: TMA tile::gather4, P producer warps, all 32 lanes issue (one gather4 each)
//  mode 2: cp.async 16 B, W warps, each warp gathers its own 32-row slice (coalesced lanes per row)
// Every CTA walks tiles of 128 indices (all indices valid, in [0, M)).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstdio>

#define DEV __device__ __forceinline__
DEV uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
DEV void mbar_init(uint32_t a, uint32_t c) { asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(a), "r"(c) : "memory"); }
DEV bool mbar_try(uint32_t a, uint32_t p) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred P;\n\tmbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\tselp.b32 %0, 1, 0, P;\n\t}" : "=r"(ok) : "r"(a), "r"(p) : "memory");
    return ok;
}
DEV uint64_t gtime() { uint64_t t; asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t)); return t; }
DEV bool mbar_wait(uint32_t a, uint32_t p) {
    uint64_t t0 = gtime();
    while (!mbar_try(a, p)) if (gtime() - t0 > 1000000000ull) return false;
    return true;
}
DEV void mbar_arrive(uint32_t a) { asm volatile("{\n\t.reg .b64 s;\n\tmbarrier.arrive.shared::cta.b64 s, [%0];\n\t}" :: "r"(a) : "memory"); }
DEV void mbar_expect(uint32_t a, uint32_t b) { asm volatile("{\n\t.reg .b64 s;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 s, [%0], %1;\n\t}" :: "r"(a), "r"(b) : "memory"); }
DEV void gather4(uint32_t dst, const void *map, int x, int4 r, uint32_t bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, %6}], [%7];"
                 :: "r"(dst), "l"(map), "r"(x), "r"(r.x), "r"(r.y), "r"(r.z), "r"(r.w), "r"(bar) : "memory");
}
DEV void cpa16(uint32_t dst, const void *src) { asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(dst), "l"(src) : "memory"); }

__device__ int g_err;

// TMA gather. Warps 0..P-1 produce, warp P consumes. Stage = 128 rows x RB bytes.
template <int RB, int S, bool ALL_LANES>
__global__ void k_tma(const __grid_constant__ CUtensorMap map, const int32_t *idx, int ntiles, int P) {
    extern __shared__ uint8_t smraw[];
    uint8_t *base = (uint8_t *)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
    uint64_t *full = (uint64_t *)(base + S * 128 * RB), *empty = full + S;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) { mbar_init(smem_u32(&full[s]), P); mbar_init(smem_u32(&empty[s]), 1); }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const int G = gridDim.x;
    int nt = blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / G + 1 : 0;
    if (warp < P) {
        const int groups = 32 / P;             // gather4 groups per producer warp
        for (int k = 0; k < nt; ++k) {
            const int tile = blockIdx.x + k * G;
            const int s = k % S, u = k / S;
            if (u > 0 && !mbar_wait(smem_u32(&empty[s]), (u - 1) & 1)) { g_err = 1; return; }
            const uint32_t dst0 = smem_u32(base + s * 128 * RB);
            if (ALL_LANES) {
                if (lane == 0) mbar_expect(smem_u32(&full[s]), groups * 4 * RB);
                __syncwarp();
                if (lane < groups) {
                    const int gidx = warp * groups + lane;
                    const int4 r = *(const int4 *)(idx + (int64_t)tile * 128 + gidx * 4);
                    gather4(dst0 + gidx * 4 * RB, &map, 0, r, smem_u32(&full[s]));
                }
            } else if (lane == 0) {
                mbar_expect(smem_u32(&full[s]), groups * 4 * RB);
                for (int q = 0; q < groups; ++q) {
                    const int gidx = warp * groups + q;
                    const int4 r = *(const int4 *)(idx + (int64_t)tile * 128 + gidx * 4);
                    gather4(dst0 + gidx * 4 * RB, &map, 0, r, smem_u32(&full[s]));
                }
            }
        }
    } else if (warp == P && lane == 0) {
        for (int k = 0; k < nt; ++k) {
            const int s = k % S, u = k / S;
            if (!mbar_wait(smem_u32(&full[s]), u & 1)) { g_err = 2; return; }
            mbar_arrive(smem_u32(&empty[s]));
        }
    }
}

// cp.async gather: each warp owns a 32-row slice of every tile, D-deep pipeline per warp.
template <int RB, int D>
__global__ void k_cpasync(const uint8_t *feats, const int32_t *idx, int ntiles, int64_t M) {
    extern __shared__ uint8_t smraw[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, W = blockDim.x >> 5;
    constexpr int LPR = RB / 16, RPI = 32 / LPR, NQ = 32 / RPI;   // instructions per 32 rows
    uint8_t *mine = smraw + warp * D * 32 * RB;
    const int G = gridDim.x;
    // warp w handles slices w % 4 of tiles (blockIdx + G * (k * (W/4) + w/4))
    const int wpt = W / 4 > 0 ? W / 4 : 1;
    int k = 0;
    for (int tile = blockIdx.x + G * (warp / 4); tile < ntiles; tile += G * wpt, ++k) {
        const int slice = warp % 4;
        uint8_t *dst = mine + (k % D) * 32 * RB;
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
            const int r = q * RPI + lane / LPR;
            const int n = idx[(int64_t)tile * 128 + slice * 32 + r];
            cpa16(smem_u32(dst + r * RB + (lane % LPR) * 16), feats + (int64_t)n * RB + (lane % LPR) * 16);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_group %0;" :: "n"(D - 1) : "memory");
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
}

typedef CUresult (*EncFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *, const cuuint64_t *,
                          const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                          CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

template <int RB>
static float run_tma(const void *feats, int64_t M, const int32_t *idx, int ntiles, int P, bool all, int grid) {
    void *p = nullptr; cudaDriverEntryPointQueryResult q;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    CUtensorMap map;
    cuuint64_t dims[2] = {(cuuint64_t)(RB / 2), (cuuint64_t)M}, str[1] = {(cuuint64_t)RB};
    cuuint32_t box[2] = {(cuuint32_t)(RB / 2), 1}, es[2] = {1, 1};
    CUtensorMapSwizzle sw = RB == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : (RB == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
    if (((EncFn)p)(&map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(feats), dims, str, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return -1.f;
    constexpr int S = 8;
    const int smem = S * 128 * RB + 2 * S * 8 + 1024;
    auto kern = all ? k_tma<RB, S, true> : k_tma<RB, S, false>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaEvent_t a, b; cudaEventCreate(&a); cudaEventCreate(&b);
    kern<<<grid, (P + 1) * 32, smem>>>(map, idx, ntiles, P);
    cudaEventRecord(a);
    kern<<<grid, (P + 1) * 32, smem>>>(map, idx, ntiles, P);
    cudaEventRecord(b); cudaEventSynchronize(b);
    float ms; cudaEventElapsedTime(&ms, a, b);
    return ms;
}

template <int RB>
static float run_cpa(const void *feats, int64_t M, const int32_t *idx, int ntiles, int W, int grid) {
    constexpr int D = 6;
    const int smem = W * D * 32 * RB;
    auto kern = k_cpasync<RB, D>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaEvent_t a, b; cudaEventCreate(&a); cudaEventCreate(&b);
    kern<<<grid, W * 32, smem>>>((const uint8_t *)feats, idx, ntiles, M);
    cudaEventRecord(a);
    kern<<<grid, W * 32, smem>>>((const uint8_t *)feats, idx, ntiles, M);
    cudaEventRecord(b); cudaEventSynchronize(b);
    float ms; cudaEventElapsedTime(&ms, a, b);
    return ms;
}

extern "C" float gb_run(int mode, int rb, const void *feats, long long M, const int32_t *idx, int ntiles, int P, int grid) {
    if (mode == 0 || mode == 1) {
        const bool all = mode == 1;
        if (rb == 32) return run_tma<32>(feats, M, idx, ntiles, P, all, grid);
        if (rb == 64) return run_tma<64>(feats, M, idx, ntiles, P, all, grid);
        return run_tma<128>(feats, M, idx, ntiles, P, all, grid);
    }
    if (rb == 32) return run_cpa<32>(feats, M, idx, ntiles, P, grid);
    if (rb == 64) return run_cpa<64>(feats, M, idx, ntiles, P, grid);
    return run_cpa<128>(feats, M, idx, ntiles, P, grid);
}
extern "C" int gb_err() { int e = 0; cudaMemcpyFromSymbol(&e, g_err, 4); cudaError_t c = cudaGetLastError(); return c ? 1000 + (int)c : e; }
