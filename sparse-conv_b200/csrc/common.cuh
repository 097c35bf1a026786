// Shared helpers for the sm_100a kernels of the submanifold-conv library:
// status bits, error plumbing, and thin inline-PTX wrappers for mbarriers, cp.async,
// the async-proxy fence and the tcgen05 (5th-generation tensor core / TMEM) instructions.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include "../../include/sparseconv_b200.h"

namespace spconv {

// ---------------------------------------------------------------------------------------
// Host-side error message (thread-local) and launch checking.
// ---------------------------------------------------------------------------------------
void set_error(const char *fmt, ...);
int check_launch(const char *what);
// Records the start (which = 0) or end (which = 1) event of a stage when stage timing is on.
void stage_mark(int stage, int which, cudaStream_t stream);

#define SPCONV_REQUIRE(cond, code, ...)   \
    do {                                  \
        if (!(cond)) {                    \
            ::spconv::set_error(__VA_ARGS__); \
            return (code);                \
        }                                 \
    } while (0)

// ---------------------------------------------------------------------------------------
// Device-side status: kernels OR bits into a caller-provided int32 word.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void raise_status(int32_t *status, int32_t bits) {
    if (status) atomicOr(status, bits);
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Default upper bound on a spin-wait inside a kernel. A wait that exceeds its limit raises
// SPCONV_STATUS_WAIT_TIMEOUT and the kernel abandons its remaining work. The limit of the
// pipeline waits is a kernel argument (spconv_set_wait_limit_ns sets it for later launches);
// the clean-up waits of an abandoned kernel (for its own copies and MMAs, which always
// complete) keep this fixed bound.
constexpr uint64_t kWaitLimitNs = 2000000000ull;   // 2 s
// The pipeline-wait limit the next conv launches pass to their kernels (process-wide).
uint64_t wait_limit_ns();

// 32-bit murmur3 finaliser (a well-mixed bijection on uint32).
__device__ __forceinline__ uint32_t fmix32(uint32_t k) {
    k ^= k >> 16;
    k *= 0x85ebca6bu;
    k ^= k >> 13;
    k *= 0xc2b2ae35u;
    k ^= k >> 16;
    return k;
}

__device__ __forceinline__ uint64_t fmix64(uint64_t k) {
    k ^= k >> 33;
    k *= 0xff51afd7ed558ccdull;
    k ^= k >> 33;
    k *= 0xc4ceb9fe1a85ec53ull;
    k ^= k >> 33;
    return k;
}

// ---------------------------------------------------------------------------------------
// Shared-memory address helpers.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------------------
// cp.async (Ampere-style, 16 B, L2-only) with zero fill when src_bytes == 0.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n"
                 :: "r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_4(uint32_t dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" :: "r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" :: "n"(N) : "memory");
}

// Makes generic-proxy writes to shared memory visible to the async proxy (tcgen05.mma).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

// ---------------------------------------------------------------------------------------
// Programmatic dependent launch. A kernel launched with launch_pdl may start while the
// previous kernel on the stream is still finishing (its own setup overlaps that kernel's
// tail); it calls grid_dependency_wait() before it reads anything that kernel wrote. Without
// a programmatic launch the wait returns at once.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void grid_dependency_wait() {
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
}

// Lets the next kernel on the stream (if launched with launch_pdl) start its blocks now
// instead of when this grid exits. Safe at any point: the next kernel still waits, in
// grid_dependency_wait(), for this whole grid to complete and its writes to be visible; it
// starts only once every block of this grid has made the call or exited, so its waiting
// blocks never hold resources this grid's blocks still need.
__device__ __forceinline__ void grid_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// ---------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t addr, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" :: "r"(addr), "r"(count) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, P;\n\t}\n"
        : "=r"(ok) : "r"(addr), "r"(parity) : "memory");
    return ok != 0;
}
// Non-blocking test: has the phase with the given parity completed?
__device__ __forceinline__ bool mbar_test(uint32_t addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, P;\n\t}\n"
        : "=r"(ok) : "r"(addr), "r"(parity) : "memory");
    return ok != 0;
}
// Bounded wait for the phase with the given parity to complete. Returns false on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t addr, uint32_t parity,
                                                  uint64_t limit_ns = kWaitLimitNs) {
    if (mbar_try_wait(addr, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait(addr, parity)) return true;
        if (globaltimer_ns() - t0 > limit_ns) return false;
    }
}
// Clean-up bound of an abandoned kernel waiting for its own weight-tile TMA loads: their
// barrier phase may never complete (a gatherer that gave up does not arrive), and a load of a
// few KB from L2/HBM lands within microseconds, so 200 us covers it with a wide margin.
constexpr uint64_t kTmaDrainNs = 200000ull;

__device__ __forceinline__ void mbar_arrive(uint32_t addr) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}\n"
                 :: "r"(addr) : "memory");
}
// Arrive and add `bytes` to the phase's expected transaction count (TMA completions).
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t addr, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}\n"
                 :: "r"(addr), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor) into this CTA's shared memory, completion on one of its mbarriers.
// ---------------------------------------------------------------------------------------
// One box of a 2-D tensor at (x, y).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void *tmap, int x, int y, uint32_t mbar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];\n"
        :: "r"(dst), "l"(tmap), "r"(x), "r"(y), "r"(mbar) : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const void *tmap) {
    asm volatile("prefetch.tensormap [%0];\n" :: "l"(tmap) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;\n" ::: "memory");
}
// Named barrier among `count` threads (id 1..15; id 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;\n" :: "r"(id), "r"(count) : "memory");
}
// Bounded wait that also gives up when another role of the CTA has flagged an abort.
// On timeout it sets the flag itself. Returns false when the caller must abandon its work.
__device__ __forceinline__ bool mbar_wait_or_abort(uint32_t addr, uint32_t parity,
                                                   volatile int *abort_flag, uint64_t limit_ns) {
    if (mbar_try_wait(addr, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait(addr, parity)) return true;
        if (*abort_flag) return false;
        if (globaltimer_ns() - t0 > limit_ns) {
            *abort_flag = 1;
            return false;
        }
    }
}

// ---------------------------------------------------------------------------------------
// tcgen05 (sm_100a): TMEM allocation, MMA issue/commit, TMEM -> register loads.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n"
                 :: "r"(dst_smem), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n"
                 :: "r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (fp16/bf16 in, fp32 accumulate).
__device__ __forceinline__ void tc_mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
        :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
// Arrive (once) on the mbarrier when every tcgen05.mma issued so far by this thread is done.
__device__ __forceinline__ void tc_commit(uint32_t mbar_addr) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n"
                 :: "r"(mbar_addr) : "memory");
}
__device__ __forceinline__ void tc_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}
// 32 lanes x 32 bits, 8 consecutive columns: thread l of the warp gets lane (base+l).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t *r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
          "=r"(r[6]), "=r"(r[7])
        : "r"(taddr) : "memory");
}
// 32 lanes x 32 bits, 16 consecutive columns: thread l of the warp gets lane (base+l).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
          "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
          "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr) : "memory");
}

// Shared-memory matrix descriptor for tcgen05.mma, K-major operand without swizzle
// ("interleaved" canonical layout): 8-row x 16-byte core matrices; `lbo` is the byte
// distance between core matrices adjacent in K, `sbo` between core matrices adjacent in
// M/N. Bits 46-47 hold the descriptor version (1 on sm_100); layout type 0 = no swizzle.
__device__ __forceinline__ uint64_t smem_desc_kmajor_noswizzle(uint32_t saddr, uint32_t lbo,
                                                               uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    return d;
}

// Shared-memory matrix descriptor, K-major with a 32/64/128-byte swizzle (the layout a TMA
// load with the same swizzle writes): rows of `row_bytes` (= the swizzle width) one after
// another, 8-row groups 8 * row_bytes apart, and within each row the 16-byte chunk index
// XOR-ed with address bits 7 and up (bits [4, 4+log2(row_bytes/16)) ^= bits [7, ...)).
// The tile must start on a multiple of 8 * row_bytes; a K step of 16 elements inside the
// row advances `saddr` by 32 bytes.
__device__ __forceinline__ uint64_t smem_desc_kmajor_swizzled(uint32_t saddr, uint32_t row_bytes) {
    const uint64_t layout = row_bytes == 128 ? 2u : (row_bytes == 64 ? 4u : 6u);
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1 << 16;                                   // leading offset: unused, 1
    d |= (uint64_t)(((8u * row_bytes) >> 4) & 0x3FFFu) << 32; // 8-row group stride
    d |= (uint64_t)1 << 46;                                   // descriptor version
    d |= layout << 61;
    return d;
}

// Instruction descriptor, kind::f16: D = f32, A/B = f16 (0) or bf16 (1), both K-major.
__host__ __device__ constexpr uint32_t instr_desc_f16(int ab_format, int M, int N) {
    return (1u << 4)                                   // D format: f32
         | ((uint32_t)ab_format << 7)                  // A format
         | ((uint32_t)ab_format << 10)                 // B format
         | ((uint32_t)(N >> 3) << 17)                  // N / 8
         | ((uint32_t)(M >> 4) << 24);                 // M / 16
}

template <typename T> struct dtype_traits;
template <> struct dtype_traits<float> {
    static __device__ __forceinline__ float to_f(float x) { return x; }
    static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <> struct dtype_traits<__half> {
    static constexpr int mma_format = 0;
    static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
    static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};
template <> struct dtype_traits<__nv_bfloat16> {
    static constexpr int mma_format = 1;
    static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

}  // namespace spconv
