// Coordinate hash table + submanifold kernel-map builder for sm_100a.
//
// Replaces the reference's three-step build (neighbor_map.cu:179-237): the 3-D insert
// kernel (hash.cu:367-409, one atomicCAS per voxel into a table sized int(2M)), a
// torch::full pre-fill of the [M,V] map, and one lookup thread per (voxel, offset)
// (neighbor_map.cu:132-177) that writes only the found entries.
//
// Here:
//   1. one cudaMemsetAsync clears the workspace (table, histogram, counters);
//   2. insert_kernel: one thread per voxel, a coalesced int4 load, a bounded linear probe
//      into a power-of-two table of packed 64-bit slots ((key << 32) | row, stored
//      complemented so that all-zero means empty). Capacity >= 2M keeps the load <= 0.5 and
//      the table L2-resident (32 MB at 2M voxels);
//   3. map_kernel: one warp per voxel probes all V offsets (lane l takes offsets l, l+32, ..)
//      and writes the voxel's V entries as one contiguous store (no pre-fill pass); a ballot
//      gives each 32-bit word of the voxel's offset mask. A block owns 512 consecutive
//      voxels, histograms them by an order key (popcount class, mask hash), and the last
//      block to finish turns the histogram into bucket offsets;
//   4. order_kernel: a counting-sort scatter of voxel ids by that key, aggregated per block
//      so the hot bucket takes one global atomic per block.
// The map is a pure function of the coordinates: for duplicate-free inputs any correct
// table gives the reference's map bit for bit. The row order used by the conv kernels
// (`order`) depends on atomics and is unspecified within a bucket; the conv results do not.
#include <cstdio>
#include <cstdarg>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace spconv {

constexpr int kOrderBuckets = 4096;    // 16 popcount classes x 256 mask-hash buckets
constexpr int kMapThreads = 256;
constexpr int kMapVoxels = 512;        // voxels per map_kernel block
constexpr int kOrderThreads = 256;
constexpr int kOrderPerThread = 8;     // voxels per thread in order_kernel
constexpr int kMaxKernelVolume = 1024;

static int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

struct WsLayout {
    int64_t cap = 0;
    bool key64 = false;
    int64_t table = 0, vals = 0, hist = 0, cursor = 0, counter = 0, total = 0;
};

static bool volume_fits_32(int batch, int W, int H, int D) {
    const long double vol = (long double)batch * W * H * D;
    return vol < 4294967296.0L;
}

static WsLayout ws_layout(int64_t M, bool key64) {
    WsLayout L;
    L.cap = spconv_hashmap_capacity(M);
    L.key64 = key64;
    int64_t off = 0;
    L.table = off; off += align256(L.cap * 8);
    if (key64) { L.vals = off; off += align256(L.cap * 4); }
    L.hist = off; off += align256(kOrderBuckets * 4);
    L.cursor = off; off += align256(kOrderBuckets * 4);
    L.counter = off; off += 256;
    L.total = off;
    return L;
}

// Warp-aggregated shared-memory increment: returns this lane's rank among all increments
// of `counter[key]` made so far (lanes with equal keys take consecutive ranks).
__device__ __forceinline__ uint32_t aggregated_inc(uint32_t *counter, uint32_t key, uint32_t active) {
    const uint32_t peers = __match_any_sync(active, key);
    const int lane = threadIdx.x & 31;
    const int leader = __ffs(peers) - 1;
    const uint32_t lt = peers & ((1u << lane) - 1u);
    uint32_t base = 0;
    if (lane == leader) base = atomicAdd(counter + key, (uint32_t)__popc(peers));
    base = __shfl_sync(peers, base, leader);
    return base + __popc(lt);
}

// ---------------------------------------------------------------------------------------
// Table: packed 64-bit slots for volumes < 2^32 (key = flat index), or 64-bit keys plus a
// separate value array otherwise. Stored complemented; 0 = empty.
// ---------------------------------------------------------------------------------------
template <bool KEY64>
__device__ __forceinline__ bool table_insert(unsigned long long *table, uint32_t *vals,
                                             uint64_t mask, uint64_t flat, uint32_t row,
                                             int32_t *status) {
    if (!KEY64) {
        const uint32_t key = (uint32_t)flat;
        const unsigned long long desired = ~((((unsigned long long)key) << 32) | row);
        uint64_t s = fmix32(key) & mask;
        for (uint64_t p = 0; p <= mask; ++p) {
            const unsigned long long prev = atomicCAS(table + s, 0ull, desired);
            if (prev == 0ull) return true;
            if ((uint32_t)((~prev) >> 32) == key) {
                // Duplicate coordinate: keep the highest row (min of the complement).
                atomicMin(table + s, desired);
                raise_status(status, SPCONV_STATUS_DUPLICATE);
                return true;
            }
            s = (s + 1) & mask;
        }
        return false;
    } else {
        const unsigned long long kst = ~(unsigned long long)flat;
        uint64_t s = fmix64(flat) & mask;
        for (uint64_t p = 0; p <= mask; ++p) {
            const unsigned long long prev = atomicCAS(table + s, 0ull, kst);
            if (prev == 0ull || prev == kst) {
                if (prev == kst) raise_status(status, SPCONV_STATUS_DUPLICATE);
                atomicMax(vals + s, row);
                return true;
            }
            s = (s + 1) & mask;
        }
        return false;
    }
}

// Returns the row of `flat`, -1 if absent, -2 if the probe wrapped the whole table.
template <bool KEY64>
__device__ __forceinline__ int32_t table_lookup(const unsigned long long *__restrict__ table,
                                                const uint32_t *__restrict__ vals,
                                                uint64_t mask, uint64_t flat) {
    if (!KEY64) {
        const uint32_t key = (uint32_t)flat;
        uint64_t s = fmix32(key) & mask;
        for (uint64_t p = 0; p <= mask; ++p) {
            const unsigned long long w = __ldg(table + s);
            if (w == 0ull) return -1;
            if ((uint32_t)((~w) >> 32) == key) return (int32_t)(uint32_t)(~w);
            s = (s + 1) & mask;
        }
        return -2;
    } else {
        const unsigned long long kst = ~(unsigned long long)flat;
        uint64_t s = fmix64(flat) & mask;
        for (uint64_t p = 0; p <= mask; ++p) {
            const unsigned long long w = __ldg(table + s);
            if (w == 0ull) return -1;
            if (w == kst) return (int32_t)__ldg(vals + s);
            s = (s + 1) & mask;
        }
        return -2;
    }
}

// ---------------------------------------------------------------------------------------
// 1. Insert (replaces hash.cu:367-389 + hash.cuh:22-63).
// ---------------------------------------------------------------------------------------
template <bool KEY64>
__global__ void __launch_bounds__(256)
insert_kernel(const int4 *__restrict__ coords, int64_t M, int N, int W, int H, int D,
              unsigned long long *table, uint32_t *vals, uint64_t mask, int32_t *status) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < M;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int4 c = __ldg(coords + i);
        if (c.x < 0 || c.x >= N || c.y < 0 || c.y >= W || c.z < 0 || c.z >= H || c.w < 0 || c.w >= D) {
            raise_status(status, SPCONV_STATUS_COORD_RANGE);
            continue;
        }
        const uint64_t flat = ((((uint64_t)c.x * W + c.y) * H + c.z) * D) + c.w;
        if (!table_insert<KEY64>(table, vals, mask, flat, (uint32_t)i, status))
            raise_status(status, SPCONV_STATUS_TABLE_FULL);
    }
}

// ---------------------------------------------------------------------------------------
// 2. Fused map + masks + order histogram (replaces torch::full + neighbor_map.cu:132-177).
//    One warp per voxel: lane l handles offsets l, l+32, ...; a ballot yields each 32-bit
//    word of the voxel's offset mask directly, and the V entries of the voxel are one
//    contiguous store. Successive voxels of a block are adjacent, so the block writes one
//    contiguous range of the map.
// ---------------------------------------------------------------------------------------
template <bool KEY64>
__global__ void __launch_bounds__(kMapThreads)
map_kernel(const int4 *__restrict__ coords, int64_t M, int W, int H, int D,
           int Kw, int Kh, int Kd, int Dw, int Dh, int Dd, int V, int MW,
           const unsigned long long *__restrict__ table, const uint32_t *__restrict__ vals,
           uint64_t tmask, int32_t *__restrict__ nbr, uint32_t *__restrict__ masks,
           uint32_t *hist, uint32_t *cursor, uint32_t *done_counter, int32_t *status) {
    __shared__ uint32_t s_hist[kOrderBuckets];
    __shared__ uint32_t s_is_last;
    __shared__ uint32_t s_warp[kMapThreads / 32];
    extern __shared__ int4 s_off[];                   // [V] (ox, oy, oz, unused)

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t i0 = (int64_t)blockIdx.x * kMapVoxels;
    const int nvox = (M - i0) < (int64_t)kMapVoxels ? (int)(M - i0) : kMapVoxels;

    for (int v = tid; v < V; v += kMapThreads) {
        const int KhKd = Kh * Kd;
        const int ox = (v / KhKd) * Dw - (Kw / 2) * Dw;
        const int oy = ((v / Kd) % Kh) * Dh - (Kh / 2) * Dh;
        const int oz = (v % Kd) * Dd - (Kd / 2) * Dd;
        s_off[v] = make_int4(ox, oy, oz, 0);
    }
    for (int j = tid; j < kOrderBuckets; j += kMapThreads) s_hist[j] = 0u;
    __syncthreads();

    const int center = V / 2;
    bool wrapped = false;
    for (int j = warp; j < nvox; j += kMapThreads / 32) {
        const int64_t i = i0 + j;
        const int4 c = __ldg(coords + i);
        int32_t *out = nbr + i * (int64_t)V;
        uint32_t *mrow = masks + i * (int64_t)MW;
        uint32_t pc = 0, h = 0x9e3779b9u;
        for (int vb = 0; vb < V; vb += 32) {
            const int v = vb + lane;
            int32_t value = -1;
            if (v < V) {
                if (v == center) {
                    value = (int32_t)i;
                } else {
                    const int4 o = s_off[v];
                    const int kx = c.y + o.x, ky = c.z + o.y, kz = c.w + o.z;
                    if (kx >= 0 && kx < W && ky >= 0 && ky < H && kz >= 0 && kz < D) {
                        const uint64_t flat = ((((uint64_t)(int64_t)c.x * W + kx) * H + ky) * D) + kz;
                        value = table_lookup<KEY64>(table, vals, tmask, flat);
                        if (value == -2) { wrapped = true; value = -1; }
                    }
                }
                out[v] = value;
            }
            const uint32_t bits = __ballot_sync(0xffffffffu, value >= 0);
            if (lane == 0) mrow[vb >> 5] = bits;
            pc += __popc(bits);
            h = fmix32(h ^ bits);
        }
        if (lane == 0) {
            const uint32_t cls = pc == 0 ? 0u : min(pc - 1u, 15u);
            atomicAdd(&s_hist[cls * 256u + (h & 255u)], 1u);
        }
    }
    if (wrapped) raise_status(status, SPCONV_STATUS_TABLE_FULL);
    __syncthreads();
    for (int b = tid; b < kOrderBuckets; b += kMapThreads)
        if (s_hist[b]) atomicAdd(hist + b, s_hist[b]);

    // The last block to finish converts the global histogram into bucket start offsets.
    __threadfence();
    __syncthreads();
    if (tid == 0) s_is_last = (atomicAdd(done_counter, 1u) == gridDim.x - 1) ? 1u : 0u;
    __syncthreads();
    if (!s_is_last) return;
    __threadfence();
    constexpr int per = kOrderBuckets / kMapThreads;   // 16 buckets per thread
    uint32_t local[per];
    uint32_t sum = 0;
#pragma unroll
    for (int k = 0; k < per; ++k) { local[k] = __ldcg(hist + tid * per + k); sum += local[k]; }
    uint32_t incl = sum;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const uint32_t n = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += n;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    uint32_t run = incl - sum;
    for (int w = 0; w < warp; ++w) run += s_warp[w];
#pragma unroll
    for (int k = 0; k < per; ++k) { cursor[tid * per + k] = run; run += local[k]; }
}

// ---------------------------------------------------------------------------------------
// 3. Counting-sort scatter of voxel ids by order key.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kOrderThreads)
order_kernel(const uint32_t *__restrict__ masks, int64_t M, int MW, uint32_t *cursor,
             int32_t *__restrict__ order, int32_t *status) {
    __shared__ uint32_t s_cnt[kOrderBuckets];
    __shared__ uint32_t s_base[kOrderBuckets];
    const int tid = threadIdx.x;
    const int64_t i0 = (int64_t)blockIdx.x * (kOrderThreads * kOrderPerThread);
    for (int b = tid; b < kOrderBuckets; b += kOrderThreads) s_cnt[b] = 0u;
    __syncthreads();
    uint32_t key[kOrderPerThread], rank[kOrderPerThread];
#pragma unroll
    for (int k = 0; k < kOrderPerThread; ++k) {
        const int64_t i = i0 + k * kOrderThreads + tid;
        const bool valid = i < M;
        key[k] = 0;
        if (valid) {
            const uint32_t *g = masks + i * (int64_t)MW;
            uint32_t pc = 0, h = 0x9e3779b9u;
            for (int w = 0; w < MW; ++w) { const uint32_t x = __ldg(g + w); pc += __popc(x); h = fmix32(h ^ x); }
            const uint32_t cls = pc == 0 ? 0u : min(pc - 1u, 15u);
            key[k] = cls * 256u + (h & 255u);
        }
        const uint32_t active = __ballot_sync(0xffffffffu, valid);
        rank[k] = valid ? aggregated_inc(s_cnt, key[k], active) : 0u;
    }
    __syncthreads();
    for (int b = tid; b < kOrderBuckets; b += kOrderThreads)
        if (s_cnt[b]) s_base[b] = atomicAdd(cursor + b, s_cnt[b]);
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kOrderPerThread; ++k) {
        const int64_t i = i0 + k * kOrderThreads + tid;
        if (i < M) {
            const uint32_t pos = s_base[key[k]] + rank[k];
            if (pos < (uint64_t)M) order[pos] = (int32_t)i;
            else raise_status(status, SPCONV_STATUS_TABLE_FULL);   // inconsistent histogram
        }
    }
}

}  // namespace spconv

using namespace spconv;

extern "C" int64_t spconv_hashmap_capacity(int64_t num_coords) {
    int64_t need = num_coords > 0 ? 2 * num_coords : 0;
    int64_t cap = 1024;
    while (cap < need) cap <<= 1;
    return cap;
}

extern "C" int spconv_mask_words(int kernel_volume) {
    return kernel_volume <= 0 ? 0 : (kernel_volume + 31) / 32;
}

extern "C" int64_t spconv_neighbor_map_workspace_bytes(int64_t num_coords, int batch, int W, int H, int D) {
    if (num_coords < 0) return -1;
    return ws_layout(num_coords, !volume_fits_32(batch, W, H, D)).total;
}

extern "C" int spconv_build_submanifold_neighbor_map(
    const int32_t *coords, int64_t M,
    int batch, int W, int H, int D,
    int Kw, int Kh, int Kd, int Dw, int Dh, int Dd,
    void *workspace, int64_t workspace_bytes,
    int32_t *neighbor_map, uint32_t *masks, int32_t *order,
    int32_t *status, void *stream_ptr) {
    SPCONV_REQUIRE(M >= 0, SPCONV_ERR_ARG, "num_coords must be >= 0 (got %lld)", (long long)M);
    SPCONV_REQUIRE(M <= 0x7fffffffLL, SPCONV_ERR_ARG, "num_coords %lld exceeds 2^31-1 rows", (long long)M);
    SPCONV_REQUIRE(batch > 0 && W > 0 && H > 0 && D > 0, SPCONV_ERR_ARG,
                   "spatial shape must be positive (N=%d W=%d H=%d D=%d)", batch, W, H, D);
    SPCONV_REQUIRE(Kw > 0 && Kh > 0 && Kd > 0, SPCONV_ERR_ARG, "kernel size must be positive");
    SPCONV_REQUIRE(Dw > 0 && Dh > 0 && Dd > 0, SPCONV_ERR_ARG, "dilation must be positive");
    const int V = Kw * Kh * Kd;
    SPCONV_REQUIRE(V <= kMaxKernelVolume, SPCONV_ERR_ARG, "kernel volume %d exceeds %d", V, kMaxKernelVolume);
    {
        const long double vol = (long double)batch * W * H * D;
        SPCONV_REQUIRE(vol < 18446744073709551615.0L, SPCONV_ERR_ARG,
                       "volume N*W*H*D does not fit in 64 bits");
    }
    if (M == 0) return SPCONV_OK;
    SPCONV_REQUIRE(coords && neighbor_map && masks && order && workspace, SPCONV_ERR_ARG,
                   "null pointer argument");
    SPCONV_REQUIRE(((uintptr_t)coords & 15u) == 0, SPCONV_ERR_ARG, "coords must be 16-byte aligned");
    SPCONV_REQUIRE(((uintptr_t)workspace & 255u) == 0, SPCONV_ERR_ARG, "workspace must be 256-byte aligned");
    const bool key64 = !volume_fits_32(batch, W, H, D);
    const WsLayout L = ws_layout(M, key64);
    SPCONV_REQUIRE(workspace_bytes >= L.total, SPCONV_ERR_ARG,
                   "workspace too small: %lld < %lld bytes", (long long)workspace_bytes, (long long)L.total);
    cudaStream_t stream = (cudaStream_t)stream_ptr;
    char *ws = (char *)workspace;
    unsigned long long *table = (unsigned long long *)(ws + L.table);
    uint32_t *vals = key64 ? (uint32_t *)(ws + L.vals) : nullptr;
    uint32_t *hist = (uint32_t *)(ws + L.hist);
    uint32_t *cursor = (uint32_t *)(ws + L.cursor);
    uint32_t *counter = (uint32_t *)(ws + L.counter);
    const uint64_t tmask = (uint64_t)L.cap - 1;
    const int MW = spconv_mask_words(V);

    stage_mark(SPCONV_STAGE_MEMSET, 0, stream);
    if (cudaMemsetAsync(workspace, 0, (size_t)L.total, stream) != cudaSuccess)
        return check_launch("workspace memset");
    stage_mark(SPCONV_STAGE_MEMSET, 1, stream);
    const int64_t gi = (M + 255) / 256;
    const int ins_grid = (int)(gi < 65535LL * 32 ? gi : 65535LL * 32);
    stage_mark(SPCONV_STAGE_INSERT, 0, stream);
    if (key64)
        insert_kernel<true><<<ins_grid, 256, 0, stream>>>((const int4 *)coords, M, batch, W, H, D, table, vals, tmask, status);
    else
        insert_kernel<false><<<ins_grid, 256, 0, stream>>>((const int4 *)coords, M, batch, W, H, D, table, vals, tmask, status);
    if (int rc = check_launch("insert_kernel")) return rc;
    stage_mark(SPCONV_STAGE_INSERT, 1, stream);

    const int map_grid = (int)((M + kMapVoxels - 1) / kMapVoxels);
    const size_t map_smem = (size_t)V * sizeof(int4);
    stage_mark(SPCONV_STAGE_MAP, 0, stream);
    if (key64)
        map_kernel<true><<<map_grid, kMapThreads, map_smem, stream>>>(
            (const int4 *)coords, M, W, H, D, Kw, Kh, Kd, Dw, Dh, Dd, V, MW, table, vals, tmask,
            neighbor_map, masks, hist, cursor, counter, status);
    else
        map_kernel<false><<<map_grid, kMapThreads, map_smem, stream>>>(
            (const int4 *)coords, M, W, H, D, Kw, Kh, Kd, Dw, Dh, Dd, V, MW, table, vals, tmask,
            neighbor_map, masks, hist, cursor, counter, status);
    if (int rc = check_launch("map_kernel")) return rc;
    stage_mark(SPCONV_STAGE_MAP, 1, stream);

    const int per_block = kOrderThreads * kOrderPerThread;
    const int ord_grid = (int)((M + per_block - 1) / per_block);
    stage_mark(SPCONV_STAGE_ORDER, 0, stream);
    order_kernel<<<ord_grid, kOrderThreads, 0, stream>>>(masks, M, MW, cursor, order, status);
    if (int rc = check_launch("order_kernel")) return rc;
    stage_mark(SPCONV_STAGE_ORDER, 1, stream);
    return SPCONV_OK;
}

// ---------------------------------------------------------------------------------------
// Allocation-free variant: the workspace is a fixed file-scope device array.
//
// Callers that cannot allocate device memory at the point of the call (operator plugin
// hosts that pass only input/output buffers, fixed-memory real-time loops, runtimes whose
// allocator must not run there) get the same map from here without a workspace argument.
// The array is sized for SPCONV_NOALLOC_MAX_COORDS voxels with 64-bit keys (the larger
// layout), about 12 MiB; every GPU that loads the library holds it until the process exits.
// In host code `g_noalloc_scratch` names a host-side stand-in, not device memory: its device
// address is looked up per device with cudaGetSymbolAddress and only that address is passed on.
// ---------------------------------------------------------------------------------------
namespace spconv {

constexpr int64_t noalloc_capacity() {
    int64_t cap = 1024;
    while (cap < 2 * (int64_t)SPCONV_NOALLOC_MAX_COORDS) cap <<= 1;
    return cap;
}
constexpr int64_t align256c(int64_t x) { return (x + 255) & ~int64_t(255); }
constexpr int64_t kNoAllocScratchBytes =
    align256c(noalloc_capacity() * 8) + align256c(noalloc_capacity() * 4) +
    2 * align256c(kOrderBuckets * 4) + 256;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
static std::mutex g_noalloc_mu;
static void *g_noalloc_dev_ptr[kNoAllocMaxDevices] = {};

// Device address of the scratch array on the current device; looked up once per device.
static int noalloc_scratch(void **out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return check_launch("cudaGetDevice");
    SPCONV_REQUIRE(dev >= 0 && dev < kNoAllocMaxDevices, SPCONV_ERR_ARG,
                   "device ordinal %d exceeds the %d devices the scratch table tracks", dev, kNoAllocMaxDevices);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (g_noalloc_dev_ptr[dev] == nullptr) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            set_error("cudaGetSymbolAddress of the no-alloc scratch failed on device %d: %s",
                      dev, cudaGetErrorString(e));
            return SPCONV_ERR_CUDA;
        }
        g_noalloc_dev_ptr[dev] = p;
    }
    *out = g_noalloc_dev_ptr[dev];
    return SPCONV_OK;
}

}  // namespace spconv

extern "C" int spconv_build_submanifold_neighbor_map_noalloc(
    const int32_t *coords, int64_t M,
    int batch, int W, int H, int D,
    int Kw, int Kh, int Kd, int Dw, int Dh, int Dd,
    int32_t *neighbor_map, uint32_t *masks, int32_t *order,
    int32_t *status, void *stream) {
    SPCONV_REQUIRE(M <= (int64_t)SPCONV_NOALLOC_MAX_COORDS, SPCONV_ERR_ARG,
                   "num_coords %lld exceeds the no-alloc limit of %d coordinates "
                   "(use spconv_build_submanifold_neighbor_map with a workspace)",
                   (long long)M, (int)SPCONV_NOALLOC_MAX_COORDS);
    void *scratch = nullptr;
    if (M > 0) {
        if (int rc = noalloc_scratch(&scratch)) return rc;
    }
    return spconv_build_submanifold_neighbor_map(
        coords, M, batch, W, H, D, Kw, Kh, Kd, Dw, Dh, Dd, scratch, kNoAllocScratchBytes,
        neighbor_map, masks, order, status, stream);
}
