// Coordinate hash table + submanifold kernel-map builder for sm_100a.
//
// Replaces the reference's three-step build (neighbor_map.cu:179-237): the 3-D insert
// kernel (hash.cu:367-409, one atomicCAS per voxel into a table sized int(2M)), a
// torch::full pre-fill of the [M,V] map, and one lookup thread per (voxel, offset)
// (neighbor_map.cu:132-177) that writes only the found entries.
//
// Here:
//   1. one cudaMemsetAsync clears the workspace (table, bitmap, histogram, cursors); for
//      3x3x3 kernels the prep kernel of the sorted-input path (section 2c') runs first and the
//      table and bitmap are cleared by a kernel only when the input takes the hash path;
//   2. insert_kernel: one thread per voxel, a coalesced int4 load, a CAS into the first free
//      slot of its 32-byte group of a power-of-two table of packed 64-bit slots
//      ((key << 32) | row, stored complemented so that all-zero means empty), and the
//      voxel's bit in an occupancy bitmap of the grid (grids of <= 2^30 cells);
//   3. a map kernel (map_kernel_k3 for 3x3x3, map_kernel_cols / map_kernel_bm for other
//      shapes with a bitmap, map_kernel otherwise): one thread per voxel screens its
//      offsets against the bitmap, probes the table only for occupied cells, stages the
//      voxel's map row in shared memory (written out coalesced) and builds its offset mask;
//      each block adds its voxels' order keys (popcount class, mask hash) to a histogram, or,
//      when the radix order follows, the low digits of their radix keys to the sort's counts;
//   4. order: order_kernel scans the histogram in every block and scatters voxel ids by key
//      (block-aggregated cursor atomics) - or, for maps of >= 2^19 voxels of kernels of
//      <= 27 offsets, a stable radix sort by (class, mask) (sort_*_kernel).
// The map is a pure function of the coordinates: for duplicate-free inputs any correct
// table gives the reference's map bit for bit. The bucket order (`order`) depends on
// atomics and is unspecified within a bucket; the radix order is deterministic; the conv
// results depend on neither.
#include <cstdio>
#include <cstdarg>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace spconv {

constexpr int kOrderBuckets = 4096;    // 16 popcount classes x 256 mask-hash buckets
constexpr int kMapThreads = 128;      // one thread per voxel
constexpr int kOrderThreads = 256;      // kOrderBuckets / kOrderThreads must be a multiple of 4
constexpr int kOrderPerThread = 2;     // voxels per thread in order_kernel
// Radix-sort order (kernels of at most kSortMaxV offsets; see radix_order for the sizes):
// tiles of kSortTile voxels, 8-bit digits, keys of at most 31 bits.
constexpr int kSortThreads = 512;
constexpr int kSortWarpItems = 128;                                  // 4 rounds of 32 per warp
constexpr int kSortTile = (kSortThreads / 32) * kSortWarpItems;      // 2048 (4096 left SMs idle)
constexpr int kSortMaxPasses = 4;
constexpr int kSortMaxV = 27;
constexpr int64_t kSortMinVoxels = 1 << 19;
// Sparse grids (surfaces) gain from the radix order at smaller sizes too: measured per-rank
// sizes of the benchmark's batch split, map build + conv, B200: indoor 2 samples (500k voxels,
// 0.19 % of the grid) 469 -> 386 us, 1 sample (250k) 272 -> 256 us; dense random occupancy
// loses (cube 168k at 2 %: 80 -> 104 us; wide3 4 samples, 335k at 0.5 %: 147 -> 175 us), and so
// do clustered LiDAR points at 0.11 % (2 samples, 207k: 156 -> 176 us), the cost of this rule.
constexpr int64_t kSortSparseMinVoxels = 1 << 17;     // exclusive
constexpr long double kSortSparseDensity = 0.003L;
constexpr int kMaxKernelVolume = 1024;

static int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

// Sorted-input path (section 2c'): at most this many (b, x, y) columns (64 MB of ranges).
constexpr int64_t kSortedMaxCols = 1ll << 23;
// Columns of the grid when the sorted-input path can serve it (32-bit keys), else 0.
static int64_t sorted_cols(int batch, int W, int H, int D) {
    const long double vol = (long double)batch * W * H * D;
    const long double cols = (long double)batch * W * H;
    if (vol >= 4294967296.0L || cols > (long double)kSortedMaxCols) return 0;
    return (int64_t)cols;
}

// Table capacity for M voxels: the next power of two >= 4M (load <= 0.25) while the table
// stays within 64 MB (L2-resident next to the streams it serves), else >= 2M (load <= 0.5).
// Slots are probed in aligned groups of kGroup = 4 (one 32-byte sector per probe).
constexpr int kGroup = 4;
constexpr int64_t kLowLoadTableBytes = 64ll << 20;
constexpr int64_t capacity_for(int64_t M) {
    int64_t cap = 1024;
    while (cap < 4 * M) cap <<= 1;
    if (cap * 8 > kLowLoadTableBytes) {
        cap = 1024;
        while (cap < 2 * M) cap <<= 1;
    }
    return cap;
}

struct WsLayout {
    int64_t cap = 0;
    bool key64 = false;
    int64_t bitmap_words = 0;
    int64_t table = 0, vals = 0, bitmap = 0, hist = 0, cursor = 0, flags = 0, total = 0;
    int sort_tiles = 0;            // > 0: room for the radix-sort order (keys alias the table)
    int64_t sort_counts = 0;       // [kSortMaxPasses][256][sort_tiles] + [kSortMaxPasses][256] totals
    int64_t cols = 0;              // > 0: room for the sorted-input path (column ranges + keys)
    int64_t colrange = 0, keys = 0;
};

// Grids of at most 2^30 cells (a 128 MB bitmap, cleared with the table) get an occupancy
// bitmap, one bit per cell, that screens neighbour probes: a clear bit settles a probe with
// one cached 4-byte load. Clearing 128 MB costs ~40 us; without the bitmap every absent
// neighbour of a surface scene (about half of 26) probes the table.
constexpr long double kBitmapMaxCells = 1073741824.0L;
static int64_t bitmap_words_for(int batch, int W, int H, int D) {
    const long double vol = (long double)batch * W * H * D;
    if (vol > kBitmapMaxCells) return 0;
    return (int64_t)((vol + 31.0L) / 32.0L);
}

// Lets a map kernel use up to 160 KB of dynamic shared memory. The attribute belongs to the
// device's context, so it is set once per device and kernel (`slot` names the kernel).
static void raise_smem_limit(const void *fn, int slot) {
    constexpr int kDevs = 64, kSlots = 5;
    static std::mutex mu;
    static bool done[kDevs][kSlots] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kDevs || slot < 0 || slot >= kSlots) {
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
        return;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (!done[dev][slot]) {
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
        done[dev][slot] = true;
    }
}

static bool volume_fits_32(int batch, int W, int H, int D) {
    const long double vol = (long double)batch * W * H * D;
    return vol < 4294967296.0L;
}

// Whether a map of M voxels on an N x W x H x D grid is ordered by the radix sort (when its
// kernel has at most kSortMaxV offsets): from 2^19 voxels, or above 2^17 voxels on grids they
// fill to at most 0.3 %. (Measured: see kSortSparseMinVoxels.)
static bool radix_order(int64_t M, int batch, int W, int H, int D) {
    if (M >= kSortMinVoxels) return true;
    const long double vol = (long double)batch * W * H * D;
    return M > kSortSparseMinVoxels && (long double)M <= kSortSparseDensity * vol;
}

// `cols` > 0 adds the sorted-input path's regions: [cols] int2 column ranges (cleared with the
// histogram and flags) and [M] uint32 flat keys.
static WsLayout ws_layout(int64_t M, bool key64, int64_t bitmap_words, bool sort, int64_t cols = 0) {
    WsLayout L;
    L.cap = capacity_for(M);
    L.key64 = key64;
    L.bitmap_words = key64 ? 0 : bitmap_words;
    int64_t off = 0;
    L.table = off; off += align256(L.cap * 8);
    if (key64) { L.vals = off; off += align256(L.cap * 4); }
    if (L.bitmap_words) { L.bitmap = off; off += align256(L.bitmap_words * 4); }
    L.hist = off; off += align256(kOrderBuckets * 4);
    L.cursor = off; off += align256(kOrderBuckets * 4);
    L.flags = off; off += 256;          // per-call flags, cleared with the rest (word 0: duplicate seen)
    if (sort) {
        // Sort keys and values (4 x M words) reuse the table, dead once the map is built:
        // its capacity is at least 2M slots of 8 bytes.
        L.sort_tiles = (int)((M + kSortTile - 1) / kSortTile);
        L.sort_counts = off;
        off += align256((int64_t)kSortMaxPasses * 256 * (L.sort_tiles + 1) * 4);
    }
    if (cols > 0 && !key64) {
        L.cols = cols;
        L.colrange = off; off += align256(cols * 8);
        L.keys = off; off += align256(M * 4);
    }
    L.total = off;
    return L;
}

// Adds a block's shared-memory order histogram to the global one (after a __syncthreads).
// The order kernel turns the global histogram into bucket offsets; nothing here waits on
// other blocks.
__device__ __forceinline__ void block_hist_flush(const uint32_t *s_hist, uint32_t *hist) {
    for (int b = threadIdx.x; b < kOrderBuckets; b += blockDim.x)
        if (s_hist[b]) atomicAdd(hist + b, s_hist[b]);
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

constexpr int kSortCompBits = 20;

__device__ __host__ __forceinline__ int order_key_drop(int V) {
    return V - 1 > kSortCompBits ? V - 1 - kSortCompBits : 0;
}

__device__ __forceinline__ uint32_t order_key(uint32_t m, int V) {
    const int c = V / 2, drop = order_key_drop(V);
    m &= (1u << V) - 1u;                                        // V <= 27
    const uint32_t comp = (m & ((1u << c) - 1u)) | ((m >> (c + 1)) << c);
    const uint32_t pc = (uint32_t)__popc(m);
    const uint32_t cls = pc == 0 ? 0u : min(pc - 1u, 15u);
    return (cls << (V - 1 - drop)) | (comp >> drop);
}

// Order histogram entry of a voxel with offset mask word `m0` (the first), popcount `pc` and
// mask hash `h`. With sort_nt > 0 (the radix order) the map kernels make the sort's first
// counts: the low 8-bit digit of the voxel's radix key, counted per 2048-voxel sort tile (every
// map block lies inside one tile); otherwise the bucket order's (class, hash) bucket.
__device__ __forceinline__ uint32_t order_bucket(uint32_t m0, uint32_t pc, uint32_t h, int V, int sort_nt) {
    if (sort_nt > 0) return order_key(m0, V) & 255u;
    const uint32_t cls = pc == 0 ? 0u : min(pc - 1u, 15u);
    return cls * 256u + (h & 255u);
}

// Adds a block's shared-memory histogram (after a __syncthreads) to the global one: the bucket
// histogram, or (sort_nt > 0) column tile = i0 / kSortTile of the radix sort's pass-0 digit
// counts [256][sort_nt], which the workspace clear zeroes.
__device__ __forceinline__ void order_hist_flush(const uint32_t *s_hist, uint32_t *hist, int sort_nt, int64_t i0) {
    if (sort_nt > 0) {
        const int64_t tile = i0 / kSortTile;
        for (int d = threadIdx.x; d < 256; d += blockDim.x)
            if (s_hist[d]) atomicAdd(hist + (int64_t)d * sort_nt + tile, s_hist[d]);
    } else {
        block_hist_flush(s_hist, hist);
    }
}

// ---------------------------------------------------------------------------------------
// Table: packed 64-bit slots for volumes < 2^32 (key = flat index), or 64-bit keys plus a
// separate row array otherwise; stored complemented, so 0 = empty. A key hashes to a group
// of kGroup consecutive slots (32 bytes); inserts take the first empty slot of the first
// group with room (linear probing over groups), so a lookup that finds an empty slot in a
// group without a match can stop: one 32-byte probe settles almost every lookup.
// ---------------------------------------------------------------------------------------
// Home group of a 32-bit key: Fibonacci hashing, the top log2(groups) bits of
// key * 2654435761 (shift = 32 - log2(groups)); consecutive grid keys land far apart.
__device__ __forceinline__ uint32_t home32(uint32_t key, uint32_t shift) {
    return (key * 0x9E3779B1u) >> shift;
}

template <bool KEY64>
__device__ __forceinline__ uint64_t home_group(uint64_t flat, uint64_t gmask, uint32_t shift) {
    return KEY64 ? (fmix64(flat) & gmask) : (uint64_t)home32((uint32_t)flat, shift);
}

template <bool KEY64>
__device__ __forceinline__ bool table_insert(unsigned long long *table, uint32_t *vals,
                                             uint64_t gmask, uint32_t shift, uint64_t flat,
                                             uint32_t row, int32_t *status, int32_t *dup_flag) {
    const unsigned long long desired =
        KEY64 ? ~(unsigned long long)flat : ~((((unsigned long long)(uint32_t)flat) << 32) | row);
    uint64_t g = home_group<KEY64>(flat, gmask, shift);
    for (uint64_t pg = 0; pg <= gmask; ++pg) {
        unsigned long long *grp = table + g * kGroup;
#pragma unroll
        for (int i = 0; i < kGroup; ++i) {
            // CAS straight away: at the table's low load it usually succeeds, and on an
            // occupied slot it returns the occupant for the duplicate test.
            const unsigned long long cur = atomicCAS(grp + i, 0ull, desired);
            if (cur == 0ull) {
                if (KEY64) atomicMax(vals + g * kGroup + i, row);
                return true;
            }
            const bool same = KEY64 ? (cur == desired) : ((uint32_t)(cur >> 32) == (uint32_t)(desired >> 32));
            if (same) {
                // Duplicate coordinate: keep the highest row.
                if (KEY64) atomicMax(vals + g * kGroup + i, row);
                else atomicMin(grp + i, desired);        // min of the complement = max row
                raise_status(status, SPCONV_STATUS_DUPLICATE);
                *dup_flag = 1;                           // this call's own record of it
                return true;
            }
        }
        g = (g + 1) & gmask;
    }
    return false;
}

__device__ __forceinline__ void load_group(const unsigned long long *__restrict__ table, uint64_t g,
                                           unsigned long long (&w)[kGroup]) {
    const ulonglong2 *p = reinterpret_cast<const ulonglong2 *>(table + g * kGroup);
    const ulonglong2 a = __ldg(p), b = __ldg(p + 1);
    w[0] = a.x; w[1] = a.y; w[2] = b.x; w[3] = b.y;
}

// Row of `flat` given its home group's loaded words; continues to later groups while they
// are full. Returns the row, -1 if absent, -2 if every group was full (table overflow).
template <bool KEY64>
__device__ __forceinline__ int32_t table_resolve(const unsigned long long *__restrict__ table,
                                                 const uint32_t *__restrict__ vals, uint64_t gmask,
                                                 uint64_t flat, uint64_t g, unsigned long long (&w)[kGroup]) {
    const uint32_t nk = ~(uint32_t)flat;
    const unsigned long long nk64 = ~(unsigned long long)flat;
    for (uint64_t pg = 0; pg <= gmask; ++pg) {
        bool empty = false;
#pragma unroll
        for (int i = 0; i < kGroup; ++i) {
            if (KEY64) {
                if (w[i] == nk64) return (int32_t)__ldg(vals + g * kGroup + i);
            } else {
                if ((uint32_t)(w[i] >> 32) == nk && w[i] != 0ull) return (int32_t)(~(uint32_t)w[i]);
            }
            empty |= (w[i] == 0ull);
        }
        if (empty) return -1;
        g = (g + 1) & gmask;
        load_group(table, g, w);
    }
    return -2;
}

// ---------------------------------------------------------------------------------------
// 1. Insert (replaces hash.cu:367-389 + hash.cuh:22-63).
// ---------------------------------------------------------------------------------------
template <bool KEY64>
__global__ void __launch_bounds__(256)
insert_kernel(const int4 *__restrict__ coords, int64_t M, int N, int W, int H, int D,
              unsigned long long *table, uint32_t *vals, uint32_t *bitmap, uint64_t gmask,
              uint32_t shift, int32_t *status, int32_t *dup_flag, const int32_t *unsorted) {
    grid_launch_dependents();                                   // the map kernel's setup overlaps this
    grid_dependency_wait();                                     // the cleared table (launched with PDL)
    if (unsorted && *unsorted == 0) return;                     // sorted input: the column path builds the map
    const int lane = threadIdx.x & 31;
    // Whole warps iterate together (the bitmap update below shuffles across the warp).
    for (int64_t w0 = (int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31); w0 < M;
         w0 += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = w0 + lane;
        bool ok = i < M;
        int4 c = make_int4(0, 0, 0, 0);
        if (ok) c = __ldg(coords + i);
        if (ok && (c.x < 0 || c.x >= N || c.y < 0 || c.y >= W || c.z < 0 || c.z >= H || c.w < 0 || c.w >= D)) {
            raise_status(status, SPCONV_STATUS_COORD_RANGE);
            ok = false;
        }
        const uint64_t flat = ((((uint64_t)c.x * W + c.y) * H + c.z) * D) + c.w;
        if (bitmap) {
            // Voxels next to each other in z, adjacent in sorted input, share a bitmap word:
            // each run of lanes with the same word ORs its bits together (segmented doubling
            // over consecutive lanes) and the run's first lane sets them with one atomic.
            // Words are < 2^25 (the bitmap covers at most 2^30 cells), so ~0 marks no voxel.
            const uint32_t wi = ok ? (uint32_t)(flat >> 5) : 0xffffffffu;
            uint32_t bits = ok ? 1u << (flat & 31) : 0u;
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const uint32_t ob = __shfl_down_sync(0xffffffffu, bits, d);
                const uint32_t ow = __shfl_down_sync(0xffffffffu, wi, d);
                if (ow == wi) bits |= ob;
            }
            const uint32_t pw = __shfl_up_sync(0xffffffffu, wi, 1);
            if (ok && (lane == 0 || pw != wi)) atomicOr(bitmap + wi, bits);
        }
        if (ok && !table_insert<KEY64>(table, vals, gmask, shift, flat, (uint32_t)i, status, dup_flag))
            raise_status(status, SPCONV_STATUS_TABLE_FULL);
    }
}

// ---------------------------------------------------------------------------------------
// 2. Fused map + masks + order histogram (replaces torch::full + neighbor_map.cu:132-177).
//    One thread per voxel walks the voxel's V offsets in chunks of kMapChunk, with the
//    chunk's table probes (one 32-byte group each) in flight together; the in-bounds test
//    and key of each offset are one add against per-offset constants in shared memory. The
//    thread builds the voxel's mask words in registers and stages its map row in shared
//    memory, and the block then writes its voxels' rows as one contiguous, coalesced range.
//    Blocks histogram their voxels by order key (popcount class, mask hash); the last
//    block to finish turns the histogram into bucket offsets.
// ---------------------------------------------------------------------------------------
constexpr int kMapChunk = 8;
constexpr int kMapStageMaxBytes = 96 * 1024;

template <bool KEY64, bool BITMAP>
__global__ void __launch_bounds__(kMapThreads)
map_kernel(const int4 *__restrict__ coords, int64_t M, int W, int H, int D,
           int Kw, int Kh, int Kd, int Dw, int Dh, int Dd, int V, int MW, int vstride,
           const unsigned long long *__restrict__ table, const uint32_t *__restrict__ vals,
           const uint32_t *__restrict__ bitmap, uint64_t gmask, uint32_t shift, int32_t *__restrict__ nbr, uint32_t *__restrict__ masks,
           uint32_t *hist, int sort_nt, int32_t *status) {
    __shared__ uint32_t s_hist[kOrderBuckets];
    extern __shared__ int4 s_off[];                                   // [V] (ox, oy, oz, 0)
    long long *s_delta = reinterpret_cast<long long *>(s_off + V);   // [V] flat-key deltas
    int32_t *s_stage = reinterpret_cast<int32_t *>(s_delta + V);     // [kMapThreads][vstride]

    const int tid = threadIdx.x;
    const int64_t i0 = (int64_t)blockIdx.x * kMapThreads;
    const int nvox = (M - i0) < (int64_t)kMapThreads ? (int)(M - i0) : kMapThreads;
    const bool staged = vstride > 0;
    grid_dependency_wait();                                     // the insert's table and bitmap
    grid_launch_dependents();

    for (int v = tid; v < V; v += kMapThreads) {
        const int KhKd = Kh * Kd;
        const int ox = (v / KhKd) * Dw - (Kw / 2) * Dw;
        const int oy = ((v / Kd) % Kh) * Dh - (Kh / 2) * Dh;
        const int oz = (v % Kd) * Dd - (Kd / 2) * Dd;
        s_off[v] = make_int4(ox, oy, oz, 0);
        // For in-bounds neighbours key(n) = key(c) + delta exactly.
        s_delta[v] = ((long long)ox * H + oy) * D + oz;
    }
    for (int j = tid; j < kOrderBuckets; j += kMapThreads) s_hist[j] = 0u;
    __syncthreads();

    const bool valid = tid < nvox;
    const int64_t i = i0 + tid;
    int4 c = make_int4(0, 0, 0, 0);
    if (valid) c = __ldg(coords + i);
    const unsigned long long base = ((((unsigned long long)(long long)c.x * W + c.y) * H + c.z) * D) + c.w;
    const int center = V / 2;
    bool wrapped = false;
    uint32_t pc = 0, h = 0x9e3779b9u, m0 = 0u;
    for (int vb = 0; vb < V; vb += 32) {
        const int vend = min(vb + 32, V);
        uint32_t bits = 0;
        for (int v0 = vb; v0 < vend; v0 += kMapChunk) {
            int32_t val[kMapChunk];
            bool need[kMapChunk];
            uint64_t flat[kMapChunk], grp[kMapChunk];
            unsigned long long word[kMapChunk][kGroup];
            uint32_t occ[kMapChunk];
#pragma unroll
            for (int k = 0; k < kMapChunk; ++k) {
                const int v = v0 + k;
                val[k] = -1;
                need[k] = false;
                if (valid && v < vend) {
                    if (v == center) {
                        val[k] = (int32_t)i;
                    } else {
                        const int4 o = s_off[v];
                        if ((unsigned)(c.y + o.x) < (unsigned)W && (unsigned)(c.z + o.y) < (unsigned)H &&
                            (unsigned)(c.w + o.z) < (unsigned)D) {
                            flat[k] = base + (unsigned long long)s_delta[v];
                            need[k] = true;
                            if (BITMAP) occ[k] = __ldg(bitmap + (flat[k] >> 5));   // screens in flight together
                        }
                    }
                }
            }
#pragma unroll
            for (int k = 0; k < kMapChunk; ++k) {
                if (BITMAP && need[k]) need[k] = (occ[k] >> (flat[k] & 31)) & 1u;
                if (need[k]) {
                    grp[k] = home_group<KEY64>(flat[k], gmask, shift);
                    load_group(table, grp[k], word[k]);              // chunk probes in flight together
                }
            }
#pragma unroll
            for (int k = 0; k < kMapChunk; ++k) {
                const int v = v0 + k;
                if (need[k]) {
                    val[k] = table_resolve<KEY64>(table, vals, gmask, flat[k], grp[k], word[k]);
                    if (val[k] == -2) { wrapped = true; val[k] = -1; }
                }
                if (valid && v < vend) {
                    if (staged) s_stage[tid * vstride + v] = val[k];
                    else nbr[i * (int64_t)V + v] = val[k];
                    if (val[k] >= 0) bits |= 1u << (v - vb);
                }
            }
        }
        if (valid) masks[i * (int64_t)MW + (vb >> 5)] = bits;
        if (vb == 0) m0 = bits;
        pc += __popc(bits);
        h = fmix32(h ^ bits);
    }
    if (wrapped) raise_status(status, SPCONV_STATUS_TABLE_FULL);
    {
        const uint32_t key = order_bucket(m0, pc, h, V, sort_nt);
        const uint32_t active = __ballot_sync(0xffffffffu, valid);
        if (valid && hist) aggregated_inc(s_hist, key, active);
    }
    __syncthreads();

    // The block's rows form one contiguous range of the map.
    if (staged) {
        int32_t *out = nbr + i0 * (int64_t)V;
        const int total = nvox * V;
        int il = tid / V, v = tid - il * V;
        const int step_i = kMapThreads / V, step_v = kMapThreads - step_i * V;
        for (int e = tid; e < total; e += kMapThreads) {
            out[e] = s_stage[il * vstride + v];
            v += step_v; il += step_i;
            if (v >= V) { v -= V; ++il; }
        }
    }
    if (hist) order_hist_flush(s_hist, hist, sort_nt, i0);
}

// ---------------------------------------------------------------------------------------
// 2b. Map build for grids with an occupancy bitmap (32-bit keys). One thread per voxel
//     walks the kernel column by column: a (dx, dy) column's z-offsets span at most 32
//     cells, so one funnel-shifted pair of bitmap words screens all of them; only cells
//     whose bit is set are probed in the hash table (the column's probes in flight
//     together). Mask words are built in a register and flushed as v crosses a multiple
//     of 32; map rows are staged in shared memory and written out coalesced.
// ---------------------------------------------------------------------------------------
constexpr int kMapBmMaxThreads = 256;
constexpr int kColBatchMax = 8;          // Kd <= 8 (longer columns use map_kernel)

template <int kColBatch>
__global__ void __launch_bounds__(kMapBmMaxThreads, 3)
map_kernel_bm(const int4 *__restrict__ coords, int64_t M, int W, int H, int D,
              int Kw, int Kh, int Kd, int Dw, int Dh, int Dd, int V, int MW, int vstride,
              const unsigned long long *__restrict__ table, const uint32_t *__restrict__ bitmap,
              int64_t bm_words, uint64_t gmask, uint32_t shift, int32_t *__restrict__ nbr,
              uint32_t *__restrict__ masks, uint32_t *hist, int sort_nt,
              int32_t *status) {
    __shared__ uint32_t s_hist[kOrderBuckets];
    extern __shared__ int32_t s_stage[];                       // [blockDim.x][vstride]

    const int tid = threadIdx.x, nthr = blockDim.x;
    const int64_t i0 = (int64_t)blockIdx.x * nthr;
    const int nvox = (M - i0) < (int64_t)nthr ? (int)(M - i0) : nthr;
    const bool staged = vstride > 0;
    grid_dependency_wait();                                     // the insert's table and bitmap
    grid_launch_dependents();
    for (int j = tid; j < kOrderBuckets; j += nthr) s_hist[j] = 0u;
    __syncthreads();

    const bool valid = tid < nvox;
    const int64_t i = i0 + tid;
    int4 c = make_int4(0, 0, 0, 0);
    if (valid) c = __ldg(coords + i);
    const int64_t HD = (int64_t)H * D;
    const int64_t key_c = (((int64_t)c.x * W + c.y) * H + c.z) * D + c.w;
    const int rw = Kw / 2, rh = Kh / 2, rd = Kd / 2;
    const int span = (Kd - 1) * Dd + 1;
    const int center = V / 2;
    bool wrapped = false;
    uint32_t pc = 0, h = 0x9e3779b9u, cur_bits = 0;
    int cur_w = 0, v = 0;
    for (int cx = 0; cx < Kw; ++cx) {
        const int ox = (cx - rw) * Dw;
        const bool xin = (unsigned)(c.y + ox) < (unsigned)W;
        for (int cy = 0; cy < Kh; ++cy) {
            const int oy = (cy - rh) * Dh;
            const bool yin = valid && xin && (unsigned)(c.z + oy) < (unsigned)H;
            const int64_t col = key_c + ox * HD + (int64_t)oy * D;     // key of (x+ox, y+oy, z)
            const int zlo = max(c.w - rd * Dd, 0);
            const int64_t kbase = col + (zlo - c.w);
            uint32_t win = 0;
            if (yin && span <= 32) {
                const int64_t wi = kbase >> 5;
                const uint32_t lo = __ldg(bitmap + wi);
                const uint32_t hi = __ldg(bitmap + (wi + 1 < bm_words ? wi + 1 : wi));
                win = __funnelshift_r(lo, hi, (uint32_t)(kbase & 31));  // bits kbase .. kbase+31
            }
            int32_t val[kColBatch];
            uint32_t key[kColBatch];
            uint64_t grp[kColBatch];
            bool need[kColBatch];
            unsigned long long word[kColBatch][kGroup];
#pragma unroll
            for (int cz = 0; cz < kColBatch; ++cz) {
                val[cz] = -1;
                need[cz] = false;
                if (cz < Kd) {
                    const int oz = (cz - rd) * Dd;
                    if (v + cz == center) {
                        val[cz] = (int32_t)i;
                    } else if (yin && (unsigned)(c.w + oz) < (unsigned)D) {
                        const int64_t kn = col + oz;
                        const bool present = span <= 32 ? ((win >> (uint32_t)(kn - kbase)) & 1u)
                                                        : ((__ldg(bitmap + (kn >> 5)) >> (kn & 31)) & 1u);
                        if (present) {
                            key[cz] = (uint32_t)kn;
                            grp[cz] = home32(key[cz], shift);
                            load_group(table, grp[cz], word[cz]);    // the column's probes in flight together
                            need[cz] = true;
                        }
                    }
                }
            }
#pragma unroll
            for (int cz = 0; cz < kColBatch; ++cz) {
                if (cz < Kd) {
                    if (need[cz]) {
                        val[cz] = table_resolve<false>(table, nullptr, gmask, key[cz], grp[cz], word[cz]);
                        if (val[cz] == -2) { wrapped = true; val[cz] = -1; }
                    }
                    if ((v >> 5) != cur_w) {                         // mask word complete
                        if (valid) masks[i * (int64_t)MW + cur_w] = cur_bits;
                        pc += __popc(cur_bits);
                        h = fmix32(h ^ cur_bits);
                        cur_w = v >> 5;
                        cur_bits = 0;
                    }
                    if (valid) {
                        if (staged) s_stage[tid * vstride + v] = val[cz];
                        else nbr[i * (int64_t)V + v] = val[cz];
                    }
                    if (val[cz] >= 0) cur_bits |= 1u << (v & 31);
                    ++v;
                }
            }
        }
    }
    if (valid) masks[i * (int64_t)MW + cur_w] = cur_bits;
    pc += __popc(cur_bits);
    h = fmix32(h ^ cur_bits);
    if (wrapped) raise_status(status, SPCONV_STATUS_TABLE_FULL);
    {
        // (the radix order needs V <= 27: cur_bits is then the only mask word)
        const uint32_t k = order_bucket(cur_bits, pc, h, V, sort_nt);
        const uint32_t active = __ballot_sync(0xffffffffu, valid);
        if (valid && hist) aggregated_inc(s_hist, k, active);
    }
    __syncthreads();

    // The block's rows form one contiguous range of the map.
    if (staged) {
        int32_t *out = nbr + i0 * (int64_t)V;
        const int total = nvox * V;
        if (vstride == V && ((uintptr_t)out & 15u) == 0) {
            const int n4 = total >> 2;
            const int4 *src = reinterpret_cast<const int4 *>(s_stage);
            int4 *dst = reinterpret_cast<int4 *>(out);
            for (int e = tid; e < n4; e += nthr) dst[e] = src[e];
            for (int e = (n4 << 2) + tid; e < total; e += nthr) out[e] = s_stage[e];
        } else {
            int il = tid / V, vv = tid - il * V;
            const int step_i = nthr / V, step_v = nthr - step_i * V;
            for (int e = tid; e < total; e += nthr) {
                out[e] = s_stage[il * vstride + vv];
                vv += step_v; il += step_i;
                if (vv >= V) { vv -= V; ++il; }
            }
        }
    }
    if (hist) order_hist_flush(s_hist, hist, sort_nt, i0);
}

// ---------------------------------------------------------------------------------------
// 2c. Map build for 3x3x3 kernels (any dilation). Phase 1 forms a 27-bit candidate mask
//     per voxel: six per-voxel in-bounds flags and, with a bitmap, one funnel-shifted window
//     per (dx, dy) column (all 18 window loads issued up front). Phase 2 probes the hash
//     table only for candidate offsets, four in flight at a time. The block's map rows are
//     pre-filled with -1 in shared memory, so only found neighbours and the centre are
//     stored before the rows are written out coalesced.
// ---------------------------------------------------------------------------------------
constexpr int kMapK3Threads = 256;
constexpr int kK3Batch = 4;

template <bool BITMAP>
__device__ __forceinline__ void
k3_hash_block(const int4 *__restrict__ coords, int64_t M, int W, int H, int D, int Dw, int Dh, int Dd,
              const unsigned long long *__restrict__ table, const uint32_t *__restrict__ bitmap,
              int64_t bm_words, uint64_t gmask, uint32_t shift, int32_t *__restrict__ nbr,
              uint32_t *__restrict__ masks, uint32_t *hist, int sort_nt,
              int32_t *status, const int32_t *dup_flag, uint32_t *s_hist, int32_t *s_stage) {
    constexpr int V = 27;

    const int tid = threadIdx.x;
    const int64_t i0 = (int64_t)blockIdx.x * kMapK3Threads;
    const int nvox = (M - i0) < (int64_t)kMapK3Threads ? (int)(M - i0) : kMapK3Threads;
    for (int j = tid; j < kOrderBuckets; j += kMapK3Threads) s_hist[j] = 0u;
    {
        int4 *st4 = reinterpret_cast<int4 *>(s_stage);
        for (int j = tid; j < kMapK3Threads * V / 4; j += kMapK3Threads) st4[j] = make_int4(-1, -1, -1, -1);
    }

    const bool valid = tid < nvox;
    const int64_t i = i0 + tid;
    int4 c = make_int4(0, 0, 0, 0);
    if (valid) c = __ldg(coords + i);
    const int64_t HD = (int64_t)H * D;
    const int64_t key_c = (((int64_t)c.x * W + c.y) * H + c.z) * D + c.w;
    const int64_t sx = (int64_t)Dw * HD, sy = (int64_t)Dh * D;
    const bool in_x[3] = {c.y - Dw >= 0, true, c.y + Dw < W};
    const bool in_y[3] = {c.z - Dh >= 0, true, c.z + Dh < H};
    const bool in_z[3] = {c.w - Dd >= 0, true, c.w + Dd < D};
    const uint32_t zbits = (in_z[0] ? 1u : 0u) | 2u | (in_z[2] ? 4u : 0u);

    grid_launch_dependents();
    // Phase 1: candidate offsets.
    uint32_t cand = 0;
    if (valid) {
        if (BITMAP && 2 * Dd + 1 <= 32) {
            uint32_t lo[9], hi[9];
            const int zoff = in_z[0] ? Dd : 0;                 // window starts at the lowest in-range cell
#pragma unroll
            for (int q = 0; q < 9; ++q) {
                const int dx = q / 3, dy = q % 3;
                lo[q] = hi[q] = 0;
                if (in_x[dx] && in_y[dy]) {
                    const int64_t kb = key_c + (dx - 1) * sx + (dy - 1) * sy - zoff;
                    const int64_t wi = kb >> 5;
                    lo[q] = __ldg(bitmap + wi);
                    hi[q] = __ldg(bitmap + (wi + 1 < bm_words ? wi + 1 : wi));
                }
            }
            const int64_t k0 = key_c - zoff;                   // same low-bit phase for every column
#pragma unroll
            for (int q = 0; q < 9; ++q) {
                const int dx = q / 3, dy = q % 3;
                if (in_x[dx] && in_y[dy]) {
                    const int64_t kb = k0 + (dx - 1) * sx + (dy - 1) * sy;
                    const uint32_t win = __funnelshift_r(lo[q], hi[q], (uint32_t)(kb & 31));
                    const uint32_t b0 = in_z[0] ? (win & 1u) : 0u;                 // z - Dd
                    const uint32_t b1 = (win >> zoff) & 1u;                          // z
                    const uint32_t b2 = in_z[2] ? ((win >> (zoff + Dd)) & 1u) : 0u;  // z + Dd
                    cand |= (b0 | (b1 << 1) | (b2 << 2)) << (3 * q);
                }
            }
        } else {
#pragma unroll
            for (int q = 0; q < 9; ++q)
                if (in_x[q / 3] && in_y[q % 3]) cand |= zbits << (3 * q);
            if (BITMAP) {                                       // wide dilation: one load per cell
                uint32_t keep = 0;
                for (uint32_t m = cand; m; m &= m - 1) {
                    const int v = __ffs(m) - 1;
                    const int64_t kn = key_c + (v / 9 - 1) * sx + ((v / 3) % 3 - 1) * sy + (int64_t)(v % 3 - 1) * Dd;
                    if ((__ldg(bitmap + (kn >> 5)) >> (kn & 31)) & 1u) keep |= 1u << v;
                }
                cand = keep;
            }
        }
    }
    cand &= ~(1u << (V / 2));                                   // the centre is the voxel itself

    __syncthreads();                                            // hist zeroed, stage pre-filled
    uint32_t bits = valid ? (1u << (V / 2)) : 0u;
    if (valid) s_stage[tid * V + V / 2] = (int32_t)i;

    // Sorted input keeps a voxel's z - Dd and z + Dd neighbours in the adjacent rows. With
    // unique coordinates (this call's insert found no duplicate: a flag in its own workspace,
    // so neither an earlier call nor another stream's affects it) a row holding that
    // coordinate is the neighbour, so those offsets need no probe; otherwise they are probed.
    if (valid && (cand & ((1u << (V / 2 - 1)) | (1u << (V / 2 + 1)))) && *dup_flag == 0) {
        if ((cand >> (V / 2 + 1)) & 1u) {
            if (i + 1 < M) {
                const int4 n = __ldg(coords + i + 1);
                if (n.x == c.x && n.y == c.y && n.z == c.z && n.w == c.w + Dd) {
                    s_stage[tid * V + V / 2 + 1] = (int32_t)(i + 1);
                    bits |= 1u << (V / 2 + 1);
                    cand &= ~(1u << (V / 2 + 1));
                }
            }
        }
        if ((cand >> (V / 2 - 1)) & 1u) {
            if (i > 0) {
                const int4 n = __ldg(coords + i - 1);
                if (n.x == c.x && n.y == c.y && n.z == c.z && n.w == c.w - Dd) {
                    s_stage[tid * V + V / 2 - 1] = (int32_t)(i - 1);
                    bits |= 1u << (V / 2 - 1);
                    cand &= ~(1u << (V / 2 - 1));
                }
            }
        }
    }

    // Phase 2: probe candidate offsets, kK3Batch in flight.
    bool wrapped = false;
    while (cand) {
        int vv[kK3Batch];
        uint32_t key[kK3Batch];
        uint64_t grp[kK3Batch];
        unsigned long long word[kK3Batch][kGroup];
#pragma unroll
        for (int b = 0; b < kK3Batch; ++b) {
            vv[b] = -1;
            if (cand) {
                const int v = __ffs(cand) - 1;
                cand &= cand - 1;
                vv[b] = v;
                const int64_t kn = key_c + (v / 9 - 1) * sx + ((v / 3) % 3 - 1) * sy + (int64_t)(v % 3 - 1) * Dd;
                key[b] = (uint32_t)kn;
                grp[b] = home32(key[b], shift);
                load_group(table, grp[b], word[b]);
            }
        }
#pragma unroll
        for (int b = 0; b < kK3Batch; ++b) {
            if (vv[b] >= 0) {
                int32_t r = table_resolve<false>(table, nullptr, gmask, key[b], grp[b], word[b]);
                if (r == -2) { wrapped = true; r = -1; }
                if (r >= 0) {
                    s_stage[tid * V + vv[b]] = r;
                    bits |= 1u << vv[b];
                }
            }
        }
    }
    if (wrapped) raise_status(status, SPCONV_STATUS_TABLE_FULL);
    if (valid) masks[i] = bits;
    {
        const uint32_t pc = __popc(bits);
        const uint32_t h = fmix32(0x9e3779b9u ^ bits);
        const uint32_t k = order_bucket(bits, pc, h, V, sort_nt);
        const uint32_t active = __ballot_sync(0xffffffffu, valid);
        if (valid && hist) aggregated_inc(s_hist, k, active);
    }
    __syncthreads();
    {
        // The block's rows form one contiguous range of the map (16-byte aligned: i0 % 256 == 0).
        int32_t *out = nbr + i0 * (int64_t)V;
        const int total = nvox * V;
        const int n4 = total >> 2;
        const int4 *src = reinterpret_cast<const int4 *>(s_stage);
        int4 *dst = reinterpret_cast<int4 *>(out);
        for (int e = tid; e < n4; e += kMapK3Threads) dst[e] = src[e];
        for (int e = (n4 << 2) + tid; e < total; e += kMapK3Threads) out[e] = s_stage[e];
    }
    if (hist) order_hist_flush(s_hist, hist, sort_nt, i0);
}

// ---------------------------------------------------------------------------------------
// 2c'. Sorted-input path for 3x3x3 kernels (grids of < 2^32 cells and at most
//      kSortedMaxCols (b, x, y) columns). Coordinates as SparseConvTensor.from_dense and
//      voxelisers produce them - strictly increasing in (b, x, y, z) - need no hash table:
//      the rows of a column (b, x, y) are one contiguous range of the input, sorted by z, so
//      a neighbour is found by a binary search of the flat keys inside its column's range.
//      sorted_prep_kernel writes the flat keys, each occupied column's [first, last + 1) row
//      range (the array is cleared per call, so empty columns read as (0, 0)) and a per-call
//      word that is set when any row is out of range or not above its predecessor (unsorted
//      or duplicate input). The hash kernels above return at once when that word is clear,
//      map_sorted_k3 when it is set, so one of the two paths builds the map, with no host
//      synchronisation. For unique coordinates every neighbour is one row, so both paths
//      give the same map, masks and order keys bit for bit.
// ---------------------------------------------------------------------------------------
constexpr int kPrepThreads = 256;

__global__ void __launch_bounds__(kPrepThreads)
sorted_prep_kernel(const int4 *__restrict__ coords, int64_t M, int N, int W, int H, int D,
                   uint32_t *__restrict__ keys, int2 *__restrict__ colrange, int32_t *unsorted) {
    const int64_t i = (int64_t)blockIdx.x * kPrepThreads + threadIdx.x;
    auto in_range = [&](const int4 &c) {
        return c.x >= 0 && c.x < N && c.y >= 0 && c.y < W && c.z >= 0 && c.z < H && c.w >= 0 && c.w < D;
    };
    auto column = [&](const int4 &c) { return ((int64_t)c.x * W + c.y) * H + c.z; };
    bool bad = false;
    if (i < M) {
        const int4 c = __ldg(coords + i);
        if (!in_range(c)) {
            bad = true;
        } else {
            const int64_t col = column(c);
            const int64_t key = col * D + c.w;
            keys[i] = (uint32_t)key;
            bool first = true, last = true;
            if (i > 0) {
                const int4 p = __ldg(coords + i - 1);
                if (in_range(p)) {               // an out-of-range row flags itself
                    const int64_t pcol = column(p);
                    if (pcol * D + p.w >= key) bad = true;
                    first = pcol != col;
                }
            }
            if (i + 1 < M) {
                const int4 n = __ldg(coords + i + 1);
                if (in_range(n)) last = column(n) != col;
            }
            if (first) colrange[col].x = (int32_t)i;
            if (last) colrange[col].y = (int32_t)(i + 1);
        }
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) *unsorted = 1;
}

// Clears the hash path's table and bitmap (`n16` 16-byte words from `p`), unless the input
// took the sorted path. Highest addresses first, so the table (at the start) is the most
// recently written when the insert's atomics reach it.
__global__ void __launch_bounds__(256)
clear_unless_sorted_kernel(uint4 *__restrict__ p, int64_t n16, const int32_t *unsorted) {
    grid_dependency_wait();                                     // the prep kernel's word
    grid_launch_dependents();
    if (*unsorted == 0) return;
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n16; j += (int64_t)gridDim.x * blockDim.x)
        p[n16 - 1 - j] = z;
}

// One thread per voxel, 256 voxels per block, for strictly increasing coordinates. The nine
// (dx, dy) columns' ranges are loaded together; the nine lower-bound searches (for the lowest
// in-range z target of each column) advance in lockstep, so their key loads are in flight
// together; then the next 2*Dd + 1 rows of every column (those inside it) are loaded together
// and matched against z - Dd, z and z + Dd. With Dd = 1 the voxel's own z - 1 / z + 1
// neighbours can only be rows i - 1 / i + 1. Rows are staged in shared memory and written out
// coalesced; masks and order histogram as in k3_hash_block.
template <bool DD1>
__device__ __forceinline__ void
k3_sorted_block(const int4 *__restrict__ coords, const uint32_t *__restrict__ keys,
                const int2 *__restrict__ colrange, int64_t M, int W, int H, int D, int Dw, int Dh, int Dd,
                int32_t *__restrict__ nbr, uint32_t *__restrict__ masks, uint32_t *hist, int sort_nt,
                uint32_t *s_hist, int32_t *s_stage) {
    constexpr int V = 27;
    const int tid = threadIdx.x;
    const int64_t i0 = (int64_t)blockIdx.x * kMapK3Threads;
    const int nvox = (M - i0) < (int64_t)kMapK3Threads ? (int)(M - i0) : kMapK3Threads;
    for (int j = tid; j < kOrderBuckets; j += kMapK3Threads) s_hist[j] = 0u;
    {
        int4 *st4 = reinterpret_cast<int4 *>(s_stage);
        for (int j = tid; j < kMapK3Threads * V / 4; j += kMapK3Threads) st4[j] = make_int4(-1, -1, -1, -1);
    }
    grid_launch_dependents();
    const bool valid = tid < nvox;
    const int64_t i = i0 + tid;
    int4 c = make_int4(0, 0, 0, 0);
    if (valid) c = __ldg(coords + i);
    const int64_t col_c = ((int64_t)c.x * W + c.y) * H + c.z;
    const int64_t key_c = col_c * D + c.w;
    const bool in_x[3] = {c.y - Dw >= 0, true, c.y + Dw < W};
    const bool in_y[3] = {c.z - Dh >= 0, true, c.z + Dh < H};
    const bool lo_z = c.w - Dd >= 0, hi_z = c.w + Dd < D;
    const int zlo = lo_z ? Dd : 0;                              // lowest target: z - zlo

    int lo[9], len[9], end[9];
    uint32_t target[9];
#pragma unroll
    for (int q = 0; q < 9; ++q) {
        const int dx = q / 3 - 1, dy = q % 3 - 1;
        lo[q] = 0;
        len[q] = 0;
        end[q] = 0;
        const int64_t cq = col_c + (int64_t)dx * Dw * H + (int64_t)dy * Dh;
        target[q] = (uint32_t)(cq * D + c.w - zlo);
        if (valid && in_x[dx + 1] && in_y[dy + 1] && !(DD1 && q == 4)) {
            const int2 r = __ldg(colrange + cq);
            lo[q] = r.x;
            end[q] = r.y;
            len[q] = r.y > r.x ? r.y - r.x : 0;
            // A column no longer than the walk below is walked whole from its first row: no
            // search (most surface columns hold one to three voxels).
            if (len[q] <= (DD1 ? 3 : 2 * Dd + 1)) len[q] = 0;
        }
    }
    // Lockstep lower bounds: lo[q] = first row of the column whose key >= target[q].
    for (;;) {
        bool more = false;
#pragma unroll
        for (int q = 0; q < 9; ++q) {
            if (len[q] > 0) {
                const int half = len[q] >> 1;
                if (__ldg(keys + lo[q] + half) < target[q]) {
                    lo[q] += half + 1;
                    len[q] -= half + 1;
                } else {
                    len[q] = half;
                }
                more |= len[q] > 0;
            }
        }
        if (!more) break;
    }

    __syncthreads();                                            // hist zeroed, stage pre-filled
    uint32_t bits = valid ? (1u << (V / 2)) : 0u;
    if (valid) {
        s_stage[tid * V + V / 2] = (int32_t)i;
        // rel = key - target: the z distance above the lowest target; the targets z - Dd, z and
        // z + Dd sit at rel = 0 (when z - Dd is in range), zlo and zlo + Dd (when in range).
        auto match = [&](int q, int j, uint32_t key) {
            const uint32_t rel = key - target[q];
            int e = -1;
            if (lo_z && rel == 0u) e = 0;
            else if (rel == (uint32_t)zlo) e = 1;
            else if (hi_z && rel == (uint32_t)(zlo + Dd)) e = 2;
            const int v = q * 3 + e;
            if (e >= 0 && v != V / 2) {
                s_stage[tid * V + v] = j;
                bits |= 1u << v;
            }
        };
        if (DD1) {
            // every column's next three rows (those inside the column) and rows i - 1, i + 1
            const bool has_m = lo_z && i > 0, has_p = hi_z && i + 1 < M;
            const uint32_t km = has_m ? __ldg(keys + i - 1) : 0u;
            const uint32_t kp = has_p ? __ldg(keys + i + 1) : 0u;
            // The next three rows of columns 0-3, then of columns 5-8, loaded together (twelve
            // loads in flight, registers for no more); rows outside the column read as
            // target + 3 (e >= 3 below: no match).
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                uint32_t kk[4][3];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int q = half * 5 + u;
#pragma unroll
                    for (int s = 0; s < 3; ++s) {
                        const int j = lo[q] + s;
                        kk[u][s] = j < end[q] ? __ldg(keys + j) : target[q] + 3u;
                    }
                }
                // Dd = 1: the targets z - 1, z, z + 1 are e = rel + 1 - zlo = 0, 1, 2. A row of this
                // column at z - 1 exists only when z >= 1 and at z + 1 only when z + 1 < D, so no
                // range test is needed; rows below the lowest target wrap to large e.
#pragma unroll
                for (int u = 0; u < 4; ++u)
#pragma unroll
                    for (int s = 0; s < 3; ++s) {
                        const int q = half * 5 + u;
                        const uint32_t e = kk[u][s] - target[q] + 1u - (uint32_t)zlo;
                        if (e <= 2u) {
                            const int v = q * 3 + (int)e;
                            s_stage[tid * V + v] = lo[q] + s;
                            bits |= 1u << v;
                        }
                    }
            }
            if (has_m && km == (uint32_t)(key_c - 1)) {
                s_stage[tid * V + V / 2 - 1] = (int32_t)(i - 1);
                bits |= 1u << (V / 2 - 1);
            }
            if (has_p && kp == (uint32_t)(key_c + 1)) {
                s_stage[tid * V + V / 2 + 1] = (int32_t)(i + 1);
                bits |= 1u << (V / 2 + 1);
            }
        } else {
            const int walk = 2 * Dd + 1;
#pragma unroll
            for (int q = 0; q < 9; ++q)
                for (int s = 0; s < walk; ++s) {
                    const int j = lo[q] + s;
                    if (j < end[q]) match(q, j, __ldg(keys + j));
                }
        }
        masks[i] = bits;
    }
    {
        const uint32_t pc = __popc(bits);
        const uint32_t h = fmix32(0x9e3779b9u ^ bits);
        const uint32_t k = order_bucket(bits, pc, h, V, sort_nt);
        const uint32_t active = __ballot_sync(0xffffffffu, valid);
        if (valid && hist) aggregated_inc(s_hist, k, active);
    }
    __syncthreads();
    {
        int32_t *out = nbr + i0 * (int64_t)V;
        const int total = nvox * V;
        const int n4 = total >> 2;
        const int4 *src = reinterpret_cast<const int4 *>(s_stage);
        int4 *dst = reinterpret_cast<int4 *>(out);
        for (int e = tid; e < n4; e += kMapK3Threads) dst[e] = src[e];
        for (int e = (n4 << 2) + tid; e < total; e += kMapK3Threads) out[e] = s_stage[e];
    }
    if (hist) order_hist_flush(s_hist, hist, sort_nt, i0);
}

// The 3x3x3 map kernel: the column path when this call's input is strictly increasing (the
// prep kernel left `unsorted` clear), else the hash path; the word is read once per block
// after the previous kernels are complete, so every block takes the same path.
template <bool BITMAP, bool DD1>
__global__ void __launch_bounds__(kMapK3Threads, 4)
map_kernel_k3(const int4 *__restrict__ coords, int64_t M, int W, int H, int D, int Dw, int Dh, int Dd,
              const unsigned long long *__restrict__ table, const uint32_t *__restrict__ bitmap,
              int64_t bm_words, uint64_t gmask, uint32_t shift, int32_t *__restrict__ nbr,
              uint32_t *__restrict__ masks, uint32_t *hist, int sort_nt, int32_t *status, const int32_t *dup_flag,
              const uint32_t *__restrict__ keys, const int2 *__restrict__ colrange, const int32_t *unsorted) {
    __shared__ uint32_t s_hist[kOrderBuckets];
    __shared__ __align__(16) int32_t s_stage[kMapK3Threads * 27];   // read back as int4
    grid_dependency_wait();                                     // the insert's table / the prep's keys
    if (unsorted && *unsorted == 0)
        k3_sorted_block<DD1>(coords, keys, colrange, M, W, H, D, Dw, Dh, Dd, nbr, masks, hist, sort_nt, s_hist,
                             s_stage);
    else
        k3_hash_block<BITMAP>(coords, M, W, H, D, Dw, Dh, Dd, table, bitmap, bm_words, gmask, shift, nbr, masks,
                              hist, sort_nt, status, dup_flag, s_hist, s_stage);
}

// ---------------------------------------------------------------------------------------
// 2d. Map build for other kernels with V <= 128 offsets whose z extent spans <= 32 cells
//     (e.g. 5x5x5), with the occupancy bitmap: the same two phases as 2c with the kernel
//     shape at run time. Phase 1 reads one funnel-shifted bitmap window per (dx, dy) column
//     (four columns' loads in flight) and keeps the in-range z cells of it; phase 2 probes
//     the candidates, four at a time, 32 offset columns at a time: the chunk's row segments
//     are staged in shared memory pre-filled with -1 and written a warp per row segment,
//     which keeps the stage at 16.5 KB whatever V is (six blocks per SM instead of two).
// ---------------------------------------------------------------------------------------
constexpr int kMapColsThreads = 128;
constexpr int kMapColsMaxV = 128;
constexpr int kMapColsStride = 33;
constexpr int kMapColsMinBlocks = 6;

__device__ __forceinline__ void or_word4(uint32_t (&m)[4], int w, uint32_t x) {
    if (w == 0) m[0] |= x;
    else if (w == 1) m[1] |= x;
    else if (w == 2) m[2] |= x;
    else if (w == 3) m[3] |= x;
}
__device__ __forceinline__ void clear_bit4(uint32_t (&m)[4], int v) {
    const uint32_t x = ~(1u << (v & 31));
    if ((v >> 5) == 0) m[0] &= x;
    else if ((v >> 5) == 1) m[1] &= x;
    else if ((v >> 5) == 2) m[2] &= x;
    else m[3] &= x;
}
// Lowest set bit of a 128-bit mask (cleared), or -1.
__device__ __forceinline__ int pop_lowest4(uint32_t (&m)[4]) {
    if (m[0]) { const int b = __ffs(m[0]) - 1; m[0] &= m[0] - 1u; return b; }
    if (m[1]) { const int b = __ffs(m[1]) - 1; m[1] &= m[1] - 1u; return 32 + b; }
    if (m[2]) { const int b = __ffs(m[2]) - 1; m[2] &= m[2] - 1u; return 64 + b; }
    if (m[3]) { const int b = __ffs(m[3]) - 1; m[3] &= m[3] - 1u; return 96 + b; }
    return -1;
}

__device__ __forceinline__ uint32_t get_word4(const uint32_t (&m)[4], int w) {
    return w == 0 ? m[0] : w == 1 ? m[1] : w == 2 ? m[2] : m[3];
}

__global__ void __launch_bounds__(kMapColsThreads, kMapColsMinBlocks)
map_kernel_cols(const int4 *__restrict__ coords, int64_t M, int W, int H, int D, int Kw, int Kh, int Kd,
                int Dw, int Dh, int Dd, int V, int MW, const unsigned long long *__restrict__ table,
                const uint32_t *__restrict__ bitmap, int64_t bm_words, uint64_t gmask, uint32_t shift,
                int32_t *__restrict__ nbr, uint32_t *__restrict__ masks, uint32_t *hist, int sort_nt,
                int32_t *status) {
    __shared__ uint32_t s_hist[kOrderBuckets];
    // 32 offset columns of every row of the block; stride 33 keeps both the per-thread
    // row writes and the per-warp row-segment reads free of bank conflicts.
    __shared__ int32_t s_stage[kMapColsThreads * kMapColsStride];

    // Block-invariant offset tables: the key offset of every kernel offset v, and per (dx, dy)
    // column its key offset and its x / y displacement (no divisions in the per-voxel loops).
    __shared__ long long s_voff[kMapColsMaxV];
    __shared__ int4 s_col[kMapColsMaxV];                       // {key offset lo, hi, dx, dy}

    const int tid = threadIdx.x;
    const int64_t i0 = (int64_t)blockIdx.x * kMapColsThreads;
    const int nvox = (M - i0) < (int64_t)kMapColsThreads ? (int)(M - i0) : kMapColsThreads;
    for (int j = tid; j < kOrderBuckets; j += kMapColsThreads) s_hist[j] = 0u;
    {
        const int64_t sxw = (int64_t)Dw * H * D, syw = (int64_t)Dh * D;
        const int rw0 = Kw / 2, rh0 = Kh / 2, rd0 = Kd / 2;
        if (tid < V) {                                          // V <= kMapColsThreads
            const int cx = tid / (Kh * Kd), rem = tid - cx * (Kh * Kd);
            const int cy = rem / Kd, cz = rem - cy * Kd;
            s_voff[tid] = (cx - rw0) * sxw + (cy - rh0) * syw + (int64_t)(cz - rd0) * Dd;
        }
        if (tid < Kw * Kh) {
            const int cx = tid / Kh, cy = tid - cx * Kh;
            const int64_t dk = (cx - rw0) * sxw + (cy - rh0) * syw;
            s_col[tid] = make_int4((int)(uint32_t)dk, (int)(dk >> 32), (cx - rw0) * Dw, (cy - rh0) * Dh);
        }
    }
    __syncthreads();

    const bool valid = tid < nvox;
    const int64_t i = i0 + tid;
    int4 c = make_int4(0, 0, 0, 0);
    if (valid) c = __ldg(coords + i);
    const int64_t key_c = (((int64_t)c.x * W + c.y) * H + c.z) * D + c.w;
    const int rd = Kd / 2;
    const int zlo = max(c.w - rd * Dd, 0);                      // window starts at the lowest in-range cell
    // in-range z cells of a column and their bit positions in the window
    uint32_t zsel = 0;
    for (int cz = 0; cz < Kd; ++cz) {
        const int z = c.w + (cz - rd) * Dd;
        if (z >= 0 && z < D) zsel |= 1u << cz;
    }
    auto extract = [&](uint32_t win) -> uint32_t {              // window bits -> Kd column bits
        if (Dd == 1) {
            const int s0 = zlo - (c.w - rd);                    // cells below z = 0 (>= 0)
            return (s0 < 32 ? (win << s0) : 0u) & zsel;
        }
        uint32_t r = 0;
        for (int cz = 0; cz < Kd; ++cz)
            if ((zsel >> cz) & 1u) r |= ((win >> (c.w + (cz - rd) * Dd - zlo)) & 1u) << cz;
        return r;
    };

    grid_dependency_wait();                                     // the insert's table and bitmap
    grid_launch_dependents();
    // Phase 1: candidate offsets.
    uint32_t cand[4] = {0u, 0u, 0u, 0u};
    const int ncol = Kw * Kh;
    if (valid) {
        const int64_t kz = key_c + (zlo - c.w);                 // key of the window start, centre column
        for (int q0 = 0; q0 < ncol; q0 += 4) {
            uint32_t lo[4], hi[4];
            int64_t kb[4];
            bool in[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int q = q0 + u;
                in[u] = false;
                lo[u] = hi[u] = 0u;
                kb[u] = 0;
                if (q < ncol) {
                    const int4 e = s_col[q];
                    const int x = c.y + e.z, y = c.z + e.w;
                    in[u] = (unsigned)x < (unsigned)W && (unsigned)y < (unsigned)H;
                    kb[u] = kz + (int64_t)(((uint64_t)(uint32_t)e.y << 32) | (uint32_t)e.x);
                }
                if (in[u]) {
                    const int64_t wi = kb[u] >> 5;
                    lo[u] = __ldg(bitmap + wi);
                    hi[u] = __ldg(bitmap + (wi + 1 < bm_words ? wi + 1 : wi));
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (in[u]) {
                    const uint32_t bits = extract(__funnelshift_r(lo[u], hi[u], (uint32_t)(kb[u] & 31)));
                    const int v0 = (q0 + u) * Kd, w = v0 >> 5, sft = v0 & 31;
                    or_word4(cand, w, bits << sft);
                    if (sft + Kd > 32 && sft > 0) or_word4(cand, w + 1, bits >> (32 - sft));
                }
            }
        }
    }
    const int vc = V / 2;                                       // the centre entry is the voxel itself
    clear_bit4(cand, vc);

    // Phase 2, one 32-column chunk of the rows at a time: probe the chunk's candidates
    // (kK3Batch in flight), then the block writes the chunk's row segments, a warp per row.
    uint32_t bits[4] = {0u, 0u, 0u, 0u};
    bool wrapped = false;
    int32_t *row = s_stage + tid * kMapColsStride;
    const int warp = tid >> 5, lane = tid & 31;
    const int nch = (V + 31) >> 5;
    for (int ch = 0; ch < nch; ++ch) {
#pragma unroll 8
        for (int j = 0; j < 32; ++j) row[j] = -1;
        uint32_t got = 0u;
        if (valid && (vc >> 5) == ch) {
            row[vc & 31] = (int32_t)i;
            got = 1u << (vc & 31);
        }
        uint32_t cw = valid ? get_word4(cand, ch) : 0u;
        while (cw) {
            int vv[kK3Batch];
            uint32_t key[kK3Batch];
            uint64_t grp[kK3Batch];
            unsigned long long word[kK3Batch][kGroup];
#pragma unroll
            for (int b = 0; b < kK3Batch; ++b) {
                vv[b] = -1;
                if (cw) {
                    const int bl = __ffs(cw) - 1;
                    cw &= cw - 1u;
                    const int v = (ch << 5) + bl;
                    vv[b] = bl;
                    const int64_t kn = key_c + s_voff[v];
                    key[b] = (uint32_t)kn;
                    grp[b] = home32(key[b], shift);
                    load_group(table, grp[b], word[b]);
                }
            }
#pragma unroll
            for (int b = 0; b < kK3Batch; ++b) {
                if (vv[b] >= 0) {
                    int32_t r = table_resolve<false>(table, nullptr, gmask, key[b], grp[b], word[b]);
                    if (r == -2) { wrapped = true; r = -1; }
                    if (r >= 0) {
                        row[vv[b]] = r;
                        got |= 1u << vv[b];
                    }
                }
            }
        }
        or_word4(bits, ch, got);
        __syncthreads();                                        // the chunk's rows are staged
        const int col = (ch << 5) + lane;
        if (col < V) {
            int32_t *out = nbr + i0 * (int64_t)V + col;
            for (int r = warp; r < nvox; r += kMapColsThreads / 32)
                out[(int64_t)r * V] = s_stage[r * kMapColsStride + lane];
        }
        __syncthreads();                                        // the stage is free again
    }
    if (wrapped) raise_status(status, SPCONV_STATUS_TABLE_FULL);
    {
        uint32_t pc = 0, h = 0x9e3779b9u;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            if (w < MW) {
                if (valid) masks[i * (int64_t)MW + w] = bits[w];
                pc += __popc(bits[w]);
                h = fmix32(h ^ bits[w]);
            }
        }
        const uint32_t k = order_bucket(bits[0], pc, h, V, sort_nt);
        const uint32_t active = __ballot_sync(0xffffffffu, valid);
        if (valid && hist) aggregated_inc(s_hist, k, active);
    }
    __syncthreads();
    if (hist) order_hist_flush(s_hist, hist, sort_nt, i0);
}

// ---------------------------------------------------------------------------------------
// 3. Counting-sort scatter of voxel ids by order key. Every block scans the map kernel's
//    global histogram (16 KB from L2) into bucket starts itself, so no block of the map
//    kernel waits for the others; a bucket's voxels of one block take one cursor atomic.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kOrderThreads)
order_kernel(const uint32_t *__restrict__ masks, int64_t M, int MW, const uint32_t *hist,
             uint32_t *cursor, int32_t *__restrict__ order, int32_t *status) {
    constexpr int kPer = kOrderBuckets / kOrderThreads;        // 16 buckets per thread
    __shared__ uint32_t s_cnt[kOrderBuckets];
    __shared__ __align__(16) uint32_t s_base[kOrderBuckets];
    __shared__ uint32_t s_warp[kOrderThreads / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t i0 = (int64_t)blockIdx.x * (kOrderThreads * kOrderPerThread);
    for (int b = tid; b < kOrderBuckets; b += kOrderThreads) s_cnt[b] = 0u;
    grid_dependency_wait();                                     // the map kernel's masks and histogram
    grid_launch_dependents();
    {
        // bucket starts: exclusive scan of the histogram, buckets tid*kPer .. tid*kPer+kPer-1 here
        uint32_t local[kPer];
        uint32_t sum = 0;
        const uint4 *h4 = reinterpret_cast<const uint4 *>(hist + tid * kPer);
#pragma unroll
        for (int q = 0; q < kPer / 4; ++q) {
            const uint4 v = __ldcg(h4 + q);
            local[4 * q] = v.x; local[4 * q + 1] = v.y; local[4 * q + 2] = v.z; local[4 * q + 3] = v.w;
            sum += v.x + v.y + v.z + v.w;
        }
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
        for (int k = 0; k < kPer; ++k) { s_base[tid * kPer + k] = run; run += local[k]; }
    }
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
        if (s_cnt[b]) s_base[b] += atomicAdd(cursor + b, s_cnt[b]);
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

// ---------------------------------------------------------------------------------------
// 3b. Order by a stable LSD radix sort of the voxels' mask keys (V <= 27, M >= 2^19).
//     key = neighbour-count class (4 bits: min(popcount - 1, 15)) above the top 20 bits of
//     the mask without its centre bit (all V - 1 bits when V <= 21). The order groups voxels
//     by class and, inside a class, by the mask read as a number: masks next to each other
//     share their high offsets, so a 128-voxel tile of the order needs few offsets beyond its
//     voxels' own. Equal keys keep input order (the (b,x,y,z) order of the coordinates), so
//     their feature rows are gathered with spatial locality.
//     Per 8-bit digit pass: the tile digit counts (made for the first pass by the map kernels,
//     which add each block's low key digits to its tile's column, and for later passes by
//     sort_count_kernel),
//     sort_scan_kernel (one block per digit) scans the counts over tiles, and
//     sort_scatter_kernel ranks each tile's keys stably (lanes with equal digits found by
//     eight ballots, per-warp digit counters, warps in input order) and writes them to their
//     sorted positions.
// ---------------------------------------------------------------------------------------
// Number of 8-bit passes for the keys of a V-offset kernel.
static int sort_passes(int V) {
    return (4 + V - 1 - order_key_drop(V) + 7) / 8;
}

// Lanes of the warp whose 8-bit digit equals this lane's, among `active`.
__device__ __forceinline__ uint32_t digit_peers(uint32_t d, uint32_t active) {
    uint32_t peers = active;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
        const bool bit = (d >> b) & 1u;
        const uint32_t bb = __ballot_sync(0xffffffffu, bit);
        peers &= bit ? bb : ~bb;
    }
    return peers;
}

// Digit counts of each 2048-key tile for passes after the first (the map kernels count the
// first pass's digits as they build the masks).
__global__ void __launch_bounds__(kSortThreads)
sort_count_kernel(const uint32_t *__restrict__ keys, int64_t M, int ntiles, int shift,
                  uint32_t *__restrict__ counts) {
    __shared__ uint32_t s_cnt[256];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid < 256) s_cnt[tid] = 0u;
    grid_dependency_wait();                                     // the masks / the previous pass's keys
    grid_launch_dependents();
    __syncthreads();
    const int64_t e0 = (int64_t)blockIdx.x * kSortTile + warp * kSortWarpItems + lane;
    uint32_t d[kSortWarpItems / 32];
#pragma unroll
    for (int k = 0; k < kSortWarpItems / 32; ++k) {
        const int64_t e = e0 + 32 * k;
        d[k] = 0xffffffffu;
        if (e < M) d[k] = (__ldg(keys + e) >> shift) & 255u;
    }
#pragma unroll
    for (int k = 0; k < kSortWarpItems / 32; ++k) {
        const bool valid = d[k] != 0xffffffffu;
        const uint32_t peers = digit_peers(d[k], __ballot_sync(0xffffffffu, valid));
        if (valid && lane == __ffs(peers) - 1) atomicAdd(&s_cnt[d[k]], (uint32_t)__popc(peers));
    }
    __syncthreads();
    if (tid < 256) counts[(int64_t)tid * ntiles + blockIdx.x] = s_cnt[tid];
}

// Exclusive block scan of one value per thread (blockDim.x = kSortThreads); also returns
// the block total. Uses s_warp[kSortThreads / 32 + 1].
__device__ __forceinline__ uint32_t sort_block_scan(uint32_t x, uint32_t *s_warp, uint32_t &total) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int kWarps = kSortThreads / 32;
    uint32_t incl = x;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const uint32_t n = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += n;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const uint32_t w = lane < kWarps ? s_warp[lane] : 0u;
        uint32_t wi = w;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const uint32_t n = __shfl_up_sync(0xffffffffu, wi, d);
            if (lane >= d) wi += n;
        }
        if (lane < kWarps) s_warp[lane] = wi - w;
        if (lane == kWarps - 1) s_warp[kWarps] = wi;
    }
    __syncthreads();
    const uint32_t r = s_warp[warp] + incl - x;
    total = s_warp[kWarps];
    __syncthreads();                                            // s_warp reusable
    return r;
}

// counts[d][0..ntiles) -> exclusive prefix over tiles, in place; totals[d] = the digit's count.
__global__ void __launch_bounds__(kSortThreads)
sort_scan_kernel(uint32_t *__restrict__ counts, int ntiles, uint32_t *__restrict__ totals) {
    __shared__ uint32_t s_warp[kSortThreads / 32 + 1];
    uint32_t *row = counts + (int64_t)blockIdx.x * ntiles;
    grid_dependency_wait();                                     // counts of this pass
    grid_launch_dependents();
    uint32_t carry = 0;
    for (int base = 0; base < ntiles; base += kSortThreads) {
        const int t = base + (int)threadIdx.x;
        const uint32_t x = t < ntiles ? row[t] : 0u;
        uint32_t tot;
        const uint32_t ex = sort_block_scan(x, s_warp, tot);
        if (t < ntiles) row[t] = carry + ex;
        carry += tot;
    }
    if (threadIdx.x == 0) totals[blockIdx.x] = carry;
}

template <bool FIRST, bool LAST>
__global__ void __launch_bounds__(kSortThreads)
sort_scatter_kernel(const uint32_t *__restrict__ masks, int V, const uint32_t *__restrict__ keys_in,
                    const uint32_t *__restrict__ vals_in, int64_t M, int ntiles, int shift,
                    const uint32_t *__restrict__ offsets, const uint32_t *__restrict__ totals,
                    uint32_t *__restrict__ keys_out, uint32_t *__restrict__ vals_out, int32_t *status) {
    constexpr int kWarps = kSortThreads / 32, kRounds = kSortWarpItems / 32;
    __shared__ uint32_t s_wcnt[kWarps][256];                    // per-warp digit counts, then bases
    __shared__ uint32_t s_dbase[256];
    __shared__ uint32_t s_warp[kWarps + 1];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int tile = blockIdx.x;
    for (int j = tid; j < kWarps * 256; j += kSortThreads) (&s_wcnt[0][0])[j] = 0u;
    grid_dependency_wait();                                     // this pass's scanned counts
    grid_launch_dependents();
    __syncthreads();

    const int64_t e0 = (int64_t)tile * kSortTile + warp * kSortWarpItems + lane;
    uint32_t key[kRounds], val[kRounds], loc[kRounds];
    const uint32_t lt = (1u << lane) - 1u;
#pragma unroll
    for (int k = 0; k < kRounds; ++k) {
        const int64_t e = e0 + 32 * k;
        key[k] = 0u;
        val[k] = 0xffffffffu;                                   // marks lanes past the end
        if (e < M) {
            if (FIRST) { key[k] = order_key(__ldg(masks + e), V); val[k] = (uint32_t)e; }
            else { key[k] = __ldg(keys_in + e); val[k] = __ldg(vals_in + e); }
        }
    }
#pragma unroll
    for (int k = 0; k < kRounds; ++k) {
        const bool valid = val[k] != 0xffffffffu;
        const uint32_t d = (key[k] >> shift) & 255u;
        const uint32_t peers = digit_peers(d, __ballot_sync(0xffffffffu, valid));
        const uint32_t before = valid ? s_wcnt[warp][d] : 0u;
        __syncwarp();
        if (valid && lane == __ffs(peers) - 1) s_wcnt[warp][d] = before + (uint32_t)__popc(peers);
        __syncwarp();
        loc[k] = before + (uint32_t)__popc(peers & lt);
    }
    __syncthreads();
    // Per digit: warps' exclusive prefix in warp order; digit start = all smaller digits of
    // every tile + this digit in earlier tiles.
    uint32_t dtot = 0u;
    if (tid < 256) {
        uint32_t run = 0u;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const uint32_t c = s_wcnt[w][tid];
            s_wcnt[w][tid] = run;
            run += c;
        }
        dtot = totals[tid];
    }
    uint32_t all;
    const uint32_t dex = sort_block_scan(tid < 256 ? dtot : 0u, s_warp, all);
    if (tid < 256) s_dbase[tid] = dex + offsets[(int64_t)tid * ntiles + tile];
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kRounds; ++k) {
        if (val[k] == 0xffffffffu) continue;
        const uint32_t d = (key[k] >> shift) & 255u;
        const uint32_t pos = s_dbase[d] + s_wcnt[warp][d] + loc[k];
        if (pos < (uint64_t)M) {
            if (!LAST) keys_out[pos] = key[k];
            vals_out[pos] = val[k];
        } else {
            raise_status(status, SPCONV_STATUS_TABLE_FULL);   // inconsistent counts
        }
    }
}

}  // namespace spconv

using namespace spconv;

extern "C" int64_t spconv_hashmap_capacity(int64_t num_coords) {
    return capacity_for(num_coords > 0 ? num_coords : 0);
}

extern "C" int spconv_mask_words(int kernel_volume) {
    return kernel_volume <= 0 ? 0 : (kernel_volume + 31) / 32;
}

extern "C" int64_t spconv_neighbor_map_workspace_bytes(int64_t num_coords, int batch, int W, int H, int D) {
    if (num_coords < 0) return -1;
    return ws_layout(num_coords, !volume_fits_32(batch, W, H, D), bitmap_words_for(batch, W, H, D),
                     radix_order(num_coords, batch, W, H, D), sorted_cols(batch, W, H, D)).total;
}

namespace spconv {
// The map build; allow_radix = false keeps the bucket order at every size (the fixed scratch of
// the allocation-free entry point has no room for the radix sort's counts).
static int build_map(const int32_t *coords, int64_t M, int batch, int W, int H, int D, int Kw, int Kh, int Kd,
                     int Dw, int Dh, int Dd, void *workspace, int64_t workspace_bytes, int32_t *neighbor_map,
                     uint32_t *masks, int32_t *order, int32_t *status, void *stream_ptr, bool allow_radix,
                     bool allow_sorted) {
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
    // The occupancy bitmap is used when the workspace has room for it.
    const bool sort = allow_radix && radix_order(M, batch, W, H, D);
    // The sorted-input path serves 3x3x3 kernels (section 2c'); its regions are used when the
    // workspace has room for them, the occupancy bitmap when it has room for that.
    const int64_t cols = (allow_sorted && Kw == 3 && Kh == 3 && Kd == 3) ? sorted_cols(batch, W, H, D) : 0;
    WsLayout L = ws_layout(M, key64, bitmap_words_for(batch, W, H, D), sort, cols);
    if (L.cols && workspace_bytes < L.total) L = ws_layout(M, key64, bitmap_words_for(batch, W, H, D), sort);
    if (L.bitmap_words && workspace_bytes < L.total) L = ws_layout(M, key64, 0, sort);
    SPCONV_REQUIRE(workspace_bytes >= L.total, SPCONV_ERR_ARG,
                   "workspace too small: %lld < %lld bytes", (long long)workspace_bytes, (long long)L.total);
    cudaStream_t stream = (cudaStream_t)stream_ptr;
    char *ws = (char *)workspace;
    unsigned long long *table = (unsigned long long *)(ws + L.table);
    uint32_t *vals = key64 ? (uint32_t *)(ws + L.vals) : nullptr;
    uint32_t *bitmap = L.bitmap_words ? (uint32_t *)(ws + L.bitmap) : nullptr;
    uint32_t *hist = (uint32_t *)(ws + L.hist);
    uint32_t *cursor = (uint32_t *)(ws + L.cursor);
    int32_t *dup_flag = (int32_t *)(ws + L.flags);
    const uint64_t gmask = (uint64_t)(L.cap / kGroup) - 1;
    uint32_t shift = 32;
    for (int64_t c = L.cap / kGroup; c > 1; c >>= 1) --shift;   // 32 - log2(groups)
    const int MW = spconv_mask_words(V);
    // Stable radix-sort order for kernels of <= kSortMaxV offsets when the workspace has room
    // (radix_order); the map kernels then skip the bucket histogram.
    const bool radix = L.sort_tiles > 0 && V <= kSortMaxV;
    // The radix order's first digit counts come from the map kernels themselves (into the sort
    // counts, zeroed with the workspace), so its first pass needs no counting launch.
    const int sort_nt = radix ? L.sort_tiles : 0;
    if (radix) hist = (uint32_t *)(ws + L.sort_counts);

    int32_t *unsorted = L.cols ? dup_flag + 1 : nullptr;       // per-call word: the hash path runs
    uint32_t *keys = L.cols ? (uint32_t *)(ws + L.keys) : nullptr;

    stage_mark(SPCONV_STAGE_MEMSET, 0, stream);
    if (L.cols) {
        // Histogram, cursors, flags, sort counts and column ranges are cleared for every input;
        // the table and bitmap only when the input takes the hash path.
        if (cudaMemsetAsync(ws + L.hist, 0, (size_t)(L.keys - L.hist), stream) != cudaSuccess)
            return check_launch("workspace memset");
        const int64_t pb = (M + kPrepThreads - 1) / kPrepThreads;
        sorted_prep_kernel<<<(unsigned)pb, kPrepThreads, 0, stream>>>(
            (const int4 *)coords, M, batch, W, H, D, keys, (int2 *)(ws + L.colrange), unsorted);
        if (int rc = check_launch("sorted_prep_kernel")) return rc;
        const int64_t n16 = L.hist / 16;                        // table (+ rows) + bitmap
        launch_pdl(clear_unless_sorted_kernel, dim3(148 * 8), dim3(256), 0, stream, (uint4 *)ws, n16,
                   (const int32_t *)unsorted);
        if (int rc = check_launch("clear_unless_sorted_kernel")) return rc;
    } else if (L.bitmap_words && M >= kSortMinVoxels) {
        // Everything after the table first (the bitmap is the bulk of it), the table last, so
        // the table's lines are the most recently written when the insert's atomics reach them
        // (indoor: insert 71 -> 60 us for +3 us of memset; below 2^19 voxels the second memset
        // costs more than it saves).
        const int64_t tail = L.table + align256(L.cap * 8) + (key64 ? align256(L.cap * 4) : 0);
        if (cudaMemsetAsync(ws + tail, 0, (size_t)(L.total - tail), stream) != cudaSuccess ||
            cudaMemsetAsync(ws, 0, (size_t)tail, stream) != cudaSuccess)
            return check_launch("workspace memset");
    } else if (cudaMemsetAsync(workspace, 0, (size_t)L.total, stream) != cudaSuccess) {
        return check_launch("workspace memset");
    }
    stage_mark(SPCONV_STAGE_MEMSET, 1, stream);
    const int64_t gi = (M + 255) / 256;
    // Where the input may take the sorted path the insert usually returns at once: a grid of
    // 16 blocks per SM (grid-stride) keeps that cheap; otherwise one thread per voxel.
    const int64_t gcap = L.cols ? 148LL * 16 : 65535LL * 32;
    const int ins_grid = (int)(gi < gcap ? gi : gcap);
    stage_mark(SPCONV_STAGE_INSERT, 0, stream);
    if (key64)
        insert_kernel<true><<<ins_grid, 256, 0, stream>>>((const int4 *)coords, M, batch, W, H, D, table, vals, bitmap, gmask, shift, status, dup_flag, unsorted);
    else if (L.cols)     // after the clear kernel: its launch overlaps that kernel's tail
        launch_pdl(insert_kernel<false>, dim3(ins_grid), dim3(256), 0, stream, (const int4 *)coords, M, batch, W, H, D,
                   table, vals, bitmap, gmask, shift, status, dup_flag, (const int32_t *)unsorted);
    else
        insert_kernel<false><<<ins_grid, 256, 0, stream>>>((const int4 *)coords, M, batch, W, H, D, table, vals, bitmap, gmask, shift, status, dup_flag, unsorted);
    if (int rc = check_launch("insert_kernel")) return rc;
    stage_mark(SPCONV_STAGE_INSERT, 1, stream);

    if (!key64 && Kw == 3 && Kh == 3 && Kd == 3) {
        auto k3_fn = bitmap ? (Dd == 1 ? map_kernel_k3<true, true> : map_kernel_k3<true, false>)
                            : (Dd == 1 ? map_kernel_k3<false, true> : map_kernel_k3<false, false>);
        const int grid = (int)((M + kMapK3Threads - 1) / kMapK3Threads);
        stage_mark(SPCONV_STAGE_MAP, 0, stream);
        launch_pdl(k3_fn, dim3(grid), dim3(kMapK3Threads), 0, stream,
                   (const int4 *)coords, M, W, H, D, Dw, Dh, Dd, (const unsigned long long *)table,
                   (const uint32_t *)bitmap, L.bitmap_words, gmask, shift, neighbor_map, masks, hist,
                   sort_nt, status, (const int32_t *)dup_flag, (const uint32_t *)keys,
                   (const int2 *)(L.cols ? ws + L.colrange : nullptr), (const int32_t *)unsorted);
    } else if (!key64 && bitmap && V <= kMapColsMaxV && (Kd - 1) * Dd + 1 <= 32) {
        const int grid = (int)((M + kMapColsThreads - 1) / kMapColsThreads);
        stage_mark(SPCONV_STAGE_MAP, 0, stream);
        launch_pdl(map_kernel_cols, dim3(grid), dim3(kMapColsThreads), 0, stream,
                   (const int4 *)coords, M, W, H, D, Kw, Kh, Kd, Dw, Dh, Dd, V, MW,
                   (const unsigned long long *)table, (const uint32_t *)bitmap, L.bitmap_words, gmask,
                   shift, neighbor_map, masks, hist, sort_nt, status);
    } else if (bitmap && Kd <= kColBatchMax) {
        // 256 voxels per block while their staged rows fit in 64 KB, else 128.
        const int nthr = ((size_t)kMapBmMaxThreads * (V | 1) * 4 <= 64 * 1024) ? kMapBmMaxThreads : 128;
        int vstride = (V % 2 == 0) ? V + 1 : V;
        if ((size_t)nthr * vstride * 4 > (size_t)kMapStageMaxBytes) vstride = 0;
        const size_t smem = (size_t)nthr * (size_t)vstride * sizeof(int32_t);
        auto bm_fn = Kd <= 4 ? map_kernel_bm<4> : map_kernel_bm<kColBatchMax>;
        raise_smem_limit((const void *)bm_fn, Kd <= 4 ? 0 : 1);
        const int grid = (int)((M + nthr - 1) / nthr);
        stage_mark(SPCONV_STAGE_MAP, 0, stream);
        bm_fn<<<grid, nthr, smem, stream>>>(
            (const int4 *)coords, M, W, H, D, Kw, Kh, Kd, Dw, Dh, Dd, V, MW, vstride, table, bitmap,
            L.bitmap_words, gmask, shift, neighbor_map, masks, hist, sort_nt, status);
    } else {
        const int map_grid = (int)((M + kMapThreads - 1) / kMapThreads);
        // Rows are staged in shared memory (odd row stride: conflict-free) unless V is so
        // large that the stage would not fit; then rows are stored directly.
        int vstride = (V % 2 == 0) ? V + 1 : V;
        if ((size_t)kMapThreads * vstride * 4 > (size_t)kMapStageMaxBytes) vstride = 0;
        const size_t map_smem = (size_t)V * (sizeof(int4) + sizeof(long long)) +
                                (size_t)kMapThreads * (size_t)vstride * sizeof(int32_t);
        auto map_fn = key64 ? map_kernel<true, false> : (bitmap ? map_kernel<false, true> : map_kernel<false, false>);
        if (map_smem > 48 * 1024) raise_smem_limit((const void *)map_fn, 2 + (key64 ? 0 : (bitmap ? 2 : 1)));
        stage_mark(SPCONV_STAGE_MAP, 0, stream);
        map_fn<<<map_grid, kMapThreads, map_smem, stream>>>(
            (const int4 *)coords, M, W, H, D, Kw, Kh, Kd, Dw, Dh, Dd, V, MW, vstride, table, vals, bitmap,
            gmask, shift, neighbor_map, masks, hist, sort_nt, status);
    }
    if (int rc = check_launch("map_kernel")) return rc;
    stage_mark(SPCONV_STAGE_MAP, 1, stream);

    stage_mark(SPCONV_STAGE_ORDER, 0, stream);
    if (radix) {
        const int nt = L.sort_tiles, passes = sort_passes(V);
        uint32_t *counts = (uint32_t *)(ws + L.sort_counts);
        uint32_t *totals = counts + (int64_t)kSortMaxPasses * 256 * nt;
        uint32_t *tbl = (uint32_t *)table;                      // 4 x M words
        uint32_t *kb[2] = {tbl, tbl + 2 * M}, *vb[2] = {tbl + M, tbl + 3 * M};
        for (int p = 0; p < passes; ++p) {
            uint32_t *cp = counts + (int64_t)p * 256 * nt, *tp = totals + p * 256;
            const bool first = p == 0, last = p + 1 == passes;
            uint32_t *ko = kb[p & 1], *vo = last ? (uint32_t *)order : vb[p & 1];
            const uint32_t *ki = first ? nullptr : kb[(p + 1) & 1], *vi = first ? nullptr : vb[(p + 1) & 1];
            if (!first) {                    // the first pass's counts come from the map kernel
                launch_pdl(sort_count_kernel, dim3(nt), dim3(kSortThreads), 0, stream, ki, M, nt, 8 * p, cp);
                if (int rc = check_launch("sort_count_kernel")) return rc;
            }
            launch_pdl(sort_scan_kernel, dim3(256), dim3(kSortThreads), 0, stream, cp, nt, tp);
            if (int rc = check_launch("sort_scan_kernel")) return rc;
            auto fn = first ? (last ? sort_scatter_kernel<true, true> : sort_scatter_kernel<true, false>)
                            : (last ? sort_scatter_kernel<false, true> : sort_scatter_kernel<false, false>);
            launch_pdl(fn, dim3(nt), dim3(kSortThreads), 0, stream, (const uint32_t *)masks, V, ki, vi, M, nt,
                       8 * p, (const uint32_t *)cp, (const uint32_t *)tp, ko, vo, status);
            if (int rc = check_launch("sort_scatter_kernel")) return rc;
        }
    } else {
        const int per_block = kOrderThreads * kOrderPerThread;
        const int ord_grid = (int)((M + per_block - 1) / per_block);
        launch_pdl(order_kernel, dim3(ord_grid), dim3(kOrderThreads), 0, stream, (const uint32_t *)masks, M, MW,
                   (const uint32_t *)hist, cursor, order, status);
        if (int rc = check_launch("order_kernel")) return rc;
    }
    stage_mark(SPCONV_STAGE_ORDER, 1, stream);
    return SPCONV_OK;
}
}  // namespace spconv

extern "C" int spconv_build_submanifold_neighbor_map(
    const int32_t *coords, int64_t M,
    int batch, int W, int H, int D,
    int Kw, int Kh, int Kd, int Dw, int Dh, int Dd,
    void *workspace, int64_t workspace_bytes,
    int32_t *neighbor_map, uint32_t *masks, int32_t *order,
    int32_t *status, void *stream_ptr) {
    return build_map(coords, M, batch, W, H, D, Kw, Kh, Kd, Dw, Dh, Dd, workspace, workspace_bytes,
                     neighbor_map, masks, order, status, stream_ptr, true, true);
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

constexpr int64_t noalloc_capacity() { return capacity_for((int64_t)SPCONV_NOALLOC_MAX_COORDS); }
constexpr int64_t align256c(int64_t x) { return (x + 255) & ~int64_t(255); }
// The largest layout ws_layout gives for at most SPCONV_NOALLOC_MAX_COORDS voxels: 64-bit keys
// (table + row array), no bitmap, histogram, cursors and the per-call flags. The radix-sort counts are absent
// because that entry point keeps the bucket order at every size it accepts; a 32-bit-key layout is smaller,
// and its bitmap is dropped when it does not fit.
constexpr int64_t kNoAllocScratchBytes =
    align256c(noalloc_capacity() * 8) + align256c(noalloc_capacity() * 4) +
    2 * align256c(kOrderBuckets * 4) + 256 /* per-call flags */ + 256;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
static std::mutex g_noalloc_mu;
static void *g_noalloc_dev_ptr[kNoAllocMaxDevices] = {};

// Device address of the scratch array on the current device; looked up once per device and
// kept for the life of the process, so the entry point must not be used on a device after
// cudaDeviceReset (or anything else that destroys its primary context) in the same process.
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
    return build_map(
        coords, M, batch, W, H, D, Kw, Kh, Kd, Dw, Dh, Dd, scratch, kNoAllocScratchBytes,
        neighbor_map, masks, order, status, stream, false, false);
}

// ---------------------------------------------------------------------------------------
// 2-D submanifold map (replaces hashmap_build_submanifold_conv2d_neighbor_map_cuda_naive,
// neighbor_map.cu:10-111): (b, x, y) coordinates on a W x H grid with a Kw x Kh kernel. Its
// offset order v = dx * Kh + dy, centre rule v == V/2 and flat key b*W*H + x*H + y are those
// of the 3-D map with D = 1, Kd = 1 and z = 0, so the coordinates are widened to (b, x, y, 0)
// in the workspace and the 3-D builder runs on them.
// ---------------------------------------------------------------------------------------
namespace spconv {

__global__ void __launch_bounds__(256)
widen_coords_2d_kernel(const int32_t *__restrict__ c3, int64_t M, int4 *__restrict__ c4) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < M; i += (int64_t)gridDim.x * blockDim.x)
        c4[i] = make_int4(__ldg(c3 + 3 * i), __ldg(c3 + 3 * i + 1), __ldg(c3 + 3 * i + 2), 0);
}

static int64_t coords4_bytes(int64_t M) { return align256(M * 16); }

}  // namespace spconv

extern "C" int64_t spconv_neighbor_map_2d_workspace_bytes(int64_t num_coords, int batch, int W, int H) {
    if (num_coords < 0) return -1;
    // the 3-D layout with D = 1 and no sorted-input regions (the 2-D kernel is not 3x3x3)
    const int64_t b3 = ws_layout(num_coords, !volume_fits_32(batch, W, H, 1), bitmap_words_for(batch, W, H, 1),
                                 radix_order(num_coords, batch, W, H, 1)).total;
    return b3 < 0 ? -1 : b3 + coords4_bytes(num_coords);
}

extern "C" int spconv_build_submanifold_neighbor_map_2d(
    const int32_t *coords, int64_t M, int batch, int W, int H, int Kw, int Kh, int Dw, int Dh,
    void *workspace, int64_t workspace_bytes,
    int32_t *neighbor_map, uint32_t *masks, int32_t *order, int32_t *status, void *stream) {
    SPCONV_REQUIRE(M >= 0, SPCONV_ERR_ARG, "num_coords must be >= 0 (got %lld)", (long long)M);
    if (M == 0) return SPCONV_OK;
    SPCONV_REQUIRE(coords && workspace, SPCONV_ERR_ARG, "null pointer argument");
    SPCONV_REQUIRE(((uintptr_t)workspace & 255u) == 0, SPCONV_ERR_ARG, "workspace must be 256-byte aligned");
    const int64_t need = spconv_neighbor_map_2d_workspace_bytes(M, batch, W, H);
    SPCONV_REQUIRE(need >= 0 && workspace_bytes >= need, SPCONV_ERR_ARG,
                   "workspace too small: %lld < %lld bytes", (long long)workspace_bytes, (long long)need);
    int4 *c4 = (int4 *)workspace;
    cudaStream_t s = (cudaStream_t)stream;
    int64_t blocks = (M + 255) / 256;
    if (blocks > 148LL * 32) blocks = 148LL * 32;
    widen_coords_2d_kernel<<<(unsigned)blocks, 256, 0, s>>>(coords, M, c4);
    if (int rc = check_launch("widen_coords_2d_kernel")) return rc;
    const int64_t off = coords4_bytes(M);
    return spconv_build_submanifold_neighbor_map(
        (const int32_t *)c4, M, batch, W, H, 1, Kw, Kh, 1, Dw, Dh, 1, (char *)workspace + off,
        workspace_bytes - off, neighbor_map, masks, order, status, stream);
}
