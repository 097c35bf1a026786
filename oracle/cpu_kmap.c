/*
 * ORACLE -- test infrastructure only. Nothing in the product (the sparseconv package,
 * its CUDA library) links, loads or calls this file. Only tests/, the smoke check and
 * the CPU-baseline leg of bench.py use it, as the checker or as the CPU timing arm.
 *
 * CPU restatement of the reference's submanifold 3D kernel-map build, in plain C with
 * OpenMP over voxels. It follows the reference step by step:
 *
 *   - key flattening of (b,x,y,z):         src/sparseconv/kernels/cuda/hash/hash.cu:376-388
 *   - 32/64-bit murmur3 finaliser % N:    src/sparseconv/kernels/cuda/hash/hash.cuh:1-20
 *   - linear-probing insert (CAS, then
 *     value store; an existing key is
 *     overwritten):                        src/sparseconv/kernels/cuda/hash/hash.cuh:22-63
 *   - linear-probing lookup:               src/sparseconv/kernels/cuda/hash/hash.cuh:65-87
 *   - per (voxel, offset) neighbour
 *     decomposition, centre rule v==V/2
 *     -> own row, bounds check on x/y/z
 *     only (batch not checked):            src/sparseconv/kernels/cuda/neighbor_map/neighbor_map.cu:145-176
 *   - map pre-filled with 0xFFFFFFFF:      src/sparseconv/kernels/cuda/neighbor_map/neighbor_map.cu:196-200
 *   - table capacity int(2.0 * M), uint32
 *     keys when N*W*H*D < 2^32 else
 *     uint64:                              src/sparseconv/ops/utils.py:3-16, ops/submanifold_conv3d.py:43-45
 *
 * The insert runs sequentially in row order, so where a coordinate repeats, the last
 * (highest) row is the one the table keeps. The reference inserts in parallel and keeps
 * whichever duplicate store lands last; the sequential order is one of its outcomes.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline uint64_t oracle_hash32(uint32_t k, uint64_t n) {
    k ^= k >> 16;
    k *= 0x85ebca6bu;
    k ^= k >> 13;
    k *= 0xc2b2ae35u;
    k ^= k >> 16;
    return (uint64_t)k % n;
}

static inline uint64_t oracle_hash64(uint64_t k, uint64_t n) {
    k ^= k >> 33;
    k *= 0xff51afd7ed558ccdULL;
    k ^= k >> 33;
    k *= 0xc4ceb9fe1a85ec53ULL;
    k ^= k >> 33;
    return k % n;
}

/* Flat key exactly as the reference computes it: size_t arithmetic on int coordinates. */
static inline uint64_t oracle_flat(int b, int x, int y, int z, int W, int H, int D) {
    return (uint64_t)(int64_t)b * (uint64_t)W * (uint64_t)H * (uint64_t)D
         + (uint64_t)(int64_t)x * (uint64_t)H * (uint64_t)D
         + (uint64_t)(int64_t)y * (uint64_t)D
         + (uint64_t)(int64_t)z;
}

/* Returns the table capacity the reference would allocate for M coordinates. */
int64_t oracle_table_capacity(int64_t M) {
    return (int64_t)(2.0 * (double)M);
}

/*
 * Build the [M, V] neighbour map (row-major, uint32, missing = 0xFFFFFFFF).
 * key64 = 0 uses 32-bit keys (N*W*H*D < 2^32), 1 uses 64-bit keys.
 * Returns 0 on success, -1 on bad arguments, -2 on allocation failure,
 * -3 when a probe sequence wraps the whole table (the reference would spin forever).
 */
int oracle_build_neighbor_map(const int32_t *coords, int64_t M,
                              int W, int H, int D,
                              int Kw, int Kh, int Kd,
                              int Dw, int Dh, int Dd,
                              int key64, int nthreads,
                              uint32_t *out) {
    if (M <= 0 || !coords || !out) return -1;
    const int V = Kw * Kh * Kd;
    const int64_t cap = oracle_table_capacity(M);
    if (cap <= 0) return -1;

    void *keys = key64 ? malloc((size_t)cap * sizeof(uint64_t)) : malloc((size_t)cap * sizeof(uint32_t));
    uint32_t *vals = (uint32_t *)malloc((size_t)cap * sizeof(uint32_t));
    if (!keys || !vals) { free(keys); free(vals); return -2; }
    if (key64) memset(keys, 0xFF, (size_t)cap * sizeof(uint64_t));
    else memset(keys, 0xFF, (size_t)cap * sizeof(uint32_t));
    memset(vals, 0, (size_t)cap * sizeof(uint32_t));

    /* Insert, row order (hash.cu:376-388 + hash.cuh:22-63). */
    for (int64_t i = 0; i < M; ++i) {
        const int32_t *c = coords + 4 * i;
        uint64_t flat = oracle_flat(c[0], c[1], c[2], c[3], W, H, D);
        int64_t probes = 0;
        if (key64) {
            uint64_t *k = (uint64_t *)keys;
            uint64_t key = flat;
            uint64_t slot = oracle_hash64(key, (uint64_t)cap);
            for (;;) {
                if (k[slot] == UINT64_MAX || k[slot] == key) { k[slot] = key; vals[slot] = (uint32_t)i; break; }
                slot = (slot + 1) % (uint64_t)cap;
                if (++probes > cap) { free(keys); free(vals); return -3; }
            }
        } else {
            uint32_t *k = (uint32_t *)keys;
            uint32_t key = (uint32_t)flat;
            uint64_t slot = oracle_hash32(key, (uint64_t)cap);
            for (;;) {
                if (k[slot] == UINT32_MAX || k[slot] == key) { k[slot] = key; vals[slot] = (uint32_t)i; break; }
                slot = slot + 1;
                if (slot >= (uint64_t)cap) slot = 0;
                if (++probes > cap) { free(keys); free(vals); return -3; }
            }
        }
    }

    /* Lookup, one (voxel, offset) pair at a time (neighbor_map.cu:145-176). */
    int failed = 0;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static) reduction(| : failed)
#endif
    for (int64_t i = 0; i < M; ++i) {
        const int32_t *c = coords + 4 * i;
        const int b = c[0];
        const int x = c[1] - Kw / 2 * Dw;
        const int y = c[2] - Kh / 2 * Dh;
        const int z = c[3] - Kd / 2 * Dd;
        const int KhKd = Kh * Kd;
        uint32_t *row = out + (size_t)i * (size_t)V;
        for (int v = 0; v < V; ++v) {
            uint32_t value = UINT32_MAX;
            if (v == V / 2) {
                value = (uint32_t)i;
            } else {
                const int kx = x + v / KhKd * Dw;
                const int ky = y + v / Kd % Kh * Dh;
                const int kz = z + v % Kd * Dd;
                if (kx >= 0 && kx < W && ky >= 0 && ky < H && kz >= 0 && kz < D) {
                    uint64_t flat = oracle_flat(b, kx, ky, kz, W, H, D);
                    int64_t probes = 0;
                    if (key64) {
                        const uint64_t *k = (const uint64_t *)keys;
                        uint64_t slot = oracle_hash64(flat, (uint64_t)cap);
                        for (;;) {
                            if (k[slot] == UINT64_MAX) break;
                            if (k[slot] == flat) { value = vals[slot]; break; }
                            slot = (slot + 1) % (uint64_t)cap;
                            if (++probes > cap) { failed = 1; break; }
                        }
                    } else {
                        const uint32_t *k = (const uint32_t *)keys;
                        const uint32_t key = (uint32_t)flat;
                        uint64_t slot = oracle_hash32(key, (uint64_t)cap);
                        for (;;) {
                            if (k[slot] == UINT32_MAX) break;
                            if (k[slot] == key) { value = vals[slot]; break; }
                            slot = slot + 1;
                            if (slot >= (uint64_t)cap) slot = 0;
                            if (++probes > cap) { failed = 1; break; }
                        }
                    }
                }
            }
            row[v] = value;
        }
    }
    free(keys);
    free(vals);
    return failed ? -3 : 0;
}

/*
 * EXPLICIT_GEMM forward restated in float64 (ops/submanifold_conv3d.py:76-86):
 * out[i, co] = bias[co] + sum_v sum_ci feats[nbr[i, v], ci] * weight[co, v, ci],
 * skipping nbr == 0xFFFFFFFF. feats [M, Ci], weight [Co, V, Ci], out [M, Co], all float64.
 */
void oracle_conv_gather_f64(const double *feats, const uint32_t *nbr, const double *weight,
                            const double *bias, int64_t M, int Ci, int Co, int V,
                            int nthreads, double *out) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static)
#endif
    for (int64_t i = 0; i < M; ++i) {
        double *o = out + (size_t)i * (size_t)Co;
        for (int co = 0; co < Co; ++co) o[co] = bias ? bias[co] : 0.0;
        for (int v = 0; v < V; ++v) {
            const uint32_t n = nbr[(size_t)i * (size_t)V + (size_t)v];
            if (n == UINT32_MAX) continue;
            const double *f = feats + (size_t)n * (size_t)Ci;
            for (int co = 0; co < Co; ++co) {
                const double *w = weight + ((size_t)co * (size_t)V + (size_t)v) * (size_t)Ci;
                double acc = 0.0;
                for (int ci = 0; ci < Ci; ++ci) acc += f[ci] * w[ci];
                o[co] += acc;
            }
        }
    }
}
