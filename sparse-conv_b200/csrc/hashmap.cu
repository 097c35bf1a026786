// Generic GPU hash table bindings (the reference's hashmap_insert_cuda / hashmap_lookup_cuda,
// hash.cu:8-146, hash.cuh:1-87): a caller-owned open-addressing table of `capacity` slots —
// keys (uint32 or uint64, empty = all ones) and values (uint32 or uint64) in two arrays, the
// layout the reference's Python allocates (ops/utils.py:3-16). The slot of a key is the
// MurmurHash3 finaliser of the key modulo the capacity, probed linearly, so tables built here
// and by the reference read the same. Differences: every probe loop is bounded by the
// capacity (a full table sets SPCONV_STATUS_TABLE_FULL instead of spinning), and the kernels
// are grid-stride over the keys. As in the reference, a key inserted twice in one call keeps
// one of its values (whichever store lands last).
#include <limits>

#include "common.cuh"

namespace spconv {

__device__ __forceinline__ uint64_t slot_of(uint32_t k, uint64_t n) { return (uint64_t)fmix32(k) % n; }
__device__ __forceinline__ uint64_t slot_of(uint64_t k, uint64_t n) { return fmix64(k) % n; }

__device__ __forceinline__ uint32_t cas_key(uint32_t *p, uint32_t cmp, uint32_t val) { return atomicCAS(p, cmp, val); }
__device__ __forceinline__ uint64_t cas_key(uint64_t *p, uint64_t cmp, uint64_t val) {
    return (uint64_t)atomicCAS(reinterpret_cast<unsigned long long *>(p), (unsigned long long)cmp,
                               (unsigned long long)val);
}

template <typename K, typename V>
__global__ void __launch_bounds__(256)
hashmap_insert_kernel(K *__restrict__ tkeys, V *__restrict__ tvals, uint64_t cap, const K *__restrict__ keys,
                      const V *__restrict__ vals, int64_t n, int32_t *status) {
    constexpr K kEmpty = std::numeric_limits<K>::max();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const K key = __ldg(keys + i);
        const V val = __ldg(vals + i);
        uint64_t s = slot_of(key, cap);
        bool done = false;
        for (uint64_t p = 0; p < cap; ++p) {
            const K prev = cas_key(tkeys + s, kEmpty, key);
            if (prev == kEmpty || prev == key) {
                tvals[s] = val;
                done = true;
                break;
            }
            if (++s == cap) s = 0;
        }
        if (!done) raise_status(status, SPCONV_STATUS_TABLE_FULL);
    }
}

template <typename K, typename V>
__global__ void __launch_bounds__(256)
hashmap_lookup_kernel(const K *__restrict__ tkeys, const V *__restrict__ tvals, uint64_t cap,
                      const K *__restrict__ keys, V *__restrict__ out, int64_t n) {
    constexpr K kEmpty = std::numeric_limits<K>::max();
    constexpr V kMissing = std::numeric_limits<V>::max();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const K key = __ldg(keys + i);
        uint64_t s = slot_of(key, cap);
        V v = kMissing;
        for (uint64_t p = 0; p < cap; ++p) {
            const K k = __ldg(tkeys + s);
            if (k == key) { v = __ldg(tvals + s); break; }
            if (k == kEmpty) break;
            if (++s == cap) s = 0;
        }
        out[i] = v;
    }
}

template <typename K, typename V>
static int hashmap_op(bool insert, void *tk, void *tv, int64_t cap, const void *keys, const void *vals, void *out,
                      int64_t n, int32_t *status, cudaStream_t s) {
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148LL * 64) blocks = 148LL * 64;
    if (insert) {
        hashmap_insert_kernel<K, V><<<(unsigned)blocks, 256, 0, s>>>((K *)tk, (V *)tv, (uint64_t)cap, (const K *)keys,
                                                                     (const V *)vals, n, status);
        return check_launch("hashmap_insert_kernel");
    }
    hashmap_lookup_kernel<K, V><<<(unsigned)blocks, 256, 0, s>>>((const K *)tk, (const V *)tv, (uint64_t)cap,
                                                                 (const K *)keys, (V *)out, n);
    return check_launch("hashmap_lookup_kernel");
}

static int hashmap_dispatch(bool insert, void *tk, void *tv, int64_t cap, int key_bits, int value_bits,
                            const void *keys, const void *vals, void *out, int64_t n, int32_t *status,
                            cudaStream_t s) {
    if (key_bits == 32 && value_bits == 32) return hashmap_op<uint32_t, uint32_t>(insert, tk, tv, cap, keys, vals, out, n, status, s);
    if (key_bits == 32 && value_bits == 64) return hashmap_op<uint32_t, uint64_t>(insert, tk, tv, cap, keys, vals, out, n, status, s);
    if (key_bits == 64 && value_bits == 32) return hashmap_op<uint64_t, uint32_t>(insert, tk, tv, cap, keys, vals, out, n, status, s);
    return hashmap_op<uint64_t, uint64_t>(insert, tk, tv, cap, keys, vals, out, n, status, s);
}

}  // namespace spconv

using namespace spconv;

extern "C" int spconv_hashmap_insert(void *table_keys, void *table_values, int64_t capacity, int key_bits,
                                     int value_bits, const void *keys, const void *values, int64_t n,
                                     int32_t *status, void *stream) {
    SPCONV_REQUIRE((key_bits == 32 || key_bits == 64) && (value_bits == 32 || value_bits == 64), SPCONV_ERR_ARG,
                   "key/value bits must be 32 or 64 (got %d/%d)", key_bits, value_bits);
    SPCONV_REQUIRE(capacity > 0 && n >= 0, SPCONV_ERR_ARG, "capacity must be > 0 and n >= 0");
    if (n == 0) return SPCONV_OK;
    SPCONV_REQUIRE(table_keys && table_values && keys && values, SPCONV_ERR_ARG, "null pointer argument");
    return hashmap_dispatch(true, table_keys, table_values, capacity, key_bits, value_bits, keys, values, nullptr, n,
                            status, (cudaStream_t)stream);
}

extern "C" int spconv_hashmap_lookup(const void *table_keys, const void *table_values, int64_t capacity,
                                     int key_bits, int value_bits, const void *keys, void *values_out, int64_t n,
                                     void *stream) {
    SPCONV_REQUIRE((key_bits == 32 || key_bits == 64) && (value_bits == 32 || value_bits == 64), SPCONV_ERR_ARG,
                   "key/value bits must be 32 or 64 (got %d/%d)", key_bits, value_bits);
    SPCONV_REQUIRE(capacity > 0 && n >= 0, SPCONV_ERR_ARG, "capacity must be > 0 and n >= 0");
    if (n == 0) return SPCONV_OK;
    SPCONV_REQUIRE(table_keys && table_values && keys && values_out, SPCONV_ERR_ARG, "null pointer argument");
    return hashmap_dispatch(false, const_cast<void *>(table_keys), const_cast<void *>(table_values), capacity,
                            key_bits, value_bits, keys, nullptr, values_out, n, nullptr, (cudaStream_t)stream);
}
