// Internal interface between the conv entry points (conv.cu) and the kernel launchers.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace spconv {

struct ConvArgs {
    const void *feats;
    int dtype;
    int64_t M;
    int Ci;
    const void *weight;
    const void *bias;
    int Co;
    int V;
    int MW;
    const int32_t *nbr;
    const uint32_t *masks;
    const int32_t *order;
    void *out;
    int32_t *status;
    cudaStream_t stream;
    // 1: read the map with offsets reversed (column V-1-v for offset v) and the masks likewise:
    // for odd kernel sizes that is the transposed map, so the input gradient needs no copy
    int flip = 0;
    // non-null: tcgen05 kernel with split tiles, this workspace holding the per-tile counters
    // and fp32 partials (conv_split_workspace_bytes)
    void *split_ws = nullptr;
};

bool tc_supported(int dtype, int Ci, int Co, int V);

// Resident CTAs per SM for `kern` at `threads` threads and `smem_dynamic` bytes of dynamic
// shared memory, from the kernel's attributes and the device limits (shared memory incl. the
// per-CTA reservation, registers at warp granularity, threads, CTAs).
int occupancy_per_sm(const void *kern, int threads, int smem_dynamic);
int launch_conv_tc(const ConvArgs &a);
int64_t split_counter_bytes();
int64_t conv_split_workspace_bytes(int64_t M, int Co);
int launch_conv_simt(const ConvArgs &a);

// tcgen05 weight gradient (wgrad_tc.cu): 16-bit features with Ci = Co = 64; `masks` may be null
// (every offset of a tile is then gathered, missing neighbours as zeros).
bool wgrad_tc_supported(int dtype, int Ci, int Co, int V);
int launch_wgrad_tc(int dtype, const void *feats, const void *gout, const int32_t *nbr, const int32_t *order,
                    const uint32_t *masks, int64_t M, int V, float *gw, int32_t *status, cudaStream_t stream);

}  // namespace spconv
