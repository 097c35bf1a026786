/*
 * sparseconv_b200 -- C ABI of the B200 (sm_100a) submanifold 3D sparse-convolution library.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream (as void*,
 * NULL = legacy default stream), launches asynchronously on that stream, and returns an
 * SPCONV_* code. Host-side validation failures return SPCONV_ERR_ARG; a failed CUDA launch
 * returns SPCONV_ERR_CUDA; in both cases spconv_last_error() holds a message (per thread).
 * Problems found on the device (coordinates out of range, a full hash table, duplicate
 * coordinates, a spin-wait limit reached) are OR-ed as SPCONV_STATUS_* bits into the
 * caller's int32 `status` word in device memory; the caller reads it when it next syncs.
 *
 * Reference interfaces replaced (paths inside Arktetra/sparse-conv):
 *   - spconv_hashmap_capacity / spconv_neighbor_map_workspace_bytes
 *       replace the table allocation policy of src/sparseconv/ops/utils.py:3-16
 *       (init_hashmap) and ops/submanifold_conv3d.py:43-45 (capacity = 2.0 * M).
 *   - spconv_build_submanifold_neighbor_map
 *       replaces hashmap_build_submanifold_conv_neighbor_map_cuda_naive,
 *       src/sparseconv/kernels/cuda/neighbor_map/neighbor_map.h:16-28
 *       (implementation neighbor_map.cu:179-237, bound in kernels/cuda/ext.cpp:9).
 *   - spconv_submanifold_conv_forward
 *       replaces sparse_submanifold_conv_fwd_implicit_gemm,
 *       src/sparseconv/kernels/triton/implicit_gemm.py:59-86, and the EXPLICIT_GEMM
 *       forward of ops/submanifold_conv3d.py:76-86.
 */
#ifndef SPARSECONV_B200_H
#define SPARSECONV_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes. */
#define SPCONV_OK 0
#define SPCONV_ERR_ARG 1
#define SPCONV_ERR_CUDA 2
#define SPCONV_ERR_UNSUPPORTED 3

/* Device status bits (OR-ed into *status by kernels). */
#define SPCONV_STATUS_COORD_RANGE 1   /* a coordinate lies outside [0,N)x[0,W)x[0,H)x[0,D) */
#define SPCONV_STATUS_TABLE_FULL 2    /* a probe sequence visited every slot */
#define SPCONV_STATUS_DUPLICATE 4     /* a coordinate occurs twice; the highest row is kept */
#define SPCONV_STATUS_WAIT_TIMEOUT 8  /* a kernel-internal wait hit its time limit */

/* Feature dtypes. */
#define SPCONV_F32 0
#define SPCONV_F16 1
#define SPCONV_BF16 2

/* Conv kernel selection for spconv_submanifold_conv_forward_ex. */
#define SPCONV_KERNEL_AUTO 0
#define SPCONV_KERNEL_SIMT 1      /* CUDA-core FMA kernel, any channel count, fp32 exact path */
#define SPCONV_KERNEL_TCGEN05 2   /* tcgen05/TMEM tensor-core kernel, fp16/bf16, C in {16,32,64,128} */

/* ABI version of this header. */
#define SPCONV_ABI_VERSION 1

int spconv_abi_version(void);

/* Time limit, in nanoseconds, of the pipeline waits inside the tensor-core conv kernels
 * launched after this call (process-wide; default 2 s; 0 restores the default). A wait that
 * reaches it makes the kernel abandon its work, wait (bounded) for its own copies and MMAs,
 * free its tensor memory, return, and set SPCONV_STATUS_WAIT_TIMEOUT; the context stays
 * usable. Returns the previous limit. Lowering it is for tests of that path.
 * No counterpart in the reference (its probe loops have no bound). */
uint64_t spconv_set_wait_limit_ns(uint64_t limit_ns);

/* Message of the last host-side error on the calling thread ("" if none). */
const char *spconv_last_error(void);

/* Slots of the coordinate hash table for num_coords voxels: the next power of two
 * >= 4 * num_coords while that table stays <= 64 MB (load <= 0.25), else the next power of
 * two >= 2 * num_coords (load <= 0.5); at least 1024.
 * Replaces the sizing of ops/utils.py:3-16 + ops/submanifold_conv3d.py:43-45. */
int64_t spconv_hashmap_capacity(int64_t num_coords);

/* Number of uint32 words of the per-voxel offset mask: ceil(kernel_volume / 32). */
int spconv_mask_words(int kernel_volume);

/* Device workspace (bytes) that spconv_build_submanifold_neighbor_map needs for
 * num_coords voxels on a grid of batch*W*H*D cells. 256-byte alignment suffices. */
int64_t spconv_neighbor_map_workspace_bytes(int64_t num_coords, int batch, int W, int H, int D);

/* Build the submanifold kernel map of num_coords voxels.
 *   coords       [M,4] int32 (b,x,y,z), device, 16-byte aligned
 *   batch,W,H,D  the NCWHD sizes without C (ops/submanifold_conv3d.py:41)
 *   Kw,Kh,Kd     kernel size; Dw,Dh,Dd dilation
 *   workspace    >= spconv_neighbor_map_workspace_bytes(...) bytes of device memory;
 *                its contents on entry do not matter (the call clears what it uses)
 *   neighbor_map [M,V] int32 output, V = Kw*Kh*Kd, row-major in the reference's offset
 *                order (v = ((dx*Kh)+dy)*Kd+dz); -1 (0xFFFFFFFF) for a missing neighbour;
 *                entry v == V/2 is the voxel's own row. Bit-identical to the reference's
 *                uint32 map (neighbor_map.cu:145-176).
 *   masks        [M, spconv_mask_words(V)] uint32 output: bit v set iff neighbor_map[i,v] >= 0
 *   order        [M] int32 output: a permutation of 0..M-1, the conv kernels' tile order.
 *                For M >= 2^19 and V <= 27 it is the stable sort of the voxels by
 *                key = min(popcount(mask) - 1, 15) << b | (mask without bit V/2) >> d, where
 *                d = max(V - 21, 0) and b = V - 1 - d (deterministic). Otherwise it groups
 *                voxels by that class and a hash of the mask, in an unspecified order inside
 *                a group. Conv results do not depend on it.
 *   status       device int32, OR-ed with SPCONV_STATUS_* bits
 * Replaces neighbor_map.h:16-28 (hashmap_build_submanifold_conv_neighbor_map_cuda_naive). */
int spconv_build_submanifold_neighbor_map(
    const int32_t *coords, int64_t num_coords,
    int batch, int W, int H, int D,
    int Kw, int Kh, int Kd, int Dw, int Dh, int Dd,
    void *workspace, int64_t workspace_bytes,
    int32_t *neighbor_map, uint32_t *masks, int32_t *order,
    int32_t *status, void *stream);

/* Workspace (bytes) for spconv_build_submanifold_neighbor_map_2d. */
int64_t spconv_neighbor_map_2d_workspace_bytes(int64_t num_coords, int batch, int W, int H);

/* 2-D submanifold kernel map: coords [M,3] int32 (b, x, y) on a batch x W x H grid, kernel
 * Kw x Kh, dilation Dw x Dh; neighbor_map [M, Kw*Kh] with v = dx*Kh + dy, -1 = missing,
 * v == V/2 the voxel's own row; masks / order as for the 3-D map. The reference's 2-D map is
 * its 3-D map with D = 1, Kd = 1, z = 0 (same offsets, centre rule and keys), and so is this.
 * Replaces hashmap_build_submanifold_conv2d_neighbor_map_cuda_naive (neighbor_map.h:4-14,
 * neighbor_map.cu:10-111). */
int spconv_build_submanifold_neighbor_map_2d(
    const int32_t *coords, int64_t num_coords, int batch, int W, int H,
    int Kw, int Kh, int Dw, int Dh,
    void *workspace, int64_t workspace_bytes,
    int32_t *neighbor_map, uint32_t *masks, int32_t *order,
    int32_t *status, void *stream);

/* Dense <-> sparse conversion (SparseConvTensor.from_dense / .dense, core.py:52-77).
 * spconv_from_dense: a voxel of the channels-last dense [batch, W, H, D, C] tensor is active
 * iff any of its C values is non-zero (x != 0: NaN counts, -0 does not). Phase 0 writes the
 * number of active voxels to *count (device int64); the caller reads it, allocates indices
 * [count, 4] int32 (16-byte aligned) and feats [count, C], and calls phase 1, which writes
 * (b, x, y, z) and the features in (b, x, y, z) order. The workspace
 * (spconv_from_dense_workspace_bytes) must be the same for both phases.
 * spconv_to_dense: zeroes out [batch, C, W, H, D] (channels_first) or [batch, W, H, D, C] and
 * writes feats [M, C] at indices [M, 4]; indices outside the grid set SPCONV_STATUS_COORD_RANGE. */
int64_t spconv_from_dense_workspace_bytes(int batch, int W, int H, int D);
int spconv_from_dense(const void *dense, int dtype, int batch, int W, int H, int D, int C,
                      void *workspace, int64_t workspace_bytes, int64_t *count,
                      int32_t *indices, void *feats, int64_t capacity, int phase, void *stream);
int spconv_to_dense(const void *feats, int dtype, const int32_t *indices, int64_t num_coords, int C,
                    int batch, int W, int H, int D, int channels_first, void *out,
                    int32_t *status, void *stream);

/* Generic caller-owned hash table (hashmap_insert_cuda / hashmap_lookup_cuda, hash.cu:8-146):
 * table_keys [capacity] uint32/uint64 (key_bits), filled with all ones when empty;
 * table_values [capacity] uint32/uint64 (value_bits). The slot of a key is the MurmurHash3
 * finaliser of the key modulo capacity, probed linearly (the reference's layout and slots, so
 * its tables read the same here and back). Insert stores values (a key given twice in one call
 * keeps one of its values) and sets SPCONV_STATUS_TABLE_FULL in *status when no slot is left;
 * lookup writes the value, or all ones for an absent key. Probing is bounded by capacity. */
int spconv_hashmap_insert(void *table_keys, void *table_values, int64_t capacity, int key_bits,
                          int value_bits, const void *keys, const void *values, int64_t n,
                          int32_t *status, void *stream);
int spconv_hashmap_lookup(const void *table_keys, const void *table_values, int64_t capacity,
                          int key_bits, int value_bits, const void *keys, void *values_out, int64_t n,
                          void *stream);

/* Largest num_coords that spconv_build_submanifold_neighbor_map_noalloc accepts. */
#define SPCONV_NOALLOC_MAX_COORDS 262144

/* Kernel-map build that allocates nothing: the same result as
 * spconv_build_submanifold_neighbor_map, but the hash table and order histogram live in a
 * fixed scratch array compiled into this library (a file-scope __device__ array of about
 * 12 MiB, resident on every GPU that loads the library until the process exits), so the
 * caller passes only coords and the outputs.
 *
 * For callers that cannot allocate device memory where the map is built: plugin hosts that
 * hand an operator only its input and output buffers and no allocator, loops whose memory is
 * fixed at start-up and must not call cudaMalloc (it can synchronise the device and can fail
 * under memory pressure), and runtimes whose allocator is not safe to call at that point.
 *
 * Limits and rules:
 *   - num_coords <= SPCONV_NOALLOC_MAX_COORDS; larger inputs return SPCONV_ERR_ARG (use the
 *     workspace entry point for them);
 *   - the first call on a device looks up the scratch array's device address for that device
 *     (cudaGetSymbolAddress, with the stream's device current); make that first call before
 *     any stream capture begins. The address is kept for the life of the process: do not call
 *     this entry point on a device after cudaDeviceReset (or any other teardown of its primary
 *     context) in the same process;
 *   - every call on a device shares the one scratch array and leaves it holding that call's
 *     table; each call clears what it uses first. Calls whose execution overlaps on the GPU
 *     (different streams without ordering, or several host threads) race on the array and
 *     give wrong maps: order them on one stream or synchronise between them.
 * No counterpart in the reference (its table is always allocated by the caller,
 * ops/utils.py:3-16). */
int spconv_build_submanifold_neighbor_map_noalloc(
    const int32_t *coords, int64_t num_coords,
    int batch, int W, int H, int D,
    int Kw, int Kh, int Kd, int Dw, int Dh, int Dd,
    int32_t *neighbor_map, uint32_t *masks, int32_t *order,
    int32_t *status, void *stream);

/* Submanifold conv forward over a kernel map:
 *   out[i, co] = bias[co] + sum_v sum_ci feats[nbr[i,v], ci] * weight[co, v, ci]
 * with fp32 accumulation, rounded once to `dtype` (no atomics, each output row written once).
 *   feats   [M, Ci] in dtype; weight [Co, V, Ci] (= [Co,Kw,Kh,Kd,Ci]) in dtype;
 *   bias    [Co] in dtype or NULL; out [M, Co] in dtype
 *   neighbor_map [M, V] int32 (-1 = missing); masks / order from the map build, or NULL
 *   (NULL masks = every offset treated as active; NULL order = identity)
 * Replaces implicit_gemm.py:59-86 and the EXPLICIT_GEMM forward of ops:76-86. */
int spconv_submanifold_conv_forward(
    const void *feats, int dtype, int64_t num_coords, int Ci,
    const void *weight, const void *bias, int Co, int kernel_volume,
    const int32_t *neighbor_map, const uint32_t *masks, const int32_t *order,
    void *out, int32_t *status, void *stream);

/* As spconv_submanifold_conv_forward, with an explicit kernel choice (SPCONV_KERNEL_*).
 * SPCONV_KERNEL_TCGEN05 returns SPCONV_ERR_UNSUPPORTED for shapes or dtypes it does not
 * cover. Same reference interface as above. */
int spconv_submanifold_conv_forward_ex(
    const void *feats, int dtype, int64_t num_coords, int Ci,
    const void *weight, const void *bias, int Co, int kernel_volume,
    const int32_t *neighbor_map, const uint32_t *masks, const int32_t *order,
    void *out, int32_t *status, void *stream, int kernel_choice);

/* Split-K forward: the same result as spconv_submanifold_conv_forward (within fp32 rounding),
 * with the heaviest tiles' work spread over two CTAs. Of the first 256 tiles of 128 voxels
 * that the tensor-core kernel takes (the end of the voxel order, where the voxels with the most
 * neighbours sort), each one with more than 16 active offsets runs as two halves of its
 * offsets on different CTAs; each half writes fp32 partial rows into `workspace`, and the
 * second half to finish adds the two (fp32 addition of two terms commutes, so results do not
 * vary from run to run) and writes the output. Rows of split tiles therefore round
 * differently from the unsplit kernel's, within the same tolerance. For shapes or dtypes
 * the tensor-core kernel does not cover it runs the ordinary kernel (nothing to split).
 *   workspace: 256-byte aligned, spconv_conv_splitk_workspace_bytes(num_coords, Co) bytes.
 * Replaces the reference's empty IMPLICIT_GEMM_SPLITK / MASKED_IMPLICIT_GEMM_SPLITK slots
 * (ops/submanifold_conv3d.py:13-15, 94-99). */
int64_t spconv_conv_splitk_workspace_bytes(int64_t num_coords, int Co);
int spconv_submanifold_conv_forward_splitk(
    const void *feats, int dtype, int64_t num_coords, int Ci,
    const void *weight, const void *bias, int Co, int kernel_volume,
    const int32_t *neighbor_map, const uint32_t *masks, const int32_t *order,
    void *workspace, int64_t workspace_bytes,
    void *out, int32_t *status, void *stream);

/* Input gradient of the submanifold conv:
 *   grad_in[j, ci] = sum_v sum_co grad_out[nbr_t[j, v], co] * weight_t[ci, v, co]
 * with weight_t[ci, v, co] = weight[co, v, ci] and nbr_t the transposed map. For odd kernel
 * volumes (every side odd, so the offsets are symmetric) nbr_t[j, v] = nbr[j, V-1-v]: the
 * kernels read neighbor_map / masks with the offsets reversed and nbr_t / masks_t may be NULL.
 * Even volumes need nbr_t / masks_t from spconv_transpose_neighbor_map. order: the map
 * build's (any permutation). Replaces the EXPLICIT_GEMM input gradient of
 * ops/submanifold_conv3d.py:117-127. */
int spconv_submanifold_conv_backward_input(
    const void *grad_out, int dtype, int64_t num_coords, int Co, const void *weight_t, int Ci,
    int kernel_volume, const int32_t *neighbor_map, const uint32_t *masks, const int32_t *order,
    const int32_t *neighbor_map_t, const uint32_t *masks_t, void *grad_in,
    int32_t *status, void *stream);

/* Transposed kernel map for the input gradient: neighbor_map_t[j, v] = i where
 * neighbor_map[i, v] = j (at most one such i for distinct coordinates; the largest if the
 * coordinates repeat), -1 if none; masks_t (optional, [M, spconv_mask_words(V)]) its offset
 * masks. For odd kernel sizes this equals the reference's flipped map
 * torch.flip(neighbor_map, [1]) (ops/submanifold_conv3d.py:123-126); for even sizes it is
 * the exact transpose (the flip is not, as the offsets are not symmetric).
 * The input gradient is then spconv_submanifold_conv_forward(grad_out, ..., weight_t, NULL,
 * ..., neighbor_map_t, masks_t, order) with weight_t[ci, v, co] = weight[co, v, ci]. */
int spconv_transpose_neighbor_map(
    const int32_t *neighbor_map, int64_t num_coords, int kernel_volume,
    int32_t *neighbor_map_t, uint32_t *masks_t, int32_t *status, void *stream);

/* Bytes of workspace spconv_submanifold_conv_weight_grad uses for num_coords voxels (tile
 * offset unions and per-offset-group tile lists), or -1 for invalid arguments. */
int64_t spconv_weight_grad_workspace_bytes(int64_t num_coords, int kernel_volume);

/* Weight and bias gradients of the submanifold conv (fp32, overwritten):
 *   grad_weight[co, v, ci] = sum_i grad_out[i, co] * feats[neighbor_map[i, v], ci]
 *   grad_bias[co]          = sum_i grad_out[i, co]           (grad_bias may be NULL)
 * feats [M, Ci] and grad_out [M, Co] in dtype; masks / order (optional) from the map build.
 * 16-bit features with 16/32/64/128 channels run on the tensor cores when a 16-byte aligned
 * workspace of spconv_weight_grad_workspace_bytes() is given: 128-voxel tiles of the order
 * that have no neighbour at an offset are skipped. Other cases run on the CUDA cores.
 * Accumulates with fp32 atomics, so the last bits may differ from run to run.
 * Replaces the EXPLICIT_GEMM weight / bias gradient of ops/submanifold_conv3d.py:132-143. */
int spconv_submanifold_conv_weight_grad(
    const void *feats, const void *grad_out, int dtype, int64_t num_coords, int Ci, int Co,
    int kernel_volume, const int32_t *neighbor_map, const uint32_t *masks, const int32_t *order,
    float *grad_weight, float *grad_bias, void *workspace, int64_t workspace_bytes,
    int32_t *status, void *stream);

/* Stage timing, for profiling and for the benchmark's roofline figures.
 * spconv_stage_timing(max_calls > 0) creates CUDA events on the current device for
 * max_calls calls of each stage and starts recording, on the launch stream, the device
 * time of every stage: the workspace memset, insert_kernel, map_kernel and order_kernel of
 * the map build, and the conv kernel. spconv_stage_timing(0) stops recording and frees the
 * events. spconv_stage_times_ms waits for the recorded events and writes, for the first
 * n stages (SPCONV_STAGE_*), the summed milliseconds and the number of recorded launches;
 * it returns the number of stages written. No reference counterpart (instrumentation). */
#define SPCONV_STAGE_MEMSET 0
#define SPCONV_STAGE_INSERT 1
#define SPCONV_STAGE_MAP 2
#define SPCONV_STAGE_ORDER 3
#define SPCONV_STAGE_CONV 4
#define SPCONV_NUM_STAGES 5

int spconv_stage_timing(int max_calls);
int spconv_stage_times_ms(double *total_ms, int64_t *launches, int n);

#ifdef __cplusplus
}
#endif

#endif /* SPARSECONV_B200_H */
