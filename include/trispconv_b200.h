/*
 * trispconv_b200 — C ABI of the B200 (sm_100a) sparse-convolution hot path.
 *
 * This library replaces the compute behind the reference's pure-Python
 * `trispconv.pytorch` package (mrpulford/trispconv):
 *   - indice-pair (kernel-map) generation   trispconv/pytorch/indices.py:67-259,
 *                                           trispconv/pytorch/modules.py:175-213
 *   - gather-GEMM-scatter convolution        trispconv/pytorch/functional.py:14-51,
 *                                           trispconv/pytorch/triton_kernels.py:31-135
 *
 * Conventions
 *   - Every pointer argument named *_dev / device buffer is CUDA device memory
 *     allocated by the caller (the Python host uses torch's caching
 *     allocator).  The library holds no device memory of its own, except
 *     the fixed table behind tsc_subm_kmap_noalloc.
 *   - `stream` is a cudaStream_t passed as void*.  All work is enqueued on it;
 *     no entry point synchronises the stream.
 *   - Host-side problems (bad arguments, misaligned pointers, launch failures)
 *     are returned as a TSC_ERR_* code; tsc_last_error() gives the message.
 *   - Problems only the device can see (coordinates outside the grid, a full
 *     hash table) are OR-ed into the caller's int64 status word as
 *     TSC_STATUS_* bits.  The caller checks it at its next synchronisation.
 *   - Coordinates are int32 rows [b, z, y, x] (16-byte rows, the reference's
 *     SparseConvTensor.indices layout, trispconv/pytorch/tensor.py:23-25).
 *   - Kernel offsets are numbered k = (kz*kH + ky)*kW + kx, the reference's
 *     loop order (indices.py:92-94 and the itertools.product at :177).
 *   - Gather maps are k-major int32 arrays map[k][row]; -1 means "no pair".
 */
#ifndef TRISPCONV_B200_H
#define TRISPCONV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TSC_ABI_VERSION 1

#if defined(__GNUC__)
#define TSC_API __attribute__((visibility("default")))
#else
#define TSC_API
#endif

/* Host-side return codes. */
#define TSC_OK                 0
#define TSC_ERR_INVALID_ARG    1
#define TSC_ERR_WORKSPACE      2
#define TSC_ERR_CUDA           3
#define TSC_ERR_UNSUPPORTED    4
#define TSC_ERR_GRID_TOO_LARGE 5

/* Device status bits, OR-ed into the caller's int64 status word. */
#define TSC_STATUS_KEY_RANGE      0x1  /* a coordinate lies outside [0,batch) x spatial_shape */
#define TSC_STATUS_HASH_FULL      0x2  /* open-addressing table ran out of probes */
#define TSC_STATUS_OVERFLOW_FULL  0x4  /* duplicate-pair overflow list ran out of room */
#define TSC_STATUS_WAIT_TIMEOUT   0x8  /* a kernel gave up waiting on one of its own barriers */
#define TSC_STATUS_INTERNAL       0x10 /* a kernel found an out-of-range index in its own shared state and skipped it */

/* Feature / weight element types. */
#define TSC_F32  0
#define TSC_F16  1
#define TSC_BF16 2
#define TSC_F64  3

/* Conv flags. */
#define TSC_CONV_RELU       0x1
#define TSC_CONV_FORCE_SIMT 0x100  /* testing: use the CUDA-core kernel even when a tensor-core one applies */
#define TSC_CONV_USE_TC     0x200  /* use the tcgen05 (TMEM) kernel where it applies */
#define TSC_CONV_TC_SIMPLE  0x400  /* testing: one-tile-per-CTA tcgen05 kernel instead of the persistent one */
#define TSC_CONV_NO_RESIDENT_W 0x800  /* testing: mma.sync kernel without resident weights */
#define TSC_CONV_NO_RG      0x2000 /* testing: skip the register-gather kernel (C_in <= 32 layers then run
                                      on the shared-memory mma.sync kernel) */
#define TSC_CONV_TEST_WAIT_TIMEOUT 0x1000  /* testing: the persistent tcgen05 kernel computes nothing; one
                                              thread waits on a barrier nothing arrives at with a ~0.1 ms
                                              limit, which runs out and sets TSC_STATUS_WAIT_TIMEOUT (the
                                              output is left unwritten) */

/* Activations of the convolution epilogue (tsc_conv_extras.act). */
#define TSC_ACT_NONE       0
#define TSC_ACT_RELU       1  /* same as TSC_CONV_RELU */
#define TSC_ACT_LEAKY_RELU 2  /* x >= 0 ? x : act_alpha * x */
#define TSC_ACT_SILU       3  /* x * sigmoid(x) */

/* Weight layouts accepted by tsc_conv_forward. */
#define TSC_W_KCC  0  /* (K, C_in, C_out): the reference's internal layout (weight.py:36) */
#define TSC_W_KRSC 1  /* (C_out, kD, kH, kW, C_in): spconv KRSC, the modules' parameter */

/* Layout of the per-kernel-map int64 "meta" buffer (length TSC_META_COUNTS + K). */
#define TSC_META_N_OUT      0  /* number of output voxels (strided) */
#define TSC_META_N_PART     1  /* input rows with at least one pair (strided) */
#define TSC_META_N_OVERFLOW 3  /* entries in the duplicate-pair overflow list */
#define TSC_META_STATUS     4  /* snapshot of the status word at the count step */
#define TSC_META_COUNTS     8  /* pair_num[k], k = 0..K-1 */

/* Geometry of one convolution.  For submanifold convs out_shape == in_shape,
 * stride = 1, padding = 0.  Shapes are (D, H, W) = (z, y, x) extents. */
typedef struct tsc_geometry {
  int32_t batch;
  int32_t in_shape[3];
  int32_t out_shape[3];
  int32_t ksize[3];
  int32_t stride[3];
  int32_t padding[3];
  int32_t dilation[3];
} tsc_geometry;

/* ---- introspection -------------------------------------------------------- */
TSC_API int tsc_abi_version(void);
TSC_API const char* tsc_last_error(void);
/* Number of CUDA kernels this library has launched in this process. */
TSC_API unsigned long long tsc_launch_count(void);

/* ---- submanifold kernel map ----------------------------------------------
 * Replaces generate_subm_indice_pairs (indices.py:67-140) and its dense
 * B*D*H*W lookup table (_build_hash_table, indices.py:54-64) with an
 * open-addressing hash of packed (b,z,y,x) keys.
 *
 * gather_map[k][i] = row j whose coordinate equals coord(i) + (k - K//2)*d,
 * or -1.  With duplicate coordinates j is the LAST such row (the reference's
 * `table[encoded] = arange` write order).  meta[TSC_META_COUNTS + k] receives
 * pair_num[k].  Keys are 32-bit up to batch*D*H*W = 2^32 - 2 cells and
 * 64-bit above (the reference's int64 key, indices.py:45-51), up to 2^62
 * cells; tsc_subm_kmap_workspace covers both.  The hash takes 2^ceil(log2 8n)
 * slots when the workspace holds them (tsc_subm_kmap_workspace's size), and
 * at least 2^ceil(log2 2n): a smaller workspace fails with TSC_ERR_WORKSPACE. */
TSC_API size_t tsc_subm_kmap_workspace(int64_t n);
TSC_API int tsc_subm_kmap(const int32_t* indices, int64_t n, const tsc_geometry* geo,
                  void* workspace, size_t workspace_bytes,
                  int32_t* gather_map, int64_t* meta, int64_t* status, void* stream);

/* Direct-address variant: the same map as tsc_subm_kmap from a caller-held
 * int32 table of at least batch*D*H*W cells (table_cells) indexed by the
 * packed key, which must hold -1 in every cell on entry and holds -1 again
 * when the call's work has run (the call writes the cells of its voxels, reads
 * the neighbours' cells and clears its cells).  The reference builds the same
 * kind of table (int64, filled anew per call, indices.py:54-64); keeping it
 * all -1 between calls makes a build cost O(n) instead of O(cells).  Calls
 * sharing a table must be serialised on one stream. */
TSC_API int tsc_subm_kmap_dense(const int32_t* indices, int64_t n, const tsc_geometry* geo,
                  int32_t* table, int64_t table_cells,
                  int32_t* gather_map, int64_t* meta, int64_t* status, void* stream);

/* Rank variant: the same map as tsc_subm_kmap for `indices` that are the
 * output coordinates of a strided map over this grid (the out_indices of
 * tsc_strided_kmap_emit, unchanged), taken from that map's workspace after
 * its emit step: a cell's row is the rank of its bit in the occupancy
 * bitmap, so no table is built or cleared.  geo is the submanifold geometry
 * (in_shape == the strided map's out_shape, same batch); strided_workspace
 * and workspace_bytes are that strided map's.  Any grid up to 2^62 cells. */
TSC_API int tsc_subm_kmap_ranked(const int32_t* indices, int64_t n, const tsc_geometry* geo,
                  const void* strided_workspace, size_t workspace_bytes,
                  int32_t* gather_map, int64_t* meta, int64_t* status, void* stream);

/* ---- strided kernel map --------------------------------------------------
 * Replaces generate_strided_indice_pairs (indices.py:143-259).  The output
 * set is found with an occupancy bitmap over the output grid (1 bit per
 * cell) and a prefix popcount, which yields the reference's
 * `torch.unique(sorted=True)` order (:219-220) without a sort.  Bitmap
 * positions are 32-bit up to 2^32 - 2 output cells and 64-bit above, up to
 * 2^62 output cells (the bitmap takes batch*D*H*W/8 bytes of workspace).
 *
 * Step 1 (count): marks the bitmap, counts pairs per offset and the
 * participating input rows, and writes meta[N_OUT], meta[N_PART] and
 * meta[STATUS].  The caller reads meta to size the outputs of step 2.
 * Step 2 (emit): writes the sorted output coordinates, the output-stationary
 * gather map gather_map[k][o] (-1 prefilled by this call), the
 * input-stationary scatter map scatter_map[k][i] = o or -1, and, for
 * duplicate input coordinates only, (k, o, i) triples that did not fit the
 * gather map into `overflow` (capacity overflow_cap triples; count in
 * meta[N_OVERFLOW]).  The same workspace must be passed to both steps. */
TSC_API size_t tsc_strided_kmap_workspace(const tsc_geometry* geo);
TSC_API int tsc_strided_kmap_count(const int32_t* indices, int64_t n_in, const tsc_geometry* geo,
                           void* workspace, size_t workspace_bytes,
                           int64_t* meta, int64_t* status, void* stream);
/* Step 1 with the counts also delivered to the host: the last count kernel
 * copies meta[0 .. TSC_META_COUNTS + K) into host_meta, page-locked host
 * memory the device can address (cudaHostAlloc / pinned tensors); other
 * host memory gets an ordinary asynchronous copy on `stream`.  The caller
 * waits on an event recorded after this call instead of copying meta back,
 * which keeps the copy engine out of the stream. */
TSC_API int tsc_strided_kmap_count_host(const int32_t* indices, int64_t n_in, const tsc_geometry* geo,
                           void* workspace, size_t workspace_bytes,
                           int64_t* meta, int64_t* host_meta, int64_t* status, void* stream);
TSC_API int tsc_strided_kmap_emit(const int32_t* indices, int64_t n_in, const tsc_geometry* geo,
                          void* workspace, size_t workspace_bytes, int64_t n_out,
                          int32_t* out_indices, int32_t* gather_map, int32_t* scatter_map,
                          int32_t* overflow, int64_t overflow_cap,
                          int64_t* meta, int64_t* status, void* stream);

/* ---- inverse kernel maps -------------------------------------------------
 * Replace the pair swap of SparseInverseConvolution (modules.py:175-213).
 *
 * From a strided forward map: keeps the forward-input rows that have at
 * least one pair (ascending row order, modules.py:178-182), writes their
 * coordinates to out_indices[n_part][4], the inverse gather map
 * inv_gather[k][r] = scatter_map[k][row_r], and compact[i] = r or -1.  When
 * n_part == n_in the gather map is the scatter map itself; pass
 * inv_gather == scatter_map to skip the copy. */
TSC_API size_t tsc_inverse_kmap_workspace(int64_t n_in);
TSC_API int tsc_inverse_kmap_strided(const int32_t* in_indices, int64_t n_in,
                             const int32_t* scatter_map, int32_t k_vol, int64_t n_part,
                             void* workspace, size_t workspace_bytes,
                             int32_t* out_indices, int32_t* inv_gather, int32_t* compact,
                             int64_t* status, void* stream);

/* From a submanifold forward map (an inverse conv keyed on a SubM
 * indice_key).  Step 1 flags every row that some pair reads, compacts them
 * and writes meta[N_PART].  Step 2 writes out_indices, the transposed gather
 * map inv_gather[k][compact[j]] = i for gather_map[k][i] = j, and duplicate
 * overflow triples as in tsc_strided_kmap_emit. */
TSC_API int tsc_inverse_kmap_subm_count(const int32_t* gather_map, int32_t k_vol, int64_t n,
                                void* workspace, size_t workspace_bytes,
                                int32_t* compact, int64_t* meta, int64_t* status, void* stream);
TSC_API int tsc_inverse_kmap_subm_emit(const int32_t* in_indices, const int32_t* gather_map,
                               int32_t k_vol, int64_t n, const int32_t* compact, int64_t n_part,
                               int32_t* out_indices, int32_t* inv_gather,
                               int32_t* overflow, int64_t overflow_cap,
                               int64_t* meta, int64_t* status, void* stream);

/* ---- pair lists in the reference's order ---------------------------------
 * Materialises IndiceData.pairs_in / pairs_out (K lists of int64) as two
 * flat int64 arrays of length sum(pair_num), k-major, from a map[k][idx]:
 *   mode 0: for each k, idx ascending with map >= 0: in = map, out = idx
 *           (submanifold, indices.py:123-124; inverse of strided)
 *   mode 1: for each k, idx ascending with map >= 0: in = idx,
 *           out = remap ? remap[map] : map
 *           (strided, indices.py:235-240; inverse of submanifold)
 * `capacity` is the length of pairs_in / pairs_out (sum of pair_num); no
 * write goes past it. */
TSC_API size_t tsc_pairs_workspace(int32_t k_vol, int64_t n);
TSC_API int tsc_pairs_materialize(const int32_t* map, int32_t k_vol, int64_t n, int32_t mode,
                          const int32_t* remap, int64_t* pairs_in, int64_t* pairs_out,
                          int64_t capacity, void* workspace, size_t workspace_bytes,
                          int64_t* status, void* stream);

/* Builds a gather map (and duplicate overflow) from explicit pair lists, for
 * IndiceData objects a user built by hand.  pairs are flat int64 arrays with
 * per-offset offsets offsets[k]..offsets[k+1] (host array, K+1 entries). */
TSC_API int tsc_gather_from_pairs(const int64_t* pairs_in, const int64_t* pairs_out,
                          const int64_t* offsets_host, int32_t k_vol, int64_t n_out,
                          int32_t* gather_map, int32_t* overflow, int64_t overflow_cap,
                          int64_t* meta, int64_t* status, void* stream);

/* ---- convolution ----------------------------------------------------------
 * Output-stationary implicit GEMM replacing sparse_conv_forward
 * (functional.py:14-51):
 *   out[o, :] = sum_k features[gather_map[k][o], :] @ weight[k]  (+ bias, ReLU)
 * in k order, fp32 accumulation, one store per output row, no atomics.
 * features [n_in][c_in], weight (layout TSC_W_KCC or TSC_W_KRSC), bias
 * [c_out] (or NULL) and out [n_out][c_out] all share `dtype`.  Reading the
 * KRSC parameter in place replaces normalize_spconv_weight (weight.py:8-50)
 * for K > 1; the 1x1x1 quirk (weight.py:29-34) is the same storage read as
 * TSC_W_KCC.  gather_map NULL means the identity map
 * (K == 1, n_in == n_out: the inverse 1x1x1 path, modules.py:162-173).
 * overflow (capacity overflow_cap triples) and meta carry the
 * duplicate-coordinate pairs of the kernel-map builders; the kernel reads
 * their count from meta[TSC_META_N_OVERFLOW] on the device.  Pass NULL when
 * the map cannot have any (submanifold maps).  row_order (NULL = identity)
 * is a permutation of [0, n_out) giving the order in which output rows are
 * grouped into tiles; results do not depend on it (an entry outside
 * [0, n_out) sets TSC_STATUS_INTERNAL and no row is written for it).
 * Kernels, for 16-bit dtypes with KRSC weights: with TSC_CONV_USE_TC,
 * layers with C_in % 64 == 0, C_out % 32 == 0 and K <= 27 run on the
 * persistent tcgen05/TMEM kernel; C_in in {4, 8} with C_out in {16, 32, 64},
 * or C_in in {16, 32} with C_out in {16, 32} (K <= 64), on the
 * register-gather mma.sync kernel (TSC_CONV_NO_RG: not); other shapes with
 * C_in % 8 == 0 (or C_in % 4 == 0 and C_in <= 16), C_out % 8 == 0 and
 * K <= 64 on the shared-memory mma.sync kernel.  Everything else runs on the
 * CUDA cores.  tile_counter (NULL allowed) is one device uint32 through which the
 * persistent kernel's CTAs take tiles dynamically (the call zeroes it on
 * `stream`); calls that may run concurrently need distinct counters.  With
 * NULL, tiles are dealt round robin. */
TSC_API int tsc_conv_forward(const void* features, int32_t dtype, int64_t n_in, int32_t c_in,
                     const void* weight, int32_t weight_layout, const void* bias,
                     const int32_t* gather_map, const int32_t* row_order,
                     int32_t k_vol, int64_t n_out, int32_t c_out,
                     const int32_t* overflow, int64_t overflow_cap, const int64_t* meta,
                     void* out, int32_t flags, int64_t* status, uint32_t* tile_counter, void* stream);

/* ---- per-plane input halos for the convolution ----------------------------
 * No counterpart in the reference (its CPU path has no tiles): a faster
 * variant of tsc_conv_forward for 16-bit 3x3x3 layers with 64 input and 64
 * or 128 output channels on maps whose output rows are spatially ordered
 * (the outputs of a strided map and the submanifold maps built on them).
 * The persistent tcgen05 kernel computes tiles of TSC_HALO_TILE_ROWS
 * consecutive output rows.  A plane is one kz of the kernel (offsets
 * k = p*kH*kW .. +kH*kW-1); the sub-halo of (tile, plane) lists the distinct
 * input rows the plane's pairs of the tile read, ascending.  The kernel
 * loads each sub-halo once into shared memory (TMA gather4) and builds the A
 * operand of every pair from it in tensor memory, instead of fetching an
 * input row from L2 once per pair.  Results are identical with and without
 * halos (same pairs, same offset order, same fp32 accumulation).
 *   tsc_conv_halo_capacity: rows per (tile, plane) sub-halo the halo kernel
 *     holds for this layer (dtype, c_in, c_out, K, conv flags), or 0 when it
 *     does not apply.
 *   tsc_tile_halo: from a k-major gather map [k_vol][n_out] (K <= 32,
 *     `planes` dividing K) writes, per tile t = o / TSC_HALO_TILE_ROWS and
 *     plane p, halo_rows[t][p][capacity] (16-byte aligned; the first
 *     halo_count[t][p] entries, padded to a multiple of 4 with copies of the
 *     last), plane_kmask[t][p] (bit k set when offset k of the plane has a
 *     pair in the tile) and halo_map [k_vol][n_out] int16: the position of
 *     gather_map[k][o] in its (tile, plane) list, -1 for no pair, -2 for a
 *     row beyond the capacity or a plane whose rows span more than 65536
 *     rows (read from the gather map instead).
 *   The convolution takes the halo buffers through tsc_conv_forward_ex
 *     (below).  Layers the halo kernel does not take (or a row_order, or an
 *     overflow list) run as in tsc_conv_forward. */
#define TSC_HALO_TILE_ROWS 256
TSC_API int32_t tsc_conv_halo_capacity(int32_t dtype, int32_t c_in, int32_t c_out, int32_t k_vol, int32_t flags);
TSC_API int tsc_tile_halo(const int32_t* gather_map, int32_t k_vol, int32_t planes, int64_t n_in, int64_t n_out,
                  int32_t capacity, int32_t* halo_rows, int32_t* halo_count, uint32_t* plane_kmask,
                  int16_t* halo_map, int64_t* status, void* stream);

/* ---- convolution with extras -------------------------------------------------
 * tsc_conv_forward plus optional extras (extras NULL or zero-filled = none):
 *   epilogue  scale/shift (float [c_out] each, or NULL): the store becomes
 *             act(acc * scale[n] + shift[n]) in fp32, rounded once; the
 *             `bias` argument is then ignored (fold it into shift).  This is
 *             an eval-mode BatchNorm1d on the features fused into the
 *             convolution: scale = gamma / sqrt(running_var + eps), shift =
 *             beta + (bias - running_mean) * scale.  The reference applies it
 *             as a separate module over x.features (modules.py:320-329).
 *             act: TSC_ACT_* (TSC_CONV_RELU in flags also selects ReLU),
 *             act_alpha the LeakyReLU slope.
 *   halos     the four tsc_tile_halo buffers with halo_planes == 3 and
 *             halo_capacity == tsc_conv_halo_capacity of the layer (see
 *             above); NULL halo_map = none. */
typedef struct tsc_conv_extras {
  const float* scale;
  const float* shift;
  int32_t act;
  float act_alpha;
  const int32_t* halo_rows;
  const int32_t* halo_count;
  const uint32_t* plane_kmask;
  const int16_t* halo_map;
  int32_t halo_planes;
  int32_t halo_capacity;
} tsc_conv_extras;
TSC_API int tsc_conv_forward_ex(const void* features, int32_t dtype, int64_t n_in, int32_t c_in,
                     const void* weight, int32_t weight_layout, const void* bias,
                     const int32_t* gather_map, const int32_t* row_order,
                     int32_t k_vol, int64_t n_out, int32_t c_out,
                     const int32_t* overflow, int64_t overflow_cap, const int64_t* meta,
                     void* out, int32_t flags, int64_t* status, uint32_t* tile_counter,
                     const tsc_conv_extras* extras, void* stream);

/* ---- dense scatter ---------------------------------------------------------
 * SparseConvTensor.dense() (tensor.py:72-99): writes features into a zeroed
 * (B, C, D, H, W) (channels_first = 1) or (B, D, H, W, C) tensor.  Rows with
 * coordinates outside the grid set TSC_STATUS_KEY_RANGE and are skipped. */
TSC_API int tsc_to_dense(const void* features, int32_t dtype, const int32_t* indices, int64_t n, int32_t c,
                 int32_t batch, const int32_t* shape3, int32_t channels_first,
                 void* out, int64_t* status, void* stream);

/* ---- row order for the convolution kernels --------------------------------
 * No counterpart in the reference (its CPU path has no tiles).  Groups the
 * output rows of a gather map by neighbour mask (bit k set when
 * gather_map[k][o] >= 0), masks ascending, so that the rows of a conv tile
 * share their kernel offsets; writes a permutation of [0, n_out) to
 * row_order, to be passed to tsc_conv_forward.  Convolution results do not
 * depend on it.  1 <= K <= 32.  More than 16384 distinct masks, or a mask
 * that finds no table slot within 128 probes, leave the identity order. */
TSC_API size_t tsc_row_order_workspace(int64_t n_out);
TSC_API int tsc_row_order(const int32_t* gather_map, int32_t k_vol, int64_t n_out, void* workspace,
                  size_t workspace_bytes, int32_t* row_order, int64_t* status, void* stream);

/* ---- voxelisation: points -> unique voxels ----------------------------------
 * No counterpart in the reference (its SparseConvTensor takes voxels that
 * the user built, trispconv/pytorch/tensor.py:12-22): the step before the
 * sparse convolutions.  points is float32 [n][point_dim] with columns x, y,
 * z and then point_dim-3 features; batch_ids int32 [n] (NULL: all 0).  A
 * point lies in voxel v_d = floor((p_d - range_lo_d) / voxel_size_d) for
 * d = x, y, z (float32 arithmetic, IEEE division) and is kept when
 * 0 <= v_x < W, 0 <= v_y < H, 0 <= v_z < D and 0 <= b < batch; the others
 * are dropped (a batch id outside [0, batch) also sets TSC_STATUS_KEY_RANGE).
 * Voxels come out sorted by their (b, z, y, x) key, the order strided maps
 * produce, found with an occupancy bitmap over the batch*D*H*W grid (keys
 * 64-bit above 2^32 - 2 cells).  A voxel's features are the mean of
 * point_dim columns over its kept points: the max_points points of smallest
 * index (all when max_points <= 0), summed in ascending index order in fp32.
 * Step 1 (count) writes meta[TSC_META_N_OUT] = voxels and
 * meta[TSC_META_N_PART] = points inside the range; step 2 (emit), with the
 * same workspace, writes coords [n_vox][4] (b, z, y, x), features
 * [n_vox][point_dim] and num_points [n_vox] (kept points per voxel). */
typedef struct tsc_voxel_params {
  int32_t batch;
  int32_t grid[3];      /* (D, H, W): voxels along z, y, x */
  float range_lo[3];    /* x, y, z of the grid's lower corner */
  float voxel_size[3];  /* x, y, z voxel extent */
  int32_t max_points;   /* points kept per voxel; <= 0 keeps all */
} tsc_voxel_params;
TSC_API size_t tsc_voxelize_workspace(const tsc_voxel_params* vp, int64_t n_points);
TSC_API int tsc_voxelize_count(const float* points, int64_t n, int32_t point_dim, const int32_t* batch_ids,
                       const tsc_voxel_params* vp, void* workspace, size_t workspace_bytes,
                       int64_t* meta, int64_t* status, void* stream);
TSC_API int tsc_voxelize_emit(const float* points, int64_t n, int32_t point_dim, const int32_t* batch_ids,
                      const tsc_voxel_params* vp, void* workspace, size_t workspace_bytes, int64_t n_vox,
                      int32_t* coords, float* features, int32_t* num_points, int64_t* meta, int64_t* status,
                      void* stream);

/* ---- allocation-free submanifold kernel map ------------------------------
 * No counterpart in the reference: an addition for callers that cannot
 * allocate device memory when they build a map (a host that owns a fixed
 * memory budget or pool, code that must not let cudaMalloc/cudaFree
 * synchronise the device, bindings without a device allocator).  Same result
 * as tsc_subm_kmap, but its hash table lives in a fixed 16 MiB device array
 * inside this library (held on every GPU that loads the library until the
 * process exits) instead of a caller workspace; it calls no allocator.
 *   - n must not exceed tsc_subm_kmap_noalloc_max_voxels() (2^20); larger
 *     inputs fail with TSC_ERR_WORKSPACE and a message naming the limit.
 *     Grids above 2^32 - 2 cells (64-bit keys) fail with
 *     TSC_ERR_GRID_TOO_LARGE; use tsc_subm_kmap for them.
 *   - The first call on each device looks up the array's device address
 *     (cudaGetSymbolAddress); make that first call before any stream capture.
 *   - The current device must be the one that owns `stream` (the array's
 *     address is per device); otherwise the call returns
 *     TSC_ERR_UNSUPPORTED.
 *   - The launches are those of tsc_subm_kmap (one fill kernel for meta and
 *     the table, then the build and the query).
 *   - All calls on a device share the one array: calls whose work overlaps
 *     on the GPU (different streams, or threads) race and give wrong maps;
 *     serialise them.  Each call clears the part of the table it uses. */
TSC_API int64_t tsc_subm_kmap_noalloc_max_voxels(void);
TSC_API int tsc_subm_kmap_noalloc(const int32_t* indices, int64_t n, const tsc_geometry* geo,
                          int32_t* gather_map, int64_t* meta, int64_t* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TRISPCONV_B200_H */
