/*
 * sparsevox -- C ABI of the B200 (sm_100a) sparse-voxel library that replaces
 * mlx_diffuser's TRELLIS sparse-voxel hot path.
 *
 * Every entry point takes plain device pointers and sizes, never a framework type, and
 * enqueues its work on the given CUDA stream (`sv_stream_t` is a `cudaStream_t`). Outputs
 * and scratch ("workspace") are allocated by the caller; the library allocates nothing.
 * Functions return an `sv_status`; on failure `sv_last_error()` (thread-local) describes it.
 * Kernels that can detect a data error at run time (hash table full, neighbour index out of
 * range, a bounded wait that expired) OR a bit into the optional device word `status`.
 *
 * Reference interfaces replaced (paths relative to the mlx_diffuser project root):
 *   src/mlx_diffuser/layers/sparse.py:146-175   build_neighbor_map
 *   src/mlx_diffuser/layers/sparse.py:217-235   SparseConv3D.__call__
 *   src/mlx_diffuser/kernels/sparse.py:58-105   sparse_conv3d (+ the Metal kernel :9-36)
 *   src/mlx_diffuser/layers/sparse.py:245-284   sparse_downsample
 *   src/mlx_diffuser/layers/sparse.py:287-295   sparse_upsample
 *   src/mlx_diffuser/layers/sparse.py:298-318   sparse_subdivide
 *   src/mlx_diffuser/layers/sparse.py:321-342   _attention_groups (sparse_self_attention)
 *   src/mlx_diffuser/models/trellis.py:278-285  occupied_coordinates (np.argwhere step)
 *   src/mlx_diffuser/models/trellis_slat.py:71-82 _SparseResBlock3D norms, modulation, skip add
 */
#ifndef SPARSEVOX_H_
#define SPARSEVOX_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SV_API __attribute__((visibility("default")))
#else
#define SV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef void* sv_stream_t; /* cudaStream_t */

typedef enum sv_status {
  SV_OK = 0,
  SV_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, bad enum value */
  SV_ERR_BAD_SHAPE = 2,        /* shape contract violated (the reference raises ValueError) */
  SV_ERR_BAD_DTYPE = 3,
  SV_ERR_TABLE_FULL = 4,       /* coordinate hash table too small for the input */
  SV_ERR_CUDA = 5,             /* a CUDA runtime/driver call failed */
  SV_ERR_UNSUPPORTED = 6,      /* valid input outside what the library implements */
  SV_ERR_WORKSPACE = 7         /* workspace pointer null or smaller than required */
} sv_status;

typedef enum sv_dtype { SV_FLOAT32 = 0, SV_FLOAT16 = 1, SV_BFLOAT16 = 2 } sv_dtype;

/* Weight layouts accepted by the convolution.
 *  SV_WEIGHT_KIO: (K, Cin, Cout), the view `sparse_conv3d` receives
 *                 (src/mlx_diffuser/kernels/sparse.py:72).
 *  SV_WEIGHT_OKI: (Cout, kD, kH, kW, Cin), spconv's checkpoint layout held by
 *                 `_SparseConv3DCore.weight` (src/mlx_diffuser/layers/sparse.py:178-193). */
typedef enum sv_weight_layout { SV_WEIGHT_KIO = 0, SV_WEIGHT_OKI = 1 } sv_weight_layout;

/* Convolution algorithm. AUTO picks a tcgen05 tensor-core kernel when the shape allows it
 * (Cin and Cout multiples of 32 -- or, for fp16/bf16, 8 or 16 --, K <= 27, 16-byte aligned
 * pointers) -- fp16/bf16 directly,
 * fp32 as 3xTF32 (each operand split into a TF32 high part and an fp32 remainder; three
 * products per K step) -- and the CUDA-core kernel otherwise. */
typedef enum sv_conv_algo { SV_CONV_AUTO = 0, SV_CONV_SIMT = 1, SV_CONV_TCGEN05 = 2 } sv_conv_algo;

/* Bits a kernel ORs into the optional device status word. */
#define SV_DEVICE_TABLE_FULL 0x1    /* an insert gave up after probing every slot */
#define SV_DEVICE_BAD_INDEX 0x2     /* a neighbour / row index out of range, treated as empty */
#define SV_DEVICE_WAIT_TIMEOUT 0x4  /* a bounded in-kernel wait expired; output invalid */

SV_API const char* sv_last_error(void);
SV_API int sv_abi_version(void);

/* ---- kernel map (build_neighbor_map, src/mlx_diffuser/layers/sparse.py:146-175) -------- */

/* Slots of the open-addressing coordinate table used for n rows (a power of two >= 2n). */
SV_API int64_t sv_kmap_table_slots(int64_t n);
/* Workspace bytes for sv_kmap_build with `table_slots` slots (48 bytes per slot: a 3x3x3,
 * dilation-1 map uses a table of 2x2x2 voxel blocks, other kernels a table of voxels). */
SV_API size_t sv_kmap_workspace_bytes(int64_t table_slots);

/* nbr[p, k] = the row of (b, c1+d1, c2+d2, c3+d3), or -1, for the offsets (d1, d2, d3) of a
 * kernel (kernel[0..2] odd) and dilation in the reference's order: offset index
 * k = (a*kernel[1] + b)*kernel[2] + c with d = ((a - kernel[0]/2)*dilation[0], ...), added to
 * coords columns 1, 2, 3. Duplicate coordinate rows resolve to the largest row index.
 * coords: [n, 4] int32 (batch, c1, c2, c3), 16-byte aligned; nbr: [n, kernel volume] int32.
 * The hash table lives in `workspace` (sv_kmap_workspace_bytes(table_slots) bytes). A table
 * with fewer slots than the distinct rows (2x2x2 blocks, for a 3x3x3 map) it has to hold is
 * detected on the device: SV_DEVICE_TABLE_FULL is ORed into `status` (the return value only
 * reports what the host can see). */
SV_API int sv_kmap_build(const int32_t* coords, int64_t n, const int32_t kernel[3],
                         const int32_t dilation[3], int32_t* nbr, int64_t table_slots,
                         void* workspace, size_t workspace_bytes, int32_t* status,
                         sv_stream_t stream);

/* Allocation-free kernel map. No counterpart in mlx_diffuser: it exists for callers that
 * cannot allocate device memory -- e.g. a host program that keeps all GPU memory to itself and
 * does not let plugins call cudaMalloc, or a caller from another language that has only its
 * input and output buffers and no device allocator. Same result as sv_kmap_build, but the hash
 * table is a fixed array inside this library (4 MiB per GPU that loads the library, held until
 * the process exits) instead of caller workspace; nothing is allocated.
 * Limits and rules:
 *  - n <= SV_KMAP_STATIC_MAX_ROWS, otherwise SV_ERR_UNSUPPORTED (with a message) and no work;
 *  - a call outside stream capture looks up the array's device address (cudaGetSymbolAddress),
 *    so it stays valid after the caller resets the device; a call on a capturing stream reuses
 *    the address found by that device's last call outside capture, so make one call on the
 *    device before capturing (and again after a reset);
 *  - all calls on a device share the one table: calls that overlap on the GPU race. Each call
 *    clears the slots it uses before inserting, so back-to-back calls are independent. */
#define SV_KMAP_STATIC_MAX_ROWS 524288
SV_API int sv_kmap_build_static(const int32_t* coords, int64_t n, const int32_t kernel[3],
                                const int32_t dilation[3], int32_t* nbr, int32_t* status,
                                sv_stream_t stream);

/* The same map through a dense grid of row indices over the coordinates' bounding box instead
 * of a hash table: one atomicMax per row, one load per neighbour. lo [4] is the box's minimum
 * (batch, c1, c2, c3) and extent [4] its size (max - min + 1), e.g. from sv_coords_bounds; rows
 * outside the box are not inserted and OR SV_DEVICE_BAD_INDEX into `status`. Workspace:
 * sv_kmap_grid_workspace_bytes(extent) = 4 bytes per cell (0 for an invalid extent). Worth it
 * when the box holds at most a few tens of cells per row. */
/* sv_coords_bounds: bounds_out (host int32 [8]) = min then max of each coords column
 * (synchronises `stream`; 32 bytes of workspace). */
SV_API int sv_coords_bounds(const int32_t* coords, int64_t n, int32_t* bounds_out,
                            void* workspace, size_t workspace_bytes, sv_stream_t stream);
SV_API size_t sv_kmap_grid_workspace_bytes(const int64_t extent[4]);
SV_API int sv_kmap_build_grid(const int32_t* coords, int64_t n, const int32_t kernel[3],
                              const int32_t dilation[3], int32_t* nbr, const int32_t lo[4],
                              const int64_t extent[4], void* workspace, size_t workspace_bytes,
                              int32_t* status, sv_stream_t stream);

/* The same map with the table chosen on the device, no host synchronisation: from 2^17 rows the
 * kernels read the coordinates' bounding box on the GPU and build a dense grid when the box holds
 * at most 16 cells per row (and fits the workspace), the hash table of sv_kmap_build otherwise
 * (sv_kmap_table_slots(n) slots); fewer rows always take the hash table. The map is the same
 * either way. Workspace: sv_kmap_auto_workspace_bytes(n), 16-byte aligned. */
SV_API size_t sv_kmap_auto_workspace_bytes(int64_t n);
SV_API int sv_kmap_build_auto(const int32_t* coords, int64_t n, const int32_t kernel[3],
                              const int32_t dilation[3], int32_t* nbr, void* workspace,
                              size_t workspace_bytes, int32_t* status, sv_stream_t stream);

/* Schedule for the tensor-core convolution, derived from a kernel map:
 *  row_order [n]: a permutation of 0..n-1 that groups rows with equal neighbour-validity masks
 *                 (stable, so rows with one mask keep their spatial order);
 *  tile_order [sv_conv_plan_tiles(n)] (nullable): the 128-row tiles of row_order, the ones
 *                 with the most neighbour offsets first (the convolution starts long work early).
 * Needs kvol <= 32. Workspace: sv_conv_plan_workspace_bytes(n). */
SV_API int64_t sv_conv_plan_tiles(int64_t n);
SV_API size_t sv_conv_plan_workspace_bytes(int64_t n);
SV_API int sv_conv_plan(const int32_t* nbr, int64_t n, int kvol, int32_t* row_order,
                        int32_t* tile_order, void* workspace, size_t workspace_bytes,
                        sv_stream_t stream);

/* ---- convolution (sparse_conv3d / SparseConv3D.__call__) ------------------------------ */

/* out[p, o] = bias[o] + sum_k sum_i features[nbr[p,k], i] * W[k, i, o] over nbr[p,k] >= 0,
 * accumulated in fp32 and rounded once to `dtype` (the Metal kernel's semantics,
 * src/mlx_diffuser/kernels/sparse.py:14-34). features [n, cin], weight in `layout`, bias
 * [cout] (nullable = zero), out [n, cout]; all of `dtype`. row_order and tile_order
 * (nullable) come from sv_conv_plan and only change the schedule, never the result.
 * The tensor-core path needs sv_conv3d_workspace_bytes() of workspace (a scheduler word, plus
 * the repacked weight for a KIO layout); the CUDA-core path needs none (0 bytes, may be null).
 * Calls that share one workspace must not overlap on the GPU. */
SV_API size_t sv_conv3d_workspace_bytes(int64_t n, int cin, int cout, int kvol, int dtype,
                                        int layout, int algo);
SV_API int sv_conv3d_forward(const void* features, int64_t n, int cin, const int32_t* nbr,
                             int kvol, const int32_t* row_order, const int32_t* tile_order,
                             const void* weight, int layout,
                             const void* bias, int cout, int dtype, void* out, int algo,
                             void* workspace, size_t workspace_bytes, int32_t* status,
                             sv_stream_t stream);

/* sv_conv3d_forward plus a residual: out = conv + bias + residual, summed in fp32 and rounded
 * once. residual [n, cout] in `dtype` (nullable = none; 16-byte aligned for the tensor-core
 * path) may be the same buffer as `out` (an in-place add), but must not partially overlap it.
 * It is the `h + skip` of the reference's sparse residual block
 * (src/mlx_diffuser/models/trellis_slat.py:82), folded into the convolution's epilogue. */
SV_API int sv_conv3d_forward_residual(const void* features, int64_t n, int cin,
                                      const int32_t* nbr, int kvol, const int32_t* row_order,
                                      const int32_t* tile_order, const void* weight, int layout,
                                      const void* bias, const void* residual, int cout, int dtype,
                                      void* out, int algo, void* workspace,
                                      size_t workspace_bytes, int32_t* status,
                                      sv_stream_t stream);

/* sv_conv3d_forward_residual over a subset of the output rows: rows [n_rows] lists the rows to
 * compute, in schedule order (e.g. the rows of one partition sorted by sv_conv_plan of their
 * map rows; -1 entries are padding), tile_order (nullable) its 128-row tiles; other rows of
 * `out` are left untouched.
 * Features, map and bounds checks still span all n rows. Used to convolve the rows whose
 * neighbours are all local while a halo exchange is in flight. */
SV_API int sv_conv3d_forward_rows(const void* features, int64_t n, int cin, const int32_t* nbr,
                                  int kvol, const int32_t* rows, int64_t n_rows,
                                  const int32_t* tile_order, const void* weight, int layout,
                                  const void* bias, const void* residual, int cout, int dtype,
                                  void* out, int algo, void* workspace, size_t workspace_bytes,
                                  int32_t* status, sv_stream_t stream);

/* sv_conv3d_forward_rows on the tcgen05 kernel (fp16/bf16, spconv weight layout) for a
 * partitioned scene whose halo rows other GPUs push into `features` (sv_halo_push): the rows
 * list holds the rows that read only local rows first, then -- from tile-order position
 * halo_from_tile on -- the rows that read halo rows (entries -1 pad the first segment to whole
 * 128-row tiles). The first item at or past that position waits, inside the kernel, until each
 * of the flag_count <= 8 flags (this GPU's data flags, raised by sv_halo_signal) is >= epoch
 * (system-scope acquire, at most 1 s per CTA; an expired wait ORs SV_DEVICE_WAIT_TIMEOUT into
 * `status`, marking the output invalid, and the launch still completes). One launch thus
 * overlaps the local rows' convolution with the peers' pushes. Workspace: 256 B. */
SV_API int sv_conv3d_forward_halo(const void* features, int64_t n, int cin, const int32_t* nbr,
                                  int kvol, const int32_t* rows, int64_t n_rows,
                                  const int32_t* tile_order, int32_t halo_from_tile,
                                  int64_t* const* flags, int flag_count, int64_t epoch,
                                  const void* weight, const void* bias, const void* residual,
                                  int cout, int dtype, void* out, void* workspace,
                                  size_t workspace_bytes, int32_t* status, sv_stream_t stream);

/* ---- narrow-channel convolution on deduplicated tiles ---------------------------------------
 * The same convolution as sv_conv3d_forward (the Metal kernel of
 * src/mlx_diffuser/kernels/sparse.py:9-36, reached from SparseConv3D.__call__,
 * src/mlx_diffuser/layers/sparse.py:217-235) for fp16/bf16 3x3x3 convolutions with Cin = 64 or
 * 128 and Cout a multiple of 32. Its tiles are 128 rows adjacent in space (Morton order); each
 * tile's distinct source rows are read from global memory once, into shared memory, and every
 * A operand is assembled from there into tensor memory. Best on surfaces and dense scenes
 * (many neighbours per row); sv_conv3d_forward stays better for very sparse maps.
 *
 * sv_conv_dd_plan builds the tile plan from the coordinates and the kernel map (cache it with
 * the map): `plan` holds sv_conv_dd_plan_bytes(n, cin) bytes, 256-byte aligned, and the build
 * needs sv_conv_dd_plan_workspace_bytes(n) bytes of scratch. sv_conv3d_forward_dd then runs the
 * convolution (weight in the spconv (Cout, 3, 3, 3, Cin) layout; residual optional as in
 * sv_conv3d_forward_residual; 4 bytes of workspace for its scheduler). */
SV_API int sv_conv_dd_supported(int64_t n, int cin, int cout, int kvol, int dtype);
SV_API size_t sv_conv_dd_plan_bytes(int64_t n, int cin);
SV_API size_t sv_conv_dd_plan_workspace_bytes(int64_t n);
SV_API int sv_conv_dd_plan(const int32_t* coords, const int32_t* nbr, int64_t n, int kvol,
                           int cin, void* plan, size_t plan_bytes, void* workspace,
                           size_t workspace_bytes, int32_t* status, sv_stream_t stream);
SV_API int sv_conv3d_forward_dd(const void* features, int64_t n, int cin, const int32_t* nbr,
                                int kvol, const void* plan, size_t plan_bytes,
                                const void* weight, const void* bias, const void* residual,
                                int cout, int dtype, void* out, void* workspace,
                                size_t workspace_bytes, int32_t* status, sv_stream_t stream);

/* Repack a (K, Cin, Cout) weight into spconv's (Cout, K, Cin) layout. */
SV_API int sv_weight_kio_to_oki(const void* w_kio, int kvol, int cin, int cout, int dtype,
                                void* w_oki, sv_stream_t stream);

/* ---- pooling (sparse_downsample / sparse_upsample) ------------------------------------- */

/* Workspace bytes for sv_downsample_coords on n rows. */
SV_API size_t sv_downsample_workspace_bytes(int64_t n);

/* new coords = unique rows of (b, c1 // f, c2 // f, c3 // f) (floor division) in
 * lexicographic signed order, as np.unique(axis=0) returns them
 * (src/mlx_diffuser/layers/sparse.py:250-253); inverse[i] = coarse row of fine row i.
 * Also emits the fine rows grouped by coarse row (sorted_rows [n], stable) and the group
 * boundaries seg_offsets [m + 1], which sv_downsample_features consumes.
 * out_coords must hold n rows. The coarse count m is written to *out_m (host memory); this
 * call synchronises `stream`. */
SV_API int sv_downsample_coords(const int32_t* coords, int64_t n, int factor,
                                int32_t* out_coords, int32_t* inverse, int32_t* sorted_rows,
                                int32_t* seg_offsets, int64_t* out_m, void* workspace,
                                size_t workspace_bytes, sv_stream_t stream);

/* out[j] = (sum of features over the fine rows of coarse row j) / (count_j + 1)
 * (src/mlx_diffuser/layers/sparse.py:254-266); fp32 sums in fine-row order. */
SV_API int sv_downsample_features(const void* features, int64_t n, int channels, int dtype,
                                  const int32_t* sorted_rows, const int32_t* seg_offsets,
                                  int64_t m, void* out, sv_stream_t stream);

/* out[i] = coarse[inverse[i]] (src/mlx_diffuser/layers/sparse.py:295). */
SV_API int sv_upsample_features(const void* coarse, int64_t m, int channels, int dtype,
                                const int32_t* inverse, int64_t n, void* out, int32_t* status,
                                sv_stream_t stream);

/* ---- halo exchange over NVLink peer memory (Morton-partitioned scenes) ---------------- */

/* CUDA IPC: sv_ipc_handle gives the 64-byte handle of the allocation holding `ptr` and ptr's
 * offset in it; a peer process opens it with sv_ipc_open (base address out; add the offset) and
 * releases it with sv_ipc_close(base). */
SV_API int sv_ipc_handle(const void* ptr, void* handle_out, int64_t* offset_out);
SV_API int sv_ipc_open(const void* handle, void** base_out);
SV_API int sv_ipc_close(void* base);

/* Push halo rows: for j < m, row rows[j] of `local` ([local_rows, row_bytes]) is stored into
 * row dst_rows[j] of peer peers[j]'s buffer, whose (IPC-mapped) address is peer_bases[peers[j]]
 * and whose row count is peer_rows[peers[j]] (host arrays of npeers <= 8 entries). rows /
 * dst_rows / peers are device int32 arrays; an index outside its buffer is skipped and
 * SV_DEVICE_BAD_INDEX is ORed into `status`. Each store is followed by a system-scope fence. */
SV_API int sv_halo_push(const void* local, int64_t local_rows, int row_bytes,
                        const int32_t* rows, const int32_t* dst_rows, const int32_t* peers,
                        int64_t m, void* const* peer_bases, const int64_t* peer_rows, int npeers,
                        int32_t* status, sv_stream_t stream);

/* Flags (int64 device words, local or IPC-mapped): sv_halo_signal stores `value` into each of
 * count <= 8 flags with a system-scope release; sv_halo_wait waits on the stream until every
 * flag is >= value (system-scope acquire), for at most 2 s, after which it ORs
 * SV_DEVICE_WAIT_TIMEOUT into `status` and returns. */
SV_API int sv_halo_signal(int64_t* const* flags, int count, int64_t value, sv_stream_t stream);
SV_API int sv_halo_wait(int64_t* const* flags, int count, int64_t value, int32_t* status,
                        sv_stream_t stream);

/* ---- backward (the gradients MLX takes through src/mlx_diffuser/kernels/sparse.py:39-55) -- */

/* Pair lists of a kernel map: for each offset k, the pairs (src = nbr[p, k], dst = p) with
 * nbr[p, k] >= 0, destinations ascending; offsets [kvol + 1] delimit the offsets' runs in
 * pair_src / pair_dst [total]. Two calls on one workspace (sv_kmap_pairs_workspace_bytes):
 * sv_kmap_pairs_count writes the number of pairs to *out_total (host memory; synchronises
 * `stream`); sv_kmap_pairs_emit then fills the lists from the same map. */
SV_API size_t sv_kmap_pairs_workspace_bytes(int64_t n, int kvol);
SV_API int sv_kmap_pairs_count(const int32_t* nbr, int64_t n, int kvol, int64_t* out_total,
                               void* workspace, size_t workspace_bytes, int32_t* status,
                               sv_stream_t stream);
SV_API int sv_kmap_pairs_emit(const int32_t* nbr, int64_t n, int kvol, int32_t* offsets,
                              int32_t* pair_src, int32_t* pair_dst, int64_t total,
                              void* workspace, size_t workspace_bytes, int32_t* status,
                              sv_stream_t stream);

/* Input gradient through the forward convolution: W'[i][j][o] = W[o][K-1-j][i] (spconv layout
 * in and out; w_oki [cout, kvol, cin] -> out [cin, kvol, cout]). For a map with unique
 * coordinates, d features = sv_conv3d_forward(dOut, nbr, W'); nbr[p, k] == q exactly when
 * nbr[q, K-1-k] == p because offset K-1-k negates offset k. */
SV_API int sv_weight_flip_transpose(const void* w_oki, int cout, int kvol, int cin, int dtype,
                                    void* out, sv_stream_t stream);

/* Weight gradient dW[o][k][i] = sum over offset k's pairs of dOut[dst][o] * features[src][i],
 * written in spconv's (Cout, K, Cin) layout in `dtype`, fp32 accumulation, one rounding.
 * features [n, cin], dout [n, cout]; the pair lists come from sv_kmap_pairs_*. AUTO takes the
 * tcgen05 kernel for fp16/bf16 with Cin % 64 == 0 and Cout % 128 == 0 (16-byte aligned), which
 * needs sv_conv3d_wgrad_workspace_bytes() of workspace; otherwise the CUDA-core kernel. */
SV_API size_t sv_conv3d_wgrad_workspace_bytes(int cin, int cout, int kvol, int dtype, int algo);
SV_API int sv_conv3d_wgrad(const void* features, const void* dout, int cin, int cout, int kvol,
                           const int32_t* offsets, const int32_t* pair_src,
                           const int32_t* pair_dst, int dtype, void* dweight, int algo,
                           void* workspace, size_t workspace_bytes, int32_t* status,
                           sv_stream_t stream);

/* Bias gradient: column sums of dout [n, channels] in fp32, in a fixed order (deterministic),
 * rounded to `dtype`. Workspace: sv_conv3d_dbias_workspace_bytes(n, channels). */
SV_API size_t sv_conv3d_dbias_workspace_bytes(int64_t n, int channels);
SV_API int sv_conv3d_dbias(const void* dout, int64_t n, int channels, int dtype, void* dbias,
                           void* workspace, size_t workspace_bytes, sv_stream_t stream);

/* ---- residual-block row normalisation ------------------------------------------------- */

/* out[r] = act(mod(LayerNorm32(x[r]))) per row r of x [n, channels] (even, <= 4096):
 *   LayerNorm32: (x - mean) * rsqrt(mean((x - mean)^2) + eps), fp32, then * weight + bias when
 *     weight [channels] (fp32) is given (src/mlx_diffuser/layers/trellis.py:16-43);
 *   mod: * (1 + scale[b]) + shift[b] when scale / shift (rows of `channels` values in `dtype`,
 *     `mod_stride` elements apart -- e.g. the two halves of one [batch, 2C] projection; 0 =
 *     one row shared by every batch element) are
 *     given, b = coords[r, 0] (the modulation of src/mlx_diffuser/models/trellis_slat.py:79);
 *   act: silu when `silu` is nonzero.
 * Computed in fp32 and rounded once to `dtype`; out may be x (in place). A batch index outside
 * [0, batch) ORs SV_DEVICE_BAD_INDEX into `status` and that row is not modulated. */
SV_API int sv_rownorm(const void* x, int64_t n, int channels, int dtype, float eps,
                      const float* weight, const float* bias, const void* scale,
                      const void* shift, int64_t mod_stride, const int32_t* coords,
                      int64_t batch, int silu, void* out, int32_t* status, sv_stream_t stream);

/* ---- topology: occupancy -> coordinates, subdivision, attention windows --------------- */

/* Coordinates of the cells of a [B, D, H, W] logits grid (element strides `strides`, so a
 * [..., 0] view of a channels-last tensor works) whose value is above `threshold`, as
 * np.argwhere(logits > threshold) lists them (src/mlx_diffuser/models/trellis.py:278-285):
 * (b, d, h, w) int32 rows in row-major order. The threshold is rounded to float32 and then to
 * the logits' dtype before the comparison; NaN is never above it. Two calls on one workspace
 * (sv_occupancy_workspace_bytes(shape) bytes):
 *   sv_occupancy_count writes the number of rows m to *out_m (host memory; synchronises
 *     `stream`) and leaves per-tile offsets in the workspace;
 *   sv_occupancy_emit then writes the m rows to out_coords ([m, 4], 16-byte aligned), with the
 *     same logits, shape, strides and threshold. Rows past m (logits changed in between) are
 *     dropped and SV_DEVICE_BAD_INDEX is ORed into `status`.
 * Grids of up to 2^31 - 1025 cells. */
SV_API size_t sv_occupancy_workspace_bytes(const int64_t shape[4]);
SV_API int sv_occupancy_count(const void* logits, int dtype, const int64_t shape[4],
                              const int64_t strides[4], double threshold, int64_t* out_m,
                              void* workspace, size_t workspace_bytes, sv_stream_t stream);
SV_API int sv_occupancy_emit(const void* logits, int dtype, const int64_t shape[4],
                             const int64_t strides[4], double threshold, int32_t* out_coords,
                             int64_t m, int32_t* status, void* workspace, size_t workspace_bytes,
                             sv_stream_t stream);

/* sparse_subdivide (src/mlx_diffuser/layers/sparse.py:298-318): row i becomes rows 8i + j,
 * j = 4z + 2y + x, with coordinates (b, 2*c1 + z, 2*c2 + y, 2*c3 + x) (int32, wrapping) and a
 * copy of feature row i (row_bytes bytes; features may be null when row_bytes == 0).
 * out_coords [8n, 4], out_features [8n, row_bytes]. */
SV_API int sv_subdivide(const int32_t* coords, int64_t n, const void* features,
                        int64_t row_bytes, int32_t* out_coords, void* out_features,
                        sv_stream_t stream);

/* Attention windows, _attention_groups (src/mlx_diffuser/layers/sparse.py:321-342): rows are
 * grouped by (b, (c1 + shift[0]) // window, (c2 + shift[1]) // window, (c3 + shift[2]) // window)
 * (int32 wrapping addition, floor division), or by b alone when window == 0 (the reference's
 * window_size=None). Groups are listed in the order of their first row, each group's rows
 * ascending -- the order of the reference's dict of lists. perm [n]: the rows, group after
 * group; offsets [G + 1] (allocate n + 1): group g is perm[offsets[g] : offsets[g + 1]].
 * The group count G is written to *out_groups (host memory); this call synchronises `stream`.
 * Workspace: sv_window_groups_workspace_bytes(n). */
SV_API size_t sv_window_groups_workspace_bytes(int64_t n);
SV_API int sv_window_groups(const int32_t* coords, int64_t n, int window, const int32_t shift[3],
                            int32_t* perm, int32_t* offsets, int64_t* out_groups,
                            void* workspace, size_t workspace_bytes, sv_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* SPARSEVOX_H_ */
