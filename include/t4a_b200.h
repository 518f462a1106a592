/*
 * t4a_b200: B200-native (sm_100a) implementation of the t4a-cuda-kernels hot path.
 *
 * C ABI of the host library libt4a_b200.so.  It replaces two reference interfaces:
 *
 *  1. The Rust planner `t4a_cuda_kernels::plan_*` (reference src/lib.rs), restated
 *     here as `t4a_plan_*`: the same inputs, the same validation and the same
 *     error codes (the order of the Rust `Error` enum, src/lib.rs:219-280, plus one),
 *     returning the launch geometry of this library's kernels.
 *  2. The caller's `cuLaunchKernel` on a module symbol (reference
 *     tests/gpu/mod.rs:297-331): `t4a_launch_*` takes the planned `t4a_launch`, the
 *     caller's stream and exactly the argument list of the kernel symbol it stands
 *     for (docs/abi/c-kernel-abi.md entry tables), and launches it.
 *
 * The modules lib/{reduce,movement,gather_scatter,rrqr,linalg_aux}.cubin built beside
 * the library export the same
 * `extern "C" __global__` symbols as the reference (t4a_cuda_reduce, ...), for
 * callers that load kernels by name.
 *
 * Ownership is the reference's: the caller owns streams, device buffers and
 * workspace; nothing here allocates device memory, frees it or synchronizes
 * (t4a_reduce's workspace is caller-provided too).  Every function returns a
 * t4a_status code.  `stream` is a cudaStream_t (NULL = legacy default stream).
 */
#ifndef T4A_B200_H_
#define T4A_B200_H_

#include <stddef.h>

#include "t4a_b200/abi.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes: 0 = success; 1..25 = the reference planner's Error variants in
 * declaration order (src/lib.rs:219-270, the fusion-only variants excluded);
 * 64.. = runtime conditions of this library. */
typedef enum {
  T4A_OK = 0,
  T4A_ERR_RANK_OUT_OF_RANGE = 1,
  T4A_ERR_RANK_LENGTH = 2,
  T4A_ERR_NEGATIVE_EXTENT = 3,
  T4A_ERR_NEGATIVE_COUNT = 4,
  T4A_ERR_OVERFLOW = 5,
  T4A_ERR_COUNT_MISMATCH = 6,
  T4A_ERR_OFFSET_OUT_OF_SPAN = 7,
  T4A_ERR_BROADCAST_DESTINATION = 8,
  T4A_ERR_UNSUPPORTED_DTYPE = 9,
  T4A_ERR_NOT_ELEMENTWISE = 10,
  T4A_ERR_LAUNCH_LIMIT = 11,
  T4A_ERR_INVALID_TRANSPOSE_CONFIG = 12,
  T4A_ERR_INVALID_AXIS = 13,
  T4A_ERR_DUPLICATE_AXIS = 14,
  T4A_ERR_NOT_COMPACT = 15,
  T4A_ERR_SHAPE_MISMATCH = 16,
  T4A_ERR_INVALID_STEP = 17,
  T4A_ERR_INVALID_PADDING = 18,
  T4A_ERR_DOMAIN_TOO_LARGE = 19,
  T4A_ERR_INVALID_STRIDE = 20,
  T4A_ERR_STRATEGY_MISMATCH = 21,
  T4A_ERR_INVALID_PLANE_WIDTH = 22,
  T4A_ERR_INVALID_SPLIT = 23,
  T4A_ERR_INDEX_VECTOR_MISMATCH = 24,
  T4A_ERR_UNSUPPORTED_OP = 25,
  T4A_ERR_CUDA = 64,          /* a CUDA runtime call failed (launch or copy) */
  T4A_ERR_WORKSPACE = 65,     /* caller workspace missing or too small */
  T4A_ERR_NULL_ARGUMENT = 66  /* a required pointer argument is NULL */
} t4a_status;

/* Launch geometry of one kernel invocation (reference `Launch`, src/lib.rs:842-848).
 * `variant` names the kernel path this library chose; a grid with a zero
 * dimension means "no work" and the launchers skip it. */
typedef struct {
  unsigned grid[3];
  unsigned block[3];
  unsigned shared_bytes;
  int variant;
} t4a_launch;

const char* t4a_status_string(int status);
int t4a_abi_revision(void);
/* Last CUDA error seen by a launcher of this thread (cudaError_t), 0 if none. */
int t4a_last_cuda_error(void);

/* ------------------------------------------------------------------------- */
/* Single-axis reductions (reference src/lib.rs:3033-3557, reduce.cu:765-852)  */
/* ------------------------------------------------------------------------- */

typedef struct {
  long long splits;
  long long chunk_len;
} t4a_split;

/* Reference ReductionPlan (src/lib.rs:3170-3182): a direct pass, or pass 1 over
 * `split` chunks plus a combine pass with `combine_op`. */
typedef struct {
  int is_split;
  int strategy;
  t4a_launch launch;
  t4a_split split;
  t4a_launch pass1;
  int combine_strategy;
  int combine_op;
  t4a_launch pass2;
} t4a_reduction_plan;

/* split_policy (src/lib.rs:3152): splits = clamp(len / (W*8), 1, 4096), floor
 * chunk; *has_split = 0 means one direct pass. */
int t4a_split_policy(long long reduce_len, unsigned plane_width, int* has_split, t4a_split* split);

/* plan_reduce (src/lib.rs:3318). */
int t4a_plan_reduce(int dtype, int op, int strategy, const t4a_cuda_layout* out, long long out_len,
                    const t4a_cuda_layout* in, long long in_len, unsigned axis, unsigned plane_width,
                    t4a_launch* launch);

/* plan_reduce_partials (src/lib.rs:3342). */
int t4a_plan_reduce_partials(int dtype, int op, const t4a_cuda_layout* partials, long long partials_len,
                             const t4a_cuda_layout* in, long long in_len, unsigned axis,
                             t4a_split split, unsigned plane_width, t4a_launch* launch);

/* plan_reduction (src/lib.rs:3457): the whole Auto policy. */
int t4a_plan_reduction(int dtype, int op, const t4a_cuda_layout* out, long long out_len,
                       const t4a_cuda_layout* in, long long in_len, unsigned axis,
                       unsigned plane_width, t4a_reduction_plan* plan);

/* reduction_partials_layout (src/lib.rs:3535): the input extents with the axis set
 * to `splits`, compact. */
int t4a_reduction_partials_layout(const t4a_cuda_layout* in, unsigned axis, long long splits,
                                  t4a_cuda_layout* partials);

/* Launch t4a_cuda_reduce (reduce.cu:765) / t4a_cuda_reduce_partials (reduce.cu:813)
 * with a planned geometry on `stream`. */
int t4a_launch_reduce(const t4a_launch* launch, void* stream, void* out, const void* in, int dtype,
                      int op, int strategy, t4a_cuda_layout out_layout, t4a_cuda_layout in_layout,
                      int axis, long long output_len);
int t4a_launch_reduce_partials(const t4a_launch* launch, void* stream, void* partials, const void* in,
                               int dtype, int op, t4a_cuda_layout partials_layout,
                               t4a_cuda_layout in_layout, int axis, long long output_len,
                               long long splits, long long chunk_len);

/* Workspace bytes of t4a_reduce (the pass-1 partials; 0 for a direct pass). */
int t4a_reduce_workspace_bytes(int dtype, int op, const t4a_cuda_layout* out, long long out_len,
                               const t4a_cuda_layout* in, long long in_len, unsigned axis,
                               unsigned plane_width, size_t* bytes);

/* One call for a whole reduction: plans, then launches pass 1 and the combine pass
 * (or the direct pass) on `stream`, partials in the caller's `workspace`. */
int t4a_reduce(void* stream, int dtype, int op, void* out, const t4a_cuda_layout* out_layout,
               long long out_len, const void* in, const t4a_cuda_layout* in_layout, long long in_len,
               unsigned axis, unsigned plane_width, void* workspace, size_t workspace_bytes);

/* Bytes of device memory the library keeps per GPU for t4a_reduce_noalloc. */
#define T4A_REDUCE_NOALLOC_SCRATCH_BYTES (16u << 20)

/* No counterpart in the reference.  t4a_reduce for callers that cannot allocate
 * device memory or hand over a workspace: the pass-1 partials go to an array of
 * T4A_REDUCE_NOALLOC_SCRATCH_BYTES that the library's module holds on every GPU that
 * loads it.  Allocates nothing.  Returns T4A_ERR_WORKSPACE when the partials would
 * not fit that array.  The first call on a device looks the array up (make it before
 * any stream capture) and caches its address for the life of the process: after a
 * cudaDeviceReset of a device, do not call it on that device again.  All calls on a
 * device share the array, so calls that may overlap on the GPU race on it. */
int t4a_reduce_noalloc(void* stream, int dtype, int op, void* out, const t4a_cuda_layout* out_layout,
                       long long out_len, const void* in, const t4a_cuda_layout* in_layout, long long in_len,
                       unsigned axis, unsigned plane_width);

/* General-rank reductions, the `_any` twins (reference cuda/src/reduce.cu:854, :902;
 * module symbols t4a_cuda_reduce_any / t4a_cuda_reduce_partials_any in reduce.cubin):
 * the same folds as t4a_launch_reduce / t4a_launch_reduce_partials, with the layouts'
 * extents and strides in device memory, so any rank works.  The launchers take the
 * kernels' argument lists; any geometry is correct, and t4a_reduce_any_geometry gives
 * the one they are tuned for (UNIT: a thread per output; PLANE: planes of w lanes,
 * w in {8, 16, 32}, or one block of w in {64 .. 512} per output for a direct pass).
 * The host checks what it can without device access (layout rank and reserved field,
 * NULL arrays, axis, split); extents and strides are the caller's, as in the reference. */
int t4a_reduce_any_geometry(int strategy, unsigned plane_width, long long output_len, long long splits,
                            t4a_launch* launch);
int t4a_launch_reduce_any(const t4a_launch* launch, void* stream, void* out, const void* in, int dtype, int op,
                          int strategy, t4a_cuda_layout_any out_layout, t4a_cuda_layout_any in_layout, int axis,
                          long long output_len);
int t4a_launch_reduce_partials_any(const t4a_launch* launch, void* stream, void* partials, const void* in,
                                   int dtype, int op, t4a_cuda_layout_any partials_layout,
                                   t4a_cuda_layout_any in_layout, int axis, long long output_len, long long splits,
                                   long long chunk_len);


/* ------------------------------------------------------------------------- */
/* Strided movement (reference src/lib.rs:1465-1737, movement.cu:514-656)      */
/* Every planner validates like its reference counterpart; the launch carries  */
/* this library's path (variant 32 + kind) and geometry.                        */
/* ------------------------------------------------------------------------- */

/* plan_materialize_strided (src/lib.rs:1630): compact dst <- strided src. */
int t4a_plan_materialize_strided(int dtype, const t4a_cuda_layout* src, long long src_len, t4a_launch* launch);
/* plan_contiguous_to_view (src/lib.rs:1645): strided dst <- compact src. */
int t4a_plan_contiguous_to_view(int dtype, const t4a_cuda_layout* dst, long long dst_len, t4a_launch* launch);
/* plan_strided_to_strided (src/lib.rs:1660): both layouts share the extents. */
int t4a_plan_strided_to_strided(int dtype, const t4a_cuda_layout* src, long long src_len,
                                const t4a_cuda_layout* dst, long long dst_len, t4a_launch* launch);
/* plan_copy_exact (src/lib.rs:1624), plan_fill_zero (:1601), plan_fill_zero_view (:1609). */
int t4a_plan_copy_exact(int dtype, long long len, t4a_launch* launch);
int t4a_plan_fill_zero(int dtype, long long len, t4a_launch* launch);
int t4a_plan_fill_zero_view(int dtype, const t4a_cuda_layout* dst, long long dst_len, t4a_launch* launch);
/* plan_tiled_transpose (src/lib.rs:1685): dst[b*S + i + j*M] = src[src_offset + b*S + i*N + j],
 * M = dst_fast_extent, N = src_fast_extent; grid[2] is the batch count. */
int t4a_plan_tiled_transpose(int dtype, t4a_cuda_transpose_config config, long long src_offset,
                             long long batch_stride, long long dst_fast_extent, long long src_fast_extent,
                             long long batches, long long src_len, long long dst_len, t4a_launch* launch);
/* plan_broadcast_in_dim (src/lib.rs:1498): dims[s] is the destination axis of input axis s. */
int t4a_plan_broadcast_in_dim(int dtype, const t4a_cuda_layout* out, long long out_len,
                              const t4a_cuda_layout* in, long long in_len, const long long* dims, int ndims,
                              t4a_launch* launch);

/* Launchers with the argument lists of movement.cu:535, :544, :553, :528, :571, :648, :514 and
 * fill_zero_view (:519). */
int t4a_launch_materialize_strided(const t4a_launch* launch, void* stream, void* dst, const void* src, int dtype,
                                   t4a_cuda_layout src_layout, long long len);
int t4a_launch_contiguous_to_view(const t4a_launch* launch, void* stream, void* dst, const void* src, int dtype,
                                  t4a_cuda_layout dst_layout, long long len);
int t4a_launch_strided_to_strided(const t4a_launch* launch, void* stream, void* dst, const void* src, int dtype,
                                  t4a_cuda_layout src_layout, t4a_cuda_layout dst_layout, long long len);
int t4a_launch_copy_exact(const t4a_launch* launch, void* stream, void* dst, const void* src, int dtype,
                          long long len);
int t4a_launch_tiled_transpose(const t4a_launch* launch, void* stream, void* dst, const void* src, int dtype,
                               long long src_offset, long long batch_stride, long long dst_fast_extent,
                               long long src_fast_extent, t4a_cuda_transpose_config config);
int t4a_launch_broadcast_in_dim(const t4a_launch* launch, void* stream, void* out, const void* in, int dtype,
                                t4a_cuda_layout out_layout, t4a_cuda_layout in_layout, t4a_cuda_axis_values dims,
                                long long out_len);
int t4a_launch_fill_zero(const t4a_launch* launch, void* stream, void* out, int dtype, long long len);
int t4a_launch_fill_zero_view(const t4a_launch* launch, void* stream, void* out, int dtype, t4a_cuda_layout layout,
                              long long len);

/* One call: validate (as t4a_plan_strided_to_strided) and copy. */
int t4a_copy_strided(void* stream, int dtype, void* dst, const t4a_cuda_layout* dst_layout, long long dst_len,
                     const void* src, const t4a_cuda_layout* src_layout, long long src_len);

/* ------------------------------------------------------------------------- */
/* Gather and additive scatter (reference src/lib.rs:2779-3029,               */
/* gather_scatter.cu:454-492).  The plans are the by-value mirrors             */
/* (CGatherPlan / CScatterPlan, src/lib.rs:4192-4303).                         */
/* ------------------------------------------------------------------------- */

/* General-rank movement, the `_any` twins (reference cuda/src/movement.cu:612-665;
 * module symbols t4a_cuda_{fill_zero_view,materialize_strided,contiguous_to_view,
 * strided_to_strided,broadcast_in_dim}_any in movement.cubin): element-wise walks over
 * layouts whose extents and strides (and broadcast dimensions) are in device memory,
 * so any rank works.  The launchers take the kernels' argument lists; any geometry is
 * correct, t4a_movement_any_geometry gives the one they are tuned for.  The host checks
 * what it can without device access (rank and reserved fields, NULL arrays, matching
 * ranks); extents and strides are the caller's, as in the reference. */
int t4a_movement_any_geometry(long long len, t4a_launch* launch);
int t4a_launch_fill_zero_view_any(const t4a_launch* launch, void* stream, void* out, int dtype,
                                  t4a_cuda_layout_any layout, long long len);
int t4a_launch_materialize_strided_any(const t4a_launch* launch, void* stream, void* dst, const void* src, int dtype,
                                       t4a_cuda_layout_any src_layout, long long len);
int t4a_launch_contiguous_to_view_any(const t4a_launch* launch, void* stream, void* dst, const void* src, int dtype,
                                      t4a_cuda_layout_any dst_layout, long long len);
int t4a_launch_strided_to_strided_any(const t4a_launch* launch, void* stream, void* dst, const void* src, int dtype,
                                      t4a_cuda_layout_any src_layout, t4a_cuda_layout_any dst_layout,
                                      long long len);
int t4a_launch_broadcast_in_dim_any(const t4a_launch* launch, void* stream, void* out, const void* in, int dtype,
                                    t4a_cuda_layout_any out_layout, t4a_cuda_layout_any in_layout,
                                    t4a_cuda_axis_values_any dims, long long out_len);

/* plan_gather (src/lib.rs:2867): validates the maps and the derived output extents;
 * *output_len receives the output element count the launch expects. */
int t4a_plan_gather(int dtype, int index_dtype, const t4a_cuda_layout* out, long long out_len,
                    const t4a_cuda_layout* operand, long long operand_len, const t4a_cuda_layout* indices,
                    long long indices_len, const t4a_cuda_gather_plan* plan, t4a_launch* launch,
                    long long* output_len);
/* plan_scatter_add (src/lib.rs:2970): `out` already holds the operand (copy_exact first).
 * Updates whose window does not fit the destination are skipped, as in the reference. */
int t4a_plan_scatter_add(int dtype, int index_dtype, const t4a_cuda_layout* out, long long out_len,
                         const t4a_cuda_layout* indices, long long indices_len, const t4a_cuda_layout* updates,
                         long long updates_len, const t4a_cuda_scatter_plan* plan, t4a_launch* launch);

/* Launchers with the argument lists of gather_scatter.cu:454 and :486 (layouts by pointer). */
int t4a_launch_gather(const t4a_launch* launch, void* stream, void* out, const void* operand, const void* indices,
                      int dtype, int index_dtype, const t4a_cuda_layout* out_layout,
                      const t4a_cuda_layout* operand_layout, const t4a_cuda_layout* indices_layout,
                      const t4a_cuda_gather_plan* plan, long long output_len);
/* One-kernel scatter (the exported symbol's path): each block sorts a chunk of 2048
 * update pieces by destination in shared memory and folds it.  Collisions are summed
 * in update order inside a chunk and atomically across chunks, so the floating result
 * depends on the schedule (the reference's atomics are order-free as well). */
int t4a_launch_scatter_add(const t4a_launch* launch, void* stream, void* out, const void* indices,
                           const void* updates, int dtype, int index_dtype, const t4a_cuda_layout* out_layout,
                           const t4a_cuda_layout* indices_layout, const t4a_cuda_layout* updates_layout,
                           const t4a_cuda_scatter_plan* plan, long long update_len);
/* Workspace of the two-kernel scatter (a grouping pass writes each chunk's sorted
 * (destination, source) list, 16 bytes an update piece; a streaming pass folds it). */
int t4a_scatter_add_workspace_bytes(int dtype, int index_dtype, const t4a_cuda_layout* out_layout,
                                    const t4a_cuda_layout* indices_layout, const t4a_cuda_layout* updates_layout,
                                    const t4a_cuda_scatter_plan* plan, size_t* bytes);

/* One call each: plan and launch. */
int t4a_gather(void* stream, int dtype, int index_dtype, void* out, const t4a_cuda_layout* out_layout,
               long long out_len, const void* operand, const t4a_cuda_layout* operand_layout, long long operand_len,
               const void* indices, const t4a_cuda_layout* indices_layout, long long indices_len,
               const t4a_cuda_gather_plan* plan);
/* t4a_scatter_add: with a workspace of t4a_scatter_add_workspace_bytes (16-byte
 * aligned) the two-kernel path, with NULL the one-kernel path; a smaller workspace
 * is T4A_ERR_WORKSPACE.  The workspace's first int is a status word: the grouping
 * pass sets it to 0, and the fold sets it to 1 when a bulk copy's completion wait
 * ran out (the fold then stops); it is left untouched when there is no work. */
int t4a_scatter_add(void* stream, int dtype, int index_dtype, void* out, const t4a_cuda_layout* out_layout,
                    long long out_len, const void* indices, const t4a_cuda_layout* indices_layout,
                    long long indices_len, const void* updates, const t4a_cuda_layout* updates_layout,
                    long long updates_len, const t4a_cuda_scatter_plan* plan, void* workspace,
                    size_t workspace_bytes);

/* No counterpart in the reference: t4a_scatter_add restricted to the elements
 * [range_begin, range_end) of the destination, for owner-computes sharding (each GPU
 * holds a slice of the destination and applies, from the whole index list, only the
 * updates that land in its slice).  out_layout describes the whole destination, which
 * must be compact (element e at offset e, layout offset 0); `out` holds elements
 * [range_begin, range_end) (out[0] is element range_begin).  Elements outside the range
 * are neither read nor written, and update rows whose destination lies outside it are
 * not read.  Each contiguous run of an update window must cover whole leading
 * destination axes and both ends must be multiples of it (e.g. whole rows for a scatter
 * of rows), otherwise T4A_ERR_SHAPE_MISMATCH.  Two kernels over a caller workspace of
 * t4a_scatter_add_workspace_bytes (required); its leading status word is 1 when a
 * bounded wait ran out.  Results equal t4a_scatter_add's on the range up to the order
 * of floating additions. */
int t4a_scatter_add_range(void* stream, int dtype, int index_dtype, void* out, const t4a_cuda_layout* out_layout,
                          long long out_len, long long range_begin, long long range_end, const void* indices,
                          const t4a_cuda_layout* indices_layout, long long indices_len, const void* updates,
                          const t4a_cuda_layout* updates_layout, long long updates_len,
                          const t4a_cuda_scatter_plan* plan, void* workspace, size_t workspace_bytes);

/* The same with block-cyclic ownership: the destination's elements form blocks of
 * `block` elements, block b belongs to owner b % owners, and `out` holds this owner's
 * blocks back to back in block order (for a scatter of rows: rows r with
 * r % owners == owner, out row k = row k * owners + owner).  `block` must be a multiple
 * of each contiguous run of an update window.  Cyclic ownership spreads skewed (e.g.
 * Zipf) destination rows evenly across owners, where contiguous slabs would not. */
int t4a_scatter_add_cyclic(void* stream, int dtype, int index_dtype, void* out, const t4a_cuda_layout* out_layout,
                           long long out_len, long long block, long long owners, long long owner, const void* indices,
                           const t4a_cuda_layout* indices_layout, long long indices_len, const void* updates,
                           const t4a_cuda_layout* updates_layout, long long updates_len,
                           const t4a_cuda_scatter_plan* plan, void* workspace, size_t workspace_bytes);

/* General-rank gather / scatter_add, the `_any` twins (reference
 * cuda/src/gather_scatter.cu:587, :619; module symbols t4a_cuda_gather_any and
 * t4a_cuda_scatter_add_any in gather_scatter.cubin): element-wise walks over layouts
 * and maps in device memory, with the kernels' argument lists (layouts and plans by
 * value).  Any geometry is correct; t4a_gather_scatter_any_geometry(elements) gives
 * the one they are tuned for (elements = output_len / update_len).  The host checks
 * dtypes, ranks, the maps' counts, null arrays and the index tensor's rank; the
 * kernels check the maps' values (axes in range, distinct window positions) and that
 * the count fits the walked layout, and a block that finds them malformed does
 * nothing.  Elements are accessed as wide as the buffers' bases allow, so complex64
 * needs 4-byte and complex128 8-byte alignment only. */
int t4a_gather_scatter_any_geometry(long long elements, t4a_launch* launch);
int t4a_launch_gather_any(const t4a_launch* launch, void* stream, void* out, const void* operand,
                          const void* indices, int dtype, int index_dtype, t4a_cuda_layout_any out_layout,
                          t4a_cuda_layout_any operand_layout, t4a_cuda_layout_any indices_layout,
                          t4a_cuda_gather_plan_any plan, long long output_len);
int t4a_launch_scatter_add_any(const t4a_launch* launch, void* stream, void* out, const void* indices,
                               const void* updates, int dtype, int index_dtype, t4a_cuda_layout_any out_layout,
                               t4a_cuda_layout_any indices_layout, t4a_cuda_layout_any updates_layout,
                               t4a_cuda_scatter_plan_any plan, long long update_len);


/* ------------------------------------------------------------------------- */
/* RRQR primitives (reference src/lib.rs:2460-2774, rrqr.cu:513-705).          */
/* Plane entries run one task (a reference 32-lane block) per warp, with the   */
/* reference's lane order, so F32/F64 results are bit-identical.               */
/* ------------------------------------------------------------------------- */

/* plan_initialize_permutation (src/lib.rs:2512): permutation[pos] = pos % n. */
int t4a_plan_initialize_permutation(long long n, long long len, t4a_launch* launch);
/* plan_column_norms (src/lib.rs:2521): columns step..n measured over rows step..m. */
int t4a_plan_column_norms(int dtype, const t4a_cuda_layout* work, long long work_len, const t4a_cuda_layout* norms,
                          long long norms_len, long long step, t4a_launch* launch);
/* plan_select_pivot (src/lib.rs:2561). */
int t4a_plan_select_pivot(int dtype, const t4a_cuda_layout* norms, long long norms_len,
                          const t4a_cuda_layout* permutation, long long permutation_len, long long pivots_len,
                          long long status_len, long long step, t4a_launch* launch);
/* plan_swap_columns (src/lib.rs:2598). */
int t4a_plan_swap_columns(int dtype, const t4a_cuda_layout* work, long long work_len,
                          const t4a_cuda_layout* permutation, long long permutation_len, long long pivots_len,
                          long long step, t4a_launch* launch);
/* plan_reflector (src/lib.rs:2635). */
int t4a_plan_reflector(int dtype, const t4a_cuda_layout* work, long long work_len, const t4a_cuda_layout* coeff,
                       long long coeff_len, long long step, t4a_launch* launch);
/* plan_apply_reflector (src/lib.rs:2664): columns first_column..first_column+column_count. */
int t4a_plan_apply_reflector(int dtype, const t4a_cuda_layout* packed, long long packed_len,
                             const t4a_cuda_layout* target, long long target_len, const t4a_cuda_layout* coeff,
                             long long coeff_len, long long step, long long first_column, long long column_count,
                             t4a_launch* launch);
/* plan_extract_r (src/lib.rs:2719), plan_prefix_rank (src/lib.rs:2748). */
int t4a_plan_extract_r(int dtype, const t4a_cuda_layout* work, long long work_len, const t4a_cuda_layout* r,
                       long long r_len, t4a_launch* launch);
int t4a_plan_prefix_rank(int dtype, const t4a_cuda_layout* r, long long r_len, long long rank_len,
                         long long status_len, double rtol, double atol, t4a_launch* launch);

/* Launchers with the argument lists of rrqr.cu:513, :524, :546, :567, :576, :620, :678, :684. */
int t4a_launch_initialize_permutation(const t4a_launch* launch, void* stream, void* permutation, long long n,
                                      long long len);
int t4a_launch_column_norms(const t4a_launch* launch, void* stream, const void* work, void* norms, int dtype,
                            t4a_cuda_layout work_layout, t4a_cuda_layout norms_layout, long long step);
int t4a_launch_select_pivot(const t4a_launch* launch, void* stream, const void* norms, const void* permutation,
                            void* pivots, void* status, int dtype, t4a_cuda_layout norms_layout,
                            t4a_cuda_layout permutation_layout, long long step);
int t4a_launch_swap_columns(const t4a_launch* launch, void* stream, void* work, void* permutation,
                            const void* pivots, int dtype, t4a_cuda_layout work_layout,
                            t4a_cuda_layout permutation_layout, long long step);
int t4a_launch_reflector(const t4a_launch* launch, void* stream, void* work, void* coeff, int dtype,
                         t4a_cuda_layout work_layout, t4a_cuda_layout coeff_layout, long long step);
int t4a_launch_apply_reflector(const t4a_launch* launch, void* stream, const void* packed, void* target,
                               const void* coeff, int dtype, t4a_cuda_layout packed_layout,
                               t4a_cuda_layout target_layout, t4a_cuda_layout coeff_layout, long long step,
                               long long first_column, long long column_count);
int t4a_launch_extract_r(const t4a_launch* launch, void* stream, const void* work, void* r, int dtype,
                         t4a_cuda_layout work_layout, t4a_cuda_layout r_layout);
int t4a_launch_prefix_rank(const t4a_launch* launch, void* stream, const void* r, void* rank, void* status, int dtype,
                           t4a_cuda_layout r_layout, double rtol, double atol);


/* General-rank RRQR primitives, the `_any` twins (reference cuda/src/rrqr.cu:930-1108;
 * module symbols t4a_cuda_*_any in rrqr.cubin): the same bodies as the launchers above,
 * with layouts whose extents and strides are in device memory, so any rank works.
 * The kernels count their tasks from the layouts on the device; the grid must cover
 * them: t4a_rrqr_any_geometry(tasks, flat) gives one task per warp for the plane
 * entries (column_norms: batches * (n - step); select_pivot, reflector, prefix_rank:
 * batches; apply_reflector: batches * column_count) and a grid-stride walk for the
 * flat ones (swap_columns: rows * batches; extract_r: elements of R). */
int t4a_rrqr_any_geometry(long long tasks, int flat, t4a_launch* launch);
int t4a_launch_column_norms_any(const t4a_launch* launch, void* stream, const void* work, void* norms, int dtype,
                                t4a_cuda_layout_any work_layout, t4a_cuda_layout_any norms_layout, long long step);
int t4a_launch_select_pivot_any(const t4a_launch* launch, void* stream, const void* norms, const void* permutation,
                                void* pivots, void* status, int dtype, t4a_cuda_layout_any norms_layout,
                                t4a_cuda_layout_any permutation_layout, long long step);
int t4a_launch_swap_columns_any(const t4a_launch* launch, void* stream, void* work, void* permutation,
                                const void* pivots, int dtype, t4a_cuda_layout_any work_layout,
                                t4a_cuda_layout_any permutation_layout, long long step);
int t4a_launch_reflector_any(const t4a_launch* launch, void* stream, void* work, void* coeff, int dtype,
                             t4a_cuda_layout_any work_layout, t4a_cuda_layout_any coeff_layout, long long step);
int t4a_launch_apply_reflector_any(const t4a_launch* launch, void* stream, const void* packed, void* target,
                                   const void* coeff, int dtype, t4a_cuda_layout_any packed_layout,
                                   t4a_cuda_layout_any target_layout, t4a_cuda_layout_any coeff_layout,
                                   long long step, long long first_column, long long column_count);
int t4a_launch_extract_r_any(const t4a_launch* launch, void* stream, const void* work, void* r, int dtype,
                             t4a_cuda_layout_any work_layout, t4a_cuda_layout_any r_layout);
int t4a_launch_prefix_rank_any(const t4a_launch* launch, void* stream, const void* r, void* rank, void* status,
                               int dtype, t4a_cuda_layout_any r_layout, double rtol, double atol);

/* RRQR epilogue: the shifted identity Q formation starts from (reference
 * linalg_aux.cu:506, :960; plan_identity_shifted src/lib.rs:2158; module symbols
 * t4a_cuda_identity_shifted / _any in linalg_aux.cubin): out(i, j, ..) = 1 where
 * i == start + j, else 0, for F32/F64/I32/I64/C32/C64.  The `_any` launcher takes a
 * geometry from t4a_rrqr_any_geometry(elements, 1). */
int t4a_plan_identity_shifted(int dtype, const t4a_cuda_layout* out, long long out_len, long long start,
                              t4a_launch* launch);
int t4a_launch_identity_shifted(const t4a_launch* launch, void* stream, void* out, int dtype,
                                t4a_cuda_layout out_layout, long long start);
int t4a_launch_identity_shifted_any(const t4a_launch* launch, void* stream, void* out, int dtype,
                                    t4a_cuda_layout_any out_layout, long long start);
/* No single counterpart in the reference (its bench drives the same steps,
 * examples/bench_kernels.rs:2560-2590): Q formation after a factorization,
 * q = identity_shifted(start 0), then apply_reflector for step = k-1 .. 0 over all k
 * columns of q (k = q's columns) with the reflectors of `work` and `coeff`.  Every
 * step is planned before the first launch, so an invalid argument launches nothing.
 * Results equal that loop of primitives bit for bit.  F32/F64 column-major matrices
 * (row stride 1) with contiguous coefficients, naturally aligned, and a non-NULL
 * `status` (device, one long long the caller zeroes) take the column pass: one block
 * per column of q per step, status bit 1 set if a bounded wait ran out.  Everything
 * else runs the primitives' launches. */
int t4a_rrqr_form_q(void* stream, int dtype, const void* work, const t4a_cuda_layout* work_layout,
                    long long work_len, const void* coeff, const t4a_cuda_layout* coeff_layout, long long coeff_len,
                    void* q, const t4a_cuda_layout* q_layout, long long q_len, long long* status);

/* No single counterpart in the reference (its loop lives with the caller, bench
 * examples/bench_kernels.rs:2390-2623): `steps` steps of column_norms, select_pivot,
 * swap_columns, reflector and apply_reflector over the trailing columns, for one
 * column-major F32/F64 matrix (row stride 1), with results bit-identical to that loop
 * of primitives.  permutation: n int64 (initialized here); coeff: `steps` entries;
 * pivots: the pivot of each step (`steps` int64); status: one sticky int64 (bit 0 set
 * when a column norm is non-finite, as the reference's select_pivot does; bit 1 set
 * when a bounded wait for a bulk copy ran out, the results are then invalid; the
 * caller zeroes it).  work and status must be naturally aligned
 * (T4A_ERR_INVALID_STRIDE otherwise).  The workspace holds the norms and per-step
 * scalars (t4a_rrqr_workspace_bytes). */
/* F32/F64 column_norms, reflector and apply_reflector over columns of unit row stride
 * and at least 2048 rows from the step are planned on this library's column engine
 * (t4a_launch.variant 66: one block of 384 threads per task, the same bits as the warp
 * entries, which also run correctly under that geometry).  Their waits on bulk copies
 * are bounded; one that runs out leaves the task's outputs unwritten and sets bit 1 of
 * a device word that this call returns and clears (reference: no counterpart, the
 * reference's primitives have no staged copies).  Synchronizes the current device. */
int t4a_rrqr_primitive_faults(unsigned long long* faults);
int t4a_rrqr_workspace_bytes(int dtype, const t4a_cuda_layout* work, size_t* bytes);
int t4a_rrqr(void* stream, int dtype, void* work, const t4a_cuda_layout* work_layout, long long work_len,
             long long steps, void* permutation, void* coeff, void* pivots, void* status, void* workspace,
             size_t workspace_bytes);

/* ------------------------------------------------------------------------- */
/* RRQR over GPUs (rows sharded; no counterpart in the reference, which has no */
/* multi-device code: this is the row-sharded form of the step loop of its     */
/* bench, examples/bench_kernels.rs:2398-2530)                                 */
/* ------------------------------------------------------------------------- */

/* NCCL communicator set-up for the sharded driver (NCCL is loaded on first use; without
 * libnccl.so.2 these return T4A_ERR_CUDA).  t4a_dist_unique_id writes the 128-byte
 * ncclUniqueId that rank 0 hands to every rank (by the caller's own channel);
 * t4a_dist_comm_init is collective over the `world` ranks, each with its device
 * current. */
int t4a_dist_unique_id(void* id);
int t4a_dist_comm_init(void** comm, const void* id, int world, int rank);
int t4a_dist_comm_destroy(void* comm);

/* Workspace of t4a_dist_rrqr: exchange buffers for n columns over `world` ranks. */
int t4a_dist_rrqr_workspace_bytes(int dtype, long long n, int world, size_t* bytes);

/* `steps` steps of the reference RRQR loop over a [global_rows, n] F32/F64 matrix whose
 * rows [row0, row0 + local_rows) this rank holds as the column-major `work` (layout
 * [local_rows, n], row stride 1); every rank of `comm` calls it with its own rows, on
 * its own stream.  Per step: the pivot from the column norms combined in rank order,
 * the swap and the reflector on each rank's rows, the dot parts (NCCL all-gather), the
 * update and the next norm parts (NCCL all-gather).  perm (n), coeff (steps), pivots
 * (steps) and status (bit 0: a non-finite norm; bit 1: a bounded wait ran out) come out
 * the same on every rank.  With one rank the results equal t4a_rrqr bit for bit; with
 * several the norms and dots round differently, so pivots agree where the column norms
 * are well separated (the rank-revealing prefix).  Nothing is allocated; the caller
 * synchronizes. */
int t4a_dist_rrqr(void* comm, void* stream, int dtype, void* work, const t4a_cuda_layout* local_layout,
                  long long work_len, long long row0, long long global_rows, long long steps, void* permutation,
                  void* coeff, void* pivots, void* status, void* workspace, size_t workspace_bytes);

/* The same row-sharded RRQR with its exchanges fused into the step kernels: each rank
 * stores its norm and dot parts into every rank's exchange region over NVLink and
 * publishes them with a per-rank flag, and the kernel that needs them waits (bounded)
 * for every rank's flag.  No collective call sits between the step's kernels.
 *
 * t4a_p2p_create allocates this GPU's region for matrices of n columns and a world of
 * `world` ranks, and writes its 64-byte CUDA IPC handle to ipc_handle; the caller
 * gathers every rank's handle (rank order, world x 64 bytes) and passes them to
 * t4a_p2p_open, which maps the peers' regions.  t4a_dist_rrqr_p2p takes the arguments
 * of t4a_dist_rrqr without a workspace, and gives its bits; every rank must make the
 * same calls in the same order.  Before t4a_p2p_destroy every rank must have finished
 * its calls (the caller synchronizes and waits for the others), since peers write into
 * the region.  A wait that ran out sets status bit 1. */
int t4a_p2p_region_bytes(long long n, int world, size_t* bytes);
int t4a_p2p_create(long long n, int world, int rank, void** comm, void* ipc_handle);
int t4a_p2p_open(void* comm, const void* ipc_handles);
int t4a_p2p_destroy(void* comm);
int t4a_dist_rrqr_p2p(void* comm, void* stream, int dtype, void* work, const t4a_cuda_layout* local_layout,
                      long long work_len, long long row0, long long global_rows, long long steps, void* permutation,
                      void* coeff, void* pivots, void* status);

#ifdef __cplusplus
}
#endif

#endif /* T4A_B200_H_ */
