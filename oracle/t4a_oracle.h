/*
 * t4a_oracle: CPU restatement of the t4a-cuda-kernels hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (the t4a_b200 library, its
 * kernels or its Python mirror) links, loads or calls this code.  Only the test
 * suite, the smoke check and the CPU-baseline leg of bench.py use it, as the
 * checker and as the timed CPU baseline.
 *
 * Every entry restates the reference's semantics for one kernel entry, including
 * the fold topology the reference ABI documents for reductions, so that results
 * can be compared bit for bit.  The file that implements each entry cites the
 * reference source lines it follows.
 */
#ifndef T4A_ORACLE_H_
#define T4A_ORACLE_H_

#include "../include/t4a_b200/abi.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Reduction topology the reference planner picks (src/lib.rs:3152-3166,
 * :3235-3241, :3435-3455).  kind 0 = direct, 1 = split. */
typedef struct {
  int kind;
  int direct_strategy;     /* T4A_CUDA_REDUCE_UNIT / _PLANE when kind == 0 */
  long long splits;        /* kind == 1 */
  long long chunk_len;     /* kind == 1 */
  int combine_strategy;    /* kind == 1 */
  int combine_width;       /* kind == 1: block width of the combine pass */
  int combine_op;          /* kind == 1 */
} t4a_oracle_reduce_topology;

/* Restated split policy + strategy choice.  Returns 0, or -1 on a bad width. */
int t4a_oracle_reduce_topology_for(int op, long long reduce_len, int plane_width,
                                   t4a_oracle_reduce_topology* topo);

/* Whole reduction with the reference topology.  `partials` (may be NULL) receives
 * pass-1 partials in the compact partials layout (input extents with the axis set
 * to `splits`) when the topology splits.  Returns 0 on success, -1 on an
 * unsupported dtype/op pair or bad metadata. */
int t4a_oracle_reduce(int dtype, int op, void* out, const t4a_cuda_layout* out_layout,
                      const void* in, const t4a_cuda_layout* in_layout, int axis,
                      int plane_width, void* partials, t4a_oracle_reduce_topology* topo_out);

/* Plain fold of one axis for the threaded CPU baseline: same topology, each
 * thread owns a contiguous range of outputs. */
int t4a_oracle_reduce_threaded(int dtype, int op, void* out, const t4a_cuda_layout* out_layout,
                               const void* in, const t4a_cuda_layout* in_layout, int axis,
                               int plane_width, int threads);

/* Movement (reference cuda/src/movement.cu). */
int t4a_oracle_strided_to_strided(int dtype, void* dst, const void* src,
                                  const t4a_cuda_layout* src_layout,
                                  const t4a_cuda_layout* dst_layout, int threads);
int t4a_oracle_materialize_strided(int dtype, void* dst, const void* src,
                                   const t4a_cuda_layout* src_layout, int threads);
int t4a_oracle_contiguous_to_view(int dtype, void* dst, const void* src,
                                  const t4a_cuda_layout* dst_layout, int threads);
int t4a_oracle_tiled_transpose(int dtype, void* dst, const void* src, long long src_offset,
                               long long batch_stride, long long dst_fast_extent,
                               long long src_fast_extent, long long batches, int threads);
int t4a_oracle_broadcast_in_dim(int dtype, void* out, const void* in,
                                const t4a_cuda_layout* out_layout,
                                const t4a_cuda_layout* in_layout,
                                const t4a_cuda_axis_values* dims, int threads);

/* Gather and additive scatter (reference cuda/src/gather_scatter.cu). */
int t4a_oracle_gather(int dtype, int index_dtype, void* out, const void* operand,
                      const void* indices, const t4a_cuda_layout* out_layout,
                      const t4a_cuda_layout* operand_layout,
                      const t4a_cuda_layout* indices_layout,
                      const t4a_cuda_gather_plan* plan, int threads);
/* Serial scatter in update order (the device order is nondeterministic). */
int t4a_oracle_scatter_add(int dtype, int index_dtype, void* out, const void* indices,
                           const void* updates, const t4a_cuda_layout* out_layout,
                           const t4a_cuda_layout* indices_layout,
                           const t4a_cuda_layout* updates_layout,
                           const t4a_cuda_scatter_plan* plan, int threads);

/* RRQR primitives (reference cuda/src/rrqr.cu), with the reference's 32-lane
 * fold order so that norms, reflectors and pivots are reproduced bit for bit. */
int t4a_oracle_initialize_permutation(long long* permutation, long long n, long long len);
int t4a_oracle_column_norms(int dtype, const void* work, void* norms,
                            const t4a_cuda_layout* work_layout,
                            const t4a_cuda_layout* norms_layout, long long step, int threads);
int t4a_oracle_select_pivot(int dtype, const void* norms, const long long* permutation,
                            long long* pivots, long long* status,
                            const t4a_cuda_layout* norms_layout,
                            const t4a_cuda_layout* permutation_layout, long long step);
int t4a_oracle_swap_columns(int dtype, void* work, long long* permutation,
                            const long long* pivots, const t4a_cuda_layout* work_layout,
                            const t4a_cuda_layout* permutation_layout, long long step);
int t4a_oracle_reflector(int dtype, void* work, void* coeff, const t4a_cuda_layout* work_layout,
                         const t4a_cuda_layout* coeff_layout, long long step);
int t4a_oracle_apply_reflector(int dtype, const void* packed, void* target, const void* coeff,
                               const t4a_cuda_layout* packed_layout,
                               const t4a_cuda_layout* target_layout,
                               const t4a_cuda_layout* coeff_layout, long long step,
                               long long first_column, long long column_count, int threads);
int t4a_oracle_extract_r(int dtype, const void* work, void* r,
                         const t4a_cuda_layout* work_layout, const t4a_cuda_layout* r_layout);
int t4a_oracle_prefix_rank(int dtype, const void* r, long long* rank, long long* status,
                           const t4a_cuda_layout* r_layout, double rtol, double atol);

/* identity_shifted (reference cuda/src/linalg_aux.cu:200-211): out(i, j, ..) = 1
 * where i == start + j, else 0, over every element of a rank >= 2 layout. */
int t4a_oracle_identity_shifted(int dtype, void* out, const t4a_cuda_layout* out_layout, long long start);

/* Whole tall-skinny RRQR loop as the reference bench drives it
 * (examples/bench_kernels.rs:2390-2623): work is an m x n column-major F64
 * matrix, updated in place; perm/coeff receive n entries; returns the rank. */
long long t4a_oracle_rrqr_f64(double* work, long long m, long long n, long long steps,
                              long long* perm, double* coeff, double rtol, double atol,
                              int threads);

/* Row-sharded RRQR, one rank's share of a step (the restatement of t4a_dist_rrqr): a rank
 * holds rows [row0, row0 + mr) of every column, column-major with column stride ld.
 * Parts are 8 doubles per column (scale, ssq, rscale, rssq, xrow, bad, own, pad). */
int t4a_oracle_dist_norm_parts(const double* local, long long mr, long long n, long long ld, long long row0,
                               long long s, long long first_col, double* parts);
int t4a_oracle_dist_select_swap(double* local, long long mr, long long n, long long ld, long long row0, long long s,
                                const double* parts, int world, long long* perm, double* coeff, long long* pivots,
                                long long* status);
int t4a_oracle_dist_dot_parts(const double* local, long long mr, long long n, long long ld, long long row0,
                              long long s, double* dots);
int t4a_oracle_dist_update(double* local, long long mr, long long n, long long ld, long long row0, long long s,
                           const double* dots, int world, const double* coeff);
/* The ranks of one [m, n] matrix run in turn; returns the status word. */
long long t4a_oracle_rrqr_rows_sharded_f64(double* work, long long m, long long n, long long steps, int world,
                                           long long* perm, double* coeff, long long* pivots);

#ifdef __cplusplus
}
#endif

#endif /* T4A_ORACLE_H_ */
