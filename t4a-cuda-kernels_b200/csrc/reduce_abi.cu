// The exported reduction symbols of the kernel ABI, for callers that load the module
// and launch by name (reference signatures cuda/src/reduce.cu:765-768, :813-817).
// Each launch picks its path at run time from the layouts, the block shape and the
// dynamic shared memory it was given (see reduce_core.cuh); the host launchers of
// this library use the per-path kernels of reduce_fast.cu instead.
#include "reduce_core.cuh"

extern "C" __global__ void __launch_bounds__(512) t4a_cuda_reduce(
    void* out, const void* in, int dtype, int op, int strategy, t4a_cuda_layout out_layout,
    t4a_cuda_layout in_layout, int axis, long long output_len) {
#define T4A_CALL(OP, T) \
  t4a::reduce_abi_body<OP, T>(out, in, strategy, out_layout, in_layout, axis, output_len, OP())
  T4A_REDUCE_SWITCH(op, dtype, T4A_CALL)
#undef T4A_CALL
}

extern "C" __global__ void __launch_bounds__(256) t4a_cuda_reduce_partials(
    void* partials, const void* in, int dtype, int op, t4a_cuda_layout partials_layout,
    t4a_cuda_layout in_layout, int axis, long long output_len, long long splits,
    long long chunk_len) {
#define T4A_CALL(OP, T)                                                                            \
  t4a::partials_abi_body<OP, T>(partials, in, partials_layout, in_layout, axis, output_len, splits, \
                                chunk_len, OP())
  T4A_REDUCE_SWITCH(op, dtype, T4A_CALL)
#undef T4A_CALL
}

// General-rank twins (reference cuda/src/reduce.cu:854-940): the same folds with the
// layouts' arrays in device memory.
extern "C" __global__ void __launch_bounds__(512) t4a_cuda_reduce_any(
    void* out, const void* in, int dtype, int op, int strategy, t4a_cuda_layout_any out_layout,
    t4a_cuda_layout_any in_layout, int axis, long long output_len) {
#define T4A_CALL(OP, T) \
  t4a::reduce_any_body<OP, T>(out, in, strategy, out_layout, in_layout, axis, output_len, OP())
  T4A_REDUCE_SWITCH(op, dtype, T4A_CALL)
#undef T4A_CALL
}

extern "C" __global__ void __launch_bounds__(256) t4a_cuda_reduce_partials_any(
    void* partials, const void* in, int dtype, int op, t4a_cuda_layout_any partials_layout,
    t4a_cuda_layout_any in_layout, int axis, long long output_len, long long splits, long long chunk_len) {
#define T4A_CALL(OP, T)                                                                                \
  t4a::partials_any_body<OP, T>(partials, in, partials_layout, in_layout, axis, output_len, splits, \
                                chunk_len, OP())
  T4A_REDUCE_SWITCH(op, dtype, T4A_CALL)
#undef T4A_CALL
}
