/*
 * t4a_b200 kernel ABI types.
 *
 * By-value metadata structs, dtype/op tags and size constants of the
 * t4a-cuda-kernels kernel ABI (revision 14, symbol set of revision 10).  Every
 * struct here is layout-identical to its counterpart in the reference header
 * `cuda/include/t4a/abi.cuh` (t4a_cuda_layout at abi.cuh:51-57, the reduce tags
 * at :60-71, t4a_cuda_axis_values at :75-79, the gather/scatter plans at :82-107,
 * t4a_cuda_transpose_config at :240-245, the size asserts at :247-280), because
 * a kernel module built from this tree must accept the exact argument bytes a
 * caller of the reference module passes to cuLaunchKernel.
 *
 * The header is plain C99/C++ with no device code, so host code in any language
 * that speaks the C ABI (C, C++, Rust, Go, Python ctypes) can use it.
 *
 * Layout convention: axis 0 is the fastest-varying logical axis.  A flat index
 * f decodes as coordinate = f % extent, f /= extent from axis 0 upward; the
 * element address is offset + sum(coordinate * stride), in signed elements.
 */
#ifndef T4A_B200_ABI_H_
#define T4A_B200_ABI_H_

#ifdef __cplusplus
extern "C" {
#endif

#define T4A_CUDA_MAX_RANK 8
#define T4A_CUDA_ABI_REVISION 14

/* Element type tags (reference abi.cuh:25-33). */
typedef enum {
  T4A_CUDA_F32 = 0,
  T4A_CUDA_F64 = 1,
  T4A_CUDA_I32 = 2,
  T4A_CUDA_I64 = 3,
  T4A_CUDA_BOOL = 4,
  T4A_CUDA_C32 = 5,
  T4A_CUDA_C64 = 6
} t4a_cuda_dtype;

/* Interleaved complex with the component's alignment (not float2/double2). */
typedef struct {
  float re;
  float im;
} t4a_cuda_c32;

typedef struct {
  double re;
  double im;
} t4a_cuda_c64;

/* Strided logical layout, passed by value (144 bytes). */
typedef struct {
  int rank;
  int reserved;
  long long offset;
  long long extents[T4A_CUDA_MAX_RANK];
  long long strides[T4A_CUDA_MAX_RANK];
} t4a_cuda_layout;

/* Reduction operation and strategy tags (ABI revision 3). */
typedef enum {
  T4A_CUDA_REDUCE_SUM = 0,
  T4A_CUDA_REDUCE_PROD = 1,
  T4A_CUDA_REDUCE_SUM_SQUARES = 2,
  T4A_CUDA_REDUCE_MAX = 3,
  T4A_CUDA_REDUCE_MIN = 4
} t4a_cuda_reduce_op;

typedef enum {
  T4A_CUDA_REDUCE_UNIT = 0,
  T4A_CUDA_REDUCE_PLANE = 1
} t4a_cuda_reduce_strategy;

/* Per-axis runtime values (broadcast_in_dim's destination-axis map). */
typedef struct {
  int rank;
  int reserved;
  long long values[T4A_CUDA_MAX_RANK];
} t4a_cuda_axis_values;

/* XLA-style gather dimension maps (ABI revision 4). */
typedef struct {
  int operand_rank;
  int out_rank;
  int index_vector_dim;
  int window_rank;
  int start_map_len;
  int reserved;
  long long window_dims[T4A_CUDA_MAX_RANK];
  long long offset_dims[T4A_CUDA_MAX_RANK];
  long long start_index_map[T4A_CUDA_MAX_RANK];
  long long slice_sizes[T4A_CUDA_MAX_RANK];
} t4a_cuda_gather_plan;

/* Additive-scatter dimension maps (ABI revision 4). */
typedef struct {
  int operand_rank;
  int updates_rank;
  int index_vector_dim;
  int window_rank;
  int scatter_map_len;
  int reserved;
  long long window_dims[T4A_CUDA_MAX_RANK];
  long long update_window_dims[T4A_CUDA_MAX_RANK];
  long long scatter_dims[T4A_CUDA_MAX_RANK];
} t4a_cuda_scatter_plan;

/* Tile configuration of the batched transpose. */
typedef struct {
  int tile;
  int block_rows;
  int padding;
  int vector_width;
} t4a_cuda_transpose_config;

/* General-rank layout of the `_any` entries (reference abi.cuh "Dynamic rank"): the
 * same fields as t4a_cuda_layout with the extents and strides in caller-owned device
 * memory, so any rank is representable; a zero-length array may be NULL. */
typedef struct {
  int rank;
  int reserved;  /* must be 0 */
  long long offset;
  const long long* extents;  /* rank values, device memory */
  const long long* strides;  /* rank values, device memory */
} t4a_cuda_layout_any;

/* Per-axis values of the `_any` entries (broadcast dimensions), in device memory. */
typedef struct {
  int rank;
  int reserved;  /* must be 0 */
  const long long* values;  /* rank values, device memory */
} t4a_cuda_axis_values_any;

/* Gather dimension maps of the `_any` entries: the fields of t4a_cuda_gather_plan with
 * the maps in caller-owned device memory (window_dims / offset_dims: window_rank
 * values; start_index_map: start_map_len; slice_sizes: operand_rank). */
typedef struct {
  int operand_rank;
  int out_rank;
  int index_vector_dim;
  int window_rank;
  int start_map_len;
  int reserved;  /* must be 0 */
  const long long* window_dims;
  const long long* offset_dims;
  const long long* start_index_map;
  const long long* slice_sizes;
} t4a_cuda_gather_plan_any;

/* Additive-scatter dimension maps of the `_any` entries (window_dims /
 * update_window_dims: window_rank values; scatter_dims: scatter_map_len), device
 * memory. */
typedef struct {
  int operand_rank;
  int updates_rank;
  int index_vector_dim;
  int window_rank;
  int scatter_map_len;
  int reserved;  /* must be 0 */
  const long long* window_dims;
  const long long* update_window_dims;
  const long long* scatter_dims;
} t4a_cuda_scatter_plan_any;

#ifdef __cplusplus
}  /* extern "C" */

static_assert(sizeof(t4a_cuda_gather_plan_any) == 56, "t4a_cuda_gather_plan_any size");
static_assert(__builtin_offsetof(t4a_cuda_gather_plan_any, window_dims) == 24, "gather_any.window_dims");
static_assert(__builtin_offsetof(t4a_cuda_gather_plan_any, slice_sizes) == 48, "gather_any.slice_sizes");
static_assert(sizeof(t4a_cuda_scatter_plan_any) == 48, "t4a_cuda_scatter_plan_any size");
static_assert(__builtin_offsetof(t4a_cuda_scatter_plan_any, scatter_dims) == 40, "scatter_any.scatter_dims");
static_assert(sizeof(t4a_cuda_axis_values_any) == 16, "t4a_cuda_axis_values_any size");
static_assert(sizeof(t4a_cuda_layout_any) == 32, "t4a_cuda_layout_any size");
static_assert(alignof(t4a_cuda_layout_any) == 8, "t4a_cuda_layout_any alignment");
static_assert(__builtin_offsetof(t4a_cuda_layout_any, extents) == 16, "layout_any.extents");
static_assert(sizeof(t4a_cuda_layout) == 144, "t4a_cuda_layout size");
static_assert(alignof(t4a_cuda_layout) == 8, "t4a_cuda_layout alignment");
static_assert(__builtin_offsetof(t4a_cuda_layout, offset) == 8, "layout.offset");
static_assert(__builtin_offsetof(t4a_cuda_layout, extents) == 16, "layout.extents");
static_assert(__builtin_offsetof(t4a_cuda_layout, strides) == 80, "layout.strides");
static_assert(sizeof(t4a_cuda_axis_values) == 72, "t4a_cuda_axis_values size");
static_assert(sizeof(t4a_cuda_gather_plan) == 280, "t4a_cuda_gather_plan size");
static_assert(__builtin_offsetof(t4a_cuda_gather_plan, window_dims) == 24, "gather.window_dims");
static_assert(sizeof(t4a_cuda_scatter_plan) == 216, "t4a_cuda_scatter_plan size");
static_assert(__builtin_offsetof(t4a_cuda_scatter_plan, window_dims) == 24, "scatter.window_dims");
static_assert(sizeof(t4a_cuda_transpose_config) == 16, "t4a_cuda_transpose_config size");
static_assert(alignof(t4a_cuda_transpose_config) == 4, "t4a_cuda_transpose_config alignment");
static_assert(sizeof(t4a_cuda_c32) == 8 && alignof(t4a_cuda_c32) == 4, "t4a_cuda_c32");
static_assert(sizeof(t4a_cuda_c64) == 16 && alignof(t4a_cuda_c64) == 8, "t4a_cuda_c64");
#endif

#endif /* T4A_B200_ABI_H_ */
