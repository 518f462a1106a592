// RRQR planning (reference src/lib.rs:2460-2774) and the host launchers of the RRQR
// primitives.  Plane entries run one task per warp, kTaskWarps tasks per block;
// flat entries are grid-stride walks.
#include <cuda_runtime.h>

#include <atomic>

#include "plan_common.h"
#include "rrqr_core.cuh"
#include "rrqr_entries.cuh"
#include "rrqr_step.cuh"
#include "runtime.h"

namespace t4a {
namespace {

using namespace rrqr;

constexpr int kTaskWarps = 8;
constexpr int kTaskThreads = kTaskWarps * 32;
constexpr int kFlatThreads = 256;
constexpr int kRrqrVariant = 64;  // t4a_launch.variant of the RRQR entries

// ---- kernels (this library's geometry) -----------------------------------------
__global__ void __launch_bounds__(kFlatThreads) k_init_perm(long long* perm, long long n, long long len,
                                                           unsigned* done) {
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long p = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; p < len; p += stride)
    perm[p] = p % n;
  if (done != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *done = 0;
}

// The primitives' kernels, templated on the layout type: t4a_cuda_layout for the
// launchers of the by-value entries, t4a_cuda_layout_any for the general-rank twins.
// Both run the module's entry bodies (rrqr_entries.cuh).
template <typename L>
__global__ void __launch_bounds__(kTaskThreads) k_norms(const void* w, void* norms, int dtype, L wl, L nl,
                                                        long long step) {
  entry::column_norms_entry(w, norms, dtype, wl, nl, step);
}
template <typename L>
__global__ void __launch_bounds__(kTaskThreads) k_pivot(const void* norms, const void* perm, void* pivots,
                                                        void* status, int dtype, L nl, L pl, long long step) {
  entry::select_pivot_entry(norms, perm, pivots, status, dtype, nl, pl, step);
}
template <typename L>
__global__ void __launch_bounds__(kFlatThreads) k_swap(void* w, void* perm, const void* pivots, int dtype, L wl, L pl,
                                                       long long step) {
  entry::swap_entry(w, perm, pivots, dtype, wl, pl, step);
}
template <typename L>
__global__ void __launch_bounds__(kTaskThreads) k_reflector(void* w, void* coeff, int dtype, L wl, L cl,
                                                            long long step) {
  entry::reflector_entry(w, coeff, dtype, wl, cl, step);
}
template <typename L>
__global__ void __launch_bounds__(kTaskThreads) k_apply(const void* packed, void* target, const void* coeff,
                                                        int dtype, L pl, L tl, L cl, long long step,
                                                        long long first_column, long long column_count) {
  entry::apply_entry(packed, target, coeff, dtype, pl, tl, cl, step, first_column, column_count);
}
template <typename L>
__global__ void __launch_bounds__(kFlatThreads) k_extract_r(const void* w, void* r, int dtype, L wl, L rl) {
  entry::extract_entry(w, r, dtype, wl, rl);
}
template <typename L>
__global__ void __launch_bounds__(kTaskThreads) k_prefix_rank(const void* r, void* rank, void* status, int dtype,
                                                              L rl, double rtol, double atol) {
  entry::prefix_rank_entry(r, rank, status, dtype, rl, rtol, atol);
}

__global__ void __launch_bounds__(kFlatThreads) k_identity(void* out, int dtype, t4a_cuda_layout l, long long start) {
  entry::identity_entry(out, dtype, l, start);
}
__global__ void __launch_bounds__(kFlatThreads) k_identity_any(void* out, int dtype, t4a_cuda_layout_any l,
                                                               long long start) {
  entry::identity_entry(out, dtype, l, start);
}

// Host checks of a general-rank layout that need no device access.
int check_rrqr_any(const t4a_cuda_layout_any& l, int min_rank) {
  if (l.rank < min_rank || l.reserved != 0) return T4A_ERR_RANK_OUT_OF_RANGE;
  if (l.extents == nullptr || l.strides == nullptr) return T4A_ERR_NULL_ARGUMENT;
  return T4A_OK;
}

// ---- fused step driver kernels ---------------------------------------------------
// The driver's launches form one chain on the caller's stream and are launched with
// programmatic stream serialization: a kernel may launch as each block of the previous
// one exits (the implicit trigger), and waits (griddepcontrol.wait) for the previous one
// to finish and its writes to be visible before it touches any data.  This hides the
// launch gap between the links; on config 5 the factorization went from 20.06 ms
// (plain launches) to 19.04 ms.  Triggering explicitly at kernel start
// (griddepcontrol.launch_dependents) made it 22.06 ms: the next kernel's waiting blocks
// took issue slots from the running chains.  Without the attribute the wait returns at
// once.
__device__ __forceinline__ void chain_enter() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename F>
__global__ void __launch_bounds__(kColThreads, 2) k_col_first(FusedArgs<F> a) {
  extern __shared__ __align__(128) unsigned char smem[];
  chain_enter();
  column_first<F>(a, *reinterpret_cast<ColSmem<F>*>(smem));
}
template <typename F>
__global__ void __launch_bounds__(kFlatThreads) k_fused_swap(FusedArgs<F> a, long long step) {
  chain_enter();
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long row = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; row < a.m; row += stride)
    fused_swap<F>(a, step, row);
}
template <typename F>
__global__ void __launch_bounds__(kColThreads, 2) k_col_step(FusedArgs<F> a, long long step, int next_norm) {
  extern __shared__ __align__(128) unsigned char smem[];
  chain_enter();
  column_step<F>(a, step, next_norm != 0, *reinterpret_cast<ColSmem<F>*>(smem));
}

// The clustered column pass (steps with few trailing columns): `csize` blocks per
// column, launched with that cluster size.
template <typename F>
__global__ void __launch_bounds__(kColThreads, 2) k_col_step_cluster(FusedArgs<F> a, long long step, int next_norm,
                                                                    unsigned csize) {
  extern __shared__ __align__(128) unsigned char smem[];
  chain_enter();
  column_step_cluster<F>(a, step, next_norm != 0, *reinterpret_cast<ColSmem<F>*>(smem), csize);
}

// Q formation pass for reflector `step`: one block per column of Q.
template <typename F>
__global__ void __launch_bounds__(kColThreads, 2) k_q_step(FusedArgs<F> a, long long step, F* q, long long qld,
                                                          long long qcols) {
  extern __shared__ __align__(128) unsigned char smem[];
  chain_enter();
  column_q<F>(a, step, q, qld, qcols, *reinterpret_cast<ColSmem<F>*>(smem));
}

// ---- the primitives on the column engine -------------------------------------------
// F32/F64 columns with unit row stride and at least kEngineRows rows from `step` run one
// block per task on the column engine instead of one warp per task; the results are
// the same bits.  A bounded wait that runs out sets bit 1 of g_engine_faults (read and
// cleared by t4a_rrqr_primitive_faults) and leaves that task's outputs unwritten.
constexpr int kRrqrEngineVariant = kRrqrVariant + 2;
constexpr long long kEngineRows = 2048;

__device__ unsigned long long g_engine_faults;

__device__ __forceinline__ long long* engine_faults() { return reinterpret_cast<long long*>(&g_engine_faults); }

template <typename F>
__global__ void __launch_bounds__(kColThreads, 2) k_eng_norms(const F* w, F* norms, t4a_cuda_layout wl,
                                                             t4a_cuda_layout nl, long long step) {
  extern __shared__ __align__(128) unsigned char smem[];
  const long long width = wl.extents[1] - step;
  const long long b = blockIdx.x / width;
  const long long col = step + (blockIdx.x - b * width);
  engine_norms_task<F>(w + wl.offset + col * wl.strides[1] + batch_base(wl, 2, b), step, wl.extents[0],
                       norms + nl.offset + col * nl.strides[0] + batch_base(nl, 1, b), engine_faults(),
                       *reinterpret_cast<ColSmem<F>*>(smem));
}

template <typename F>
__global__ void __launch_bounds__(kColThreads, 2) k_eng_reflector(F* w, F* coeff, t4a_cuda_layout wl,
                                                                 t4a_cuda_layout cl, long long step) {
  extern __shared__ __align__(128) unsigned char smem[];
  const long long b = blockIdx.x;
  engine_reflect_task<F>(w + wl.offset + step * wl.strides[1] + batch_base(wl, 2, b), step, wl.extents[0],
                         coeff + cl.offset + step * cl.strides[0] + batch_base(cl, 1, b), engine_faults(),
                         *reinterpret_cast<ColSmem<F>*>(smem));
}

template <typename F>
__global__ void __launch_bounds__(kColThreads, 2) k_eng_apply(const F* packed, F* target, const F* coeff,
                                                             t4a_cuda_layout pl, t4a_cuda_layout tl,
                                                             t4a_cuda_layout cl, long long step,
                                                             long long first_column, long long column_count) {
  extern __shared__ __align__(128) unsigned char smem[];
  const long long b = blockIdx.x / column_count;
  const long long col = first_column + (blockIdx.x - b * column_count);
  const F* v = packed + pl.offset + step * pl.strides[1] + batch_base(pl, 2, b) + step;
  F* t = target + tl.offset + col * tl.strides[1] + batch_base(tl, 2, b) + step;
  const F c = coeff[cl.offset + step * cl.strides[0] + batch_base(cl, 1, b)];
  engine_apply_task<F>(v, t, pl.extents[0] - step, c, engine_faults(), *reinterpret_cast<ColSmem<F>*>(smem));
}

// Raises a kernel's dynamic shared memory limit once on each device.
template <typename K>
int allow_smem(K kernel, unsigned bytes, std::atomic<unsigned long long>& raised) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return runtime::check_launch();
  const unsigned long long bit = 1ull << (dev & 63);
  if ((raised.load(std::memory_order_relaxed) & bit) == 0) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
      return runtime::check_launch();
    raised.fetch_or(bit);
  }
  return T4A_OK;
}

struct FusedLayout {
  size_t norms, rec, done, total;
};

FusedLayout fused_layout(long long n, int fsize) {
  auto up = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
  FusedLayout l;
  l.norms = 0;
  l.rec = up(l.norms + n * fsize);
  l.done = up(l.rec + 64);
  l.total = up(l.done + 4);
  return l;
}

// Launches `kernel` as the next link of a driver chain (see chain_enter); `csize` > 1:
// with thread-block clusters of that many blocks along x.
template <typename... KArgs, typename... Args>
int chain_launch_clustered(void (*kernel)(KArgs...), unsigned csize, dim3 grid, dim3 block, unsigned smem,
                           cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (csize > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = csize;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) {
    runtime::last_error() = static_cast<int>(e);
    return T4A_ERR_CUDA;
  }
  return T4A_OK;
}
template <typename... KArgs, typename... Args>
int chain_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, unsigned smem, cudaStream_t s, Args... args) {
  return chain_launch_clustered(kernel, 1u, grid, block, smem, s, args...);
}

// The clustered column pass runs one block per SM: its dynamic shared memory is raised
// above half an SM's, so the cluster scheduler cannot pair two blocks (two leaders' chains
// and feeds) on one SM.  Measured on config 5 with two blocks per SM allowed: clusters
// gained 8-11 us per step at 4-19 trailing columns and lost up to 3 us once the pass
// neared 148 blocks.
unsigned cluster_smem(unsigned need) {
  int dev = 0, per_sm = 0, optin = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return need;
  if (cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
    return need;
  const unsigned half = static_cast<unsigned>(per_sm) / 2 + 1024;
  const unsigned want = half > need ? half : need;
  return want <= static_cast<unsigned>(optin) ? want : need;
}

// Cluster size of the column pass over `trailing` columns: the largest of 8, 4, 2 for
// which every cluster of the pass is resident at once (cudaOccupancyMaxActiveClusters at
// one block per SM), else 1 (the plain pass).  Capacities are asked once per device.
template <typename K>
unsigned column_cluster_size(K kernel, unsigned smem, long long trailing) {
  static std::atomic<int> cap[64][4];  // [device][log2 size]: resident clusters + 1 (0: not asked)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return 1;
  for (int lg = 3; lg >= 1; --lg) {
    int c = cap[dev][lg].load(std::memory_order_relaxed);
    if (c == 0) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(1u << lg);
      cfg.blockDim = dim3(kColThreads);
      cfg.dynamicSmemBytes = smem;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 1u << lg;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess) {
        cudaGetLastError();
        clusters = 0;
      }
      c = clusters + 1;
      cap[dev][lg].store(c, std::memory_order_relaxed);
    }
    if (trailing <= c - 1) return 1u << lg;
  }
  return 1;
}

template <typename F>
int run_fused(cudaStream_t s, F* w, long long m, long long n, long long ld, long long steps, long long* perm, F* coeff,
              long long* pivots, long long* status, unsigned char* ws) {
  const FusedLayout L = fused_layout(n, sizeof(F));
  FusedArgs<F> a;
  a.w = w;
  a.m = m;
  a.n = n;
  a.ld = ld;
  a.perm = perm;
  a.coeff = coeff;
  a.pivots = pivots;
  a.status = status;
  a.norms = reinterpret_cast<F*>(ws + L.norms);
  a.rec = reinterpret_cast<StepRecord<F>*>(ws + L.rec);
  a.done = reinterpret_cast<unsigned*>(ws + L.done);
  static std::atomic<unsigned long long> raised_first{0}, raised_step{0}, raised_cluster{0};
  const unsigned smem = sizeof(ColSmem<F>);
  T4A_TRY(allow_smem(k_col_first<F>, smem, raised_first));
  T4A_TRY(allow_smem(k_col_step<F>, smem, raised_step));
  const unsigned csmem = cluster_smem(smem);
  T4A_TRY(allow_smem(k_col_step_cluster<F>, csmem, raised_cluster));
  k_init_perm<<<dim3(static_cast<unsigned>((n + kFlatThreads - 1) / kFlatThreads)), dim3(kFlatThreads), 0, s>>>(
      perm, n, n, a.done);
  if (steps == 0) return runtime::check_launch();
  const unsigned swap_grid = static_cast<unsigned>(m < 148ll * 8 * kFlatThreads ? (m + kFlatThreads - 1) / kFlatThreads
                                                                                : 148 * 8);
  T4A_TRY(chain_launch(k_col_first<F>, dim3(static_cast<unsigned>(n)), dim3(kColThreads), smem, s, a));
  // The first pass and every column pass end with the next step's pivot (last block).
  for (long long step = 0; step < steps; ++step) {
    T4A_TRY(chain_launch(k_fused_swap<F>, dim3(swap_grid), dim3(kFlatThreads), 0, s, a, step));
    const long long trailing = n - step - 1;
    if (trailing <= 0) continue;
    const int next_norm = step + 1 < steps ? 1 : 0;
    const unsigned csize = column_cluster_size(k_col_step_cluster<F>, csmem, trailing);
    if (csize > 1)
      T4A_TRY(chain_launch_clustered(k_col_step_cluster<F>, csize, dim3(static_cast<unsigned>(trailing) * csize),
                                     dim3(kColThreads), csmem, s, a, step, next_norm, csize));
    else
      T4A_TRY(chain_launch(k_col_step<F>, dim3(static_cast<unsigned>(trailing)), dim3(kColThreads), smem, s, a,
                           step, next_norm));
  }
  return runtime::check_launch();
}

// Q formation through the column pass: identity, then for step = k-1 .. 0 one block per
// column of Q applies reflector `step` (dot and update phases, the primitives' bits).
template <typename F>
int run_form_q(cudaStream_t s, const F* w, long long m, long long ld, long long w_span, const F* coeff, F* q,
               long long qld, long long k, long long q_span, long long* status) {
  FusedArgs<F> a{};
  a.w = const_cast<F*>(w);
  a.m = m;
  a.n = k;
  a.ld = ld;
  a.coeff = const_cast<F*>(coeff);
  a.status = status;
  static std::atomic<unsigned long long> raised{0};
  const unsigned smem = sizeof(ColSmem<F>);
  T4A_TRY(allow_smem(k_q_step<F>, smem, raised));
  for (long long step = k - 1; step >= 0; --step)
    T4A_TRY(chain_launch(k_q_step<F>, dim3(static_cast<unsigned>(k)), dim3(kColThreads), smem, s, a, step, q, qld, k));
  return runtime::check_launch();
}

// ---- planning helpers (src/lib.rs:2460-2774) -------------------------------------
int check_algebra(int dtype) {
  return dtype == T4A_CUDA_F32 || dtype == T4A_CUDA_F64 || dtype == T4A_CUDA_C32 || dtype == T4A_CUDA_C64
             ? T4A_OK
             : T4A_ERR_UNSUPPORTED_DTYPE;
}

int check_numeric(int dtype) {
  return check_algebra(dtype) == T4A_OK || dtype == T4A_CUDA_I32 || dtype == T4A_CUDA_I64 ? T4A_OK
                                                                                          : T4A_ERR_UNSUPPORTED_DTYPE;
}

int component_size(int dtype) {
  switch (dtype) {
    case T4A_CUDA_C32: return 4;
    case T4A_CUDA_C64: return 8;
    default: return plan::dtype_size(dtype);
  }
}

int batches_of(const t4a_cuda_layout& l, int first, long long* out) {
  return plan::extent_product(l.extents + first, l.rank > first ? l.rank - first : 0, out);
}

// require_shorter (src/lib.rs:2493).
int require_shorter(const t4a_cuda_layout& shorter, const t4a_cuda_layout& matrix) {
  T4A_TRY(plan::require_matrix(matrix));
  if (shorter.rank + 1 != matrix.rank) return T4A_ERR_SHAPE_MISMATCH;
  for (int ax = 1; ax < shorter.rank; ++ax)
    if (shorter.extents[ax] != matrix.extents[ax + 1]) return T4A_ERR_SHAPE_MISMATCH;
  return T4A_OK;
}

bool same_batch(const t4a_cuda_layout& a, const t4a_cuda_layout& b) {
  if (a.rank != b.rank) return false;
  for (int ax = 2; ax < a.rank; ++ax)
    if (a.extents[ax] != b.extents[ax]) return false;
  return true;
}

// plane_launch (src/lib.rs:2472): one task per warp here.
int plane_geometry(long long tasks, t4a_launch* launch) {
  using namespace plan;
  if (tasks < 0) return T4A_ERR_NEGATIVE_COUNT;
  if (tasks == 0) {
    *launch = empty_launch();
    return T4A_OK;
  }
  unsigned long long grid = 0;
  T4A_TRY(grid_of(static_cast<unsigned long long>(tasks), kTaskWarps, &grid));
  *launch = make_launch(grid, kTaskThreads, 1, 0, kRrqrVariant);
  return T4A_OK;
}

// flat_launch (src/lib.rs:1465), grid capped: the walks are grid-stride.
int flat_geometry(long long len, t4a_launch* launch) {
  using namespace plan;
  if (len < 0) return T4A_ERR_NEGATIVE_COUNT;
  if (len == 0) {
    *launch = empty_launch();
    return T4A_OK;
  }
  unsigned long long grid = ceil_div(static_cast<unsigned long long>(len), kFlatThreads);
  if (grid > 148ull * 64) grid = 148ull * 64;
  *launch = make_launch(grid, kFlatThreads, 1, 0, kRrqrVariant + 1);
  return T4A_OK;
}

// One block per task on the column engine (F32/F64, unit row stride, at least
// kEngineRows rows from the step).  The module's warp entries run correctly under this
// geometry too (one task per warp; the extra warps return).
bool engine_eligible(int dtype, long long rows, long long row_stride) {
  return (dtype == T4A_CUDA_F32 || dtype == T4A_CUDA_F64) && row_stride == 1 && rows >= kEngineRows;
}

int task_geometry(int dtype, long long tasks, long long rows, long long row_stride, t4a_launch* launch) {
  if (tasks > 0 && tasks <= 0x7fffffffll && engine_eligible(dtype, rows, row_stride)) {
    *launch = plan::make_launch(static_cast<unsigned long long>(tasks), kColThreads, 1, 0, kRrqrEngineVariant);
    return T4A_OK;
  }
  return plane_geometry(tasks, launch);
}

// The engine path at launch: the planned variant, and a layout and pointers that still
// qualify (the launchers take layouts by value).
template <typename F>
bool engine_runs(const t4a_launch* launch, const void* p, const void* q, long long rows, long long s0,
                 long long s1) {
  const auto a = [](const void* x) { return reinterpret_cast<unsigned long long>(x) % sizeof(F) == 0; };
  return launch->variant == kRrqrEngineVariant && s0 == 1 && s1 == 1 && rows >= kEngineRows && a(p) && a(q);
}

// Launches a column-engine kernel: one block of kColThreads per planned task, with the
// engine's shared memory (its limit raised once per device and kernel).
template <typename F, typename... KArgs, typename... Args>
int launch_engine(void (*kernel)(KArgs...), const t4a_launch* launch, cudaStream_t s, Args... args) {
  static std::atomic<unsigned long long> raised{0};
  const unsigned smem = sizeof(ColSmem<F>);
  T4A_TRY(allow_smem(kernel, smem, raised));
  kernel<<<dim3(launch->grid[0]), dim3(kColThreads), smem, s>>>(args...);
  return runtime::check_launch();
}

dim3 grid_of_launch(const t4a_launch* l) { return dim3(l->grid[0], l->grid[1] ? l->grid[1] : 1, l->grid[2] ? l->grid[2] : 1); }
dim3 block_of_launch(const t4a_launch* l) { return dim3(l->block[0], l->block[1] ? l->block[1] : 1, l->block[2] ? l->block[2] : 1); }
bool launch_empty(const t4a_launch* l) { return l->grid[0] == 0 || l->block[0] == 0; }

}  // namespace
}  // namespace t4a

using namespace t4a;
using namespace t4a::plan;
using namespace t4a::rrqr;

extern "C" {

int t4a_plan_initialize_permutation(long long n, long long len, t4a_launch* launch) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (n <= 0) return T4A_ERR_NEGATIVE_COUNT;
  return flat_geometry(len, launch);
}

int t4a_plan_column_norms(int dtype, const t4a_cuda_layout* work, long long work_len, const t4a_cuda_layout* norms,
                          long long norms_len, long long step, t4a_launch* launch) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_layout(work));
  T4A_TRY(check_layout(norms));
  T4A_TRY(check_algebra(dtype));
  T4A_TRY(require_shorter(*norms, *work));
  const long long rows = work->extents[0], cols = work->extents[1];
  if (norms->extents[0] != cols) return T4A_ERR_SHAPE_MISMATCH;
  if (step < 0 || step > cols) return T4A_ERR_SHAPE_MISMATCH;
  if (step < cols && step >= rows) return T4A_ERR_SHAPE_MISMATCH;
  T4A_TRY(require_destination(*norms));
  T4A_TRY(check_span(*work, work_len, dtype_size(dtype)));
  T4A_TRY(check_span(*norms, norms_len, component_size(dtype)));
  long long batches = 0, tasks = 0;
  T4A_TRY(batches_of(*work, 2, &batches));
  if (mul_overflows(batches, cols - step, &tasks)) return T4A_ERR_OVERFLOW;
  return task_geometry(dtype, tasks, rows - step, work->strides[0], launch);
}

int t4a_plan_select_pivot(int dtype, const t4a_cuda_layout* norms, long long norms_len,
                          const t4a_cuda_layout* permutation, long long permutation_len, long long pivots_len,
                          long long status_len, long long step, t4a_launch* launch) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_layout(norms));
  T4A_TRY(check_layout(permutation));
  if (dtype != T4A_CUDA_F32 && dtype != T4A_CUDA_F64) return T4A_ERR_UNSUPPORTED_DTYPE;
  if (norms->rank == 0 || permutation->rank != norms->rank) return T4A_ERR_SHAPE_MISMATCH;
  for (int ax = 0; ax < norms->rank; ++ax)
    if (permutation->extents[ax] != norms->extents[ax]) return T4A_ERR_SHAPE_MISMATCH;
  const long long cols = norms->extents[0];
  if (step < 0 || step > cols) return T4A_ERR_SHAPE_MISMATCH;
  long long batches = 0;
  T4A_TRY(batches_of(*norms, 1, &batches));
  if (pivots_len < batches || status_len < batches) return T4A_ERR_SHAPE_MISMATCH;
  T4A_TRY(check_span(*norms, norms_len, dtype_size(dtype)));
  T4A_TRY(check_span(*permutation, permutation_len, 8));
  return plane_geometry(batches, launch);
}

int t4a_plan_swap_columns(int dtype, const t4a_cuda_layout* work, long long work_len,
                          const t4a_cuda_layout* permutation, long long permutation_len, long long pivots_len,
                          long long step, t4a_launch* launch) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_layout(work));
  T4A_TRY(check_layout(permutation));
  T4A_TRY(check_numeric(dtype));
  T4A_TRY(require_shorter(*permutation, *work));
  const long long cols = work->extents[1];
  if (permutation->extents[0] != cols) return T4A_ERR_SHAPE_MISMATCH;
  if (step < 0 || step >= cols) return T4A_ERR_SHAPE_MISMATCH;
  T4A_TRY(require_destination(*work));
  T4A_TRY(require_destination(*permutation));
  T4A_TRY(check_span(*work, work_len, dtype_size(dtype)));
  T4A_TRY(check_span(*permutation, permutation_len, 8));
  long long batches = 0, len = 0;
  T4A_TRY(batches_of(*work, 2, &batches));
  if (pivots_len < batches) return T4A_ERR_SHAPE_MISMATCH;
  if (mul_overflows(work->extents[0], batches, &len)) return T4A_ERR_OVERFLOW;
  return flat_geometry(len, launch);
}

int t4a_plan_reflector(int dtype, const t4a_cuda_layout* work, long long work_len, const t4a_cuda_layout* coeff,
                       long long coeff_len, long long step, t4a_launch* launch) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_layout(work));
  T4A_TRY(check_layout(coeff));
  T4A_TRY(check_algebra(dtype));
  T4A_TRY(require_shorter(*coeff, *work));
  long long limit = work->extents[0] < work->extents[1] ? work->extents[0] : work->extents[1];
  if (coeff->extents[0] < limit) limit = coeff->extents[0];
  if (step < 0 || step >= limit) return T4A_ERR_SHAPE_MISMATCH;
  T4A_TRY(require_destination(*work));
  T4A_TRY(require_destination(*coeff));
  T4A_TRY(check_span(*work, work_len, dtype_size(dtype)));
  T4A_TRY(check_span(*coeff, coeff_len, dtype_size(dtype)));
  long long batches = 0;
  T4A_TRY(batches_of(*work, 2, &batches));
  return task_geometry(dtype, batches, work->extents[0] - step, work->strides[0], launch);
}

int t4a_plan_apply_reflector(int dtype, const t4a_cuda_layout* packed, long long packed_len,
                             const t4a_cuda_layout* target, long long target_len, const t4a_cuda_layout* coeff,
                             long long coeff_len, long long step, long long first_column, long long column_count,
                             t4a_launch* launch) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_layout(packed));
  T4A_TRY(check_layout(target));
  T4A_TRY(check_layout(coeff));
  T4A_TRY(check_algebra(dtype));
  T4A_TRY(require_destination(*target));
  T4A_TRY(require_matrix(*packed));
  if (packed->rank != target->rank || packed->extents[0] != target->extents[0] || !same_batch(*packed, *target))
    return T4A_ERR_SHAPE_MISMATCH;
  T4A_TRY(require_shorter(*coeff, *packed));
  if (coeff->extents[0] <= step) return T4A_ERR_SHAPE_MISMATCH;
  if (step < 0 || step >= packed->extents[0] || step >= packed->extents[1]) return T4A_ERR_SHAPE_MISMATCH;
  if (first_column < 0 || column_count < 0) return T4A_ERR_NEGATIVE_COUNT;
  long long last = 0;
  if (add_overflows(first_column, column_count, &last)) return T4A_ERR_OVERFLOW;
  if (last > target->extents[1]) return T4A_ERR_SHAPE_MISMATCH;
  T4A_TRY(check_span(*packed, packed_len, dtype_size(dtype)));
  T4A_TRY(check_span(*target, target_len, dtype_size(dtype)));
  T4A_TRY(check_span(*coeff, coeff_len, dtype_size(dtype)));
  long long batches = 0, tasks = 0;
  T4A_TRY(batches_of(*packed, 2, &batches));
  if (mul_overflows(batches, column_count, &tasks)) return T4A_ERR_OVERFLOW;
  return task_geometry(dtype, tasks, packed->extents[0] - step,
                       packed->strides[0] == 1 && target->strides[0] == 1 ? 1 : 0, launch);
}

int t4a_plan_extract_r(int dtype, const t4a_cuda_layout* work, long long work_len, const t4a_cuda_layout* r,
                       long long r_len, t4a_launch* launch) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_layout(work));
  T4A_TRY(check_layout(r));
  T4A_TRY(check_algebra(dtype));
  T4A_TRY(require_destination(*r));
  T4A_TRY(require_matrix(*work));
  T4A_TRY(require_matrix(*r));
  if (r->rank != work->rank || r->extents[1] != work->extents[1] || !same_batch(*r, *work))
    return T4A_ERR_SHAPE_MISMATCH;
  if (r->extents[0] > work->extents[0]) return T4A_ERR_SHAPE_MISMATCH;
  long long len = 0;
  T4A_TRY(element_count(*r, &len));
  T4A_TRY(check_span(*r, r_len, dtype_size(dtype)));
  T4A_TRY(check_span(*work, work_len, dtype_size(dtype)));
  return flat_geometry(len, launch);
}

int t4a_plan_prefix_rank(int dtype, const t4a_cuda_layout* r, long long r_len, long long rank_len,
                         long long status_len, double rtol, double atol, t4a_launch* launch) {
  (void)rtol;
  (void)atol;
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_layout(r));
  T4A_TRY(check_algebra(dtype));
  T4A_TRY(require_matrix(*r));
  const long long rows = r->extents[0], cols = r->extents[1];
  if (rows < 1 || cols < 1 || rows > cols) return T4A_ERR_SHAPE_MISMATCH;
  long long batches = 0;
  T4A_TRY(batches_of(*r, 2, &batches));
  if (rank_len < batches || status_len < batches) return T4A_ERR_SHAPE_MISMATCH;
  T4A_TRY(check_span(*r, r_len, dtype_size(dtype)));
  return plane_geometry(batches, launch);
}

// ---- launchers (argument lists of rrqr.cu:513-705) ---------------------------------

int t4a_launch_initialize_permutation(const t4a_launch* launch, void* stream, void* permutation, long long n,
                                      long long len) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (launch_empty(launch) || len <= 0 || n <= 0) return T4A_OK;
  k_init_perm<<<grid_of_launch(launch), block_of_launch(launch), 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<long long*>(permutation), n, len, nullptr);
  return runtime::check_launch();
}

int t4a_launch_column_norms(const t4a_launch* launch, void* stream, const void* work, void* norms, int dtype,
                            t4a_cuda_layout work_layout, t4a_cuda_layout norms_layout, long long step) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (launch_empty(launch)) return T4A_OK;
  T4A_TRY(check_algebra(dtype));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long rows = work_layout.extents[0] - step;
  if (dtype == T4A_CUDA_F64 && engine_runs<double>(launch, work, norms, rows, work_layout.strides[0], 1))
    return launch_engine<double>(k_eng_norms<double>, launch, s, static_cast<const double*>(work),
                         static_cast<double*>(norms), work_layout, norms_layout, step);
  if (dtype == T4A_CUDA_F32 && engine_runs<float>(launch, work, norms, rows, work_layout.strides[0], 1))
    return launch_engine<float>(k_eng_norms<float>, launch, s, static_cast<const float*>(work), static_cast<float*>(norms),
                         work_layout, norms_layout, step);
  k_norms<t4a_cuda_layout><<<grid_of_launch(launch), block_of_launch(launch), 0, s>>>(work, norms, dtype, work_layout,
                                                                                     norms_layout, step);
  return runtime::check_launch();
}

int t4a_launch_select_pivot(const t4a_launch* launch, void* stream, const void* norms, const void* permutation,
                            void* pivots, void* status, int dtype, t4a_cuda_layout norms_layout,
                            t4a_cuda_layout permutation_layout, long long step) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (launch_empty(launch)) return T4A_OK;
  if (dtype != T4A_CUDA_F32 && dtype != T4A_CUDA_F64) return T4A_ERR_UNSUPPORTED_DTYPE;
  k_pivot<t4a_cuda_layout><<<grid_of_launch(launch), block_of_launch(launch), 0, static_cast<cudaStream_t>(stream)>>>(
      norms, permutation, pivots, status, dtype, norms_layout, permutation_layout, step);
  return runtime::check_launch();
}

int t4a_launch_swap_columns(const t4a_launch* launch, void* stream, void* work, void* permutation,
                            const void* pivots, int dtype, t4a_cuda_layout work_layout,
                            t4a_cuda_layout permutation_layout, long long step) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (launch_empty(launch)) return T4A_OK;
  T4A_TRY(check_numeric(dtype));
  k_swap<t4a_cuda_layout><<<grid_of_launch(launch), block_of_launch(launch), 0, static_cast<cudaStream_t>(stream)>>>(
      work, permutation, pivots, dtype, work_layout, permutation_layout, step);
  return runtime::check_launch();
}

int t4a_launch_reflector(const t4a_launch* launch, void* stream, void* work, void* coeff, int dtype,
                         t4a_cuda_layout work_layout, t4a_cuda_layout coeff_layout, long long step) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (launch_empty(launch)) return T4A_OK;
  T4A_TRY(check_algebra(dtype));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long rows = work_layout.extents[0] - step;
  if (dtype == T4A_CUDA_F64 && engine_runs<double>(launch, work, coeff, rows, work_layout.strides[0], 1))
    return launch_engine<double>(k_eng_reflector<double>, launch, s, static_cast<double*>(work), static_cast<double*>(coeff),
                         work_layout, coeff_layout, step);
  if (dtype == T4A_CUDA_F32 && engine_runs<float>(launch, work, coeff, rows, work_layout.strides[0], 1))
    return launch_engine<float>(k_eng_reflector<float>, launch, s, static_cast<float*>(work), static_cast<float*>(coeff),
                         work_layout, coeff_layout, step);
  k_reflector<t4a_cuda_layout><<<grid_of_launch(launch), block_of_launch(launch), 0, s>>>(work, coeff, dtype,
                                                                                         work_layout, coeff_layout,
                                                                                         step);
  return runtime::check_launch();
}

int t4a_launch_apply_reflector(const t4a_launch* launch, void* stream, const void* packed, void* target,
                               const void* coeff, int dtype, t4a_cuda_layout packed_layout,
                               t4a_cuda_layout target_layout, t4a_cuda_layout coeff_layout, long long step,
                               long long first_column, long long column_count) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (launch_empty(launch) || column_count <= 0) return T4A_OK;
  T4A_TRY(check_algebra(dtype));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long rows = packed_layout.extents[0] - step;
  if (dtype == T4A_CUDA_F64 &&
      engine_runs<double>(launch, packed, target, rows, packed_layout.strides[0], target_layout.strides[0]))
    return launch_engine<double>(k_eng_apply<double>, launch, s, static_cast<const double*>(packed),
                         static_cast<double*>(target), static_cast<const double*>(coeff), packed_layout, target_layout,
                         coeff_layout, step, first_column, column_count);
  if (dtype == T4A_CUDA_F32 &&
      engine_runs<float>(launch, packed, target, rows, packed_layout.strides[0], target_layout.strides[0]))
    return launch_engine<float>(k_eng_apply<float>, launch, s, static_cast<const float*>(packed), static_cast<float*>(target),
                         static_cast<const float*>(coeff), packed_layout, target_layout, coeff_layout, step,
                         first_column, column_count);
  k_apply<t4a_cuda_layout><<<grid_of_launch(launch), block_of_launch(launch), 0, s>>>(
      packed, target, coeff, dtype, packed_layout, target_layout, coeff_layout, step, first_column, column_count);
  return runtime::check_launch();
}

int t4a_launch_extract_r(const t4a_launch* launch, void* stream, const void* work, void* r, int dtype,
                         t4a_cuda_layout work_layout, t4a_cuda_layout r_layout) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (launch_empty(launch)) return T4A_OK;
  T4A_TRY(check_algebra(dtype));
  k_extract_r<t4a_cuda_layout><<<grid_of_launch(launch), block_of_launch(launch), 0,
                                 static_cast<cudaStream_t>(stream)>>>(work, r, dtype, work_layout, r_layout);
  return runtime::check_launch();
}

int t4a_launch_prefix_rank(const t4a_launch* launch, void* stream, const void* r, void* rank, void* status, int dtype,
                           t4a_cuda_layout r_layout, double rtol, double atol) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (launch_empty(launch)) return T4A_OK;
  T4A_TRY(check_algebra(dtype));
  k_prefix_rank<t4a_cuda_layout><<<grid_of_launch(launch), block_of_launch(launch), 0,
                                   static_cast<cudaStream_t>(stream)>>>(r, rank, status, dtype, r_layout, rtol, atol);
  return runtime::check_launch();
}

// ---- whole factorization (fused steps) ----------------------------------------------

int t4a_rrqr_any_geometry(long long tasks, int flat, t4a_launch* launch) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (tasks < 0) return T4A_ERR_NEGATIVE_COUNT;
  if (tasks == 0) {
    *launch = plan::empty_launch();
    return T4A_OK;
  }
  if (flat) {
    unsigned long long grid = plan::ceil_div(static_cast<unsigned long long>(tasks), kFlatThreads);
    if (grid > 148ull * 64) grid = 148ull * 64;
    *launch = plan::make_launch(grid, kFlatThreads, 1, 0, 0);
  } else {
    *launch = plan::make_launch(plan::ceil_div(static_cast<unsigned long long>(tasks), kTaskWarps), kTaskThreads, 1,
                                0, 0);
  }
  return T4A_OK;
}

#define T4A_ANY_PROLOGUE                                        \
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;          \
  if (launch_empty(launch)) return T4A_OK;                      \
  const dim3 g = grid_of_launch(launch), b = block_of_launch(launch); \
  cudaStream_t s = static_cast<cudaStream_t>(stream)

int t4a_launch_column_norms_any(const t4a_launch* launch, void* stream, const void* work, void* norms, int dtype,
                                t4a_cuda_layout_any work_layout, t4a_cuda_layout_any norms_layout, long long step) {
  T4A_TRY(check_algebra(dtype));
  T4A_TRY(check_rrqr_any(work_layout, 2));
  T4A_TRY(check_rrqr_any(norms_layout, 1));
  T4A_ANY_PROLOGUE;
  k_norms<t4a_cuda_layout_any><<<g, b, 0, s>>>(work, norms, dtype, work_layout, norms_layout, step);
  return runtime::check_launch();
}

int t4a_launch_select_pivot_any(const t4a_launch* launch, void* stream, const void* norms, const void* permutation,
                                void* pivots, void* status, int dtype, t4a_cuda_layout_any norms_layout,
                                t4a_cuda_layout_any permutation_layout, long long step) {
  if (dtype != T4A_CUDA_F32 && dtype != T4A_CUDA_F64) return T4A_ERR_UNSUPPORTED_DTYPE;
  T4A_TRY(check_rrqr_any(norms_layout, 1));
  T4A_TRY(check_rrqr_any(permutation_layout, 1));
  T4A_ANY_PROLOGUE;
  k_pivot<t4a_cuda_layout_any><<<g, b, 0, s>>>(norms, permutation, pivots, status, dtype, norms_layout, permutation_layout, step);
  return runtime::check_launch();
}

int t4a_launch_swap_columns_any(const t4a_launch* launch, void* stream, void* work, void* permutation,
                                const void* pivots, int dtype, t4a_cuda_layout_any work_layout,
                                t4a_cuda_layout_any permutation_layout, long long step) {
  T4A_TRY(check_numeric(dtype));
  T4A_TRY(check_rrqr_any(work_layout, 2));
  T4A_TRY(check_rrqr_any(permutation_layout, 1));
  T4A_ANY_PROLOGUE;
  k_swap<t4a_cuda_layout_any><<<g, b, 0, s>>>(work, permutation, pivots, dtype, work_layout, permutation_layout, step);
  return runtime::check_launch();
}

int t4a_launch_reflector_any(const t4a_launch* launch, void* stream, void* work, void* coeff, int dtype,
                             t4a_cuda_layout_any work_layout, t4a_cuda_layout_any coeff_layout, long long step) {
  T4A_TRY(check_algebra(dtype));
  T4A_TRY(check_rrqr_any(work_layout, 2));
  T4A_TRY(check_rrqr_any(coeff_layout, 1));
  T4A_ANY_PROLOGUE;
  k_reflector<t4a_cuda_layout_any><<<g, b, 0, s>>>(work, coeff, dtype, work_layout, coeff_layout, step);
  return runtime::check_launch();
}

int t4a_launch_apply_reflector_any(const t4a_launch* launch, void* stream, const void* packed, void* target,
                                   const void* coeff, int dtype, t4a_cuda_layout_any packed_layout,
                                   t4a_cuda_layout_any target_layout, t4a_cuda_layout_any coeff_layout,
                                   long long step, long long first_column, long long column_count) {
  T4A_TRY(check_algebra(dtype));
  T4A_TRY(check_rrqr_any(packed_layout, 2));
  T4A_TRY(check_rrqr_any(target_layout, 2));
  T4A_TRY(check_rrqr_any(coeff_layout, 1));
  T4A_ANY_PROLOGUE;
  k_apply<t4a_cuda_layout_any><<<g, b, 0, s>>>(packed, target, coeff, dtype, packed_layout, target_layout, coeff_layout, step,
                              first_column, column_count);
  return runtime::check_launch();
}

int t4a_launch_extract_r_any(const t4a_launch* launch, void* stream, const void* work, void* r, int dtype,
                             t4a_cuda_layout_any work_layout, t4a_cuda_layout_any r_layout) {
  T4A_TRY(check_algebra(dtype));
  T4A_TRY(check_rrqr_any(work_layout, 2));
  T4A_TRY(check_rrqr_any(r_layout, 2));
  T4A_ANY_PROLOGUE;
  k_extract_r<t4a_cuda_layout_any><<<g, b, 0, s>>>(work, r, dtype, work_layout, r_layout);
  return runtime::check_launch();
}

int t4a_launch_prefix_rank_any(const t4a_launch* launch, void* stream, const void* r, void* rank, void* status,
                               int dtype, t4a_cuda_layout_any r_layout, double rtol, double atol) {
  T4A_TRY(check_algebra(dtype));
  T4A_TRY(check_rrqr_any(r_layout, 2));
  T4A_ANY_PROLOGUE;
  k_prefix_rank<t4a_cuda_layout_any><<<g, b, 0, s>>>(r, rank, status, dtype, r_layout, rtol, atol);
  return runtime::check_launch();
}
#undef T4A_ANY_PROLOGUE

int t4a_rrqr_workspace_bytes(int dtype, const t4a_cuda_layout* work, size_t* bytes) {
  if (work == nullptr || bytes == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_layout(work));
  if (dtype != T4A_CUDA_F32 && dtype != T4A_CUDA_F64) return T4A_ERR_UNSUPPORTED_DTYPE;
  T4A_TRY(require_matrix(*work));
  *bytes = fused_layout(work->extents[1], dtype_size(dtype)).total;
  return T4A_OK;
}

int t4a_rrqr(void* stream, int dtype, void* work, const t4a_cuda_layout* work_layout, long long work_len,
             long long steps, void* permutation, void* coeff, void* pivots, void* status, void* workspace,
             size_t workspace_bytes) {
  if (work_layout == nullptr || work == nullptr || permutation == nullptr || coeff == nullptr || pivots == nullptr ||
      status == nullptr)
    return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_layout(work_layout));
  if (dtype != T4A_CUDA_F32 && dtype != T4A_CUDA_F64) return T4A_ERR_UNSUPPORTED_DTYPE;
  if (work_layout->rank != 2) return T4A_ERR_RANK_OUT_OF_RANGE;
  const long long m = work_layout->extents[0], n = work_layout->extents[1];
  // One column-major matrix: unit row stride, columns apart by at least a column.
  if (work_layout->strides[0] != 1 || work_layout->strides[1] < m) return T4A_ERR_INVALID_STRIDE;
  if (steps < 0 || steps > (m < n ? m : n)) return T4A_ERR_SHAPE_MISMATCH;
  T4A_TRY(check_span(*work_layout, work_len, dtype_size(dtype)));
  size_t need = 0;
  T4A_TRY(t4a_rrqr_workspace_bytes(dtype, work_layout, &need));
  if (workspace == nullptr || workspace_bytes < need) return T4A_ERR_WORKSPACE;
  // The chain passes read columns with bulk copies placed by address modulo 16, so the
  // matrix (and the int64 status word) must be naturally aligned.
  if (reinterpret_cast<unsigned long long>(work) % dtype_size(dtype) != 0 ||
      reinterpret_cast<unsigned long long>(status) % 8 != 0)
    return T4A_ERR_INVALID_STRIDE;
  if (m == 0 || n == 0) return T4A_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto* ws = static_cast<unsigned char*>(workspace);
  auto* perm = static_cast<long long*>(permutation);
  auto* piv = static_cast<long long*>(pivots);
  auto* st = static_cast<long long*>(status);
  const long long ld = work_layout->strides[1];
  if (dtype == T4A_CUDA_F64)
    return run_fused<double>(s, static_cast<double*>(work) + work_layout->offset, m, n, ld, steps, perm,
                             static_cast<double*>(coeff), piv, st, ws);
  return run_fused<float>(s, static_cast<float*>(work) + work_layout->offset, m, n, ld, steps, perm,
                          static_cast<float*>(coeff), piv, st, ws);
}

// plan_identity_shifted (src/lib.rs:2158): out(i, j, ..) = (i == start + j).
int t4a_plan_identity_shifted(int dtype, const t4a_cuda_layout* out, long long out_len, long long start,
                              t4a_launch* launch) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_layout(out));
  T4A_TRY(check_numeric(dtype));
  T4A_TRY(require_destination(*out));
  T4A_TRY(require_matrix(*out));
  if (start < 0) return T4A_ERR_NEGATIVE_COUNT;
  long long end = 0;
  if (__builtin_add_overflow(start, out->extents[1], &end)) return T4A_ERR_OVERFLOW;
  long long len = 0;
  T4A_TRY(element_count(*out, &len));
  T4A_TRY(check_span(*out, out_len, dtype_size(dtype)));
  return flat_geometry(len, launch);
}

int t4a_launch_identity_shifted(const t4a_launch* launch, void* stream, void* out, int dtype,
                                t4a_cuda_layout out_layout, long long start) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_numeric(dtype));
  if (out_layout.rank < 2 || out_layout.rank > T4A_CUDA_MAX_RANK) return T4A_ERR_RANK_OUT_OF_RANGE;
  if (launch_empty(launch)) return T4A_OK;
  if (out == nullptr) return T4A_ERR_NULL_ARGUMENT;
  k_identity<<<grid_of_launch(launch), block_of_launch(launch), 0, static_cast<cudaStream_t>(stream)>>>(
      out, dtype, out_layout, start);
  return runtime::check_launch();
}

int t4a_launch_identity_shifted_any(const t4a_launch* launch, void* stream, void* out, int dtype,
                                    t4a_cuda_layout_any out_layout, long long start) {
  if (launch == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_numeric(dtype));
  T4A_TRY(check_rrqr_any(out_layout, 2));
  if (launch_empty(launch)) return T4A_OK;
  if (out == nullptr) return T4A_ERR_NULL_ARGUMENT;
  k_identity_any<<<grid_of_launch(launch), block_of_launch(launch), 0, static_cast<cudaStream_t>(stream)>>>(
      out, dtype, out_layout, start);
  return runtime::check_launch();
}

// Q formation of the RRQR epilogue as the reference bench drives it
// (examples/bench_kernels.rs:2560-2590): q = identity_shifted(start 0), then
// apply_reflector for step = k-1 .. 0 over all k columns of q, the reflectors read from
// the factorized `work` and `coeff`; k = the columns of q.
int t4a_rrqr_form_q(void* stream, int dtype, const void* work, const t4a_cuda_layout* work_layout,
                    long long work_len, const void* coeff, const t4a_cuda_layout* coeff_layout, long long coeff_len,
                    void* q, const t4a_cuda_layout* q_layout, long long q_len, long long* status) {
  if (work_layout == nullptr || coeff_layout == nullptr || q_layout == nullptr) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_algebra(dtype));
  t4a_launch l;
  T4A_TRY(t4a_plan_identity_shifted(dtype, q_layout, q_len, 0, &l));
  const long long k = q_layout->extents[1];
  for (long long step = k - 1; step >= 0; --step) {
    t4a_launch a;
    T4A_TRY(t4a_plan_apply_reflector(dtype, work_layout, work_len, q_layout, q_len, coeff_layout, coeff_len, step, 0,
                                     k, &a));
  }
  if (q == nullptr || (k > 0 && (work == nullptr || coeff == nullptr))) return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(t4a_launch_identity_shifted(&l, stream, q, dtype, *q_layout, 0));
  // The column-pass route: F32/F64 column-major matrices (row stride 1), contiguous
  // coefficients, naturally aligned buffers and a status word.
  const int es = dtype_size(dtype);
  const auto aligned = [es](const void* p, long long off) {
    return ((reinterpret_cast<unsigned long long>(p) + static_cast<unsigned long long>(off) * es) % es) == 0;
  };
  if ((dtype == T4A_CUDA_F32 || dtype == T4A_CUDA_F64) && status != nullptr && k > 0 && work_layout->rank == 2 &&
      q_layout->rank == 2 && work_layout->strides[0] == 1 && q_layout->strides[0] == 1 &&
      work_layout->strides[1] > 0 && q_layout->strides[1] > 0 && coeff_layout->rank == 1 &&
      (coeff_layout->strides[0] == 1 || coeff_layout->extents[0] <= 1) && aligned(work, work_layout->offset) &&
      aligned(q, q_layout->offset) && aligned(coeff, coeff_layout->offset) &&
      (reinterpret_cast<unsigned long long>(status) & 7ull) == 0) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const long long m = work_layout->extents[0];
    if (dtype == T4A_CUDA_F64)
      return run_form_q<double>(s, static_cast<const double*>(work) + work_layout->offset, m, work_layout->strides[1],
                                work_len - work_layout->offset, static_cast<const double*>(coeff) + coeff_layout->offset,
                                static_cast<double*>(q) + q_layout->offset, q_layout->strides[1], k,
                                q_len - q_layout->offset, status);
    return run_form_q<float>(s, static_cast<const float*>(work) + work_layout->offset, m, work_layout->strides[1],
                             work_len - work_layout->offset, static_cast<const float*>(coeff) + coeff_layout->offset,
                             static_cast<float*>(q) + q_layout->offset, q_layout->strides[1], k,
                             q_len - q_layout->offset, status);
  }
  for (long long step = k - 1; step >= 0; --step) {
    t4a_launch a;
    T4A_TRY(t4a_plan_apply_reflector(dtype, work_layout, work_len, q_layout, q_len, coeff_layout, coeff_len, step, 0,
                                     k, &a));
    T4A_TRY(t4a_launch_apply_reflector(&a, stream, work, q, coeff, dtype, *work_layout, *q_layout, *coeff_layout,
                                       step, 0, k));
  }
  return T4A_OK;
}

// Faults of the column-engine primitives since the last call (bit 1: a bounded wait ran
// out and a task's outputs were left unwritten); reading clears them.  Synchronizes the
// current device.
int t4a_rrqr_primitive_faults(unsigned long long* faults) {
  if (faults == nullptr) return T4A_ERR_NULL_ARGUMENT;
  unsigned long long zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(faults, g_engine_faults, sizeof(zero));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_engine_faults, &zero, sizeof(zero));
  if (e != cudaSuccess) {
    runtime::last_error() = static_cast<int>(e);
    return T4A_ERR_CUDA;
  }
  return T4A_OK;
}

}  // extern "C"
