// RRQR of a tall matrix whose rows are split across GPUs (one process per GPU), with
// NCCL over NVLink for the two exchanges every step has.  The reference has no
// multi-device code; this is the row-sharded form of its step loop (reference bench
// examples/bench_kernels.rs:2398-2530): column_norms, select_pivot, swap_columns,
// reflector, apply_reflector.
//
// The step's arithmetic is rrqr_shard.cuh's.  Per step: select+swap (from the gathered
// norm parts), dot, an all-gather of the dot parts, update with the next step's norm
// parts, an all-gather of the norm parts.
//
// NCCL is loaded on first use (dlopen of libnccl.so.2), so the library loads on hosts
// without it; the entry points then return T4A_ERR_CUDA.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <atomic>
#include <mutex>

#include "plan_common.h"
#include "rrqr_shard.cuh"
#include "runtime.h"

namespace t4a {
namespace {

using namespace rrqr;

// ---- NCCL, loaded on first use ---------------------------------------------------

struct Nccl {
  bool ok = false;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_count)(const ncclComm_t, int*) = nullptr;
  ncclResult_t (*comm_user_rank)(const ncclComm_t, int*) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
};

const Nccl& nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) return;
    n.get_unique_id = reinterpret_cast<decltype(n.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    n.comm_init_rank = reinterpret_cast<decltype(n.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    n.comm_destroy = reinterpret_cast<decltype(n.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    n.comm_count = reinterpret_cast<decltype(n.comm_count)>(dlsym(h, "ncclCommCount"));
    n.comm_user_rank = reinterpret_cast<decltype(n.comm_user_rank)>(dlsym(h, "ncclCommUserRank"));
    n.all_gather = reinterpret_cast<decltype(n.all_gather)>(dlsym(h, "ncclAllGather"));
    n.ok = n.get_unique_id && n.comm_init_rank && n.comm_destroy && n.comm_count && n.comm_user_rank && n.all_gather;
  });
  return n;
}

int nccl_status(ncclResult_t r) { return r == ncclSuccess ? T4A_OK : T4A_ERR_CUDA; }

// ---- kernels ------------------------------------------------------------------------

template <typename F>
__global__ void __launch_bounds__(256) k_dist_init(DistArgs<F> a) {
  for (long long c = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; c < a.n;
       c += static_cast<long long>(gridDim.x) * blockDim.x)
    a.perm[c] = c;
}

// Step 0's norm parts: block per column.
template <typename F>
__global__ void __launch_bounds__(kColThreads, 2) k_dist_first(DistArgs<F> a) {
  extern __shared__ __align__(128) unsigned char smem[];
  ColSmem<F>& sm = *reinterpret_cast<ColSmem<F>*>(smem);
  const long long j = blockIdx.x;
  engine_init(sm);
  NormPart<F>* out = a.nsend + j;
  norm_parts(a, sm, a.w + j * a.ld, 0, 0, F(0), false, false, [&](const NormPart<F>& p) { *out = p; });
}

// Pivot of step s from the gathered parts (every block decides the same), then the swap
// of columns s and pivot over this rank's rows and the reflector's scaling.
template <typename F>
__global__ void __launch_bounds__(256) k_dist_select_swap(DistArgs<F> a, long long s) {
  __shared__ DistRecord<F> rec;
  const long long count = a.n - s;  // gathered parts cover columns s .. n-1
  if (threadIdx.x < 32) {
    const DistRecord<F> r = shard_pivot<F, 1>(a, s, count, s, blockIdx.x == 0,
                                        [&](long long c) { return combined_norm<F, false>(a, count, c - s); });
    if (lane_id() == 0) rec = r;
  }
  __syncthreads();
  shard_swap(a, s, rec);
}

// Dot parts of step s: block per trailing column (and block 0 swaps the permutation).
template <typename F>
__global__ void __launch_bounds__(kColThreads, 2) k_dist_dot(DistArgs<F> a, long long s) {
  extern __shared__ __align__(128) unsigned char smem[];
  ColSmem<F>& sm = *reinterpret_cast<ColSmem<F>*>(smem);
  const long long j = s + 1 + blockIdx.x;
  if (blockIdx.x == 0 && threadIdx.x == 0) shard_perm_swap(a, s, a.rec->pivot);
  const long long lo = local_from(a, s);
  const long long rows = a.mr - lo;
  if (rows <= 0) {
    if (threadIdx.x == 0) a.dsend[blockIdx.x] = F(0);
    return;
  }
  engine_init(sm);
  Producer pr = producer_start();
  const F d = ring_dot(sm, pr, 0, a.w + s * a.ld + lo, a.w + j * a.ld + lo, rows, F(1), a.status, holds(a, s));
  drain(sm, pr, a.status);
  if (threadIdx.x == 0) a.dsend[blockIdx.x] = d;
}

// Update of step s and the next step's norm parts: block per trailing column.
template <typename F>
__global__ void __launch_bounds__(kColThreads, 2) k_dist_update(DistArgs<F> a, long long s, int next_norm) {
  extern __shared__ __align__(128) unsigned char smem[];
  ColSmem<F>& sm = *reinterpret_cast<ColSmem<F>*>(smem);
  const long long j = s + 1 + blockIdx.x;
  const long long count = a.n - s - 1;
  engine_init(sm);
  if (threadIdx.x == 0) sm.dot = combined_dot(a, count, blockIdx.x, a.coeff[s]);
  __syncthreads();
  const F d = sm.dot;
  const long long lo = local_from(a, s);
  const long long rows = a.mr - lo;
  F* col = a.w + j * a.ld;
  F peak = F(0);
  bool flagged = false;
  if (rows > 0) update_direct<true>(a.w + s * a.ld + lo, col + lo, rows, d, &peak, &flagged, holds(a, s));
  NormPart<F>* out = a.nsend + blockIdx.x;
  if (next_norm)
    norm_parts(a, sm, col, local_from(a, s + 1), s + 1, peak, flagged, true, [&](const NormPart<F>& p) { *out = p; });
}

template <typename F>
struct DistLayout {
  size_t nsend, nrecv, dsend, drecv, rec, total;
};

template <typename F>
DistLayout<F> dist_layout(long long n, int world) {
  auto up = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
  DistLayout<F> l;
  l.nsend = 0;
  l.nrecv = up(l.nsend + sizeof(NormPart<F>) * n);
  l.dsend = up(l.nrecv + sizeof(NormPart<F>) * n * world);
  l.drecv = up(l.dsend + sizeof(F) * n);
  l.rec = up(l.drecv + sizeof(F) * n * world);
  l.total = up(l.rec + sizeof(DistRecord<F>));
  return l;
}

template <typename K>
int raise_smem(K kernel, unsigned bytes, std::atomic<unsigned long long>& raised) {
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

template <typename F>
ncclDataType_t nccl_type() {
  return sizeof(F) == 8 ? ncclFloat64 : ncclFloat32;
}

template <typename F>
int run_dist(ncclComm_t comm, cudaStream_t st, F* w, long long mr, long long n, long long ld, long long row0,
             int world, long long steps, long long* perm, F* coeff, long long* pivots, long long* status,
             unsigned char* ws) {
  const Nccl& nc = nccl();
  const DistLayout<F> L = dist_layout<F>(n, world);
  DistArgs<F> a;
  a.w = w;
  a.mr = mr;
  a.n = n;
  a.ld = ld;
  a.row0 = row0;
  a.world = world;
  a.perm = perm;
  a.coeff = coeff;
  a.pivots = pivots;
  a.status = status;
  a.nsend = reinterpret_cast<NormPart<F>*>(ws + L.nsend);
  a.nrecv = reinterpret_cast<NormPart<F>*>(ws + L.nrecv);
  a.dsend = reinterpret_cast<F*>(ws + L.dsend);
  a.drecv = reinterpret_cast<F*>(ws + L.drecv);
  a.rec = reinterpret_cast<DistRecord<F>*>(ws + L.rec);
  static std::atomic<unsigned long long> r_first{0}, r_dot{0}, r_update{0};
  const unsigned smem = sizeof(ColSmem<F>);
  T4A_TRY(raise_smem(k_dist_first<F>, smem, r_first));
  T4A_TRY(raise_smem(k_dist_dot<F>, smem, r_dot));
  T4A_TRY(raise_smem(k_dist_update<F>, smem, r_update));
  const ncclDataType_t type = nccl_type<F>();
  constexpr size_t kPartElems = sizeof(NormPart<F>) / sizeof(F);
  k_dist_init<F><<<dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, st>>>(a);
  if (steps == 0) return runtime::check_launch();
  k_dist_first<F><<<dim3(static_cast<unsigned>(n)), dim3(kColThreads), smem, st>>>(a);
  T4A_TRY(runtime::check_launch());
  T4A_TRY(nccl_status(nc.all_gather(a.nsend, a.nrecv, static_cast<size_t>(n) * kPartElems, type, comm, st)));
  const long long swap_blocks = mr < 148ll * 8 * 256 ? (mr + 255) / 256 : 148ll * 8;
  for (long long s = 0; s < steps; ++s) {
    k_dist_select_swap<F><<<dim3(static_cast<unsigned>(swap_blocks > 0 ? swap_blocks : 1)), dim3(256), 0, st>>>(a, s);
    const long long trailing = n - s - 1;
    if (trailing <= 0) continue;
    k_dist_dot<F><<<dim3(static_cast<unsigned>(trailing)), dim3(kColThreads), smem, st>>>(a, s);
    T4A_TRY(runtime::check_launch());
    T4A_TRY(nccl_status(nc.all_gather(a.dsend, a.drecv, static_cast<size_t>(trailing), type, comm, st)));
    const int next = s + 1 < steps ? 1 : 0;
    k_dist_update<F><<<dim3(static_cast<unsigned>(trailing)), dim3(kColThreads), smem, st>>>(a, s, next);
    T4A_TRY(runtime::check_launch());
    if (next)
      T4A_TRY(nccl_status(nc.all_gather(a.nsend, a.nrecv, static_cast<size_t>(trailing) * kPartElems, type, comm,
                                        st)));
  }
  return runtime::check_launch();
}

}  // namespace
}  // namespace t4a

using namespace t4a;
using namespace t4a::plan;

extern "C" {

int t4a_dist_unique_id(void* id) {
  if (id == nullptr) return T4A_ERR_NULL_ARGUMENT;
  const Nccl& nc = nccl();
  if (!nc.ok) return T4A_ERR_CUDA;
  return nccl_status(nc.get_unique_id(static_cast<ncclUniqueId*>(id)));
}

int t4a_dist_comm_init(void** comm, const void* id, int world, int rank) {
  if (comm == nullptr || id == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (world < 1 || rank < 0 || rank >= world) return T4A_ERR_SHAPE_MISMATCH;
  const Nccl& nc = nccl();
  if (!nc.ok) return T4A_ERR_CUDA;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclComm_t c = nullptr;
  T4A_TRY(nccl_status(nc.comm_init_rank(&c, world, uid, rank)));
  *comm = c;
  return T4A_OK;
}

int t4a_dist_comm_destroy(void* comm) {
  if (comm == nullptr) return T4A_ERR_NULL_ARGUMENT;
  const Nccl& nc = nccl();
  if (!nc.ok) return T4A_ERR_CUDA;
  return nccl_status(nc.comm_destroy(static_cast<ncclComm_t>(comm)));
}

int t4a_dist_rrqr_workspace_bytes(int dtype, long long n, int world, size_t* bytes) {
  if (bytes == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (n < 0) return T4A_ERR_NEGATIVE_EXTENT;
  if (world < 1) return T4A_ERR_SHAPE_MISMATCH;
  if (dtype == T4A_CUDA_F64) {
    *bytes = dist_layout<double>(n, world).total;
  } else if (dtype == T4A_CUDA_F32) {
    *bytes = dist_layout<float>(n, world).total;
  } else {
    return T4A_ERR_UNSUPPORTED_DTYPE;
  }
  return T4A_OK;
}

int t4a_dist_rrqr(void* comm, void* stream, int dtype, void* work, const t4a_cuda_layout* local_layout,
                  long long work_len, long long row0, long long global_rows, long long steps, void* permutation,
                  void* coeff, void* pivots, void* status, void* workspace, size_t workspace_bytes) {
  if (comm == nullptr || local_layout == nullptr || work == nullptr || permutation == nullptr || coeff == nullptr ||
      pivots == nullptr || status == nullptr)
    return T4A_ERR_NULL_ARGUMENT;
  T4A_TRY(check_layout(local_layout));
  if (dtype != T4A_CUDA_F32 && dtype != T4A_CUDA_F64) return T4A_ERR_UNSUPPORTED_DTYPE;
  if (local_layout->rank != 2) return T4A_ERR_RANK_OUT_OF_RANGE;
  const long long mr = local_layout->extents[0], n = local_layout->extents[1];
  if (local_layout->strides[0] != 1 || local_layout->strides[1] < mr) return T4A_ERR_INVALID_STRIDE;
  if (row0 < 0 || global_rows < 0 || row0 + mr > global_rows) return T4A_ERR_SHAPE_MISMATCH;
  if (steps < 0 || steps > (global_rows < n ? global_rows : n)) return T4A_ERR_SHAPE_MISMATCH;
  T4A_TRY(check_span(*local_layout, work_len, dtype_size(dtype)));
  const Nccl& nc = nccl();
  if (!nc.ok) return T4A_ERR_CUDA;
  int world = 0, rank = 0;
  T4A_TRY(nccl_status(nc.comm_count(static_cast<ncclComm_t>(comm), &world)));
  T4A_TRY(nccl_status(nc.comm_user_rank(static_cast<ncclComm_t>(comm), &rank)));
  size_t need = 0;
  T4A_TRY(t4a_dist_rrqr_workspace_bytes(dtype, n, world, &need));
  if (workspace == nullptr || workspace_bytes < need) return T4A_ERR_WORKSPACE;
  const unsigned long long es = static_cast<unsigned long long>(dtype_size(dtype));
  if (reinterpret_cast<unsigned long long>(work) % es != 0 || reinterpret_cast<unsigned long long>(status) % 8 != 0)
    return T4A_ERR_INVALID_STRIDE;
  if (n == 0) return T4A_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* ws = static_cast<unsigned char*>(workspace);
  auto* perm = static_cast<long long*>(permutation);
  auto* piv = static_cast<long long*>(pivots);
  auto* stt = static_cast<long long*>(status);
  const long long ld = local_layout->strides[1];
  if (dtype == T4A_CUDA_F64)
    return run_dist<double>(static_cast<ncclComm_t>(comm), st, static_cast<double*>(work) + local_layout->offset, mr, n,
                            ld, row0, world, steps, perm, static_cast<double*>(coeff), piv, stt, ws);
  return run_dist<float>(static_cast<ncclComm_t>(comm), st, static_cast<float*>(work) + local_layout->offset, mr, n, ld,
                         row0, world, steps, perm, static_cast<float*>(coeff), piv, stt, ws);
}

}  // extern "C"
