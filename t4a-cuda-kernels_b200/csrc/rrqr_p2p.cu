// Row-sharded RRQR with the step's two exchanges fused into one column pass: every rank
// stores its norm parts and dot parts straight into every peer's memory over NVLink
// (CUDA IPC mappings of a region this library allocates on each GPU) and publishes each
// column's part with a flag; the block that needs a column's parts waits for that
// column's flag from every rank.  Like the single-GPU driver, a step is two launches
// on one chain (programmatic stream serialization) with no collective call or host
// round trip between them:
//   swap    flat over this rank's rows: column and permutation swap, the reflector's
//           scaling of the new column s, from the step record;
//   column  block per trailing column j: the dot part over this rank's rows (ring_dot);
//           push it to every rank and flag it; wait for column j's dot parts of every
//           rank and sum them in rank order; the update of this rank's rows; the next
//           step's norm part, pushed and flagged; wait for column j's norm parts of
//           every rank and store the combined norm.  The block that draws the last
//           ticket chooses the next pivot from the combined norms and writes the step
//           record.
// The arithmetic is rrqr_shard.cuh's, so the results equal the NCCL driver's
// (rrqr_dist.cu) bit for bit, and a world of one equals t4a_rrqr.  The blocks of one
// column pass are all resident (at most n - 1 of them, two per SM), and each block
// stores its own parts before it waits for other ranks', so no wait depends on a block
// that has not started (the host refuses a column count whose pass cannot be resident).
//
// Region of rank q (in q's memory; peers write into it):
//   norms [world][n] NormPart   rank r's part of column c at r * n + c
//   dots  [world][n] F          the same for dot parts
//   nflag [world][n]            rank r's part of column c of epoch e has landed when
//   dflag [world][n]            flag[r * n + c] >= e
//   done  [world]               rank r has read every part of call g from its region
//                               when done[r] >= g (no rank writes call g + 1's parts
//                               into a region before its owner has read call g's)
// and, written only by q: the ticket, the step record and the combined norms of the
// trailing columns (each block combines its own column's parts).  Epochs are
// (call << 32) + step + 1, so flags only grow and are never reset.  A part is
// overwritten only after its readers are done with it: a rank writes step s + 1's dot
// part of a column after its step-s column pass has ended, every block of which waited
// for every rank's norm part of its column, which each rank stores only after reading
// its step-s dot parts of that column; it writes step s + 2's norm part of a column only
// after every rank's dot part of that column for step s + 1, which a rank stores only
// after its step-s column pass, last block included, has ended.
//
// Every wait is bounded; one that runs out sets status bit 1, and every later wait of
// the call then returns at once (the results are then undefined, but nothing waits for
// good).
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>
#include <vector>

#include "plan_common.h"
#include "rrqr_shard.cuh"
#include "runtime.h"

namespace t4a {
namespace {

using namespace rrqr;

constexpr unsigned kFlagWaitLimit = 1u << 22;  // polls of 128 ns or more: about half a second at least

struct P2pLayout {
  size_t norms, dots, nflag, dflag, done, ticket, rec, cnorm, total;
};

// One layout for F32 and F64 (sized for 8-byte elements).
P2pLayout p2p_layout(long long n, int world) {
  auto up = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
  const size_t cells = static_cast<size_t>(n) * static_cast<size_t>(world);
  P2pLayout l;
  l.norms = 0;
  l.dots = up(l.norms + sizeof(NormPart<double>) * cells);
  l.nflag = up(l.dots + sizeof(double) * cells);
  l.dflag = up(l.nflag + 8 * cells);
  l.done = up(l.dflag + 8 * cells);
  l.ticket = up(l.done + 8 * static_cast<size_t>(world));
  l.rec = up(l.ticket + 16);
  l.cnorm = up(l.rec + sizeof(DistRecord<double>));
  l.total = up(l.cnorm + sizeof(double) * static_cast<size_t>(n));
  return l;
}

template <typename F>
struct P2pArgs {
  DistArgs<F> a;           // nrecv / drecv / rec point into this rank's region
  void* const* peers;      // device array: every rank's region as mapped on this GPU
  int rank;
  size_t norms, dots, nflag, dflag, done;  // region offsets
  unsigned* ticket;
  F* cnorm;                 // combined norms (column_norms form), one per column
  unsigned long long call;  // this call's number (1, 2, ...)
};

__device__ __forceinline__ unsigned long long epoch(unsigned long long call, long long step) {
  return (call << 32) + static_cast<unsigned long long>(step) + 1;
}

__device__ __forceinline__ unsigned long long load_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool stopped(const long long* status) {
  return (*reinterpret_cast<const volatile long long*>(status) & 2) != 0;
}
__device__ __forceinline__ void stop(long long* status) {
  atomicOr(reinterpret_cast<unsigned long long*>(status), 2ull);
}

template <typename F>
__device__ __forceinline__ unsigned char* region(const P2pArgs<F>& q, int r) {
  return static_cast<unsigned char*>(q.peers[r]);
}
template <typename F>
__device__ __forceinline__ const unsigned long long* own_flags(const P2pArgs<F>& q, size_t off) {
  return reinterpret_cast<const unsigned long long*>(region(q, q.rank) + off);
}

// One thread: wait until flags[r * n + c] >= target for every rank r (bounded).
template <typename F>
__device__ __forceinline__ void wait_column(const P2pArgs<F>& q, size_t off, long long c, unsigned long long target) {
  if (stopped(q.a.status)) return;
  const unsigned long long* flags = own_flags(q, off);
  for (unsigned it = 0; it < kFlagWaitLimit; ++it) {
    bool all = true;
    for (int r = 0; r < q.a.world && all; ++r) all = load_acquire_sys(flags + r * q.a.n + c) >= target;
    if (all) return;
    __nanosleep(128);
  }
  stop(q.a.status);
}

__device__ __forceinline__ void store_relaxed_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// One thread, after storing a part into every region: the part's flag in every region.
// The fence orders the part before the flags: system scope when peers read them, GPU
// scope for a world of one.
template <typename F>
__device__ __forceinline__ void flag_everywhere(const P2pArgs<F>& q, size_t off, long long cell, unsigned long long e) {
  if (q.a.world > 1) {
    __threadfence_system();
  } else {
    __threadfence();
  }
  for (int r = 0; r < q.a.world; ++r)
    store_relaxed_sys(reinterpret_cast<unsigned long long*>(region(q, r) + off) + cell, e);
}

// One thread: store this rank's part of column c into every region, then its flag.
template <typename F>
__device__ __forceinline__ void push_norm(const P2pArgs<F>& q, long long c, const NormPart<F>& p,
                                          unsigned long long e) {
  const long long cell = static_cast<long long>(q.rank) * q.a.n + c;
  for (int r = 0; r < q.a.world; ++r) reinterpret_cast<NormPart<F>*>(region(q, r) + q.norms)[cell] = p;
  flag_everywhere(q, q.nflag, cell, e);
}
template <typename F>
__device__ __forceinline__ void push_dot(const P2pArgs<F>& q, long long c, F d, unsigned long long e) {
  const long long cell = static_cast<long long>(q.rank) * q.a.n + c;
  for (int r = 0; r < q.a.world; ++r) reinterpret_cast<F*>(region(q, r) + q.dots)[cell] = d;
  flag_everywhere(q, q.dflag, cell, e);
}

__device__ __forceinline__ void chain_enter() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// After a block has pushed its norm part of column c for step s: wait for column c's
// parts of every rank and store the combined norm; the block that draws the last ticket
// then sees every trailing column's combined norm and records step s (pivot and scalars).
template <typename F>
__device__ __forceinline__ void combine_and_pivot(const P2pArgs<F>& q, long long s, long long c, ColSmem<F>& sm) {
  if (threadIdx.x == 0) {
    wait_column(q, q.nflag, c, epoch(q.call, s));
    q.cnorm[c] = combined_norm<F, false>(q.a, q.a.n, c);
    __threadfence();
    sm.last = atomicAdd(q.ticket, 1u) == gridDim.x - 1 ? 1 : 0;
  }
  __syncthreads();
  if (sm.last && threadIdx.x < 32) {
    __threadfence();
    const F* cn = q.cnorm;
    shard_pivot(q.a, s, q.a.n, 0, true, [&](long long col) { return cn[col]; });
    if (threadIdx.x == 0) *q.ticket = 0;  // rearmed for the next column pass (stream-ordered)
  }
}

template <typename F>
__global__ void __launch_bounds__(256) k_p2p_init(P2pArgs<F> q) {
  chain_enter();
  for (long long c = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; c < q.a.n;
       c += static_cast<long long>(gridDim.x) * blockDim.x)
    q.a.perm[c] = c;
}

// Step 0's norm parts, block per column, once every rank has read the previous call's
// parts from its region; the last block records step 0.
template <typename F>
__global__ void __launch_bounds__(kColThreads, 2) k_p2p_first(P2pArgs<F> q) {
  extern __shared__ __align__(128) unsigned char smem[];
  ColSmem<F>& sm = *reinterpret_cast<ColSmem<F>*>(smem);
  chain_enter();
  const long long j = blockIdx.x;
  if (threadIdx.x == 0 && !stopped(q.a.status)) {
    const unsigned long long* done = own_flags(q, q.done);
    bool ok = false;
    for (unsigned it = 0; it < kFlagWaitLimit && !ok; ++it) {
      ok = true;
      for (int r = 0; r < q.a.world && ok; ++r) ok = load_acquire_sys(done + r) >= q.call - 1;
      if (!ok) __nanosleep(128);
    }
    if (!ok) stop(q.a.status);
  }
  engine_init(sm);  // its barrier also holds the block until the wait is over
  norm_parts(q.a, sm, q.a.w + j * q.a.ld, 0, 0, F(0), false, false,
             [&](const NormPart<F>& p) { push_norm(q, j, p, epoch(q.call, 0)); });
  combine_and_pivot(q, 0, j, sm);
}

// Swap of step s over this rank's rows, from the step record.
template <typename F>
__global__ void __launch_bounds__(256) k_p2p_swap(P2pArgs<F> q, long long s) {
  chain_enter();
  const DistRecord<F> r = *q.a.rec;
  if (blockIdx.x == 0 && threadIdx.x == 0) shard_perm_swap(q.a, s, r.pivot);
  shard_swap(q.a, s, r);
}

// Column pass of step s: block per trailing column j = s + 1 + blockIdx.x.
template <typename F>
__global__ void __launch_bounds__(kColThreads, 2) k_p2p_column(P2pArgs<F> q, long long s, int next_norm) {
  extern __shared__ __align__(128) unsigned char smem[];
  ColSmem<F>& sm = *reinterpret_cast<ColSmem<F>*>(smem);
  chain_enter();
  const DistArgs<F>& a = q.a;
  const long long j = s + 1 + blockIdx.x;
  const long long lo = local_from(a, s);
  const long long rows = a.mr - lo;
  const F* v = a.w + s * a.ld + lo;
  F* t = a.w + j * a.ld + lo;
  engine_init(sm);
  F part = F(0);
  if (rows > 0) {
    Producer pr = producer_start();
    part = ring_dot(sm, pr, 0, v, t, rows, F(1), a.status, holds(a, s));
    drain(sm, pr, a.status);
  }
  if (threadIdx.x == 0) {
    push_dot(q, j, part, epoch(q.call, s));
    wait_column(q, q.dflag, j, epoch(q.call, s));
    sm.dot = combined_dot(a, a.n, j, a.coeff[s]);
  }
  __syncthreads();
  const F d = sm.dot;
  F peak = F(0);
  bool flagged = false;
  if (rows > 0) update_direct<true>(v, t, rows, d, &peak, &flagged, holds(a, s));
  if (next_norm) {
    norm_parts(a, sm, a.w + j * a.ld, local_from(a, s + 1), s + 1, peak, flagged, true,
               [&](const NormPart<F>& p) { push_norm(q, j, p, epoch(q.call, s + 1)); });
    combine_and_pivot(q, s + 1, j, sm);
  }
}

// End of a call: this rank has read every part of the call from its region.
template <typename F>
__global__ void k_p2p_leave(P2pArgs<F> q) {
  chain_enter();
  if (threadIdx.x == 0) flag_everywhere(q, q.done, q.rank, q.call);
}

// The host side of one rank's exchange: its region, every rank's region as mapped here
// (IPC), and the number of calls made so far (the same on every rank, since every rank
// makes the same calls).
struct P2pComm {
  int world = 1, rank = 0;
  long long n = 0;
  P2pLayout layout{};
  void* local = nullptr;
  std::vector<void*> peers;    // host copy; peers[rank] == local
  std::vector<bool> opened;    // IPC mappings to close
  void** dev_peers = nullptr;  // device copy
  unsigned long long calls = 0;
};

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return T4A_OK;
  runtime::last_error() = static_cast<int>(e);
  return T4A_ERR_CUDA;
}

template <typename... KArgs, typename... Args>
int chain(void (*kernel)(KArgs...), dim3 grid, dim3 block, unsigned smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
}

template <typename K>
int raise_smem(K kernel, unsigned bytes, std::atomic<unsigned long long>& raised) {
  int dev = 0;
  T4A_TRY(cuda_status(cudaGetDevice(&dev)));
  const unsigned long long bit = 1ull << (dev & 63);
  if ((raised.load(std::memory_order_relaxed) & bit) == 0) {
    T4A_TRY(cuda_status(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes)));
    raised.fetch_or(bit);
  }
  return T4A_OK;
}

template <typename F>
int run_p2p(P2pComm& c, cudaStream_t st, F* w, long long mr, long long n, long long ld, long long row0,
            long long steps, long long* perm, F* coeff, long long* pivots, long long* status) {
  static std::atomic<unsigned long long> r_first{0}, r_column{0};
  const unsigned smem = sizeof(ColSmem<F>);
  T4A_TRY(raise_smem(k_p2p_first<F>, smem, r_first));
  T4A_TRY(raise_smem(k_p2p_column<F>, smem, r_column));
  // Every block of a column pass must be resident at once (a block waits for the blocks
  // of the same column on the other ranks).
  int dev = 0, sms = 0, per_sm = 0;
  T4A_TRY(cuda_status(cudaGetDevice(&dev)));
  T4A_TRY(cuda_status(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)));
  T4A_TRY(cuda_status(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_p2p_column<F>, kColThreads, smem)));
  if (n - 1 > static_cast<long long>(sms) * per_sm) return T4A_ERR_LAUNCH_LIMIT;
  auto* base = static_cast<unsigned char*>(c.local);
  P2pArgs<F> q;
  q.a.w = w;
  q.a.mr = mr;
  q.a.n = n;
  q.a.ld = ld;
  q.a.row0 = row0;
  q.a.world = c.world;
  q.a.perm = perm;
  q.a.coeff = coeff;
  q.a.pivots = pivots;
  q.a.status = status;
  q.a.nsend = nullptr;
  q.a.dsend = nullptr;
  q.a.nrecv = reinterpret_cast<NormPart<F>*>(base + c.layout.norms);
  q.a.drecv = reinterpret_cast<F*>(base + c.layout.dots);
  q.a.rec = reinterpret_cast<DistRecord<F>*>(base + c.layout.rec);
  q.peers = c.dev_peers;
  q.rank = c.rank;
  q.norms = c.layout.norms;
  q.dots = c.layout.dots;
  q.nflag = c.layout.nflag;
  q.dflag = c.layout.dflag;
  q.done = c.layout.done;
  q.ticket = reinterpret_cast<unsigned*>(base + c.layout.ticket);
  q.cnorm = reinterpret_cast<F*>(base + c.layout.cnorm);
  q.call = c.calls;
  T4A_TRY(chain(k_p2p_init<F>, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, st, q));
  if (steps == 0) return T4A_OK;
  q.call = ++c.calls;
  T4A_TRY(chain(k_p2p_first<F>, dim3(static_cast<unsigned>(n)), dim3(kColThreads), smem, st, q));
  const long long swap_blocks = mr < 148ll * 8 * 256 ? (mr + 255) / 256 : 148ll * 8;
  for (long long s = 0; s < steps; ++s) {
    T4A_TRY(chain(k_p2p_swap<F>, dim3(static_cast<unsigned>(swap_blocks > 0 ? swap_blocks : 1)), dim3(256), 0, st, q,
                  s));
    const long long trailing = n - s - 1;
    if (trailing > 0)
      T4A_TRY(chain(k_p2p_column<F>, dim3(static_cast<unsigned>(trailing)), dim3(kColThreads), smem, st, q, s,
                    s + 1 < steps ? 1 : 0));
  }
  return chain(k_p2p_leave<F>, dim3(1), dim3(32), 0, st, q);
}

}  // namespace
}  // namespace t4a

using namespace t4a;
using namespace t4a::plan;

extern "C" {

int t4a_p2p_region_bytes(long long n, int world, size_t* bytes) {
  if (bytes == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (n < 0) return T4A_ERR_NEGATIVE_EXTENT;
  if (world < 1) return T4A_ERR_SHAPE_MISMATCH;
  *bytes = p2p_layout(n, world).total;
  return T4A_OK;
}

int t4a_p2p_create(long long n, int world, int rank, void** comm, void* ipc_handle) {
  if (comm == nullptr || ipc_handle == nullptr) return T4A_ERR_NULL_ARGUMENT;
  if (n < 0) return T4A_ERR_NEGATIVE_EXTENT;
  if (world < 1 || rank < 0 || rank >= world) return T4A_ERR_SHAPE_MISMATCH;
  auto* c = new P2pComm;
  c->world = world;
  c->rank = rank;
  c->n = n;
  c->layout = p2p_layout(n, world);
  int st = cuda_status(cudaMalloc(&c->local, c->layout.total));
  if (st == T4A_OK) st = cuda_status(cudaMemset(c->local, 0, c->layout.total));
  if (st == T4A_OK) st = cuda_status(cudaDeviceSynchronize());  // zeroed before any peer can write
  cudaIpcMemHandle_t h;
  memset(&h, 0, sizeof(h));
  if (st == T4A_OK && world > 1) st = cuda_status(cudaIpcGetMemHandle(&h, c->local));
  if (st != T4A_OK) {
    if (c->local != nullptr) cudaFree(c->local);
    delete c;
    return st;
  }
  memcpy(ipc_handle, &h, sizeof(h));
  c->peers.assign(world, nullptr);
  c->opened.assign(world, false);
  c->peers[rank] = c->local;
  *comm = c;
  return T4A_OK;
}

int t4a_p2p_open(void* comm, const void* ipc_handles) {
  if (comm == nullptr || ipc_handles == nullptr) return T4A_ERR_NULL_ARGUMENT;
  auto* c = static_cast<P2pComm*>(comm);
  if (c->dev_peers != nullptr) return T4A_ERR_SHAPE_MISMATCH;  // opened already
  const auto* hs = static_cast<const unsigned char*>(ipc_handles);
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, hs + static_cast<size_t>(r) * sizeof(h), sizeof(h));
    T4A_TRY(cuda_status(cudaIpcOpenMemHandle(&c->peers[r], h, cudaIpcMemLazyEnablePeerAccess)));
    c->opened[r] = true;
  }
  T4A_TRY(cuda_status(cudaMalloc(&c->dev_peers, sizeof(void*) * c->world)));
  return cuda_status(cudaMemcpy(c->dev_peers, c->peers.data(), sizeof(void*) * c->world, cudaMemcpyHostToDevice));
}

int t4a_p2p_destroy(void* comm) {
  if (comm == nullptr) return T4A_ERR_NULL_ARGUMENT;
  auto* c = static_cast<P2pComm*>(comm);
  int st = cuda_status(cudaDeviceSynchronize());
  for (int r = 0; r < c->world; ++r)
    if (c->opened[r]) {
      const int e = cuda_status(cudaIpcCloseMemHandle(c->peers[r]));
      if (st == T4A_OK) st = e;
    }
  if (c->dev_peers != nullptr) cudaFree(c->dev_peers);
  if (c->local != nullptr) cudaFree(c->local);
  delete c;
  return st;
}

int t4a_dist_rrqr_p2p(void* comm, void* stream, int dtype, void* work, const t4a_cuda_layout* local_layout,
                      long long work_len, long long row0, long long global_rows, long long steps, void* permutation,
                      void* coeff, void* pivots, void* status) {
  if (comm == nullptr || local_layout == nullptr || work == nullptr || permutation == nullptr || coeff == nullptr ||
      pivots == nullptr || status == nullptr)
    return T4A_ERR_NULL_ARGUMENT;
  auto* c = static_cast<P2pComm*>(comm);
  if (c->dev_peers == nullptr) return T4A_ERR_SHAPE_MISMATCH;  // t4a_p2p_open first
  T4A_TRY(check_layout(local_layout));
  if (dtype != T4A_CUDA_F32 && dtype != T4A_CUDA_F64) return T4A_ERR_UNSUPPORTED_DTYPE;
  if (local_layout->rank != 2) return T4A_ERR_RANK_OUT_OF_RANGE;
  const long long mr = local_layout->extents[0], n = local_layout->extents[1];
  if (n != c->n) return T4A_ERR_SHAPE_MISMATCH;
  if (local_layout->strides[0] != 1 || local_layout->strides[1] < mr) return T4A_ERR_INVALID_STRIDE;
  if (row0 < 0 || global_rows < 0 || row0 + mr > global_rows) return T4A_ERR_SHAPE_MISMATCH;
  if (steps < 0 || steps > (global_rows < n ? global_rows : n)) return T4A_ERR_SHAPE_MISMATCH;
  T4A_TRY(check_span(*local_layout, work_len, dtype_size(dtype)));
  const unsigned long long es = static_cast<unsigned long long>(dtype_size(dtype));
  if (reinterpret_cast<unsigned long long>(work) % es != 0 || reinterpret_cast<unsigned long long>(status) % 8 != 0)
    return T4A_ERR_INVALID_STRIDE;
  if (n == 0) return T4A_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* perm = static_cast<long long*>(permutation);
  auto* piv = static_cast<long long*>(pivots);
  auto* stt = static_cast<long long*>(status);
  const long long ld = local_layout->strides[1];
  if (dtype == T4A_CUDA_F64)
    return run_p2p<double>(*c, st, static_cast<double*>(work) + local_layout->offset, mr, n, ld, row0, steps, perm,
                           static_cast<double*>(coeff), piv, stt);
  return run_p2p<float>(*c, st, static_cast<float*>(work) + local_layout->offset, mr, n, ld, row0, steps, perm,
                        static_cast<float*>(coeff), piv, stt);
}

}  // extern "C"
