// t4a_reduce_noalloc: a whole single-axis reduction that allocates no device memory
// and takes no workspace argument.
//
// Some callers cannot hand this library a workspace: code that runs where the CUDA
// allocator must not be touched (a cudaMalloc can synchronize the whole device and
// stall every other stream of a serving process), hosts whose device memory is all
// reserved up front by another allocator, and foreign-language callers whose binding
// has no device-allocation call at all.  For them the split reduction keeps its pass-1
// partials in a fixed array that lives in this library's module: every GPU that loads
// the library holds T4A_REDUCE_NOALLOC_SCRATCH_BYTES of device memory for it until
// the process exits.
//
// The first call on a device looks up the array's device address with that device
// current (cudaGetSymbolAddress; host code cannot use the array's name as a device
// pointer), so make that first call before any stream capture.  The address is cached
// for the life of the process: after a cudaDeviceReset of a device this library must not
// be called on that device again (the reset unloads the module and the cached address
// no longer names the array).  Devices with an ordinal of kMaxDevices or more are looked
// up on every call.  Every call on a device
// shares the one array and leaves its partials there: calls whose kernels may overlap
// on the GPU (different streams without ordering between them) race on it.  Nothing
// needs to start at zero: pass 1 writes every partial before the combine pass reads it.
#include <cuda_runtime.h>

#include <mutex>

#include "plan_common.h"
#include "runtime.h"

namespace t4a {
namespace {

static __device__ __align__(256) unsigned char t4a_reduce_scratch[T4A_REDUCE_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;

struct DeviceScratch {
  std::once_flag once;
  void* ptr = nullptr;
  cudaError_t err = cudaSuccess;
};

DeviceScratch g_scratch[kMaxDevices];

// Device address of the scratch array on the current device, looked up once per device.
int scratch_of_current_device(void** out) {
  int dev = 0;
  const cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    runtime::last_error() = static_cast<int>(e);
    return T4A_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    const cudaError_t u = cudaGetSymbolAddress(out, t4a_reduce_scratch);
    if (u != cudaSuccess) {
      runtime::last_error() = static_cast<int>(u);
      return T4A_ERR_CUDA;
    }
    return T4A_OK;
  }
  DeviceScratch& s = g_scratch[dev];
  std::call_once(s.once, [&s]() { s.err = cudaGetSymbolAddress(&s.ptr, t4a_reduce_scratch); });
  if (s.err != cudaSuccess) {
    runtime::last_error() = static_cast<int>(s.err);
    return T4A_ERR_CUDA;
  }
  *out = s.ptr;
  return T4A_OK;
}

}  // namespace
}  // namespace t4a

extern "C" int t4a_reduce_noalloc(void* stream, int dtype, int op, void* out, const t4a_cuda_layout* out_layout,
                                  long long out_len, const void* in, const t4a_cuda_layout* in_layout,
                                  long long in_len, unsigned axis, unsigned plane_width) {
  size_t need = 0;
  T4A_TRY(t4a_reduce_workspace_bytes(dtype, op, out_layout, out_len, in_layout, in_len, axis, plane_width, &need));
  if (need > static_cast<size_t>(T4A_REDUCE_NOALLOC_SCRATCH_BYTES)) return T4A_ERR_WORKSPACE;
  void* scratch = nullptr;
  if (need > 0) T4A_TRY(t4a::scratch_of_current_device(&scratch));
  return t4a_reduce(stream, dtype, op, out, out_layout, out_len, in, in_layout, in_len, axis, plane_width, scratch,
                    need);
}
