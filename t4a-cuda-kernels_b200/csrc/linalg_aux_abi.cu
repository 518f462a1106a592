// Exported linear-algebra auxiliary symbols of the kernel ABI that the RRQR epilogue
// uses (reference cuda/src/linalg_aux.cu:506 and its `_any` twin :960): the shifted
// identity that Q formation starts from.  Flat grid-stride walks, so any geometry is
// correct.  The module is linalg_aux.cubin, like the reference's per-file module.
#include "rrqr_entries.cuh"

using namespace t4a::rrqr::entry;

extern "C" __global__ void t4a_cuda_identity_shifted(void* out, int dtype, t4a_cuda_layout out_layout,
                                                     long long start) {
  identity_entry(out, dtype, out_layout, start);
}

extern "C" __global__ void t4a_cuda_identity_shifted_any(void* out, int dtype, t4a_cuda_layout_any out_layout,
                                                         long long start) {
  identity_entry(out, dtype, out_layout, start);
}
