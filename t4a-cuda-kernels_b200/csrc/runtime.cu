#include "runtime.h"

namespace t4a {
namespace runtime {

int& last_error() {
  static thread_local int error = 0;
  return error;
}

}  // namespace runtime
}  // namespace t4a

extern "C" int t4a_last_cuda_error(void) { return t4a::runtime::last_error(); }
