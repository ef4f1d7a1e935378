#include "fa_ptx.cuh"
#include "fa_internal.h"
namespace fa {
size_t bwd_workspace_bytes(const fa_bwd_args_t* a) { return 0; }
int launch_bwd(const fa_bwd_args_t* a, void* ws, size_t ws_bytes, int* err, cudaStream_t st) {
  return FA_ERR_UNSUPPORTED;
}
}  // namespace fa
