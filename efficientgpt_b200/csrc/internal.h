// Host-side helpers shared by the library's translation units (not part of the public C-ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/egpt_b200.h"

namespace egpt {

// Upper bound on CTAs of the lm_head/argmax kernel (sizes its workspace).
constexpr int kArgmaxMaxCtas = 1024;

// Thread-local error message; set_error returns `code` so call sites can `return set_error(...)`.
int set_error(int code, const char *fmt, ...);
void clear_error();
// Maps a CUDA launch result to EGPT_OK / EGPT_ERR_LAUNCH (with the runtime's message).
int check_launch(cudaError_t e, const char *what);
// SM count of the current device (cached per device).
int num_sms();
// Largest dynamic shared memory one CTA may opt in to on the current device (bytes).
size_t smem_limit();

// cudaLaunchKernelExC wrapper: optional programmatic-stream-serialization attribute (PDL).
template <typename... Args>
inline cudaError_t launch_kernel(const void *fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                                 const Args &...args) {
  void *argv[] = {(void *)&args...};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelExC(&cfg, fn, argv);
}

}  // namespace egpt
