// Single translation unit of libegpt_b200.so: the kernels share one device error word
// (egpt::g_device_error), which a unity build lets every kernel reach without relocatable device code.
#include "capi.cu"
#include "elementwise.cu"
#include "gemv_i8.cu"
#include "attention.cu"
#include "decode_step.cu"
#include "decode_dataflow.cu"
#include "gemv_tc.cu"
#include "sampling.cu"
#include "gemm_tc.cu"
#include "attn_prefill.cu"
#include "attn_stream.cu"
