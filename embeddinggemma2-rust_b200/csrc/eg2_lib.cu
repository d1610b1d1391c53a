// Single translation unit of libeg2_b200.so: the kernels share the device status word
// `eg2_dev_status`, which needs one definition visible to every kernel without relocatable
// device code.
#include "common.cuh"


#include "gemm_tc.cu"
#include "simt.cu"
#include "rowops.cu"
#include "attention_tc.cu"
#include "noalloc.cu"
#include "probe.cu"
#include "runtime.cu"
