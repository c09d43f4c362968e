// tjb200.cu -- single translation unit of libtjb200.so (keeps the device
// status word and all kernels in one module without relocatable device code).
#include "runtime.cu"
#include "layernorm.cu"
#include "gemm.cu"
#include "gemm_ln.cu"
#include "attention.cu"
#include "ffn.cu"
#include "ffn_fused.cu"
#include "forward_small.cu"
