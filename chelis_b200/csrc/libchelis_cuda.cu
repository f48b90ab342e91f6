// libchelis_cuda.cu -- the library is compiled as one translation unit so
// that device globals (the bounded-wait error word) have a single
// definition without relocatable device code.
#include "runtime.cu"
#include "gemm_tf32x3.cu"
#include "gemm_f64.cu"
#include "host_gemm.cu"
#include "rows.cu"
#include "chain.cu"
#include "portfolio.cu"
#include "mlp.cu"
#include "attention.cu"
#include "block.cu"
#include "abi.cu"
#include "chain_noalloc.cu"
#include "fused.cu"
#include "fused_jit.cu"
#include "activations.cu"
#include "dp.cu"
