// Single translation unit for libharsh4b_b200.so: the kernels share device
// globals (the status word) without relocatable device code.
#include "gemv.cu"
#include "attention.cu"
#include "decode.cu"
#include "persistent.cu"
#include "sample.cu"
#include "gemm.cu"
#include "gemm_tc.cu"
#include "prefill_tc.cu"
#include "batch.cu"
#include "prefill.cu"
#include "tp.cu"
#include "lattice.cu"
