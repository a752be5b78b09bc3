// tcgen05 / TMEM / TMA GEMM for sm_100a (bf16 operands, fp32 accumulate).
#include "common.cuh"
#include "internal.h"

bool gemm_tc_available() { return false; }
bool gemm_tc(const GemmArgs&, cudaStream_t) { return false; }
