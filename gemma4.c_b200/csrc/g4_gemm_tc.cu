// g4_gemm_tc.cu — prefill int8 GEMM on the 5th-generation tensor cores
// (tcgen05, TMEM accumulators). Not yet enabled: every shape reports
// "unsupported" and the engine uses the SIMT GEMM.
#include "g4_common.cuh"
#include "g4_internal.h"

bool g4_gemm_tc_supported(const GemmArgs &a) {
    (void)a;
    return false;
}

cudaError_t g4_launch_gemm_tc(const GemmArgs &a, cudaStream_t st, bool pdl) {
    (void)a;
    (void)st;
    (void)pdl;
    return cudaErrorNotSupported;
}
