// Placeholder tensor-core entry points; replaced by gemm_tcgen05.cu / fmha.cu.
#include <cuda_runtime.h>
#include "../../include/ktir_b200.h"
extern "C" int ktir_gemm_f16(const KtirGemmDesc*, void*) { return KTIR_ERR_UNSUPPORTED; }
extern "C" int ktir_fmha_f16(const KtirFmhaDesc*, void*) { return KTIR_ERR_UNSUPPORTED; }
