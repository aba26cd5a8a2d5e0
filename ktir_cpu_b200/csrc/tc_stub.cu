// Placeholder for the attention entry point until fmha_tcgen05.cu lands.
#include <cuda_runtime.h>
#include "../../include/ktir_b200.h"
extern "C" int ktir_fmha_f16(const KtirFmhaDesc*, void*) { return KTIR_ERR_UNSUPPORTED; }
