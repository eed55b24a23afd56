// Causal GQA prefill on the 5th-generation tensor cores (tcgen05 + TMA + TMEM).
#include "b2_common.cuh"
#include "prefill.h"

namespace b2 {

int launch_prefill_sm100(const PrefillArgs& a, uint32_t batch, cudaStream_t stream) {
    (void)a;
    (void)batch;
    (void)stream;
    return B2_ERR_UNSUPPORTED;
}

}  // namespace b2
