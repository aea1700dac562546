// Fused attention entry point. The tcgen05/TMEM kernel is built in attention_sm100.cu when
// present; until then the launcher reports the request as unsupported instead of computing it
// any other way.
#include "common.cuh"
#include "launch.h"

namespace nb200 {

int launch_attention(const void*, const void*, const void*, void*, float*, int64_t, int64_t, int64_t,
                     int64_t, int, float, cudaStream_t) {
    set_error("nb200_attention: the tcgen05 attention kernel is not built in this library");
    return NB200_ERR_UNSUPPORTED;
}

}  // namespace nb200
