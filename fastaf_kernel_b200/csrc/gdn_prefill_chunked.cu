// gdn_prefill_chunked.cu -- chunked (C = 64) Gated DeltaNet prefill on tensor cores.
// (placeholder: reports unsupported until the tensor-core kernel lands)
#include "gdn_common.cuh"
#include "gdn_launch.h"

namespace gdn {

bool prefill_chunked_supported(const PrefillArgs &) { return false; }

cudaError_t launch_prefill_chunked(const PrefillArgs &, cudaStream_t) {
    return cudaErrorNotSupported;
}

cudaError_t read_chunked_device_error(cudaStream_t, int *code, bool) {
    *code = 0;
    return cudaSuccess;
}

cudaError_t read_chunked_check_record(cudaStream_t, int rec[4]) {
    rec[0] = rec[1] = rec[2] = rec[3] = 0;
    return cudaSuccess;
}

}  // namespace gdn
