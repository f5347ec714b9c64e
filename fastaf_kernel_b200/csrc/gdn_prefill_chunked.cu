// gdn_prefill_chunked.cu -- chunked (C=64) WY/UT Gated DeltaNet prefill on tcgen05.
// (tensor-core kernel under construction; reports unsupported until it lands)
#include "gdn_common.cuh"
#include "gdn_launch.h"

namespace gdn {

bool prefill_chunked_supported(const PrefillArgs &) { return false; }

cudaError_t launch_prefill_chunked(const PrefillArgs &, cudaStream_t) {
    return cudaErrorNotSupported;
}

}  // namespace gdn
