// IQ codebook encoders (src/quant_iq.rs) for sm_100a.
#include "kernels.cuh"

namespace shc {

bool iq_supported(uint32_t type) {
    (void)type;
    return false;
}

cudaError_t launch_iq(uint32_t type, const EncArgs &a, const IqTables &iq, int num_sms, cudaStream_t st) {
    (void)type; (void)a; (void)iq; (void)num_sms; (void)st;
    return cudaErrorNotSupported;
}

}  // namespace shc
