// tcgen05 convolution: placeholder until the kernel lands; the BF16 mode falls back to nothing
// here because tc_available() reports false (the engine then runs the fp32 kernels).
#include "kk_tc.h"

namespace kk {
bool tc_available() { return false; }
cudaError_t tc_make_weights(const float*, int, int, int, TcWeights*) { return cudaErrorNotSupported; }
bool tc_supported(const ConvArgs&, const TcWeights&) { return false; }
cudaError_t tc_conv(const ConvArgs&, const TcWeights&, cudaStream_t) { return cudaErrorNotSupported; }
}  // namespace kk
