// tcgen05 implicit-GEMM modulated conv (f16): placeholder until the kernel lands.
#include "tpmd_internal.h"

namespace tpmd {
bool conv_tc_supported(bool, int, int) { return false; }
cudaError_t launch_conv_tc(bool, const conv_params &, cudaStream_t) { return cudaErrorNotSupported; }
}  // namespace tpmd
