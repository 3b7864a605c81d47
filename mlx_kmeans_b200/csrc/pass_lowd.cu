// pass_lowd.cu -- placeholder until the specialised low-dimensional pass lands.
#include "kmc_internal.h"
namespace kmc {
cudaError_t launch_pass_lowd(PassArgs, cudaStream_t) { return cudaErrorNotSupported; }
}  // namespace kmc
