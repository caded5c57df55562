// Placeholder until the tcgen05 implicit-GEMM convolution lands.
#include "kernels.h"
namespace fb {
int launch_conv_tc(const ConvArgs&, void*) { return FB_ERR_UNSUPPORTED; }
}  // namespace fb
