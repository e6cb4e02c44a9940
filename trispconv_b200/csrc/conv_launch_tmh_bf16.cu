// Halo convolution kernels instantiated for __nv_bfloat16.
#include "conv_launch_impl.cuh"

namespace tsc {

int launch_tmh_bf16(const ConvArgs& a) { return detail::launch_tmh<__nv_bfloat16>(a); }

}  // namespace tsc
