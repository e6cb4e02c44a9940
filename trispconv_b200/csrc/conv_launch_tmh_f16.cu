// Halo convolution kernels instantiated for __half, and the halo capacity
// (independent of the element type).
#include "conv_launch_impl.cuh"

namespace tsc {

int launch_tmh_f16(const ConvArgs& a) { return detail::launch_tmh<__half>(a); }

int tmh_capacity(int c_out) { return detail::tmh_capacity_of(c_out); }

}  // namespace tsc
