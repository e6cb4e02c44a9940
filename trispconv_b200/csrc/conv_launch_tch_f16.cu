// Halo convolution kernels instantiated for __half, and the halo capacity
// (independent of the element type).
#include "conv_launch_impl.cuh"

namespace tsc {

int launch_tch_f16(const ConvArgs& a) { return detail::launch_tch<__half>(a); }

int tch_capacity(int c_out) { return detail::tch_capacity_of(c_out); }

}  // namespace tsc
