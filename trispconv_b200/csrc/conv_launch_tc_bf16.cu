// tc convolution kernels instantiated for __nv_bfloat16.
#include "conv_launch_impl.cuh"

namespace tsc {

int launch_tc_bf16(const ConvArgs& a) {
  return detail::launch_tc<__nv_bfloat16>(a.features, a.n_in, a.c_in, a.weight, a.bias, a.gather_map, a.row_order,
                                     a.k_vol, a.n_out, a.c_out, a.overflow, a.overflow_cap, a.meta, a.out, a.flags, a.epi,
                                     a.status, a.stream);
}

}  // namespace tsc
