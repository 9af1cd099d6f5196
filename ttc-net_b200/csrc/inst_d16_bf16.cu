// Kernel instantiations for h_dim = u_dim = 16, __nv_bfloat16 activations.
#define TTC_DEFINE_LAUNCHERS
#include "lqr_launch.cuh"

TTC_INSTANTIATE(16, 16, __nv_bfloat16)
