// Kernel instantiations for h_dim = u_dim = 64, __nv_bfloat16 activations.
#define TTC_DEFINE_LAUNCHERS
#include "lqr_launch.cuh"

TTC_INSTANTIATE(64, 64, __nv_bfloat16)
