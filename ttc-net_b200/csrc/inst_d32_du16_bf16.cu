// Kernel instantiations for h_dim = 32, u_dim = 16, bfloat16 activations.
#define TTC_DEFINE_LAUNCHERS
#include "lqr_launch.cuh"

TTC_INSTANTIATE(32, 16, __nv_bfloat16)
