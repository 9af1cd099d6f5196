// Kernel instantiations for h_dim = 32, u_dim = 16, float activations.
#define TTC_DEFINE_LAUNCHERS
#include "lqr_launch.cuh"

TTC_INSTANTIATE(32, 16, float)
