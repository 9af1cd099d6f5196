// Kernel instantiations for h_dim = 64, u_dim = 32, float activations.
#define TTC_DEFINE_LAUNCHERS
#include "lqr_launch.cuh"

TTC_INSTANTIATE(64, 32, float)
