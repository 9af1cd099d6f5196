"""ttc_b200 -- B200-native (sm_100a) LQR solve for TTC-Net's TTCLayer.

    from ttc_b200 import TTCLayer            # drop-in for `from ttc import TTCLayer`
    layer = TTCLayer(in_dim, out_dim, h_dim, num_heads, b_rank, q_rank).cuda()
    y = layer(x, T=64)

The solver is libttc_b200.so (include/ttc_b200.h), bound with ctypes.
"""
from .layer import TTCLayer, l2norm
from .solver import (LQR_SOLVER_IMPL_MAP, LQRSolveFunction, cuda_lqr_solve, fused_lqr_solve,
                     kkt_lqr_solve, lqr_solve_with_status)
from .trajectory import lqr_trajectory

__all__ = ["TTCLayer", "LQR_SOLVER_IMPL_MAP", "LQRSolveFunction", "cuda_lqr_solve",
           "fused_lqr_solve", "kkt_lqr_solve", "lqr_solve_with_status", "lqr_trajectory", "l2norm"]
