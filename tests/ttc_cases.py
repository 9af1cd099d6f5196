"""Test-case definitions shared by the golden-vector generator, the CPU tests,
the GPU parity tests and bench.py.

The five layer configurations are BASELINE.json's ``configs`` (rows N = B*L*H
after the reshape x[B,L,H,in] -> [B, L*H, in]); layer weights are drawn from a
numpy PCG64 stream with the reference's init distributions
(ttc/layers/ttc_layer.py:56-96: nn.Linear default U(-1/sqrt(fan_in), +), Bs ~ N(0,
0.02), Qs = G G^T / sqrt(h) with G ~ N(0, 0.02)), so every machine rebuilds the
same weights without shipping them.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class LayerConfig:
    name: str
    B: int
    L: int
    H: int
    in_dim: int
    out_dim: int
    h_dim: int
    rank: int
    T: int
    dtype: str        # activation dtype: "float32" or "bfloat16"
    seed: int
    backward: bool

    @property
    def num_heads(self) -> int:
        return self.H

    @property
    def rows(self) -> int:
        return self.B * self.L * self.H

    @property
    def tokens(self) -> int:
        return self.B * self.L

    @property
    def problems(self) -> int:
        return self.rows * self.H

    @property
    def width(self) -> int:
        d = self.h_dim
        return (6 * d + 1) * self.H + 2 * self.rank


CONFIGS = {
    1: LayerConfig("cfg1", 2, 128, 8, 32, 32, 16, 16, 64, "float32", 0, False),
    2: LayerConfig("cfg2", 4, 1024, 16, 64, 64, 16, 16, 64, "float32", 1, True),
    3: LayerConfig("cfg3", 8, 4096, 32, 128, 128, 32, 32, 128, "bfloat16", 2, True),
    4: LayerConfig("cfg4", 2, 8192, 32, 128, 128, 64, 64, 512, "float32", 3, True),
    5: LayerConfig("cfg5", 64, 4096, 32, 128, 128, 32, 32, 128, "bfloat16", 4, True),
}


def layer_weights(cfg: LayerConfig, seed: int | None = None) -> dict:
    """Deterministic float32 weights with the reference's init distributions."""
    rng = np.random.default_rng(1000 + (cfg.seed if seed is None else seed))
    d, r, nh = cfg.h_dim, cfg.rank, cfg.H
    b_in = 1.0 / math.sqrt(cfg.in_dim)
    b_out = 1.0 / math.sqrt(d * nh)
    w = {
        "in_proj.weight": rng.uniform(-b_in, b_in, size=(cfg.width, cfg.in_dim)),
        "out_proj.weight": rng.uniform(-b_out, b_out, size=(cfg.out_dim, d * nh)),
        "Bs": rng.normal(0.0, 0.02, size=(r, d, d)),
    }
    g = rng.normal(0.0, 0.02, size=(r, d, d))
    w["Qs"] = g @ g.transpose(0, 2, 1) / math.sqrt(d)
    return {k: v.astype(np.float32) for k, v in w.items()}


def layer_input(cfg: LayerConfig, rows: int, seed: int | None = None):
    """x ~ N(0,1) [rows, in_dim] and dy ~ N(0,1) [rows, out_dim] (float32)."""
    rng = np.random.default_rng(2000 + (cfg.seed if seed is None else seed))
    x = rng.standard_normal((rows, cfg.in_dim)).astype(np.float32)
    dy = rng.standard_normal((rows, cfg.out_dim)).astype(np.float32)
    return x, dy


def solver_inputs_synthetic(N: int, nh: int, d: int, du: int, seed: int):
    """Solver-level inputs in the style of the reference's bench generator
    (ttc/solvers/bench_lqr_solvers.py:71-101): normalised A in [0,1), B ~ N(0,1),
    PSD normalised Q/Q_f (symmetrised as in :125,127), R_inv = softplus(U[0,1)),
    h0 ~ N(0,1), log-gammas = -softplus(N(0,1)) - 1.328.  Returns float64 numpy arrays."""
    rng = np.random.default_rng(3000 + seed)

    def softplus(v):
        return np.log1p(np.exp(v))

    A = rng.random((N, nh, d))
    A = A / np.linalg.norm(A, axis=-1, keepdims=True)
    B = rng.standard_normal((N, d, du))
    Q = rng.standard_normal((N, d, d))
    Q = Q / np.linalg.norm(Q, axis=(-2, -1), keepdims=True)
    Q = Q @ Q.transpose(0, 2, 1) / math.sqrt(d)
    Qf = rng.standard_normal((N, nh, d, d))
    Qf = Qf / np.linalg.norm(Qf, axis=(-2, -1), keepdims=True)
    Qf = Qf @ Qf.transpose(0, 1, 3, 2) / math.sqrt(d)
    Rinv = softplus(rng.random((N, nh, du)))
    h0 = rng.standard_normal((N, nh, d))
    lgA = -softplus(rng.standard_normal((N, nh))) - 1.328
    lgB = -softplus(rng.standard_normal((N, nh, du))) - 1.328
    lgQ = -softplus(rng.standard_normal((N, nh, d))) - 1.328
    Q = (Q + Q.transpose(0, 2, 1)) / 2
    Qf = (Qf + Qf.transpose(0, 1, 3, 2)) / 2
    return [A, B, Q, Rinv, Qf, lgA, lgB, lgQ, h0]


SOLVER_ARG_NAMES = ["A_diag", "B", "Q", "R_inv_diag", "Q_f",
                    "log_gamma_A", "log_gamma_B", "log_gamma_Q", "h0"]
