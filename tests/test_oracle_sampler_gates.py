"""The sampler-gate oracle (oracle.front.sampler_gates), no GPU: its edge cases, its
agreement with the MLX op-by-op gates where the two formulas round alike, and the
elements where they differ (log(1 + e) in fp32 against a full-precision softplus)."""

import math

import numpy as np

from oracle import front as ofront


def test_padding_clamp_and_plain_values():
    a = np.array([[-np.inf, np.inf, 0.0, 1.0]], np.float32)
    b = np.array([[-np.inf, np.inf, 0.0, 2.0]], np.float32)
    gate, log_gate, beta, tie = ofront.sampler_gates(a, b, np.zeros(4, np.float32),
                                                     np.zeros(4, np.float32))
    assert gate[0, 0] == 1.0 and log_gate[0, 0] == 0.0 and beta[0, 0] == 0.0
    assert gate[0, 1] == 0.0 and log_gate[0, 1] == np.float32(math.log(1e-6))
    assert beta[0, 1] == 1.0
    # a = 0, a_log = 0: gate = bf16(exp(-bf16(log 2))); beta = sigmoid(0) = 0.5.
    ln2 = ofront.bf(np.float32(math.log(2.0))).reshape(-1)[0]
    assert gate[0, 2] == ofront.bf(np.float32(math.exp(-float(ln2)))).reshape(-1)[0]
    assert beta[0, 2] == 0.5
    assert not tie.any()


def test_agrees_with_the_mlx_gates_except_where_log1p_matters():
    rng = np.random.default_rng(0)
    a = ofront.bf((2 * rng.standard_normal((2000, 6)) - 2).astype(np.float32))
    b = ofront.bf(rng.standard_normal((2000, 6)).astype(np.float32))
    a_log = rng.uniform(-2, 1, 6).astype(np.float32)
    dt_bias = (0.5 * rng.standard_normal(6)).astype(np.float32)
    gate, _, beta, _ = ofront.sampler_gates(a, b, a_log, dt_bias)
    g_mlx, b_mlx = ofront.gates_bf16(a, b, a_log, dt_bias)
    assert np.array_equal(beta, b_mlx)
    same = gate == g_mlx
    assert same.mean() > 0.97
    # Where they differ, the fp32 log(1 + exp(-|x|)) lost the low bits of a small
    # exp(-|x|): only for clearly negative x, and by one bf16 step at most.
    x = ofront.bf(a + ofront.bf(dt_bias))
    assert np.all(x[~same] < -2.0)
    step = np.abs(g_mlx[~same]) * 2.0 ** -7
    assert np.all(np.abs(gate[~same] - g_mlx[~same]) <= 1.01 * step)
