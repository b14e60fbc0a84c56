"""One hybrid decode cache-step on the host cores (TEST INFRASTRUCTURE / CPU baseline).

The reference's decode step cannot run here (MLX is Darwin-only); its own CPU
code for this path is the float64 NumPy oracles, restated in oracle.gdn and
oracle.attention. This module times that math on a bounded sample of
sequences: for each sampled sequence, every GDN layer advances its recurrent
state one token and every attention layer appends one K/V row and attends
over the sequence's whole context, exactly the per-token work of the GPU step.

Only bench.py (cpu_baseline, --impl reference) and tests import this.
"""

from __future__ import annotations

import os
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from . import attention as oatt
from . import gdn as ogdn


class SampledSequence:
    """Host caches of one sequence: a state per GDN layer and a K/V buffer."""

    def __init__(self, rng: np.random.Generator, length: int, n_gdn: int, n_attn: int,
                 Hk: int, Hv: int, dk: int, dv: int, Hq: int, Hkv: int, D: int,
                 capacity: int):
        self.length = length
        self.states = [np.zeros((1, Hv, dv, dk), np.float32) for _ in range(n_gdn)]
        cap = length + capacity
        # One K/V buffer per attention layer would multiply host memory by the
        # layer count; the math per layer is identical, so the layers share one
        # buffer and each writes the step's new row at the same position.
        self.k = rng.standard_normal((cap, Hkv, D)).astype(np.float32)
        self.v = rng.standard_normal((cap, Hkv, D)).astype(np.float32)
        self.shape = (Hk, Hv, dk, dv, Hq, Hkv, D)
        self.n_attn = n_attn

    def step(self, rng: np.random.Generator, layers: list, scale: float) -> None:
        Hk, Hv, dk, dv, Hq, Hkv, D = self.shape
        g_i = a_i = 0
        pos = self.length
        for is_attn in layers:
            if is_attn:
                q = rng.standard_normal((Hq, D))
                self.k[pos] = rng.standard_normal((Hkv, D))
                self.v[pos] = rng.standard_normal((Hkv, D))
                oatt.decode_attention(q, self.k[:pos + 1], self.v[:pos + 1], scale)
                a_i += 1
            else:
                q = rng.standard_normal((1, Hk, dk))
                k = rng.standard_normal((1, Hk, dk))
                v = rng.standard_normal((1, Hv, dv))
                g = np.full((1, Hv), 0.9)
                beta = np.full((1, Hv), 0.5)
                _, s = ogdn.token_step(q, k, v, g, beta, self.states[g_i])
                self.states[g_i] = s.astype(np.float32)
                g_i += 1
        self.length += 1


def run_sample(seqs: list, layers: list, scale: float, threads: int, seed: int) -> float:
    """Advance every sampled sequence one token; returns elapsed seconds."""
    rngs = [np.random.default_rng(seed + i) for i in range(len(seqs))]
    start = time.perf_counter()
    if threads <= 1:
        for s, r in zip(seqs, rngs):
            s.step(r, layers, scale)
    else:
        with ThreadPoolExecutor(max_workers=threads) as pool:
            list(pool.map(lambda pair: pair[0].step(pair[1], layers, scale), zip(seqs, rngs)))
    return time.perf_counter() - start


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1
