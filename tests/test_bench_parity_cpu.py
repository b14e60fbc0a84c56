"""The bench's in-run parity checks (no GPU): its float64 torch restatements of the
paged-pool read, split attention and the GDN token step agree with the CPU oracle, and
they reject a planted error. The bench runs them on the device after its timed windows,
on every rank, so the multi-GPU lines carry a parity result."""

import math

import numpy as np
import torch

import bench
from oracle import attention as oatt
from oracle import gdn as ogdn


def _pool(rng, num_pages=12, hkv=2, P=16, D=256):
    return torch.from_numpy(rng.standard_normal((num_pages, hkv, 2, P, D)).astype(np.float32)
                            ).to(torch.bfloat16)


def test_pool_tokens_unswizzles_like_the_oracle():
    rng = np.random.default_rng(0)
    pool = _pool(rng)
    pages = [7, 2, 11, 0]
    for L in (1, 16, 17, 50, 64):
        k, v = bench.pool_tokens(pool, pages, L)
        wk, wv = oatt.pool_read_pages(pool.float().numpy(), pages, L, 2, 16, 256)
        assert np.array_equal(k.float().numpy(), wk) and np.array_equal(v.float().numpy(), wv)


def test_split_partials_merge_to_the_oracle_attention():
    rng = np.random.default_rng(1)
    q = torch.from_numpy(rng.standard_normal((3, 64)))
    k = torch.from_numpy(rng.standard_normal((300, 64)))
    v = torch.from_numpy(rng.standard_normal((300, 64)))
    parts = [bench.partial_fp64(q, k[a:b], v[a:b], 0.125) for a, b in ((0, 7), (7, 160),
                                                                        (160, 300))]
    empty = (torch.zeros((3, 64), dtype=torch.float64),
             torch.full((3,), -math.inf, dtype=torch.float64))
    out, lse = bench.merge_fp64(parts + [empty])
    want, want_lse = oatt.decode_attention(q.numpy(), k.numpy()[:, None], v.numpy()[:, None],
                                           0.125)
    np.testing.assert_allclose(out.numpy(), want, atol=1e-12)
    np.testing.assert_allclose(lse.numpy(), want_lse, atol=1e-12)


def test_attention_row_check_accepts_bf16_output_and_rejects_a_planted_error():
    rng = np.random.default_rng(2)
    hq, hkv, L, D = 16, 2, 200, 256
    q = torch.from_numpy(rng.standard_normal((hq, D)).astype(np.float32)).to(torch.bfloat16)
    k = torch.from_numpy(rng.standard_normal((L, hkv, D)).astype(np.float32)).to(torch.bfloat16)
    v = torch.from_numpy(rng.standard_normal((L, hkv, D)).astype(np.float32)).to(torch.bfloat16)
    want, _ = oatt.decode_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                    1 / 16)
    out = torch.from_numpy(want.astype(np.float32)).to(torch.bfloat16)
    assert bench.attention_row_ok(out, q, k, v, 1 / 16)
    bad = out.clone()
    bad[9, 100] += 0.05
    assert not bench.attention_row_ok(bad, q, k, v, 1 / 16)


def test_gdn_row_check_matches_the_oracle_step_and_rejects_a_planted_error():
    rng = np.random.default_rng(3)
    hk, hv, d = 2, 4, 32
    q = rng.standard_normal((1, hk, d))
    k = rng.standard_normal((1, hk, d)) / math.sqrt(d)
    v = rng.standard_normal((1, hv, d))
    decay = rng.uniform(0.2, 1.0, (1, hv))
    beta = rng.uniform(0.0, 1.0, (1, hv))
    state = rng.standard_normal((1, hv, d, d)) * 0.05
    out, after = ogdn.token_step(q, k, v, decay, beta, state)
    t = lambda x: torch.from_numpy(np.asarray(x)[0])  # noqa: E731
    args = (t(state), t(after), t(out), t(q), t(k), t(v), t(decay), t(beta))
    assert bench.gdn_row_ok(*args)
    planted = t(after).clone()
    planted[1, 3, 5] += 2e-4
    assert not bench.gdn_row_ok(args[0], planted, *args[2:])
