"""Pin the CPU oracle to the reference's own code (golden fixtures) and known answers."""

from pathlib import Path

import numpy as np
import pytest

from oracle import attention as oatt
from oracle import gdn as ogdn

GOLDEN = Path(__file__).resolve().parent / "golden"


def _cases(path):
    data = np.load(path)
    names = sorted({k.split("/")[0] for k in data.files})
    return data, names


GDN, GDN_NAMES = _cases(GOLDEN / "gdn_sequential.npz")
ATT, ATT_NAMES = _cases(GOLDEN / "attention.npz")


def _gdn_inputs(name):
    return [GDN[f"{name}/{k}"].astype(np.float64) for k in ("q", "k", "v", "g", "beta", "s0")]


@pytest.mark.parametrize("name", GDN_NAMES)
def test_sequential_matches_reference_sequential(name):
    y, s = ogdn.sequential(*_gdn_inputs(name))
    np.testing.assert_allclose(y, GDN[f"{name}/y"], rtol=1e-12, atol=1e-14)
    np.testing.assert_allclose(s, GDN[f"{name}/state"], rtol=1e-12, atol=1e-14)


@pytest.mark.parametrize("name", GDN_NAMES)
def test_token_steps_match_reference_sequential(name):
    q, k, v, g, beta, s = _gdn_inputs(name)
    ys = []
    for t in range(q.shape[1]):
        y, s = ogdn.token_step(q[:, t], k[:, t], v[:, t], g[:, t], beta[:, t], s)
        ys.append(y)
    np.testing.assert_allclose(np.stack(ys, 1), GDN[f"{name}/y"], rtol=1e-12, atol=1e-14)
    np.testing.assert_allclose(s, GDN[f"{name}/state"], rtol=1e-12, atol=1e-14)


@pytest.mark.parametrize("name", GDN_NAMES)
def test_chunked_form_matches_reference_sequential(name):
    """The chunk-64 WY/UT form (with tail padding) equals the sequential recurrence."""
    inputs = _gdn_inputs(name)
    inputs[3] = np.clip(inputs[3], 1e-6, 1.0)  # the chunk path clamps gates before the log
    y, s = ogdn.chunked(*inputs)
    np.testing.assert_allclose(y, GDN[f"{name}/y"], rtol=1e-9, atol=1e-11)
    np.testing.assert_allclose(s, GDN[f"{name}/state"], rtol=1e-9, atol=1e-11)


def test_chunked_small_chunks_and_tails():
    q, k, v, g, beta, s = _gdn_inputs("ref_test_L70_gated")
    y_seq, s_seq = ogdn.sequential(q, k, v, g, beta, s)
    for chunk in (8, 16, 64):
        y, st = ogdn.chunked(q, k, v, g, beta, s, chunk=chunk)
        np.testing.assert_allclose(y, y_seq, rtol=1e-9, atol=1e-11)
        np.testing.assert_allclose(st, s_seq, rtol=1e-9, atol=1e-11)


def test_bf16_round_is_nearest_even():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, 1e-40], np.float32)
    got = ogdn.bf16_round(x)
    assert got[0] == 1.0 and got[1] == 1.0 and got[2] == 1.0 + 2 ** -6 and got[3] == -2.5


def test_gates_match_reference_formula():
    a = np.array([-3.0, 0.0, 2.0])
    b = np.array([0.0, 1.0, -2.0])
    g, beta = ogdn.gates(a, b, np.array([0.5]), np.array([0.1]))
    sp = np.log1p(np.exp(a + 0.1))
    np.testing.assert_allclose(g, np.exp(-np.exp(0.5) * sp))
    np.testing.assert_allclose(beta, 1 / (1 + np.exp(-b)))


@pytest.mark.parametrize("name", ATT_NAMES)
def test_attention_matches_reference_numpy_attention(name):
    q, k, v, y = (ATT[f"{name}/{x}"] for x in ("q", "k", "v", "y"))
    queries, keys, offset, scale = ATT[f"{name}/meta"]
    got, lse = oatt.attention(q, k, v, float(scale), query_offset=int(offset))
    np.testing.assert_allclose(got, y, rtol=1e-12, atol=1e-13)
    assert np.all(np.isfinite(lse))


def test_known_answer_causal_offset():
    """The reference's known answer: v = [1, 3, 8] seen by queries at offsets 1 and 2."""
    got, _ = oatt.attention(np.zeros((1, 2, 2, 1)), np.zeros((1, 1, 3, 1)),
                            np.array([[[[1.0], [3.0], [8.0]]]]), 1.0)
    np.testing.assert_allclose(got[0, :, 0, 0], [2.0, 2.0])
    np.testing.assert_allclose(got[0, :, 1, 0], [4.0, 4.0])


@pytest.mark.parametrize("tokens_per_split", [1, 16, 100, 1000])
def test_split_partials_combine_to_single_pass(tokens_per_split):
    name = "decode_k300"
    q, k, v, y = (ATT[f"{name}/{x}"] for x in ("q", "k", "v", "y"))
    po, pl = oatt.split_partials(q[0, :, 0], k[0].transpose(1, 0, 2), v[0].transpose(1, 0, 2),
                                 1 / 16, tokens_per_split)
    out, lse = oatt.combine(po, pl)
    np.testing.assert_allclose(out, y[0, :, 0], rtol=1e-12, atol=1e-13)
    _, want_lse = oatt.decode_attention(q[0, :, 0], k[0].transpose(1, 0, 2),
                                        v[0].transpose(1, 0, 2), 1 / 16)
    np.testing.assert_allclose(lse, want_lse, rtol=1e-12)


def test_pool_layout_roundtrip_and_swizzle():
    rng = np.random.default_rng(0)
    hkv, P, D, pages = 2, 16, 64, 5
    pool = np.zeros(pages * hkv * 2 * P * D, np.float32)
    slots = rng.permutation(pages * P)[:30]
    k = rng.standard_normal((30, hkv, D)).astype(np.float32)
    v = rng.standard_normal((30, hkv, D)).astype(np.float32)
    oatt.pool_write(pool, slots, k, v, hkv, P, D)
    k2, v2 = oatt.pool_read(pool, slots, hkv, P, D)
    assert np.array_equal(k, k2) and np.array_equal(v, v2)
    # Token at page offset 3: its chunk 0 sits at chunk position 3.
    slot = int(slots[0])
    page, off = divmod(slot, P)
    row = (((page * hkv + 0) * 2 + 0) * P + off) * D
    assert np.array_equal(pool[row + 8 * (0 ^ (off & 7)):row + 8 * (0 ^ (off & 7)) + 8],
                          k[0, 0, :8])
