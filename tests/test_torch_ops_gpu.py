"""torch.ops.shellcache.* on the GPU: each registered operator gives the same bits as the
direct call of the same C-ABI entry point (numerics / paged shims), state and pools
included, and the operators pass torch.library.opcheck's schema and fake-kernel checks."""

import math

import numpy as np
import pytest
import torch

from shellsmith_b200 import numerics, paged, torch_ops  # noqa: F401 (registers the ops)
from shellsmith_b200.workloads import gdn_token_inputs_device

pytestmark = pytest.mark.gpu


def test_gdn_operators_match_direct_calls(cuda):
    gen = torch.Generator(device=cuda)
    gen.manual_seed(3)
    q, k, v, g, beta = gdn_token_inputs_device(gen, 6, 2, 4, 128, 128, device=cuda)
    s0 = torch.randn((6, 4, 128, 128), generator=gen, device=cuda) * 0.1
    a, b = s0.clone(), s0.clone()
    out_op = torch.ops.shellcache.gdn_decode(q, k, v, g, beta, a)
    out = numerics.gdn_decode(q, k, v, g, beta, b)
    assert torch.equal(out_op, out) and torch.equal(a, b)
    a, b = s0.clone(), s0.clone()
    y_op = torch.ops.shellcache.gated_delta_token(q[:, None], k[:, None], v[:, None], g[:, None],
                                                  beta[:, None], a)
    y, _ = numerics.gated_delta_token(q[:, None], k[:, None], v[:, None], g[:, None],
                                      beta[:, None], b)
    assert torch.equal(y_op, y) and torch.equal(a, b)
    T = 70
    qs, ks, vs, gs, bs = gdn_token_inputs_device(gen, 2 * T, 2, 4, 128, 128, device=cuda)
    shape = lambda x: x.view(2, T, *x.shape[1:])  # noqa: E731
    st0 = torch.randn((2, 4, 128, 128), generator=gen, device=cuda) * 0.1
    a, b = st0.clone(), st0.clone()
    y_op = torch.ops.shellcache.gated_delta_chunked(*map(shape, (qs, ks, vs, gs, bs)), a)
    y, _ = numerics.gated_delta_chunked(*map(shape, (qs, ks, vs, gs, bs)), b)
    assert torch.equal(y_op, y) and torch.equal(a, b)
    logits = torch.randn((2, T, 4), generator=gen, device=cuda).to(torch.bfloat16)
    a_log = torch.rand(4, generator=gen, device=cuda)
    dt = torch.randn(4, generator=gen, device=cuda)
    a, b = st0.clone(), st0.clone()
    y_op = torch.ops.shellcache.gated_delta_chunks(*map(shape, (qs, ks, vs)), logits, logits,
                                                   a_log, dt, a)
    y, _ = numerics.gated_delta_chunks(*map(shape, (qs, ks, vs)), logits, logits, a_log, dt, b)
    assert torch.equal(y_op, y) and torch.equal(a, b)


def test_paged_operators_match_direct_calls(cuda):
    rng = np.random.default_rng(4)
    P, hq, hkv, D = paged.PAGE_SIZE, 16, 2, 256
    lengths = [40, 300, 1, 129]
    need = [math.ceil(L / P) for L in lengths]
    table = np.zeros((4, max(need)), np.int32)
    perm, cursor = rng.permutation(64), 0
    for i, n in enumerate(need):
        table[i, :n] = perm[cursor:cursor + n]
        cursor += n
    bt = torch.from_numpy(table).to(cuda)
    ctx = torch.tensor(lengths, dtype=torch.int32, device=cuda)
    pool0 = torch.randn((64, hkv, 2, P, D), device=cuda).to(torch.bfloat16)
    q = torch.randn((4, hq, D), device=cuda).to(torch.bfloat16)
    kn = torch.randn((4, hkv, D), device=cuda).to(torch.bfloat16)
    vn = torch.randn((4, hkv, D), device=cuda).to(torch.bfloat16)
    slots = torch.tensor([int(table[i, (L - 1) // P]) * P + (L - 1) % P
                          for i, L in enumerate(lengths)], dtype=torch.int64, device=cuda)
    a, b = pool0.clone(), pool0.clone()
    torch.ops.shellcache.kv_append(kn, vn, a, slots)
    paged.kv_append(kn, vn, b, slots)
    assert torch.equal(a, b)
    out_op = torch.ops.shellcache.paged_decode_attention(q, a, bt, ctx, 1 / 16, 4)
    out = paged.paged_decode_attention(q, b, bt, ctx, 1 / 16, pages_per_split=4)
    assert torch.equal(out_op, out)
    a, b = pool0.clone(), pool0.clone()
    out_op = torch.ops.shellcache.paged_decode_attention_fused(q, kn, vn, slots, a, bt, ctx,
                                                               1 / 16, 4)
    out = paged.paged_decode_attention_fused(q, kn, vn, slots, b, bt, ctx, 1 / 16,
                                             pages_per_split=4)
    torch.cuda.synchronize()
    assert torch.equal(out_op, out) and torch.equal(a, b)


def test_opcheck_schema_and_fake_kernels(cuda):
    gen = torch.Generator(device=cuda)
    gen.manual_seed(5)
    q, k, v, g, beta = gdn_token_inputs_device(gen, 3, 2, 4, 128, 128, device=cuda)
    state = torch.zeros((3, 4, 128, 128), device=cuda)
    checks = ("test_schema", "test_faketensor")
    torch.library.opcheck(torch.ops.shellcache.gdn_decode.default, (q, k, v, g, beta, state),
                          test_utils=checks)
    pool = torch.zeros((8, 2, 2, 16, 128), dtype=torch.bfloat16, device=cuda)
    kn = torch.randn((3, 2, 128), device=cuda).to(torch.bfloat16)
    slots = torch.tensor([0, 17, -1], dtype=torch.int64, device=cuda)
    torch.library.opcheck(torch.ops.shellcache.kv_append.default, (kn, kn, pool, slots),
                          test_utils=checks)
