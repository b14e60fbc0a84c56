"""Config 3's shapes at full batch and context: the engine's decode step over 256 ragged
sequences (contexts U[512, 16k], 16/32 GDN heads with fp32 128 x 128 states, 16/2
attention heads of 256) checked against the CPU oracle on samples. Four layers (three GDN,
one attention) stand in for the 48: every layer runs the same kernels on its own data."""

import math

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import gdn as ogdn
from shellsmith_b200 import _capi, paged
from shellsmith_b200.engine import HybridCacheEngine, HybridConfig
from shellsmith_b200.workloads import gdn_token_inputs_device

pytestmark = pytest.mark.gpu

STATE_ATOL = 1e-4
RTOL, ATOL = 2e-2, 3e-3


def test_decode_step_at_config3_scale(cuda):
    cfg = HybridConfig(layers=4, max_seqs=256, num_pages=150_000)
    eng = HybridCacheEngine(cfg, cuda, seed=3)
    gen = torch.Generator(device=cuda)
    gen.manual_seed(3)
    rng = np.random.default_rng(3)
    drawn = rng.integers(512, 16384 + 1, size=cfg.max_seqs)
    lengths = np.zeros(cfg.max_seqs, np.int64)   # rows are slots
    for i, n in enumerate(drawn):
        lengths[eng.blocks.admit(i, int(n) - 1)] = n
    flat = eng.kv.view(-1)
    for start in range(0, flat.numel(), 1 << 26):
        part = flat[start:start + (1 << 26)]
        part.copy_(torch.randn(part.shape, generator=gen, device=cuda))
    eng.state.copy_(torch.randn(eng.state.shape, generator=gen, device=cuda) * 0.05)
    B = cfg.max_seqs
    inputs, outputs = {}, {}
    for layer in range(cfg.layers):
        if cfg.is_attention(layer):
            inputs[layer] = tuple(torch.randn((B, h, cfg.head_dim), generator=gen,
                                              device=cuda).to(torch.bfloat16)
                                  for h in (cfg.q_heads, cfg.kv_heads, cfg.kv_heads))
            outputs[layer] = torch.empty((B, cfg.q_heads, cfg.head_dim), dtype=torch.bfloat16,
                                         device=cuda)
        else:
            inputs[layer] = gdn_token_inputs_device(gen, B, cfg.gdn_key_heads,
                                                    cfg.gdn_value_heads, cfg.key_dim,
                                                    cfg.value_dim, device=cuda)
            outputs[layer] = torch.empty((B, cfg.gdn_value_heads, cfg.value_dim),
                                         dtype=torch.bfloat16, device=cuda)
    state_before = eng.state.clone()
    assert eng.begin_step() == B
    eng.decode_step(inputs, outputs)
    torch.cuda.synchronize()
    _capi.check_device()

    # Attention: the appended token of every row, then sampled rows against the oracle.
    layer = cfg.attention_layers[0]
    pool = eng.kv[eng.attn_index[layer]]
    q, k_new, v_new = inputs[layer]
    slots = torch.from_numpy(np.array([eng.blocks.prompt_slots(b, int(lengths[b]) - 1,
                                                               int(lengths[b]))[0]
                                       for b in range(B)], np.int64)).to(cuda)
    kg, vg = paged.kv_gather(pool, slots)
    assert torch.equal(kg, k_new) and torch.equal(vg, v_new)
    scale = 1.0 / math.sqrt(cfg.head_dim)
    for b in (int(np.argmin(lengths)), int(np.argmax(lengths)), 101):
        n = int(lengths[b])
        pos = torch.from_numpy(eng.blocks.prompt_slots(b, 0, n).astype(np.int64)).to(cuda)
        k, v = paged.kv_gather(pool, pos)
        want, _ = oatt.decode_attention(q[b].float().cpu().numpy(), k.float().cpu().numpy(),
                                        v.float().cpu().numpy(), scale)
        np.testing.assert_allclose(outputs[layer][b].float().cpu().numpy(), want, rtol=RTOL,
                                   atol=ATOL, err_msg=f"row {b}")

    # GDN: sampled rows of every GDN layer against the float64 token step.
    for layer in cfg.gdn_layers:
        i = eng.gdn_index[layer]
        qg, kg_, vg_, decay, beta = (t.float().cpu().numpy() for t in inputs[layer])
        for b in (0, 77, B - 1):
            want, s = ogdn.token_step(qg[b:b + 1], kg_[b:b + 1], vg_[b:b + 1],
                                      decay[b:b + 1], beta[b:b + 1],
                                      state_before[i, b:b + 1].cpu().numpy())
            np.testing.assert_allclose(outputs[layer][b].float().cpu().numpy(), want[0],
                                       rtol=RTOL, atol=ATOL, err_msg=f"layer {layer} row {b}")
            err = np.abs(eng.state[i, b].cpu().numpy() - s[0]).max()
            assert err <= STATE_ATOL, (layer, b, err)
