"""torch.ops.shellcache registration (no GPU): every operator exists with its schema and
its fake kernel propagates shapes and dtypes of CUDA tensors without running a kernel."""

import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from shellsmith_b200 import torch_ops


def test_operators_are_registered_with_their_mutations():
    for name in torch_ops.OPERATORS:
        op = getattr(torch.ops.shellcache, name).default
        mutated = [a.name for a in op._schema.arguments if a.alias_info and a.alias_info.is_write]
        expect = {"gdn_decode": ["state"], "gated_delta_token": ["state_BHVK"],
                  "gated_delta_chunked": ["state"], "gated_delta_chunks": ["state"],
                  "kv_append": ["kv_pool"], "paged_decode_attention": [],
                  "paged_decode_attention_fused": ["kv_pool"]}[name]
        assert mutated == expect, (name, mutated)


def test_fake_kernels_propagate_shapes():
    bf, f32 = torch.bfloat16, torch.float32
    with FakeTensorMode():
        dev = "cuda"
        q = torch.empty((5, 2, 128), dtype=bf, device=dev)
        v = torch.empty((5, 4, 128), dtype=bf, device=dev)
        g = torch.empty((5, 4), dtype=f32, device=dev)
        state = torch.empty((5, 4, 128, 128), dtype=f32, device=dev)
        out = torch.ops.shellcache.gdn_decode(q, q, v, g, g, state)
        assert out.shape == (5, 4, 128) and out.dtype == bf
        out = torch.ops.shellcache.gated_delta_token(q[:, None], q[:, None], v[:, None],
                                                     g[:, None], g[:, None], state)
        assert out.shape == (5, 1, 4, 128)
        qs = torch.empty((2, 70, 2, 128), dtype=bf, device=dev)
        vs = torch.empty((2, 70, 4, 128), dtype=bf, device=dev)
        gs = torch.empty((2, 70, 4), dtype=f32, device=dev)
        st = torch.empty((2, 4, 128, 128), dtype=f32, device=dev)
        assert torch.ops.shellcache.gated_delta_chunked(qs, qs, vs, gs, gs, st).shape == vs.shape
        logits = torch.empty((2, 70, 4), dtype=bf, device=dev)
        w = torch.empty((4,), dtype=f32, device=dev)
        y = torch.ops.shellcache.gated_delta_chunks(qs, qs, vs, logits, logits, w, w, st)
        assert y.shape == vs.shape and y.dtype == bf
        pool = torch.empty((64, 2, 2, 16, 256), dtype=bf, device=dev)
        qa = torch.empty((3, 16, 256), dtype=bf, device=dev)
        kn = torch.empty((3, 2, 256), dtype=bf, device=dev)
        slots = torch.empty((3,), dtype=torch.int64, device=dev)
        table = torch.empty((3, 8), dtype=torch.int32, device=dev)
        ctx = torch.empty((3,), dtype=torch.int32, device=dev)
        torch.ops.shellcache.kv_append(kn, kn, pool, slots)
        assert torch.ops.shellcache.paged_decode_attention(qa, pool, table, ctx, 0.0625).shape \
            == qa.shape
        out = torch.ops.shellcache.paged_decode_attention_fused(qa, kn, kn, slots, pool, table,
                                                                ctx, 0.0625, 4)
        assert out.shape == qa.shape and out.dtype == bf
