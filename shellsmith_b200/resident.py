"""A resident model over the paged cache engine, and the runtime engine around it.

The reference's model-level plug point: `mlx_decode.decode_rows(engine,
requests)` forwards to `engine.resident.decode_rows(engine, requests)`
(studio_compute/mlx_decode.py:24-26), and `inference.prefill_request`
(inference.py:124-163) advances a prompt by at most `engine.prefill_tokens`
tokens per scheduler step. `PagedResident` implements both over one
`HybridCacheEngine`: a request's cache is a `runtime.PagedSequence` (one slot:
its batch row, block-table row, GDN state and tap-ring row), decode batches
every row of a group into one launch per layer, and prefill runs a prompt
chunk through every layer's cache work (GDN layers through the front /
tcgen05 chunk kernel / gated norm, attention layers through the K/V scatter).

The projections, norms, attention over the prompt itself and the LM head are
not part of the cache path; `ToyHybridModel` supplies them with small seeded
weights (torch GEMMs, torch SDPA for the prompt's own attention) so that the
reference's scheduler can drive the paged engine end to end in tests.

`PagedRuntimeEngine` carries the attributes the reference's request
lifecycle reads (`resident`, `prefixes`, `policies`, `reserved`, `admit`,
`lm.make_cache`, `mx`, `prefill_tokens` ...) and builds the
`ContinuousBatcher` whose callbacks are runtime.create_request /
prefill_request / advance_requests / sample_requests / release_request, as
`RuntimeEngine.inference_scheduler` does (studio_compute/runtime.py:135-148).
"""

from __future__ import annotations

import math
from collections import OrderedDict
from contextlib import contextmanager
from types import SimpleNamespace

import numpy as np
import torch

from . import admission, gdn_layer, paged
from .engine import HybridCacheEngine, HybridConfig
from .runtime import PagedSequence, paged_prefix_cache


def _rms(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    x = x.float()
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)


class ToyHybridModel:
    """Seeded projections for a hybrid GDN / attention stack (not the cache path)."""

    def __init__(self, cfg: HybridConfig, d_model: int = 256, vocab: int = 97, seed: int = 0,
                 device="cuda"):
        self.cfg, self.d_model, self.vocab = cfg, d_model, vocab
        dev = torch.device(device)
        gen = torch.Generator(device="cpu").manual_seed(seed)

        def w(rows, cols, scale=None):
            t = torch.randn((rows, cols), generator=gen) * (scale or 1.0 / math.sqrt(rows))
            return t.to(dev, torch.bfloat16)

        self.embed = torch.randn((vocab, d_model), generator=gen).to(dev, torch.float32)
        self.layers = {}
        C = (2 * cfg.gdn_key_heads + cfg.gdn_value_heads) * 128
        for layer in range(cfg.layers):
            if cfg.is_attention(layer):
                self.layers[layer] = SimpleNamespace(
                    wq=w(d_model, cfg.q_heads * cfg.head_dim),
                    wk=w(d_model, cfg.kv_heads * cfg.head_dim),
                    wv=w(d_model, cfg.kv_heads * cfg.head_dim),
                    wo=w(cfg.q_heads * cfg.head_dim, d_model))
            else:
                Hv = cfg.gdn_value_heads
                weights = gdn_layer.GDNWeights(
                    conv_w=(torch.randn((C, 4), generator=gen) * 0.5).to(dev, torch.bfloat16),
                    a_log=torch.log(torch.rand(Hv, generator=gen) * 15 + 1).to(dev),
                    dt_bias=torch.randn(Hv, generator=gen).to(dev),
                    norm_w=(1 + 0.1 * torch.randn(128, generator=gen)).to(dev, torch.bfloat16),
                    eps=1e-6, key_heads=cfg.gdn_key_heads, value_heads=Hv)
                self.layers[layer] = SimpleNamespace(
                    w_qkv=w(d_model, C), w_z=w(d_model, Hv * 128), w_a=w(d_model, Hv),
                    w_b=w(d_model, Hv), wo=w(Hv * 128, d_model), glue=weights)
        self.head = w(d_model, vocab)

    def hidden(self, ids) -> torch.Tensor:
        return self.embed[torch.as_tensor(ids, device=self.embed.device, dtype=torch.long)]

    def gdn_inputs(self, layer: int, h: torch.Tensor) -> tuple:
        L = self.layers[layer]
        x = _rms(h).to(torch.bfloat16)
        return ((x @ L.w_qkv).contiguous(), (x @ L.w_z).contiguous(), (x @ L.w_a).contiguous(),
                (x @ L.w_b).contiguous())

    def attention_inputs(self, layer: int, h: torch.Tensor) -> tuple:
        L, c = self.layers[layer], self.cfg
        x = _rms(h).to(torch.bfloat16)
        n = x.shape[0]
        return ((x @ L.wq).view(n, c.q_heads, c.head_dim).contiguous(),
                (x @ L.wk).view(n, c.kv_heads, c.head_dim).contiguous(),
                (x @ L.wv).view(n, c.kv_heads, c.head_dim).contiguous())

    def residual(self, layer: int, h: torch.Tensor, mixed: torch.Tensor) -> torch.Tensor:
        return h + (mixed.reshape(h.shape[0], -1) @ self.layers[layer].wo).float()

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        return (_rms(h).to(torch.bfloat16) @ self.head).float()


class PagedResident:
    """decode_rows / prefill over a HybridCacheEngine (with tap rings) and a model."""

    def __init__(self, cache: HybridCacheEngine, model: ToyHybridModel):
        if cache.taps is None:
            raise ValueError("PagedResident runs GDN layers from projections: gdn_taps=True")
        self.cache, self.model = cache, model
        c = cache.cfg
        self._glue_ws = gdn_layer.SplitWorkspace(c.max_seqs, model.layers[c.gdn_layers[0]].glue,
                                                 cache.device)

    # ---------------------------------------------------------------- prefill
    def prefill(self, seq: PagedSequence, ids: list, start: int) -> torch.Tensor:
        """Run prompt tokens `ids` at positions start.. of `seq` through every layer;
        returns the last token's logits [1, vocab]."""
        eng, model, c = self.cache, self.model, self.cache.cfg
        stop = start + len(ids)
        if eng.blocks.lengths[seq.slot] < stop:
            eng.extend(seq.slot, stop)
        dev = eng.device
        one = torch.zeros(2, dtype=torch.int32, device=dev)
        one[1] = len(ids)
        slot_t = torch.tensor([seq.slot], dtype=torch.int32, device=dev)
        start_t = torch.tensor([start], dtype=torch.int32, device=dev)
        kv_slots = torch.from_numpy(eng.blocks.prompt_slots(seq.slot, start, stop)).to(dev)
        all_slots = torch.from_numpy(eng.blocks.prompt_slots(seq.slot, 0, stop)).to(dev)
        h = model.hidden(ids)
        for layer in range(c.layers):
            if c.is_attention(layer):
                q, k, v = model.attention_inputs(layer, h)
                pool = eng.kv[eng.attn_index[layer]]
                paged.kv_append(k, v, pool, kv_slots)
                kk, vv = paged.kv_gather(pool, all_slots)          # [stop, Hkv, D]
                group = c.q_heads // c.kv_heads
                kk = kk.float().repeat_interleave(group, 1).transpose(0, 1)
                vv = vv.float().repeat_interleave(group, 1).transpose(0, 1)
                qq = q.float().transpose(0, 1)                      # [Hq, n, D]
                mask = (torch.arange(stop, device=dev)[None, :]
                        <= torch.arange(start, stop, device=dev)[:, None])
                o = torch.nn.functional.scaled_dot_product_attention(
                    qq, kk, vv, attn_mask=mask, scale=eng.scale).transpose(0, 1)
                h = model.residual(layer, h, o.to(torch.bfloat16))
            else:
                qkv, z, a, b = model.gdn_inputs(layer, h)
                i = eng.gdn_index[layer]
                out = gdn_layer.gdn_prefill(qkv, z, a, b, model.layers[layer].glue, eng.taps[i],
                                            eng.state[i], one, slot_t, start_t)
                h = model.residual(layer, h, out)
        return model.logits(h[-1:])

    # ---------------------------------------------------------------- decode
    def decode_rows(self, engine, requests: list) -> None:
        """One token per request through every layer: the reference's decode_rows
        contract (mlx_decode.py:18-77) — feeds each request's last token, writes
        request.logits and clears needs_decode."""
        eng, model, c = self.cache, self.model, self.cache.cfg
        slots = [r.cache.slot for r in requests]
        eng.begin_step(slots)
        rows = torch.tensor(slots, dtype=torch.long, device=eng.device)
        h = model.hidden([r.tokens[-1] for r in requests])
        B = c.max_seqs
        for layer in range(c.layers):
            if c.is_attention(layer):
                q, k, v = model.attention_inputs(layer, h)
                qf = torch.zeros((B, c.q_heads, c.head_dim), dtype=torch.bfloat16, device=eng.device)
                kf = torch.zeros((B, c.kv_heads, c.head_dim), dtype=torch.bfloat16,
                                 device=eng.device)
                vf = torch.zeros_like(kf)
                qf[rows], kf[rows], vf[rows] = q, k, v
                out = torch.empty_like(qf)
                eng.attention_layer(layer, qf, kf, vf, out)
                h = model.residual(layer, h, out[rows])
            else:
                qkv, z, a, b = model.gdn_inputs(layer, h)
                full = [torch.zeros((B,) + t.shape[1:], dtype=t.dtype, device=eng.device)
                        for t in (qkv, z, a, b)]
                for dst, src in zip(full, (qkv, z, a, b)):
                    dst[rows] = src
                out = torch.empty((B, c.gdn_value_heads * 128), dtype=torch.bfloat16,
                                  device=eng.device)
                i = eng.gdn_index[layer]
                gdn_layer.gdn_decode_split(*full, model.layers[layer].glue, eng.taps[i],
                                           eng.position, eng.state[i], eng.state_slot, out=out,
                                           workspace=self._glue_ws)
                h = model.residual(layer, h, out[rows])
        logits = model.logits(h)
        for row, request in enumerate(requests):
            request.logits = logits[row:row + 1]
            request.needs_decode = False


class _Mx:
    """The mx calls the request lifecycle makes (RNG keys, live device bytes)."""

    uint32 = np.uint32

    @staticmethod
    def get_active_memory():
        return int(torch.cuda.memory_allocated())

    @staticmethod
    def array(values, dtype):
        return np.asarray(values, dtype=dtype)

    class random:  # noqa: N801 -- the reference's attribute name
        @staticmethod
        def key(seed):
            return np.asarray([0, seed], dtype=np.uint32)


class PagedRuntimeEngine:
    """The engine object the reference's request lifecycle and batcher expect."""

    def __init__(self, cfg: HybridConfig, model: ToyHybridModel | None = None, *,
                 budget_bytes: int = 1 << 40, prefix_limit_bytes: int = 1 << 30,
                 prefill_tokens: int = 32, concurrency: int = 8, device="cuda"):
        self.cache = HybridCacheEngine(cfg, device)
        self.model = model or ToyHybridModel(cfg, device=device)
        paged_resident = PagedResident(self.cache, self.model)
        budget = admission.ResidentBudget(cfg, budget_bytes, SimpleNamespace(
            get_active_memory=lambda: int(torch.cuda.memory_allocated(self.cache.device))))
        self.resident = SimpleNamespace(
            estimate_inference=budget.estimate_inference, admit=budget.admit,
            budget=budget_bytes, mx=budget.mx, decode_rows=paged_resident.decode_rows,
            prefill=paged_resident.prefill)
        self.prefixes = paged_prefix_cache(self.cache, prefix_limit_bytes)
        self.policies = OrderedDict(p=SimpleNamespace())
        self.idle_factors: dict = {}
        self.reserved: dict = {}
        self.prefix_identity = "toy-hybrid"
        self.prefill_tokens = prefill_tokens
        self.inference_concurrency = concurrency
        self.mx = _Mx
        self.lm = SimpleNamespace(make_cache=lambda: PagedSequence(self.cache, None))

    def persistent_bytes(self) -> int:
        return self.prefixes.bytes

    def admission_budget_bytes(self) -> int:
        return self.resident.budget

    def admit(self, additional: int) -> None:
        self.prefixes.trim(admission.cache_capacity(self, additional=additional))
        reserved = sum(self.reserved.values())
        self.resident.admit(additional, reserved, persistent=self.persistent_bytes())

    @contextmanager
    def _borrow_policy(self, reference):
        yield {"policy": reference}

    def inference_scheduler(self, *, finish, fail):
        from . import runtime
        from .scheduler import ContinuousBatcher

        return ContinuousBatcher(
            self.inference_concurrency,
            create=lambda request_id, body: runtime.create_request(self, request_id, body),
            prefill=lambda request: runtime.prefill_request(self, request),
            advance=lambda requests: runtime.advance_requests(self, requests),
            sample=lambda requests: runtime.sample_requests(self, requests),
            finish=finish, fail=fail,
            release=lambda request: runtime.release_request(self, request))
