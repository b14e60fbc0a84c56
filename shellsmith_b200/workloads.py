"""Seeded synthetic inputs with the distributions of the benchmark configs.

The reference measures on private replayed conversations; these generators
stand in for them with the configs' stated shapes and distributions:
  q, k ~ N(0, 1) then L2-normalised per head; v ~ N(0, 1);
  beta = sigmoid(N(0, 1)); gate log g ~ -softplus(N(0, 1)), decay a = exp(g).
NumPy generators feed the small parity cases (so the CPU oracle sees the
same bf16-representable values); torch generators fill large device buffers.
"""

from __future__ import annotations

import numpy as np
import torch


def bf16_np(x: np.ndarray) -> np.ndarray:
    """Round to bfloat16 and return float32 (the values a bf16 tensor holds)."""
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(
        torch.bfloat16).float().numpy()


def _l2(x: np.ndarray) -> np.ndarray:
    return x / np.linalg.norm(x, axis=-1, keepdims=True)


def gdn_token_inputs(rng: np.random.Generator, B: int, Hk: int, Hv: int, dk: int, dv: int):
    """One decode token: q, k [B,Hk,dk], v [B,Hv,dv] (bf16 values), decay and beta [B,Hv] fp32."""
    q = bf16_np(_l2(rng.standard_normal((B, Hk, dk))))
    k = bf16_np(_l2(rng.standard_normal((B, Hk, dk))))
    v = bf16_np(rng.standard_normal((B, Hv, dv)))
    log_g = -np.logaddexp(0.0, rng.standard_normal((B, Hv)))
    decay = np.exp(log_g).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((B, Hv))))).astype(np.float32)
    return q, k, v, decay, beta


def gdn_sequence_inputs(rng: np.random.Generator, B: int, T: int, Hk: int, Hv: int, dk: int,
                        dv: int):
    """A prompt: q, k [B,T,Hk,dk], v [B,T,Hv,dv] (bf16 values), decay, beta [B,T,Hv] fp32."""
    q = bf16_np(_l2(rng.standard_normal((B, T, Hk, dk))))
    k = bf16_np(_l2(rng.standard_normal((B, T, Hk, dk))))
    v = bf16_np(rng.standard_normal((B, T, Hv, dv)))
    decay = np.exp(-np.logaddexp(0.0, rng.standard_normal((B, T, Hv)))).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((B, T, Hv))))).astype(np.float32)
    return q, k, v, decay, beta


def to_device(*arrays, dtype=torch.bfloat16, device="cuda"):
    return [torch.from_numpy(np.ascontiguousarray(a)).to(device=device, dtype=dtype)
            for a in arrays]


# ----------------------------------------------------------------- device-side
def l2_normalise_(x: torch.Tensor) -> torch.Tensor:
    return x.div_(x.float().norm(dim=-1, keepdim=True).to(x.dtype))


def gdn_token_inputs_device(gen: torch.Generator, B: int, Hk: int, Hv: int, dk: int, dv: int,
                            device="cuda"):
    """Device-resident decode-token inputs with the same distributions."""
    q = torch.randn((B, Hk, dk), generator=gen, device=device)
    k = torch.randn((B, Hk, dk), generator=gen, device=device)
    q = (q / q.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    k = (k / k.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    v = torch.randn((B, Hv, dv), generator=gen, device=device).to(torch.bfloat16)
    decay = torch.exp(-torch.nn.functional.softplus(
        torch.randn((B, Hv), generator=gen, device=device)))
    beta = torch.sigmoid(torch.randn((B, Hv), generator=gen, device=device))
    return q, k, v, decay.contiguous(), beta.contiguous()


def fill_normal_bf16_(t: torch.Tensor, gen: torch.Generator, chunk: int = 1 << 28) -> None:
    """Fill a large bf16 buffer with N(0,1) values, chunk by chunk (bounded temporaries)."""
    flat = t.view(-1)
    for start in range(0, flat.numel(), chunk):
        part = flat[start:start + chunk]
        part.copy_(torch.randn(part.shape, generator=gen, device=t.device))
