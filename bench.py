"""Benchmark of the continuous-batching decode cache step.

Workload (per GPU; sequences shard across ranks with no collective, so the
per-GPU work is fixed as N grows -- weak scaling):
  48 layers, 3 GDN : 1 full attention (36 + 12), GDN 16 key / 32 value heads
  128 x 128 fp32 state, attention 16 q / 2 kv heads, D = 256, page 16;
  256 ragged sequences, context lengths U[512, 16k]. Each step every
  sequence finishes with probability 0.02 (pages and state slot released)
  and a new sequence with a U[256, 2k] prompt is admitted in its place; the
  prompt's KV pages are written (prefill, timed separately) and it decodes in
  the same step.
A step = one decode token for every active sequence through all 48 layers'
cache work: GDN state update, paged KV append, split-K paged attention.
Inputs are seeded synthetic tensors with the config's distributions; the
per-step working set (~90 GB) exceeds L2, so no flush is needed.

Arms:
  default           the CUDA path (libshellcache.so through its C ABI)
  --impl reference  the reference's CPU math for the path (float64 NumPy
                    oracles restated in oracle/) on the host cores, on a
                    bounded sample of sequences per step
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode cache-step tokens/sec at batch 256 ragged; achieved HBM GB/s vs B200 peak"
# DRAM bytes (read + write) / algorithmic bytes of one launch, from an ncu
# capture of this workload at a smaller size (4 layers, ctx U[512, 8k]; the
# attention figure from the kernel with the append folded in).
# Traffic grows in proportion to the K/V tokens read (attention) and the rows
# updated (GDN), so a full launch's traffic is its algorithmic bytes times this.
ATTN_TRAFFIC_RATIO = 1.004
GDN_TRAFFIC_RATIO = 0.950
UNIT = "tokens/s"
SEED = 3  # configs 1-4 use seeds 1-4


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--layers", type=int, default=48,
                    help="decoder layers (3 GDN : 1 attention); fewer only for profiling")
    ap.add_argument("--min-len", type=int, default=512)
    ap.add_argument("--max-len", type=int, default=16_384)
    ap.add_argument("--churn", type=float, default=0.02)
    ap.add_argument("--num-pages", type=int, default=150_000)
    ap.add_argument("--pages-per-split", type=int, default=0,
                    help="attention split size in pages (0 = adapt to the batch)")
    ap.add_argument("--cpu-sample", type=int, default=0,
                    help="sequences in the CPU baseline sample (0 = auto)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-config1", action="store_true",
                    help="skip the measurements beside config 3: configs 2 and 4 (every rank, "
                         "sharded), configs 0 and 1, the GDN front and 8-bit KV (rank 0)")
    ap.add_argument("--front-only", action="store_true",
                    help="only time one GDN layer run from its projections (fused glue) "
                         "against the plain state update, with --batch rows; prints a JSON "
                         "object (a profiling entry, not a bench line)")
    ap.add_argument("--prefill-only", action="store_true",
                    help="only time the config-1 chunked prefill; prints a JSON "
                         "object (a profiling entry, not a bench line)")
    ap.add_argument("--kv8-only", action="store_true",
                    help="only time one attention layer on 8-bit pages beside bf16 pages for "
                         "--batch sequences of U[--min-len, --max-len] tokens; prints a JSON "
                         "object (a profiling entry, not a bench line)")
    ap.add_argument("--exchange", choices=("fused", "p2p", "nccl"), default="p2p",
                    help="config 4, N > 1: exchange the attention partials by NVLink peer "
                         "stores with epoch flags, issued by the attention merge itself "
                         "(fused) or by a separate put/wait kernel pair (p2p), or by an "
                         "NCCL all-gather (nccl)")
    ap.add_argument("--config", type=int, choices=(3, 4), default=3,
                    help="3: ragged batch decode step (default); 4: one long sequence with its "
                         "KV pages split across the GPUs")
    ap.add_argument("--ctx4", type=int, default=131_072, help="config-4 context length")
    return ap.parse_args()


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples the SM clock and the clock-event (throttle) reasons while the timed region
    runs: through NVML every 20 ms when its binding loads, else nvidia-smi every 200 ms.
    It only reads: no GPU setting is changed."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, index: int):
        visible = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
        self.index = visible[index].strip() if index < len(visible) and visible[index].strip() \
            else str(index)
        self.rows = []   # (sm MHz, max sm MHz, frozenset of active reasons)
        self._nvml = self._open_nvml(index)
        self.source = "nvml" if self._nvml is not None else "nvidia-smi"
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)

    def _open_nvml(self, local: int):
        """NVML handle of CUDA device `local`, found by its UUID (the CUDA and NVML
        orders can differ), or None."""
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            uuid = "GPU-" + str(torch.cuda.get_device_properties(local).uuid)
            handle = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            self._pynvml = pynvml
            self._bits = {"hw_slowdown": pynvml.nvmlClocksEventReasonHwSlowdown,
                          "hw_thermal_slowdown": pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                          "sw_thermal_slowdown": pynvml.nvmlClocksEventReasonSwThermalSlowdown,
                          "sw_power_cap": pynvml.nvmlClocksEventReasonSwPowerCap}
            return handle
        except Exception:  # noqa: BLE001 -- fall back to nvidia-smi
            return None

    def _sample_nvml(self):
        p, h = self._pynvml, self._nvml
        sm = p.nvmlDeviceGetClockInfo(h, p.NVML_CLOCK_SM)
        mx = p.nvmlDeviceGetMaxClockInfo(h, p.NVML_CLOCK_SM)
        bits = p.nvmlDeviceGetCurrentClocksEventReasons(h)
        return float(sm), float(mx), frozenset(n for n, b in self._bits.items() if bits & b)

    def _sample_smi(self):
        out = subprocess.run(
            ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
             "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
        r = [x.strip() for x in out.stdout.strip().split(",")]
        if out.returncode != 0 or len(r) < 9:
            return None
        num = lambda x: float(x) if x.replace(".", "").isdigit() else None  # noqa: E731
        return num(r[1]), num(r[2]), frozenset(
            n for i, n in enumerate(self.REASONS) if r[5 + i].lower() == "active")

    def _run(self):
        sample = self._sample_nvml if self._nvml is not None else self._sample_smi
        period = 0.02 if self._nvml is not None else 0.2
        while not self._stop.is_set():
            try:
                row = sample()
                if row is not None:
                    self.rows.append(row)
            except Exception:  # noqa: BLE001 -- clocks are advisory
                pass
            self._stop.wait(period)

    def __enter__(self):
        self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._thread.join(timeout=10)

    def summary(self) -> dict:
        sm = [r[0] for r in self.rows if r[0] is not None]
        mx = [r[1] for r in self.rows if r[1] is not None]
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clocks unavailable"],
                    "samples": 0, "source": self.source}
        return {"sm_mhz": statistics.median(sm), "sm_min_mhz": min(sm),
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(set().union(*(r[2] for r in self.rows))),
                "samples": len(self.rows), "source": self.source}


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": float(data["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


# ------------------------------------------------------------------ distributed
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ------------------------------------------------------------------ workload
def balanced_share(args, rank: int, world: int) -> np.ndarray:
    """This rank's running sequences when the batch is sharded over `world` GPUs: every
    rank draws the same global set of batch x world contexts and the sequences are dealt
    longest first in snake order (0..N-1, N-1..0, ...), so each GPU holds `batch`
    sequences with nearly equal resident K/V bytes."""
    glob = np.random.default_rng(SEED).integers(args.min_len, args.max_len + 1,
                                                size=args.batch * world)
    return glob[snake_deal(glob, rank, world)]


def strong_share(args, rank: int, world: int) -> np.ndarray:
    """This rank's running sequences when config 3's one batch of `batch` sequences (the
    draw the 1-GPU run uses) is sharded over `world` GPUs: batch / world per GPU, dealt
    longest first in snake order (strong scaling: the global batch is fixed)."""
    glob = np.random.default_rng(SEED).integers(args.min_len, args.max_len + 1,
                                                size=args.batch)
    return glob[snake_deal(glob, rank, world)]


def snake_deal(lengths: np.ndarray, rank: int, world: int) -> np.ndarray:
    """Indices of `lengths` that rank `rank` holds when they are dealt longest first in
    snake order (seats 0..N-1, then N-1..0, ...): the per-rank sums stay nearly equal."""
    order = np.argsort(-np.asarray(lengths), kind="stable")
    pos = np.arange(order.size)
    turn, seat = pos // world, pos % world
    owner = np.where(turn % 2 == 0, seat, world - 1 - seat)
    return order[owner == rank]


class Workload:
    """Engine, caches, per-layer inputs and the churn process of one rank."""

    def __init__(self, args, rank: int, device, world: int = 1):
        import torch

        from shellsmith_b200.engine import HybridCacheEngine, HybridConfig
        from shellsmith_b200.workloads import gdn_token_inputs_device

        self.args = args
        self.device = device
        self.cfg = HybridConfig(layers=args.layers, max_seqs=args.batch, num_pages=args.num_pages,
                                max_context=args.max_len + 2048 + args.steps + args.warmup + 64,
                                pages_per_split=args.pages_per_split or None)
        cfg = self.cfg
        self.engine = HybridCacheEngine(cfg, device, seed=SEED + 1000 * rank)
        self.rng = np.random.default_rng(SEED + 1000 * rank)
        gen = torch.Generator(device=device)
        gen.manual_seed(SEED + 1000 * rank)
        # Pool and state contents: tile one random block over the buffers
        # (the values never steer control flow; tiling keeps setup short).
        block = torch.randn(1 << 27, generator=gen, device=device)
        kv_flat = self.engine.kv.view(-1)
        tile = block.to(torch.bfloat16)
        for start in range(0, kv_flat.numel(), tile.numel()):
            part = kv_flat[start:start + tile.numel()]
            part.copy_(tile[:part.numel()])
        st_flat = self.engine.state.view(-1)
        tile = block.mul(0.05).to(self.engine.state.dtype)
        for start in range(0, st_flat.numel(), tile.numel()):
            part = st_flat[start:start + tile.numel()]
            part.copy_(tile[:part.numel()])
        del block, tile
        # Running sequences: admitted with their current context (already
        # prefilled); each decode step appends one token.
        lengths = self.rng.integers(args.min_len, args.max_len + 1, size=args.batch)
        if world > 1:
            lengths = balanced_share(args, rank, world)
        self.initial = np.asarray(lengths).copy()
        self.next_id = 0
        for length in lengths:
            self.engine.blocks.admit(self._new_id(), int(length) - 1)
        # Per-layer inputs and outputs (device-resident, reused every step).
        self.inputs, self.outputs = {}, {}
        B = cfg.max_seqs
        for layer in range(cfg.layers):
            if cfg.is_attention(layer):
                q = torch.randn((B, cfg.q_heads, cfg.head_dim), generator=gen,
                                device=device).to(torch.bfloat16)
                k = torch.randn((B, cfg.kv_heads, cfg.head_dim), generator=gen,
                                device=device).to(torch.bfloat16)
                v = torch.randn((B, cfg.kv_heads, cfg.head_dim), generator=gen,
                                device=device).to(torch.bfloat16)
                self.inputs[layer] = (q, k, v)
                self.outputs[layer] = torch.empty((B, cfg.q_heads, cfg.head_dim),
                                                  dtype=torch.bfloat16, device=device)
            else:
                self.inputs[layer] = gdn_token_inputs_device(
                    gen, B, cfg.gdn_key_heads, cfg.gdn_value_heads, cfg.key_dim, cfg.value_dim,
                    device=device)
                self.outputs[layer] = torch.empty((B, cfg.gdn_value_heads, cfg.value_dim),
                                                  dtype=torch.bfloat16, device=device)
        # Prompt inputs for the prefill of admitted sequences: one packed
        # buffer of PROMPT_CAP tokens, shared by every layer (values are
        # synthetic; their distributions match the decode inputs).
        cap = self.PROMPT_CAP
        self.prompt_k = torch.randn((cap, cfg.kv_heads, cfg.head_dim), generator=gen,
                                    device=device).to(torch.bfloat16)
        self.prompt_v = torch.randn_like(self.prompt_k)
        self.prompt_gdn = gdn_token_inputs_device(gen, cap, cfg.gdn_key_heads,
                                                  cfg.gdn_value_heads, cfg.key_dim,
                                                  cfg.value_dim, device=device)
        self.prompt_out = torch.empty((cap, cfg.gdn_value_heads, cfg.value_dim),
                                      dtype=torch.bfloat16, device=device)
        self.finished = 0
        self.admitted = 0
        self.prefill_tokens = 0
        self.prefill_launches = 0

    PROMPT_CAP = 16384

    def _new_id(self):
        self.next_id += 1
        return self.next_id

    def reset(self, lengths) -> None:
        """Release every running sequence and admit `lengths` afresh (contexts already
        prefilled; the next decode step appends token `length`), so a timed window
        starts from the config's stated draw rather than a batch the churn of earlier
        phases has shortened. Churn draws continue from the same generator."""
        blocks = self.engine.blocks
        for slot in np.flatnonzero(blocks.active).tolist():
            self.engine.release(slot)
        for length in lengths:
            blocks.admit(self._new_id(), int(length) - 1)

    def churn(self) -> list:
        """Retire Bernoulli(p) finishers and admit replacements; returns new slots."""
        blocks = self.engine.blocks
        active = np.flatnonzero(blocks.active)
        done = active[self.rng.random(len(active)) < self.args.churn]
        for slot in done.tolist():
            self.engine.release(slot)
        self.finished += len(done)
        new = []
        for _ in range(len(done)):
            prompt = int(self.rng.integers(256, 2048 + 1))
            if not blocks.can_admit(prompt + 1):
                break
            new.append((self.engine.admit(self._new_id(), prompt), prompt))
        self.admitted += len(new)
        return new

    def prefill(self, new: list) -> None:
        """Prefill the admitted prompts: chunked GDN prefill into their state
        rows (all GDN layers) and their K/V into every attention layer's pages."""
        gdn = lambda layer, n: tuple(t[:n] for t in self.prompt_gdn)  # noqa: E731
        kv = lambda layer, n: (self.prompt_k[:n], self.prompt_v[:n])  # noqa: E731
        group, total = [], 0
        for slot, prompt in new + [(None, None)]:
            if slot is None or total + prompt > self.PROMPT_CAP:
                # GDN chunk launches only: the K/V writes are counted by paged as they launch.
                launched = self.engine.prefill(group, gdn, kv, self.prompt_out)
                self.prefill_launches += max(0, launched - len(self.cfg.attention_layers))
                group, total = [], 0
            if slot is not None:
                group.append((slot, prompt))
                total += prompt
                self.prefill_tokens += prompt


# ------------------------------------------------------------------ parity checks
# Checks of the measured paths, run on the device after their timed windows (never
# timed): plain PyTorch float64 restatements of the kernels' math, so every rank of a
# multi-GPU run checks its own share. The test suite checks the same kernels against
# the CPU oracle.
ATTN_RTOL, ATTN_ATOL = 2e-2, 3e-3   # bf16 outputs; the kernel's P.V uses bf16 probabilities
GDN_RTOL, GDN_ATOL, STATE_ATOL = 2e-2, 2e-3, 1e-4


def pool_tokens(pool, pages, length: int):
    """Logical K, V [length, Hkv, D] of one sequence from a bf16 page pool
    [num_pages, Hkv, 2, P, D], whose token row t stores its 16-byte chunk c at chunk
    position c ^ (t & 7) (the layout include/shellcache.h documents)."""
    import torch

    dev = pool.device
    P, D = pool.shape[3], pool.shape[4]
    n = -(-length // P)
    idx = torch.as_tensor(np.asarray(pages[:n], np.int64), device=dev)
    blocks = pool.index_select(0, idx)                              # [n, Hkv, 2, P, D]
    hkv, ch = blocks.shape[1], D // 8
    swz = torch.arange(ch, device=dev)[None, :] ^ (torch.arange(P, device=dev)[:, None] & 7)
    x = torch.gather(blocks.view(n, hkv, 2, P, ch, 8), 4,
                     swz.view(1, 1, 1, P, ch, 1).expand(n, hkv, 2, P, ch, 8))
    x = x.reshape(n, hkv, 2, P, D).permute(2, 0, 3, 1, 4).reshape(2, n * P, hkv, D)
    return x[0, :length], x[1, :length]


def partial_fp64(q, k, v, scale: float) -> tuple:
    """Attention of query rows q [R, D] over k, v [L, D] in float64: (normalised out
    [R, D], natural-log lse [R])."""
    import torch

    s = (k.double() @ q.double().T) * scale                         # [L, R]
    m = s.max(dim=0).values
    p = torch.exp(s - m)
    total = p.sum(dim=0)
    return (p.T @ v.double()) / total[:, None], m + torch.log(total)


def merge_fp64(parts) -> tuple:
    """Merge (out [R, D], lse [R]) float64 partials of disjoint key ranges."""
    import torch

    lse = torch.stack([p[1] for p in parts])
    top = lse.max(dim=0).values
    w = torch.exp(lse - top)
    out = (w[:, :, None] * torch.stack([p[0] for p in parts])).sum(dim=0) / w.sum(dim=0)[:, None]
    return out, top + torch.log(w.sum(dim=0))


def close(got, want, rtol: float, atol: float) -> bool:
    import torch

    return bool(torch.all((got.double().cpu() - want.double().cpu()).abs()
                          <= atol + rtol * want.double().cpu().abs()))


def attention_row_ok(out, q, k, v, scale: float) -> bool:
    """out, q [Hq, D] of one sequence against float64 attention over its k, v
    [L, Hkv, D] (query head h reads kv head h // (Hq / Hkv))."""
    hq, hkv = q.shape[0], k.shape[1]
    g = hq // hkv
    ok = True
    for j in range(hkv):
        want, _ = partial_fp64(q[j * g:(j + 1) * g], k[:, j], v[:, j], scale)
        ok &= close(out[j * g:(j + 1) * g], want, ATTN_RTOL, ATTN_ATOL)
    return ok


def gdn_row_ok(before, after, out, q, k, v, decay, beta) -> bool:
    """One sequence's GDN token update against float64: state [Hv, dv, dk] before and
    after, out [Hv, dv]; q, k [Hk, dk], v [Hv, dv], decay, beta [Hv]; key head of
    value head h is h // (Hv / Hk). Decayed S = a S; pred = S k; S' = S + beta (v -
    pred) k^T; out = S' q."""
    import torch

    g = v.shape[0] // q.shape[0]
    qq = q.double().repeat_interleave(g, 0)
    kk = k.double().repeat_interleave(g, 0)
    dec = decay.double()[:, None, None] * before.double()
    pred = torch.einsum("hvk,hk->hv", dec, kk)
    want = dec + (beta.double()[:, None] * (v.double() - pred))[:, :, None] * kk[:, None, :]
    o = torch.einsum("hvk,hk->hv", want, qq)
    state_ok = float((after.double() - want).abs().max()) <= STATE_ATOL
    return state_ok and close(out, o, GDN_RTOL, GDN_ATOL)


def step_parity(wl) -> tuple:
    """One more decode step of the workload (untimed) with two of this rank's rows
    checked, its longest and its shortest sequence: the first GDN layer's state update
    and output, and the first attention layer's output over the row's whole paged
    context, its appended token included. Returns (rows failing, rows checked)."""
    import torch

    eng, cfg = wl.engine, wl.cfg
    active = np.flatnonzero(eng.blocks.active)
    lens = eng.blocks.lengths[active]
    rows = sorted({int(active[np.argmax(lens)]), int(active[np.argmin(lens)])})
    gl, al = cfg.gdn_layers[0], cfg.attention_layers[0]
    gi = eng.gdn_index[gl]
    before = eng.state[gi, rows].clone()
    eng.begin_step()
    eng.decode_step(wl.inputs, wl.outputs)
    torch.cuda.synchronize()
    bad = 0
    q, k, v, decay, beta = wl.inputs[gl]
    for i, r in enumerate(rows):
        bad += not gdn_row_ok(before[i], eng.state[gi, r], wl.outputs[gl][r], q[r], k[r], v[r],
                              decay[r], beta[r])
    pool = eng.kv[eng.attn_index[al]]
    for r in rows:
        kk, vv = pool_tokens(pool, eng.blocks.pages[r], int(eng.blocks.lengths[r]))
        bad += not attention_row_ok(wl.outputs[al][r], wl.inputs[al][0][r], kk, vv, eng.scale)
    return bad, 2 * len(rows)


def parity_word(bad: float, checked: float) -> str:
    return "ok" if bad == 0 else f"FAILED {int(bad)} of {int(checked)}"


def run_ours(args, world, rank, local):
    import torch

    from shellsmith_b200 import _build, _capi, paged

    _build.build()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    wl = Workload(args, rank, device, world)
    eng = wl.engine
    cfg = wl.cfg
    stream = torch.cuda.current_stream(device)

    # Launch counter: kernels this build launches per decode step: one update per GDN
    # layer; the attention layers' kernels are counted as they launch (paged counts
    # them: one when the append folds into the split-K launch, else the append, the
    # split-K kernel and, when a sequence spans splits, the merge).
    def launches_per_step():
        return len(cfg.gdn_layers)

    def step(timed_events=None, layer_events=None):
        new = wl.churn()
        p0 = torch.cuda.Event(enable_timing=True)
        p1 = torch.cuda.Event(enable_timing=True)
        p0.record(stream)
        wl.prefill(new)
        p1.record(stream)
        n = eng.begin_step()
        lengths = eng.blocks.lengths[eng.blocks.active].copy()
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        if layer_events is None:
            eng.decode_step(wl.inputs, wl.outputs)
        else:
            for layer in range(cfg.layers):
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                if cfg.is_attention(layer):
                    eng.attention_layer(layer, *wl.inputs[layer], wl.outputs[layer])
                else:
                    eng.gdn_layer(layer, *wl.inputs[layer], wl.outputs[layer],
                                  chained=layer > 0)
                e1.record(stream)
                layer_events.append((cfg.is_attention(layer), e0, e1, lengths))
        s1.record(stream)
        if timed_events is not None:
            timed_events.append((s0, s1, p0, p1, n, lengths, len(new)))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    _capi.check_device()

    # Each measured window starts from config 3's stated draw (contexts U[min, max]):
    # churn replaces finished sequences with shorter prompts, so a window that ran after
    # earlier phases would measure a lighter batch.
    e2e = None
    if not args.no_e2e:
        wl.reset(wl.initial)
        e2e = run_e2e(args, wl, world)
        _capi.check_device()

    wl.reset(wl.initial)
    barrier(world)
    torch.cuda.synchronize()
    events, layer_events = [], []
    launches_before = wl.prefill_launches
    attn_before = paged.attention_launches
    with ClockSampler(local) as clocks:
        t0 = time.perf_counter()
        for i in range(args.steps):
            step(events)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    barrier(world)
    _capi.check_device()
    timed_launches = (launches_per_step() * args.steps + paged.attention_launches - attn_before
                      + wl.prefill_launches - launches_before)
    # Per-layer rates (the roofline of each kernel) from a separate pass over the same
    # starting draw, after the timed window: an event between two layers keeps the next
    # layer's launch from overlapping the tail of the one before it (1.4 % of the step
    # at 256 sequences, 7 % at 32), so the timed steps carry none.
    sample_layers(wl, step, layer_events, args.steps, wl.initial)

    decode_ms = [s0.elapsed_time(s1) for s0, s1, *_ in events]
    prefill_ms = [p0.elapsed_time(p1) for _, _, p0, p1, *_ in events]
    tokens = sum(e[4] for e in events)
    decode_s = sum(decode_ms) / 1e3
    bytes_total = sum(eng.step_bytes(e[5])["total"] for e in events)
    # Per-layer bytes over the steps that carried per-layer events.
    gdn_bytes = sum(eng.step_bytes(le[3])["gdn"] / len(cfg.gdn_layers)
                    for le in layer_events if not le[0])
    attn_ms = sum(a.elapsed_time(b) for is_attn, a, b, _ in layer_events if is_attn)
    gdn_ms = sum(a.elapsed_time(b) for is_attn, a, b, _ in layer_events if not is_attn)
    attn_bytes = sum(eng.step_bytes(le[3])["attention_per_layer"]
                     for le in layer_events if le[0])
    n_attn_launch = sum(1 for le in layer_events if le[0])
    n_gdn_launch = sum(1 for le in layer_events if not le[0])
    timed_ctx = np.concatenate([e[5] for e in events]).astype(np.float64)
    ctx_stats = [float(timed_ctx.sum()), float(timed_ctx.size), float(timed_ctx.min()),
                 float(timed_ctx.max())]

    decode_s_max = max_over_ranks(decode_s, world)
    tokens_all = sum_over_ranks(tokens, world)
    wall_max = max_over_ranks(wall, world)
    ctx_sum, ctx_n = sum_over_ranks(ctx_stats[0], world), sum_over_ranks(ctx_stats[1], world)
    ctx_min = -max_over_ranks(-ctx_stats[2], world)
    ctx_max = max_over_ranks(ctx_stats[3], world)
    peaks = measured_peaks()
    hbm = peaks["hbm_gbs"]
    bad, checked = step_parity(wl)
    bad, checked = sum_over_ranks(bad, world), sum_over_ranks(checked, world)
    _capi.check_device()

    strong = attention_c2 = long_c4 = None
    prefill_c1 = front = kv8 = decode_c0 = None
    if not args.no_config1:
        # Config 3 as stated (256 sequences in all, sharded over the GPUs), then the
        # other sharded configs, on every rank (each with its own collectives, in the
        # same order everywhere): config 2 by sequence, config 4 by KV page.
        barrier(world)
        strong = config3_strong(args, wl, world, rank, step)
        attention_c2 = config2_attention(device, rank=rank, world=world)
        long_c4 = config4_measure(args, world, rank, local, steps=200, warmup=5,
                                  exchange=args.exchange)
        barrier(world)
    if not args.no_config1 and rank == 0:
        prefill_c1 = config1_prefill(device)
        decode_c0 = config0_decode(device)
        front = gdn_front_layer(device)
        kv8 = kv8_attention_layer(wl, device)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args, wl)

    if rank != 0:
        return None
    step_gbs = bytes_total / decode_s / 1e9
    attn_gbs = attn_bytes / (attn_ms / 1e3) / 1e9
    gdn_gbs = gdn_bytes / (gdn_ms / 1e3) / 1e9
    line = {
        "metric": METRIC,
        "value": round(tokens_all / decode_s_max, 1),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(decode_s_max * 1e3 / args.steps, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16 kv / fp32 gdn state",
        "data": "synthetic (seeded; config 3 shapes and distributions)",
        "config": {
            "workload": f"config3 hybrid decode cache step: {cfg.layers} layers "
                        f"({len(cfg.gdn_layers)} GDN + {len(cfg.attention_layers)} attention), "
                        f"{args.batch} ragged sequences per GPU, ctx U[{args.min_len},"
                        f"{args.max_len}], churn {args.churn}/step",
            "global_batch": args.batch * world, "seq_len": f"U[{args.min_len},{args.max_len}]",
            "mean_ctx_timed": round(ctx_sum / ctx_n, 1),
            "ctx_timed_range": [int(ctx_min), int(ctx_max)],
            "timed_from": "the stated draw (batch re-admitted at U[min, max] before the window)",
            "parallelism": f"sequence-sharded x{world}, no collective",
            "gdn": "Hk16/Hv32 dk=dv=128 fp32 state", "attention": "Hq16/Hkv2 D256 page16",
            "pages_per_split": args.pages_per_split or "adaptive (<= 1024, >= 3 waves of CTAs)",
            "l2": "working set ~90 GB/step > L2 (no flush needed)",
        },
        "parity": parity_word(bad, checked),
        "hbm": {"step_gbs": round(step_gbs, 1), "peak_gbs": hbm,
                "frac": round(step_gbs / hbm, 4), "peak_source": peaks["source"],
                "bytes_per_step": round(bytes_total / max(1, len(events))),
                "gdn_gbs": round(gdn_gbs, 1), "attention_gbs": round(attn_gbs, 1),
                "gdn_traffic_per_launch": round(GDN_TRAFFIC_RATIO * gdn_bytes
                                                / max(1, n_gdn_launch))},
        "roofline": {"bound": "hbm",
                     "kernel": "paged_decode_attention_fused (append folded into split-K; "
                               "+ merge when a sequence spans splits)",
                     "achieved": round(attn_gbs, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(attn_gbs / hbm, 4),
                     "traffic": round(ATTN_TRAFFIC_RATIO * attn_bytes / max(1, n_attn_launch)),
                     "bytes_per_launch": round(attn_bytes / max(1, n_attn_launch)),
                     "peak_source": peaks["source"]},
        "prefill": {"ms_per_step": round(statistics.mean(prefill_ms), 3),
                    "tokens": wl.prefill_tokens, "admitted": wl.admitted,
                    "finished": wl.finished,
                    "note": "admitted prompts: chunked GDN prefill (tcgen05) into their state "
                            "rows for every GDN layer + K/V written to every attention layer; "
                            "timed separately, excluded from decode bytes"},
        "wall_ms_per_step": round(wall_max * 1e3 / args.steps, 3),
        "gpu_launches": timed_launches,
        "clocks": clocks.summary(),
    }
    if e2e is not None:
        line["e2e"] = e2e
    if prefill_c1 is not None:
        line["config1_prefill"] = prefill_c1
        line["config0_decode"] = decode_c0
    if front is not None:
        line["gdn_front"] = front
    if kv8 is not None:
        line["kv8_attention"] = kv8
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if strong is not None:
        # The sharded configs last and compact, so the tail of the line carries them.
        line["sharded_workloads"] = SHARDED_WORKLOADS
        line["config3_strong"] = strong
        line["config2_attention"] = attention_c2
        line["config4_long_sequence"] = long_c4
    print(json.dumps(line), flush=True)
    return line


SHARDED_WORKLOADS = (
    "config3_strong: config 3's 256 sequences in all, 256/N per GPU; config2_attention: 64 "
    "seqs U[1k,32k] dealt over the GPUs; config4_long_sequence: one 131,072-token sequence, "
    "KV pages split over the GPUs, partials exchanged over NVLink. tokens_per_s: all GPUs; "
    "fractions of measured HBM; parity: float64 checks on every rank")


def sample_layers(wl, step, layer_events, steps: int, start) -> None:
    """Runs min(steps, 4) steps from the draw `start` with CUDA events around every
    layer, appending (is_attention, start, end, lengths) to layer_events."""
    import torch

    from shellsmith_b200 import _capi

    wl.reset(start)
    for _ in range(max(1, min(steps, 4))):
        step(None, layer_events)
    torch.cuda.synchronize()
    _capi.check_device()


def config3_strong(args, wl, world, rank, step, warmup: int = 2) -> dict | None:
    """Config 3 as stated: one batch of `batch` sequences (the 1-GPU draw) sharded by
    sequence over the ranks, batch / world per GPU (strong scaling), timed like the
    headline window from the stated draw. Every rank calls it; returns the record on
    rank 0."""
    import torch

    from shellsmith_b200 import _capi

    eng = wl.engine
    wl.reset(strong_share(args, rank, world))
    for _ in range(warmup):
        step()
    wl.reset(strong_share(args, rank, world))
    torch.cuda.synchronize()
    barrier(world)
    events, layer_events = [], []
    for i in range(args.steps):
        step(events)
    torch.cuda.synchronize()
    _capi.check_device()
    decode_s = sum(e[0].elapsed_time(e[1]) for e in events) / 1e3
    # Per-layer rates from a separate sampled pass: what limits the strong-scaling curve.
    sample_layers(wl, step, layer_events, args.steps, strong_share(args, rank, world))
    n_gdn = len(wl.cfg.gdn_layers)
    attn_s = sum(a.elapsed_time(b) for is_attn, a, b, _ in layer_events if is_attn) / 1e3
    gdn_s = sum(a.elapsed_time(b) for is_attn, a, b, _ in layer_events if not is_attn) / 1e3
    attn_b = sum(eng.step_bytes(le[3])["attention_per_layer"] for le in layer_events if le[0])
    gdn_b = sum(eng.step_bytes(le[3])["gdn"] / n_gdn for le in layer_events if not le[0])
    tokens = sum(e[4] for e in events)
    nbytes = sum(eng.step_bytes(e[5])["total"] for e in events)
    ctx = np.concatenate([e[5] for e in events]).astype(np.float64)
    seqs = len(events[0][5])
    decode_max = max_over_ranks(decode_s, world)
    tokens_all = sum_over_ranks(tokens, world)
    gbs_per_gpu = sum_over_ranks(nbytes, world) / world / decode_max / 1e9
    peak = measured_peaks()["hbm_gbs"]
    attn_frac = -max_over_ranks(-(attn_b / max(attn_s, 1e-9) / 1e9 / peak), world)
    gdn_frac = -max_over_ranks(-(gdn_b / max(gdn_s, 1e-9) / 1e9 / peak), world)
    ctx_sum, ctx_n = sum_over_ranks(float(ctx.sum()), world), sum_over_ranks(ctx.size, world)
    bad, checked = step_parity(wl)
    bad, checked = sum_over_ranks(bad, world), sum_over_ranks(checked, world)
    _capi.check_device()
    if rank != 0:
        return None
    return {"n_gpus": world, "seqs_per_gpu": seqs, "steps": args.steps,
            "ms_per_step": round(decode_max * 1e3 / args.steps, 3),
            "tokens_per_s": round(tokens_all / decode_max, 1),
            "hbm_frac_per_gpu": round(gbs_per_gpu / peak, 4),
            "layer_frac_min_rank": {"gdn": round(gdn_frac, 3), "attention": round(attn_frac, 3)},
            "mean_ctx": round(ctx_sum / ctx_n), "parity": parity_word(bad, checked)}


def gdn_front_layer(device, batch: int = 256, rounds: int = 5) -> dict:
    """A config-3 GDN layer run from its projections: the fused front kernel
    (conv taps + SiLU + q/k norm + gates + state update + gated norm, one launch)
    beside the plain state update over the same rows. Four layers' states rotate
    (2 GiB > L2). Algorithmic bytes per fused launch: per row the state read and
    written, qkv, z, a, b, three tap rows read and one written, the output; plus
    the layer's weights once."""
    import torch

    from shellsmith_b200 import gdn_layer, numerics
    from shellsmith_b200.workloads import gdn_token_inputs_device

    B, Hk, Hv, d, layers = batch, 16, 32, 128, 4
    C = (2 * Hk + Hv) * d
    gen = torch.Generator(device=device)
    gen.manual_seed(5)
    states = [torch.zeros((B, Hv, d, d), dtype=torch.float32, device=device)
              for _ in range(layers)]
    taps = [torch.zeros((B, gdn_layer.RING, C), dtype=torch.bfloat16, device=device)
            for _ in range(layers)]
    weights = [gdn_layer.GDNWeights(
        conv_w=(torch.randn((C, 4), generator=gen, device=device) * 0.5).to(torch.bfloat16),
        a_log=torch.rand(Hv, generator=gen, device=device) * 2.7,
        dt_bias=torch.randn(Hv, generator=gen, device=device),
        norm_w=torch.ones(d, dtype=torch.bfloat16, device=device), eps=1e-6,
        key_heads=Hk, value_heads=Hv) for _ in range(layers)]
    qkv = torch.randn((B, C), generator=gen, device=device).to(torch.bfloat16)
    z = torch.randn((B, Hv * d), generator=gen, device=device).to(torch.bfloat16)
    a = torch.randn((B, Hv), generator=gen, device=device).to(torch.bfloat16)
    b = torch.randn((B, Hv), generator=gen, device=device).to(torch.bfloat16)
    out = torch.empty((B, Hv * d), dtype=torch.bfloat16, device=device)
    q, k, v, decay, beta = gdn_token_inputs_device(gen, B, Hk, Hv, d, d, device=device)
    out3 = out.view(B, Hv, d)
    pos = torch.full((B,), 5, dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream(device)

    def fused(i):
        gdn_layer.gdn_decode_fused(qkv, z, a, b, weights[i], taps[i], pos, states[i], out=out)

    ws = gdn_layer.SplitWorkspace(B, weights[0], device)

    def split(i):
        gdn_layer.gdn_decode_split(qkv, z, a, b, weights[i], taps[i], pos, states[i], out=out,
                                   workspace=ws)

    def plain(i):
        numerics.gdn_decode(q, k, v, decay, beta, states[i], out=out3)

    # Each form runs rounds x layers back to back between one pair of events, so
    # host-side launch work overlaps the device work as it does inside a decode step.
    result = {}
    for name, fn in (("fused", fused), ("split", split), ("plain", plain)):
        for i in range(layers):
            fn(i)
        samples = []
        for _ in range(3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record(stream)
            for _ in range(rounds):
                for i in range(layers):
                    fn(i)
            e1.record(stream)
            torch.cuda.synchronize()
            samples.append(e0.elapsed_time(e1) / (rounds * layers))
        result[name] = statistics.median(samples)
    state_rw = 2 * Hv * d * d * 4
    fused_bytes = B * (state_rw + C * 2 + Hv * d * 2 + 2 * Hv * 2 + 4 * C * 2 + Hv * d * 2) + (
        C * 4 * 2 + Hv * 8 + d * 2)
    plain_bytes = B * (state_rw + (2 * Hk * d + 2 * Hv * d) * 2 + 2 * Hv * 4)
    peaks = measured_peaks()
    gbs = fused_bytes / (result["fused"] / 1e3) / 1e9
    split_gbs = fused_bytes / (result["split"] / 1e3) / 1e9
    return {"workload": f"config3 GDN layer from projections, B={B}, Hk16/Hv32 128x128 fp32 "
                        f"state, conv K=4 tap ring",
            "fused_ms": round(result["fused"], 4), "split_ms": round(result["split"], 4),
            "plain_update_ms": round(result["plain"], 4),
            "fused_gbs": round(gbs, 1), "fused_frac": round(gbs / peaks["hbm_gbs"], 4),
            "split_gbs": round(split_gbs, 1),
            "split_frac": round(split_gbs / peaks["hbm_gbs"], 4),
            "plain_gbs": round(plain_bytes / (result["plain"] / 1e3) / 1e9, 1),
            "bytes_per_launch": fused_bytes, "layer_calls": 3 * rounds * layers,
            "note": "fused = the whole GDN glue of bf16.py:44-139 around the update in one "
                    "launch (2-CTA clusters); split = the same in three launches (front + tap "
                    "rows, update, gated norm); plain = the state update alone on "
                    "pre-made q/k/v/g/beta. GB/s use the fused bytes for both forms"}


def kv8_attention_layer(wl, device, rounds: int = 5) -> dict:
    """One attention layer of the step just measured (append + split-K attention
    over the same block tables and context lengths) on 8-bit pages beside bf16
    pages. Algorithmic bytes per launch as step_bytes, with a cached token
    costing 2 * Hkv * D code bytes plus 8 * Hkv * D / 64 of bf16 scale and bias."""
    import torch

    from shellsmith_b200 import paged

    eng, cfg = wl.engine, wl.cfg
    layer = cfg.attention_layers[0]
    q, k, v = wl.inputs[layer]
    out = wl.outputs[layer]
    D = cfg.head_dim
    pool8 = paged.new_pool_q8(cfg.num_pages, cfg.kv_heads, D, device)
    pool8.random_(0, 256)
    pool8[:, :, 32 * D:].view(torch.bfloat16).fill_(0.01)   # scales and biases
    stream = torch.cuda.current_stream(device)

    plan = dict(max_pages_in_batch=eng.max_pages_in_batch, pages_per_split=cfg.pages_per_split,
                total_pages=eng.total_pages, workspace=eng.workspace, out=out,
                seq_order=eng.seq_order)

    def run(pool):   # the engine's attention layer on either pool
        paged.append_and_attend(q, k, v, eng.slot_map, pool, eng.table, eng.ctx_len, eng.scale,
                                **plan)

    def run_two(pool):   # the append and the attention as separate launches
        paged.kv_append(k, v, pool, eng.slot_map)
        paged.paged_decode_attention(q, pool, eng.table, eng.ctx_len, eng.scale, **plan)

    ms = {}
    bf16_pool = eng.kv[eng.attn_index[layer]]
    for name, fn, pool in (("bf16", run, bf16_pool), ("bf16_two", run_two, bf16_pool),
                           ("8bit", run, pool8)):
        fn(pool)
        fn(pool)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(rounds):
            fn(pool)
        e1.record(stream)
        torch.cuda.synchronize()
        ms[name] = e0.elapsed_time(e1) / rounds
    del pool8
    active = np.flatnonzero(eng.blocks.active)
    lengths = eng.blocks.lengths[active].astype(np.float64)
    n = len(lengths)
    rows = {"bf16": cfg.kv_heads * D * 4, "bf16_two": cfg.kv_heads * D * 4,
            "8bit": cfg.kv_heads * (2 * D + 8 * D / 64)}
    extra = n * cfg.q_heads * D * 4 + float(np.ceil(lengths / cfg.page_size).sum()) * 4
    nbytes = {key: float(lengths.sum()) * r + n * r + extra for key, r in rows.items()}
    peaks = measured_peaks()
    gbs = {key: nbytes[key] / (ms[key] / 1e3) / 1e9 for key in ms}
    return {"workload": f"one config-3 attention layer, {n} sequences, mean ctx "
                        f"{lengths.mean():.0f}, Hq{cfg.q_heads}/Hkv{cfg.kv_heads} D{D}",
            "bf16_ms": round(ms["bf16"], 4), "kv8_ms": round(ms["8bit"], 4),
            "bf16_two_launch_ms": round(ms["bf16_two"], 4),
            "speedup": round(ms["bf16"] / ms["8bit"], 3),
            "bf16_gbs": round(gbs["bf16"], 1), "kv8_gbs": round(gbs["8bit"], 1),
            "kv8_frac": round(gbs["8bit"] / peaks["hbm_gbs"], 4),
            "kv8_bytes_per_launch": round(nbytes["8bit"]), "launches": rounds,
            "note": "8-bit pages hold random codes with bf16 scale/bias 0.01; timing does not "
                    "depend on the values"}


def kv8_layer_standalone(args, device, rounds: int = 10) -> dict:
    """One config-3 attention layer (append + split-K attention + combine) over
    --batch sequences of U[--min-len, --max-len] tokens, on 8-bit and on bf16
    pages (random contents; timing does not depend on the values)."""
    import torch

    from shellsmith_b200 import paged

    rng = np.random.default_rng(SEED)
    B, Hq, Hkv, D, P = args.batch, 16, 2, 256, paged.PAGE_SIZE
    lengths = rng.integers(args.min_len, args.max_len + 1, size=B)
    need = np.ceil(lengths / P).astype(np.int64)
    num_pages, width = int(need.sum()) + 16, int(need.max())
    perm = rng.permutation(num_pages)
    table = np.zeros((B, width), np.int32)
    cursor = 0
    for b, n in enumerate(need):
        table[b, :n] = perm[cursor:cursor + n]
        cursor += n
    slots = (table[np.arange(B), (lengths - 1) // P].astype(np.int64) * P + (lengths - 1) % P)
    bt = torch.from_numpy(table).to(device)
    ctx = torch.from_numpy(lengths.astype(np.int32)).to(device)
    slot_t = torch.from_numpy(slots).to(device)
    gen = torch.Generator(device=device)
    gen.manual_seed(SEED)
    q = torch.randn((B, Hq, D), generator=gen, device=device).to(torch.bfloat16)
    kn = torch.randn((B, Hkv, D), generator=gen, device=device).to(torch.bfloat16)
    out = torch.empty_like(q)
    total = int(need.sum())
    ws = paged.AttentionWorkspace(B, Hq, D, paged.split_plan(width, 16)[1], device=device)
    stream = torch.cuda.current_stream(device)
    ms, nbytes = {}, {}
    for name in ("bf16", "8bit"):
        if name == "8bit":
            pool = paged.new_pool_q8(num_pages, Hkv, D, device)
            pool.random_(0, 256)
            pool[:, :, 32 * D:].view(torch.bfloat16).fill_(0.01)
            row = Hkv * (2 * D + 8 * D / 64)
        else:
            pool = paged.new_pool(num_pages, Hkv, D, device=device)
            pool.view(torch.int16).random_(0, 16000)  # finite bf16 values below 1
            row = Hkv * D * 4

        def run():
            paged.append_and_attend(q, kn, kn, slot_t, pool, bt, ctx, 1.0 / 16,
                                    max_pages_in_batch=width, total_pages=total, workspace=ws,
                                    out=out)

        for _ in range(3):
            run()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(rounds):
            run()
        e1.record(stream)
        torch.cuda.synchronize()
        ms[name] = e0.elapsed_time(e1) / rounds
        nbytes[name] = float(lengths.sum()) * row + B * row + B * Hq * D * 4 + total * 4
        del pool
    peaks = measured_peaks()
    return {"workload": f"attention layer, {B} sequences U[{args.min_len},{args.max_len}] "
                        f"(mean {lengths.mean():.0f}), Hq16/Hkv2 D256",
            "bf16_ms": round(ms["bf16"], 4), "kv8_ms": round(ms["8bit"], 4),
            "bf16_gbs": round(nbytes["bf16"] / ms["bf16"] / 1e6, 1),
            "kv8_gbs": round(nbytes["8bit"] / ms["8bit"] / 1e6, 1),
            "kv8_frac": round(nbytes["8bit"] / ms["8bit"] / 1e6 / peaks["hbm_gbs"], 4),
            "kv8_bytes_per_launch": round(nbytes["8bit"]), "launches": rounds + 3}


def config0_decode(device, steps: int = 256, rounds: int = 5) -> dict:
    """Config 0: GDN one-token decode, B=4 sequences, 8 heads, 128 x 128 fp32 state, 256
    steps from a zero state (each step reads the state the previous one wrote). The 2 MiB
    state stays in L2, so the step is bound by launch and dependency latency; tokens/s =
    B x steps / time. Inputs of all steps are made before the timed region. Timed twice:
    256 calls from Python (each call's host work included) and the same 256 launches
    replayed as one CUDA graph (the device-side chain)."""
    import torch

    from shellsmith_b200 import numerics
    from shellsmith_b200.workloads import gdn_token_inputs_device

    B, H, d = 4, 8, 128
    gen = torch.Generator(device=device)
    gen.manual_seed(0)
    inputs = [gdn_token_inputs_device(gen, B, H, H, d, d, device=device) for _ in range(steps)]
    state = torch.zeros((B, H, d, d), dtype=torch.float32, device=device)
    out = torch.empty((B, H, d), dtype=torch.bfloat16, device=device)
    stream = torch.cuda.current_stream(device)

    def run():
        for q, k, v, g, beta in inputs:
            numerics.gdn_decode(q, k, v, g, beta, state, out=out)

    def timed(fn):
        times = []
        for _ in range(rounds):
            state.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            times.append((e0, e1))
        torch.cuda.synchronize()
        return statistics.median(a.elapsed_time(b) for a, b in times)

    run()
    ms_calls = timed(run)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run()
    torch.cuda.synchronize()
    ms = timed(graph.replay)
    del graph
    return {"workload": "config0 GDN decode B=4 H=8 128x128 fp32 state, 256 dependent steps",
            "ms_per_256_steps": round(ms, 3), "us_per_step": round(ms * 1e3 / steps, 2),
            "tokens_per_s": round(B * steps / (ms / 1e3), 1),
            "python_calls": {"us_per_step": round(ms_calls * 1e3 / steps, 2),
                             "tokens_per_s": round(B * steps / (ms_calls / 1e3), 1)},
            "note": "graph replay of the 256 launches; state (2 MiB) L2-resident: "
                    "latency-bound, HBM fraction not meaningful",
            "launches": steps}


def config2_attention(device, steps: int = 20, warmup: int = 3, rank: int = 0,
                      world: int = 1) -> dict | None:
    """Config 2: paged KV append + split-K decode attention, bf16. 64 sequences with
    contexts U[1k, 32k], 16 query / 2 KV heads, D 256, pages of 16 tokens handed out from a
    random permutation of a 150k-page pool. Each step appends one token per sequence and
    attends over the grown context. Slots, lengths and the launch order (longest first) of
    every step are made before the timed region; 2.2 GB per step, well above L2.

    Sharded by sequence over `world` ranks with no collective on the data path (every
    rank calls this): the 64 sequences are dealt longest first in snake order, each rank
    runs its share on its own pool, and the step time is the max over ranks (strong
    scaling: the 64 sequences are fixed). Returns the record on rank 0, else None."""
    import torch

    from shellsmith_b200 import paged

    B_all, hq, hkv, D, P, NP = 64, 16, 2, 256, 16, 150_000
    total = warmup + steps
    rng = np.random.default_rng(2)
    lengths_all = rng.integers(1024, 32 * 1024 + 1, size=B_all)
    lengths = lengths_all[np.sort(snake_deal(lengths_all, rank, world))] if world > 1 \
        else lengths_all
    B = len(lengths)
    need = -(-(lengths + total) // P)
    perm = rng.permutation(NP).astype(np.int32)
    table = np.zeros((B, int(need.max())), np.int32)
    cursor = 0
    for b in range(B):
        table[b, :need[b]] = perm[cursor:cursor + need[b]]
        cursor += need[b]
    pos = lengths[None, :] + np.arange(total)[:, None]            # [step, B] new token index
    slots = table[np.arange(B)[None, :], pos // P].astype(np.int64) * P + pos % P
    ctx = (pos + 1).astype(np.int32)
    gen = torch.Generator(device=device)
    gen.manual_seed(2)
    pool = torch.empty((NP, hkv, 2, P, D), dtype=torch.bfloat16, device=device)
    flat, block = pool.view(-1), 1 << 26
    for start in range(0, flat.numel(), block):
        part = flat[start:start + block]
        part.copy_(torch.randn(part.shape, generator=gen, device=device))
    table_d = torch.from_numpy(table).to(device)
    slots_d = torch.from_numpy(slots).to(device)
    ctx_d = torch.from_numpy(ctx).to(device)
    order = torch.from_numpy(np.argsort(-lengths, kind="stable").astype(np.int32)).to(device)
    q = torch.randn((B, hq, D), generator=gen, device=device).to(torch.bfloat16)
    kn = torch.randn((B, hkv, D), generator=gen, device=device).to(torch.bfloat16)
    vn = torch.randn((B, hkv, D), generator=gen, device=device).to(torch.bfloat16)
    out = torch.empty((B, hq, D), dtype=torch.bfloat16, device=device)
    max_pages = int(-(-ctx.max() // P))
    total_pages = int((-(-ctx[-1] // P)).sum())
    # The split is the library's own choice (total_pages given); the scratch
    # fits the smallest split it can pick.
    ws = paged.AttentionWorkspace(B, hq, D, paged.split_plan(max_pages, 16)[1], device=device)
    stream = torch.cuda.current_stream(device)

    def step(s):
        paged.append_and_attend(q, kn, vn, slots_d[s], pool, table_d, ctx_d[s], 1 / 16,
                                max_pages_in_batch=max_pages, total_pages=total_pages,
                                workspace=ws, out=out, seq_order=order)

    for s in range(warmup):
        step(s)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    launched = paged.attention_launches
    e0.record(stream)
    for s in range(warmup, total):
        step(s)
    e1.record(stream)
    launched = paged.attention_launches - launched
    torch.cuda.synchronize()
    from shellsmith_b200 import _capi

    _capi.check_device()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    c = ctx[warmup:].astype(np.float64)
    nbytes = (c.sum() * hkv * D * 2 * 2 + steps * B * hkv * D * 2 * 2
              + steps * B * hq * D * 2 * 2 + np.ceil(c / P).sum() * 4) / steps
    nbytes = sum_over_ranks(float(nbytes), world)
    gbs = nbytes / world / (ms / 1e3) / 1e9   # per GPU
    peak = measured_peaks()["hbm_gbs"]
    # Parity of the last step on this rank's longest and shortest sequence.
    bad = 0
    for b in sorted({int(np.argmax(lengths)), int(np.argmin(lengths))}):
        L = int(ctx[-1, b])
        kk, vv = pool_tokens(pool, table[b], L)
        bad += not attention_row_ok(out[b], q[b], kk, vv, 1 / 16)
    bad = sum_over_ranks(bad, world)
    checked = sum_over_ranks(min(2, B), world)
    del pool
    if rank != 0:
        return None
    return {"n_gpus": world, "seqs_per_gpu": B, "ms_per_step": round(ms, 4),
            "tokens_per_s": round(B_all / (ms / 1e3), 1), "hbm_frac_per_gpu": round(gbs / peak, 4),
            "launches_per_step": launched / steps,
            "parity": parity_word(bad, checked)}


def config1_prefill(device, steps: int = 5, warmup: int = 2) -> dict:
    """Config 1: chunked GDN prefill, B=8, T=4096, 16 key / 32 value heads, 128 x 128,
    fp32 state, on the tensor cores. Algorithmic FLOPs and bytes of the reference
    chunk algorithm (per (sequence, value head, chunk): QK^T/KK^T, two solves, two
    m-products, three state products, the inverse)."""
    import torch

    from shellsmith_b200 import numerics
    from shellsmith_b200.workloads import gdn_token_inputs_device

    B, T, Hk, Hv, d, C = 8, 4096, 16, 32, 128, 64
    gen = torch.Generator(device=device)
    gen.manual_seed(1)
    q, k, v, decay, beta = gdn_token_inputs_device(gen, B * T, Hk, Hv, d, d, device=device)
    state = torch.zeros((B, Hv, d, d), dtype=torch.float32, device=device)
    out = torch.empty((B * T, Hv, d), dtype=torch.bfloat16, device=device)
    stream = torch.cuda.current_stream(device)
    for _ in range(warmup):
        numerics.gdn_chunk_prefill(q, k, v, decay, beta, state, T=T, out=out)
    times = []
    for _ in range(steps):
        state.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        numerics.gdn_chunk_prefill(q, k, v, decay, beta, state, T=T, out=out)
        e1.record(stream)
        times.append((e0, e1))
    torch.cuda.synchronize()
    ms = statistics.median(a.elapsed_time(b) for a, b in times)
    per_chunk = 3 * (2 * 2 * C * C * d) + 3 * 2 * C * d * d + 2 * C ** 3 / 3
    flops = per_chunk * B * Hv * (T // C)
    nbytes = (2 * B * T * Hk * d * 2 + 2 * B * T * Hv * d * 2 + 2 * B * T * Hv * 4
              + 2 * B * Hv * d * d * 4)
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (
        ROOT / "MEASURED_PEAKS.json").exists() else {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0}
    tflops = flops / (ms / 1e3) / 1e12
    gbs = nbytes / (ms / 1e3) / 1e9
    return {"workload": "config1 chunked GDN prefill B=8 T=4096 Hk16/Hv32 128x128 fp32 state",
            "ms": round(ms, 3), "tokens_per_s": round(B * T / (ms / 1e3), 1),
            "algorithmic_gflop": round(flops / 1e9, 1), "tflops": round(tflops, 1),
            "tensor_peak_tflops": peaks["bf16_tflops"],
            "tensor_frac": round(tflops / peaks["bf16_tflops"], 4),
            "hbm_gbs": round(gbs, 1), "hbm_frac": round(gbs / peaks["hbm_gbs"], 4),
            "launches": steps}


def run_e2e(args, wl, world):
    """Same step through the public API with host buffers: every step stages its
    tables (host bookkeeping), copies every layer's inputs host->device from
    pinned memory and every output back, copies overlapped with compute on side
    streams; wall clock per step, summed over the steps. A layer's input copies
    are issued a few layers ahead of its kernels, interleaved with the launches,
    so the GPU starts on layer 0 while the host is still queueing copies."""
    import torch

    eng, cfg = wl.engine, wl.cfg
    comp = torch.cuda.current_stream(wl.device)
    h2d = torch.cuda.Stream(wl.device)
    d2h = torch.cuda.Stream(wl.device)
    host_in = {l: tuple(t.cpu().pin_memory() for t in wl.inputs[l]) for l in range(cfg.layers)}
    host_out = {l: torch.empty(wl.outputs[l].shape, dtype=wl.outputs[l].dtype).pin_memory()
                for l in range(cfg.layers)}
    bytes_in = sum(t.numel() * t.element_size() for ts in host_in.values() for t in ts)
    bytes_out = sum(t.numel() * t.element_size() for t in host_out.values())

    ahead = 3  # layers whose inputs are in flight before a layer's kernels are queued
    spans = []  # device time of each timed step's kernels (first layer to last)

    def step(span=None):
        ready = {}
        h2d.wait_stream(comp)  # the last step's kernels are done with the input buffers

        def copy_in(l):
            with torch.cuda.stream(h2d):
                for dst, src in zip(wl.inputs[l], host_in[l]):
                    dst.copy_(src, non_blocking=True)
                ready[l] = torch.cuda.Event()
                ready[l].record(h2d)

        # The first layers' inputs go out before the host stages the step's tables
        # (begin_step), so the copies run while the host does its bookkeeping.
        for l in range(min(ahead, cfg.layers)):
            copy_in(l)
        n = eng.begin_step()
        if span is not None:
            span[0].record(comp)
        for l in range(cfg.layers):
            if l + ahead < cfg.layers:
                copy_in(l + ahead)
            comp.wait_event(ready.pop(l))
            if cfg.is_attention(l):
                eng.attention_layer(l, *wl.inputs[l], wl.outputs[l])
            else:
                eng.gdn_layer(l, *wl.inputs[l], wl.outputs[l], chained=l > 0)
            done = torch.cuda.Event()
            done.record(comp)
            with torch.cuda.stream(d2h):
                d2h.wait_event(done)
                host_out[l].copy_(wl.outputs[l], non_blocking=True)
        if span is not None:
            span[1].record(comp)
        comp.wait_stream(d2h)
        return n

    def admit():
        # Churn and prefill of admitted prompts are reported separately; they
        # run before the timed part of each step.
        wl.prefill(wl.churn())
        torch.cuda.synchronize()

    for _ in range(2):
        admit()
        step()
    torch.cuda.synchronize()
    barrier(world)
    tokens, elapsed = 0, 0.0
    for _ in range(args.steps):
        admit()
        span = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        t0 = time.perf_counter()
        tokens += step(span)
        torch.cuda.synchronize()
        elapsed += time.perf_counter() - t0
        spans.append(span)
    elapsed = max_over_ranks(elapsed, world)
    tokens = sum_over_ranks(tokens, world)
    return {"value": round(tokens / elapsed, 1), "unit": UNIT,
            "h2d_bytes_per_step": int(bytes_in), "d2h_bytes_per_step": int(bytes_out),
            "ms_per_step": round(elapsed * 1e3 / args.steps, 3),
            # The kernels of the same steps alone (their batches are the run's first,
            # longest ones): the rest of ms_per_step is host work and copies.
            "device_ms_per_step": round(sum(a.elapsed_time(b) for a, b in spans) / len(spans), 3)
            if spans else None}


def cpu_baseline(args, wl):
    """The oracle step on the host cores for a bounded sample of the same sequences."""
    from oracle import cpu_step

    cfg = wl.cfg
    threads = cpu_step.host_threads()
    active = np.flatnonzero(wl.engine.blocks.active)
    sample = args.cpu_sample or min(len(active), 32, max(4, threads))
    picked = np.random.default_rng(SEED).choice(active, size=sample, replace=False)
    lengths = wl.engine.blocks.lengths[picked]
    rng = np.random.default_rng(SEED)
    seqs = [cpu_step.SampledSequence(rng, int(L), len(cfg.gdn_layers), len(cfg.attention_layers),
                                     cfg.gdn_key_heads, cfg.gdn_value_heads, cfg.key_dim,
                                     cfg.value_dim, cfg.q_heads, cfg.kv_heads, cfg.head_dim, 8)
            for L in lengths]
    layers = [cfg.is_attention(l) for l in range(cfg.layers)]
    elapsed = cpu_step.run_sample(seqs, layers, 1.0 / math.sqrt(cfg.head_dim), threads, SEED)
    return {"value": round(len(seqs) / elapsed, 2), "unit": UNIT, "cores": threads,
            "kind": "port",
            "sample": f"{len(seqs)} of the step's sequences, drawn at random (mean ctx "
                      f"{int(np.mean(lengths))}) x {cfg.layers} layers, one decode token each, "
                      f"float64/fp32 NumPy oracle, {threads} threads"}


def config4_measure(args, world, rank, local, steps: int, warmup: int,
                    exchange: str = "p2p") -> dict | None:
    """Config 4: one sequence of --ctx4 tokens; its KV pages are split evenly across the
    ranks (contiguous ranges), the GDN state (32 heads) is updated on every rank, and each
    attention layer sends the per-rank (out, lse) partial to every rank: NVLink peer
    stores with epoch flags (exchange p2p or fused) or an NCCL all-gather (nccl).
    Every rank calls it; returns the measurement on rank 0, else None."""
    import torch
    import torch.distributed as dist

    from shellsmith_b200 import _build, _capi, numerics
    from shellsmith_b200.longctx import ShardedSequence
    from shellsmith_b200.workloads import gdn_token_inputs_device

    _build.build()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    L, n_attn = 48, 12
    hq, hkv, d = 16, 2, 256
    # Page headroom on the tail rank for every token this run appends (the
    # warm-up, the captured pass, the first replay and the timed steps).
    headroom = -(-(warmup + steps + 4) // 16) + 1
    shard = ShardedSequence(args.ctx4, rank, world, attention_layers=n_attn, kv_heads=hkv,
                            head_dim=d, q_heads=hq, headroom_pages=headroom, device=device)
    use_p2p = world > 1 and exchange != "nccl"
    if use_p2p:
        shard.enable_peer_exchange(fused=exchange == "fused")
    gen = torch.Generator(device=device)
    gen.manual_seed(4)
    block = torch.randn(1 << 26, generator=gen, device=device).to(torch.bfloat16)
    flat = shard.kv.view(-1)
    for start in range(0, flat.numel(), block.numel()):
        part = flat[start:start + block.numel()]
        part.copy_(block[:part.numel()])
    del block
    state = torch.zeros((36, 1, 32, 128, 128), dtype=torch.float32, device=device)
    gdn_in = [gdn_token_inputs_device(gen, 1, 16, 32, 128, 128, device=device) for _ in range(36)]
    gdn_out = torch.empty((1, 32, 128), dtype=torch.bfloat16, device=device)
    attn_in = [(torch.randn((1, hq, d), generator=gen, device=device).to(torch.bfloat16),
                torch.randn((1, hkv, d), generator=gen, device=device).to(torch.bfloat16),
                torch.randn((1, hkv, d), generator=gen, device=device).to(torch.bfloat16))
               for _ in range(n_attn)]
    stream = torch.cuda.current_stream(device)

    def layers():
        g_i = a_i = 0
        for layer in range(L):
            if layer % 4 == 3:
                q, k, v = attn_in[a_i]
                shard.attention(a_i, q, k, v, 1 / 16)
                a_i += 1
            else:
                # Each layer has its own state: the update may stream it in early.
                numerics.gdn_decode(*gdn_in[g_i], state[g_i], out=gdn_out, chained=True)
                g_i += 1

    for _ in range(warmup):
        shard.begin_token()
        layers()
    torch.cuda.synchronize()
    # The step is launch-bound (~100 small kernels for ~0.5 ms of HBM time at
    # 1 GPU): capture the 48 layers, all-gathers included, in one CUDA graph.
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        layers()
    torch.cuda.synchronize()

    def step():
        shard.begin_token()
        graph.replay()

    step()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    local_ms = e0.elapsed_time(e1)
    ms = max_over_ranks(local_ms, world)
    parity = config4_parity(shard, attn_in[0], world, rank)
    # The exchange alone: one layer's packed partial to every rank. It runs last: its
    # epochs lie above every layer epoch this run still had to use.
    ag_ms = None
    if use_p2p:
        for i in range(5):
            shard.peer.put_and_wait(shard.packed, shard.epoch, 1 << 20 | i, i & 1)
        torch.cuda.synchronize()
        barrier(world)
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for i in range(50):
            shard.peer.put_and_wait(shard.packed, shard.epoch, (1 << 20) + 8 + i, i & 1)
        a1.record(stream)
        torch.cuda.synchronize()
        ag_ms = max_over_ranks(a0.elapsed_time(a1) / 50, world)
    elif world > 1:
        for _ in range(5):
            dist.all_gather_into_tensor(shard.gathered, shard.packed)
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for _ in range(50):
            dist.all_gather_into_tensor(shard.gathered, shard.packed)
        a1.record(stream)
        torch.cuda.synchronize()
        ag_ms = max_over_ranks(a0.elapsed_time(a1) / 50, world)
    _capi.check_device()
    del graph  # release the graph (it holds NCCL work) before the process group goes
    barrier(world)
    shard.close()
    bytes_rank = n_attn * (shard.local_tokens * hkv * d * 2 * 2) + 36 * 4210944
    bytes_all = sum_over_ranks(float(bytes_rank), world)
    del shard, state
    if rank != 0:
        return None
    peaks = measured_peaks()
    per_step = ms / 1e3 / steps
    # Compact: this record closes the bench line. exchange_us is one layer's partial to
    # every rank timed alone (the put/wait kernel pair for p2p and fused, the all-gather
    # for nccl); the step is one CUDA graph replay.
    return {
        "n_gpus": world, "steps": steps,
        "ms_per_step": round(per_step * 1e3, 4), "tokens_per_s": round(1 / per_step, 1),
        "hbm_frac_per_gpu": round(bytes_all / world / per_step / 1e9 / peaks["hbm_gbs"], 4),
        "exchange": exchange if world > 1 else None,
        "exchange_us": None if ag_ms is None else round(ag_ms * 1e3, 2),
        "parity": parity,
    }


def config4_parity(shard, attn_in, world: int, rank: int) -> str:
    """One more token through attention layer 0 on the measured path (untimed). At
    N > 1 the same per-rank partials through an NCCL all-gather and the packed merge
    must give the same bits; on every N, query heads 0, 9 and 15 must match float64
    attention over the whole context (each rank's float64 partial over its own pages,
    merged on rank 0). Every rank calls it (its collectives run on all ranks)."""
    import torch
    import torch.distributed as dist

    from shellsmith_b200 import _capi, paged

    q, k, v = attn_in
    shard.begin_token()
    got = shard.attention(0, q, k, v, 1 / 16).clone()
    identical = True
    if world > 1:
        # The same partial again, by the kernel the measured path used (the fused layer
        # rewrites the same appended rows), gathered by NCCL instead.
        plan = dict(max_pages_in_batch=shard.capacity, pages_per_split=shard.pages_per_split,
                    total_pages=shard.capacity, workspace=shard.workspace, packed=shard.packed)
        if shard.peer_fused or shard.num_splits > 1:
            paged.paged_decode_attention_packed(q, shard.kv[0], shard.table, shard.ctx, 1 / 16,
                                                **plan)
        else:
            paged.paged_decode_attention_fused(q, k, v, shard.slot, shard.kv[0], shard.table,
                                               shard.ctx, 1 / 16, **plan)
        dist.all_gather_into_tensor(shard.gathered, shard.packed)
        ref, _ = paged.attention_combine_packed(shard.gathered)
        torch.cuda.synchronize()
        identical = torch.equal(ref, got)
    torch.cuda.synchronize()
    _capi.check_device()
    heads = (0, 9, 15)
    group = shard.q_heads // shard.kv.shape[2]
    mine = [(torch.zeros((1, shard.head_dim), dtype=torch.float64),
             torch.full((1,), -math.inf, dtype=torch.float64))] * len(heads)
    if shard.local_tokens:
        kk, vv = pool_tokens(shard.kv[0], list(range(shard.capacity)), shard.local_tokens)
        mine = []
        for h in heads:
            o, l = partial_fp64(q[0, h:h + 1], kk[:, h // group], vv[:, h // group], 1 / 16)
            mine.append((o.cpu(), l.cpu()))
        del kk, vv
    parts = [mine]
    if world > 1:
        parts = [None] * world
        dist.all_gather_object(parts, mine)
        identical = bool(sum_over_ranks(float(not identical), world) == 0)
    if rank != 0:
        return ""
    ok = True
    for i, h in enumerate(heads):
        want, _ = merge_fp64([p[i] for p in parts])
        ok &= close(got[h:h + 1], want, ATTN_RTOL, ATTN_ATOL)
    if ok and identical:
        return "ok" + (" (exchange == nccl bit for bit)" if world > 1 else "")
    fails = ([] if ok else ["FAILED vs float64 (heads 0, 9, 15)"]) + (
        [] if identical else ["FAILED exchange != nccl"])
    return "; ".join(fails)


def run_config4(args, world, rank, local):
    """--config 4: the config-4 measurement as the run's own JSON line."""
    c4 = config4_measure(args, world, rank, local, args.steps, args.warmup, args.exchange)
    if c4 is None:
        return None
    line = {
        "metric": "config4 long-context decode tokens/sec (one 128k sequence, KV sharded)",
        "value": c4["tokens_per_s"], "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": c4["ms_per_step"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16 kv / fp32 gdn state", "data": "synthetic",
        "config": {"workload": f"config4: one sequence of {args.ctx4} tokens, 48 layers (36 GDN "
                               f"replicated + 12 attention with KV pages split over {world} "
                               f"GPU)",
                   "parallelism": f"KV-page sharding x{world}, exchange {c4['exchange']}",
                   "all_gather_bytes_per_rank": 16 * 257 * 4},
        "hbm_frac_per_gpu": c4["hbm_frac_per_gpu"], "exchange_us": c4["exchange_us"],
        "parity": c4["parity"],
    }
    print(json.dumps(line), flush=True)
    return line


def run_reference(args, world, rank):
    """--impl reference: the reference's CPU math (oracle port) on the host cores."""
    if rank != 0:
        return None
    from oracle import cpu_step

    rng = np.random.default_rng(SEED)
    threads = cpu_step.host_threads()
    sample = args.cpu_sample or min(32, max(4, threads))
    lengths = rng.integers(args.min_len, args.max_len + 1, size=sample)
    layers = [l % 4 == 3 for l in range(48)]
    seqs = [cpu_step.SampledSequence(rng, int(L), 36, 12, 16, 32, 128, 128, 16, 2, 256,
                                     args.steps + args.warmup + 1) for L in lengths]
    for i in range(args.warmup):
        cpu_step.run_sample(seqs, layers, 1.0 / 16.0, threads, SEED + i)
    elapsed = 0.0
    for i in range(args.steps):
        elapsed += cpu_step.run_sample(seqs, layers, 1.0 / 16.0, threads, SEED + 100 + i)
    value = len(seqs) * args.steps / elapsed
    desc = (f"{len(seqs)} sequences (ctx U[{args.min_len},{args.max_len}]) x 48 layers per step, "
            f"float64/fp32 NumPy oracle port, {threads} threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(elapsed * 1e3 / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64/f32", "data": "synthetic",
        "config": {"workload": "config3 hybrid decode cache step (CPU oracle sample)",
                   "global_batch": len(seqs), "seq_len": f"U[{args.min_len},{args.max_len}]",
                   "parallelism": "host threads"},
        "cpu_baseline": {"value": round(value, 2), "unit": UNIT, "cores": threads,
                         "kind": "port", "sample": desc},
        "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return line


def main():
    args = parse()
    world, rank, local = dist_setup(args) if args.impl == "ours" else (
        int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        elif args.prefill_only:
            import torch

            print(json.dumps(config1_prefill(torch.device("cuda", local))), flush=True)
        elif args.kv8_only:
            import torch

            print(json.dumps(kv8_layer_standalone(args, torch.device("cuda", local))),
                  flush=True)
        elif args.front_only:
            import torch

            print(json.dumps(gdn_front_layer(torch.device("cuda", local), batch=args.batch)),
                  flush=True)
        elif args.config == 4:
            run_config4(args, world, rank, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        if args.impl == "ours" and world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
