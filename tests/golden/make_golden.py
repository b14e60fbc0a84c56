"""Generate the golden fixtures in this folder from the reference's own code.

Run where the shellsmith source tree is available (it is not needed to run
the tests):
    python tests/golden/make_golden.py --reference <path to shellsmith>

It executes, without copying, these reference functions and classes:
  tests/test_gdn_sequential.py `sequential`  -- the float64 GDN oracle. The
      module imports MLX at its top, so only the function's own AST is
      compiled, with numpy as its one global.
  scripts/mlx_attention_qualify.py `numpy_attention` -- causal GQA oracle.
  src/studio_compute/mlx_racing.py `ContinuousBatcher` -- the scheduler.
  src/studio_compute/cache.py `PrefixCache` -- the prefix snapshot pool.
  src/studio_compute/inference.py `create_request`, `release_request` -- the
      admission, deferral, failure and release rules of a request.
Inputs are seeded NumPy draws (the reference tests draw with mx.random,
whose bits are not reproducible without MLX), rounded to bf16 where the
reference feeds bf16. Outputs are written as .npz / .json next to this file.
"""

from __future__ import annotations

import argparse
import ast
import importlib.util
import json
import sys
from collections import OrderedDict
from pathlib import Path
from types import SimpleNamespace

import numpy as np

HERE = Path(__file__).resolve().parent


def bf16(x):
    x = np.ascontiguousarray(np.asarray(x, np.float32))
    bits = x.view(np.uint32).astype(np.uint64)
    bits = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
    return bits.astype(np.uint32).view(np.float32).reshape(x.shape)


def load_sequential(ref: Path):
    tree = ast.parse((ref / "tests/test_gdn_sequential.py").read_text())
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "sequential")
    module = ast.Module(body=[fn], type_ignores=[])
    scope = {"np": np}
    exec(compile(module, "test_gdn_sequential.py", "exec"), scope)
    return scope["sequential"]


def load_numpy_attention(ref: Path):
    sys.path.insert(0, str(ref / "scripts"))
    spec = importlib.util.spec_from_file_location(
        "attention_qualify", ref / "scripts/mlx_attention_qualify.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module.numpy_attention


# ---------------------------------------------------------------- GDN
def gdn_cases(rng):
    """(name, q, k, v, g, beta, initial) in float64, values bf16-representable."""
    cases = []
    for length in (17, 70, 193):
        for unit in (False, True):
            q = bf16(rng.standard_normal((1, length, 1, 64)) * 0.02)
            k = bf16(rng.standard_normal((1, length, 1, 64)) * 0.08)
            v = bf16(rng.standard_normal((1, length, 2, 16)) * 0.1)
            g = bf16(rng.uniform(0.96, 0.995, (1, length, 2)))
            if unit:
                g = np.ones_like(g)
            beta = bf16(rng.uniform(0.1, 0.6, (1, length, 2)))
            s0 = bf16(rng.standard_normal((1, 2, 16, 64)) * 0.02)
            cases.append((f"ref_test_L{length}_{'unit' if unit else 'gated'}",
                          q, k, v, g, beta, s0))
    # Config-0 distributions (L2-normalised q/k, sigmoid beta, exp(-softplus) decay).
    def l2(x):
        return x / np.linalg.norm(x, axis=-1, keepdims=True)

    B, T, Hk, Hv, d = 1, 24, 2, 4, 128
    q = bf16(l2(rng.standard_normal((B, T, Hk, d))))
    k = bf16(l2(rng.standard_normal((B, T, Hk, d))))
    v = bf16(rng.standard_normal((B, T, Hv, d)))
    g = np.exp(-np.logaddexp(0.0, rng.standard_normal((B, T, Hv)))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((B, T, Hv))))).astype(np.float32)
    cases.append(("config0_dist_gqa", q, k, v, g, beta, np.zeros((B, Hv, d, d), np.float32)))
    # Token-test shapes: 6 value / 2 key heads, dk 32, dv 16, nonzero state.
    q = bf16(rng.standard_normal((2, 8, 2, 32)) * 0.05)
    k = bf16(rng.standard_normal((2, 8, 2, 32)) * 0.08)
    v = bf16(rng.standard_normal((2, 8, 6, 16)) * 0.1)
    g = np.full((2, 8, 6), 0.984375, np.float32)
    beta = np.full((2, 8, 6), 0.5, np.float32)
    s0 = bf16(rng.standard_normal((2, 6, 16, 32)) * 0.02)
    cases.append(("token_test_gqa3", q, k, v, g, beta, s0))
    return cases


def make_gdn(ref: Path):
    sequential = load_sequential(ref)
    rng = np.random.default_rng(7)
    out = {}
    for name, q, k, v, g, beta, s0 in gdn_cases(rng):
        inputs = [np.asarray(x, np.float64) for x in (q, k, v, g, beta, s0)]
        cot = [np.zeros_like(inputs[2]), np.zeros_like(inputs[5])]
        (y, state), _ = sequential(inputs, cot)
        for key, value in zip(("q", "k", "v", "g", "beta", "s0"), (q, k, v, g, beta, s0)):
            out[f"{name}/{key}"] = np.asarray(value, np.float32)
        out[f"{name}/y"] = y
        out[f"{name}/state"] = state
    np.savez_compressed(HERE / "gdn_sequential.npz", **out)
    return sorted({k.split("/")[0] for k in out})


# ---------------------------------------------------------------- attention
def make_attention(ref: Path):
    numpy_attention = load_numpy_attention(ref)
    rng = np.random.default_rng(19)
    out = {}
    cases = [(1, 1, 0), (1, 17, 16), (8, 41, 33), (17, 41, 24), (194, 194, 0), (33, 47, 7)]
    for queries, keys, offset in cases:
        name = f"q{queries}_k{keys}_o{offset}"
        q = bf16(rng.standard_normal((1, 4, queries, 64)))
        k = bf16(rng.standard_normal((1, 2, keys, 64)))
        v = bf16(rng.standard_normal((1, 2, keys, 64)))
        y = numpy_attention(q, k, v, np.zeros_like(q), scale=0.125, query_offset=offset)[0]
        out.update({f"{name}/q": q, f"{name}/k": k, f"{name}/v": v, f"{name}/y": y,
                    f"{name}/meta": np.array([queries, keys, offset, 0.125])})
    for keys in (1, 17, 300):  # decode: one query at the last position, 16/2 heads, D 256
        name = f"decode_k{keys}"
        q = bf16(rng.standard_normal((1, 16, 1, 256)))
        k = bf16(rng.standard_normal((1, 2, keys, 256)))
        v = bf16(rng.standard_normal((1, 2, keys, 256)))
        y = numpy_attention(q, k, v, np.zeros_like(q), scale=1 / 16)[0]
        out.update({f"{name}/q": q, f"{name}/k": k, f"{name}/v": v, f"{name}/y": y,
                    f"{name}/meta": np.array([1, keys, keys - 1, 1 / 16])})
    # The reference's known answer (tests/test_attention_oracle.py:44-57).
    q = np.zeros((1, 2, 2, 1))
    k = np.zeros((1, 1, 3, 1))
    v = np.array([[[[1.0], [3.0], [8.0]]]])
    y = numpy_attention(q, k, v, np.ones_like(q), scale=1.0)[0]
    out.update({"known/q": q, "known/k": k, "known/v": v, "known/y": y,
                "known/meta": np.array([2, 3, 1, 1.0])})
    np.savez_compressed(HERE / "attention.npz", **out)
    return sorted({k.split("/")[0] for k in out})


# ---------------------------------------------------------------- scheduler
def scheduler_harness(ContinuousBatcher, concurrency, memory_slots=None, churn_rng=None):
    """Stub callbacks in the manner of the reference scheduler tests: every
    callback appends to one event trace, and the batcher's records are kept."""
    events, released, completed, failed, live = [], [], {}, {}, set()

    def create(request_id, body):
        if body.get("invalid"):
            raise ValueError("invalid request")
        if memory_slots is not None and len(live) >= memory_slots:
            events.append(("defer", request_id))
            return None
        live.add(request_id)
        events.append(("admit", request_id))
        return SimpleNamespace(request_id=request_id, body=body, tokens=[], offset=0,
                               logits=None, needs_decode=False, reason=None)

    def prefill(request):
        step = request.body.get("chunk", 2)
        request.offset += min(step, request.body["prompt_length"] - request.offset)
        events.append(("prefill", request.request_id, request.offset))
        if request.offset == request.body["prompt_length"]:
            request.logits = True

    def advance(requests):
        events.append(("advance", [r.request_id for r in requests]))
        for r in requests:
            r.needs_decode = False

    def sample(requests):
        events.append(("sample", [r.request_id for r in requests]))
        for r in requests:
            if r.body.get("fail"):
                raise RuntimeError("kernel failed")
            r.tokens.append(len(r.tokens))
            done = len(r.tokens) == r.body["maximum"]
            if churn_rng is not None and not done:
                done = churn_rng.random() < r.body.get("finish_p", 0.0)
            r.reason = "length" if done else None
            r.needs_decode = r.reason is None

    def release(request):
        live.discard(request.request_id)
        released.append(request.request_id)
        events.append(("release", request.request_id))

    batcher = ContinuousBatcher(
        concurrency, create=create, prefill=prefill, advance=advance, sample=sample,
        finish=lambda r: (completed.__setitem__(r.request_id, list(r.tokens)),
                          events.append(("finish", r.request_id))),
        fail=lambda name, error: (failed.__setitem__(name, str(error)),
                                  events.append(("fail", name, str(error)))),
        release=release)
    return batcher, events, released, completed, failed


def run_scenario(ContinuousBatcher, scenario):
    """Scenario = dict(concurrency, memory_slots, seed, script=[(op, ...)])."""
    churn = np.random.default_rng(scenario["seed"]) if scenario.get("churn") else None
    batcher, events, released, completed, failed = scheduler_harness(
        ContinuousBatcher, scenario["concurrency"], scenario.get("memory_slots"), churn)
    records = []
    for op in scenario["script"]:
        if op[0] == "enqueue":
            batcher.enqueue(op[1], op[2])
        elif op[0] == "cancel":
            batcher.cancel(op[1])
        elif op[0] == "step":
            for _ in range(op[1]):
                records.append(batcher.step())
        elif op[0] == "drain":
            guard = 0
            while batcher.pending or batcher.active:
                records.append(batcher.step())
                guard += 1
                assert guard < 5000
        elif op[0] == "close":
            batcher.close()
    return {"records": records, "events": [list(e) for e in events], "released": released,
            "completed": completed, "failed": failed,
            "active": sorted(batcher.active), "pending": [p[0] for p in batcher.pending]}


def scheduler_scenarios():
    def body(length=2, maximum=8, policy="p", **extra):
        return {"policy": policy, "prompt_length": length, "maximum": maximum, **extra}

    scenarios = {}
    for c in (1, 2, 3, 5, 8):
        script = [("enqueue", str(i), body(length=1 + i % 7, maximum=1 + i % 9))
                  for i in range(20)] + [("drain",)]
        scenarios[f"mixed_lengths_c{c}"] = {"concurrency": c, "script": script}
    scenarios["live_arrival"] = {"concurrency": 2, "script": [
        ("enqueue", "long", body(maximum=10)), ("enqueue", "short", body(maximum=1)),
        ("step", 2), ("enqueue", "new", body(maximum=2)), ("step", 1), ("close",)]}
    scenarios["deferral_cancel_failure"] = {"concurrency": 7, "memory_slots": 2, "script": [
        ("enqueue", "bad", body(invalid=True)), ("enqueue", "a", body(maximum=2)),
        ("enqueue", "b", body(length=5)), ("enqueue", "c", body(policy="other", fail=True)),
        ("enqueue", "queued-cancel", body()), ("step", 1), ("cancel", "queued-cancel"),
        ("cancel", "b"), ("drain",)]}
    scenarios["policy_groups"] = {"concurrency": 6, "script": [
        ("enqueue", "a", body(policy="p")), ("enqueue", "b", body(policy="other")),
        ("enqueue", "c", body(policy="p")), ("step", 5), ("close",)]}
    # Continuous churn: 64 slots, 300 requests with ragged prompts and
    # Bernoulli(0.02) finishing, prompts prefilled in 2048-token chunks.
    rng = np.random.default_rng(3)
    script = []
    for i in range(300):
        script.append(("enqueue", f"r{i}", body(length=int(rng.integers(256, 4097)),
                                                maximum=int(rng.integers(8, 200)),
                                                chunk=2048, finish_p=0.02)))
    script.append(("drain",))
    scenarios["churn_c64"] = {"concurrency": 64, "seed": 3, "churn": True, "script": script}
    return scenarios


def make_scheduler(ref: Path):
    sys.path.insert(0, str(ref / "src"))
    from studio_compute.mlx_racing import ContinuousBatcher

    scenarios = scheduler_scenarios()
    result = {}
    for name, scenario in scenarios.items():
        result[name] = {"scenario": scenario, "trace": run_scenario(ContinuousBatcher, scenario)}
    (HERE / "scheduler_traces.json").write_text(json.dumps(result, separators=(",", ":")))
    return list(result)


# ---------------------------------------------------------------- prefix cache
class FakeArray:
    def __init__(self, size):
        self.nbytes = size


def prefix_script(seed, n_ops=400):
    rng = np.random.default_rng(seed)
    ops = []
    vocab = 6
    for _ in range(n_ops):
        kind = rng.choice(["put", "get", "get_fork", "contains", "trim"], p=[.35, .3, .1, .15, .1])
        identity = ["m", "m2"][int(rng.random() < 0.1)]
        policy = ["p", "q"][int(rng.random() < 0.2)]
        precision = ["bf16", "8bit"][int(rng.random() < 0.15)]
        tokens = [int(t) for t in rng.integers(0, vocab, size=int(rng.integers(1, 7)))]
        if kind == "put":
            ops.append(["put", identity, policy, precision, tokens,
                        int(rng.integers(1, 40)), int(rng.integers(0, 5))])
        elif kind in ("get", "get_fork", "contains"):
            ops.append([kind, identity, policy, precision, tokens])
        else:
            ops.append(["trim", int(rng.integers(0, 150))])
    return ops


def run_prefix(PrefixCache, limit, capacity_mode, ops):
    mx = SimpleNamespace(array=FakeArray, stop_gradient=lambda x: x, eval=lambda *a: None)
    state = {"spare": 120}
    capacity = None
    if capacity_mode == "spare":
        capacity = lambda size: state["spare"] - size  # noqa: E731
    cache = PrefixCache(mx, limit, capacity=capacity)
    cache._copy = lambda c: list(c)
    outcomes = []
    for op in ops:
        if op[0] == "put":
            _, ident, pol, prec, tokens, size, logits = op
            cache.put(ident, pol, prec, tokens, [SimpleNamespace(state=[FakeArray(size)])],
                      FakeArray(logits))
            outcomes.append(None)
        elif op[0] == "get":
            hit = cache.get(*op[1:5])
            outcomes.append(None if hit is None else hit[2])
        elif op[0] == "get_fork":
            # fork=True only changes how the snapshot is copied (MLX arrays);
            # the bookkeeping is that of get(), so the fixture uses get().
            hit = cache.get(*op[1:5])
            outcomes.append(None if hit is None else hit[2])
        elif op[0] == "contains":
            outcomes.append(cache.contains(*op[1:5]))
        else:
            cache.trim(op[1])
            outcomes.append(None)
        outcomes[-1] = {"result": outcomes[-1], "metrics": cache.metrics(),
                        "keys": [[k[0], k[1], k[2], list(k[3])] for k in cache.entries]}
    return outcomes


def make_prefix(ref: Path):
    sys.path.insert(0, str(ref / "src"))
    from studio_compute.cache import PrefixCache

    result = {}
    for seed, limit, mode in ((1, 100, None), (2, 60, None), (3, 100, "spare"), (4, 0, None),
                              (5, 1000, None)):
        ops = prefix_script(seed)
        result[f"seed{seed}_limit{limit}_{mode}"] = {
            "limit": limit, "capacity": mode, "ops": ops,
            "outcomes": run_prefix(PrefixCache, limit, mode, ops)}
    (HERE / "prefix_cache_traces.json").write_text(json.dumps(result, separators=(",", ":")))
    return list(result)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    args = ap.parse_args()
    ref = args.reference.resolve()
    print("gdn:", make_gdn(ref))
    print("attention:", make_attention(ref))
    print("scheduler:", make_scheduler(ref))
    print("prefix:", make_prefix(ref))
    print("lifecycle:", make_lifecycle(ref))
    print("admission:", make_admission(ref))



# ---------------------------------------------------------------- request lifecycle
class _Lease:
    def __init__(self, log, name, fail):
        self.log, self.name, self.fail = log, name, fail

    def __enter__(self):
        if self.fail:
            raise MemoryError("policy reload does not fit")
        self.log.append(("enter", self.name))
        return {"factors": self.name}

    def __exit__(self, *exc):
        self.log.append(("exit", self.name))
        return False


def lifecycle_engine(spec, log):
    """A fake engine with the attributes inference.create_request reads."""
    state = {"persistent": spec["persistent"]}
    prefix_hit = spec.get("prefix_hit")

    def estimate(length, batch=1, **options):
        return spec["per_token"] * length * batch + spec["base"]

    def admit(needed):
        log.append(("admit", needed))
        if needed > spec["admit_limit"]:
            raise MemoryError("live memory pressure")

    def get(identity, policy, precision, tokens, fork=False):
        log.append(("prefix_get", identity, policy, precision, len(tokens), fork))
        if spec.get("prefix_error"):
            raise ValueError("corrupt cache")
        if prefix_hit is None or prefix_hit > len(tokens):
            return None
        return (["snapshot"], "logits", prefix_hit)

    mx = SimpleNamespace(uint32="uint32", array=lambda v, t: ("key", tuple(v)),
                         random=SimpleNamespace(key=lambda seed: ("seed", seed)))
    return SimpleNamespace(
        resident=SimpleNamespace(estimate_inference=estimate),
        prefixes=SimpleNamespace(limit=spec["prefix_limit"], bytes=spec["prefix_bytes"], get=get),
        policies=dict.fromkeys(spec["policies"], {}),
        idle_factors={"a": SimpleNamespace(nbytes=spec["idle_bytes"])},
        reserved=dict(spec["reserved"]),
        persistent_bytes=lambda: state["persistent"],
        admission_budget_bytes=lambda: spec["budget"],
        admit=admit,
        _borrow_policy=lambda ref: _Lease(log, ref, spec.get("lease_fail", False)),
        prefix_identity="ident",
        lm=SimpleNamespace(make_cache=lambda: ["fresh"]),
        mx=mx,
    )


def lifecycle_scenarios(n=160, seed=8):
    rng = np.random.default_rng(seed)
    out = []
    for i in range(n):
        prompt = int(rng.integers(1, 60))
        body = {"policy": ["p", "q"][int(rng.integers(0, 2))],
                "prompt_token_ids": [int(t) for t in rng.integers(0, 9, size=prompt)],
                "max_tokens": int(rng.integers(1, 40))}
        if rng.random() < 0.3:
            body["target_token_ids"] = [1] * int(rng.integers(1, 10))
        if rng.random() < 0.3:
            body["use_prefix_cache"] = bool(rng.integers(0, 2))
        if rng.random() < 0.2:
            body["cache_precision"] = "8bit"
        if rng.random() < 0.5:
            body["rng_key"] = [int(rng.integers(0, 99)), 1]
        else:
            body["seed"] = int(rng.integers(0, 99))
        spec = {
            "per_token": int(rng.integers(1, 4)), "base": int(rng.integers(0, 20)),
            "persistent": int(rng.integers(20, 120)), "budget": int(rng.integers(80, 260)),
            "admit_limit": int(rng.integers(0, 200)), "prefix_limit": int(rng.integers(0, 80)),
            "prefix_bytes": int(rng.integers(0, 20)), "idle_bytes": int(rng.integers(0, 30)),
            "policies": ["p"] if rng.random() < 0.6 else [],
            "reserved": {"replay": int(rng.integers(1, 80))} if rng.random() < 0.5 else {},
            "lease_fail": bool(rng.random() < 0.1),
            "prefix_error": bool(rng.random() < 0.05),
            "prefix_hit": (int(rng.integers(0, prompt + 1)) if rng.random() < 0.5 else None),
        }
        out.append({"id": f"r{i}", "body": body, "spec": spec})
    return out


def run_lifecycle(create_request, release_request, scenario):
    log = []
    engine = lifecycle_engine(scenario["spec"], log)
    try:
        request = create_request(engine, scenario["id"], scenario["body"])
    except Exception as error:  # noqa: BLE001 -- recorded as the outcome
        return {"outcome": f"{type(error).__name__}: {error}", "log": log,
                "reserved": engine.reserved}
    if request is None:
        return {"outcome": "defer", "log": log, "reserved": engine.reserved}
    record = {"outcome": "request", "offset": request.offset,
              "cached_tokens": request.cached_tokens, "has_logits": request.logits is not None,
              "cache": list(request.cache), "rng": list(request.rng)}
    release_request(engine, request)
    return {**record, "log": log, "reserved": engine.reserved}


def make_lifecycle(ref: Path):
    sys.path.insert(0, str(ref / "src"))
    from studio_compute.inference import create_request, release_request

    result = []
    for scenario in lifecycle_scenarios():
        result.append({"scenario": scenario,
                       "trace": run_lifecycle(create_request, release_request, scenario)})
    (HERE / "lifecycle_traces.json").write_text(
        json.dumps(result, separators=(",", ":"), default=list))
    return len(result)



# ---------------------------------------------------------------- byte admission
def load_methods(path: Path, cls: str, names, new_name: str, bases, scope: dict):
    """Compile chosen methods of a reference class into a new class (AST only, so
    the module's own imports -- MLX among them -- are never executed)."""
    tree = ast.parse(path.read_text())
    node = next(n for n in tree.body if isinstance(n, ast.ClassDef) and n.name == cls)
    body = [n for n in node.body if isinstance(n, ast.FunctionDef) and n.name in names]
    assert len(body) == len(names), (cls, names)
    new = ast.ClassDef(name=new_name, bases=[ast.Name(b, ast.Load()) for b in bases],
                       keywords=[], body=body, decorator_list=[], type_params=[])
    module = ast.fix_missing_locations(ast.Module(body=[new], type_ignores=[]))
    exec(compile(module, str(path), "exec"), scope)
    return scope[new_name]


def reference_admission_classes(ref: Path):
    src = ref / "src/studio_compute"
    scope = {"math": __import__("math")}
    resident = load_methods(src / "model.py", "Qwen27Model", ["estimate_inference", "admit"],
                            "Resident", [], scope)
    engine = load_methods(src / "engine.py", "ResidentEngine",
                          ["_evict_policy", "admission_budget_bytes", "admit"], "Engine", [],
                          scope)
    runtime = load_methods(src / "runtime.py", "RuntimeEngine",
                           ["_cache_capacity", "admit", "inference_batch_capacity"], "Runtime",
                           ["Engine"], scope)
    return resident, runtime


class AdmissionPrefixes:
    """Snapshot pool stand-in: bytes, limit, and trim() dropping the oldest first."""

    def __init__(self, limit, sizes, log):
        self.limit, self.sizes, self.log = limit, list(sizes), log

    @property
    def bytes(self):
        return sum(self.sizes)

    def trim(self, limit_bytes):
        self.log.append(["trim", limit_bytes])
        target = max(0, min(self.limit, limit_bytes))
        while self.bytes > target and self.sizes:
            self.sizes.pop(0)


def admission_engine(classes, spec, log):
    """A fake runtime engine with the attributes the admission methods read."""
    resident_cls, runtime_cls = classes
    engine = runtime_cls()
    every = spec["attention_every"]
    layers = [SimpleNamespace(
        is_linear=l % every != every - 1,
        self_attn=SimpleNamespace(num_key_value_heads=spec["kv_heads"],
                                  head_dim=spec["head_dim"]),
        linear_attn=SimpleNamespace(num_v_heads=spec["v_heads"], head_v_dim=spec["dv"],
                                    head_k_dim=spec["dk"])) for l in range(spec["layers"])]
    policies = OrderedDict((name, {"factors": SimpleNamespace(name=name, nbytes=size)})
                           for name, size, _ in spec["policies"])
    idle = SimpleNamespace(name="idle", nbytes=spec["idle_bytes"])

    def policy_bytes():
        return sum(p["factors"].nbytes for p in engine.policies.values())

    def active():
        return spec["base_active"] + policy_bytes() + engine.prefixes.bytes

    mx = SimpleNamespace(get_active_memory=active)
    resident = resident_cls()
    resident.lm = SimpleNamespace(layers=layers)
    resident.mx = mx
    resident.budget = spec["budget"]
    resident.selected = (policies[spec["selected"]]["factors"] if spec["selected"] else
                         {"idle": idle})
    resident.select = lambda factors: (log.append(["select", sorted(factors)]),
                                       setattr(resident, "selected", factors))
    resident.spec = spec
    engine.resident = resident
    engine.mx = mx
    engine.policies = policies
    engine.policy_users = {name: users for name, _, users in spec["policies"] if users}
    engine.idle_factors = {"idle": idle}
    engine.reserved = dict(spec["reserved"])
    engine.prefixes = AdmissionPrefixes(spec["prefix_limit"], spec["prefix_sizes"], log)
    engine.execution_profile = spec["profile"]
    engine.capabilities = ({"recommended_working_set_bytes": spec["recommended"]}
                           if spec["recommended"] is not None else {})
    engine.persistent_bytes = lambda: (spec["base_persistent"] + spec["idle_bytes"]
                                       + policy_bytes() + engine.prefixes.bytes)
    if spec["concurrency"] is not None:
        engine.inference_concurrency = spec["concurrency"]
    return engine


def admission_scenarios(n=60, seed=12):
    rng = np.random.default_rng(seed)
    gib = 1 << 30
    out = []
    for i in range(n):
        npol = int(rng.integers(0, 4))
        policies = [[f"p{j}", int(rng.integers(1, 6)) * gib // 4, int(rng.integers(0, 2))]
                    for j in range(npol)]
        spec = {
            "layers": int(rng.choice([8, 48, 64])), "attention_every": int(rng.choice([2, 4])),
            "kv_heads": int(rng.choice([2, 4])), "head_dim": int(rng.choice([128, 256])),
            "v_heads": int(rng.choice([16, 32, 48])), "dv": 128, "dk": 128,
            "base_active": int(rng.integers(10, 60)) * gib,
            "base_persistent": int(rng.integers(10, 60)) * gib,
            "idle_bytes": int(rng.integers(0, 3)) * gib // 2,
            "policies": policies,
            "selected": (policies[int(rng.integers(0, npol))][0]
                         if npol and rng.random() < 0.7 else None),
            "budget": int(rng.integers(60, 180)) * gib,
            "recommended": (int(rng.integers(50, 200)) * gib if rng.random() < 0.4 else None),
            "profile": ["bf16-fast", "legacy"][int(rng.random() < 0.3)],
            "reserved": ({"replay": int(rng.integers(1, 30)) * gib} if rng.random() < 0.5
                         else {}),
            "prefix_limit": int(rng.integers(0, 40)) * gib,
            "prefix_sizes": [int(x) * gib // 2 for x in rng.integers(1, 8, size=int(
                rng.integers(0, 6)))],
            "concurrency": int(rng.integers(1, 12)) if rng.random() < 0.7 else None,
        }
        ops = []
        for _ in range(14):
            kind = rng.choice(["estimate", "admit", "capacity", "batch", "reserve", "unreserve"],
                              p=[.2, .3, .15, .15, .1, .1])
            precision = ["bf16", "8bit", "fp8"][int(rng.choice(3, p=[.6, .3, .1]))]
            if kind == "estimate":
                ops.append(["estimate", int(rng.integers(0, 300_000)),
                            int(rng.integers(1, 9)), precision])
            elif kind == "admit":
                ops.append(["admit", int(rng.integers(0, 80)) * gib // 2])
            elif kind == "capacity":
                ops.append(["capacity", int(rng.integers(0, 20)) * gib // 2,
                            int(rng.integers(0, 20)) * gib // 2])
            elif kind == "batch":
                ops.append(["batch", int(rng.integers(1, 40_000)), int(rng.integers(1, 40_000)),
                            ["bf16", "8bit"][int(rng.random() < 0.3)], int(rng.integers(1, 16))])
            elif kind == "reserve":
                ops.append(["reserve", f"r{len(ops)}", int(rng.integers(1, 20)) * gib])
            else:
                ops.append(["unreserve"])
        out.append({"id": f"a{i}", "spec": spec, "ops": ops})
    return out


def run_admission(classes, scenario):
    log = []
    engine = admission_engine(classes, scenario["spec"], log)
    steps = []
    for op in scenario["ops"]:
        start = len(log)
        try:
            if op[0] == "estimate":
                result = engine.resident.estimate_inference(op[1], op[2], cache_precision=op[3])
            elif op[0] == "admit":
                result = engine.admit(op[1])
            elif op[0] == "capacity":
                result = engine._cache_capacity(op[1], additional=op[2])
            elif op[0] == "batch":
                body = {"prompt_token_ids": [0] * op[1], "max_tokens": op[2],
                        "cache_precision": op[3]}
                result = engine.inference_batch_capacity(body, op[4])
            elif op[0] == "reserve":
                engine.reserved[op[1]] = op[2]
                result = None
            else:
                result = engine.reserved.popitem()[0] if engine.reserved else None
        except Exception as error:  # noqa: BLE001 -- recorded as the outcome
            result = f"{type(error).__name__}: {error}"
        steps.append({"result": result, "log": log[start:], "policies": list(engine.policies),
                      "prefix_sizes": list(engine.prefixes.sizes),
                      "reserved": sorted(engine.reserved.items())})
    return steps


def make_admission(ref: Path):
    classes = reference_admission_classes(ref)
    result = [{"scenario": sc, "trace": run_admission(classes, sc)}
              for sc in admission_scenarios()]
    (HERE / "admission_traces.json").write_text(json.dumps(result, separators=(",", ":")))
    return len(result)


if __name__ == "__main__":
    main()
