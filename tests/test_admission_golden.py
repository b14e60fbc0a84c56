"""Byte admission reproduces the reference's estimates and decisions exactly.

Fixtures: the reference methods (model.py estimate_inference/admit,
engine.py _evict_policy/admission_budget_bytes/admit, runtime.py
_cache_capacity/admit/inference_batch_capacity) run on seeded fake engines
(tests/golden/make_golden.py). The same scenarios run here through
shellsmith_b200.admission; every result, error text, snapshot trim target,
policy eviction and reservation table must be equal.
"""

import json
import sys
from pathlib import Path

import pytest

from shellsmith_b200 import admission
from shellsmith_b200.engine import HybridConfig

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import make_golden  # noqa: E402  (the fake engine the fixtures were recorded on)

TRACES = json.loads((GOLDEN / "admission_traces.json").read_text())


class Resident(admission.ResidentBudget):
    def __init__(self):  # attributes are set by the fake-engine builder
        pass

    @property
    def cfg(self):
        s = self.spec
        return HybridConfig(layers=s["layers"], attention_every=s["attention_every"],
                            kv_heads=s["kv_heads"], head_dim=s["head_dim"],
                            gdn_value_heads=s["v_heads"], value_dim=s["dv"], key_dim=s["dk"])


class Runtime(admission.AdmissionMixin):
    pass


def _normal(x):
    return json.loads(json.dumps(x))


def test_fixture_covers_rejections_evictions_and_errors():
    results = [st["result"] for t in TRACES for st in t["trace"]]
    assert any(isinstance(r, str) and r.startswith("MemoryError") for r in results)
    assert any(isinstance(r, str) and r.startswith("ValueError") for r in results)
    logs = [entry[0] for t in TRACES for st in t["trace"] for entry in st["log"]]
    assert "trim" in logs and "select" in logs


@pytest.mark.parametrize("case", range(len(TRACES)))
def test_admission_matches_reference(case):
    item = TRACES[case]
    got = make_golden.run_admission((Resident, Runtime), item["scenario"])
    assert _normal(got) == item["trace"]


def test_paged_bytes_against_estimate():
    """The paged footprint of a request never exceeds the reference's bound minus
    its 2 GiB headroom by more than one page per attention layer."""
    cfg = HybridConfig()
    for length in (1, 15, 16, 17, 1000, 16_384):
        est = admission.estimate_inference(cfg, length) - admission.HEADROOM
        paged = admission.paged_cache_bytes(cfg, length)
        page = cfg.kv_heads * 2 * cfg.page_size * cfg.head_dim * 2
        assert est <= paged <= est + page * len(cfg.attention_layers)
