"""Production MECO adapter: identity checks, asynchronous fail-closed
inference, request capture, fallback monitor, export and profiling."""
import hashlib

import pytest
import torch

from autodrive_b200.meco.adapter import (DiagnosticMonitor, ProductionMecoAdapter, capture_request, export_scorer,
                                         profile_latency)
from autodrive_b200.meco.tracks import DecisionRequest, choose_candidate, make_meco_track

SHA = hashlib.sha256(b"weights").hexdigest()
IDS = tuple(f"action-{k}" for k in range(8))


def _inputs():
    g = torch.Generator().manual_seed(0)
    return {"globals_": torch.rand(1, 7, generator=g), "candidate_features": torch.rand(1, 8, 16, generator=g)}


def test_identity_and_device_checks():
    model = make_meco_track("C1")
    with pytest.raises(ValueError):
        ProductionMecoAdapter("C1", model, checkpoint_sha256="abc", protocol_id="p")
    with pytest.raises(ValueError):
        ProductionMecoAdapter("Z9", model, checkpoint_sha256=SHA, protocol_id="p", allow_cpu=True)
    with pytest.raises(RuntimeError):
        ProductionMecoAdapter("C1", model, checkpoint_sha256=SHA, protocol_id="p")      # CPU model refused


def test_async_inference_feeds_the_arbiter():
    ad = ProductionMecoAdapter("C1", make_meco_track("C1"), checkpoint_sha256=SHA, protocol_id="p", allow_cpu=True)
    try:
        req = ad.next_request(IDS, 10., ("globals_", "candidate_features"))
        handle = ad.submit_inference(req, _inputs())
        out = ad.wait(req, handle, now=10.05)
        assert out is not None and out.candidate_ids == IDS and len(out.utility) == 8
        choice, why = choose_candidate(DecisionRequest(IDS, (True,) * 8, "action-7", 10.05), out)
        assert why == "scorer" and choice in IDS
        # stale: answered after the request's age limit
        req2 = ad.next_request(IDS, 11., ("globals_", "candidate_features"))
        h2 = ad.submit_inference(req2, _inputs())
        assert ad.wait(req2, h2, now=12.) is None
        # superseded by a reload
        req3 = ad.next_request(IDS, 13., ("globals_", "candidate_features"))
        h3 = ad.submit_inference(req3, _inputs())
        ad.reload(make_meco_track("C1"), SHA)
        assert ad.wait(req3, h3, now=13.) is None
        c = ad.inference_counters
        assert c["submitted"] == 3 and c["stale"] == 1 and c["superseded"] == 1
    finally:
        ad.close()


def test_faulting_or_invalid_scorer_fails_closed():
    class Broken(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.w = torch.nn.Parameter(torch.zeros(1))

        def forward(self, **_):
            return {"utility": torch.full((1, 8), float("nan")), "penalty": torch.zeros(1, 8)}

    ad = ProductionMecoAdapter("C1", Broken(), checkpoint_sha256=SHA, protocol_id="p", allow_cpu=True)
    try:
        req = ad.next_request(IDS, 1., ())
        assert ad.wait(req, ad.submit_inference(req, {}), now=1.) is None
        assert ad.inference_counters["invalid"] == 1
    finally:
        ad.close()


def test_request_capture_is_bounded(tmp_path):
    ad = ProductionMecoAdapter("C1", make_meco_track("C1"), checkpoint_sha256=SHA, protocol_id="p", allow_cpu=True)
    try:
        for k in range(3):
            req = ad.next_request(IDS, float(k), ("globals_", "candidate_features"))
            capture_request(req, _inputs(), directory=tmp_path, max_requests=2)
        assert len(list(tmp_path.glob("request-*.pt"))) == 2
        assert len((tmp_path / "manifest.jsonl").read_text().splitlines()) == 2
    finally:
        ad.close()


def test_monitor_alarm_and_export(tmp_path):
    mon = DiagnosticMonitor(window=64, max_fallback_rate=.25)
    for k in range(64):
        mon.record("scorer" if k % 2 else "stale-output")
    assert mon.alarm and abs(mon.fallback_rate - .5) < 1e-9
    model = make_meco_track("C1")
    rep = export_scorer(model, _inputs(), tmp_path / "c1.pt2")
    assert rep["format"] == "torch.export" and len(rep["sha256"]) == 64
    loaded = torch.export.load(str(tmp_path / "c1.pt2")).module()
    u, p = loaded(*_inputs().values())
    assert u.shape == (1, 8)
    prof = profile_latency(model, _inputs(), iters=5, warmup=1)
    assert prof["p50_ms"] > 0
