"""Production MECO adapter: validated, asynchronous, fail-closed inference.

Parity with frc_defense/meco_tracks.py:236-520 (``ProductionMecoAdapter``,
``_AsyncInferenceBroker``), meco_request_capture.py (opt-in bounded request
capture), meco_diagnostic_monitor.py (fallback-rate monitor) and
meco_deployment.py (scorer export and latency profiling).

The adapter never decides by itself: it returns a ``ScorerOutput`` for a
request or ``None`` (not ready, stale, superseded, faulted or invalid), and
the caller keeps its deterministic, already-feasible fallback via
``choose_candidate``. Inference runs on a worker thread; on CUDA every job
gets its own stream and the worker (not the control loop) waits for it, so
the control loop never blocks on the scorer.
"""
from __future__ import annotations

import hashlib
import json
import os
import queue
import threading
import time
import uuid
from dataclasses import dataclass
from pathlib import Path
from typing import Mapping

import torch
from torch import nn

from .tracks import TRACKS, ScorerOutput


@dataclass(frozen=True)
class MecoInferenceRequest:
    sequence: int
    generation: str
    candidate_ids: tuple[str, ...]
    observation_time: float
    input_names: tuple[str, ...]
    max_age_s: float = .25


def _is_sha256(text: str) -> bool:
    return len(text) == 64 and all(c in "0123456789abcdef" for c in text)


class _AsyncInferenceBroker:
    """One worker thread; a job is (request, inputs). Results are kept per
    sequence number until polled."""

    def __init__(self, adapter: "ProductionMecoAdapter"):
        self.adapter = adapter
        self.jobs: queue.Queue = queue.Queue()
        self.results: dict[int, tuple[str, object]] = {}
        self.lock = threading.Lock()
        self.counts = {"submitted": 0, "completed": 0, "failed": 0, "invalid": 0, "stale": 0, "superseded": 0}
        self.thread = threading.Thread(target=self._run, name="meco-inference", daemon=True)
        self.thread.start()

    def _run(self):
        while True:
            job = self.jobs.get()
            if job is None:
                return
            request, inputs = job
            status, value = "failed", None
            try:
                value = self.adapter._infer(request, inputs)
                status = "ok" if value is not None else "invalid"
            except Exception as exc:              # a faulting scorer is a fallback, never a crash
                self.adapter.last_exception_type = type(exc).__name__
            with self.lock:
                self.results[request.sequence] = (status, value)
                self.counts["completed" if status == "ok" else status] += 1

    def submit(self, request, inputs):
        with self.lock:
            self.counts["submitted"] += 1
        self.jobs.put((request, inputs))
        return request.sequence

    def poll(self, request, handle, now: float | None = None):
        with self.lock:
            if handle not in self.results:
                return None
            status, value = self.results.pop(handle)
            if status != "ok":
                return None
            if request.generation != self.adapter.generation:
                self.counts["superseded"] += 1
                return None
            if now is not None and now - request.observation_time > request.max_age_s:
                self.counts["stale"] += 1
                return None
            return value

    def close(self):
        self.jobs.put(None)
        self.thread.join(timeout=10.)


class ProductionMecoAdapter:
    """Identity-checked scorer with asynchronous inference. The model must sit
    on one CUDA device unless ``allow_cpu`` (host testing)."""

    def __init__(self, track: str, model: nn.Module, *, checkpoint_sha256: str, protocol_id: str,
                 source_snapshot_sha256: str = "", allow_cpu: bool = False):
        if track not in TRACKS:
            raise ValueError(f"unsupported MECO track: {track}")
        if not _is_sha256(checkpoint_sha256) or not protocol_id:
            raise ValueError("production adapter requires checkpoint and protocol identity")
        params = tuple(model.parameters())
        if not params:
            raise RuntimeError("production MECO model has no parameters")
        devices = {p.device for p in params}
        if len(devices) != 1:
            raise RuntimeError("production MECO model spans several devices")
        self.device = next(iter(devices))
        if self.device.type != "cuda" and not allow_cpu:
            raise RuntimeError("production MECO adapter rejects CPU models")
        self.track, self.model = track, model.eval()
        self.checkpoint_sha256, self.protocol_id = checkpoint_sha256, protocol_id
        self.source_snapshot_sha256 = source_snapshot_sha256
        self.last_exception_type = None
        self._lock = threading.Lock()
        self._sequence = 0
        self.generation = uuid.uuid4().hex
        self._broker = _AsyncInferenceBroker(self)

    # -------------------------------------------------------------- requests
    def next_request(self, candidate_ids, observation_time: float, input_names, max_age_s: float = .25):
        with self._lock:
            self._sequence += 1
            seq = self._sequence
        return MecoInferenceRequest(seq, self.generation, tuple(candidate_ids), float(observation_time),
                                    tuple(input_names), float(max_age_s))

    def reload(self, model: nn.Module, checkpoint_sha256: str) -> None:
        """Swap the scorer; outstanding results of the old generation are dropped."""
        if not _is_sha256(checkpoint_sha256):
            raise ValueError("checkpoint identity must be a SHA-256 hex digest")
        with self._lock:
            self.model, self.checkpoint_sha256 = model.eval(), checkpoint_sha256
            self.generation = uuid.uuid4().hex

    def submit_inference(self, request: MecoInferenceRequest, inputs: Mapping[str, torch.Tensor]):
        if os.environ.get("MECO_REQUEST_CAPTURE_DIR"):
            try:
                capture_request(request, {k: inputs[k] for k in request.input_names if k in inputs},
                                source_snapshot_sha256=self.source_snapshot_sha256)
            except OSError:
                pass                                # capture never changes scoring
        return self._broker.submit(request, dict(inputs))

    def poll_inference(self, request: MecoInferenceRequest, handle, now: float | None = None):
        return self._broker.poll(request, handle, now)

    def wait(self, request, handle, timeout_s: float = 5., now: float | None = None):
        """Poll until a result or `timeout_s` (tests and offline evaluation)."""
        end = time.monotonic() + timeout_s
        while time.monotonic() < end:
            with self._broker.lock:
                ready = handle in self._broker.results
            if ready:
                return self.poll_inference(request, handle, now)
            time.sleep(.001)
        return None

    @property
    def inference_counters(self) -> dict:
        with self._broker.lock:
            return dict(self._broker.counts)

    def close(self) -> None:
        self._broker.close()

    # -------------------------------------------------------------- worker side
    def _infer(self, request: MecoInferenceRequest, inputs: Mapping[str, torch.Tensor]):
        model = self.model
        moved = {k: v.to(self.device, non_blocking=True) if isinstance(v, torch.Tensor) else v
                 for k, v in inputs.items()}
        with torch.no_grad():
            if self.device.type == "cuda":
                stream = torch.cuda.Stream(device=self.device)
                with torch.cuda.stream(stream):
                    out = model(**moved)
                    utility, penalty = out["utility"].float().cpu(), out["penalty"].float().cpu()
                stream.synchronize()
            else:
                out = model(**moved)
                utility, penalty = out["utility"].float(), out["penalty"].float()
        utility, penalty = utility.reshape(-1), penalty.reshape(-1)
        if utility.numel() != len(request.candidate_ids) or penalty.numel() != utility.numel():
            return None
        if not bool(torch.isfinite(utility).all() and torch.isfinite(penalty).all() and (penalty >= 0).all()):
            return None
        return ScorerOutput(request.candidate_ids, tuple(utility.tolist()), tuple(penalty.tolist()),
                            request.observation_time)


# --------------------------------------------------------------------------- capture
def capture_request(request: MecoInferenceRequest, inputs: Mapping[str, torch.Tensor], *,
                    source_snapshot_sha256: str = "", directory=None, max_requests: int | None = None):
    """Save one request's inputs (opt-in: MECO_REQUEST_CAPTURE_DIR, at most
    MECO_REQUEST_CAPTURE_MAX files) with a JSON manifest line holding the
    file's SHA-256. Returns the saved path or None when the bound is reached."""
    root = Path(directory or os.environ["MECO_REQUEST_CAPTURE_DIR"])
    limit = int(max_requests if max_requests is not None else os.environ.get("MECO_REQUEST_CAPTURE_MAX", "64"))
    root.mkdir(parents=True, exist_ok=True)
    if len(list(root.glob("request-*.pt"))) >= limit:
        return None
    path = root / f"request-{request.generation[:8]}-{request.sequence:08d}.pt"
    torch.save({k: v.detach().cpu() for k, v in inputs.items()}, path)
    digest = hashlib.sha256(path.read_bytes()).hexdigest()
    with (root / "manifest.jsonl").open("a") as fh:
        fh.write(json.dumps({"file": path.name, "sha256": digest, "sequence": request.sequence,
                             "generation": request.generation, "candidates": list(request.candidate_ids),
                             "observation_time": request.observation_time,
                             "source_snapshot_sha256": source_snapshot_sha256}, sort_keys=True) + "\n")
    return path


# --------------------------------------------------------------------------- monitoring
class DiagnosticMonitor:
    """Rolling window of arbiter reasons; ``alarm`` when the share of
    fallbacks (any reason but "scorer") exceeds `max_fallback_rate`."""

    def __init__(self, window: int = 512, max_fallback_rate: float = .25):
        self.window, self.max_rate = int(window), float(max_fallback_rate)
        self.reasons: list[str] = []

    def record(self, reason: str) -> None:
        self.reasons.append(reason)
        if len(self.reasons) > self.window:
            del self.reasons[:len(self.reasons) - self.window]

    @property
    def fallback_rate(self) -> float:
        if not self.reasons:
            return 0.
        return sum(r != "scorer" for r in self.reasons) / len(self.reasons)

    @property
    def alarm(self) -> bool:
        return len(self.reasons) >= min(32, self.window) and self.fallback_rate > self.max_rate

    def summary(self) -> dict:
        counts: dict[str, int] = {}
        for r in self.reasons:
            counts[r] = counts.get(r, 0) + 1
        return {"window": len(self.reasons), "fallback_rate": self.fallback_rate, "alarm": self.alarm,
                "reasons": counts}


# --------------------------------------------------------------------------- deployment
def export_scorer(model: nn.Module, example_inputs: Mapping[str, torch.Tensor], path) -> dict:
    """``torch.export`` program of a scorer (positional inputs in the order of
    `example_inputs`, outputs (utility, penalty)) saved with its SHA-256; ONNX
    is reported as unavailable when the package is missing."""
    path = Path(path)
    names = list(example_inputs)

    class _Positional(nn.Module):
        def __init__(self, inner):
            super().__init__()
            self.inner = inner

        def forward(self, *args):
            out = self.inner(**dict(zip(names, args)))
            return out["utility"], out["penalty"]

    wrapped = _Positional(model.eval())
    program = torch.export.export(wrapped, tuple(example_inputs[k] for k in names))
    torch.export.save(program, str(path))
    try:
        import onnx  # noqa: F401
        onnx_state = "available"
    except ImportError:
        onnx_state = "unavailable"
    return {"schema": "meco-scorer-export-v1", "format": "torch.export", "path": str(path), "inputs": names,
            "sha256": hashlib.sha256(path.read_bytes()).hexdigest(), "onnx_package": onnx_state}


def profile_latency(model: nn.Module, inputs: Mapping[str, torch.Tensor], iters: int = 50, warmup: int = 5) -> dict:
    """Per-call inference latency (CUDA events on CUDA, wall clock on CPU)."""
    dev = next(model.parameters()).device
    times = []
    with torch.no_grad():
        for k in range(warmup + iters):
            if dev.type == "cuda":
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                model(**inputs)
                b.record()
                b.synchronize()
                ms = a.elapsed_time(b)
            else:
                t0 = time.perf_counter()
                model(**inputs)
                ms = (time.perf_counter() - t0) * 1e3
            if k >= warmup:
                times.append(ms)
    times.sort()
    return {"iters": iters, "p50_ms": times[len(times) // 2], "p99_ms": times[min(len(times) - 1, int(.99 * len(times)))],
            "device": str(dev)}
