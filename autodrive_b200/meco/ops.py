"""MECO research operations: device leases, task exposure scheduling, a
process supervisor, GPU / native-extension attestation and a release gate.

Parity with frc_defense/meco_device_lease.py (exclusive fcntl leases on
indexed devices, lockfiles never unlinked), meco_task_scheduler.py (resumable
exposure chunks unlocking curriculum stages), meco_supervisor.py (round-robin
tasks over devices, one process group per task, kill on timeout, restart with
exponential backoff, signal-safe shutdown), meco_gpu_attestation.py (device,
driver and loaded native-extension identity), meco_external_release_gate.py
(required artifacts and digests before a release).
"""
from __future__ import annotations

import fcntl
import hashlib
import json
import os
import random
import signal
import subprocess
import sys
import tempfile
import time
import uuid
from contextlib import AbstractContextManager
from dataclasses import dataclass, field
from datetime import datetime, timezone
from pathlib import Path

from ..train.curriculum import SCENARIOS, CurriculumState, ancestors, eligible_scenarios


# --------------------------------------------------------------------------- device lease
def device_index(device: str) -> int:
    if not isinstance(device, str) or not device.startswith("cuda:"):
        raise ValueError("device lease requires an indexed CUDA device")
    raw = device[5:]
    if not raw.isdecimal() or (len(raw) > 1 and raw.startswith("0")):
        raise ValueError("device lease requires a canonical indexed device")
    return int(raw)


class DeviceLease(AbstractContextManager):
    """Fail-fast exclusive leases (flock) on indexed devices; stable lockfile
    paths, never unlinked, holding the owner / pid / lease id as JSON."""

    def __init__(self, devices, *, owner: str = "meco", lock_root=None):
        devs = tuple(devices)
        if not devs or len(set(devs)) != len(devs):
            raise ValueError("device lease set must be nonempty and duplicate-free")
        self.devices = tuple(sorted(devs, key=device_index))
        self.owner = str(owner)
        self.lock_root = Path(lock_root or Path(tempfile.gettempdir()) / "autodrive-device-leases")
        self._handles = []
        self.lease_id = None

    @property
    def acquired(self) -> bool:
        return bool(self._handles) and len(self._handles) == len(self.devices)

    def acquire(self) -> "DeviceLease":
        if self._handles:
            raise RuntimeError("device lease is already acquired")
        self.lease_id = uuid.uuid4().hex
        self.lock_root.mkdir(parents=True, exist_ok=True)
        try:
            for dev in self.devices:
                path = self.lock_root / f"{hashlib.sha256(dev.encode()).hexdigest()[:16]}.lock"
                fh = path.open("a+")
                try:
                    fcntl.flock(fh.fileno(), fcntl.LOCK_EX | fcntl.LOCK_NB)
                except BlockingIOError as exc:
                    fh.close()
                    raise RuntimeError(f"indexed device {dev} is already leased") from exc
                self._handles.append(fh)
                fh.seek(0)
                fh.truncate()
                json.dump({"device": dev, "owner": self.owner, "pid": os.getpid(), "lease_id": self.lease_id,
                           "acquired_at": datetime.now(timezone.utc).isoformat()}, fh, sort_keys=True)
                fh.write("\n")
                fh.flush()
                os.fsync(fh.fileno())
            return self
        except BaseException:
            self.release()
            raise

    def release(self) -> None:
        while self._handles:
            fh = self._handles.pop()
            try:
                fcntl.flock(fh.fileno(), fcntl.LOCK_UN)
            finally:
                fh.close()

    def __enter__(self):
        return self.acquire()

    def __exit__(self, *exc):
        self.release()
        return False


# --------------------------------------------------------------------------- scheduler
SCHEDULER_VERSION = 1


def _digest(value) -> str:
    return hashlib.sha256(json.dumps(value, sort_keys=True, allow_nan=False).encode()).hexdigest()


@dataclass
class MecoTaskScheduler:
    """Deterministic, resumable exposure schedule: each eligible scenario is
    trained in `chunks_per_scenario` exposure chunks; a scenario's dependants
    unlock for exposure once its chunks are done (promotion itself still needs
    the qualified evaluation gates). State round-trips through JSON."""

    master_seed: int
    chunks_per_scenario: int = 10
    state: dict | None = None

    def __post_init__(self):
        if self.state is None:
            self.state = {"version": SCHEDULER_VERSION, "exposed": {}, "history": []}
        elif self.state.get("version") != SCHEDULER_VERSION:
            raise ValueError("incompatible scheduler state")

    def _unlocked(self) -> set[str]:
        done = {s for s, n in self.state["exposed"].items() if n >= self.chunks_per_scenario}
        return {s for s in SCENARIOS if ancestors(s) <= done}

    def next_task(self) -> dict | None:
        pending = sorted(s for s in self._unlocked() if self.state["exposed"].get(s, 0) < self.chunks_per_scenario)
        if not pending:
            return None
        rng = random.Random(_digest([self.master_seed, len(self.state["history"])]))
        sid = rng.choice(pending)
        chunk = self.state["exposed"].get(sid, 0)
        cats = SCENARIOS[sid].required_categories
        return {"scenario": sid, "category": cats[chunk % len(cats)], "chunk": chunk,
                "task_id": _digest([self.master_seed, sid, chunk])[:16]}

    def complete(self, task: dict) -> None:
        sid = task["scenario"]
        if self.state["exposed"].get(sid, 0) != task["chunk"]:
            raise ValueError("task completed out of order or twice")
        self.state["exposed"][sid] = task["chunk"] + 1
        self.state["history"].append(task["task_id"])

    def eligible_for_promotion(self, curriculum: CurriculumState) -> tuple[str, ...]:
        return tuple(s for s in eligible_scenarios(curriculum)
                     if self.state["exposed"].get(s, 0) >= self.chunks_per_scenario)

    def to_json(self) -> str:
        return json.dumps(self.state, sort_keys=True)

    @classmethod
    def from_json(cls, master_seed: int, text: str, chunks_per_scenario: int = 10) -> "MecoTaskScheduler":
        return cls(master_seed, chunks_per_scenario, json.loads(text))


# --------------------------------------------------------------------------- supervisor
@dataclass
class SupervisedTask:
    name: str
    argv: list[str]
    devices: tuple[str, ...] = ()
    timeout_s: float = 3600.
    max_restarts: int = 3
    env: dict = field(default_factory=dict)


class Supervisor:
    """Runs tasks round-robin over device leases, each in its own process
    group; a task past its timeout is killed with its whole group (TERM, then
    KILL after `grace_s`); a failed task restarts with exponential backoff up
    to `max_restarts`. SIGINT / SIGTERM stop every child group."""

    def __init__(self, tasks, *, lock_root=None, log_dir=None, backoff_s: float = 1., grace_s: float = 5.,
                 poll_s: float = .1):
        self.tasks = list(tasks)
        self.lock_root, self.backoff_s, self.grace_s, self.poll_s = lock_root, backoff_s, grace_s, poll_s
        self.log_dir = Path(log_dir) if log_dir else None
        self.results: dict[str, dict] = {}
        self._children: dict[int, subprocess.Popen] = {}
        self._stop = False

    def _kill_group(self, proc: subprocess.Popen) -> None:
        try:
            os.killpg(proc.pid, signal.SIGTERM)
        except ProcessLookupError:
            return
        deadline = time.monotonic() + self.grace_s
        while proc.poll() is None and time.monotonic() < deadline:
            time.sleep(.05)
        if proc.poll() is None:
            try:
                os.killpg(proc.pid, signal.SIGKILL)
            except ProcessLookupError:
                pass
            proc.wait()

    def _run_once(self, task: SupervisedTask, attempt: int) -> tuple[str, int | None]:
        lease = DeviceLease(task.devices, owner=task.name, lock_root=self.lock_root) if task.devices else None
        if lease is not None:
            lease.acquire()
        try:
            out = None
            if self.log_dir is not None:
                self.log_dir.mkdir(parents=True, exist_ok=True)
                out = open(self.log_dir / f"{task.name}.attempt{attempt}.log", "w")
            env = {**os.environ, **task.env}
            if task.devices:
                env["CUDA_VISIBLE_DEVICES"] = ",".join(str(device_index(d)) for d in task.devices)
            proc = subprocess.Popen(task.argv, env=env, stdout=out or subprocess.DEVNULL,
                                    stderr=subprocess.STDOUT if out else subprocess.DEVNULL, start_new_session=True)
            self._children[proc.pid] = proc
            start = time.monotonic()
            try:
                while proc.poll() is None:
                    if self._stop:
                        self._kill_group(proc)
                        return "stopped", proc.returncode
                    if time.monotonic() - start > task.timeout_s:
                        self._kill_group(proc)
                        return "timeout", proc.returncode
                    time.sleep(self.poll_s)
                return ("ok" if proc.returncode == 0 else "failed"), proc.returncode
            finally:
                self._children.pop(proc.pid, None)
                if out:
                    out.close()
        finally:
            if lease is not None:
                lease.release()

    def run(self) -> dict:
        previous = {}
        for sig in (signal.SIGINT, signal.SIGTERM):
            try:
                previous[sig] = signal.signal(sig, lambda *_: setattr(self, "_stop", True))
            except ValueError:  # not the main thread
                pass
        try:
            for task in self.tasks:
                attempts = []
                for attempt in range(task.max_restarts + 1):
                    status, code = self._run_once(task, attempt)
                    attempts.append({"attempt": attempt, "status": status, "returncode": code})
                    if status in ("ok", "stopped") or self._stop:
                        break
                    time.sleep(self.backoff_s * (2 ** attempt))
                self.results[task.name] = {"status": attempts[-1]["status"], "attempts": attempts}
                if self._stop:
                    break
        finally:
            for proc in list(self._children.values()):
                self._kill_group(proc)
            for sig, handler in previous.items():
                signal.signal(sig, handler)
        return self.results


# --------------------------------------------------------------------------- attestation / release gate
def native_extension_identity() -> dict:
    """Path and SHA-256 of the loaded native extension, as mapped by this process."""
    ext = None
    try:
        from ..ops import require_extension
        ext = require_extension()
    except RuntimeError:
        pass
    path = Path(getattr(ext, "__file__", "")) if ext else None
    mapped = False
    if path and path.is_file():
        try:
            mapped = str(path.resolve()) in Path("/proc/self/maps").read_text()
        except OSError:
            mapped = False
    return {"path": str(path) if path else None,
            "sha256": hashlib.sha256(path.read_bytes()).hexdigest() if path and path.is_file() else None,
            "mapped": mapped}


def gpu_attestation() -> dict:
    import torch
    rec = {"torch": torch.__version__, "cuda_available": torch.cuda.is_available(),
           "extension": native_extension_identity(), "time": datetime.now(timezone.utc).isoformat(),
           "python": sys.version.split()[0]}
    if torch.cuda.is_available():
        rec["devices"] = [{"index": i, "name": torch.cuda.get_device_name(i),
                           "capability": list(torch.cuda.get_device_capability(i)),
                           "memory_bytes": torch.cuda.get_device_properties(i).total_memory}
                          for i in range(torch.cuda.device_count())]
        rec["cuda_runtime"] = torch.version.cuda
    rec["digest"] = _digest({k: v for k, v in rec.items() if k != "time"})
    return rec


def release_gate(run_dir, *, required=("policy.pt", "status.json", "metadata.json"),
                 expected_sha256: dict | None = None) -> dict:
    """Pass only when every required artifact exists, the status is complete,
    and every listed artifact has the expected SHA-256."""
    run = Path(run_dir)
    failures = [f"missing {name}" for name in required if not (run / name).is_file()]
    status = {}
    if (run / "status.json").is_file():
        try:
            status = json.loads((run / "status.json").read_text())
        except json.JSONDecodeError:
            failures.append("status.json is not valid JSON")
    if status and status.get("state", status.get("status")) not in ("complete", "completed"):
        failures.append("run is not complete")
    for name, digest in (expected_sha256 or {}).items():
        p = run / name
        if not p.is_file() or hashlib.sha256(p.read_bytes()).hexdigest() != digest:
            failures.append(f"digest mismatch for {name}")
    return {"passed": not failures, "failures": failures, "run": str(run)}
