"""Dashboard HTTP server (frc_defense/dashboard.py:142-994, read-only).

    python -m autodrive_b200.dashboard --run-dir checkpoints/tensor-ppo --port 8765

GET endpoints (JSON unless noted):

  /                         static viewer (index.html, /assets/dashboard.js|css)
  /api/status               server identity, run directory, active jobs
  /api/training-status      newest (running first) run's status.json + generation history
  /api/curriculum-status    curriculum-status.json files under the curriculum root
  /api/field-layout         field boxes for the renderer
  /api/playback-runs        runs that have a playback.json
  /api/playback?run=R       playback.json of run R (ETag / If-None-Match)
  /api/generation?run=R&generation=N     generation-playback/generation-N.json
  /api/generation-scenario?run=R&generation=N
  /api/ablations            metrics/*/ablation*.json records
  /api/game-evaluations     evaluation playbacks available
  /api/game-evaluation-playback?name=N
  /api/zone-playback?seconds=S&seed=K[&run=R]   start a recording job -> {simulation_id}
  /api/focused-playback?...                     same, short focused window
  /api/zone-playback-progress?simulation_id=I
  /api/zone-playback-result?simulation_id=I
  /api/zone-playback-stream?simulation_id=I&offset=B   live frames of a recording from byte B
  /api/zone-playback-active
  /api/meco-status          MECO runs: latest metrics per track, ledger chain check, weights digest
  /api/scenario-replays     saved recordings
DELETE /api/scenario-replay?simulation_id=I   remove a finished saved recording

Run and file names are validated against fixed patterns; nothing outside the
run directory is served.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import re
import threading
import time
import uuid
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from pathlib import Path
from urllib.parse import parse_qs, urlparse

from .simulation import field_layout_payload, record_playback, write_json_atomic

STATIC = Path(__file__).resolve().parent / "static"
_RUN = re.compile(r"[A-Za-z0-9][A-Za-z0-9._-]{0,120}")
_SIM = re.compile(r"(?:scenario|focused)-[A-Za-z0-9_-]{1,80}")


def _read_json(path: Path, default):
    try:
        return json.loads(path.read_text())
    except (OSError, json.JSONDecodeError):
        return default


def source_identity() -> str:
    h = hashlib.sha256()
    for p in sorted(Path(__file__).resolve().parent.rglob("*")):
        if p.is_file() and p.suffix in (".py", ".js", ".css", ".html"):
            h.update(p.name.encode())
            h.update(p.read_bytes())
    return h.hexdigest()


class Jobs:
    """Background playback-recording jobs (one thread each)."""

    def __init__(self, store: Path, device: str):
        self.store, self.device = store, device
        self.lock = threading.Lock()
        self.jobs: dict[str, dict] = {}

    def start(self, kind: str, seconds: float, seed: int, checkpoint: Path | None) -> str:
        sid = f"{kind}-{uuid.uuid4().hex[:12]}"
        job = {"id": sid, "state": "running", "progress": 0., "started": time.time(), "cancel": False}
        with self.lock:
            self.jobs[sid] = job

        self.store.mkdir(parents=True, exist_ok=True)
        stream = self.store / f"{sid}.stream.jsonl"

        def emit(item: dict) -> None:
            # one JSON object per line, appended as frames are produced
            with stream.open("a") as fh:
                fh.write(json.dumps(item, separators=(",", ":")) + "\n")

        def run():
            try:
                rec = record_playback(seconds=seconds, device=self.device, seed=seed,
                                      checkpoint=str(checkpoint) if checkpoint else None,
                                      progress=lambda f: job.__setitem__("progress", round(f, 3)),
                                      cancel=lambda: job["cancel"],
                                      on_metadata=lambda m: emit({"type": "metadata", **m}),
                                      on_frame=lambda f: emit({"type": "frame", "frame": f}))
                write_json_atomic(self.store / f"{sid}.json", rec)
                job["state"] = "complete"
            except Exception as exc:  # noqa: BLE001 - reported through the API
                job["state"], job["error"] = "failed", f"{type(exc).__name__}: {exc}"
        threading.Thread(target=run, daemon=True).start()
        return sid

    def active(self) -> list[dict]:
        with self.lock:
            return [{k: v for k, v in j.items() if k != "cancel"} for j in self.jobs.values() if j["state"] == "running"]


def read_stream(jobs: "Jobs", q: dict) -> dict:
    """Frames of a running (or finished) recording from byte `offset` of its
    JSON-lines stream; `next_offset` resumes after the last complete line."""
    sid = q.get("simulation_id", [""])[0]
    if not _SIM.fullmatch(sid):
        raise ValueError("invalid simulation_id")
    offset = int(q.get("offset", ["0"])[0])
    if offset < 0:
        raise ValueError("offset must be a non-negative integer")
    job = jobs.jobs.get(sid)
    path = jobs.store / f"{sid}.stream.jsonl"
    metadata, frames, next_offset = None, [], offset
    if path.is_file():
        size = path.stat().st_size
        offset = 0 if offset > size else offset
        with path.open("rb") as fh:
            fh.seek(offset)
            chunk = fh.read(1_000_000)
        end = chunk.rfind(b"\n")
        if end >= 0:
            next_offset = offset + end + 1
            for line in chunk[:end + 1].splitlines():
                if not line:
                    continue
                item = json.loads(line)
                if item.get("type") == "metadata":
                    metadata = {k: v for k, v in item.items() if k != "type"}
                elif item.get("type") == "frame" and isinstance(item.get("frame"), dict):
                    frames.append(item["frame"])
    state = job["state"] if job else ("complete" if (jobs.store / f"{sid}.json").is_file() else "waiting")
    return {"simulation_id": sid, "metadata": metadata, "frames": frames, "next_offset": next_offset,
            "status": state}


def meco_status_payload(root: Path) -> dict:
    """MECO research runs under `root`: per run directory with a metric
    ledger, the latest update metrics per scorer track, the checkpoint digest
    and whether the ledger's hash chain verifies; runs of the same scenario
    family form one comparison group (frc_defense/meco_dashboard.py)."""
    from ..meco.train import MetricLedger
    policies, errors = [], []
    for ledger_path in sorted(Path(root).glob("*/metric-ledger.jsonl")):
        run = ledger_path.parent
        try:
            ledger = MetricLedger(ledger_path)
            records = ledger.records()
            chain_ok = ledger.verify()
        except (OSError, ValueError, KeyError) as exc:
            errors.append({"run": run.name, "error": str(exc)})
            continue
        updates = [r for r in records if r.get("kind") == "meco_update"]
        checkpoint = next((r for r in reversed(records) if r.get("kind") == "checkpoint"), None)
        last = updates[-1]["payload"] if updates else {}
        policies.append({"run": run.name, "track": last.get("track"), "updates": len(updates),
                         "latest": {k: v for k, v in last.items() if k not in ("config",)},
                         "weights_sha256": (checkpoint or {}).get("payload", {}).get("weights_sha256"),
                         "ledger_chain_verified": chain_ok, "records": len(records)})
    groups: dict = {}
    for pol in policies:
        groups.setdefault(pol["latest"].get("scenario") or "default", []).append(pol["run"])
    return {"schema_version": 1, "policies": policies,
            "comparison_groups": [{"scenario": k, "runs": v} for k, v in sorted(groups.items())],
            "errors": errors}


def create_handler(run_dir, curriculum_root=None, device: str = "cpu", meco_root=None):
    run_dir = Path(run_dir)
    meco_root = Path(meco_root) if meco_root else run_dir / "meco"
    curriculum_root = Path(curriculum_root) if curriculum_root else run_dir
    jobs = Jobs(run_dir / ".scenario-progress", device)
    identity = source_identity()

    def training_status() -> dict:
        runs = []
        for sp in run_dir.glob("*/status.json"):
            st = _read_json(sp, None)
            if isinstance(st, dict):
                st["run_name"] = sp.parent.name
                st["_age"] = time.time() - sp.stat().st_mtime
                runs.append(st)
        live = [r for r in runs if r.get("state", r.get("status")) == "running" and r["_age"] < 3 * 3600]
        pool = live or runs
        if not pool:
            return {"status": "waiting", "runs": []}
        sel = max(pool, key=lambda r: float(r.get("started_at") or 0.) - r["_age"] * 1e-9)
        hist = _read_json(run_dir / sel["run_name"] / "generation-history.json", {})
        sel["generation_history"] = hist.get("generations", []) if isinstance(hist, dict) else []
        if sel["generation_history"]:
            sel["latest_generation_metrics"] = sel["generation_history"][-1]
        sel["runs"] = [{k: r.get(k) for k in ("run_name", "task", "state", "status", "architecture", "generation",
                                               "total_generations", "completed_timesteps", "device")} for r in runs]
        for r in runs:
            r.pop("_age", None)
        return sel

    class Handler(BaseHTTPRequestHandler):
        server_version = "autodrive-dashboard/1"

        def _send(self, code: int, body: bytes, ctype="application/json", etag=None):
            self.send_response(code)
            self.send_header("Content-Type", ctype)
            self.send_header("Content-Length", str(len(body)))
            self.send_header("Cache-Control", "no-store")
            self.send_header("X-AutoDrive-Source-Identity-SHA256", identity)
            if etag:
                self.send_header("ETag", etag)
            self.end_headers()
            self.wfile.write(body)

        def _json(self, payload, code=200):
            self._send(code, json.dumps(payload, separators=(",", ":"), default=str).encode())

        def _file_json(self, path: Path, default):
            try:
                st = path.stat()
                etag = f'"{st.st_mtime_ns}-{st.st_size}"'
            except FileNotFoundError:
                return self._json(default)
            if self.headers.get("If-None-Match") == etag:
                self.send_response(304)
                self.send_header("ETag", etag)
                self.end_headers()
                return None
            self._send(200, path.read_bytes(), etag=etag)
            return None

        def _run(self, params) -> Path | None:
            name = params.get("run", [""])[0]
            if not name:
                return None
            if not _RUN.fullmatch(name) or not (run_dir / name).is_dir():
                self.send_error(400, "unknown run")
                raise LookupError
            return run_dir / name

        def log_message(self, fmt, *args):  # quiet
            pass

        def do_GET(self):  # noqa: C901 - one branch per endpoint
            u = urlparse(self.path)
            q = parse_qs(u.query)
            p = u.path
            try:
                if p in ("/", "/index.html"):
                    return self._send(200, (STATIC / "index.html").read_bytes(), "text/html; charset=utf-8")
                if p == "/assets/dashboard.js":
                    return self._send(200, (STATIC / "dashboard.js").read_bytes(), "text/javascript")
                if p == "/assets/dashboard.css":
                    return self._send(200, (STATIC / "dashboard.css").read_bytes(), "text/css")
                if p == "/api/status":
                    return self._json({"run_dir": str(run_dir), "source_identity": identity,
                                       "active_jobs": len(jobs.active()), "time": time.time()})
                if p == "/api/training-status":
                    return self._json(training_status())
                if p == "/api/curriculum-status":
                    rows = []
                    for sp in curriculum_root.glob("**/curriculum-status.json"):
                        st = _read_json(sp, None)
                        if isinstance(st, dict):
                            rows.append({"run": str(sp.parent.relative_to(curriculum_root)), **st})
                    return self._json(rows)
                if p == "/api/field-layout":
                    return self._json(field_layout_payload())
                if p == "/api/playback-runs":
                    runs = [{"id": c.name, "label": c.name.replace("-", " ").title(),
                             "mtime": (c / "playback.json").stat().st_mtime}
                            for c in run_dir.iterdir() if c.is_dir() and _RUN.fullmatch(c.name)
                            and (c / "playback.json").is_file()]
                    runs.sort(key=lambda r: -r["mtime"])
                    return self._json([{k: v for k, v in r.items() if k != "mtime"} for r in runs])
                if p == "/api/playback":
                    target = self._run(q) or run_dir
                    return self._file_json(target / "playback.json", {"frames": []})
                if p in ("/api/generation", "/api/generation-scenario"):
                    target = self._run(q) or run_dir
                    g = q.get("generation", [""])[0]
                    if not g.isdigit() or int(g) < 1:
                        return self.send_error(400, "generation must be a positive integer")
                    if p == "/api/generation":
                        return self._file_json(target / "generation-playback" / f"generation-{int(g)}.json",
                                               {"generation": int(g), "candidates": []})
                    return self._file_json(target / "scenario-simulations" / f"generation-{int(g):04d}" / "playback.json",
                                           {"generation": int(g), "scenarios": [], "status": "waiting"})
                if p == "/api/ablations":
                    recs = [_read_json(f, None) for f in sorted(run_dir.glob("**/ablation*.json"))]
                    return self._json([r for r in recs if r is not None])
                if p == "/api/game-evaluations":
                    names = sorted({f.parent.name for f in run_dir.glob("**/playback.json")
                                    if f.parent.name.startswith("ablations-")})
                    return self._json([{"id": n[len("ablations-"):], "label": n[len("ablations-"):].replace("_", " ")}
                                       for n in names])
                if p == "/api/game-evaluation-playback":
                    name = q.get("name", [""])[0]
                    if not _RUN.fullmatch(name or "-"):
                        return self.send_error(400, "invalid evaluation name")
                    hits = sorted(run_dir.glob(f"**/ablations-{name}/playback.json"))
                    return self._file_json(hits[0], {"frames": []}) if hits else self.send_error(404)
                if p in ("/api/zone-playback", "/api/focused-playback"):
                    seconds = float(q.get("seconds", ["20" if p.endswith("zone-playback") else "6"])[0])
                    if not 0 < seconds <= 160:
                        return self.send_error(400, "seconds must be in (0, 160]")
                    seed = int(q.get("seed", ["0"])[0])
                    target = self._run(q)
                    ck = target / "policy.pt" if target is not None and (target / "policy.pt").is_file() else None
                    sid = jobs.start("scenario" if p.endswith("zone-playback") else "focused", seconds, seed, ck)
                    return self._json({"simulation_id": sid, "state": "running"}, 202)
                if p in ("/api/zone-playback-progress", "/api/zone-playback-result"):
                    sid = q.get("simulation_id", [""])[0]
                    if not _SIM.fullmatch(sid):
                        return self.send_error(400, "invalid simulation id")
                    job = jobs.jobs.get(sid)
                    if p.endswith("progress"):
                        if job is None and not (jobs.store / f"{sid}.json").is_file():
                            return self.send_error(404)
                        return self._json({k: v for k, v in (job or {"id": sid, "state": "complete",
                                                                      "progress": 1.}).items() if k != "cancel"})
                    return self._file_json(jobs.store / f"{sid}.json", {"state": (job or {}).get("state", "missing")})
                if p == "/api/zone-playback-stream":
                    try:
                        return self._json(read_stream(jobs, q))
                    except ValueError as exc:
                        return self.send_error(400, str(exc))
                if p == "/api/meco-status":
                    try:
                        return self._json(meco_status_payload(meco_root))
                    except (OSError, ValueError) as exc:
                        return self._json({"schema_version": 1, "policies": [], "comparison_groups": [],
                                           "errors": [{"error": f"MECO status unavailable: {exc}"}]}, 503)
                if p == "/api/zone-playback-active":
                    return self._json(jobs.active())
                if p == "/api/scenario-replays":
                    files = sorted(jobs.store.glob("*.json")) if jobs.store.is_dir() else []
                    return self._json([{"simulation_id": f.stem, "bytes": f.stat().st_size} for f in files
                                       if _SIM.fullmatch(f.stem)])
                return self.send_error(404)
            except LookupError:
                return None

        def do_DELETE(self):
            u = urlparse(self.path)
            sid = parse_qs(u.query).get("simulation_id", [""])[0]
            if u.path != "/api/scenario-replay" or not _SIM.fullmatch(sid):
                return self._json({"error": "invalid saved scenario replay"}, 400)
            job = jobs.jobs.get(sid)
            if job is not None and job["state"] == "running":
                return self._json({"error": "this replay is still being generated"}, 409)
            path = jobs.store / f"{sid}.json"
            if not path.is_file():
                return self._json({"error": "no such replay"}, 404)
            path.unlink()
            jobs.jobs.pop(sid, None)
            return self._json({"deleted": sid})

    Handler.jobs = jobs
    return Handler


def serve(run_dir, host="127.0.0.1", port=8765, curriculum_root=None, device="cpu",
          meco_root=None) -> ThreadingHTTPServer:
    httpd = ThreadingHTTPServer((host, port), create_handler(run_dir, curriculum_root, device, meco_root))
    return httpd


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="autodrive_b200 training dashboard")
    p.add_argument("--run-dir", default="checkpoints/tensor-ppo")
    p.add_argument("--curriculum-root", default=None)
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--port", type=int, default=8765)
    p.add_argument("--device", default="cpu", help="device for playback recording jobs")
    p.add_argument("--meco-root", default=None, help="MECO run directories (default: <run-dir>/meco)")
    a = p.parse_args(argv)
    httpd = serve(a.run_dir, a.host, a.port, a.curriculum_root, a.device, a.meco_root)
    print(f"dashboard on http://{a.host}:{a.port} (run dir {a.run_dir})")
    try:
        httpd.serve_forever()
    except KeyboardInterrupt:
        pass
    finally:
        httpd.server_close()
