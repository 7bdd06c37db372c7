"""Dashboard API against a temporary run directory (CPU, real HTTP)."""
import json
import threading
import time
import urllib.error
import urllib.request

import pytest

from autodrive_b200.dashboard import serve


@pytest.fixture()
def server(tmp_path):
    run = tmp_path / "runs"
    r1 = run / "gen-run"
    r1.mkdir(parents=True)
    (r1 / "status.json").write_text(json.dumps({"state": "running", "task": "defense", "generation": 2,
                                                 "started_at": time.time()}))
    (r1 / "generation-history.json").write_text(json.dumps({"generations": [{"generation": 1}, {"generation": 2}]}))
    (r1 / "playback.json").write_text(json.dumps({"frames": [{"tick": 1}]}))
    (r1 / "generation-playback").mkdir()
    (r1 / "generation-playback" / "generation-2.json").write_text(json.dumps({"generation": 2, "candidates": [1]}))
    cur = run / "cur"
    cur.mkdir()
    (cur / "curriculum-status.json").write_text(json.dumps({"state": "complete", "qualified": ["pickup_simple"]}))
    from autodrive_b200.meco.train import MetricLedger
    ledger = MetricLedger(run / "meco" / "track-a" / "metric-ledger.jsonl")
    ledger.append("meco_update", {"track": "A1", "update": 1, "mean_return": .1})
    ledger.append("meco_update", {"track": "A1", "update": 2, "mean_return": .2})
    ledger.append("checkpoint", {"path": "meco.pt", "weights_sha256": "ab" * 32})
    httpd = serve(run, port=0)
    t = threading.Thread(target=httpd.serve_forever, daemon=True)
    t.start()
    yield f"http://127.0.0.1:{httpd.server_address[1]}"
    httpd.shutdown()
    httpd.server_close()


def _get(url, method="GET", headers=None):
    req = urllib.request.Request(url, method=method, headers=headers or {})
    try:
        with urllib.request.urlopen(req, timeout=60) as r:
            return r.status, r.headers, r.read()
    except urllib.error.HTTPError as e:
        return e.code, e.headers, e.read()


def test_endpoints(server):
    code, _, body = _get(server + "/")
    assert code == 200 and b"<canvas" in body
    assert _get(server + "/assets/dashboard.js")[0] == 200
    st = json.loads(_get(server + "/api/training-status")[2])
    assert st["run_name"] == "gen-run" and st["latest_generation_metrics"]["generation"] == 2
    lay = json.loads(_get(server + "/api/field-layout")[2])
    assert lay["length"] > 16 and any(b["kind"] == "hub" for b in lay["boxes"])
    assert json.loads(_get(server + "/api/playback-runs")[2])[0]["id"] == "gen-run"
    code, headers, body = _get(server + "/api/playback?run=gen-run")
    assert code == 200 and json.loads(body)["frames"]
    assert _get(server + "/api/playback?run=gen-run", headers={"If-None-Match": headers["ETag"]})[0] == 304
    assert _get(server + "/api/playback?run=../etc")[0] == 400
    assert json.loads(_get(server + "/api/generation?run=gen-run&generation=2")[2])["candidates"] == [1]
    assert _get(server + "/api/generation?run=gen-run&generation=0")[0] == 400
    cur = json.loads(_get(server + "/api/curriculum-status")[2])
    assert cur and cur[0]["qualified"] == ["pickup_simple"]
    assert _get(server + "/api/nope")[0] == 404
    meco = json.loads(_get(server + "/api/meco-status")[2])
    assert meco["schema_version"] == 1 and meco["policies"][0]["run"] == "track-a"
    assert meco["policies"][0]["ledger_chain_verified"] and meco["policies"][0]["updates"] == 2


def test_recording_job_and_delete(server):
    code, _, body = _get(server + "/api/zone-playback?seconds=1&seed=3")
    assert code == 202
    sid = json.loads(body)["simulation_id"]
    for _ in range(600):
        p = json.loads(_get(server + f"/api/zone-playback-progress?simulation_id={sid}")[2])
        if p["state"] != "running":
            break
        time.sleep(.1)
    assert p["state"] == "complete", p
    rec = json.loads(_get(server + f"/api/zone-playback-result?simulation_id={sid}")[2])
    assert len(rec["frames"]) == 10 and len(rec["frames"][0]["robots"]) == 6
    assert len(rec["frames"][0]["tracks"]) == 6 and len(rec["frames"][0]["possession"]) == 6
    # the live stream carries the same frames, resumable from a byte offset
    first = json.loads(_get(server + f"/api/zone-playback-stream?simulation_id={sid}&offset=0")[2])
    assert first["status"] == "complete" and first["metadata"]["teams"] == [0, 0, 0, 1, 1, 1]
    assert [f["tick"] for f in first["frames"]] == [f["tick"] for f in rec["frames"]]
    rest = json.loads(_get(server + f"/api/zone-playback-stream?simulation_id={sid}&offset={first['next_offset']}")[2])
    assert rest["frames"] == [] and rest["next_offset"] == first["next_offset"]
    assert _get(server + "/api/zone-playback-stream?simulation_id=../x")[0] == 400
    assert any(r["simulation_id"] == sid for r in json.loads(_get(server + "/api/scenario-replays")[2]))
    assert _get(server + f"/api/scenario-replay?simulation_id={sid}", method="DELETE")[0] == 200
    assert _get(server + "/api/scenario-replay?simulation_id=bad/../x", method="DELETE")[0] == 400
