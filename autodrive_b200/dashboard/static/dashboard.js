// Dashboard viewer: polls the JSON API and renders playback frames on a 2-D
// canvas (field boxes, robots as oriented 0.9 m squares with intake marker and
// held-FUEL count, free FUEL, planned routes, navigation targets, each robot's
// perceived FUEL tracks), streams a recording live while it is produced, and
// lists training, curriculum and MECO status.
"use strict";
const $ = (id) => document.getElementById(id);
const canvas = $("field");
const ctx = canvas.getContext("2d");
let layout = null, playback = null, frame = 0, playing = false, etag = null;

async function getJSON(url, opts) {
  const r = await fetch(url, opts);
  if (r.status === 304) return null;
  if (!r.ok) throw new Error(`${url}: ${r.status}`);
  return r.json();
}

function toCanvas(x, y) {
  const s = canvas.width / layout.length;
  return [x * s, canvas.height - y * s];
}

function drawField(hubActive) {
  ctx.fillStyle = "#2b3a2e";
  ctx.fillRect(0, 0, canvas.width, canvas.height);
  const s = canvas.width / layout.length;
  for (const b of layout.boxes) {
    const [cx, cy] = toCanvas(b.x, b.y);
    const w = b.length * s, h = b.width * s;
    const palette = { hub: "#8892a0", bump: "#5b4b3a", depot: "#39485a", trench: "#3c3c48", upright: "#9aa4b1", support: "#9aa4b1" };
    ctx.fillStyle = palette[b.kind] || "#444";
    ctx.globalAlpha = b.kind === "trench" ? 0.5 : 0.9;
    ctx.fillRect(cx - w / 2, cy - h / 2, w, h);
    ctx.globalAlpha = 1;
    if (b.kind === "hub") {
      const team = b.alliance === "red" ? 0 : 1;
      ctx.strokeStyle = hubActive && hubActive[team] ? (team ? "#5ea8ff" : "#ff6b6b") : "#555";
      ctx.lineWidth = 3;
      ctx.strokeRect(cx - w / 2, cy - h / 2, w, h);
    }
  }
}

function drawFrame(f) {
  drawField(f.hub_active);
  const s = canvas.width / layout.length;
  ctx.fillStyle = "#ffd43b";
  for (const [x, y] of f.fuel) {
    const [px, py] = toCanvas(x, y);
    ctx.beginPath(); ctx.arc(px, py, 0.075 * s, 0, 2 * Math.PI); ctx.fill();
  }
  const showTracks = $("show-tracks") && $("show-tracks").checked;
  f.robots.forEach((pose, r) => {
    const team = playback.teams ? playback.teams[r] : (r < 3 ? 0 : 1);
    if (showTracks && f.tracks && f.tracks[r]) {
      ctx.strokeStyle = team ? "#5ea8ff66" : "#ff6b6b66";
      ctx.lineWidth = 1;
      for (const [x, y] of f.tracks[r]) {
        const [px, py] = toCanvas(x, y);
        ctx.beginPath(); ctx.arc(px, py, 0.11 * s, 0, 2 * Math.PI); ctx.stroke();
      }
    }
    if (f.targets && f.targets[r]) {
      const [tx, ty] = toCanvas(f.targets[r][0], f.targets[r][1]);
      ctx.strokeStyle = team ? "#9cc8ff" : "#ffa3a3";
      ctx.lineWidth = 2;
      ctx.beginPath();
      ctx.moveTo(tx - 5, ty - 5); ctx.lineTo(tx + 5, ty + 5); ctx.moveTo(tx + 5, ty - 5); ctx.lineTo(tx - 5, ty + 5);
      ctx.stroke();
    }
    const route = f.routes ? f.routes[r] : [];
    if (route && route.length > 1) {
      ctx.setLineDash([6, 6]);
      ctx.strokeStyle = team ? "#5ea8ffaa" : "#ff6b6baa";
      ctx.beginPath();
      route.forEach(([x, y], i) => { const [px, py] = toCanvas(x, y); i ? ctx.lineTo(px, py) : ctx.moveTo(px, py); });
      ctx.stroke();
      ctx.setLineDash([]);
    }
    const [px, py] = toCanvas(pose[0], pose[1]);
    ctx.save();
    ctx.translate(px, py);
    ctx.rotate(-pose[2]);
    ctx.fillStyle = team ? "#2f6fc0" : "#c03a3a";
    ctx.fillRect(-0.45 * s, -0.45 * s, 0.9 * s, 0.9 * s);
    ctx.fillStyle = "#fff";
    ctx.fillRect(0.3 * s, -0.08 * s, 0.15 * s, 0.16 * s);
    ctx.restore();
    const held = f.possession ? f.possession[r] : 0;
    ctx.fillStyle = "#fff";
    ctx.font = `${Math.max(10, 0.35 * s)}px sans-serif`;
    ctx.textAlign = "center";
    ctx.fillText(held ? `${r}:${held}` : `${r}`, px, py + 0.12 * s);
  });
  $("clock").textContent = `${f.time.toFixed(1)} s  red ${f.scores[2]}  blue ${f.scores[3]}`;
}

function show(i) {
  if (!playback || !playback.frames.length) { if (layout) drawField(null); return; }
  frame = Math.max(0, Math.min(i, playback.frames.length - 1));
  $("scrub").value = frame;
  drawFrame(playback.frames[frame]);
}

async function loadPlayback(url) {
  const data = await getJSON(url);
  if (!data || !data.frames) return;
  playback = data;
  $("scrub").max = Math.max(0, data.frames.length - 1);
  show(0);
}

async function refreshStatus() {
  try {
    const st = await getJSON("/api/training-status");
    const dl = $("status");
    dl.innerHTML = "";
    for (const k of ["run_name", "state", "status", "task", "generation", "total_generations", "completed_timesteps", "transitions_per_second", "device"]) {
      if (st[k] === undefined) continue;
      dl.insertAdjacentHTML("beforeend", `<dt>${k}</dt><dd>${st[k]}</dd>`);
    }
    const body = $("generations").querySelector("tbody");
    body.innerHTML = "";
    for (const g of (st.generation_history || []).slice(-12)) {
      const m = g.metrics || g;
      body.insertAdjacentHTML("beforeend", `<tr><td>${g.generation ?? ""}</td><td>${(m.score_difference ?? m.mean_score_difference ?? "").toString().slice(0, 7)}</td><td>${(m.acquired ?? m.mean_acquired ?? "").toString().slice(0, 6)}</td><td>${(g.transitions_per_second ?? "").toString().slice(0, 8)}</td></tr>`);
    }
    const cur = await getJSON("/api/curriculum-status");
    $("curriculum").innerHTML = (cur || []).map((c) => `<li>${c.run}: ${c.state} — qualified ${(c.qualified || []).join(", ") || "none"}</li>`).join("");
  } catch (e) { /* server restarting */ }
}

async function record() {
  const run = $("run-select").value;
  const job = await getJSON(`/api/zone-playback?seconds=20&seed=${Date.now() % 1000}${run ? "&run=" + run : ""}`);
  // live stream: frames appear as the recording job produces them
  playback = { frames: [], teams: [0, 0, 0, 1, 1, 1] };
  let offset = 0;
  const poll = async () => {
    const st = await getJSON(`/api/zone-playback-stream?simulation_id=${job.simulation_id}&offset=${offset}`);
    if (st.metadata) playback = { ...st.metadata, frames: playback.frames };
    offset = st.next_offset;
    if (st.frames.length) {
      const atEnd = frame >= playback.frames.length - 1;
      playback.frames.push(...st.frames);
      $("scrub").max = Math.max(0, playback.frames.length - 1);
      if (atEnd) show(playback.frames.length - 1);
    }
    $("job").textContent = `${st.status} ${playback.frames.length} frames`;
    if (st.status === "running" || st.status === "waiting") return setTimeout(poll, 400);
  };
  poll();
}

async function refreshMeco() {
  try {
    const m = await getJSON("/api/meco-status");
    $("meco").innerHTML = (m.policies || []).map((p) =>
      `<li>${p.run}: track ${p.track ?? "?"}, ${p.updates} updates, ledger ${p.ledger_chain_verified ? "verified" : "BROKEN"}` +
      `${p.weights_sha256 ? ", weights " + p.weights_sha256.slice(0, 12) : ""}</li>`).join("") || "<li>no MECO runs</li>";
  } catch (e) { $("meco").innerHTML = "<li>MECO status unavailable</li>"; }
}

function tick() {
  if (playing && playback && frame < playback.frames.length - 1) show(frame + 1);
  setTimeout(tick, 100);
}

async function init() {
  layout = await getJSON("/api/field-layout");
  const st = await getJSON("/api/status");
  $("identity").textContent = `source ${st.source_identity.slice(0, 12)}`;
  const runs = await getJSON("/api/playback-runs");
  for (const r of runs) $("run-select").insertAdjacentHTML("beforeend", `<option value="${r.id}">${r.label}</option>`);
  $("run-select").onchange = () => { const v = $("run-select").value; if (v) loadPlayback(`/api/playback?run=${v}`); };
  $("record").onclick = record;
  $("play").onclick = () => { playing = !playing; $("play").textContent = playing ? "Pause" : "Play"; };
  $("scrub").oninput = (e) => show(+e.target.value);
  show(0);
  refreshStatus();
  refreshMeco();
  setInterval(refreshStatus, 5000);
  setInterval(refreshMeco, 15000);
  tick();
}
init();
