"""Policy-kernel micro-benchmark: tcgen05 kernels vs PyTorch eager.

    python -m autodrive_b200.bench.policy_bench --rows 6144 --iters 50

Times (CUDA events, after warm-up, median of `--iters`):

* ``act``          fused forward + masked sample + log-prob + value (one launch)
* ``train``        fused PPO minibatch forward + backward (partial gradients)
* ``minibatch``    one whole PPO minibatch step on the tensor-core path:
                   advantage stats, fused fwd+bwd, partial reduction, fused
                   clip + Adam, weight re-pack
* ``torch_*``      the same work in PyTorch eager fp32 (autograd + the fused
                   Adam kernel), the path used without the tensor-core kernels

and reports the policy FLOPs per row so the tensor-core time can be read
against the GEMM peak. Inputs are rows of a synthetic [N, 137] observation
buffer larger than L2 when ``--pool`` rows are used (default 262144 rows,
143 MB), gathered by random index like a PPO minibatch.
"""
from __future__ import annotations

import argparse
import json
import statistics

import torch


def _time(fn, iters):
    ts = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b))
    return statistics.median(ts)


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--rows", type=int, default=6144)
    p.add_argument("--pool", type=int, default=262144)
    p.add_argument("--iters", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    args = p.parse_args()
    from autodrive_b200.train.ppo import PPOConfig, PPOLearner
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    cfg = PPOConfig(epochs=1, minibatch_size=args.rows, grad_backend="local")
    fused = PPOLearner(137, 8, "categorical", dev, cfg, "mlp", 1)
    eager_cfg = PPOConfig(epochs=1, minibatch_size=args.rows, grad_backend="local", fused_policy=False)
    eager = PPOLearner(137, 8, "categorical", dev, eager_cfg, "mlp", 1)
    eager.model.load_state_dict(fused.model.state_dict())
    n = args.pool
    obs = torch.randn(n, 137, device=dev) * .7
    obs[:, -8:] = (torch.rand(n, 8, device=dev) > .3).float()
    obs[:, -8] = 1.
    tc = fused._tc_ready()
    with torch.no_grad():
        action, logp, value, mask = tc.act(obs)
    batch = {"obs": obs, "actions": action, "mask": mask, "logp": logp,
             "adv": torch.randn(n, device=dev), "returns": torch.randn(n, device=dev)}
    ent = torch.full((1,), .01, device=dev)
    stats = torch.zeros(5, device=dev)
    idx_pool = [torch.randperm(n, device=dev)[:args.rows] for _ in range(8)]
    rows_obs = [obs[i].contiguous() for i in idx_pool]
    it = {"k": 0}

    def nxt():
        it["k"] = (it["k"] + 1) % len(idx_pool)
        return it["k"]

    def act():
        tc.act(rows_obs[nxt()])

    def train():
        k = nxt()
        b = int(idx_pool[k].numel())
        tc.ext.policy_train(batch["obs"], idx_pool[k], 8, tc.images, tc.flat.flat, tc.offsets, batch["actions"],
                            batch["mask"], batch["logp"], batch["adv"], batch["returns"], tc.adv_stats, ent,
                            .2, .5, tc.partials(b), stats, tc.status)

    def minibatch():
        k = nxt()
        tc.train_minibatch(batch, idx_pool[k], ent, .2, .5, 1e-5, stats)
        fused.sync.step()
        fused.weights_version += 1
        tc.pack(fused.weights_version)

    def torch_act():
        with torch.no_grad():
            eager.act(rows_obs[nxt()])

    flat = {k2: v for k2, v in batch.items()}

    def torch_minibatch():
        k = nxt()
        idx = idx_pool[k]
        model = eager.model
        logp_n, entropy, val, _ = model.score(flat["obs"][idx], flat["actions"][idx], flat["mask"][idx])
        ratio = (logp_n - flat["logp"][idx]).exp()
        adv = flat["adv"][idx]
        adv = (adv - adv.mean()) / (adv.std(unbiased=False) + 1e-8)
        pg = torch.maximum(-adv * ratio, -adv * ratio.clamp(.8, 1.2)).mean()
        vloss = .5 * (val - flat["returns"][idx]).square().mean()
        l2 = sum(q.square().sum() for q in model.parameters() if q.ndim > 1)
        loss = pg + .5 * vloss - .01 * entropy.mean() + 1e-5 * l2
        eager.opt.zero_grad()
        loss.backward()
        eager.sync.step()

    out = {}
    for name, fn in (("act", act), ("train", train), ("minibatch", minibatch), ("torch_act", torch_act),
                     ("torch_minibatch", torch_minibatch)):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        out[name + "_ms"] = round(_time(fn, args.iters), 4)
    tc._post_status()
    tc.check()
    d, hdim, a = 137, 128, 9
    fwd = 2 * (d * hdim + hdim * hdim + hdim * a)
    out.update({"rows": args.rows, "pool_rows": n, "fwd_flops_per_row": fwd, "fwd_bwd_flops_per_row": 3 * fwd,
                "train_tflops": round(3 * fwd * args.rows / (out["train_ms"] * 1e-3) / 1e12, 3),
                "speedup_minibatch_vs_torch": round(out["torch_minibatch_ms"] / out["minibatch_ms"], 2),
                "speedup_act_vs_torch": round(out["torch_act_ms"] / out["act_ms"], 2)})
    print(json.dumps(out))


if __name__ == "__main__":
    main()
