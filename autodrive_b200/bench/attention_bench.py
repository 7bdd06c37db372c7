"""Microbenchmark of the tcgen05 variable-length attention
(``ops.attention.varlen_attention``) against PyTorch's memory-efficient
attention kernel on the entity encoder's packed minibatch: `samples` samples
whose valid-token counts are drawn uniformly from [lo, hi] (the benchmark
world's encoder sees 5-403 live tokens per sample, mean about 190), 4 heads
of dimension 64.

    python -m autodrive_b200.bench.attention_bench [--samples 768] [--lo 5] [--hi 403] [--iters 20]

Forward and forward + backward are timed with CUDA events over `iters`
launches after 3 warm-up launches, rotating over two input sets. Prints one
JSON line per case with both times and the attention FLOPs per second
(4 * sum(L^2) * 64 * heads per forward, 2.5x that for the backward).
"""
from __future__ import annotations

import argparse
import json

import torch

from ..ops.attention import varlen_attention

HEADS, DH = 4, 64


def _time(fn, iters: int) -> float:
    for i in range(3):
        fn(i)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(iters):
        fn(i)
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def _aten_forward(qkv, cu, max_len):
    x = qkv.view(1, qkv.shape[0], 3, HEADS, DH)
    q, k, v = x.select(2, 0), x.select(2, 1), x.select(2, 2)
    out, lse, seed, offset, _, _ = torch.ops.aten._efficient_attention_forward(
        q, k, v, None, cu, cu, max_len, max_len, 0.0, 0, True)
    return q, k, v, out, lse, seed, offset


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--samples", type=int, default=768)
    ap.add_argument("--lo", type=int, default=5)
    ap.add_argument("--hi", type=int, default=403)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args(argv)
    g = torch.Generator().manual_seed(args.seed)
    dev = torch.device("cuda")
    lengths = torch.randint(args.lo, args.hi + 1, (args.samples,), generator=g)
    cu = torch.zeros(args.samples + 1, dtype=torch.int32)
    cu[1:] = lengths.cumsum(0)
    cu = cu.to(dev)
    total, max_len = int(lengths.sum()), int(lengths.max())
    sets = [torch.randn((total, 3 * HEADS * DH), device=dev).bfloat16().requires_grad_(True) for _ in range(2)]
    grads = [torch.randn((total, HEADS * DH), device=dev).bfloat16() for _ in range(2)]
    flops = 4.0 * float((lengths.double() ** 2).sum()) * DH * HEADS

    ours_f = _time(lambda i: varlen_attention(sets[i % 2].detach(), cu, max_len, HEADS), args.iters)
    aten_f = _time(lambda i: _aten_forward(sets[i % 2].detach(), cu, max_len), args.iters)

    def ours_fb(i):
        x = sets[i % 2]
        varlen_attention(x, cu, max_len, HEADS).backward(grads[i % 2])

    def aten_fb(i):
        x = sets[i % 2].detach()
        q, k, v, out, lse, seed, offset = _aten_forward(x, cu, max_len)
        torch.ops.aten._efficient_attention_backward(
            grads[i % 2].view(out.shape), q, k, v, None, out, cu, cu, max_len, max_len, lse, 0.0, seed, offset, 0,
            False, shared_storage_dqdkdv=True)

    ours_b = _time(ours_fb, args.iters)
    aten_b = _time(aten_fb, args.iters)
    common = {"samples": args.samples, "tokens": total, "max_len": max_len, "heads": HEADS, "head_dim": DH}
    print(json.dumps({"case": "forward", **common, "tc_ms": round(ours_f, 4), "aten_ms": round(aten_f, 4),
                      "tc_tflops": round(flops / ours_f / 1e9, 1), "aten_tflops": round(flops / aten_f / 1e9, 1)}))
    print(json.dumps({"case": "forward+backward", **common, "tc_ms": round(ours_b, 4), "aten_ms": round(aten_b, 4),
                      "tc_tflops": round(3.5 * flops / ours_b / 1e9, 1),
                      "aten_tflops": round(3.5 * flops / aten_b / 1e9, 1)}))


if __name__ == "__main__":
    main()
