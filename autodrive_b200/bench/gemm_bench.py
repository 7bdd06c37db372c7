"""Microbenchmark of the tcgen05 GEMM (``ops.tc_linear.gemm``) against the
cuBLAS bf16 GEMM (``torch.mm``) on the linear-layer shapes of the entity
encoder's PPO minibatch (tokens x d = 256, 4 heads, feed-forward 1024).

    python -m autodrive_b200.bench.gemm_bench [--tokens 311040] [--iters 20]

Each case is timed with CUDA events over `iters` launches after 3 warm-up
launches; every operand set is larger than the 126 MB L2 or rotates through
buffers that together are, so each launch reads from HBM. Prints one JSON line
per case: time, TFLOP/s, and the same for cuBLAS. Two more cases time the
GELU epilogues (the feed-forward's first forward GEMM with GELU and the kept
pre-activation; its backward dH GEMM scaled by GELU') against cuBLAS followed
by PyTorch's GELU kernels.
"""
from __future__ import annotations

import argparse
import json

import torch

from ..ops.tc_linear import gemm


def _time(fn, iters: int) -> float:
    for _ in range(3):
        fn(0)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(iters):
        fn(i)
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=311040)
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args(argv)
    m = args.tokens
    cases = [("qkv forward", m, 768, 256, False, False), ("out_proj forward", m, 256, 256, False, False),
             ("ff1 forward", m, 1024, 256, False, False), ("ff2 forward", m, 256, 1024, False, False),
             ("ff2 dX", m, 1024, 256, False, True), ("ff1 dW", 1024, 256, m, True, True)]
    dev = torch.device("cuda")
    for name, mm, n, k, a_mn, b_mn in cases:
        nbuf = 2
        a = [torch.randn((k, mm) if a_mn else (mm, k), device=dev).bfloat16() for _ in range(nbuf)]
        b = [torch.randn((k, n) if b_mn else (n, k), device=dev).bfloat16() for _ in range(nbuf)]
        out = torch.empty((mm, n), device=dev, dtype=torch.bfloat16 if not a_mn else torch.float32)
        ours = _time(lambda i: gemm(a[i % nbuf], b[i % nbuf], a_mn=a_mn, b_mn=b_mn, out=out), args.iters)
        aa = [x.T if a_mn else x for x in a]
        bb = [x if b_mn else x.T for x in b]
        out_ref = torch.empty((mm, n), device=dev, dtype=torch.bfloat16)
        ref = _time(lambda i: torch.mm(aa[i % nbuf], bb[i % nbuf], out=out_ref), args.iters)
        flops = 2.0 * mm * n * k
        print(json.dumps({"case": name, "M": mm, "N": n, "K": k, "a_mn": a_mn, "b_mn": b_mn,
                          "tc_gemm_ms": round(ours, 4), "tc_gemm_tflops": round(flops / ours / 1e9, 1),
                          "cublas_ms": round(ref, 4), "cublas_tflops": round(flops / ref / 1e9, 1)}), flush=True)
        del a, b, out, out_ref
    # fused GELU epilogues against cuBLAS + the PyTorch GELU kernels
    x = [torch.randn((m, 256), device=dev).bfloat16() for _ in range(2)]
    w1 = torch.randn((1024, 256), device=dev).bfloat16()
    bias = torch.randn(1024, device=dev)
    z = torch.empty((m, 1024), device=dev, dtype=torch.bfloat16)
    h = torch.empty((m, 1024), device=dev, dtype=torch.bfloat16)
    ours = _time(lambda i: gemm(x[i % 2], w1, bias=bias, act="gelu", aux=z, out=h), args.iters)
    b16 = bias.bfloat16()

    def ref_fwd(i):
        zz = torch.addmm(b16, x[i % 2], w1.T)
        return torch.nn.functional.gelu(zz)
    ref = _time(ref_fwd, args.iters)
    print(json.dumps({"case": "ff1 forward + GELU (pre-activation kept)", "M": m, "N": 1024, "K": 256,
                      "tc_gemm_ms": round(ours, 4), "cublas_plus_gelu_ms": round(ref, 4)}), flush=True)
    dy = [torch.randn((m, 256), device=dev).bfloat16() for _ in range(2)]
    w2 = torch.randn((256, 1024), device=dev).bfloat16()
    dz = torch.empty((m, 1024), device=dev, dtype=torch.bfloat16)
    ours = _time(lambda i: gemm(dy[i % 2], w2, b_mn=True, act="gelu_grad", aux=z, out=dz), args.iters)

    def ref_bwd(i):
        dh = torch.mm(dy[i % 2], w2)
        return torch.ops.aten.gelu_backward(dh, z)
    ref = _time(ref_bwd, args.iters)
    print(json.dumps({"case": "ff2 dX x GELU' (backward of the above)", "M": m, "N": 1024, "K": 256,
                      "tc_gemm_ms": round(ours, 4), "cublas_plus_gelu_backward_ms": round(ref, 4)}), flush=True)


if __name__ == "__main__":
    main()
