"""Fixed workloads for profilers (ncu launch lists and single-kernel captures).

    PYTHONPATH=compute-sharding_b200 python -m stagefwd.profiling decode [--steps N] [--ctx C] [--batch B]
    PYTHONPATH=compute-sharding_b200 python -m stagefwd.profiling gemv [--launches N]
    PYTHONPATH=compute-sharding_b200 python -m stagefwd.profiling gemm [--tokens T] [--launches N]

`decode` builds the 42-layer synthetic Q4_K_M stage (d_model 2560, vocab 262144), fills the
sessions with C seeded cached positions, and runs N eager decode steps of B sequences through
the device-pointer stage calls (no CUDA graph, so every kernel is its own launch for the
profiler).  `gemv` launches the 10240 x 2560 Q4_K GEMV (one token) over cycling weight copies
larger than twice the L2, the same kernel and shape the benchmark's roofline line reports.  `gemm` runs the same weight shape
through the tensor-core GEMM with T tokens (operand preparation + tcgen05 GEMM per launch).
"""
from __future__ import annotations

import argparse

import numpy as np
import torch

from . import Q4_K, CudaStageBackend, ModelShape, lib, prepare_weights, synth_tensor


def run_decode(steps: int, ctx: int, batch: int):
    dev = torch.device("cuda")
    shape = ModelShape()
    be = CudaStageBackend(synthetic=shape, rope_theta=10000.0, max_ctx=max(ctx + steps + 8, 64),
                          max_sessions=batch + 2, max_batch_tokens=max(batch, 8)).load_layout(
        "synthetic-gemma", "full", 0, shape.n_layers - 1, True, True)
    names = [f"s{i}" for i in range(batch)]
    for i, n in enumerate(names):
        be.fill_session_synthetic(n, ctx, seed=100 + i)
    ids = torch.arange(batch, dtype=torch.int32, device=dev) * 997 + 11
    out = torch.empty(batch, shape.hidden, device=dev)
    tk = torch.empty(batch, dtype=torch.int64, device=dev)
    sc = torch.empty(batch, dtype=torch.float32, device=dev)
    for _ in range(steps):
        be.forward_dev(names, [1] * batch, ids_dev=ids, out_dev=out, append=True)
        be.sample_dev(out, tk, sc)
        ids.copy_(tk.to(torch.int32))
    torch.cuda.synchronize()
    be.close()
    print("decode", steps, "steps, batch", batch, "ctx", ctx, "tokens", tk.tolist()[:8])


def run_gemv(launches: int, tokens: int = 1):
    dev = torch.device("cuda")
    rows, k = 10240, 2560
    wbytes = rows * (k // 256) * 144
    copies = int(np.ceil(2 * (126 << 20) / wbytes)) + 2
    ws = [prepare_weights(Q4_K, synth_tensor(Q4_K, 1, f"gemv.{i}", rows, k, 0.02), rows, k) for i in range(copies)]
    x = torch.randn(tokens, k, device=dev)
    y = torch.empty(tokens, rows, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    for i in range(launches):
        rc = lib.sfc_matmul(Q4_K, ws[i % copies].data_ptr(), rows, k, x.data_ptr(), tokens, y.data_ptr(), st)
        if rc:
            raise RuntimeError(f"sfc_matmul failed: {rc}")
    torch.cuda.synchronize()
    print("matmul", launches, "launches of Q4_K", rows, "x", k, "with", tokens, "tokens over", copies, "weight copies")


def main():
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    d = sub.add_parser("decode")
    d.add_argument("--steps", type=int, default=3)
    d.add_argument("--ctx", type=int, default=512)
    d.add_argument("--batch", type=int, default=1)
    g = sub.add_parser("gemv")
    g.add_argument("--launches", type=int, default=8)
    m = sub.add_parser("gemm")
    m.add_argument("--tokens", type=int, default=64)
    m.add_argument("--launches", type=int, default=8)
    a = ap.parse_args()
    torch.cuda.set_device(0)
    if a.cmd == "decode":
        run_decode(a.steps, a.ctx, a.batch)
    elif a.cmd == "gemv":
        run_gemv(a.launches)
    else:
        run_gemv(a.launches, a.tokens)


if __name__ == "__main__":
    main()
