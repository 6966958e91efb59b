"""Benchmark: decode tokens/s of the 42-layer Q4_K_M Gemma-style model on B200
(bs1 after a 512-token prompt, and 64-sequence batched decode), plus the Q4_K GEMV's
HBM bandwidth, against the reference's CPU stage path timed on this host.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  torchrun --nproc-per-node N ... bench.py --gpus N   (one pipeline stage per GPU)
  python bench.py --case decode|prefill|gemv|gemm [...]   (fixed workloads for profilers, no JSON line)

One JSON line on rank 0.  `value` = bs1 greedy decode tokens/s (whole job); `bs64` = batched
decode tokens/s; `roofline` = the Q4_K GEMV (10240 x 2560, one token, cold L2) against the
measured HBM copy bandwidth; `e2e` = bs1 tokens/s through the stage C ABI with host buffers.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "compute-sharding_b200"))

METRIC = "decode tokens/s (bs1 and bs64) 42-layer Q4_K model at 1/2/4/8 B200; GEMV HBM GB/s"
N_LAYERS, HIDDEN, VOCAB = 42, 2560, 262144
PROMPT = 512
# algorithmic bytes of one Q4_K GEMV 10240 x 2560 with f32 x and y (14,745,600 + 10,240 + 40,960)
GEMV_BYTES = 10240 * 10 * 144 + 2560 * 4 + 10240 * 4
# algorithmic weight bytes of one decode token through all 42 layers + tied fp16 logits
LAYER_WEIGHT_BYTES = 60_518_400
EMBD_BYTES = VOCAB * HIDDEN * 2
# dram__bytes_read.sum + dram__bytes_write.sum of one qgemv_kernel<1,1> launch on that shape, from
# the ncu capture summarised in profiles/qgemv_q4k_10240x2560_1tok.md
GEMV_DRAM_BYTES = 14_816_512
# the tail stage's logits pass (262144 x 2560 fp16 table) in layers' worth of time for the split
# (64-row decode: about two layers)
TAIL_COST_LAYERS = 2.0
# greedy steps compared between the pipeline and a one-GPU run of the whole model (N > 1)
CHECK_STEPS = 64
BS64_WORKLOAD = "64 sequences, contexts uniform 512..3584 (seeded synthetic KV), 1 token each per step"
# multiply-add FLOPs of one 512-token prefill: the projections of 42 layers (q 2048, k 1024, v 1024,
# o, gate, up, down over hidden 2560 / ffn 10240), causal attention (8 query heads x 256 dims, QK and
# PV), and the logits of the last row (262144 x 2560)
LAYER_PARAMS = 2560 * (2048 + 1024 + 1024) + 2048 * 2560 + 3 * 2560 * 10240
PREFILL_FLOP = (2 * PROMPT * LAYER_PARAMS * N_LAYERS + N_LAYERS * 2 * 2 * 8 * 256 * PROMPT * (PROMPT + 1) // 2
                + 2 * HIDDEN * VOCAB)


def bs1_config(world: int = 1) -> dict:
    """`config` of the headline line, shared by both arms."""
    return {"workload": "42-layer Gemma-style Q4_K_M greedy decode, batch 1, after a 512-token prompt",
            "layers": N_LAYERS, "d_model": HIDDEN, "heads": "8q/4kv x 256", "ffn": 10240, "vocab": VOCAB,
            "prompt": PROMPT, "parallelism": f"pp{world}", "kv": "fp16",
            "l2": "inputs larger than L2 (3.9 GB of weights read per token)"}


def env_rank():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("LOCAL_RANK", "0"))


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


def bf16_sustained_tflops() -> float:
    """Dense bf16 GEMM throughput held for seconds (the denominator for a whole prefill)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text()).get("bf16_tflops_sustained", 1400.0))
    return 1400.0


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    def __init__(self, index: int, enabled: bool = True):
        self.index = index
        self.enabled = enabled
        self.proc = None
        fd, name = tempfile.mkstemp(prefix="sfc_clocks_", suffix=".csv")
        os.close(fd)
        self.path = Path(name)

    def __enter__(self):
        if not self.enabled:
            return self
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "25"], stdout=self.f, stderr=subprocess.DEVNULL)
            # the timed region starts once sampling has (nvidia-smi takes a moment to start)
            t_end = time.time() + 3.0
            while time.time() < t_end and self.path.stat().st_size == 0:
                time.sleep(0.01)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        try:
            rows = [r.split(",") for r in self.path.read_text().strip().splitlines() if r.strip()]
            self.path.unlink()
        except Exception:
            return None
        if not rows:
            return None
        sm = [float(r[1]) for r in rows]
        mx = float(rows[0][2])
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(rows)}


# ---------------------------------------------------------------- reference arm (CPU)
def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_decode_sample(n_steps: int, n_cached: int = PROMPT):
    """The reference's CPU stage path restated (oracle, kind 'port') on all host cores:
    42-layer greedy decode tokens/s after n_cached positions (seeded synthetic keys and values:
    a 512-token prefill would take minutes on the host).  Returns (tokens/s, threads, description)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import stage_oracle as so
    threads = os.cpu_count() or 1
    os.environ["ORACLE_THREADS"] = str(threads)
    spec = so.ModelSpec()
    st = so.OracleStage(so.synth_stage(spec, 0, N_LAYERS - 1, True, True),
                        so.Layout("synthetic-gemma", "full", 0, N_LAYERS - 1, True, True), rope_theta=10000.0)
    st.fill_session_synthetic("r", n_cached, seed=spec.seed)
    tok = int(so.synth_tokens(spec.seed, "bench.prompt", 1, spec.vocab)[0])
    t0 = time.perf_counter()
    for _ in range(n_steps):
        h = st.begin_token_ids("r", [tok])
        tok = st.sample_tail(h[-1])[0]
    dt = time.perf_counter() - t0
    desc = (f"{n_steps} greedy decode steps of the 42-layer model (d_model 2560, vocab 262144) after "
            f"{n_cached} cached positions (seeded synthetic K/V), f32 KV, {threads} threads (row-parallel like rayon)")
    return n_steps / dt, threads, desc


def run_reference(args):
    rank, world, _ = env_rank()
    if rank != 0:
        return
    steps = max(1, min(args.steps, 8))
    # warm-up steps are part of the same sampled loop (first-touch of weights); time `steps` after it
    tps, threads, desc = cpu_decode_sample(steps)
    line = {"impl": "reference", "metric": METRIC, "value": tps, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": args.warmup, "ms_per_step": 1e3 / tps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": bs1_config(world),
            "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": desc,
                             "cpu": cpu_model()},
            "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- our arm
def gemv_roofline(sf, torch, hbm_peak):
    """Config-1 GEMV: Q4_K 10240 x 2560, one token, cycling weight copies larger than twice the L2.

    The launches are captured once in a CUDA graph (one launch per weight copy, back to back with
    programmatic dependent launch, as inside a decode step) and the graph is replayed; CUDA events
    on the replay stream give the average device time per launch."""
    dev = torch.device("cuda")
    props = torch.cuda.get_device_properties(0)
    l2 = getattr(props, "L2_cache_size", 126 << 20)
    wbytes = 10240 * 10 * 144
    copies = int(np.ceil(2 * l2 / wbytes)) + 2
    ws = [sf.prepare_weights(sf.Q4_K, sf.synth_tensor(sf.Q4_K, 1, f"gemv.{i}", 10240, 2560, 0.02), 10240, 2560)
          for i in range(copies)]
    x = torch.randn(1, 2560, device=dev)
    y = torch.empty(1, 10240, device=dev)
    lib = sf.lib

    def launch_all():
        st = torch.cuda.current_stream().cuda_stream
        for i in range(copies):
            rc = lib.sfc_matmul(sf.Q4_K, ws[i].data_ptr(), 10240, 2560, x.data_ptr(), 1, y.data_ptr(), st)
            if rc:
                raise RuntimeError(f"sfc_matmul failed with {rc}")

    launch_all()  # first calls outside capture (device error flag lookup, etc.)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        launch_all()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    reps = 30
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    n = reps * copies
    dur_s = e0.elapsed_time(e1) / 1e3 / n
    achieved = GEMV_BYTES / dur_s / 1e9
    del g
    return {"kernel": "qgemv_kernel<1,1,Q4_K,15> (Q4_K 10240x2560, 1 token, weights cycled over > 2x L2)", "bound": "hbm",
            "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
            "us_per_launch": dur_s * 1e6, "launches_timed": n, "bytes_per_launch": GEMV_BYTES,
            "traffic": GEMV_DRAM_BYTES}


def run_single(args):
    import torch
    import stagefwd as sf
    torch.cuda.set_device(0)
    hbm_peak, peak_kind = peaks()
    shape = sf.ModelShape()  # 42 layers, Q4_K_M, vocab 262144, seed fixed
    max_ctx = 4096
    be = sf.CudaStageBackend(synthetic=shape, rope_theta=10000.0, max_ctx=max_ctx, max_sessions=66,
                             max_batch_tokens=512).load_layout("synthetic-gemma", "full", 0, N_LAYERS - 1, True, True)
    rng = np.random.default_rng(1234)
    prompt = rng.integers(0, VOCAB, PROMPT).astype(np.uint32)

    # ---- bs1 device-timed decode (one captured graph per token)
    be.generate_greedy("warm", prompt, max(args.warmup, 3) + 1)
    be.clear_decode_session("warm")
    with ClockSampler(0) as clk:
        toks = be.generate_greedy("bs1", prompt, args.steps + 1)
        prof = be.last_profile()
    be.clear_decode_session("bs1")
    bs1_s = prof.total_us / 1e6
    bs1_tps = args.steps / bs1_s
    launches = int(prof.kernels)  # kernels recorded in the decode graph x graph replays

    # ---- bs1 end-to-end through the stage C ABI (host buffers every step)
    h = be.begin_token_ids("e2e", prompt)
    tok, _ = be.sample_tail(h)
    for _ in range(args.warmup):
        h = be.begin_token_ids("e2e", [tok])
        tok, _ = be.sample_tail(h)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        h = be.begin_token_ids("e2e", [tok])
        tok, _ = be.sample_tail(h)
    e2e_s = time.perf_counter() - t0
    be.clear_decode_session("e2e")

    # ---- speculative verify: 1024 cached positions, 16-node draft tree (branching 2-2-2-2, BFS,
    # truncated), one tree-masked forward of the 42 layers + logits + acceptance walk (host API)
    sys.path.insert(0, str(ROOT / "oracle"))
    import stage_oracle as so
    parent = np.array(so.bfs_tree([2, 2, 2, 2], 16), np.int32)
    spec_res = {}
    for label, temp in (("greedy", 0.0), ("t0.8", 0.8)):
        times, accepted = [], []
        for rep in range(max(args.warmup, 3) + 4):
            be.fill_session_synthetic("verify", 1024, seed=7)
            nodes = rng.integers(0, VOCAB, 16).astype(np.uint32)
            t0 = time.perf_counter()
            rows = be.forward_tree("verify", parent, ids=nodes)
            path, _ = be.sample_tree(rows, parent, nodes, temperature=temp, seed=1000 + rep)
            be.commit_tree("verify", path)
            dt = time.perf_counter() - t0
            if rep >= max(args.warmup, 3):
                times.append(dt)
                accepted.append(len(path) - 1)
        spec_res[label] = {"ms_per_verify": 1e3 * statistics.median(times), "accepted_mean": float(np.mean(accepted))}
    be.clear_decode_session("verify")

    # ---- prefill / time to first token: the 512-token prompt into a fresh session (42 layers on the
    # tensor-core GEMM), logits of the last row and argmax; device-timed with the ids already on the
    # device, and end to end through the C ABI (host ids in, rows and the token back to the host)
    dev = torch.device("cuda")
    pids = torch.from_numpy(prompt.astype(np.int32)).to(dev)
    pout = torch.empty(PROMPT, HIDDEN, device=dev)
    ptok = torch.empty(1, dtype=torch.int64, device=dev)
    psc = torch.empty(1, dtype=torch.float32, device=dev)
    pf_dev, pf_host = [], []
    for rep in range(max(args.warmup, 3) + 5):
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        be.forward_dev(["pf"], [PROMPT], ids_dev=pids, out_dev=pout, append=False)
        be.sample_dev(pout[PROMPT - 1:], ptok, psc)
        f1.record()
        torch.cuda.synchronize()
        be.clear_decode_session("pf")
        t0 = time.perf_counter()
        rows = be.begin_token_ids("pfh", prompt)
        be.sample_tail(rows[PROMPT - 1:])
        dt = time.perf_counter() - t0
        be.clear_decode_session("pfh")
        if rep >= max(args.warmup, 3):
            pf_dev.append(f0.elapsed_time(f1))
            pf_host.append(dt * 1e3)
    pf_ms = statistics.median(pf_dev)
    bf16_peak = bf16_sustained_tflops()

    # ---- bs64 batched decode, contexts 512..3584 (seeded), one token per sequence per step
    ctx = rng.integers(512, 3585, 64)
    names = [f"b{i}" for i in range(64)]
    for i, n in enumerate(names):
        be.fill_session_synthetic(n, int(ctx[i]), seed=100 + i)
    ids = torch.from_numpy(rng.integers(0, VOCAB, 64).astype(np.int32)).to(dev)
    out = torch.empty(64, HIDDEN, device=dev)
    tk = torch.empty(64, dtype=torch.int64, device=dev)
    sc = torch.empty(64, dtype=torch.float32, device=dev)

    def bs64_step():
        be.forward_dev(names, [1] * 64, ids_dev=ids, out_dev=out, append=True)
        be.sample_dev(out, tk, sc)
        ids.copy_(tk.to(torch.int32))

    for _ in range(max(args.warmup, 3)):
        bs64_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    bsteps = max(16, args.steps // 4)
    e0.record()
    for _ in range(bsteps):
        bs64_step()
    e1.record()
    torch.cuda.synchronize()
    bs64_s = e0.elapsed_time(e1) / 1e3
    bs64_tps = 64 * bsteps / bs64_s
    be.close()

    roof = gemv_roofline(sf, torch, hbm_peak)
    roof["peak_kind"] = peak_kind

    cpu_tps, cores, desc = cpu_decode_sample(3)
    token_bytes = N_LAYERS * LAYER_WEIGHT_BYTES + EMBD_BYTES
    line = {
        "metric": METRIC, "value": bs1_tps, "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": bs1_s * 1e3 / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": bs1_config(1),
        "bs1_step_bandwidth_gbs": token_bytes / (bs1_s / args.steps) / 1e9,
        "bs64": {"value": bs64_tps, "unit": "tokens/s", "steps": bsteps, "ms_per_step": bs64_s * 1e3 / bsteps,
                 "workload": BS64_WORKLOAD},
        "gemv": {"value": roof["achieved"], "unit": "GB/s", "frac_of_hbm": roof["frac"]},
        "prefill": {"ttft_ms": pf_ms, "ttft_ms_e2e": statistics.median(pf_host), "tflops": PREFILL_FLOP / pf_ms / 1e9,
                    "frac_of_bf16_sustained": PREFILL_FLOP / pf_ms / 1e9 / bf16_peak,
                    "flop": PREFILL_FLOP,
                    "workload": "512-token prompt, fresh session, 42 layers + last-row logits + argmax; "
                                "e2e = begin_token_ids + sample_tail with host buffers"},
        "spec_verify": dict(spec_res, workload="1024 cached positions, 16-node draft tree (2-2-2-2, BFS, truncated) "
                                               "of random tokens: tree-masked forward of 42 layers, logits over "
                                               "262144, acceptance walk (greedy / seeded T=0.8), KV compaction; "
                                               "host buffers"),
        "e2e": {"value": args.steps / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": 4 + HIDDEN * 4,
                "d2h_bytes_per_step": HIDDEN * 4 + 8,
                "path": "begin_token_ids + sample_tail through the C ABI with host buffers each token"},
        "roofline": roof,
        "cpu_baseline": {"value": cpu_tps, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": desc,
                         "cpu": cpu_model()},
        "gpu_launches": launches,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def run_pipeline(args):
    import datetime
    import torch
    import torch.distributed as dist
    import stagefwd as sf
    from stagefwd.pipeline import CudaCompute, Pipeline, balanced_stage_split, make_groups
    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    ranks = make_groups(rank, world)
    split = balanced_stage_split(N_LAYERS, world, TAIL_COST_LAYERS)
    start, end = split[rank]
    be = sf.CudaStageBackend(synthetic=sf.ModelShape(), device=local, rope_theta=10000.0, max_ctx=4096,
                             max_sessions=66, max_batch_tokens=512).load_layout(
        "synthetic-gemma", f"stage-{rank}", start, end, ranks.is_head, ranks.is_tail)
    dev = torch.device("cuda", local)
    comp = CudaCompute(be, HIDDEN, 512, dev)
    pipe = Pipeline(comp, ranks, HIDDEN, dev)
    rng = np.random.default_rng(1234)
    prompt_np = rng.integers(0, VOCAB, PROMPT).astype(np.int64)
    prompt = torch.from_numpy(prompt_np).to(dev)

    def max_over_ranks(v: float) -> float:
        t = torch.tensor([v], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)

    # greedy stream of the pipeline on the seeded prompt; rank 0 also runs the whole model on one
    # GPU and compares (identical tokens for CHECK_STEPS steps)
    check = pipe.generate("check", prompt, CHECK_STEPS)
    match = None
    if rank == 0:
        full = sf.CudaStageBackend(synthetic=sf.ModelShape(), device=local, rope_theta=10000.0,
                                   max_ctx=PROMPT + CHECK_STEPS + 8, max_sessions=1).load_layout(
            "synthetic-gemma", "full", 0, N_LAYERS - 1, True, True)
        ref = full.generate_greedy("check", prompt_np.astype(np.uint32), CHECK_STEPS)
        full.close()
        match = check.cpu().tolist() == ref.tolist()
    be.clear_decode_session("check")

    # bs1
    pipe.generate("warm", prompt, max(args.warmup, 3))
    dist.barrier()
    torch.cuda.synchronize()
    tok = pipe.step(["bs1"], [PROMPT], prompt, append=False)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k0 = sf.kernel_launches()
    # clocks are sampled on rank 0's GPU only: one sampler process per rank slowed the ranks
    with ClockSampler(local, enabled=rank == 0) as clk:
        # the sampler starts on rank 0 only: line the ranks up again before the timed region
        dist.barrier()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(args.steps):
            tok = pipe.step(["bs1"], [1], tok if tok is not None else torch.zeros(1, dtype=torch.int64, device=dev))
        e1.record()
        torch.cuda.synchronize()
    dist.barrier()
    bs1_s = max_over_ranks(e0.elapsed_time(e1) / 1e3)
    launches = sf.kernel_launches() - k0

    # e2e: the same bs1 decode through the public pipeline API, each step's input token copied
    # from pinned host memory on the head and the sampled token read back to the host; timed by
    # the host clock on every rank (max over ranks)
    htok = torch.zeros(1, dtype=torch.int64, pin_memory=True)
    if ranks.is_head:
        htok.copy_(tok.view(1))
    dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        x = htok.to(dev, non_blocking=True) if ranks.is_head else None
        nxt = pipe.step(["bs1"], [1], x)
        if ranks.is_head:
            htok.copy_(nxt.view(1))
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    dist.barrier()

    # bs64: contexts 512..3584, as one microbatch per stage (the fastest schedule here) and as 8
    # microbatches of 8 sequences (the schedule the workload states)
    ctx = rng.integers(512, 3585, 64)
    names = [f"b{i}" for i in range(64)]
    bsteps = max(16, args.steps // 4)
    bs64 = {}
    for label, n_mb in (("one_microbatch_per_stage", world), ("microbatches_of_8", 8)):
        for i, n in enumerate(names):
            be.fill_session_synthetic(n, int(ctx[i]), seed=100 + i)
        mb = 64 // n_mb
        mbs = [names[mb * m: mb * m + mb] for m in range(n_mb)]
        tokens = [torch.from_numpy(rng.integers(0, VOCAB, mb).astype(np.int64)).to(dev) for _ in range(n_mb)]
        pipe.decode_microbatched(mbs, tokens, max(args.warmup, 3))
        torch.cuda.synchronize()
        dist.barrier()
        e0.record()
        pipe.decode_microbatched(mbs, tokens, bsteps)
        e1.record()
        torch.cuda.synchronize()
        dist.barrier()
        t = max_over_ranks(e0.elapsed_time(e1) / 1e3)
        bs64[label] = {"value": 64 * bsteps / t, "unit": "tokens/s", "steps": bsteps, "ms_per_step": 1e3 * t / bsteps,
                       "microbatches": f"{n_mb} x {mb} sequences"}
    be.close()
    roof = None
    if rank == 0:
        hbm_peak, peak_kind = peaks()
        roof = gemv_roofline(sf, torch, hbm_peak)
        roof["peak_kind"] = peak_kind
    dist.barrier()
    if rank == 0:
        best = max(bs64.values(), key=lambda d: d["value"])
        line = {"metric": METRIC, "value": args.steps / bs1_s, "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": bs1_s * 1e3 / args.steps,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic",
                "config": dict(bs1_config(world), split=split, tail_cost_layers=TAIL_COST_LAYERS,
                               handoff="NCCL send/recv of f32 hidden rows"),
                "tokens_match_1gpu": match,
                "tokens_match_steps": CHECK_STEPS,
                "bs64": dict(best, workload=BS64_WORKLOAD, schedules=bs64),
                "e2e": {"value": args.steps / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": 8,
                        "d2h_bytes_per_step": 8,
                        "path": "Pipeline.step per token, token from pinned host memory to the head and back; "
                                "host clock, max over ranks"},
                "roofline": roof, "gpu_launches": launches, "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    dist.destroy_process_group()


# ---------------------------------------------------------------- fixed workloads for profilers
def case_decode(steps: int, ctx: int, batch: int, layers: int = N_LAYERS):
    """`steps` eager decode steps of `batch` sequences after `ctx` seeded cached positions, through
    the device-pointer stage calls (no CUDA graph, so every kernel is its own launch); `layers` of
    the model (fewer keep a profiler's capture small)."""
    import torch
    import stagefwd as sf
    dev = torch.device("cuda")
    shape = sf.ModelShape(n_layers=layers)
    be = sf.CudaStageBackend(synthetic=shape, rope_theta=10000.0, max_ctx=max(ctx + steps + 8, 64),
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


def case_prefill(steps: int, tokens: int):
    """`steps` prefills of a `tokens`-token prompt into a fresh session (42 layers on the tensor-core
    GEMM, last-row logits and argmax), device-pointer calls."""
    import torch
    import stagefwd as sf
    dev = torch.device("cuda")
    shape = sf.ModelShape()
    be = sf.CudaStageBackend(synthetic=shape, rope_theta=10000.0, max_ctx=max(tokens + 8, 64), max_sessions=2,
                             max_batch_tokens=tokens).load_layout("synthetic-gemma", "full", 0, shape.n_layers - 1,
                                                                  True, True)
    ids = torch.arange(tokens, dtype=torch.int32, device=dev) * 997 % shape.vocab
    out = torch.empty(tokens, shape.hidden, device=dev)
    tk = torch.empty(1, dtype=torch.int64, device=dev)
    sc = torch.empty(1, dtype=torch.float32, device=dev)
    for _ in range(steps):
        be.forward_dev(["p"], [tokens], ids_dev=ids, out_dev=out, append=False)
        be.sample_dev(out[tokens - 1:], tk, sc)
        be.clear_decode_session("p")
    torch.cuda.synchronize()
    be.close()
    print("prefill", steps, "x", tokens, "tokens, first token", int(tk.item()))


def case_matmul(launches: int, tokens: int):
    """`launches` calls of sfc_matmul on the Q4_K 10240 x 2560 shape with `tokens` tokens (the GEMV
    from 1 to 7 tokens, the tensor-core GEMM from 8), over weight copies larger than twice the L2."""
    import torch
    import stagefwd as sf
    dev = torch.device("cuda")
    rows, k = 10240, 2560
    wbytes = rows * (k // 256) * 144
    copies = int(np.ceil(2 * (126 << 20) / wbytes)) + 2
    ws = [sf.prepare_weights(sf.Q4_K, sf.synth_tensor(sf.Q4_K, 1, f"gemv.{i}", rows, k, 0.02), rows, k)
          for i in range(copies)]
    x = torch.randn(tokens, k, device=dev)
    y = torch.empty(tokens, rows, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    for i in range(launches):
        rc = sf.lib.sfc_matmul(sf.Q4_K, ws[i % copies].data_ptr(), rows, k, x.data_ptr(), tokens, y.data_ptr(), st)
        if rc:
            raise RuntimeError(f"sfc_matmul failed: {rc}")
    torch.cuda.synchronize()
    print("matmul", launches, "launches of Q4_K", rows, "x", k, "with", tokens, "tokens over", copies, "weight copies")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--case", choices=["decode", "prefill", "gemv", "gemm"],
                    help="run a fixed workload for a profiler instead of the benchmark")
    ap.add_argument("--ctx", type=int, default=512, help="--case decode: cached positions per sequence")
    ap.add_argument("--batch", type=int, default=1, help="--case decode: sequences per step")
    ap.add_argument("--layers", type=int, default=N_LAYERS, help="--case decode: model layers")
    ap.add_argument("--tokens", type=int, default=64, help="--case gemm / prefill: tokens per launch / prompt")
    ap.add_argument("--launches", type=int, default=8, help="--case gemv/gemm: launches")
    args = ap.parse_args()
    if args.case:
        import torch
        torch.cuda.set_device(0)
        if args.case == "decode":
            case_decode(args.steps, args.ctx, args.batch, args.layers)
        elif args.case == "prefill":
            case_prefill(args.steps, args.tokens)
        else:
            case_matmul(args.launches, 1 if args.case == "gemv" else args.tokens)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    _, world, _ = env_rank()
    if world > 1:
        run_pipeline(args)
    else:
        run_single(args)


if __name__ == "__main__":
    main()
