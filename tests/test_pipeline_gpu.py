"""Two GPUs over NCCL: the pipeline driver (stagefwd/pipeline.py) with one stage per GPU gives the
stream of the whole model on one GPU, token for token: greedy generation after a 40-token prompt
(the reference's generate loop, bin/real_two_stage_generate_bench.rs:232-290) and decode of two
microbatches of three sequences.  Split stages compute the single stage's hidden states bit for bit,
so the streams are identical.  Skipped with fewer than two visible GPUs.

Ranks are spawned processes (one per GPU) with a short process-group timeout, so a rank that fails
ends the other's next receive with an error instead of a wait."""
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

CFG = dict(hidden=512, n_heads=4, n_kv=2, head_dim=128, ffn=1024, vocab=4096, n_layers=6, seed=91)
PROMPT, STEPS = 40, 24
MBS = [["a", "b", "c"], ["d", "e", "f"]]
MB_STEPS = 4


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def prompts():
    rng = np.random.default_rng(7)
    main = rng.integers(0, CFG["vocab"], PROMPT).astype(np.int64)
    seqs = {rid: rng.integers(0, CFG["vocab"], 5 + i).astype(np.int64) for i, rid in enumerate("abcdef")}
    return main, seqs


def backend(sf, dev, start, end, head, tail, tag):
    return sf.CudaStageBackend(synthetic=sf.ModelShape(**CFG), device=dev, rope_theta=10000.0, max_ctx=256,
                               max_sessions=8, max_batch_tokens=64).load_layout("m", tag, start, end, head, tail)


def one_gpu_reference(sf, dev):
    """The whole model on one GPU, driven call for call as the pipeline drives its stages."""
    from stagefwd.pipeline import CudaCompute
    main, seqs = prompts()
    full = backend(sf, dev.index, 0, CFG["n_layers"] - 1, True, True, "full")
    comp = CudaCompute(full, CFG["hidden"], 64, dev)
    gen = full.generate_greedy("g", main.astype(np.uint32), STEPS).astype(np.int64).tolist()
    mb_tokens = []
    for mb in MBS:
        firsts = []
        for rid in mb:
            y = comp.forward([rid], [len(seqs[rid])], torch.from_numpy(seqs[rid]).to(dev), append=False)
            firsts.append(comp.sample(y[-1:]).clone())
        mb_tokens.append(torch.cat(firsts))
    stream = []
    for _ in range(MB_STEPS):
        for m, mb in enumerate(MBS):
            y = comp.forward(mb, [1] * len(mb), mb_tokens[m], append=True)
            mb_tokens[m] = comp.sample(y).clone()
        stream.append([t.cpu().tolist() for t in mb_tokens])
    full.close()
    return gen, stream


def worker(rank, world, port, q):
    import datetime
    import os
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        import torch.distributed as dist
        import stagefwd as sf
        from stagefwd.pipeline import CudaCompute, Pipeline, even_stage_split, make_groups
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120))
        ranks = make_groups(rank, world)
        start, end = even_stage_split(CFG["n_layers"], world)[rank]
        be = backend(sf, rank, start, end, ranks.is_head, ranks.is_tail, f"s{rank}")
        pipe = Pipeline(CudaCompute(be, CFG["hidden"], 64, dev), ranks, CFG["hidden"], dev)
        main, seqs = prompts()
        gen = pipe.generate("g", torch.from_numpy(main).to(dev), STEPS)
        tokens = []
        for mb in MBS:  # each sequence's prompt as its own pipeline step
            firsts = [pipe.step([rid], [len(seqs[rid])], torch.from_numpy(seqs[rid]).to(dev), append=False)
                      for rid in mb]
            tokens.append(torch.cat(firsts) if ranks.is_head else None)
        stream = []
        for _ in range(MB_STEPS):  # one step per call: the head's tokens are read after each
            tokens = pipe.decode_microbatched(MBS, tokens, 1)
            if ranks.is_head:
                stream.append([t.cpu().tolist() for t in tokens])
        torch.cuda.synchronize()
        out = {"rank": rank}
        if rank == 0:
            ref_gen, ref_stream = one_gpu_reference(sf, dev)
            out.update(gen=gen.cpu().tolist(), ref_gen=ref_gen, stream=stream, ref_stream=ref_stream)
        dist.barrier()
        be.close()
        dist.destroy_process_group()
        q.put(out)
    except Exception as e:  # reported to the test; the peer's next receive times out
        q.put({"rank": rank, "error": repr(e)})


def test_two_gpu_pipeline_matches_one_gpu():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two visible GPUs")
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(2):
            d = q.get(timeout=600)
            results[d["rank"]] = d
    finally:
        for p in procs:
            p.join(timeout=60)
        for p in procs:
            if p.is_alive():
                p.terminate()
                p.join(timeout=10)
    for r in (0, 1):
        assert "error" not in results[r], results[r]["error"]
    r0 = results[0]
    assert r0["gen"] == r0["ref_gen"]
    assert r0["stream"] == r0["ref_stream"]
