"""CPU, world_size 2 and 3 over gloo: the pipeline driver (stagefwd/pipeline.py) splits layers
like gguf.rs:307-329, hands hidden rows rank to rank, returns tail tokens to the head, and
reproduces the single-process result.  The per-rank compute here is the CPU oracle."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import stage_oracle as so

# seed 33: every sequence's greedy token changes from step to step, so a pipeline that returned
# an earlier step's samples would be caught
SPEC = dict(hidden=256, n_heads=4, n_kv=2, head_dim=64, ffn=512, vocab=200, n_layers=5, seed=33)
# decode_microbatched calls of 1, 2 and 1 steps: the head's tokens are checked after each call
CALL_STEPS = (1, 2, 1)


class OracleCompute:
    def __init__(self, stage):
        self.s = stage

    def forward(self, request_ids, seq_tokens, x, append=True):
        outs, row = [], 0
        for rid, n in zip(request_ids, seq_tokens):
            part = x[row:row + n]
            if self.s.layout.is_head:
                o = self.s.begin_token_ids(rid, part.numpy().astype(np.uint32), append=append)
            else:
                o = self.s.continue_forward(rid, part.numpy(), append=append)
            outs.append(torch.from_numpy(o))
            row += n
        return torch.cat(outs)

    def sample(self, hidden):
        return torch.tensor([self.s.sample_tail(h.numpy())[0] for h in hidden], dtype=torch.int64)


def make_stage(start, end, head, tail):
    spec = so.ModelSpec(**SPEC)
    return so.OracleStage(so.synth_stage(spec, start, end, head, tail),
                          so.Layout("m", f"s{start}", start, end, head, tail), rope_theta=10000.0)


def run_pipeline(rank, world, port, q):
    os.environ["ORACLE_THREADS"] = "1"
    from stagefwd.pipeline import Pipeline, even_stage_split, make_groups
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    ranks = make_groups(rank, world)
    start, end = even_stage_split(SPEC["n_layers"], world)[rank]
    pipe = Pipeline(OracleCompute(make_stage(start, end, rank == 0, rank == world - 1)), ranks, SPEC["hidden"],
                    torch.device("cpu"))
    prompt = torch.from_numpy(so.synth_tokens(2, "p", 7, SPEC["vocab"]).astype(np.int64))
    gen = pipe.generate("g", prompt, 6)
    mbs = [["a", "b"], ["c", "d"]]
    for i, rid in enumerate(["a", "b", "c", "d"]):  # short prefills so every session has context
        pipe.step([rid], [3], torch.tensor([i + 1, i + 2, i + 3], dtype=torch.int64), append=False)
    toks = [torch.tensor([5, 6], dtype=torch.int64), torch.tensor([7, 8], dtype=torch.int64)]
    after = []
    for n in CALL_STEPS:
        toks = pipe.decode_microbatched(mbs, toks, n)
        after.append([t.tolist() for t in toks] if rank == 0 else None)
    if rank == 0:
        q.put((gen.tolist(), after))
    dist.barrier()
    dist.destroy_process_group()


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def single_process_reference():
    st = make_stage(0, SPEC["n_layers"] - 1, True, True)
    prompt = so.synth_tokens(2, "p", 7, SPEC["vocab"])
    h = st.begin_token_ids("g", prompt)
    gen = []
    for _ in range(6):
        t = st.sample_tail(h[-1])[0]
        gen.append(t)
        h = st.begin_token_ids("g", [t])
    for i, rid in enumerate(["a", "b", "c", "d"]):
        st.begin_token_ids(rid, [i + 1, i + 2, i + 3])
    toks = {"a": 5, "b": 6, "c": 7, "d": 8}
    after = []
    for n in CALL_STEPS:
        for _ in range(n):
            for rid in ["a", "b", "c", "d"]:
                toks[rid] = st.sample_tail(st.begin_token_ids(rid, [toks[rid]])[-1])[0]
        after.append([[toks["a"], toks["b"]], [toks["c"], toks["d"]]])
    return gen, after


def test_even_stage_split_matches_reference_rule():
    from stagefwd.pipeline import even_stage_split
    assert even_stage_split(42, 2) == [(0, 20), (21, 41)]
    assert even_stage_split(42, 4) == [(0, 10), (11, 21), (22, 31), (32, 41)]
    assert [e - s + 1 for s, e in even_stage_split(42, 8)] == [6, 6, 5, 5, 5, 5, 5, 5]
    with pytest.raises(ValueError):
        even_stage_split(3, 4)


def test_balanced_split_counts_the_tail_logits():
    from stagefwd.pipeline import balanced_stage_split, even_stage_split

    def cost(split, tc):
        return max((e - s + 1) + (tc if i == len(split) - 1 else 0) for i, (s, e) in enumerate(split))

    for n in (1, 2, 3, 4, 8):
        assert balanced_stage_split(42, n, 0.0) == even_stage_split(42, n)
        for tc in (0.5, 2.0, 4.0, 12.0):
            sp = balanced_stage_split(42, n, tc)
            assert sp[0][0] == 0 and sp[-1][1] == 41 and all(sp[i][1] + 1 == sp[i + 1][0] for i in range(n - 1))
            assert all(e >= s for s, e in sp)
            assert cost(sp, tc) <= cost(even_stage_split(42, n), tc)
    assert [e - s + 1 for s, e in balanced_stage_split(42, 8, 2.0)] == [6, 6, 6, 5, 5, 5, 5, 4]


@pytest.mark.parametrize("world", [2, 3])
def test_pipeline_matches_single_process(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=run_pipeline, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    import queue
    import time
    got, t0 = None, time.time()
    while got is None and time.time() - t0 < 240:
        try:
            got = q.get(timeout=2)
        except queue.Empty:
            if any(p.exitcode not in (None, 0) for p in procs):
                break
    for p in procs:
        if got is None:
            p.kill()
    assert got is not None, [p.exitcode for p in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = single_process_reference()
    assert got[0] == ref[0]
    assert got[1] == ref[1]
    # the sampled tokens move from call to call (the check above would see a stale step)
    assert ref[1][0] != ref[1][1] and ref[1][1] != ref[1][2]
