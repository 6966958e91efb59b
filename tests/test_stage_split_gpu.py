"""A layer range split over several stages computes the single stage's hidden states bit for bit.

Inside one stage the residual add after a layer's FFN runs in the prologue of the next layer's
q/k/v projection; at a stage boundary the stage closes with a separate residual add and the next
stage starts with a plain RMSNorm.  Both sides sum squares in one order and round every step alike,
so the pipeline's greedy stream equals the one-GPU stream exactly (the reference hands the f32
hidden state from stage to stage: crates/llama-stage-backend/src/lib.rs:1505-1562, :2308-2370).
Covered: prefill through the tensor-core GEMM (40 and 9 rows), one-token decode (GEMV, one token),
two sequences decoded in one call and a two-token append (GEMV, two tokens), at full width
(2560: more 256-element blocks than the GEMV's consumer warps) and at 512."""
import pytest

import stage_oracle as so

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

SHAPES = {
    "2560": dict(hidden=2560, n_heads=8, n_kv=4, head_dim=256, ffn=10240, vocab=8192, n_layers=4, seed=77),
    "512": dict(hidden=512, n_heads=4, n_kv=2, head_dim=128, ffn=1024, vocab=4096, n_layers=4, seed=78),
}
SPLITS = [[(0, 0), (1, 2), (3, 3)], [(0, 1), (2, 3)], [(0, 0), (1, 1), (2, 2), (3, 3)]]


@pytest.fixture(scope="module")
def sf():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import stagefwd
    return stagefwd


def stage(sf, shape, start, end, n_layers):
    return sf.CudaStageBackend(synthetic=shape, rope_theta=10000.0, max_ctx=256, max_sessions=4,
                               max_batch_tokens=64).load_layout("m", f"s{start}", start, end, start == 0,
                                                                end == n_layers - 1)


def chain(stages, hidden, ids, seqs, counts, append):
    x = None
    for i, s in enumerate(stages):
        out = torch.empty(ids.numel(), hidden, device=ids.device)
        if i == 0:
            s.forward_dev(seqs, counts, ids_dev=ids, out_dev=out, append=append)
        else:
            s.forward_dev(seqs, counts, in_dev=x, out_dev=out, append=append)
        x = out
    return x


@pytest.mark.parametrize("split", SPLITS, ids=["1-2-1", "2-2", "1-1-1-1"])
@pytest.mark.parametrize("width", list(SHAPES))
def test_split_stages_equal_one_stage_bitwise(sf, width, split):
    cfg = SHAPES[width]
    shape = sf.ModelShape(**cfg)
    L, H = cfg["n_layers"], cfg["hidden"]
    full = [stage(sf, shape, 0, L - 1, L)]
    parts = [stage(sf, shape, a, b, L) for a, b in split]
    dev = torch.device("cuda")

    def ids_of(tokens):
        return torch.tensor(tokens, dtype=torch.int32, device=dev)

    steps = [  # (request ids, tokens per sequence, token ids, append)
        (["a"], [40], so.synth_tokens(1, "a", 40, cfg["vocab"]), False),
        (["b"], [9], so.synth_tokens(2, "b", 9, cfg["vocab"]), False),
        (["a"], [1], [17], True),
        (["a"], [1], [4001], True),
        (["a", "b"], [1, 1], [5, 6], True),
        (["a"], [2], [7, 8], True),
        (["b", "a"], [3, 8], list(range(100, 111)), True),
    ]
    tok_dev = torch.empty(2, dtype=torch.int64, device=dev)
    score_dev = torch.empty(2, dtype=torch.float32, device=dev)
    for n, (seqs, counts, toks, append) in enumerate(steps):
        ids = ids_of([int(t) for t in toks])
        y_full = chain(full, H, ids, seqs, counts, append)
        y_split = chain(parts, H, ids, seqs, counts, append)
        torch.cuda.synchronize()
        diff = (y_full - y_split).abs().max().item()
        assert torch.equal(y_full, y_split), f"step {n}: split {split} differs from one stage by {diff:.3e}"
        last = torch.tensor([sum(counts[: i + 1]) - 1 for i in range(len(counts))], device=dev)
        t_full, t_split = tok_dev[: len(counts)].clone(), None
        full[0].sample_dev(y_full.index_select(0, last), t_full, score_dev[: len(counts)])
        t_split = torch.empty_like(t_full)
        parts[-1].sample_dev(y_split.index_select(0, last), t_split, score_dev[: len(counts)])
        torch.cuda.synchronize()
        assert torch.equal(t_full, t_split)
    for s in full + parts:
        s.close()
