"""GPU: stages loaded from GGUF files.  A stage opened straight from a GGUF file
(sfc_stage_open_gguf), one packed from the same file through the shard manifest bundle
(sfc_gguf_write_bundle + sfc_pack_stage, the reference's gguf.rs:636-751 and lib.rs:3512-3613
route) and one loaded from the oracle's pack of the same tensors hold the same bytes, so their
outputs are bit-identical; they also match the oracle (f32 cache, 1e-3)."""
import numpy as np
import pytest

import stage_oracle as so
from gguf_util import STR, U32, gguf_bytes, write_stage_gguf
from gpu_util import assert_close

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def sf():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import stagefwd
    return stagefwd


SPEC = dict(hidden=512, n_heads=4, n_kv=2, head_dim=128, ffn=1024, vocab=1000, n_layers=2, seed=33)
KW = dict(rope_theta=10000.0, kv_f32=True, max_ctx=256, max_sessions=2)


def model_gguf(tmp_path):
    spec = so.ModelSpec(**SPEC)
    tensors = so.synth_stage(spec, 0, 1, True, True)
    meta = [("general.architecture", STR, "gemma4"), ("general.name", STR, "synthetic-gemma"),
            ("gemma4.block_count", U32, 2)]
    return spec, tensors, write_stage_gguf(tmp_path / "model.gguf", tensors, meta)


def test_gguf_stage_matches_pack_stage(sf, tmp_path):
    from stagefwd.gguf import GgufFile, pack_stage
    spec, tensors, gg = model_gguf(tmp_path)
    idx = so.write_pack(tmp_path / "oracle_pack", "stage-0", "full", 0, tensors)
    f = GgufFile.parse_file(gg)
    f.write_bundle(f.suggest_even_stage_split(1), tmp_path / "bundle")
    idx2 = pack_stage(tmp_path / "bundle", gg, 0, tmp_path / "packed", include_optional=True)
    stages = [sf.CudaStageBackend(idx, **KW), sf.CudaStageBackend(gguf_path=gg, **KW),
              sf.CudaStageBackend(idx2, **KW)]
    stages = [s.load_layout("synthetic-gemma", "full", 0, 1, True, True) for s in stages]
    prompt = so.synth_tokens(6, "p", 11, spec.vocab)
    hs = [s.begin_token_ids("r", prompt) for s in stages]
    assert np.array_equal(hs[0], hs[1]) and np.array_equal(hs[0], hs[2])
    o = so.OracleStage(so.load_pack(idx2), so.Layout("m", "s", 0, 1, True, True), rope_theta=10000.0,
                       kv_fp16=False)
    assert_close(hs[1], o.begin_token_ids("r", prompt), what="GGUF stage vs oracle")
    toks = [s.sample_tail(h[-1])[0] for s, h in zip(stages, hs)]
    assert toks[0] == toks[1] == toks[2] == o.sample_tail(o.begin_token_ids("q", prompt)[-1])[0]
    for step in range(3):  # decode steps on the kept KV
        hs = [s.begin_token_ids("r", [toks[0]]) for s in stages]
        assert np.array_equal(hs[0], hs[1]) and np.array_equal(hs[0], hs[2]), f"step {step}"
        toks = [s.sample_tail(h[-1])[0] for s, h in zip(stages, hs)]
        assert toks[0] == toks[1] == toks[2]


def test_gguf_two_stage_split(sf, tmp_path):
    """Head (layer 0, embedding) and tail (layer 1, output norm, tied logits from token_embd: the
    file has no output.weight) opened from one GGUF file, against the whole model in one stage."""
    spec, _, gg = model_gguf(tmp_path)
    full = sf.CudaStageBackend(gguf_path=gg, **KW).load_layout("m", "full", 0, 1, True, True)
    head = sf.CudaStageBackend(gguf_path=gg, **KW).load_layout("m", "head", 0, 0, True, False)
    tail = sf.CudaStageBackend(gguf_path=gg, **KW).load_layout("m", "tail", 1, 1, False, True)
    assert head.info.n_layers == 1 and tail.info.n_layers == 1 and tail.info.vocab == spec.vocab
    prompt = so.synth_tokens(8, "p", 9, spec.vocab)
    ref = full.begin_token_ids("r", prompt)
    out = tail.continue_forward("r", head.begin_token_ids("r", prompt))
    assert_close(out, ref, what="two-stage GGUF vs one stage")
    assert tail.sample_tail(out[-1])[0] == full.sample_tail(ref[-1])[0]


def test_gguf_stage_rejects_short_tensor_slot(sf, tmp_path):
    """A tensor whose dims imply more bytes than lie before the next tensor is refused on the host."""
    spec, tensors, _ = model_gguf(tmp_path)
    items = list(tensors.items())
    # all tensors back to back in one section, but the first Q4_K matrix's slot cut to 100 bytes
    section, recs, off = b"", [], 0
    for k, (name, (t, dims, arr)) in enumerate(items):
        b = np.ascontiguousarray(arr).view(np.uint8).tobytes()
        recs.append((name, dims, t, off))
        section += b
        off += len(b)
    q = next(i for i, (_, (t, _, _)) in enumerate(items) if t == 12)
    name, dims, t, o = recs[q]
    recs = [r if i != q + 1 else (r[0], r[1], r[2], o + 100) for i, r in enumerate(recs)]
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(gguf_bytes([], recs, data=section))
    with pytest.raises(sf.StageError, match="implied by its dims"):
        sf.CudaStageBackend(gguf_path=bad, **KW).load_layout("m", "s", 0, 1, True, True)
