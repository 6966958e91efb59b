"""Per-layer embeddings (PLE) on the GPU against the oracle's restatement (compute_ple_inputs,
real_forward.rs:1157-1299; the per-layer block, :1753-1778): full-width layers (d_model 2560, 8q/4kv x
256, ffn 10240, Q4_K_M) with ple_dim 256, as one stage and as a head/tail split whose per-layer inputs
travel in the prompt aux section of the hand-off payload.  f32 cache, 1e-3 relative bar."""
import numpy as np
import pytest

import stage_oracle as so
from gpu_util import assert_close

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

SPEC = dict(hidden=2560, n_heads=8, n_kv=4, head_dim=256, ffn=10240, vocab=4096, n_layers=4, seed=0x91E,
            ple_dim=256)


@pytest.fixture(scope="module")
def sf():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import stagefwd
    return stagefwd


@pytest.fixture(scope="module")
def packs(tmp_path_factory):
    spec = so.ModelSpec(**SPEC)
    d = tmp_path_factory.mktemp("ple")
    out = {}
    for name, (a, b, head, tail) in {"full": (0, 3, True, True), "head": (0, 1, True, False),
                                     "tail": (2, 3, False, True)}.items():
        tensors = so.synth_stage(spec, a, b, head, tail)
        out[name] = (so.write_pack(d / name, f"stage-{name}", name, 0, tensors), tensors, (a, b, head, tail))
    return spec, out


def gpu(sf, pack):
    idx, _, (a, b, head, tail) = pack
    return sf.CudaStageBackend(idx, rope_theta=10000.0, kv_f32=True, max_ctx=128, max_sessions=2).load_layout(
        "synthetic-gemma", f"s{a}", a, b, head, tail)


def oracle(pack):
    _, tensors, (a, b, head, tail) = pack
    return so.OracleStage(tensors, so.Layout("synthetic-gemma", f"s{a}", a, b, head, tail), rope_theta=10000.0,
                          kv_fp16=False)


def test_ple_single_stage_prefill_and_decode(sf, packs):
    spec, p = packs
    g, o = gpu(sf, p["full"]), oracle(p["full"])
    prompt = so.synth_tokens(5, "ple.prompt", 20, spec.vocab)
    assert_close(g.begin_token_ids("r", prompt), o.begin_token_ids("r", prompt), what="PLE prefill")
    h_g, h_o = g.begin_token_ids("r", [7]), o.begin_token_ids("r", [7], append=True)
    for step in range(4):
        assert_close(h_g, h_o, what=f"PLE decode step {step}")
        t_g, t_o = g.sample_tail(h_g)[0], o.sample_tail(h_o[-1])[0]
        assert t_g == t_o
        h_g, h_o = g.begin_token_ids("r", [t_g]), o.begin_token_ids("r", [t_o], append=True)
    g.close()


def test_ple_head_tail_split_through_the_aux_section(sf, packs):
    spec, p = packs
    gh, gt = gpu(sf, p["head"]), gpu(sf, p["tail"])
    oh, ot = oracle(p["head"]), oracle(p["tail"])
    prompt = so.synth_tokens(6, "ple.split", 17, spec.vocab)
    payload = gh.begin_token_ids_bytes("r", prompt)
    hidden, aux, framed = sf.stage_tensor_byte_sections(payload)
    assert framed and aux is not None
    ple_g, hashes = so.decode_prompt_aux(aux)
    h_o = oh.begin_token_ids("r", prompt)
    assert ple_g.shape == (17, SPEC["n_layers"], SPEC["ple_dim"])
    assert hashes == so.prefix_hashes(prompt)
    assert_close(ple_g, oh.last_ple, what="per-layer inputs (compute_ple_inputs)")
    assert_close(np.frombuffer(hidden, np.float32).reshape(17, -1), h_o, what="head rows")
    out = gt.continue_forward_bytes("r", payload, SPEC["hidden"])
    rows, aux2, _ = sf.stage_tensor_byte_sections(out)
    assert aux2 == aux  # carried through unchanged
    t_o = ot.continue_forward("r", h_o, ple_all=oh.last_ple)
    assert_close(np.frombuffer(rows, np.float32).reshape(17, -1), t_o, what="tail rows")
    tok_g, tok_o = gt.sample_tail_bytes(out, SPEC["hidden"])[0], ot.sample_tail(t_o[-1])[0]
    assert tok_g == tok_o
    for step in range(3):  # decode: one token per step, its per-layer inputs in the aux section
        payload = gh.begin_token_ids_bytes("r", [tok_g])
        h_o = oh.begin_token_ids("r", [tok_o], append=True)
        out = gt.continue_forward_bytes("r", payload, SPEC["hidden"])
        t_o = ot.continue_forward("r", h_o, append=True, ple_all=oh.last_ple)
        rows = np.frombuffer(sf.stage_tensor_byte_sections(out)[0], np.float32).reshape(1, -1)
        assert_close(rows, t_o, what=f"split decode step {step}")
        tok_g, tok_o = gt.sample_tail_bytes(out, SPEC["hidden"])[0], ot.sample_tail(t_o[-1])[0]
        assert tok_g == tok_o
    # a PLE stage fed rows without the per-layer inputs refuses them
    with pytest.raises(sf.StageError, match="prompt aux"):
        gt.continue_forward("x", np.zeros((1, SPEC["hidden"]), np.float32))
    gh.close()
    gt.close()
