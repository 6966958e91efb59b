"""CPU: pin the oracle against the reference's golden vectors and known answers.

  * dequant bit-exact vs gguf-py numpy fixtures (tests/golden/dequant_golden.npz) and vs the
    reference's own ggml-quants.c compiled from source (oracle/_ref);
  * known-answer unit tests of quants.rs / real_math.rs (tests/golden/known_answers.json);
  * the oracle's stage semantics: incremental decode == full rerun (real_forward.rs:3129).
"""
import ctypes
import json
from pathlib import Path

import numpy as np
import pytest

import stage_oracle as so

ROOT = Path(__file__).resolve().parent.parent
KA = json.loads((ROOT / "tests/golden/known_answers.json").read_text())


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def constructed_q4k(d=1.0):
    row = np.zeros(144, np.uint8)
    row[0:2] = np.array([d], np.float16).view(np.uint8)
    row[4:8] = 1
    row[16:] = 0x11
    return row


def constructed_q6k(d=1.0):
    row = np.zeros(210, np.uint8)
    row[192:208] = 1
    row[208:210] = np.array([d], np.float16).view(np.uint8)
    return row


@pytest.mark.parametrize("name,t", [("q4k", so.Q4_K), ("q6k", so.Q6_K)])
def test_dequant_matches_gguf_py_bit_exact(golden_dir, name, t):
    g = np.load(golden_dir / "dequant_golden.npz")
    raw, exp = g[f"{name}_raw"], g[f"{name}_out"]
    got = so.dequantize_rows(t, raw.reshape(-1), raw.shape[0], 256)
    assert np.array_equal(_bits(got), _bits(exp))


def test_q5k_rust_layout_quirk(golden_dir):
    """quants.rs:145-146 interleaves the low/high nibble outputs of a Q5_K group (j + 2l, j + 2l + 1),
    unlike ggml/gguf-py (l, l + 32). The oracle follows the Rust; Q5_K is not on the hot path."""
    g = np.load(golden_dir / "dequant_golden.npz")
    raw, exp = g["q5k_raw"], g["q5k_out"]
    got = so.dequantize_rows(so.Q5_K, raw.reshape(-1), raw.shape[0], 256).reshape(-1, 4, 64)
    exp = exp.reshape(-1, 4, 2, 32)
    rust_order = np.stack([exp[:, :, 0, :], exp[:, :, 1, :]], axis=-1).reshape(-1, 4, 64)
    assert np.array_equal(_bits(got), _bits(rust_order))


@pytest.mark.parametrize("name,fn,t", [("q4k", "dequantize_row_q4_K", so.Q4_K), ("q6k", "dequantize_row_q6_K", so.Q6_K)])
def test_dequant_matches_reference_ggml_build(golden_dir, name, fn, t):
    path = ROOT / "oracle/_ref/libggml_quants_ref.so"
    if not path.exists():
        pytest.skip("oracle/_ref not built (make -C oracle with the reference tree present)")
    ref = ctypes.CDLL(str(path))
    f = getattr(ref, fn)
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
    rng = np.random.default_rng(7)
    bs = 144 if t == so.Q4_K else 210
    raw = rng.integers(0, 256, size=(300, bs), dtype=np.uint8)
    off = [0, 2] if t == so.Q4_K else [208]
    for o in off:
        raw[:, o:o + 2] = np.abs(rng.normal(0, 0.02, (300, 1))).astype(np.float16).view(np.uint8).reshape(300, 2)
    raw = np.ascontiguousarray(raw)
    out = np.empty(300 * 256, np.float32)
    f(raw.ctypes.data, out.ctypes.data, out.size)
    got = so.dequantize_rows(t, raw.reshape(-1), 300, 256).reshape(-1)
    assert np.array_equal(_bits(got), _bits(out))
    g = np.load(golden_dir / "dequant_golden.npz")
    raw2 = np.ascontiguousarray(g[f"{name}_raw"])
    out2 = np.empty(raw2.shape[0] * 256, np.float32)
    f(raw2.ctypes.data, out2.ctypes.data, out2.size)
    assert np.array_equal(_bits(out2), _bits(g[f"{name}_out"].reshape(-1)))


def test_zero_blocks():
    for t, bs in ((so.Q4_K, 144), (so.Q6_K, 210)):
        assert not so.dequantize_rows(t, np.zeros(bs, np.uint8), 1, 256).any()


def test_known_answer_rows():
    ka = KA["q4k_constructed_row"]
    for x, e in zip(ka["inputs"], ka["expected"]):
        assert so.matmul(so.Q4_K, constructed_q4k(), 1, 256, np.full((1, 256), x, np.float32))[0, 0] == e
    ka = KA["q6k_constructed_row"]
    for x, e in zip(ka["inputs"], ka["expected"]):
        assert so.matmul(so.Q6_K, constructed_q6k(), 1, 256, np.full((1, 256), x, np.float32))[0, 0] == e


def test_known_answer_top_k():
    ka = KA["q4k_top_k_four_rows"]
    raw = np.concatenate([constructed_q4k(d) for d in (1.0, 2.0, 3.0, 4.0)])
    am, _, top, _ = so.logits_top_k(so.Q4_K, raw, 4, 256, np.ones(256, np.float32), 2, cap=0.0)
    assert am == ka["argmax"] and top == [tuple(x) for x in ka["top"]]
    ka = KA["q6k_top_k_pair"]
    raw = np.concatenate([constructed_q6k(d) for d in (1.0, 2.0)])
    am, _, top, _ = so.logits_top_k(so.Q6_K, raw, 2, 256, np.ones(256, np.float32), 2, cap=0.0)
    assert am == ka["argmax"] and top == [tuple(x) for x in ka["top"]]
    ka = KA["f32_top_k"]
    raw = np.array(ka["rows"], np.float32).view(np.uint8).reshape(-1)
    am, sc, top, _ = so.logits_top_k(so.F32, raw, 3, 2, np.array(ka["input"], np.float32), ka["k"], cap=0.0)
    assert (am, sc) == (ka["argmax"], ka["argmax_score"]) and top == [tuple(x) for x in ka["top"]]


def test_argmax_ties_go_to_lowest_index():
    raw = np.array([[1.0], [3.0], [3.0], [2.0]], np.float32).view(np.uint8).reshape(-1)
    am, _, _, _ = so.logits_top_k(so.F32, raw, 4, 1, np.ones(1, np.float32), 0, cap=30.0)
    assert am == 1


def test_rms_norm_and_attention_known_answers():
    ka = KA["rms_norm_identity"]
    x = np.array(ka["x"], np.float32)
    out = so.rms_norm(x, np.array(ka["w"], np.float32))
    scale = 1.0 / np.sqrt((9.0 + 16.0) / 2.0 + 1e-6)
    assert np.allclose(out, x * scale, atol=ka["tol"])
    ka = KA["gqa_limit_causality"]
    q, k, v = (np.array(ka[n], np.float32) for n in ("q", "k", "v"))
    assert np.array_equal(so.gqa_attention(q, k, v, 1, 1, 2, limit=1), np.array(ka["limit1_expected"], np.float32))
    both = so.gqa_attention(q, k, v, 1, 1, 2, limit=2)
    assert 10.0 < both[0] < 100.0 and 1.0 < both[1] < 2.0
    ka = KA["gqa_window"]
    q, k, v = (np.array(ka[n], np.float32) for n in ("q", "k", "v"))
    assert np.array_equal(so.gqa_attention(q, k, v, 1, 1, 2, window=1), np.array(ka["window1_expected"], np.float32))
    assert np.array_equal(so.gqa_attention(q, k, v, 1, 1, 2), np.array(ka["full_expected"], np.float32))


def test_proportional_rope_known_answer():
    ka = KA["proportional_rope"]
    x = np.array(ka["x"], np.float32)
    out = so.rope(x, 1, 8, None, ka["position"], ka["theta"], rotary_dim=ka["rotary_dim"], proportional=True)
    for i, v in ka["unchanged"].items():
        assert out[int(i)] == v
    assert abs(out[0] - (1 * np.cos(1.0) - 5 * np.sin(1.0))) < 1e-5
    assert abs(out[1] - (2 * np.cos(0.1) - 6 * np.sin(0.1))) < 1e-5
    # norm preserved (real_math.rs:2994-3005)
    y = so.rope(np.ones(8, np.float32), 1, 8, np.ones(4, np.float32), 3, 10000.0)
    assert abs(np.linalg.norm(y) - np.sqrt(8)) < 1e-4


def test_synthetic_generator_is_deterministic_and_distributed():
    key = so.tensor_key(123, "blk.0.attn_q.weight")
    a = so.synth_tensor(so.Q4_K, key, 64, 2560, 0.02)
    b = so.synth_tensor(so.Q4_K, key, 64, 2560, 0.02)
    assert np.array_equal(a, b)
    blocks = a.reshape(-1, 144)
    d = blocks[:, 0:2].copy().view(np.float16).astype(np.float32).ravel()
    assert (d >= 0).all() and 0.01 < d.mean() < 0.02  # E|N(0, .02)| = 0.016
    q = blocks[:, 16:]
    nib = np.concatenate([q & 15, q >> 4]).ravel()
    assert abs(nib.mean() - 7.5) < 0.1
    n = so.synth_normal_f32(1, "x", 200000)
    assert abs(n.mean()) < 0.02 and abs(n.std() - 1.0) < 0.02


def _tiny_spec(**kw):
    base = dict(hidden=256, n_heads=4, n_kv=2, head_dim=64, ffn=512, vocab=300, n_layers=4, seed=11)
    base.update(kw)
    return so.ModelSpec(**base)


def test_oracle_incremental_decode_equals_full_rerun():
    """real_forward.rs:3129 cached_decode_step_matches_fresh_full_rerun, on the oracle."""
    spec = _tiny_spec()
    head = so.OracleStage(so.synth_stage(spec, 0, 1, True, False), so.Layout("m", "s0", 0, 1, True, False), 1e4)
    tail = so.OracleStage(so.synth_stage(spec, 2, 3, False, True), so.Layout("m", "s1", 2, 3, False, True), 1e4)
    prompt = so.synth_tokens(5, "prompt", 9, spec.vocab)
    h = head.begin_token_ids("r", prompt)
    t = tail.continue_forward("r", h)
    tok = tail.sample_tail(t[-1])[0]
    h2 = head.begin_token_ids("r", [tok])
    t2 = tail.continue_forward("r", h2)
    cached = tail.sample_tail(t2[-1])[0]
    head_f = so.OracleStage(head.t, head.layout, 1e4)
    tail_f = so.OracleStage(tail.t, tail.layout, 1e4)
    hf = head_f.begin_token_ids("f", np.append(prompt, tok))
    tf = tail_f.continue_forward("f", hf)
    assert np.array_equal(tf[-1], t2[-1])
    assert tail_f.sample_tail(tf[-1])[0] == cached


def test_pack_roundtrip_and_validation(tmp_path):
    spec = _tiny_spec(n_layers=2)
    tensors = so.synth_stage(spec, 0, 1, True, True)
    idx = so.write_pack(tmp_path, "stage-0", "head", 0, tensors)
    loaded = so.load_pack(idx)
    assert list(loaded) == list(tensors)
    for name in tensors:
        assert np.array_equal(np.asarray(loaded[name][2]), tensors[name][2])
    # truncated pack -> size mismatch (lib.rs:3660-3667)
    pack = idx.with_name("stage-0-required.pack")
    data = pack.read_bytes()
    pack.write_bytes(data[:-1])
    with pytest.raises(ValueError):
        so.load_pack(idx)
    pack.write_bytes(data)
    # bad offsets (lib.rs:3729-3750)
    j = json.loads(idx.read_text())
    j["tensors"][1]["pack_offset"] += 4
    idx.write_text(json.dumps(j))
    with pytest.raises(ValueError):
        so.load_pack(idx)
