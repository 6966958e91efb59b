"""CPU: the oracle's per-layer embedding (PLE) path and the stage aux section
(crates/stage-forward-lab/src/real_forward.rs:1157-1299 compute_ple_inputs, :1753-1778 the per-layer
block, :1852-1990 the "rsa1" / "rpl1" aux codec, :319-333 prefix hashes).  The B200 stage does not
run PLE yet; this pins the oracle side it will be checked against."""
import struct

import numpy as np
import pytest

import stage_oracle as so

SPEC = dict(hidden=256, n_heads=2, n_kv=1, head_dim=128, ffn=512, vocab=300, n_layers=3, seed=77, ple_dim=64)


def stage(spec, start, end, head, tail, drop_ple_layers=False):
    t = so.synth_stage(spec, start, end, head, tail)
    if drop_ple_layers:
        t = {k: v for k, v in t.items() if not k.endswith((".inp_gate.weight", ".proj.weight"))}
    return so.OracleStage(t, so.Layout("m", f"s{start}", start, end, head, tail), rope_theta=10000.0)


def test_rms_norm_chunked_matches_per_chunk_norm():
    """real_math.rs:2929-2944: a chunked norm is the norm of each chunk."""
    w = np.array([1.0, 0.5, 1.5], np.float32)
    x = np.array([1, 2, 3, 4, 5, 6, -1, 0, 1], np.float32)
    got = so.rms_norm(x.reshape(3, 3), w, 1e-6).reshape(-1)
    for c in range(3):
        ch = x[3 * c: 3 * c + 3].astype(np.float64)
        want = ch / np.sqrt(np.mean(ch * ch) + 1e-6) * w
        np.testing.assert_allclose(got[3 * c: 3 * c + 3], want, rtol=1e-6)


def test_ple_inputs_shape_and_effect():
    spec = so.ModelSpec(**SPEC)
    st = stage(spec, 0, 2, True, True)
    assert (st.ple_dim, st.ple_layers) == (64, 3)
    ids = so.synth_tokens(5, "p", 7, spec.vocab)
    out = st.begin_token_ids("r", ids)
    assert st.last_ple.shape == (7, 3, 64) and np.isfinite(st.last_ple).all()
    # the per-layer inputs are RMS-normed projections plus sqrt(64)-scaled embedding rows, times 2^-1/2
    no_ple = stage(spec, 0, 2, True, True, drop_ple_layers=True).begin_token_ids("r", ids)
    assert np.abs(out - no_ple).max() > 1e-2 * np.abs(no_ple).max()


def test_ple_incremental_decode_equals_full_rerun():
    """real_forward.rs:3129 with PLE: the decode step's PLE input comes from its own token."""
    spec = so.ModelSpec(**SPEC)
    ids = so.synth_tokens(6, "p", 10, spec.vocab)
    full = stage(spec, 0, 2, True, True).begin_token_ids("f", ids)
    inc = stage(spec, 0, 2, True, True)
    inc.begin_token_ids("i", ids[:6])
    rows = [inc.begin_token_ids("i", [t]) for t in ids[6:]]
    np.testing.assert_allclose(np.concatenate(rows), full[6:], rtol=0, atol=2e-5 * np.abs(full).max())


def test_ple_two_stages_through_the_aux_section():
    """The head computes every layer's inputs and sends them in the "rsa1" aux section; the tail
    uses its layers' slices (run_stage_layers indexes them by global layer, :1992-2052)."""
    spec = so.ModelSpec(**SPEC)
    ids = so.synth_tokens(7, "p", 8, spec.vocab)
    whole = stage(spec, 0, 2, True, True).begin_token_ids("r", ids)
    head, tail = stage(spec, 0, 1, True, False), stage(spec, 2, 2, False, True)
    h = head.begin_token_ids("r", ids)
    aux = so.encode_prompt_aux(head.last_ple, 64, so.prefix_hashes(ids))
    ple, hashes = so.decode_prompt_aux(aux)
    assert hashes == so.prefix_hashes(ids) and ple.shape == (8, 3, 64)
    out = tail.continue_forward("r", h, ple_all=ple)
    np.testing.assert_allclose(out, whole, rtol=0, atol=1e-6 * np.abs(whole).max())


def fnv1a64(data: bytes) -> int:
    h = 0xCBF29CE484222325
    for b in data:
        h = ((h ^ b) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def test_prefix_hashes_are_running_fnv1a():
    assert fnv1a64(b"a") == 0xAF63DC4C8601EC8C  # the published FNV-1a 64 test vector
    ids = [1, 70000, 3]
    le = b"".join(struct.pack("<I", t) for t in ids)
    assert so.prefix_hashes(ids) == [fnv1a64(le[:4]), fnv1a64(le[:8]), fnv1a64(le)]


def test_prompt_aux_codec():
    ple = np.arange(2 * 3 * 4, dtype=np.float32).reshape(2, 3, 4)
    b = so.encode_prompt_aux(ple, 4, [5, 6])
    assert b[:4] == b"rsa1" and len(b) == 20 + ple.nbytes + 16
    got, hashes = so.decode_prompt_aux(b)
    assert np.array_equal(got, ple) and hashes == [5, 6]
    assert so.encode_prompt_aux(None, 0, []) is None
    only_hashes = so.encode_prompt_aux(None, 0, [9])
    assert so.decode_prompt_aux(only_hashes)[1] == [9] and so.decode_prompt_aux(only_hashes)[0].size == 0
    with pytest.raises(ValueError, match="Invalid prompt-aux byte length"):
        so.decode_prompt_aux(b[:-1])
    legacy = b"rpl1" + struct.pack("<III", 2, 3, 4) + ple.tobytes()
    got, hashes = so.decode_prompt_aux(legacy)
    assert np.array_equal(got, ple) and hashes == []
    with pytest.raises(ValueError, match="Invalid prompt-aux payload"):
        so.decode_prompt_aux(b"xxxx" + bytes(16))
