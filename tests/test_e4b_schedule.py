"""CPU: the oracle's Gemma-4 e4b attention schedule table and split rule
(layer_attention_config_for_layout / validate_stage_split_constraints,
crates/stage-forward-lab/src/real_forward.rs:1407-1481)."""
import numpy as np
import pytest

import stage_oracle as so


def fake_stage(model_id, start, end, hidden=2560, head_dim=256):
    t = {}
    for i in range(start, end + 1):
        t[f"blk.{i}.attn_q.weight"] = (12, [hidden, 8 * head_dim], None)
        t[f"blk.{i}.attn_k.weight"] = (12, [hidden, 4 * head_dim], None)
        t[f"blk.{i}.attn_q_norm.weight"] = (0, [head_dim], None)
    return so.OracleStage(t, so.Layout(model_id, "s", start, end, True, True), rope_theta=10000.0)


def test_e4b_schedule_table():
    st = fake_stage("gemma-4-e4b-it", 20, 35)
    assert st.rope_freqs is not None and st.rope_freqs.size == 0  # RoPE on, packed freqs unused
    assert st._attention_config(20) == (10000.0, 256, False, None, 512)
    assert st._attention_config(23) == (1000000.0, 64, True, None, 0)
    assert st._attention_config(24) == (10000.0, 256, False, 22, 512)
    assert st._attention_config(29) == (1000000.0, 64, True, 23, 0)
    assert st._attention_config(35) == (1000000.0, 64, True, 23, 0)
    # other models, other widths or head sizes: the generic schedule
    for s in (fake_stage("gemma-3-27b", 20, 35), fake_stage("gemma-4-e4b", 20, 35, hidden=2048),
              fake_stage("gemma-4-e4b", 20, 35, head_dim=128)):
        assert all(s._attention_config(i) == (10000.0, s.head_dim, False, None, 0) for i in range(20, 36))


def test_e4b_split_rule():
    with pytest.raises(ValueError, match="layer 24 requires shared KV from layer 22 outside this stage"):
        fake_stage("gemma-4-e4b", 24, 41)
    t = {}
    for i in (22, 29):  # a stage whose layout spans 22..29 but whose layer 23 lies elsewhere is fine
        t[f"blk.{i}.attn_q.weight"] = (12, [2560, 2048], None)
        t[f"blk.{i}.attn_k.weight"] = (12, [2560, 1024], None)
    so.OracleStage(t, so.Layout("gemma-4-e4b", "s", 22, 29, True, True))
    with pytest.raises(ValueError, match="layer 29 requires shared KV from layer 23 outside this stage"):
        so.OracleStage({k: v for k, v in t.items() if k.startswith("blk.29")},
                       so.Layout("gemma-4-e4b", "s", 24, 29, True, True))


def gqa_reference(q, kc, vc, n_heads, n_kv, hd, window, limit):
    """gqa_attention_seq_with_window_and_limit (real_math.rs:2697-2744) in float64."""
    seq = min(limit, len(kc))
    w0 = max(0, seq - window) if window else 0
    out = np.zeros(n_heads * hd)
    g = n_heads // n_kv
    for h in range(n_heads):
        kv = h // g
        s = np.array([q[h * hd:(h + 1) * hd] @ kc[t][kv * hd:(kv + 1) * hd] for t in range(w0, seq)], np.float64)
        w = np.exp(s - s.max())
        w /= w.sum()
        out[h * hd:(h + 1) * hd] = sum(w[i] * vc[t][kv * hd:(kv + 1) * hd] for i, t in enumerate(range(w0, seq)))
    return out


def test_attention_window_and_limit_rule():
    rng = np.random.default_rng(5)
    nh, nkv, hd, n = 4, 2, 32, 40
    q = rng.standard_normal(nh * hd).astype(np.float32) * 0.3
    kc = [rng.standard_normal(nkv * hd).astype(np.float32) for _ in range(n)]
    vc = [rng.standard_normal(nkv * hd).astype(np.float32) for _ in range(n)]
    for window, limit in [(0, 40), (8, 40), (8, 20), (64, 30), (1, 5)]:
        want = gqa_reference(q, kc, vc, nh, nkv, hd, window, limit)
        got = so.gqa_attention_rows(q, kc, vc, nh, nkv, hd, limit=limit, window=window)
        np.testing.assert_allclose(got, want, rtol=0, atol=1e-5)


def test_e4b_oracle_incremental_equals_full_rerun():
    """Incremental decode == full rerun (real_forward.rs:3129) under the e4b schedule: sliding,
    global and shared-KV layers (22-25 of a full-width model)."""
    base = dict(hidden=2560, n_heads=8, n_kv=4, head_dim=256, ffn=512, vocab=300, n_layers=26, seed=9)
    spec = so.ModelSpec(**base)
    tensors = so.synth_stage(spec, 22, 25, True, True)
    lay = so.Layout("gemma-4-e4b", "s", 22, 25, True, True)
    ids = so.synth_tokens(4, "p", 14, spec.vocab)
    full = so.OracleStage(tensors, lay, rope_theta=10000.0).begin_token_ids("f", ids)
    inc = so.OracleStage(tensors, lay, rope_theta=10000.0)
    inc.begin_token_ids("i", ids[:11])
    assert sorted(inc.sessions["i"]["kv"]) == [22, 23]  # 24 and 25 read layer 22's cache
    rows = np.concatenate([inc.begin_token_ids("i", [t]) for t in ids[11:]])
    np.testing.assert_allclose(rows, full[11:], rtol=0, atol=2e-5 * np.abs(full).max())
