"""CPU: the oracle's Gemma-4 e4b attention schedule table and split rule
(layer_attention_config_for_layout / validate_stage_split_constraints,
crates/stage-forward-lab/src/real_forward.rs:1407-1481)."""
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
