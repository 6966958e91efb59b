"""GPU: the Gemma-4 e4b attention schedule (layer_attention_config_for_layout,
crates/stage-forward-lab/src/real_forward.rs:1407-1481) against the oracle.

Layers 5, 11, 17, 23, 29, .. are global (RoPE base 1e6, proportional rotation of head_dim/4 dims);
the others slide over 512 keys (base 1e4); from layer 24 on a layer attends over the cache of layer
23 (global) or 22 (sliding) and has no cache of its own.  The stages here hold layers 22-25 and
22-29 of a full-width (hidden 2560, head_dim 256) synthetic model: sliding, global, shared-sliding
and shared-global layers; a 530-token prompt makes the window cut.  f32 cache; the bar is stated at
check_prefill."""
import numpy as np
import pytest

import stage_oracle as so
from gpu_util import assert_close

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

E4B = "synthetic-gemma-4-e4b"
BASE = dict(hidden=2560, n_heads=8, n_kv=4, head_dim=256, ffn=512, vocab=1000, n_layers=30, seed=41)


@pytest.fixture(scope="module")
def sf():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import stagefwd
    return stagefwd


def gpu(sf, model_id, start, end, **kw):
    shape = sf.ModelShape(**BASE)
    return sf.CudaStageBackend(synthetic=shape, rope_theta=10000.0, kv_f32=True, max_ctx=1024, max_sessions=2,
                               max_batch_tokens=544, **kw).load_layout(model_id, "s", start, end, True, True)


def row_errors(got, ref):
    return np.abs(got - ref).max(axis=1) / np.abs(ref).max(axis=1)


# With hundreds of cached keys this synthetic model's unscaled, sharply peaked attention meets
# near-ties between its top keys on a few query rows, where last-bit differences move the row by up
# to a few percent (the generic schedule on the same layers shows it too: 8 of 530 prompt rows above
# 1e-3, median 3e-6).  The bar for a long prompt is therefore: median row error <= 2e-5, at most 5%
# of rows above 1e-3, and 1e-3 on the rows that matter here: those the window cuts, the last prompt
# row and every decode row; tokens identical.
def check_prefill(hg, ho, strict_rows, what):
    err = row_errors(hg, ho)
    assert np.median(err) <= 2e-5, f"{what}: median row error {np.median(err):.2e}"
    assert np.mean(err > 1e-3) <= 0.05, f"{what}: {int(np.sum(err > 1e-3))} rows above 1e-3"
    bad = [int(r) for r in strict_rows if err[r] > 1e-3]
    assert not bad, f"{what}: rows {bad} above 1e-3 ({err[bad]})"


def run_case(sf, start, end, strict_rows, decode_steps):
    spec = so.ModelSpec(**BASE)
    g = gpu(sf, E4B, start, end)
    o = so.OracleStage(so.synth_stage(spec, start, end, True, True), so.Layout(E4B, "s", start, end, True, True),
                       rope_theta=10000.0, kv_fp16=False)
    prompt = so.synth_tokens(12, "p", 530, spec.vocab)
    hg, ho = g.begin_token_ids("r", prompt), o.begin_token_ids("r", prompt)
    check_prefill(hg, ho, strict_rows, f"e4b prefill, layers {start}-{end}")
    tok = g.sample_tail(hg[-1])[0]
    assert tok == o.sample_tail(ho[-1])[0]
    for step in range(decode_steps):  # one row per step, 531+ keys: the window cuts every decode row
        hg, ho = g.begin_token_ids("r", [tok]), o.begin_token_ids("r", [tok], append=True)
        assert_close(hg, ho, what=f"e4b decode step {step}, layers {start}-{end}")
        tok = g.sample_tail(hg[-1])[0]
        assert tok == o.sample_tail(ho[-1])[0]
    return g


def test_e4b_window_and_shared_sliding_layers(sf):
    """Layers 22 (sliding), 23 (global, proportional RoPE), 24 and 25 (sliding, reading 22's cache)."""
    g = run_case(sf, 22, 25, strict_rows=range(512, 530), decode_steps=3)
    # layers 22 and 23 hold a cache; 24 and 25 read 22's (4 slabs in the generic schedule, 2 here)
    generic = gpu(sf, "synthetic-gemma", 22, 25)
    assert g.info.kv_bytes * 4 == generic.info.kv_bytes * 2


def test_e4b_shared_global_layer(sf):
    """Layers 22-29: 29 is global and reads 23's cache; 24-28 read 22's."""
    g = run_case(sf, 22, 29, strict_rows=[529], decode_steps=2)
    generic = gpu(sf, "synthetic-gemma", 22, 29)
    assert g.info.kv_bytes * 8 == generic.info.kv_bytes * 2


def test_e4b_stage_must_hold_its_shared_kv_sources(sf):
    """validate_stage_split_constraints (real_forward.rs:1459-1481)."""
    with pytest.raises(sf.StageError, match="layer 24 requires shared KV from layer 22 outside this stage"):
        gpu(sf, E4B, 24, 29)
    gpu(sf, "synthetic-gemma", 24, 29)  # the generic schedule has no shared KV
