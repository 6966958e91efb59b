"""GPU: the stage on StageTensor::bytes payloads (sfc_continue_forward_bytes / sfc_sample_tail_bytes):
bare and stb1-framed hidden rows give the same (bit-identical) rows as the float API, the aux
section ("rsa1": per-layer inputs, prefix hashes) comes back unchanged (real_forward.rs:2383-2387),
and malformed payloads are refused on the host."""
import struct

import pytest

import stage_oracle as so

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def sf():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import stagefwd
    return stagefwd


def test_payload_bytes_match_float_api(sf):
    base = dict(hidden=512, n_heads=4, n_kv=2, head_dim=128, ffn=1024, vocab=4096, n_layers=2, seed=23)
    spec, shape = so.ModelSpec(**base), sf.ModelShape(**base)
    kw = dict(rope_theta=10000.0, max_ctx=256, max_sessions=8)
    head = sf.CudaStageBackend(synthetic=shape, **kw).load_layout("m", "h", 0, 0, True, False)
    tail = sf.CudaStageBackend(synthetic=shape, **kw).load_layout("m", "t", 1, 1, False, True)
    H = shape.hidden
    h = head.begin_token_ids("r", so.synth_tokens(3, "p", 9, spec.vocab))
    ref = tail.continue_forward("a", h)
    assert tail.continue_forward_bytes("b", h.tobytes(), H) == ref.tobytes()  # bare rows
    aux = b"rsa1" + struct.pack("<IIII", 0, 0, 0, 2) + struct.pack("<QQ", 11, 22)  # prefix hashes only
    out = tail.continue_forward_bytes("c", sf.encode_stage_tensor_bytes(h.tobytes(), aux), H)
    assert sf.stage_tensor_byte_sections(out) == (ref.tobytes(), aux, True)
    assert tail.sample_tail_bytes(out, H) == tail.sample_tail(ref[-1])
    # one decode row through the bytes path continues session "c" like the float path continues "a"
    row = head.begin_token_ids("r", [5])
    assert tail.continue_forward_bytes("c", row.tobytes(), H) == tail.continue_forward("a", row).tobytes()
    with pytest.raises(sf.StageError, match="not a multiple of hidden_dim"):
        tail.continue_forward_bytes("d", h.tobytes()[:-4], H)
    with pytest.raises(sf.StageError, match="hidden_dim must be nonzero"):
        tail.sample_tail_bytes(h.tobytes(), 0)
    with pytest.raises(sf.StageError, match="stage hidden size"):
        tail.continue_forward_bytes("d", h.tobytes(), H // 2)
    with pytest.raises(sf.StageError, match="Head stage should use begin_prompt"):
        head.continue_forward_bytes("d", h.tobytes(), H)
