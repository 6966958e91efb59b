"""CPU: the stage hand-off byte layout (StageTensor::bytes) at the C ABI against the reference's
rules (stage_tensor_byte_sections / encode_stage_tensor_bytes, crates/stage-forward-lab/src/
lib.rs:36-118): bare rows, well-formed frames, and byte strings that only look like frames."""
import struct

import numpy as np
import pytest

sf = pytest.importorskip("stagefwd")


def frame(hidden: bytes, aux: bytes) -> bytes:
    return b"stb1" + struct.pack("<II", len(hidden), len(aux)) + hidden + aux


def test_sections_and_encode_roundtrip():
    hidden = np.arange(12, dtype=np.float32).tobytes()
    aux = b"rsa1" + bytes(16) + b"\x07" * 8
    framed = sf.encode_stage_tensor_bytes(hidden, aux)
    assert framed == frame(hidden, aux)
    assert sf.stage_tensor_byte_sections(framed) == (hidden, aux, True)
    # no aux: the bare rows, not a frame (encode_stage_tensor_bytes returns hidden_bytes.to_vec())
    assert sf.encode_stage_tensor_bytes(hidden) == hidden
    assert sf.encode_stage_tensor_bytes(hidden, b"") == hidden
    assert sf.stage_tensor_byte_sections(hidden) == (hidden, None, False)
    # a frame with an empty aux section parses, aux None
    assert sf.stage_tensor_byte_sections(frame(hidden, b"")) == (hidden, None, True)


def test_lookalikes_are_bare_rows():
    hidden = np.ones(4, np.float32).tobytes()
    bad_len = frame(hidden, b"xy")[:-1]  # total length disagrees with the header
    assert sf.stage_tensor_byte_sections(bad_len) == (bad_len, None, False)
    assert sf.stage_tensor_byte_sections(b"stb1") == (b"stb1", None, False)  # shorter than the header
    assert sf.stage_tensor_byte_sections(b"") == (b"", None, False)
    other = b"stb2" + struct.pack("<II", 4, 0) + bytes(4)
    assert sf.stage_tensor_byte_sections(other) == (other, None, False)
