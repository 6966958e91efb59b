"""CPU: the C-ABI library loads, exports every entry point include/stagefwd.h declares, and
rejects bad input on the host with an error message (no GPU needed for these paths)."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "stagefwd.h"
LIB = ROOT / "compute-sharding_b200" / "stagefwd" / "libstagefwd.so"


def declared():
    return sorted(set(re.findall(r"\b(sfc_[a-z0-9_]+)\s*\(", HEADER.read_text())))


def test_header_declares_entry_points():
    names = declared()
    for must in ("sfc_matmul", "sfc_dequantize_rows", "sfc_stage_open", "sfc_begin_token_ids",
                 "sfc_continue_forward", "sfc_sample_tail", "sfc_rollback_kv", "sfc_verify_greedy"):
        assert must in names


def test_library_exports_every_declared_symbol():
    assert LIB.exists(), "build with make -C compute-sharding_b200"
    lib = ctypes.CDLL(str(LIB))
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB)], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (sfc_[a-z0-9_]+)", out))
    assert set(declared()) <= exported


def test_host_validation_without_gpu():
    import stagefwd as sf
    assert sf.lib.sfc_abi_version() == 1
    # unsupported type / shape: rejected before any CUDA call
    assert sf.lib.sfc_matmul(13, None, 4, 256, None, 1, None, None) == -1
    assert b"unsupported ggml type 13" in sf.lib.sfc_last_error()
    assert sf.lib.sfc_matmul(12, None, 4, 100, None, 1, None, None) == -1
    assert sf.lib.sfc_dequantize_rows(1, None, 1, 256, None, None) == -1
    # K-quants: tiles of 16 rows (zero-padded), one record per (tile, 256-block): Q6_K 3360 B, Q4_K 2304 B
    assert sf.lib.sfc_weight_device_bytes(14, 10, 2560) == 1 * 10 * 3360
    assert sf.lib.sfc_weight_device_bytes(14, 32, 2560) == 2 * 10 * 3360
    assert sf.lib.sfc_weight_device_bytes(12, 10, 2560) == 1 * 10 * 2304
    assert sf.lib.sfc_weight_device_bytes(12, 17, 512) == 2 * 2 * 2304
    assert sf.lib.sfc_weight_device_bytes(1, 10, 2560) == 10 * 2560 * 2


def test_stage_open_rejects_bad_index_name(tmp_path):
    import stagefwd as sf
    bad = tmp_path / "stage.json"
    bad.write_text("{}")
    with pytest.raises(sf.StageError, match="index.json"):
        sf.CudaStageBackend(bad).load_layout("m", "s", 0, 0, True, True)


def test_gguf_and_payload_entry_points_validate_on_the_host(tmp_path):
    import ctypes
    import stagefwd as sf
    import stagefwd.gguf  # noqa: F401  (declares the GGUF prototypes)
    with pytest.raises(sf.StageError, match="Failed to open"):
        sf.CudaStageBackend(gguf_path=tmp_path / "absent.gguf").load_layout("m", "s", 0, 0, True, True)
    junk = tmp_path / "junk.gguf"
    junk.write_bytes(b"GGML" + bytes(60))
    with pytest.raises(sf.StageError, match="Not a GGUF file"):
        sf.CudaStageBackend(gguf_path=junk).load_layout("m", "s", 0, 0, True, True)
    n = ctypes.c_uint64()
    assert sf.lib.sfc_continue_forward_bytes(None, b"r", b"", 0, 4, None, 0, ctypes.byref(n)) == -1
    assert b"null argument" in sf.lib.sfc_last_error()
    buf = ctypes.create_string_buffer(64)
    assert sf.lib.sfc_pack_stage(str(tmp_path / "no-bundle").encode(), str(junk).encode(), 0, 0,
                                 str(tmp_path / "out").encode(), buf, 64) == -3
    assert b"Failed to read" in sf.lib.sfc_last_error() and b"model-shard-manifest.json" in sf.lib.sfc_last_error()
    assert sf.lib.sfc_gguf_open(None, None) == -1


def test_per_layer_embedding_stage_validation(tmp_path):
    """Stages whose layers carry PLE tensors are checked at load, before any device work: the chunk
    norm must be there, and a head needs the per-token table and the model projection."""
    import stagefwd as sf
    import stage_oracle as so
    spec = so.ModelSpec(hidden=256, n_heads=2, n_kv=1, head_dim=128, ffn=512, vocab=300, n_layers=2, seed=3,
                        ple_dim=64)
    full = so.synth_stage(spec, 0, 1, True, True)
    cases = [("per_layer_proj_norm.weight", "per_layer_proj_norm"),
             ("per_layer_token_embd.weight", "per_layer_token_embd"),
             ("blk.1.proj.weight", "only one of inp_gate / proj")]
    for k, (drop, msg) in enumerate(cases):
        tensors = {n: t for n, t in full.items() if n != drop}
        idx = so.write_pack(tmp_path / str(k), "stage-0", "full", 0, tensors)
        with pytest.raises(sf.StageError, match=msg):
            sf.CudaStageBackend(idx).load_layout("m", "s", 0, 1, True, True)


def test_header_is_plain_c(tmp_path):
    """include/stagefwd.h is the FFI boundary: it must compile as C99 (what a cgo / bindgen / ctypes
    binding sees), warning-free."""
    import shutil
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    r = subprocess.run([gcc, "-std=c99", "-Wall", "-Wextra", "-Werror", "-fsyntax-only", "-x", "c", str(HEADER)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
