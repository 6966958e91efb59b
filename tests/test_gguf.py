"""CPU: GGUF parsing, tensor roles, stage splits, the shard manifest bundle and stage packs
(csrc/gguf.cpp through the C ABI), against the reference's own known answers
(crates/stage-forward-lab/src/gguf.rs:925-1163, lib.rs:7930-8030) and a fixture written and read
by the reference's gguf-py (tests/golden/make_gguf_golden.py)."""
import json

import numpy as np
import pytest

import stage_oracle as so
from gguf_util import ARR, BOOL, F32, F64, I32, I64, STR, U8, U32, U64, gguf_bytes

sfg = pytest.importorskip("stagefwd.gguf")
from stagefwd import StageError  # noqa: E402
from stagefwd.gguf import GgufFile, StageSplit, materialize_stage, pack_stage  # noqa: E402
from stagefwd.pipeline import even_stage_split  # noqa: E402


# ---------------------------------------------------------------- gguf-py fixture
@pytest.fixture(scope="module")
def mixed(golden_dir):
    path = golden_dir / "gguf_mixed.gguf"
    return path, json.loads((golden_dir / "gguf_mixed.json").read_text())


def test_gguf_py_fixture_parses_identically(mixed):
    path, ref = mixed
    f = GgufFile.parse_file(path)
    assert f.version == ref["version"] == 3
    assert f.file_size_bytes == ref["file_size"]
    assert f.tensor_data_offset == ref["tensor_data_offset"]  # general.alignment = 64
    assert f.tensor_count == len(ref["tensors"])
    for got, want in zip(f.tensors, ref["tensors"]):
        assert got.name == want["name"]
        assert list(got.dimensions) == want["dims"]
        assert got.ggml_type == want["ggml_type"]
        assert got.offset == want["offset"]
        assert got.file_offset == ref["tensor_data_offset"] + want["offset"]
        assert got.byte_len == want["byte_len"]  # distance to the next tensor: padding included
        assert got.byte_len >= want["n_bytes"]
    # metadata: sorted keys, every value as the reference formats it
    assert f.metadata_keys == sorted(ref["metadata"])
    for key, m in ref["metadata"].items():
        assert f.metadata_string(key) == m["text"], key
    assert f.metadata_string("absent.key") is None
    assert f.architecture() == "gemma4"
    assert f.inferred_layer_count() == 3
    assert (f.hidden_size(), f.feed_forward_length(), f.attention_head_count()) == (256, 512, 4)
    assert f.metadata_u32("fixture.u64") is None  # 2^63 + 5 does not fit
    assert f.metadata_u32("fixture.i32") is None  # negative
    assert f.metadata_u32("fixture.u8") is None   # only u32 / u64 / i32 / i64 convert
    assert f.metadata_u32("fixture.u32") == 4000000000
    assert f.block_indices() == [0, 1, 2]
    roles = {t.name: t.role for t in f.tensors}
    assert roles == {"token_embd.weight": "PromptIngress", "rope_freqs.weight": "Positional",
                     "blk.0.attn_q.weight": "Layer", "blk.0.attn_norm.weight": "Layer",
                     "blk.1.ffn_down.weight": "Layer", "blk.2.post_ffw_norm.weight": "Layer",
                     "per_layer_token_embd.weight": "SharedAuxiliary", "output_norm.weight": "TailOnly",
                     "fixture.unknown": "UnknownGlobal"}
    # array metadata (gguf.rs:253-277)
    assert f.metadata_string_array("fixture.arr_str") == ["a", "b c", ""]
    assert f.metadata_string_array("fixture.arr_f32") == ["0.5", "1.25", "-3"]
    assert f.metadata_f32_array("fixture.arr_f32") == [0.5, 1.25, -3.0]
    assert f.metadata_f32_array("fixture.arr_i32") == [1.0, -2.0, 3.0]
    assert f.metadata_f32_array("fixture.arr_u64") == [0.0, 0.0]  # only f32 / f64 / i32 / u32 convert
    assert f.metadata_f32_array("fixture.arr_empty") is None  # gguf-py's writer drops empty arrays
    e = GgufFile.parse_bytes(gguf_bytes([("empty", ARR, (F32, [])), ("words", ARR, (STR, ["x", "é"]))], []))
    assert e.metadata_f32_array("empty") == [] and e.metadata_string_array("empty") == []
    assert e.metadata_string("empty") == "[]" and e.metadata_string_array("words") == ["x", "é"]
    assert f.metadata_f32_array("fixture.u32") is None and f.metadata_string_array("absent") is None
    # parse_bytes of the same bytes gives the same view
    g = GgufFile.parse_bytes(path.read_bytes())
    assert g.tensors == f.tensors and g.metadata_keys == f.metadata_keys


# ---------------------------------------------------------------- reference unit tests
def test_parse_synthetic_v3_gguf():
    """gguf.rs:945-996."""
    data = gguf_bytes([("general.architecture", STR, "gemma"), ("gemma.block_count", U32, 28)],
                      [("blk.0.attn_q.weight", [4, 8], 0, 0), ("blk.27.ffn_down.weight", [4, 8], 0, 128)],
                      data=b"")
    f = GgufFile.parse_bytes(data)
    assert f.version == 3 and f.tensor_count == 2
    assert f.architecture() == "gemma"
    assert f.inferred_layer_count() == 28
    assert f.block_indices() == [0, 27]
    assert f.suggest_even_stage_split(2) == [StageSplit(0, 0, 13), StageSplit(1, 14, 27)]


def test_classify_tensor_roles():
    """gguf.rs:998-1024, plus the u32 parse rule of the block index."""
    names = ["blk.7.attn_q.weight", "token_embd.weight", "output_norm.weight", "rope_freqs.weight",
             "per_layer_token_embd.weight", "general.weird", "blk.+3.x", "blk.07.x", "blk.x.y",
             "blk.4294967296.a", "blk.4294967295", "output.weight", "blk."]
    data = gguf_bytes([], [(n, [1], 0, 4 * i) for i, n in enumerate(names)], data=bytes(4 * len(names)))
    f = GgufFile.parse_bytes(data)
    got = {t.name: (t.role, t.layer_index) for t in f.tensors}
    assert got["blk.7.attn_q.weight"] == ("Layer", 7)
    assert got["token_embd.weight"] == ("PromptIngress", None)
    assert got["output_norm.weight"] == ("TailOnly", None)
    assert got["rope_freqs.weight"] == ("Positional", None)
    assert got["per_layer_token_embd.weight"] == ("SharedAuxiliary", None)
    assert got["general.weird"] == ("UnknownGlobal", None)
    assert got["blk.+3.x"] == ("Layer", 3)          # Rust's u32 parse takes a leading '+'
    assert got["blk.07.x"] == ("Layer", 7)
    assert got["blk.x.y"] == ("UnknownGlobal", None)
    assert got["blk.4294967296.a"] == ("UnknownGlobal", None)  # overflows u32
    assert got["blk.4294967295"] == ("Layer", 4294967295)
    assert got["output.weight"] == ("TailOnly", None)
    assert got["blk."] == ("UnknownGlobal", None)


def toy_gguf(tmp_path):
    """The toy model of gguf.rs:1026-1163 / lib.rs:7930-8030 as a real file: three 1-element
    tensors at offsets 0 / 100 / 200 of a 300-byte data section of the bytes 0, 1, .., 255, 0, ..."""
    section = bytes((np.arange(300) % 256).astype(np.uint8))
    meta = [("general.name", STR, "Toy"), ("general.architecture", STR, "toy"), ("llama.block_count", U32, 2)]
    tensors = [("token_embd.weight", [1], 0, 0), ("blk.0.attn_q.weight", [1], 0, 100),
               ("output_norm.weight", [1], 0, 200)]
    path = tmp_path / "toy.gguf"
    path.write_bytes(gguf_bytes(meta, tensors, data=section))
    return path, section


TOY_SPLITS = [StageSplit(0, 0, 0), StageSplit(1, 1, 1)]


def test_manifest_builds_replicated_and_owned_groups(tmp_path):
    """gguf.rs:1026-1103 and :1106-1162 (bundle files)."""
    path, _ = toy_gguf(tmp_path)
    f = GgufFile.parse_file(path)
    assert [t.byte_len for t in f.tensors] == [100, 100, 100]
    out = tmp_path / "bundle"
    f.write_bundle(TOY_SPLITS, out)
    m = json.loads((out / "model-shard-manifest.json").read_text())
    assert m["model_name"] == "Toy" and m["architecture"] == "toy"
    assert m["hidden_size"] is None and m["total_layers"] == 2
    assert len(m["stages"]) == 2
    assert m["stages"][0]["prompt_ingress"]["tensor_names"] == ["token_embd.weight"]
    assert m["stages"][0]["owned"]["tensor_names"] == ["blk.0.attn_q.weight"]
    assert m["stages"][0]["owned"]["name"] == "stage1_owned"
    assert m["stages"][1]["owned"]["tensor_names"] == []
    assert m["stages"][1]["tail_only"]["tensor_names"] == ["output_norm.weight"]
    assert m["stages"][0]["tail_only"] == {"name": "tail_only", "tensor_names": [], "total_bytes": 0}
    rp = m["runtime_plan"]
    assert [r["role"] for r in rp] == ["head", "tail"]
    assert rp[0]["required"]["tensor_names"] == ["token_embd.weight", "blk.0.attn_q.weight"]
    assert rp[0]["required"]["total_bytes"] == 200
    assert rp[1]["required"]["tensor_names"] == ["output_norm.weight"]
    assert rp[1]["optional"]["tensor_names"] == ["token_embd.weight"]
    for name in ["stage-1-owned.txt", "stage-2-tail-only.txt", "runtime-stage-1.json", "runtime-stage-2-required.txt",
                 "stage-1.json", "runtime-stage-2-slices.json"]:
        assert (out / name).exists(), name
    assert (out / "stage-2-owned.txt").read_text() == "\n"  # an empty list is one newline
    assert (out / "stage-1-owned.txt").read_text() == "blk.0.attn_q.weight\n"
    slices = json.loads((out / "runtime-stage-2-slices.json").read_text())
    assert slices["optional"][0] == {"name": "token_embd.weight", "file_offset": f.tensor_data_offset,
                                     "byte_len": 100, "dimensions": [1], "ggml_type": 0}
    # serde_json's pretty layout: two-space indent, one array element per line, `[]` when empty
    text = (out / "stage-2.json").read_text()
    assert text.startswith('{\n  "stage_index": 1,\n  "start_layer": 1,\n  "end_layer": 1,\n  "prompt_ingress": {\n'
                           '    "name": "prompt_ingress",\n    "tensor_names": [\n      "token_embd.weight"\n    ],\n')
    assert '"owned": {\n    "name": "stage2_owned",\n    "tensor_names": [],\n    "total_bytes": 0\n  },' in text
    assert not text.endswith("\n")


def test_pack_stage_roundtrip(tmp_path):
    """lib.rs:7930-8030: pack the head's required tensors, reopen, compare bytes."""
    path, section = toy_gguf(tmp_path)
    GgufFile.parse_file(path).write_bundle(TOY_SPLITS, tmp_path / "bundle")
    idx = pack_stage(tmp_path / "bundle", path, 0, tmp_path / "packs")
    assert idx.name == "stage-1-required.index.json"
    index = json.loads(idx.read_text())
    assert index["tensor_count"] == 2 and index["role"] == "head" and index["model_name"] == "Toy"
    assert [e["name"] for e in index["tensors"]] == ["token_embd.weight", "blk.0.attn_q.weight"]
    tensors = so.load_pack(idx)  # the oracle's reader of the reference format (validate_offsets)
    assert bytes(tensors["token_embd.weight"][2]) == section[:100]
    assert bytes(tensors["blk.0.attn_q.weight"][2]) == section[100:200]
    assert "output_norm.weight" not in tensors
    # the tail: required = output*, optional = the embedding (tied logits)
    idx2 = pack_stage(tmp_path / "bundle", path, 1, tmp_path / "packs")
    assert [e["name"] for e in json.loads(idx2.read_text())["tensors"]] == ["output_norm.weight"]
    idx3 = pack_stage(tmp_path / "bundle", path, 1, tmp_path / "packs_all", include_optional=True)
    t3 = so.load_pack(idx3)
    assert list(t3) == ["output_norm.weight", "token_embd.weight"]
    assert bytes(t3["output_norm.weight"][2]) == section[200:300]
    e = json.loads(idx3.read_text())["tensors"][1]
    assert e["source_file_offset"] == GgufFile.parse_file(path).tensor_data_offset and e["pack_offset"] == 100


def test_bundle_validation_errors(tmp_path):
    """LoadedRuntimeBundle::load / validate_against_gguf / stage lookup (lib.rs:3283-3440)."""
    path, _ = toy_gguf(tmp_path)
    b = tmp_path / "bundle"
    GgufFile.parse_file(path).write_bundle(TOY_SPLITS, b)
    with pytest.raises(StageError, match="Stage 3 not found in runtime bundle"):
        pack_stage(b, path, 2, tmp_path / "p")
    req = b / "runtime-stage-1-required.txt"
    good = req.read_text()
    req.write_text("token_embd.weight\n")
    with pytest.raises(StageError, match="Required runtime tensor list .* does not match manifest for stage 1"):
        pack_stage(b, path, 0, tmp_path / "p")
    req.write_text("  blk.0.attn_q.weight \n\ntoken_embd.weight\n")  # order, blanks and spaces do not matter
    pack_stage(b, path, 0, tmp_path / "p")
    req.write_text(good)
    other = tmp_path / "other.gguf"
    other.write_bytes(gguf_bytes([("llama.block_count", U32, 2)], [("token_embd.weight", [1], 0, 0)], data=bytes(4)))
    with pytest.raises(StageError, match="references tensor blk.0.attn_q.weight which is not present in GGUF"):
        pack_stage(b, other, 0, tmp_path / "p")
    rt = b / "runtime-stage-2.json"
    rt.write_text(rt.read_text().replace('"tail"', '"middle"'))
    with pytest.raises(StageError, match="does not match top-level manifest for stage 2"):
        pack_stage(b, path, 0, tmp_path / "p")


# ---------------------------------------------------------------- format edge cases
def test_version1_and_alignment():
    meta = [("general.alignment", U32, 64), ("a.b", ARR, (I32, [1, 2])), ("c", F64, 0.25), ("d", BOOL, 1),
            ("e", I64, -3), ("f", U64, 5), ("g", U8, 7), ("h", F32, 1.5)]
    data = gguf_bytes(meta, [("blk.0.x", [2, 3], 0, 0)], version=1, alignment=64, data=bytes(24))
    f = GgufFile.parse_bytes(data)
    assert f.version == 1 and f.tensor_data_offset % 64 == 0
    assert f.tensors[0].dimensions == (2, 3) and f.tensors[0].byte_len == 24
    assert [f.metadata_string(k) for k in ["a.b", "c", "d", "e", "f", "g", "h"]] == [
        "[1, 2]", "0.25", "true", "-3", "5", "7", "1.5"]
    # an alignment of 0 leaves the data right after the header; a u64 alignment counts too
    f0 = GgufFile.parse_bytes(gguf_bytes([("general.alignment", U64, 0)], [], alignment=1))
    assert f0.tensor_data_offset == f0.file_size_bytes
    # a repeated key keeps its last value
    f2 = GgufFile.parse_bytes(gguf_bytes([("k", U32, 1), ("k", U32, 9)], []))
    assert f2.metadata_u32("k") == 9 and f2.metadata_keys == ["k"]


@pytest.mark.parametrize("blob,match", [
    (b"", "truncated"),
    (b"GGUX" + bytes(20), "Not a GGUF file"),
    (b"GGUF\x03\x00\x00\x00", "truncated"),
])
def test_malformed_headers(blob, match):
    with pytest.raises(StageError, match=match):
        GgufFile.parse_bytes(blob)


def test_malformed_bodies():
    base = gguf_bytes([("general.architecture", STR, "gemma")], [("blk.0.w", [4], 0, 0)], data=bytes(16))
    for cut in (30, 40, 60, 100):  # inside the metadata and the tensor table (it ends at byte 108)
        with pytest.raises(StageError, match="truncated|past the end"):
            GgufFile.parse_bytes(base[:cut])
    GgufFile.parse_bytes(base[:108])  # the data section itself is not read: a cut there still parses
    raw = b"GGUF" + (3).to_bytes(4, "little") + (0).to_bytes(8, "little") + (1).to_bytes(8, "little")
    raw += (1).to_bytes(8, "little") + b"x" + (13).to_bytes(4, "little")
    with pytest.raises(StageError, match="Unsupported GGUF metadata type 13"):
        GgufFile.parse_bytes(raw)
    bad_utf8 = b"GGUF" + (3).to_bytes(4, "little") + (0).to_bytes(8, "little") + (1).to_bytes(8, "little")
    bad_utf8 += (2).to_bytes(8, "little") + b"\xc3\x28" + (4).to_bytes(4, "little") + (1).to_bytes(4, "little")
    with pytest.raises(StageError, match="not valid UTF-8"):
        GgufFile.parse_bytes(bad_utf8)
    huge = b"GGUF" + (3).to_bytes(4, "little") + (0).to_bytes(8, "little") + (1).to_bytes(8, "little")
    huge += (2**62).to_bytes(8, "little")
    with pytest.raises(StageError, match="past the end"):
        GgufFile.parse_bytes(huge)
    many = b"GGUF" + (3).to_bytes(4, "little") + (2**60).to_bytes(8, "little") + (0).to_bytes(8, "little")
    with pytest.raises(StageError, match="truncated"):
        GgufFile.parse_bytes(many)
    GgufFile.parse_bytes(gguf_bytes([], []))  # no metadata, no tensors
    with pytest.raises(StageError, match="Failed to open"):
        GgufFile.parse_file("/nonexistent/model.gguf")


def test_even_split_matches_pipeline_rule():
    """suggest_even_stage_split (gguf.rs:307-329) == the pipeline's split for 42 layers."""
    f = GgufFile.parse_bytes(gguf_bytes([("gemma4.block_count", U32, 42)], []))
    for n in (1, 2, 4, 8):
        got = [(s.start_layer, s.end_layer) for s in f.suggest_even_stage_split(n)]
        assert got == [tuple(x) for x in even_stage_split(42, n)]
    assert f.suggest_even_stage_split(0) is None and f.suggest_even_stage_split(43) is None
    g = GgufFile.parse_bytes(gguf_bytes([], []))
    assert g.inferred_layer_count() is None and g.suggest_even_stage_split(1) is None


def test_materialize_required_tensors(tmp_path):
    """materialize_required_tensors (lib.rs:3500-3510) with sanitize_tensor_filename (:3627-3636)."""
    path, section = toy_gguf(tmp_path)
    GgufFile.parse_file(path).write_bundle(TOY_SPLITS, tmp_path / "bundle")
    out = tmp_path / "materialized"
    assert materialize_stage(tmp_path / "bundle", path, 0, out) == 2
    assert sorted(p.name for p in out.iterdir()) == ["blk_0_attn_q_weight", "token_embd_weight"]
    assert (out / "token_embd_weight").read_bytes() == section[:100]
    assert (out / "blk_0_attn_q_weight").read_bytes() == section[100:200]
    # a multi-byte character becomes one '_'
    data = gguf_bytes([("llama.block_count", U32, 1)], [("blk.0.\u00e9-x_y", [1], 0, 0)], data=bytes(8))
    (tmp_path / "u.gguf").write_bytes(data)
    GgufFile.parse_file(tmp_path / "u.gguf").write_bundle([StageSplit(0, 0, 0)], tmp_path / "ub")
    assert materialize_stage(tmp_path / "ub", tmp_path / "u.gguf", 0, tmp_path / "um") == 1
    assert [p.name for p in (tmp_path / "um").iterdir()] == ["blk_0__-x_y"]


def test_written_json_has_serde_pretty_layout(tmp_path):
    """Every JSON file the bundle and pack writers produce is laid out exactly as serde_json's pretty
    printer lays it out (two-space indent, `"key": value`, one element per line, `[]` when empty,
    lowercase \\u00XX escapes, no trailing newline) -- which for these documents is what Python's
    json.dumps(indent=2, ensure_ascii=False) prints, field order kept."""
    section = bytes(64)
    meta = [("general.name", STR, 'q"uote\\\\ \x01 ctl é'), ("general.architecture", STR, "toy"),
            ("llama.block_count", U32, 3), ("llama.embedding_length", U32, 8)]
    tensors = [("token_embd.weight", [4, 2], 0, 0), ("blk.0.w", [2], 0, 32), ("blk.1.w", [2], 0, 40),
               ("blk.2.w", [2], 0, 48), ("output_norm.weight", [2], 0, 56)]
    path = tmp_path / "m.gguf"
    path.write_bytes(gguf_bytes(meta, tensors, data=section))
    f = GgufFile.parse_file(path)
    f.write_bundle(f.suggest_even_stage_split(3), tmp_path / "b")
    pack_stage(tmp_path / "b", path, 1, tmp_path / "p", include_optional=True)
    files = sorted((tmp_path / "b").glob("*.json")) + sorted((tmp_path / "p").glob("*.json"))
    assert len(files) == 1 + 3 + 3 + 3 + 1
    for p in files:
        text = p.read_text()
        assert text == json.dumps(json.loads(text), indent=2, ensure_ascii=False), p.name
    m = json.loads((tmp_path / "b" / "model-shard-manifest.json").read_text())
    assert m["model_name"] == 'q"uote\\\\ \x01 ctl é' and m["hidden_size"] == 8
    assert [r["role"] for r in m["runtime_plan"]] == ["head", "middle", "tail"]
