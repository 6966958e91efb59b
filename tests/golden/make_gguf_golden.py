"""Regenerate the GGUF parsing fixtures in this folder (run in a container that has the reference
tree; tests only read the committed outputs).

  python tests/golden/make_gguf_golden.py --reference <reference checkout>

Outputs
  gguf_mixed.gguf   a small GGUF v3 file written by the reference's own gguf-py writer
                    (vendor/llama.cpp/gguf-py/gguf/gguf_writer.py): every metadata value type
                    (u8 .. f64, bool, strings with escapes and non-ASCII text, typed and inferred
                    arrays), a 64-byte data alignment, and F32 / F16 / Q4_K / Q6_K tensors of every
                    tensor role, one of them 40 bytes long so that alignment padding follows it.
  gguf_mixed.json   what the reference's gguf-py reader (gguf_reader.py) sees in that file:
                    version, tensor data offset, tensor names / dims / types / offsets, and the
                    expected results of the stage tooling's rules (crates/stage-forward-lab/src/
                    gguf.rs): tensor_byte_len as the distance to the next tensor by offset
                    (:331-343), metadata values as text in Rust's `Display` form (:800-823:
                    floats as the shortest round-trip digits without exponent).
"""
import argparse
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def rust_display(v, vtype, gguf) -> str:
    T = gguf.GGUFValueType
    if vtype == T.FLOAT32:
        x = np.float32(v)
        return "NaN" if np.isnan(x) else np.format_float_positional(x, unique=True, trim="-")
    if vtype == T.FLOAT64:
        x = np.float64(v)
        return "NaN" if np.isnan(x) else np.format_float_positional(x, unique=True, trim="-")
    if vtype == T.BOOL:
        return "true" if v else "false"
    if vtype == T.STRING:
        return v
    return str(int(v))


def field_value(field, gguf):
    """(python value, text) of a reader field, following gguf_reader's part layout."""
    T = gguf.GGUFValueType
    t = field.types[0]
    if t == T.ARRAY:
        sub = field.types[1] if len(field.types) > 1 else None
        vals = []
        for idx in field.data:
            part = field.parts[idx]
            if sub == T.STRING:
                vals.append(bytes(part).decode("utf-8"))
            else:
                vals.append(part[0].item())
        text = "[" + ", ".join(rust_display(x, sub, gguf) for x in vals) + "]"
        return vals, text
    part = field.parts[field.data[0]]
    v = bytes(part).decode("utf-8") if t == T.STRING else part[0].item()
    return v, rust_display(v, t, gguf)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "vendor/llama.cpp/gguf-py"))
    import gguf

    T = gguf.GGUFValueType
    Q = gguf.GGMLQuantizationType
    path = HERE / "gguf_mixed.gguf"
    rng = np.random.default_rng(20261202)
    w = gguf.GGUFWriter(str(path), "gemma4")
    w.add_custom_alignment(64)
    w.add_name("fixture µ-model")
    w.add_uint32("gemma4.block_count", 3)
    w.add_uint32("gemma4.embedding_length", 256)
    w.add_uint64("gemma4.feed_forward_length", 512)
    w.add_int32("gemma4.attention.head_count", 4)
    w.add_uint8("fixture.u8", 200)
    w.add_int8("fixture.i8", -5)
    w.add_uint16("fixture.u16", 65000)
    w.add_int16("fixture.i16", -30000)
    w.add_uint32("fixture.u32", 4000000000)
    w.add_int32("fixture.i32", -2000000000)
    w.add_float32("fixture.f32_tenth", 0.1)
    w.add_float32("fixture.f32_small", 1e-7)
    w.add_float32("fixture.f32_large", 3.0e38)
    w.add_float32("fixture.f32_one", 1.0)
    w.add_float32("fixture.f32_negzero", -0.0)
    w.add_uint64("fixture.u64", 2**63 + 5)
    w.add_int64("fixture.i64", -(2**62))
    w.add_float64("fixture.f64", 2.5e-8)
    w.add_float64("fixture.f64_big", 1.0e22)
    w.add_bool("fixture.true", True)
    w.add_bool("fixture.false", False)
    w.add_string("fixture.escapes", 'quote " backslash \\ tab\t newline\n bell\x07 é ✓')
    w.add_array("fixture.arr_i32", [1, -2, 3])
    w.add_array("fixture.arr_f32", [0.5, 1.25, -3.0])
    w.add_array("fixture.arr_str", ["a", "b c", ""])
    w.add_array("fixture.arr_bool", [True, False])
    w.add_key_value("fixture.arr_u8", [1, 2, 255], T.ARRAY, sub_type=T.UINT8)
    w.add_key_value("fixture.arr_u64", [7, 2**40], T.ARRAY, sub_type=T.UINT64)
    w.add_array("fixture.arr_empty", [])

    def q_bytes(rows, row_bytes):
        return rng.integers(0, 256, size=(rows, row_bytes), dtype=np.uint8)

    w.add_tensor("token_embd.weight", rng.normal(0, 0.02, size=(8, 256)).astype(np.float16))
    w.add_tensor("rope_freqs.weight", np.ones(128, np.float32))
    w.add_tensor("blk.0.attn_q.weight", q_bytes(16, 144), raw_dtype=Q.Q4_K)
    w.add_tensor("blk.0.attn_norm.weight", rng.normal(1, 0.05, size=10).astype(np.float32))  # 40 B + padding
    w.add_tensor("blk.1.ffn_down.weight", q_bytes(16, 210), raw_dtype=Q.Q6_K)
    w.add_tensor("blk.2.post_ffw_norm.weight", rng.normal(1, 0.05, size=256).astype(np.float32))
    w.add_tensor("per_layer_token_embd.weight", rng.normal(0, 0.02, size=(2, 32)).astype(np.float16))
    w.add_tensor("output_norm.weight", rng.normal(1, 0.05, size=256).astype(np.float32))
    w.add_tensor("fixture.unknown", np.arange(16, dtype=np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()

    r = gguf.GGUFReader(str(path))
    size = path.stat().st_size
    meta = {}
    for name, field in r.fields.items():
        if name.startswith("GGUF."):
            continue
        value, text = field_value(field, gguf)
        meta[name] = {"type": int(field.types[0]), "text": text,
                      "value": value if not isinstance(value, float) or np.isfinite(value) else None}
    tensors = []
    for t in r.tensors:
        rel = int(t.data_offset) - int(r.data_offset)
        tensors.append({"name": t.name, "dims": [int(d) for d in t.field.parts[3]],
                        "ggml_type": int(t.tensor_type), "offset": rel, "n_bytes": int(t.n_bytes)})
    order = sorted(range(len(tensors)), key=lambda i: tensors[i]["offset"])  # stable, like sort_by_key
    data_bytes = size - int(r.data_offset)
    for k, i in enumerate(order):
        nxt = tensors[order[k + 1]]["offset"] if k + 1 < len(order) else data_bytes
        tensors[i]["byte_len"] = max(0, nxt - tensors[i]["offset"])
    version = int(r.fields["GGUF.version"].parts[-1][0])
    out = {"source": "gguf-py GGUFWriter / GGUFReader of the reference tree", "file_size": size,
           "version": version, "tensor_data_offset": int(r.data_offset), "alignment": int(r.alignment),
           "metadata": meta, "tensors": tensors}
    (HERE / "gguf_mixed.json").write_text(json.dumps(out, indent=1, ensure_ascii=False))
    print("wrote", path, size, "bytes,", len(tensors), "tensors,", len(meta), "metadata keys")


if __name__ == "__main__":
    main()
