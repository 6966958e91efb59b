"""CPU oracle for the stage-forward hot path — TEST INFRASTRUCTURE ONLY.

A restatement of the reference's Rust CPU stage (`RealGemmaBackend`,
crates/stage-forward-lab/src/real_forward.rs) on top of the C++ kernels in
stage_oracle.cpp.  Only tests/, ``__graft_entry__.smoke()`` and bench.py's
CPU-baseline leg import this module, and only as the checker; the product
(`compute-sharding_b200/`) never does.

Parity anchors:
  * dequant: bit-exact against the reference's own ggml-quants.c
    (oracle/_ref, built from the reference sources) and gguf-py numpy
    (tests/golden fixtures) — see tests/test_oracle_golden.py;
  * known-answer rows from quants.rs:3725-3772 and real_math.rs:3130-3191,
    4334-4440 (tests/golden/known_answers.json);
  * incremental decode == full rerun (real_forward.rs:3129).
"""
from __future__ import annotations

import ctypes
import json
import math
import struct
import os
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

F32, F16, Q4_K, Q5_K, Q6_K, BF16 = 0, 1, 12, 13, 14, 30
QK_K = 256
BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210}
EPS = 1e-6  # real_math.rs:5


def bytes_per_row(t: int, in_dim: int) -> int:
    if t == F32:
        return 4 * in_dim
    if t in (F16, BF16):
        return 2 * in_dim
    if t in BLOCK_BYTES:
        if in_dim % QK_K:
            raise ValueError(f"in_dim {in_dim} not a multiple of {QK_K}")
        return in_dim // QK_K * BLOCK_BYTES[t]
    raise ValueError(f"unsupported ggml type {t}")


def _threads() -> int:
    return max(1, int(os.environ.get("ORACLE_THREADS", os.cpu_count() or 1)))


class _Lib:
    def __init__(self):
        path = HERE / "_build" / "libstage_oracle.so"
        if not path.exists():
            raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
        L = ctypes.CDLL(str(path))
        P, I64, I, F, U64 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_uint64
        L.or_dequantize_rows.argtypes = [I, P, I64, I64, P]
        L.or_matmul.argtypes = [I, P, I64, I64, P, I64, P, I]
        L.or_rms_norm_inplace.argtypes = [P, I64, P, I64, F]
        L.or_per_head_rms_norm.argtypes = [P, P, I64, I, I, F]
        L.or_gelu_tanh_mul_inplace.argtypes = [P, P, I64]
        L.or_rope_apply.argtypes = [P, I, I, P, I64, ctypes.c_uint32, F, I, I]
        L.or_gqa_attention.argtypes = [P, P, P, I64, I64, I64, I, I, I, P]
        L.or_gqa_attention_rows.argtypes = [P, P, P, I64, I64, I64, I, I, I, P]
        L.or_gqa_attention_rows_batch.argtypes = [P, P, P, I64, P, I64, I64, I, I, I, P, I]
        L.or_logits_top_k.argtypes = [I, P, I64, I64, P, I, F, P, P, P, P, P, I]
        L.or_mix64.argtypes = [U64, U64]
        L.or_mix64.restype = U64
        L.or_tensor_key.argtypes = [U64, ctypes.c_char_p]
        L.or_tensor_key.restype = U64
        L.or_synth_normal.argtypes = [U64, U64]
        L.or_synth_normal.restype = F
        L.or_synth_tensor.argtypes = [I, U64, I64, I64, F, F, P, I]
        L.or_fp16_to_f32.argtypes = [ctypes.c_uint16]
        L.or_fp16_to_f32.restype = F
        L.or_f32_to_fp16.argtypes = [F]
        L.or_f32_to_fp16.restype = ctypes.c_uint16
        self.L = L


_LIB = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        _LIB = _Lib()
    return _LIB.L


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


# ---------------------------------------------------------------- kernels
def dequantize_rows(t: int, raw: np.ndarray, n_rows: int, in_dim: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.empty((n_rows, in_dim), np.float32)
    if lib().or_dequantize_rows(t, _p(raw), n_rows, in_dim, _p(out)) != 0:
        raise ValueError("dequantize shape mismatch")
    return out


def matmul(t: int, raw: np.ndarray, out_dim: int, in_dim: int, x: np.ndarray) -> np.ndarray:
    """Token-major y[T, out_dim] (real_math.rs matmul_quantized_many_refs_range_token_major)."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    if x.shape[1] != in_dim:
        raise ValueError("input width mismatch")
    y = np.empty((x.shape[0], out_dim), np.float32)
    if lib().or_matmul(t, _p(raw), out_dim, in_dim, _p(x), x.shape[0], _p(y), _threads()) != 0:
        raise ValueError("matmul shape mismatch")
    return y


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float = EPS) -> np.ndarray:
    x = np.array(x, np.float32, copy=True, order="C")
    w = np.ascontiguousarray(w, np.float32)
    for row in x.reshape(-1, x.shape[-1]):
        lib().or_rms_norm_inplace(_p(row), row.shape[0], _p(w), w.shape[0], eps)
    return x


def per_head_rms_norm(x: np.ndarray, w, n_heads: int, head_dim: int, eps: float = EPS) -> np.ndarray:
    x = np.array(x, np.float32, copy=True, order="C")
    if w is not None:
        w = np.ascontiguousarray(w, np.float32)
    for row in x.reshape(-1, n_heads * head_dim):
        lib().or_per_head_rms_norm(_p(row), None if w is None else _p(w), 0 if w is None else w.shape[0],
                                   n_heads, head_dim, eps)
    return x


def gelu_tanh_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.array(g, np.float32, copy=True, order="C")
    u = np.ascontiguousarray(u, np.float32)
    lib().or_gelu_tanh_mul_inplace(_p(g), _p(u), g.size)
    return g


def rope(x: np.ndarray, n_heads: int, head_dim: int, freqs, position: int, theta: float,
         rotary_dim: int | None = None, proportional: bool = False) -> np.ndarray:
    x = np.array(x, np.float32, copy=True, order="C")
    f = np.ascontiguousarray(freqs if freqs is not None else np.zeros(0), np.float32)
    lib().or_rope_apply(_p(x), n_heads, head_dim, _p(f), f.shape[0], position, theta,
                        head_dim if rotary_dim is None else rotary_dim, int(proportional))
    return x


def _row_pointers(rows) -> np.ndarray:
    ptr = np.empty(len(rows), np.uintp)
    for i, r in enumerate(rows):
        if r.dtype != np.float32 or not r.flags.c_contiguous:
            raise ValueError("cached rows must be contiguous float32")
        ptr[i] = r.ctypes.data
    return ptr


def gqa_attention_rows(q: np.ndarray, krows: list, vrows: list, n_heads: int, n_kv: int, head_dim: int,
                       limit: int = -1, window: int = 0) -> np.ndarray:
    """gqa_attention over a cache held as one array per position (read in place, no copy)."""
    q = np.ascontiguousarray(q, np.float32)
    kp, vp = _row_pointers(krows), _row_pointers(vrows)
    out = np.empty(n_heads * head_dim, np.float32)
    lib().or_gqa_attention_rows(_p(q), _p(kp), _p(vp), len(krows), limit, window, n_heads, n_kv, head_dim, _p(out))
    return out


def gqa_attention_rows_batch(qs: np.ndarray, krows: list, vrows: list, n_heads: int, n_kv: int, head_dim: int,
                             limits, window: int = 0) -> np.ndarray:
    """gqa_attention_rows for every query row of qs [T][n_heads*head_dim], query t seeing
    limits[t] cached positions (threads over queries; each query's arithmetic is unchanged)."""
    qs = np.ascontiguousarray(qs, np.float32)
    lim = np.ascontiguousarray(limits, np.int64)
    kp, vp = _row_pointers(krows), _row_pointers(vrows)
    out = np.empty((qs.shape[0], n_heads * head_dim), np.float32)
    lib().or_gqa_attention_rows_batch(_p(qs), _p(kp), _p(vp), len(krows), _p(lim), qs.shape[0], window, n_heads,
                                      n_kv, head_dim, _p(out), _threads())
    return out


def gqa_attention(q: np.ndarray, kc: np.ndarray, vc: np.ndarray, n_heads: int, n_kv: int, head_dim: int,
                  limit: int = -1, window: int = 0) -> np.ndarray:
    q = np.ascontiguousarray(q, np.float32)
    kc = np.ascontiguousarray(kc, np.float32)
    vc = np.ascontiguousarray(vc, np.float32)
    out = np.empty(n_heads * head_dim, np.float32)
    lib().or_gqa_attention(_p(q), _p(kc), _p(vc), kc.shape[0], limit, window, n_heads, n_kv, head_dim, _p(out))
    return out


def logits_top_k(t: int, raw: np.ndarray, vocab: int, hidden: int, h: np.ndarray, k: int = 0,
                 cap: float = 30.0, want_all: bool = False):
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    h = np.ascontiguousarray(h, np.float32)
    am = np.zeros(1, np.int64)
    asc = np.zeros(1, np.float32)
    ti = np.zeros(max(k, 1), np.int64)
    ts = np.zeros(max(k, 1), np.float32)
    allsc = np.empty(vocab, np.float32) if want_all else None
    rc = lib().or_logits_top_k(t, _p(raw), vocab, hidden, _p(h), k, cap, _p(am), _p(asc), _p(ti), _p(ts),
                               None if allsc is None else _p(allsc), _threads())
    if rc != 0:
        raise ValueError("logits shape mismatch")
    top = [(int(i), float(s)) for i, s in zip(ti[:k], ts[:k]) if i >= 0]
    return int(am[0]), float(asc[0]), top, allsc


def fp16_round(a: np.ndarray) -> np.ndarray:
    """Round f32 values to fp16 precision (used to emulate an fp16 KV cache)."""
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


# ---------------------------------------------------------------- synthetic model
def tensor_key(seed: int, name: str) -> int:
    return int(lib().or_tensor_key(seed & (2**64 - 1), name.encode()))


def synth_tensor(t: int, key: int, n_rows: int, in_dim: int, sigma: float, mean: float = 0.0) -> np.ndarray:
    out = np.empty(n_rows * bytes_per_row(t, in_dim), np.uint8)
    if lib().or_synth_tensor(t, key, n_rows, in_dim, sigma, mean, _p(out), _threads()) != 0:
        raise ValueError("bad synthetic tensor shape")
    return out


def synth_tokens(seed: int, name: str, n: int, vocab: int) -> np.ndarray:
    key = tensor_key(seed, name)
    return np.array([int(lib().or_mix64(key, i)) % vocab for i in range(n)], np.uint32)


def synth_normal_f32(seed: int, name: str, n: int, sigma: float = 1.0) -> np.ndarray:
    raw = synth_tensor(F32, tensor_key(seed, name), 1, n, sigma)
    return raw.view(np.float32).copy()


@dataclass
class ModelSpec:
    """Gemma-style decoder with GGUF tensor names (real_forward.rs:1483-1793).

    Defaults are the 42-layer Q4_K_M shape of the graded configs: d_model 2560,
    8 q heads / 4 kv heads of 256, GeGLU FFN 10240, vocab 262144, tied fp16 embedding.
    """
    hidden: int = 2560
    n_heads: int = 8
    n_kv: int = 4
    head_dim: int = 256
    ffn: int = 10240
    vocab: int = 262144
    n_layers: int = 42
    seed: int = 0x5EED
    rope_theta: float = 10000.0
    w_sigma: float = 0.02        # fp16 d/dmin ~ |N(0, 0.02)|
    embd_sigma: float = 0.02     # tied embedding ~ N(0, 0.02)
    norm_sigma: float = 0.05     # norm weights 1 + N(0, 0.05)
    types: dict = field(default_factory=lambda: {
        "attn_q": Q4_K, "attn_k": Q4_K, "attn_v": Q6_K, "attn_output": Q4_K,
        "ffn_gate": Q4_K, "ffn_up": Q4_K, "ffn_down": Q6_K, "token_embd": F16})
    ple_dim: int = 0             # > 0: per-layer embedding inputs (PLE) of this width, F16 matrices

    @property
    def q_dim(self):
        return self.n_heads * self.head_dim

    @property
    def k_dim(self):
        return self.n_kv * self.head_dim

    def layer_tensor_shapes(self, i: int):
        """(name, ggml_type, dims [in, out]) for layer i, GGUF order."""
        H, Q, K, F, D = self.hidden, self.q_dim, self.k_dim, self.ffn, self.head_dim
        p = f"blk.{i}"
        t = self.types
        return [
            (f"{p}.attn_norm.weight", F32, [H]),
            (f"{p}.attn_q.weight", t["attn_q"], [H, Q]),
            (f"{p}.attn_k.weight", t["attn_k"], [H, K]),
            (f"{p}.attn_v.weight", t["attn_v"], [H, K]),
            (f"{p}.attn_q_norm.weight", F32, [D]),
            (f"{p}.attn_k_norm.weight", F32, [D]),
            (f"{p}.attn_output.weight", t["attn_output"], [Q, H]),
            (f"{p}.post_attention_norm.weight", F32, [H]),
            (f"{p}.ffn_norm.weight", F32, [H]),
            (f"{p}.ffn_gate.weight", t["ffn_gate"], [H, F]),
            (f"{p}.ffn_up.weight", t["ffn_up"], [H, F]),
            (f"{p}.ffn_down.weight", t["ffn_down"], [F, H]),
            (f"{p}.post_ffw_norm.weight", F32, [H]),
        ] + ([(f"{p}.inp_gate.weight", F16, [H, self.ple_dim]), (f"{p}.proj.weight", F16, [self.ple_dim, H]),
              (f"{p}.post_norm.weight", F32, [H])] if self.ple_dim else [])

    def stage_tensor_shapes(self, start: int, end: int, is_head: bool, is_tail: bool):
        out = []
        if is_head or is_tail:
            out.append(("token_embd.weight", self.types["token_embd"], [self.hidden, self.vocab]))
        out.append(("rope_freqs.weight", F32, [self.head_dim // 2]))
        if self.ple_dim:  # shared auxiliary tensors (gguf.rs:774-781): every stage holds them
            P = self.ple_dim * self.n_layers
            out += [("per_layer_token_embd.weight", F16, [P, self.vocab]),
                    ("per_layer_model_proj.weight", F16, [self.hidden, P]),
                    ("per_layer_proj_norm.weight", F32, [self.ple_dim])]
        for i in range(start, end + 1):
            out.extend(self.layer_tensor_shapes(i))
        if is_tail:
            out.append(("output_norm.weight", F32, [self.hidden]))
        return out

    def synth(self, name: str, t: int, dims) -> np.ndarray:
        """Bytes of one synthetic tensor (same spec as the device generator)."""
        in_dim = dims[0]
        rows = int(np.prod(dims[1:])) if len(dims) > 1 else 1
        key = tensor_key(self.seed, name)
        if name == "rope_freqs.weight":
            return np.ones(in_dim, np.float32).view(np.uint8).copy()
        if t == F32:  # norm weights
            return synth_tensor(F32, key, rows, in_dim, self.norm_sigma, 1.0)
        if name in ("token_embd.weight", "per_layer_token_embd.weight"):
            return synth_tensor(t, key, rows, in_dim, self.embd_sigma)
        return synth_tensor(t, key, rows, in_dim, self.w_sigma)


def synth_stage(spec: ModelSpec, start: int, end: int, is_head: bool, is_tail: bool) -> dict:
    """name -> (ggml_type, dims, bytes)."""
    return {n: (t, d, spec.synth(n, t, d)) for n, t, d in spec.stage_tensor_shapes(start, end, is_head, is_tail)}


# ---------------------------------------------------------------- packed stage files
def write_pack(directory, stage_name: str, role: str, stage_index: int, tensors: dict,
               model_name: str = "synthetic-gemma") -> Path:
    """Write `<stage>-required.index.json` + `.pack` (PackedStageIndex, lib.rs:2908-2927).
    Tensors are contiguous in insertion order, as validate_offsets requires (lib.rs:3729-3750)."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    index_path = directory / f"{stage_name}-required.index.json"
    pack_path = directory / f"{stage_name}-required.pack"
    entries, off = [], 0
    with open(pack_path, "wb") as f:
        for name, (t, dims, data) in tensors.items():
            b = np.ascontiguousarray(data).view(np.uint8)
            f.write(b.tobytes())
            entries.append({"name": name, "pack_offset": off, "byte_len": int(b.size), "source_file_offset": 0,
                            "dimensions": [int(d) for d in dims], "ggml_type": int(t)})
            off += int(b.size)
    index = {"model_name": model_name, "architecture": "gemma4", "stage_index": stage_index, "role": role,
             "total_bytes": off, "tensor_count": len(entries), "tensors": entries}
    index_path.write_text(json.dumps(index, indent=2))
    return index_path


def load_pack(index_path) -> dict:
    """PackedStageArtifact::load + validate_offsets (lib.rs:3645-3675, :3729-3750)."""
    index_path = Path(index_path)
    if not index_path.name.endswith(".index.json"):
        raise ValueError("Packed stage index must end with .index.json")
    index = json.loads(index_path.read_text())
    pack = index_path.with_name(index_path.name[: -len(".index.json")] + ".pack")
    if not pack.exists():
        raise FileNotFoundError(f"Packed stage file {pack} does not exist")
    if pack.stat().st_size != index["total_bytes"]:
        raise ValueError("Packed stage size does not match index total_bytes")
    mm = np.memmap(pack, np.uint8, "r")
    out, expected = {}, 0
    for e in index["tensors"]:
        if e["pack_offset"] != expected:
            raise ValueError(f"Packed tensor {e['name']} has pack_offset {e['pack_offset']} but expected {expected}")
        expected += e["byte_len"]
        out[e["name"]] = (e["ggml_type"], e["dimensions"], mm[e["pack_offset"]: e["pack_offset"] + e["byte_len"]])
    if expected != index["total_bytes"]:
        raise ValueError("Packed tensor coverage does not match total_bytes")
    return out


# ---------------------------------------------------------------- stage backend
@dataclass
class Layout:
    """StageLayout (lib.rs:212-219)."""
    model_id: str
    stage_id: str
    start_layer: int
    end_layer: int
    is_head: bool
    is_tail: bool


class OracleStage:
    """RealGemmaBackend semantics with an explicit KV cache.

    The reference drops its KV on single-token steps when the model has no PLE
    (real_forward.rs:1006-1011, :2072-2076) and pins "incremental decode == full
    rerun" (real_forward.rs:3129); this oracle keeps the KV explicitly, which the
    tests check against a full rerun.  ``kv_fp16`` rounds stored K/V to fp16 to
    mirror a device fp16 cache; False is the reference's f32 cache.
    """

    def __init__(self, tensors: dict, layout: Layout, rope_theta: float = 1e6, softcap: float = 30.0,
                 kv_fp16: bool = False):
        self.t = tensors
        self.layout = layout
        self.kv_fp16 = kv_fp16
        self.softcap = softcap
        self.rope_theta = rope_theta
        layers = sorted({int(n.split(".")[1]) for n in tensors if n.startswith("blk.")})
        self.layers = layers
        l0 = f"blk.{layers[0]}" if layers else None
        # config inference, real_forward.rs:2258-2283 and real_math.rs:2869-2907
        self.hidden = tensors[f"{l0}.attn_q.weight"][1][0] if l0 else 2560
        q_dim = tensors[f"{l0}.attn_q.weight"][1][1] if l0 else 2048
        k_dim = tensors[f"{l0}.attn_k.weight"][1][1] if l0 else 512
        hd = None
        qn = tensors.get(f"{l0}.attn_q_norm.weight")
        if qn is not None and q_dim % qn[1][0] == 0 and k_dim % qn[1][0] == 0:
            hd = qn[1][0]
        if hd is None:
            hd = next((c for c in (256, 128, 64) if q_dim % c == 0 and k_dim % c == 0 and
                       q_dim // c >= k_dim // c and (q_dim // c) % (k_dim // c) == 0), math.gcd(q_dim, k_dim))
        self.head_dim, self.n_heads, self.n_kv = hd, q_dim // hd, max(1, k_dim // hd)
        rf = tensors.get("rope_freqs.weight")
        self.rope_freqs = None if rf is None else self._f32(rf)
        if self._e4b():
            # should_use_packed_rope_freqs (real_forward.rs:158-160): RoPE on, no frequency scales
            self.rope_freqs = np.zeros(0, np.float32)
            for i in layers:  # validate_stage_split_constraints (real_forward.rs:1459-1481)
                src = self._attention_config(i)[3]
                if src is not None and not (layout.start_layer <= src <= layout.end_layer):
                    raise ValueError(f"real_forward stage {layout.stage_id} (layers {layout.start_layer}-"
                                     f"{layout.end_layer}) is unsupported for {layout.model_id}: layer {i} requires "
                                     f"shared KV from layer {src} outside this stage")
        # PLE (real_forward.rs:2320-2338): width from per_layer_proj_norm, layer count from the projection
        pn, mp = tensors.get("per_layer_proj_norm.weight"), tensors.get("per_layer_model_proj.weight")
        self.ple_dim = int(pn[1][0]) if pn is not None else 0
        self.ple_layers = int(mp[1][1]) // self.ple_dim if self.ple_dim and mp is not None else 0
        self.last_ple = None
        self.sessions: dict[str, dict] = {}

    def compute_ple_inputs(self, ids, embeds: np.ndarray) -> np.ndarray:
        """compute_ple_inputs (real_forward.rs:1157-1299) for every model layer: [T][layers][ple_dim].
        The model projection of the scaled token embedding, times hidden^-1/2, RMS-normed per ple_dim
        chunk with per_layer_proj_norm (eps 1e-6), plus the token's per-layer embedding row times
        sqrt(ple_dim), all times 2^-1/2."""
        P, L = self.ple_dim, self.ple_layers
        if P == 0 or L == 0:
            raise ValueError(f"PLE not configured (ple_dim={P}, num_layers={L})")
        proj = self._mm("per_layer_model_proj.weight", embeds)  # [T][L*P]
        proj = proj * np.float32(np.float32(embeds.shape[1]) ** np.float32(-0.5))
        norm = self._f32(self.t["per_layer_proj_norm.weight"])
        proj = rms_norm(proj.reshape(-1, P), norm, 1e-6).reshape(len(ids), L * P)  # rms_norm_chunked_inplace
        t, dims, raw = self.t["per_layer_token_embd.weight"]
        rb = bytes_per_row(t, dims[0])
        embed_scale, combine_scale = np.float32(math.sqrt(P)), np.float32(2.0 ** -0.5)
        out = np.empty((len(ids), L * P), np.float32)
        for i, tid in enumerate(ids):
            row = dequantize_rows(t, raw[int(tid) * rb:(int(tid) + 1) * rb], 1, dims[0])[0]
            out[i] = (proj[i] + row * embed_scale) * combine_scale
        return out.reshape(len(ids), L, P)

    def _e4b(self) -> bool:
        return ("gemma-4-e4b" in self.layout.model_id and self.hidden == 2560 and self.head_dim in (256, 512))

    def _attention_config(self, i: int):
        """layer_attention_config_for_layout (real_forward.rs:1407-1457): (rope base, rotary dims,
        proportional, shared-KV source layer or None, sliding window or 0)."""
        if not self._e4b():
            return self.rope_theta, self.head_dim, False, None, 0
        if i % 6 == 5:
            return 1_000_000.0, self.head_dim // 4, True, (23 if i >= 24 else None), 0
        return 10_000.0, self.head_dim, False, (22 if i >= 24 else None), 512

    @staticmethod
    def _f32(entry) -> np.ndarray:
        t, dims, raw = entry
        if t != F32:
            raise ValueError("Expected F32 tensor")  # real_forward.rs:478-488
        return np.frombuffer(np.ascontiguousarray(raw).tobytes(), np.float32)

    def _mm(self, name: str, x: np.ndarray) -> np.ndarray:
        t, dims, raw = self.t[name]
        return matmul(t, raw, dims[1], dims[0], x)

    def embed(self, ids) -> np.ndarray:
        """embed_tokens, real_forward.rs:848-871: F16 row dequant, then * sqrt(hidden)."""
        t, dims, raw = self.t["token_embd.weight"]
        H, V = dims
        rb = bytes_per_row(t, H)
        out = np.empty((len(ids), H), np.float32)
        scale = np.float32(math.sqrt(H))
        for i, tid in enumerate(ids):
            if tid >= V:
                raise ValueError(f"Token ID {tid} exceeds vocab size {V}")
            out[i] = dequantize_rows(t, raw[int(tid) * rb:(int(tid) + 1) * rb], 1, H)[0] * scale
        return out

    def _layer(self, i: int, states: np.ndarray, pos0: int, kv: dict, ple=None) -> np.ndarray:
        """forward_layer_seq, real_forward.rs:1483-1793 (generic schedule, no PLE)."""
        p = f"blk.{i}"
        H, nh, nkv, hd = self.hidden, self.n_heads, self.n_kv, self.head_dim
        T = states.shape[0]
        theta, rot, prop, src, win = self._attention_config(i)
        x = rms_norm(states, self._f32(self.t[f"{p}.attn_norm.weight"]))
        q_all = self._mm(f"{p}.attn_q.weight", x)
        q_all = per_head_rms_norm(q_all, self._f32(self.t[f"{p}.attn_q_norm.weight"]), nh, hd)
        if src is None:
            k_all = self._mm(f"{p}.attn_k.weight", x)
            v_all = self._mm(f"{p}.attn_v.weight", x)
            k_all = per_head_rms_norm(k_all, self._f32(self.t[f"{p}.attn_k_norm.weight"]), nkv, hd)
            v_all = per_head_rms_norm(v_all, None, nkv, hd)
            kc, vc = kv.setdefault(i, ([], []))
        else:  # shared KV: the source layer's cache, already holding these positions (:1561-1640)
            kc, vc = kv[src]
        qs = np.empty((T, nh * hd), np.float32)
        for t in range(T):
            q = q_all[t]
            if self.rope_freqs is not None:
                q = rope(q, nh, hd, self.rope_freqs, pos0 + t, theta, rot, prop)
            qs[t] = q
            if src is None:
                k = k_all[t]
                if self.rope_freqs is not None:
                    k = rope(k, nkv, hd, self.rope_freqs, pos0 + t, theta, rot, prop)
                v = v_all[t]
                if self.kv_fp16:
                    k, v = fp16_round(k), fp16_round(v)
                kc.append(k)
                vc.append(v)
        # token t sees positions [0, pos0 + t] (its own k/v were appended above)
        att = gqa_attention_rows_batch(qs, kc, vc, nh, nkv, hd, pos0 + 1 + np.arange(T), window=win)
        o = self._mm(f"{p}.attn_output.weight", att)
        o = rms_norm(o, self._f32(self.t[f"{p}.post_attention_norm.weight"]))
        states = o + states
        x = rms_norm(states, self._f32(self.t[f"{p}.ffn_norm.weight"]))
        g = self._mm(f"{p}.ffn_gate.weight", x)
        u = self._mm(f"{p}.ffn_up.weight", x)
        a = gelu_tanh_mul(g, u)
        d = self._mm(f"{p}.ffn_down.weight", a)
        d = rms_norm(d, self._f32(self.t[f"{p}.post_ffw_norm.weight"]))
        states = d + states
        ig, pj = self.t.get(f"{p}.inp_gate.weight"), self.t.get(f"{p}.proj.weight")
        if ig is not None and pj is not None and ple is not None:  # real_forward.rs:1753-1778
            gated = gelu_tanh_mul(self._mm(f"{p}.inp_gate.weight", states), ple)
            pr = self._mm(f"{p}.proj.weight", gated)
            pn = self.t.get(f"{p}.post_norm.weight")
            if pn is not None:
                pr = rms_norm(pr, self._f32(pn))
            states = pr + states
        sc = self.t.get(f"{p}.layer_output_scale.weight")
        if sc is not None:
            states = states * self._f32(sc)[0]
        return states

    def run_layers(self, states: np.ndarray, pos0: int, kv: dict, ple_all=None) -> np.ndarray:
        """run_stage_layers (real_forward.rs:1992-2052): PLE inputs by global layer index."""
        for i in self.layers:
            states = self._layer(i, states, pos0, kv, None if ple_all is None else ple_all[:, i, :])
        return states

    def _session(self, req: str, n: int, fresh: bool) -> dict:
        s = self.sessions.get(req)
        if fresh or s is None:
            s = {"seq_len": 0, "kv": {}}
            self.sessions[req] = s
        return s

    def begin_token_ids(self, req: str, ids, append: bool = False) -> np.ndarray:
        """Head ingress (real_forward.rs:988-1121). A multi-token call starts a new
        session; a single-token call (or append=True) continues the session's KV."""
        if not self.layout.is_head:
            raise ValueError("Only the head stage may accept prompt ingress")
        if len(ids) == 0:
            raise ValueError("Empty prompt")
        s = self._session(req, len(ids), fresh=(len(ids) > 1 and not append))
        emb = self.embed(ids)
        # the head computes every layer's PLE inputs; later stages receive them in the aux section
        self.last_ple = self.compute_ple_inputs(ids, emb) if self.ple_dim else None
        out = self.run_layers(emb, s["seq_len"], s["kv"], self.last_ple)
        s["seq_len"] += len(ids)
        return out

    def continue_forward(self, req: str, hidden: np.ndarray, append: bool = False, ple_all=None) -> np.ndarray:
        """continue_forward_inner (real_forward.rs:2054-2254), same session rule; ple_all: the
        per-layer inputs [T][layers][ple_dim] from the head (the aux section's PLE part)."""
        if self.layout.is_head:
            raise ValueError("Head stage should use begin_prompt, not continue_forward")
        hidden = np.ascontiguousarray(np.atleast_2d(hidden), np.float32)
        s = self._session(req, hidden.shape[0], fresh=(hidden.shape[0] > 1 and not append))
        out = self.run_layers(hidden, s["seq_len"], s["kv"], ple_all)
        s["seq_len"] += hidden.shape[0]
        return out

    def fill_session_synthetic(self, req: str, n_pos: int, seed: int = 0):
        """A session whose cache holds n_pos seeded N(0,1) keys and values in every layer that has
        its own cache (benchmarks: a decode step's cost does not depend on the cached values)."""
        rng = np.random.default_rng(seed)
        kv = {}
        width = self.n_kv * self.head_dim
        for i in self.layers:
            if self._attention_config(i)[3] is None:
                kv[i] = ([r for r in rng.standard_normal((n_pos, width), np.float32)],
                         [r for r in rng.standard_normal((n_pos, width), np.float32)])
        self.sessions[req] = {"seq_len": n_pos, "kv": kv}

    def fill_session_like_device(self, req: str, n_pos: int, seed: int, kv_f32: bool):
        """The cache that sfc_session_fill_synthetic writes on the device, restated: for the
        stage's i-th layer (stage order) that has its own cache, part p (0 = K, 1 = V) of kv head h
        holds synth_tensor(F32 if kv_f32 else F16, tensor_key(seed, f"kv.{i}.{p}.{h}"), n_pos,
        head_dim, sigma 1) as [position][head_dim]; a cached row is the heads side by side."""
        kv = {}
        t = F32 if kv_f32 else F16
        dt = np.float32 if kv_f32 else np.float16
        for li, i in enumerate(self.layers):
            if self._attention_config(i)[3] is not None:
                continue
            parts = []
            for part in range(2):
                heads = [np.frombuffer(synth_tensor(t, tensor_key(seed, f"kv.{li}.{part}.{kh}"), n_pos, self.head_dim,
                                                    1.0).tobytes(), dt).astype(np.float32).reshape(n_pos, self.head_dim)
                         for kh in range(self.n_kv)]
                rows = np.ascontiguousarray(np.concatenate(heads, axis=1))
                parts.append([np.ascontiguousarray(r) for r in rows])
            kv[i] = (parts[0], parts[1])
        self.sessions[req] = {"seq_len": n_pos, "kv": kv}

    def rollback(self, req: str, keep: int):
        s = self.sessions[req]
        if keep > s["seq_len"]:
            raise ValueError("keep_count exceeds session length")
        for kc, vc in s["kv"].values():
            del kc[keep:]
            del vc[keep:]
        s["seq_len"] = keep

    def logits_entry(self):
        return self.t.get("output.weight") or self.t["token_embd.weight"]  # real_forward.rs:803-816

    def sample_tail(self, hidden_last: np.ndarray, top_k: int = 0, want_all: bool = False):
        """sample_hidden_state_with_trace (real_forward.rs:904-986): output_norm, tied
        logits with softcap 30, argmax (lowest index wins ties)."""
        if not self.layout.is_tail:
            raise ValueError("Only the tail stage may sample")
        h = np.ascontiguousarray(hidden_last, np.float32).reshape(-1)
        on = self.t.get("output_norm.weight")
        if on is not None:
            h = rms_norm(h, self._f32(on))
        t, dims, raw = self.logits_entry()
        H = self.hidden
        vocab = dims[1] if dims[0] == H else dims[0]
        return logits_top_k(t, raw, vocab, H, h, top_k, self.softcap, want_all)


# ---------------------------------------------------------------- draft-tree verification
# No counterpart in the reference, which verifies a chain greedily
# (crates/llama-stage-backend/src/lib.rs:2143-2185); these restate the library's tree rule and its
# seeded temperature sampler so the GPU path has a CPU check.

_M64 = (1 << 64) - 1


def mix64(key: int, ctr: int) -> int:
    """SplitMix64 finaliser of key + (ctr + 1) * golden ratio (the synthetic-weight hash)."""
    z = (key + (ctr + 1) * 0x9E3779B97F4A7C15) & _M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    return z ^ (z >> 31)


def sampling_uniform(seed: int, row: int) -> np.float32:
    """The per-row uniform in [0, 1): top 24 bits of mix64(seed, row), times 2^-24."""
    return np.float32(mix64(seed, row) >> 40) * np.float32(1.0 / 16777216.0)


def sample_temperature(scores: np.ndarray, temperature: float, seed: int, row: int, segments: int = 1024):
    """Draw from softmax(scores / temperature) as the GPU sampler does: float32 weights
    exp((s - max) * (1/T)) summed in index order over `segments` contiguous segments, segment
    prefixes summed in order, target = u * total, and the owning segment walked from its prefix.
    Returns the drawn index."""
    s = np.asarray(scores, np.float32)
    v = s.shape[0]
    seg = (v + segments - 1) // segments
    mx = np.float32(s.max())
    inv_t = np.float32(1.0) / np.float32(temperature)
    w = np.exp((s - mx) * inv_t).astype(np.float32)
    seg_sums = np.zeros(segments, np.float32)
    for j in range(segments):
        acc = np.float32(0.0)
        for x in w[j * seg:min((j + 1) * seg, v)]:
            acc = np.float32(acc + x)
        seg_sums[j] = acc
    pre = np.zeros(segments, np.float32)
    run = np.float32(0.0)
    for j in range(segments):
        pre[j] = run
        run = np.float32(run + seg_sums[j])
    target = np.float32(sampling_uniform(seed, row) * run)
    pick = -1
    for j in range(segments):
        lo, hi = j * seg, min((j + 1) * seg, v)
        if lo < hi and pre[j] <= target < np.float32(pre[j] + seg_sums[j]):
            r = pre[j]
            pick = hi - 1
            for i in range(lo, hi):
                r = np.float32(r + w[i])
                if r > target:
                    pick = i
                    break
            break
    if pick < 0:
        pick = v - 1
    return pick


def tree_walk(parent, node_tokens, drawn):
    """From the root, move to the first child whose token equals the token drawn at the current
    node; stop when none does.  Returns (path of node indices from 0, token drawn at the stop)."""
    n = len(parent)
    path, cur = [0], 0
    while True:
        nxt = next((c for c in range(cur + 1, n) if parent[c] == cur and node_tokens[c] == drawn[cur]), -1)
        if nxt < 0:
            return path, int(drawn[cur])
        path.append(nxt)
        cur = nxt


def bfs_tree(branching, max_nodes: int):
    """Parent array of a breadth-first tree with the given branching per level (root = node 0),
    truncated to max_nodes."""
    parent, frontier = [-1], [0]
    for b in branching:
        nxt = []
        for p in frontier:
            for _ in range(b):
                if len(parent) >= max_nodes:
                    return parent
                parent.append(p)
                nxt.append(len(parent) - 1)
        frontier = nxt
    return parent


# ---------------------------------------------------------------- stage aux section
def prefix_hashes(token_ids) -> list:
    """prefix_hashes (real_forward.rs:319-333): 64-bit FNV-1a over each token id's little-endian
    bytes, one running hash per prefix."""
    h, out = 0xCBF29CE484222325, []
    for tid in token_ids:
        for b in int(tid).to_bytes(4, "little"):
            h = ((h ^ b) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
        out.append(h)
    return out


def encode_prompt_aux(ple_all, ple_dim: int, hashes=()) -> bytes | None:
    """encode_prompt_aux (real_forward.rs:1852-1894): "rsa1" | u32 seq_len | u32 layers | u32 ple_dim |
    u32 n_hashes | f32 [seq][layers][ple_dim] | u64 hashes; None when both parts are empty."""
    seq = 0 if ple_all is None else int(ple_all.shape[0])
    layers = 0 if ple_all is None or seq == 0 else int(ple_all.shape[1])
    if seq * layers * ple_dim == 0 and not hashes:
        return None
    head = b"rsa1" + struct.pack("<IIII", seq, layers, ple_dim, len(hashes))
    body = b"" if ple_all is None else np.ascontiguousarray(ple_all, np.float32).tobytes()
    return head + body + b"".join(struct.pack("<Q", h) for h in hashes)


def decode_prompt_aux(b: bytes):
    """decode_prompt_aux (real_forward.rs:1896-1990): (ple_all [seq][layers][ple_dim], hashes) from an
    "rsa1" section, or from the older "rpl1" one (PLE only)."""
    if len(b) >= 20 and b[:4] == b"rsa1":
        seq, layers, pdim, nh = struct.unpack_from("<IIII", b, 4)
        want = 20 + seq * layers * pdim * 4 + nh * 8
        if len(b) != want:
            raise ValueError(f"Invalid prompt-aux byte length {len(b)} (expected {want})")
        ple = np.frombuffer(b, np.float32, seq * layers * pdim, 20).reshape(seq, layers, pdim)
        off = 20 + seq * layers * pdim * 4
        return ple, list(struct.unpack_from(f"<{nh}Q", b, off))
    if len(b) < 16 or b[:4] != b"rpl1":
        raise ValueError("Invalid prompt-aux payload")
    seq, layers, pdim = struct.unpack_from("<III", b, 4)
    want = 16 + seq * layers * pdim * 4
    if len(b) != want:
        raise ValueError(f"Invalid prompt-aux byte length {len(b)} (expected {want})")
    return np.frombuffer(b, np.float32, seq * layers * pdim, 16).reshape(seq, layers, pdim), []
