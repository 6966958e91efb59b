"""stagefwd — Python binding of the B200 stage-forward backend (libstagefwd.so, C ABI in
include/stagefwd.h).

Mirrors the reference's stage API (crates/stage-forward-lab/src/lib.rs:4663-4674,
`StageForwardBackend`, implemented by `RealGemmaBackend` in real_forward.rs) so that
parity tests and benchmarks read like the reference's own: `load_layout`,
`begin_token_ids`, `continue_forward`, `sample_tail`, plus the kernel-level entry points.

There is no CPU fallback: importing this module fails if the CUDA library is missing.
Device buffers are torch CUDA tensors (torch is only the allocator/stream plumbing).
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "libstagefwd.so"
HEADER_PATH = _HERE.parent.parent / "include" / "stagefwd.h"

F32, F16, Q4_K, Q5_K, Q6_K, BF16 = 0, 1, 12, 13, 14, 30

if not LIB_PATH.exists():
    raise ImportError(f"{LIB_PATH} is missing: build it with `make -C compute-sharding_b200` "
                      "(the stage backend has no CPU fallback)")

_lib = ctypes.CDLL(str(LIB_PATH))
_P, _I, _I64, _F, _U64, _U32 = (ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float,
                                ctypes.c_uint64, ctypes.c_uint32)


class Layout(ctypes.Structure):
    """StageLayout (lib.rs:212-219)."""
    _fields_ = [("model_id", ctypes.c_char_p), ("stage_id", ctypes.c_char_p), ("start_layer", _U32),
                ("end_layer", _U32), ("is_head", _I), ("is_tail", _I)]


class Options(ctypes.Structure):
    _fields_ = [("rope_theta", _F), ("logit_softcap", _F), ("eps", _F), ("kv_f32", _I), ("max_ctx", _I),
                ("max_sessions", _I), ("max_batch_tokens", _I)]


class SynthSpec(ctypes.Structure):
    _fields_ = [("seed", _U64), ("hidden", _I), ("n_heads", _I), ("n_kv", _I), ("head_dim", _I), ("ffn", _I),
                ("n_layers_total", _I), ("vocab", _I64), ("type_q", _I), ("type_k", _I), ("type_v", _I),
                ("type_o", _I), ("type_gate", _I), ("type_up", _I), ("type_down", _I), ("type_embd", _I),
                ("w_sigma", _F), ("embd_sigma", _F), ("norm_sigma", _F)]


class StageInfo(ctypes.Structure):
    _fields_ = [("hidden", _I), ("n_heads", _I), ("n_kv", _I), ("head_dim", _I), ("ffn", _I), ("n_layers", _I),
                ("vocab", _I64), ("is_head", _I), ("is_tail", _I), ("weight_bytes", _I64), ("kv_bytes", _I64)]


class Profile(ctypes.Structure):
    _fields_ = [("seq_len", _I64), ("layers", _I64), ("embed_us", ctypes.c_double), ("attn_us", ctypes.c_double),
                ("ffn_us", ctypes.c_double), ("logits_us", ctypes.c_double), ("total_us", ctypes.c_double),
                ("kernels", _I64)]


def _sig(name, res, *args):
    f = getattr(_lib, name)
    f.restype = res
    f.argtypes = list(args)
    return f


_sig("sfc_abi_version", _I)
_sig("sfc_last_error", ctypes.c_char_p)
_sig("sfc_device_error", _I, ctypes.POINTER(ctypes.c_uint))
_sig("sfc_kernel_launches", ctypes.c_int64)
_sig("sfc_selftest_bounded_wait", _I, ctypes.c_uint, _I, _P)
_sig("sfc_weight_device_bytes", _I64, _I, _I64, _I64)
_sig("sfc_prepare_weights", _I, _I, _P, _I64, _I64, _P, _P)
_sig("sfc_dequantize_rows", _I, _I, _P, _I64, _I64, _P, _P)
_sig("sfc_matmul", _I, _I, _P, _I64, _I64, _P, _I64, _P, _P)
_sig("sfc_matmul_pair_geglu", _I, _I, _P, _P, _I64, _I64, _P, _I64, _P, _P)
_sig("sfc_rms_norm", _I, _P, _P, _I64, _I64, _F, _P, _P)
_sig("sfc_logits_argmax", _I, _I, _P, _I64, _I64, _P, _I64, _F, _P, _P, _P, _P)
_sig("sfc_synth_tensor", _I, _I, _U64, ctypes.c_char_p, _I64, _I64, _F, _F, _P, _P)
_sig("sfc_stage_open", _I, ctypes.c_char_p, ctypes.POINTER(Layout), ctypes.POINTER(Options), _I, ctypes.POINTER(_P))
_sig("sfc_stage_open_synthetic", _I, ctypes.POINTER(SynthSpec), ctypes.POINTER(Layout), ctypes.POINTER(Options), _I,
     ctypes.POINTER(_P))
_sig("sfc_stage_open_gguf", _I, ctypes.c_char_p, ctypes.POINTER(Layout), ctypes.POINTER(Options), _I,
     ctypes.POINTER(_P))
_sig("sfc_stage_close", _I, _P)
_sig("sfc_stage_get_info", _I, _P, ctypes.POINTER(StageInfo))
_sig("sfc_begin_token_ids", _I, _P, ctypes.c_char_p, _P, _I64, _P)
_sig("sfc_continue_forward", _I, _P, ctypes.c_char_p, _P, _I64, _P)
_sig("sfc_sample_tail", _I, _P, _P, _I64, ctypes.POINTER(_U32), ctypes.POINTER(_F))
_sig("sfc_forward_dev", _I, _P, ctypes.POINTER(ctypes.c_char_p), _P, _I, _P, _P, _P, _I, _P)
_sig("sfc_sample_dev", _I, _P, _P, _I64, _P, _P, _P)
_sig("sfc_verify_greedy", _I, _P, _P, _P, _I64, ctypes.POINTER(_I64), ctypes.POINTER(_U32))
_sig("sfc_sample_temperature", _I, _P, ctypes.c_int64, ctypes.c_int64, ctypes.c_float, ctypes.c_uint64, _P, _P)
_sig("sfc_forward_tree", _I, _P, ctypes.c_char_p, _P, _P, _P, ctypes.c_int64, _P)
_sig("sfc_sample_tree", _I, _P, _P, _P, _P, ctypes.c_int64, ctypes.c_float, ctypes.c_uint64, _P, _P, _P)
_sig("sfc_commit_tree", _I, _P, ctypes.c_char_p, _P, ctypes.c_int64)
_sig("sfc_clear_decode_session", _I, _P, ctypes.c_char_p)
_sig("sfc_rollback_kv", _I, _P, ctypes.c_char_p, _I64)
_sig("sfc_session_len", _I64, _P, ctypes.c_char_p)
_sig("sfc_session_fill_synthetic", _I, _P, ctypes.c_char_p, _I64, _U64)
_sig("sfc_generate_greedy", _I, _P, ctypes.c_char_p, _P, _I64, _I64, _P)
_sig("sfc_last_profile", _I, _P, ctypes.POINTER(Profile))
_PU64 = ctypes.POINTER(_U64)
_sig("sfc_stage_tensor_sections", _I, ctypes.c_char_p, _U64, _PU64, _PU64, _PU64, _PU64)
_sig("sfc_encode_stage_tensor_bytes", _I, ctypes.c_char_p, _U64, ctypes.c_char_p, _U64, _P, _U64, _PU64)
_sig("sfc_continue_forward_bytes", _I, _P, ctypes.c_char_p, ctypes.c_char_p, _U64, _U64, _P, _U64, _PU64)
_sig("sfc_begin_token_ids_bytes", _I, _P, ctypes.c_char_p, _P, _I64, _P, _U64, _PU64)
_sig("sfc_sample_tail_bytes", _I, _P, ctypes.c_char_p, _U64, _U64, ctypes.POINTER(_U32), ctypes.POINTER(_F))

lib = _lib


class StageError(RuntimeError):
    pass


def _check(rc: int, what: str):
    if rc != 0:
        raise StageError(f"{what} failed ({rc}): {_lib.sfc_last_error().decode()}")


def _ptr(t) -> int | None:
    if t is None:
        return None
    if isinstance(t, np.ndarray):
        return t.ctypes.data
    return t.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return stream


def exported_symbols() -> list[str]:
    """Every `sfc_*` function the public header declares."""
    import re
    text = HEADER_PATH.read_text()
    return sorted(set(re.findall(r"\b(sfc_[a-z0-9_]+)\s*\(", text)))


# ---------------------------------------------------------------- hand-off payloads (StageTensor::bytes)
def stage_tensor_byte_sections(payload: bytes) -> tuple[bytes, bytes | None, bool]:
    """stage_tensor_byte_sections (lib.rs:75-96): (hidden bytes, aux bytes or None, framed)."""
    ho, hl, ao, al = _U64(), _U64(), _U64(), _U64()
    rc = _lib.sfc_stage_tensor_sections(payload, len(payload), ctypes.byref(ho), ctypes.byref(hl), ctypes.byref(ao),
                                        ctypes.byref(al))
    if rc not in (0, 1):
        _check(rc, "stage_tensor_byte_sections")
    hidden = payload[ho.value: ho.value + hl.value]
    aux = payload[ao.value: ao.value + al.value] if al.value else None
    return hidden, aux, rc == 0


def encode_stage_tensor_bytes(hidden: bytes, aux: bytes | None = None) -> bytes:
    """encode_stage_tensor_bytes (lib.rs:98-118)."""
    aux = aux or b""
    n = _U64()
    _check(_lib.sfc_encode_stage_tensor_bytes(hidden, len(hidden), aux, len(aux), None, 0, ctypes.byref(n)),
           "encode_stage_tensor_bytes")
    out = ctypes.create_string_buffer(max(int(n.value), 1))
    _check(_lib.sfc_encode_stage_tensor_bytes(hidden, len(hidden), aux, len(aux), out, n.value, ctypes.byref(n)),
           "encode_stage_tensor_bytes")
    return out.raw[: int(n.value)]


# ---------------------------------------------------------------- kernel-level API (torch tensors)
def weight_device_bytes(ggml_type: int, rows: int, in_dim: int) -> int:
    n = _lib.sfc_weight_device_bytes(ggml_type, rows, in_dim)
    if n < 0:
        raise StageError(_lib.sfc_last_error().decode())
    return n


def prepare_weights(ggml_type: int, gguf_dev, rows: int, in_dim: int, stream=None):
    import torch
    out = torch.empty(weight_device_bytes(ggml_type, rows, in_dim) + 16, dtype=torch.uint8, device=gguf_dev.device)
    _check(_lib.sfc_prepare_weights(ggml_type, _ptr(gguf_dev), rows, in_dim, _ptr(out), _stream(stream)),
           "sfc_prepare_weights")
    return out


def dequantize_rows(ggml_type: int, gguf_dev, rows: int, in_dim: int, stream=None):
    import torch
    out = torch.empty((rows, in_dim), dtype=torch.float32, device=gguf_dev.device)
    _check(_lib.sfc_dequantize_rows(ggml_type, _ptr(gguf_dev), rows, in_dim, _ptr(out), _stream(stream)),
           "sfc_dequantize_rows")
    return out


def matmul(ggml_type: int, w_dev, out_dim: int, in_dim: int, x, stream=None):
    import torch
    x = x.contiguous()
    n_tok = x.shape[0] if x.dim() == 2 else 1
    y = torch.empty((n_tok, out_dim), dtype=torch.float32, device=x.device)
    _check(_lib.sfc_matmul(ggml_type, _ptr(w_dev), out_dim, in_dim, _ptr(x), n_tok, _ptr(y), _stream(stream)),
           "sfc_matmul")
    return y


def matmul_pair_geglu(ggml_type: int, w_gate, w_up, out_dim: int, in_dim: int, x, stream=None):
    import torch
    x = x.contiguous()
    n_tok = x.shape[0] if x.dim() == 2 else 1
    y = torch.empty((n_tok, out_dim), dtype=torch.float32, device=x.device)
    _check(_lib.sfc_matmul_pair_geglu(ggml_type, _ptr(w_gate), _ptr(w_up), out_dim, in_dim, _ptr(x), n_tok, _ptr(y),
                                      _stream(stream)), "sfc_matmul_pair_geglu")
    return y


def rms_norm(x, w, eps: float = 1e-6, stream=None):
    import torch
    x = x.contiguous()
    out = torch.empty_like(x)
    _check(_lib.sfc_rms_norm(_ptr(x), _ptr(w), x.numel() // x.shape[-1], x.shape[-1], eps, _ptr(out),
                             _stream(stream)), "sfc_rms_norm")
    return out


def logits_argmax(ggml_type: int, w_dev, vocab: int, dim: int, h, cap: float = 30.0, want_scores: bool = False,
                  stream=None):
    import torch
    h = h.contiguous()
    n_tok = h.shape[0] if h.dim() == 2 else 1
    idx = torch.empty(n_tok, dtype=torch.int64, device=h.device)
    sc = torch.empty(n_tok, dtype=torch.float32, device=h.device)
    allsc = torch.empty((n_tok, vocab), dtype=torch.float32, device=h.device) if want_scores else None
    _check(_lib.sfc_logits_argmax(ggml_type, _ptr(w_dev), vocab, dim, _ptr(h), n_tok, cap, _ptr(allsc), _ptr(idx),
                                  _ptr(sc), _stream(stream)), "sfc_logits_argmax")
    return idx, sc, allsc


def sample_temperature(scores, temperature: float, seed: int, stream=None):
    """Seeded temperature sampling of each row of scores [n][vocab] (sfc_sample_temperature)."""
    import torch
    scores = scores.contiguous()
    out = torch.empty(scores.shape[0], dtype=torch.int64, device=scores.device)
    _check(_lib.sfc_sample_temperature(_ptr(scores), scores.shape[0], scores.shape[1], float(temperature), int(seed),
                                       _ptr(out), _stream(stream)), "sfc_sample_temperature")
    return out


def synth_tensor(ggml_type: int, seed: int, name: str, rows: int, in_dim: int, sigma: float, mean: float = 0.0,
                 device="cuda", stream=None):
    import torch
    from math import prod  # noqa: F401
    rb = {F32: 4 * in_dim, F16: 2 * in_dim, BF16: 2 * in_dim, Q4_K: in_dim // 256 * 144, Q6_K: in_dim // 256 * 210}
    out = torch.empty(rows * rb[ggml_type], dtype=torch.uint8, device=device)
    _check(_lib.sfc_synth_tensor(ggml_type, seed, name.encode(), rows, in_dim, sigma, mean, _ptr(out),
                                 _stream(stream)), "sfc_synth_tensor")
    return out


def kernel_launches() -> int:
    """Compute-kernel launches issued by the library so far (graph replays not counted)."""
    return int(_lib.sfc_kernel_launches())


def device_error() -> int:
    """Read and clear the device error word (0 none, 1 a bounded wait ran out, 2 a bad argument)."""
    c = ctypes.c_uint(0)
    _check(_lib.sfc_device_error(ctypes.byref(c)), "sfc_device_error")
    return c.value


def selftest_bounded_wait(spin_limit: int, complete: bool, stream=None):
    """One bounded mbarrier wait of `spin_limit` polls on a barrier that completes or never does."""
    _check(_lib.sfc_selftest_bounded_wait(spin_limit, int(complete), _stream(stream)), "sfc_selftest_bounded_wait")


# ---------------------------------------------------------------- stage-level API
@dataclass
class ModelShape:
    """Gemma-style stage shape for synthetic stages (defaults: the 42-layer Q4_K_M config)."""
    hidden: int = 2560
    n_heads: int = 8
    n_kv: int = 4
    head_dim: int = 256
    ffn: int = 10240
    vocab: int = 262144
    n_layers: int = 42
    seed: int = 0x5EED
    type_q: int = Q4_K
    type_k: int = Q4_K
    type_v: int = Q6_K
    type_o: int = Q4_K
    type_gate: int = Q4_K
    type_up: int = Q4_K
    type_down: int = Q6_K
    type_embd: int = F16
    w_sigma: float = 0.02
    embd_sigma: float = 0.02
    norm_sigma: float = 0.05

    def spec(self) -> SynthSpec:
        return SynthSpec(self.seed, self.hidden, self.n_heads, self.n_kv, self.head_dim, self.ffn, self.n_layers,
                         self.vocab, self.type_q, self.type_k, self.type_v, self.type_o, self.type_gate, self.type_up,
                         self.type_down, self.type_embd, self.w_sigma, self.embd_sigma, self.norm_sigma)


class CudaStageBackend:
    """StageForwardBackend on B200 (RealGemmaBackend semantics, real_forward.rs:112-2411)."""

    def __init__(self, index_path: str | os.PathLike | None = None, *, synthetic: ModelShape | None = None,
                 gguf_path: str | os.PathLike | None = None, device: int = 0, rope_theta: float = 0.0,
                 logit_softcap: float = 0.0, kv_f32: bool = False, max_ctx: int = 4096, max_sessions: int = 64,
                 max_batch_tokens: int = 512):
        """Weights from a packed stage (`<stage>.index.json`, RealGemmaBackend::new), from a GGUF
        file directly (`gguf_path`: the layout's layers and the stage's head/tail tensors), or
        generated on the device (`synthetic`)."""
        if sum(x is not None for x in (index_path, synthetic, gguf_path)) != 1:
            raise ValueError("give exactly one of index_path, gguf_path or synthetic")
        self.index_path = None if index_path is None else str(index_path)
        self.gguf_path = None if gguf_path is None else os.fspath(gguf_path)
        self.synthetic = synthetic
        self.device = device
        self.options = Options(rope_theta, logit_softcap, 0.0, int(kv_f32), max_ctx, max_sessions, max_batch_tokens)
        self.h = None
        self.info = None

    def load_layout(self, model_id: str, stage_id: str, start_layer: int, end_layer: int, is_head: bool,
                    is_tail: bool):
        """StageForwardBackend::load_layout (real_forward.rs:2258-2363)."""
        self._layout = Layout(model_id.encode(), stage_id.encode(), start_layer, end_layer, int(is_head),
                              int(is_tail))
        h = _P()
        if self.synthetic is not None:
            spec = self.synthetic.spec()
            rc = _lib.sfc_stage_open_synthetic(ctypes.byref(spec), ctypes.byref(self._layout),
                                               ctypes.byref(self.options), self.device, ctypes.byref(h))
        elif self.gguf_path is not None:
            rc = _lib.sfc_stage_open_gguf(os.fsencode(self.gguf_path), ctypes.byref(self._layout),
                                          ctypes.byref(self.options), self.device, ctypes.byref(h))
        else:
            rc = _lib.sfc_stage_open(self.index_path.encode(), ctypes.byref(self._layout), ctypes.byref(self.options),
                                     self.device, ctypes.byref(h))
        _check(rc, "load_layout")
        self.h = h
        info = StageInfo()
        _check(_lib.sfc_stage_get_info(self.h, ctypes.byref(info)), "sfc_stage_get_info")
        self.info = info
        return self

    @property
    def hidden_dim(self) -> int:
        return self.info.hidden

    def begin_token_ids(self, request_id: str, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        out = np.empty((ids.shape[0], self.hidden_dim), np.float32)
        _check(_lib.sfc_begin_token_ids(self.h, request_id.encode(), ids.ctypes.data, ids.shape[0], out.ctypes.data),
               "begin_token_ids")
        return out

    def continue_forward(self, request_id: str, hidden) -> np.ndarray:
        hidden = np.ascontiguousarray(np.atleast_2d(hidden), dtype=np.float32)
        out = np.empty_like(hidden)
        _check(_lib.sfc_continue_forward(self.h, request_id.encode(), hidden.ctypes.data, hidden.shape[0],
                                         out.ctypes.data), "continue_forward")
        return out

    def begin_token_ids_bytes(self, request_id: str, ids) -> bytes:
        """begin_prompt's StageTensor bytes: the rows framed with the prompt aux section (prefix
        hashes of a multi-token prompt, every layer's per-layer inputs for a PLE model)."""
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        n = _U64()
        _lib.sfc_begin_token_ids_bytes(self.h, request_id.encode(), ids.ctypes.data, ids.shape[0], None, 0,
                                       ctypes.byref(n))  # size query (fails on the null output)
        out = ctypes.create_string_buffer(max(int(n.value), 1))
        _check(_lib.sfc_begin_token_ids_bytes(self.h, request_id.encode(), ids.ctypes.data, ids.shape[0], out,
                                              len(out), ctypes.byref(n)), "begin_token_ids_bytes")
        return out.raw[: int(n.value)]

    def continue_forward_bytes(self, request_id: str, payload: bytes, hidden_dim: int) -> bytes:
        """continue_forward on StageTensor::bytes (bare or stb1-framed rows; the aux section is
        carried through)."""
        n = _U64()
        out = ctypes.create_string_buffer(len(payload) + 16)
        _check(_lib.sfc_continue_forward_bytes(self.h, request_id.encode(), payload, len(payload), hidden_dim, out,
                                               len(out), ctypes.byref(n)), "continue_forward_bytes")
        return out.raw[: int(n.value)]

    def sample_tail_bytes(self, payload: bytes, hidden_dim: int) -> tuple[int, float]:
        tok, sc = _U32(0), _F(0)
        _check(_lib.sfc_sample_tail_bytes(self.h, payload, len(payload), hidden_dim, ctypes.byref(tok),
                                          ctypes.byref(sc)), "sample_tail_bytes")
        return int(tok.value), float(sc.value)

    def sample_tail(self, hidden) -> tuple[int, float]:
        hidden = np.ascontiguousarray(np.atleast_2d(hidden), dtype=np.float32)
        tok, sc = _U32(0), _F(0)
        _check(_lib.sfc_sample_tail(self.h, hidden.ctypes.data, hidden.shape[0], ctypes.byref(tok), ctypes.byref(sc)),
               "sample_tail")
        return int(tok.value), float(sc.value)

    def verify_greedy(self, hidden, drafts) -> tuple[int, int]:
        hidden = np.ascontiguousarray(np.atleast_2d(hidden), dtype=np.float32)
        drafts = np.ascontiguousarray(drafts, dtype=np.uint32)
        acc, bonus = _I64(0), _U32(0)
        _check(_lib.sfc_verify_greedy(self.h, hidden.ctypes.data, drafts.ctypes.data, drafts.shape[0],
                                      ctypes.byref(acc), ctypes.byref(bonus)), "verify_greedy")
        return int(acc.value), int(bonus.value)

    def forward_tree(self, request_id: str, parent, ids=None, hidden=None) -> np.ndarray:
        """Tree-masked forward of draft-tree nodes after the session's cache (sfc_forward_tree)."""
        parent = np.ascontiguousarray(parent, dtype=np.int32)
        n = parent.shape[0]
        out = np.empty((n, self.hidden_dim), np.float32)
        idp = hp = None
        if ids is not None:
            ids = np.ascontiguousarray(ids, dtype=np.uint32)
            idp = ids.ctypes.data
        if hidden is not None:
            hidden = np.ascontiguousarray(np.atleast_2d(hidden), dtype=np.float32)
            hp = hidden.ctypes.data
        _check(_lib.sfc_forward_tree(self.h, request_id.encode(), idp, hp, parent.ctypes.data, n, out.ctypes.data),
               "forward_tree")
        return out

    def sample_tree(self, hidden, parent, node_tokens, temperature: float = 0.0, seed: int = 0):
        """Acceptance walk over a verified tree (sfc_sample_tree): (path, next_token)."""
        hidden = np.ascontiguousarray(np.atleast_2d(hidden), dtype=np.float32)
        parent = np.ascontiguousarray(parent, dtype=np.int32)
        node_tokens = np.ascontiguousarray(node_tokens, dtype=np.uint32)
        n = parent.shape[0]
        path = np.empty(n, np.int32)
        npath, nxt = _I64(0), _U32(0)
        _check(_lib.sfc_sample_tree(self.h, hidden.ctypes.data, parent.ctypes.data, node_tokens.ctypes.data, n,
                                    float(temperature), int(seed), path.ctypes.data, ctypes.byref(npath),
                                    ctypes.byref(nxt)), "sample_tree")
        return path[: npath.value].copy(), int(nxt.value)

    def commit_tree(self, request_id: str, path):
        path = np.ascontiguousarray(path, dtype=np.int32)
        _check(_lib.sfc_commit_tree(self.h, request_id.encode(), path.ctypes.data, path.shape[0]), "commit_tree")

    def forward_dev(self, request_ids, seq_tokens, ids_dev=None, in_dev=None, out_dev=None, append=True,
                    stream=None):
        n = len(request_ids)
        arr = (ctypes.c_char_p * n)(*[r.encode() for r in request_ids])
        st = np.ascontiguousarray(seq_tokens, dtype=np.int32)
        _check(_lib.sfc_forward_dev(self.h, arr, st.ctypes.data, n, _ptr(ids_dev), _ptr(in_dev), _ptr(out_dev),
                                    int(append), _stream(stream)), "forward_dev")
        return out_dev

    def sample_dev(self, hidden_dev, tokens_dev, scores_dev, stream=None):
        n = hidden_dev.shape[0]
        _check(_lib.sfc_sample_dev(self.h, _ptr(hidden_dev), n, _ptr(tokens_dev), _ptr(scores_dev), _stream(stream)),
               "sample_dev")

    def generate_greedy(self, request_id: str, prompt, n_steps: int) -> np.ndarray:
        prompt = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.empty(n_steps, np.uint32)
        _check(_lib.sfc_generate_greedy(self.h, request_id.encode(), prompt.ctypes.data, prompt.shape[0], n_steps,
                                        out.ctypes.data), "generate_greedy")
        return out

    def clear_decode_session(self, request_id: str):
        _check(_lib.sfc_clear_decode_session(self.h, request_id.encode()), "clear_decode_session")

    def rollback_kv(self, request_id: str, keep: int):
        _check(_lib.sfc_rollback_kv(self.h, request_id.encode(), keep), "rollback_kv")

    def session_len(self, request_id: str) -> int:
        return int(_lib.sfc_session_len(self.h, request_id.encode()))

    def fill_session_synthetic(self, request_id: str, n_pos: int, seed: int = 1):
        _check(_lib.sfc_session_fill_synthetic(self.h, request_id.encode(), n_pos, seed), "fill_session_synthetic")

    def last_profile(self) -> Profile:
        p = Profile()
        _check(_lib.sfc_last_profile(self.h, ctypes.byref(p)), "last_profile")
        return p

    def close(self):
        if self.h:
            _lib.sfc_stage_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
