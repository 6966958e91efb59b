"""GGUF shard files, stage splits, manifest bundles and stage packs through the C ABI.

Mirrors the reference's on-disk tooling (crates/stage-forward-lab): `GgufFile` (gguf.rs:138-365),
`plan_for_splits` / `write_bundle` (gguf.rs:366-751) and the stage pack writer
(`StageResidencyAdapter::pack_required_tensors` / `pack_all_tensors`, lib.rs:3424-3613).  The
parsing, planning and file writing run in the library's C++ (csrc/gguf.cpp); this module only
binds it.  A stage can also be opened straight from a GGUF file:
`CudaStageBackend(gguf_path=...)`.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from pathlib import Path

from . import _lib, _sig, _check

SFC_ABSENT = 1
ROLE_NAMES = {0: "Layer", 1: "PromptIngress", 2: "Positional", 3: "SharedAuxiliary", 4: "TailOnly",
              5: "UnknownGlobal"}

_U32, _U64, _I64, _P = ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int64, ctypes.c_void_p


class _Info(ctypes.Structure):
    _fields_ = [("version", _U32), ("tensor_count", _U64), ("metadata_count", _U64), ("file_size_bytes", _U64),
                ("tensor_data_offset", _U64), ("layer_count", _I64), ("hidden_size", _I64),
                ("feed_forward_length", _I64), ("attention_head_count", _I64), ("architecture", ctypes.c_char_p)]


class _Tensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("n_dims", _U32), ("dims", ctypes.POINTER(_U64)), ("ggml_type", _U32),
                ("offset", _U64), ("file_offset", _U64), ("byte_len", _U64), ("role", ctypes.c_int32),
                ("layer", _I64)]


class StageSplit(ctypes.Structure):
    """StageSplit (gguf.rs:42-47)."""
    _fields_ = [("stage_index", _U32), ("start_layer", _U32), ("end_layer", _U32)]

    def __eq__(self, other):
        return (self.stage_index, self.start_layer, self.end_layer) == (
            other.stage_index, other.start_layer, other.end_layer)

    def __repr__(self):
        return f"StageSplit({self.stage_index}, {self.start_layer}, {self.end_layer})"


_sig("sfc_gguf_open", ctypes.c_int, ctypes.c_char_p, ctypes.POINTER(_P))
_sig("sfc_gguf_parse", ctypes.c_int, ctypes.c_char_p, _U64, ctypes.POINTER(_P))
_sig("sfc_gguf_close", ctypes.c_int, _P)
_sig("sfc_gguf_get_info", ctypes.c_int, _P, ctypes.POINTER(_Info))
_sig("sfc_gguf_get_tensor", ctypes.c_int, _P, _U64, ctypes.POINTER(_Tensor))
_sig("sfc_gguf_find_tensor", ctypes.c_int, _P, ctypes.c_char_p, ctypes.POINTER(_U64))
_sig("sfc_gguf_metadata_key", ctypes.c_int, _P, _U64, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_U32))
_sig("sfc_gguf_metadata_string", ctypes.c_int, _P, ctypes.c_char_p, ctypes.c_char_p, _U64, ctypes.POINTER(_U64))
_sig("sfc_gguf_metadata_u32", ctypes.c_int, _P, ctypes.c_char_p, ctypes.POINTER(_U32))
_sig("sfc_gguf_metadata_array", ctypes.c_int, _P, ctypes.c_char_p, ctypes.POINTER(_U32), ctypes.POINTER(_U64))
_sig("sfc_gguf_metadata_f32_array", ctypes.c_int, _P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_float), _U64,
     ctypes.POINTER(_U64))
_sig("sfc_gguf_metadata_array_string", ctypes.c_int, _P, ctypes.c_char_p, _U64, ctypes.c_char_p, _U64,
     ctypes.POINTER(_U64))
_sig("sfc_gguf_block_indices", ctypes.c_int, _P, ctypes.POINTER(_U32), _U64, ctypes.POINTER(_U64))
_sig("sfc_gguf_even_split", ctypes.c_int, _P, _U32, ctypes.POINTER(StageSplit))
_sig("sfc_gguf_write_bundle", ctypes.c_int, _P, ctypes.POINTER(StageSplit), _U32, ctypes.c_char_p)
_sig("sfc_pack_stage", ctypes.c_int, ctypes.c_char_p, ctypes.c_char_p, _U32, ctypes.c_int, ctypes.c_char_p,
     ctypes.c_char_p, _U64)
_sig("sfc_materialize_stage", ctypes.c_int, ctypes.c_char_p, ctypes.c_char_p, _U32, ctypes.c_char_p,
     ctypes.POINTER(_U64))


@dataclass(frozen=True)
class TensorInfo:
    """TensorInfo (gguf.rs:24-30) with its slice (gguf.rs:101-108) and role (gguf.rs:49-57)."""
    name: str
    dimensions: tuple
    ggml_type: int
    offset: int
    file_offset: int
    byte_len: int
    role: str
    layer_index: int | None


def _fs(p) -> bytes:
    return os.fsencode(os.fspath(p))


class GgufFile:
    """GgufFile (gguf.rs:32-40): the header, metadata and tensor table of a GGUF file."""

    def __init__(self, handle: int):
        self._h = _P(handle)
        info = _Info()
        _check(_lib.sfc_gguf_get_info(self._h, ctypes.byref(info)), "sfc_gguf_get_info")
        self.version = int(info.version)
        self.tensor_count = int(info.tensor_count)
        self.file_size_bytes = int(info.file_size_bytes)
        self.tensor_data_offset = int(info.tensor_data_offset)
        self._arch = None if info.architecture is None else info.architecture.decode()
        self._layers = int(info.layer_count)
        self._hidden, self._ffn, self._heads = (int(info.hidden_size), int(info.feed_forward_length),
                                                int(info.attention_head_count))
        self.tensors = [self._tensor(i) for i in range(self.tensor_count)]
        self.metadata_keys = []
        for i in range(int(info.metadata_count)):
            k, t = ctypes.c_char_p(), _U32()
            _check(_lib.sfc_gguf_metadata_key(self._h, i, ctypes.byref(k), ctypes.byref(t)), "sfc_gguf_metadata_key")
            self.metadata_keys.append(k.value.decode())

    @classmethod
    def parse_file(cls, path) -> "GgufFile":
        h = _P()
        _check(_lib.sfc_gguf_open(_fs(path), ctypes.byref(h)), "GgufFile::parse_file")
        return cls(h.value)

    @classmethod
    def parse_bytes(cls, data: bytes) -> "GgufFile":
        h = _P()
        _check(_lib.sfc_gguf_parse(data, len(data), ctypes.byref(h)), "GgufFile::parse_bytes")
        return cls(h.value)

    def close(self):
        if self._h is not None and self._h.value:
            _lib.sfc_gguf_close(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def _tensor(self, i: int) -> TensorInfo:
        t = _Tensor()
        _check(_lib.sfc_gguf_get_tensor(self._h, i, ctypes.byref(t)), "sfc_gguf_get_tensor")
        return TensorInfo(t.name.decode(), tuple(int(t.dims[d]) for d in range(t.n_dims)), int(t.ggml_type),
                          int(t.offset), int(t.file_offset), int(t.byte_len), ROLE_NAMES[int(t.role)],
                          None if t.layer < 0 else int(t.layer))

    # ---- queries (gguf.rs:212-364)
    def architecture(self) -> str | None:
        return self._arch

    def inferred_layer_count(self) -> int | None:
        return None if self._layers < 0 else self._layers

    def hidden_size(self) -> int | None:
        return None if self._hidden < 0 else self._hidden

    def feed_forward_length(self) -> int | None:
        return None if self._ffn < 0 else self._ffn

    def attention_head_count(self) -> int | None:
        return None if self._heads < 0 else self._heads

    def block_indices(self) -> list[int]:
        n = _U64()
        _check(_lib.sfc_gguf_block_indices(self._h, None, 0, ctypes.byref(n)), "sfc_gguf_block_indices")
        buf = (_U32 * max(int(n.value), 1))()
        _check(_lib.sfc_gguf_block_indices(self._h, buf, n.value, ctypes.byref(n)), "sfc_gguf_block_indices")
        return [int(buf[i]) for i in range(int(n.value))]

    def metadata_string(self, key: str) -> str | None:
        n = _U64()
        rc = _lib.sfc_gguf_metadata_string(self._h, key.encode(), None, 0, ctypes.byref(n))
        if rc == SFC_ABSENT:
            return None
        _check(rc, "metadata_string")
        buf = ctypes.create_string_buffer(int(n.value) + 1)
        _check(_lib.sfc_gguf_metadata_string(self._h, key.encode(), buf, len(buf), ctypes.byref(n)),
               "metadata_string")
        return buf.raw[: int(n.value)].decode()

    def metadata_string_array(self, key: str) -> list[str] | None:
        """metadata_string_array (gguf.rs:253-260)."""
        t, n = _U32(), _U64()
        rc = _lib.sfc_gguf_metadata_array(self._h, key.encode(), ctypes.byref(t), ctypes.byref(n))
        if rc == SFC_ABSENT:
            return None
        _check(rc, "metadata_string_array")
        out = []
        for i in range(int(n.value)):
            ln = _U64()
            _check(_lib.sfc_gguf_metadata_array_string(self._h, key.encode(), i, None, 0, ctypes.byref(ln)),
                   "metadata_string_array")
            buf = ctypes.create_string_buffer(int(ln.value) + 1)
            _check(_lib.sfc_gguf_metadata_array_string(self._h, key.encode(), i, buf, len(buf), ctypes.byref(ln)),
                   "metadata_string_array")
            out.append(buf.raw[: int(ln.value)].decode())
        return out

    def metadata_f32_array(self, key: str) -> list[float] | None:
        """metadata_f32_array (gguf.rs:262-277)."""
        n = _U64()
        rc = _lib.sfc_gguf_metadata_f32_array(self._h, key.encode(), None, 0, ctypes.byref(n))
        if rc == SFC_ABSENT:
            return None
        _check(rc, "metadata_f32_array")
        buf = (ctypes.c_float * max(int(n.value), 1))()
        _check(_lib.sfc_gguf_metadata_f32_array(self._h, key.encode(), buf, n.value, ctypes.byref(n)),
               "metadata_f32_array")
        return [float(buf[i]) for i in range(int(n.value))]

    def metadata_u32(self, key: str) -> int | None:
        v = _U32()
        rc = _lib.sfc_gguf_metadata_u32(self._h, key.encode(), ctypes.byref(v))
        if rc == SFC_ABSENT:
            return None
        _check(rc, "metadata_u32")
        return int(v.value)

    def suggest_even_stage_split(self, stages: int) -> list[StageSplit] | None:
        out = (StageSplit * max(stages, 1))()
        rc = _lib.sfc_gguf_even_split(self._h, stages, out)
        if rc == SFC_ABSENT:
            return None
        _check(rc, "suggest_even_stage_split")
        return [StageSplit(s.stage_index, s.start_layer, s.end_layer) for s in out[:stages]]

    def _find(self, name: str) -> TensorInfo | None:
        i = _U64()
        rc = _lib.sfc_gguf_find_tensor(self._h, name.encode(), ctypes.byref(i))
        if rc == SFC_ABSENT:
            return None
        _check(rc, "sfc_gguf_find_tensor")
        return self.tensors[int(i.value)]

    def tensor_byte_len(self, name: str) -> int | None:
        t = self._find(name)
        return None if t is None else t.byte_len

    def tensor_file_offset(self, name: str) -> int | None:
        t = self._find(name)
        return None if t is None else t.file_offset

    # ---- bundle (gguf.rs:366-751)
    def write_bundle(self, splits, out_dir) -> Path:
        arr = (StageSplit * max(len(splits), 1))(*[StageSplit(s.stage_index, s.start_layer, s.end_layer)
                                                   for s in splits])
        _check(_lib.sfc_gguf_write_bundle(self._h, arr, len(splits), _fs(out_dir)), "write_bundle")
        return Path(out_dir) / "model-shard-manifest.json"


def pack_stage(bundle_dir, gguf_path, stage_index: int, out_dir, include_optional: bool = False) -> Path:
    """StageResidencyAdapter::load(bundle, gguf, stage) + pack_required_tensors (or pack_all_tensors
    with include_optional) (lib.rs:3424-3613).  Returns the `.index.json` path."""
    buf = ctypes.create_string_buffer(4096)
    _check(_lib.sfc_pack_stage(_fs(bundle_dir), _fs(gguf_path), stage_index, int(include_optional), _fs(out_dir),
                               buf, len(buf)), "pack_stage")
    return Path(os.fsdecode(buf.value))


def materialize_stage(bundle_dir, gguf_path, stage_index: int, out_dir) -> int:
    """StageResidencyAdapter::load + materialize_required_tensors (lib.rs:3424-3510): one file per
    required tensor of the stage in out_dir.  Returns the number of files written."""
    n = _U64()
    _check(_lib.sfc_materialize_stage(_fs(bundle_dir), _fs(gguf_path), stage_index, _fs(out_dir), ctypes.byref(n)),
           "materialize_stage")
    return int(n.value)
