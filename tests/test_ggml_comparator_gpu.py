"""The reference's own GPU GEMV (ggml-cuda MMVQ with its q8_1 activation quantizer, built for sm_100a
from the reference tree into oracle/_ref/libref_mmvq.so by oracle/Makefile) against the stage GEMV on
the same GGUF rows and activations: results agree within the reference's 8-bit activation
quantization, and both are timed on the same device over weight copies larger than twice the L2
(printed; the figures go to the profile summaries).  Skipped when the comparator was not built
(no reference checkout at build time)."""
import ctypes
import json
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

LIB = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "libref_mmvq.so"
SHAPES = [(12, 10240, 2560), (14, 2560, 10240), (12, 2048, 2560)]  # (GGUF type, rows, K)


@pytest.fixture(scope="module")
def sf():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import stagefwd
    return stagefwd


@pytest.fixture(scope="module")
def ref():
    if not LIB.exists():
        pytest.skip("comparator not built (oracle/Makefile with REFERENCE)")
    lib = ctypes.CDLL(str(LIB))
    lib.ref_mmvq_q8_bytes.restype = ctypes.c_size_t
    lib.ref_mmvq_q8_bytes.argtypes = [ctypes.c_int64, ctypes.c_int64]
    lib.ref_mmvq.restype = ctypes.c_int
    lib.ref_mmvq.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
                             ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    return lib


@pytest.mark.parametrize("typ,rows,k", SHAPES)
def test_reference_mmvq_against_stage_gemv(sf, ref, typ, rows, k):
    dev = torch.device("cuda")
    row_bytes = k // 256 * (144 if typ == 12 else 210)
    copies = int(np.ceil(2 * (126 << 20) / (rows * row_bytes))) + 2
    gguf = [sf.synth_tensor(typ, 1, f"cmp.{rows}.{k}.{i}", rows, k, 0.02) for i in range(copies)]
    ours = [sf.prepare_weights(typ, g, rows, k) for g in gguf]
    x = torch.randn(1, k, device=dev)
    q8 = torch.empty(ref.ref_mmvq_q8_bytes(k, 1), dtype=torch.uint8, device=dev)
    y_ref = torch.empty(1, rows, device=dev)
    y_our = torch.empty(1, rows, device=dev)
    st = torch.cuda.current_stream().cuda_stream

    def run_ref(i):
        rc = ref.ref_mmvq(typ, gguf[i % copies].data_ptr(), rows, k, x.data_ptr(), 1, y_ref.data_ptr(),
                          q8.data_ptr(), st)
        assert rc == 0, rc

    def run_our(i):
        assert sf.lib.sfc_matmul(typ, ours[i % copies].data_ptr(), rows, k, x.data_ptr(), 1, y_our.data_ptr(), st) == 0

    run_ref(0)
    run_our(0)
    torch.cuda.synchronize()
    exact = (x.double() @ sf.dequantize_rows(typ, gguf[0], rows, k).double().t()).float()
    err_our = float((y_our - exact).norm() / exact.norm())
    err_ref = float((y_ref - exact).norm() / exact.norm())
    assert err_our < 1e-5, err_our
    assert err_ref < 2e-2, err_ref  # q8_1 activations: 8-bit per 32-element block

    def timed(fn, n=400):
        for i in range(20):
            fn(i)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(n):
            fn(i)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / n

    us_ref, us_our = timed(run_ref), timed(run_our)
    wbytes = rows * row_bytes + k * 4 + rows * 4
    print(json.dumps({"type": "Q4_K" if typ == 12 else "Q6_K", "rows": rows, "k": k, "tokens": 1,
                      "ggml_mmvq_us": round(us_ref, 2), "stage_gemv_us": round(us_our, 2),
                      "ggml_mmvq_gbs": round(wbytes / us_ref / 1e3, 1), "stage_gemv_gbs": round(wbytes / us_our / 1e3, 1),
                      "rel_err_vs_exact": {"ggml_mmvq": err_ref, "stage_gemv": err_our}}))
