"""GPU: the allocation-free logits entry point (sfc_logits_argmax_noalloc) gives the same result as
sfc_logits_argmax.  It exists for callers that cannot have the library call cudaMalloc: serving
processes whose device memory is reserved up front and owned by their own allocator.  Collected last so that a run stopping at the first failure has already run every
other test; it must also pass alone in a fresh process."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def test_logits_argmax_noalloc_matches_allocating_entry_point():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import stagefwd as sf
    lib = sf.lib
    f = lib.sfc_logits_argmax_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                  ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    V, H, T = 65536, 2560, 3
    table = sf.synth_tensor(sf.F16, 41, "token_embd.weight", V, H, 0.02)
    h = torch.randn(T, H, device="cuda", generator=torch.Generator("cuda").manual_seed(0))
    st = torch.cuda.current_stream().cuda_stream
    ref_idx, ref_sc, ref_all = sf.logits_argmax(sf.F16, table, V, H, h, 30.0, want_scores=True)
    torch.cuda.synchronize()
    for _ in range(2):  # two calls in a row share (and overwrite) the fixed scratch array
        idx = torch.full((T,), -1, dtype=torch.int64, device="cuda")
        sc = torch.zeros(T, dtype=torch.float32, device="cuda")
        allsc = torch.zeros((T, V), dtype=torch.float32, device="cuda")
        rc = f(sf.F16, table.data_ptr(), V, H, h.data_ptr(), T, 30.0, allsc.data_ptr(), idx.data_ptr(),
               sc.data_ptr(), st)
        assert rc == 0, lib.sfc_last_error()
        torch.cuda.synchronize()
        assert torch.equal(idx, ref_idx)
        # the tolerance the other logits tests use: 1e-3 relative
        np.testing.assert_allclose(sc.cpu().numpy(), ref_sc.cpu().numpy(), rtol=1e-3)
        d = (allsc - ref_all).abs().max().item() / ref_all.abs().max().item()
        assert d <= 1e-3


def test_noalloc_rejects_bad_input_without_gpu_work():
    import stagefwd as sf
    f = sf.lib.sfc_logits_argmax_noalloc
    f.restype = ctypes.c_int
    assert f(12, None, 10, 256, None, 1, ctypes.c_float(30.0), None, None, None, None) == -1
    assert b"F16/F32/BF16" in sf.lib.sfc_last_error()
