"""GPU parity of the tensor-core K-quant GEMM (8 or more tokens: tcgen05 MMA, TMEM accumulators)
against the CPU oracle, through the same kernel-level C ABI as the GEMV (sfc_matmul picks the GEMM
from 8 tokens on).  Bar: 1e-3 relative (gpu_util.REL_TOL); known answers exact."""
import numpy as np
import pytest

import stage_oracle as so
from gpu_util import assert_close

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def sf():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import stagefwd
    return stagefwd


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


# (type, rows, K, token counts): graded shapes, partial row tiles (rows % 128 != 0), single-block K,
# and token counts that hit every token-tile width (8/16/32/64) and ragged last tiles
CASES = [(so.Q4_K, 10240, 2560, (8, 16, 64)), (so.Q4_K, 2048, 2560, (8, 24, 100, 130)),
         (so.Q6_K, 2560, 10240, (8, 64)), (so.Q6_K, 1024, 2560, (8, 17, 64)),
         (so.Q4_K, 200, 512, (8, 9, 33)), (so.Q6_K, 130, 256, (8, 40)), (so.Q4_K, 2560, 2048, (8, 512))]


@pytest.mark.parametrize("t,rows,k,toks", CASES)
def test_gemm_matches_oracle(sf, t, rows, k, toks):
    w = so.synth_tensor(t, so.tensor_key(17, f"g{rows}x{k}"), rows, k, 0.02)
    wd = sf.prepare_weights(t, dev(w), rows, k)
    for n_tok in toks:
        x = so.synth_normal_f32(5, f"gx{n_tok}", n_tok * k).reshape(n_tok, k)
        y = sf.matmul(t, wd, rows, k, dev(x)).cpu().numpy()
        ref = so.matmul(t, w, rows, k, x)
        assert_close(y, ref, what=f"gemm type {t} {rows}x{k} T={n_tok}")


@pytest.mark.parametrize("t", [so.Q4_K, so.Q6_K])
def test_gemm_pair_geglu(sf, t):
    rows, k = 1024, 2560
    g = so.synth_tensor(t, so.tensor_key(19, "g"), rows, k, 0.02)
    u = so.synth_tensor(t, so.tensor_key(19, "u"), rows, k, 0.02)
    gd, ud = sf.prepare_weights(t, dev(g), rows, k), sf.prepare_weights(t, dev(u), rows, k)
    for n_tok in (8, 20):
        x = so.synth_normal_f32(6, f"x{n_tok}", n_tok * k).reshape(n_tok, k) * np.float32(0.01)
        y = sf.matmul_pair_geglu(t, gd, ud, rows, k, dev(x)).cpu().numpy()
        ref = so.gelu_tanh_mul(so.matmul(t, g, rows, k, x), so.matmul(t, u, rows, k, x))
        assert_close(y, ref, what=f"gemm geglu T={n_tok}")


def test_gemm_edge_inputs(sf):
    """Per-token rows of zeros, tiny, huge and wide-range values in one batch (per (token, block)
    power-of-two scaling keeps each in fp16 range)."""
    rows, k = 256, 2560
    w = so.synth_tensor(so.Q4_K, so.tensor_key(8, "edge"), rows, k, 0.02)
    wd = sf.prepare_weights(so.Q4_K, dev(w), rows, k)
    x = np.stack([np.zeros(k, np.float32), np.full(k, 1e-30, np.float32), np.full(k, 3.0e7, np.float32),
                  np.where(np.arange(k) % 7 == 0, 1e4, 1e-3).astype(np.float32),
                  np.where(np.arange(k) < 256, 1e20, 1.0).astype(np.float32)] +
                 [so.synth_normal_f32(1, f"e{i}", k) for i in range(3)])
    y = sf.matmul(so.Q4_K, wd, rows, k, dev(x)).cpu().numpy()
    ref = so.matmul(so.Q4_K, w, rows, k, x)
    assert not y[0].any()
    for i in range(1, x.shape[0]):
        assert_close(y[i], ref[i], what=f"edge row {i}")


def test_gemm_known_answer(sf):
    """Q4_K row with d=1, sub-blocks 0-3 scale 1 (4-7 scale 0), mins 0, all quants 1 -> sum of the
    first 128 x; Q6_K d=1, sc=1, q=0 -> -32 * sum(x); 8 tokens so the GEMM runs."""
    row = np.zeros(144, np.uint8)
    row[0:2] = np.array([1.0], np.float16).view(np.uint8)
    row[4:8] = 1
    row[16:] = 0x11
    x = np.stack([np.full(256, float(i + 1), np.float32) for i in range(8)])
    y = sf.matmul(so.Q4_K, sf.prepare_weights(so.Q4_K, dev(row), 1, 256), 1, 256, dev(x)).cpu().numpy()
    assert y.ravel().tolist() == [128.0 * (i + 1) for i in range(8)]
    row6 = np.zeros(210, np.uint8)
    row6[192:208] = 1
    row6[208:210] = np.array([1.0], np.float16).view(np.uint8)
    y = sf.matmul(so.Q6_K, sf.prepare_weights(so.Q6_K, dev(row6), 1, 256), 1, 256, dev(x)).cpu().numpy()
    assert y.ravel().tolist() == [-8192.0 * (i + 1) for i in range(8)]
