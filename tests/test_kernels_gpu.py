"""GPU parity of the kernel-level C ABI against the CPU oracle.

Bar: dequant bit-exact; matmuls / logits within 1e-3 relative (normwise and max-abs over
max-ref, see gpu_util.REL_TOL); argmax identical (lowest index on ties)."""
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


def test_synthetic_bytes_match_oracle(sf):
    for t, rows, k, sigma, mean in ((so.Q4_K, 33, 2560, 0.02, 0.0), (so.Q6_K, 17, 2560, 0.02, 0.0),
                                    (so.F16, 9, 2560, 0.02, 0.0), (so.F32, 5, 2560, 0.05, 1.0)):
        g = sf.synth_tensor(t, 99, "blk.3.ffn_down.weight", rows, k, sigma, mean).cpu().numpy()
        o = so.synth_tensor(t, so.tensor_key(99, "blk.3.ffn_down.weight"), rows, k, sigma, mean)
        assert np.array_equal(g, o), t


@pytest.mark.parametrize("t", [so.Q4_K, so.Q6_K])
def test_dequant_bit_exact(sf, golden_dir, t):
    g = np.load(golden_dir / "dequant_golden.npz")
    raw = g["q4k_raw" if t == so.Q4_K else "q6k_raw"]
    out = sf.dequantize_rows(t, dev(raw.reshape(-1)), raw.shape[0], 256).cpu().numpy()
    assert np.array_equal(out.view(np.uint32), g["q4k_out" if t == so.Q4_K else "q6k_out"].view(np.uint32))
    syn = so.synth_tensor(t, so.tensor_key(5, "w"), 64, 2560, 0.02)
    out = sf.dequantize_rows(t, dev(syn), 64, 2560).cpu().numpy()
    ref = so.dequantize_rows(t, syn, 64, 2560)
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


SHAPES = [(10240, 2560), (2560, 10240), (1024, 2560), (2560, 2048), (37, 512), (5, 256)]


@pytest.mark.parametrize("t", [so.Q4_K, so.Q6_K, so.F16, so.F32])
@pytest.mark.parametrize("rows,k", SHAPES)
def test_matmul_matches_oracle(sf, t, rows, k):
    w = so.synth_tensor(t, so.tensor_key(7, f"m{rows}x{k}"), rows, k, 0.02)
    wd = sf.prepare_weights(t, dev(w), rows, k)
    for n_tok in (1, 2, 3, 4, 5, 8):
        x = so.synth_normal_f32(3, f"x{n_tok}", n_tok * k).reshape(n_tok, k)
        y = sf.matmul(t, wd, rows, k, dev(x)).cpu().numpy()
        ref = so.matmul(t, w, rows, k, x)
        assert_close(y, ref, what=f"type {t} {rows}x{k} T={n_tok}")


def test_gemv_edge_inputs(sf):
    rows, k = 64, 2560
    w = so.synth_tensor(so.Q4_K, so.tensor_key(8, "edge"), rows, k, 0.02)
    wd = sf.prepare_weights(so.Q4_K, dev(w), rows, k)
    xs = [np.zeros((1, k), np.float32),                       # all zero
          np.full((1, k), 1e-30, np.float32),                 # tiny
          np.full((1, k), 3.0e7, np.float32),                 # large
          np.where(np.arange(k) % 7 == 0, 1e4, 1e-3).astype(np.float32)[None]]  # wide range in a block
    for x in xs:
        y = sf.matmul(so.Q4_K, wd, rows, k, dev(x)).cpu().numpy()
        ref = so.matmul(so.Q4_K, w, rows, k, x)
        if not ref.any():
            assert not y.any()
        else:
            assert_close(y, ref, tol=1e-3, what="edge")


def test_known_answer_rows_on_gpu(sf):
    row = np.zeros(144, np.uint8)
    row[0:2] = np.array([1.0], np.float16).view(np.uint8)
    row[4:8] = 1
    row[16:] = 0x11
    y = sf.matmul(so.Q4_K, sf.prepare_weights(so.Q4_K, dev(row), 1, 256), 1, 256,
                  dev(np.stack([np.ones(256, np.float32), np.full(256, 0.5, np.float32)]))).cpu().numpy()
    assert y.ravel().tolist() == [128.0, 64.0]
    row6 = np.zeros(210, np.uint8)
    row6[192:208] = 1
    row6[208:210] = np.array([1.0], np.float16).view(np.uint8)
    y = sf.matmul(so.Q6_K, sf.prepare_weights(so.Q6_K, dev(row6), 1, 256), 1, 256,
                  dev(np.ones((1, 256), np.float32))).cpu().numpy()
    assert y.ravel().tolist() == [-8192.0]


@pytest.mark.parametrize("t", [so.Q4_K, so.Q6_K])
def test_pair_geglu(sf, t):
    rows, k = 1024, 2560
    g = so.synth_tensor(t, so.tensor_key(9, "g"), rows, k, 0.02)
    u = so.synth_tensor(t, so.tensor_key(9, "u"), rows, k, 0.02)
    gd, ud = sf.prepare_weights(t, dev(g), rows, k), sf.prepare_weights(t, dev(u), rows, k)
    for n_tok in (1, 4, 6):
        x = so.synth_normal_f32(4, f"x{n_tok}", n_tok * k).reshape(n_tok, k) * np.float32(0.01)
        y = sf.matmul_pair_geglu(t, gd, ud, rows, k, dev(x)).cpu().numpy()
        ref = so.gelu_tanh_mul(so.matmul(t, g, rows, k, x), so.matmul(t, u, rows, k, x))
        assert_close(y, ref, what=f"geglu T={n_tok}")


def test_rms_norm(sf):
    x = so.synth_normal_f32(1, "rx", 3 * 2560).reshape(3, 2560) * np.float32(50)
    w = so.synth_normal_f32(1, "rw", 2560) * np.float32(0.05) + np.float32(1)
    y = sf.rms_norm(dev(x), dev(w)).cpu().numpy()
    assert_close(y, so.rms_norm(x, w), tol=1e-5, what="rmsnorm")


@pytest.mark.parametrize("vocab", [262144, 1000])
def test_logits_argmax(sf, vocab):
    H = 2560
    e = so.synth_tensor(so.F16, so.tensor_key(2, "token_embd.weight"), vocab, H, 0.02)
    h = so.synth_normal_f32(2, "h", 3 * H).reshape(3, H)
    idx, sc, allsc = sf.logits_argmax(so.F16, dev(e), vocab, H, dev(h), 30.0, want_scores=True)
    for t in range(3):
        am, asc, _, ref_all = so.logits_top_k(so.F16, e, vocab, H, h[t], 0, 30.0, want_all=True)
        assert int(idx[t]) == am
        assert_close(allsc[t].cpu().numpy(), ref_all, what="logits")
        assert abs(float(sc[t]) - asc) <= 1e-3 * abs(asc)


def test_logits_tie_lowest_index(sf):
    H, V = 256, 5000
    e = np.zeros((V, H), np.float16)
    e[[17, 1234, 4999], :] = 1.0  # three identical best rows
    idx, _, _ = sf.logits_argmax(so.F16, dev(e.view(np.uint8).reshape(-1)), V, H, dev(np.ones((1, H), np.float32)))
    assert int(idx[0]) == 17
