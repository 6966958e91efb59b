"""The oracle's multi-token paths (row terms applied to 8 tokens at once; attention queries on
several threads) give bit-identical results to its one-token paths, so long prompts can be
checked against the oracle in seconds without changing a single rounding."""
import numpy as np
import pytest

import stage_oracle as so


@pytest.mark.parametrize("t", [so.Q4_K, so.Q6_K, so.F16, so.F32, so.BF16])
@pytest.mark.parametrize("n_tok", [2, 7, 8, 9, 19])
def test_multi_token_matmul_bit_identical(t, n_tok):
    rows, k = 37, 512
    raw = so.synth_tensor(t, so.tensor_key(3, f"fast.{t}"), rows, k, 0.02)
    x = so.synth_normal_f32(5, f"fast.x.{n_tok}", n_tok * k).reshape(n_tok, k)
    many = so.matmul(t, raw, rows, k, x)
    for i in range(n_tok):
        one = so.matmul(t, raw, rows, k, x[i])
        assert np.array_equal(many[i].view(np.uint32), one[0].view(np.uint32)), f"token {i}"


def test_batched_attention_bit_identical():
    nh, nkv, hd, n = 4, 2, 64, 70
    rng = np.random.default_rng(1)
    krows = [np.ascontiguousarray(r) for r in rng.standard_normal((n, nkv * hd), dtype=np.float32)]
    vrows = [np.ascontiguousarray(r) for r in rng.standard_normal((n, nkv * hd), dtype=np.float32)]
    qs = rng.standard_normal((9, nh * hd), dtype=np.float32)
    limits = np.array([1, 2, 5, 33, 64, 65, 69, 70, 70])
    for window in (0, 16):
        got = so.gqa_attention_rows_batch(qs, krows, vrows, nh, nkv, hd, limits, window=window)
        for i in range(len(limits)):
            ref = so.gqa_attention_rows(qs[i], krows, vrows, nh, nkv, hd, limit=int(limits[i]), window=window)
            assert np.array_equal(got[i].view(np.uint32), ref.view(np.uint32)), (window, i)
