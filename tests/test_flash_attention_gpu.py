"""GPU parity of the tensor-core attention (multi-row batches over an fp16 cache, fattn.cu): several
sequences with cached prefixes and ragged new chunks in one batch (query tiles that end mid-tile,
tiles of different sequences side by side, key splits over long prefixes), against the oracle
and against the same chunks run one sequence at a time.  Head dims 64 / 128 / 256 and 2 or 4
query heads per kv head (32- and 64-token query tiles)."""
import numpy as np
import pytest

import stage_oracle as so
from gpu_util import rel_errors

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def sf():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import stagefwd
    return stagefwd


def shapes(hd, n_heads, n_kv):
    base = dict(hidden=512, n_heads=n_heads, n_kv=n_kv, head_dim=hd, ffn=1024, vocab=4096, n_layers=2, seed=31)
    import stagefwd
    return so.ModelSpec(**base), stagefwd.ModelShape(**base)


# (cached prefix, new tokens) per sequence of the batch
SEQS = [(0, 70), (17, 5), (100, 130), (900, 40)]


@pytest.mark.parametrize("hd,n_heads,n_kv", [(64, 4, 2), (128, 8, 2), (256, 8, 4)])
def test_ragged_multi_sequence_chunks(sf, hd, n_heads, n_kv):
    spec, shape = shapes(hd, n_heads, n_kv)
    mk = lambda: sf.CudaStageBackend(synthetic=shape, rope_theta=10000.0, max_ctx=1024, max_sessions=8,
                                     max_batch_tokens=512).load_layout("m", "s0", 0, 1, True, True)
    g, g1 = mk(), mk()
    orc = so.OracleStage(so.synth_stage(spec, 0, 1, True, True), so.Layout("m", "s0", 0, 1, True, True),
                         rope_theta=10000.0, kv_fp16=True)
    prompts = [so.synth_tokens(40 + i, "f", pre + n, spec.vocab) for i, (pre, n) in enumerate(SEQS)]
    for i, (pre, n) in enumerate(SEQS):
        if pre:
            g.begin_token_ids(f"b{i}", prompts[i][:pre])
            g1.begin_token_ids(f"s{i}", prompts[i][:pre])
    dev = torch.device("cuda")
    ids = torch.from_numpy(np.concatenate([p[pre:] for p, (pre, _) in zip(prompts, SEQS)]).astype(np.int32)).to(dev)
    out = torch.empty(ids.numel(), shape.hidden, device=dev)
    g.forward_dev([f"b{i}" for i in range(len(SEQS))], [n for _, n in SEQS], ids_dev=ids, out_dev=out, append=True)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    row = 0
    for i, (pre, n) in enumerate(SEQS):
        # the same chunk appended alone (a batch of one sequence)
        one_ids = torch.from_numpy(prompts[i][pre:].astype(np.int32)).to(dev)
        one_out = torch.empty(n, shape.hidden, device=dev)
        g1.forward_dev([f"s{i}"], [n], ids_dev=one_ids, out_dev=one_out, append=True)
        torch.cuda.synchronize()
        one = one_out.cpu().numpy()
        ref = orc.begin_token_ids(f"o{i}", prompts[i])[pre:]
        norm_1, mx_1 = rel_errors(got[row:row + n], one)
        assert norm_1 <= 1e-4, f"seq {i}: batched vs alone normwise {norm_1:.2e}"
        # fp16 cache: the oracle rounds its cache the same way; elements whose two roundings differ
        # move this unscaled, peaked attention by up to ~1e-2 (see test_stage_gpu.stage_close)
        norm, mx = rel_errors(got[row:row + n], ref)
        assert norm <= 1e-2, f"seq {i}: vs oracle normwise {norm:.2e}, max/max {mx:.2e}"
        row += n
    g.close()
    g1.close()
