"""The TCP stage node over the CUDA backend: a head (layers 0-1) and a tail (2-3) stage on the GPU
behind loopback sockets, driven with the StageNodeRequest v1 flow of test_stage_node.py
(BeginPrompt, ContinueForward, ContinueHeadTokens decode steps, SampleTail, ContinueForwardVerifyK
with accepted and rejected drafts, RollbackKv); every token equals the oracle's."""
import pytest

from test_stage_node import SPEC, run_gateway_flow

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def test_gpu_nodes_serve_the_gateway_flow():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import stagefwd as sf
    from stagefwd import node
    shape = sf.ModelShape(**SPEC)  # the oracle's synthetic model: Q4_K_M mix, f32 cache below
    mk = lambda a, b, hd, tl: sf.CudaStageBackend(synthetic=shape, rope_theta=10000.0, kv_f32=True, max_ctx=256,
                                                  max_sessions=4).load_layout("m", f"s{a}", a, b, hd, tl)
    head, tail = mk(0, 1, True, False), mk(2, 3, False, True)
    try:
        run_gateway_flow(node, head, tail)
    finally:
        head.close()
        tail.close()
