"""CPU: the TCP stage node (stagefwd/node.py) — the StageNodeRequest v1 wire format
(crates/llama-stage-backend/src/lib.rs:606-666, :737-789, framing :2308-2370), the reference's own
wire round-trip cases (lib.rs:4849-5050) restated for MessagePack, and a loopback head/tail pair
driven like the gateway does.  The nodes here serve the oracle stage (the node is generic over the
backend), so the protocol and the handler are checked without a GPU; test_stage_node_gpu.py drives
the CUDA backend the same way."""
import socket
import struct
import threading

import msgpack
import numpy as np
import pytest

import stage_oracle as so

SPEC = dict(hidden=256, n_heads=4, n_kv=2, head_dim=64, ffn=512, vocab=300, n_layers=4, seed=33)


@pytest.fixture(scope="module")
def node():
    from stagefwd import node as nd
    return nd


def sample_tensor(nd):
    return nd.stage_tensor("req-1", 8, bytes(range(1, 9)), ["head"], max_tokens=64)


# ---------------------------------------------------------------- wire format
def round_trip(nd, obj):
    frame = nd.pack_message(obj)
    (n,) = struct.unpack_from("<I", frame)
    assert n == len(frame) - 4
    return msgpack.unpackb(frame[4:], raw=False)


def test_request_encoding_is_rmp_serde_named_map(node):
    """rmp_serde::to_vec_named of StageNodeRequest::RollbackKv: a 3-entry map, tag first."""
    req = node.request("rollback_kv", request_id="req-1", keep_count=5)
    body = node.pack_message(req)[4:]
    assert body == b"\x83\xa2op\xabrollback_kv\xaarequest_id\xa5req-1\xaakeep_count\x05"
    assert node.pack_message(req)[:4] == struct.pack("<I", len(body))


def test_stage_tensor_fields_and_bytes(node):
    t = sample_tensor(node)
    assert list(t) == ["request_id", "kind", "stage_trace", "hidden_dim", "bytes", "prompt_text", "max_tokens",
                       "continuation", "transient", "carry"]
    body = msgpack.packb(t, use_bin_type=True)
    assert b"\xa5bytes\xc4\x08\x01\x02\x03\x04\x05\x06\x07\x08" in body  # Vec<u8> as bin (not base64)
    assert b"\xa4kind\xabHiddenState" in body                            # unit variant by name


def test_continue_head_draft_k_round_trips(node):
    r = round_trip(node, node.request("continue_head_draft_k", request_id="req-1", last_token=42, draft_k=4,
                                      max_tokens=128))
    assert node.check_request(r) == {"op": "continue_head_draft_k", "request_id": "req-1", "last_token": 42,
                                     "draft_k": 4, "max_tokens": 128}


def test_continue_forward_verify_k_round_trips(node):
    r = node.check_request(round_trip(node, node.request(
        "continue_forward_verify_k", request_id="req-1", tensor=sample_tensor(node), last_token=7,
        draft_tokens=[10, 20, 30, 40], clear_memory=False)))
    assert r["request_id"] == "req-1" and r["tensor"]["hidden_dim"] == 8 and r["last_token"] == 7
    assert r["draft_tokens"] == [10, 20, 30, 40] and r["clear_memory"] is False


def test_rollback_kv_round_trips(node):
    r = node.check_request(round_trip(node, node.request("rollback_kv", request_id="req-1", keep_count=5)))
    assert r["request_id"] == "req-1" and r["keep_count"] == 5


def test_verified_batch_round_trips(node):
    r = round_trip(node, node.response("verified_batch", accepted_count=3, accepted_token_ids=[10, 20, 30, 99],
                                       accepted_pieces=["a", "b", "c", "d"], is_eog=False, profile=None))
    assert r == {"kind": "verified_batch", "accepted_count": 3, "accepted_token_ids": [10, 20, 30, 99],
                 "accepted_pieces": ["a", "b", "c", "d"], "is_eog": False}
    assert "profile" not in r


def test_stage_node_info_back_compat_default_spec_decode_flag(node):
    legacy = {"protocol_version": 1, "model_id": "gemma-4-e4b", "stage_id": "head", "start_layer": 0,
              "end_layer": 17, "is_head": True, "is_tail": False}
    info = node.node_info(round_trip(node, legacy))
    assert info["protocol_version"] == 1 and info["spec_decode_v1"] is False


def test_tensor_response_back_compat_omits_tail_sample(node):
    body = node.pack_message(node.response("tensor", tensor=sample_tensor(node), tail_sample=None, profile=None))
    assert b"tail_sample" not in body and b"profile" not in body


def test_bad_requests_answer_with_errors(node):
    n = node.StageNode(None, "m", "s", 0, 0, True, True, 8, 300)
    assert n.handle({"op": "nope"})["kind"] == "error"
    assert "missing field `keep_count`" in n.handle({"op": "rollback_kv", "request_id": "x"})["message"]
    r = n.handle(node.request("continue_head_draft_k", request_id="r", last_token=1, draft_k=2))
    assert r == {"kind": "error", "message": "ContinueHeadDraftK is not implemented on this node "
                                             "(gateway-side drafting)"}


# ---------------------------------------------------------------- loopback head / tail
class OracleBackend:
    """The node's backend interface over the oracle stage (what CudaStageBackend offers on GPUs)."""

    def __init__(self, start, end, head, tail):
        spec = so.ModelSpec(**SPEC)
        self.s = so.OracleStage(so.synth_stage(spec, start, end, head, tail),
                                so.Layout("m", f"s{start}", start, end, head, tail), rope_theta=10000.0)

    def begin_token_ids_bytes(self, req, ids):
        import stagefwd as sf
        ids = list(ids)
        h = self.s.begin_token_ids(req, ids)
        aux = so.encode_prompt_aux(None, 0, so.prefix_hashes(ids) if len(ids) > 1 else ())
        return sf.encode_stage_tensor_bytes(np.ascontiguousarray(h, np.float32).tobytes(), aux)

    def continue_forward_bytes(self, req, payload, hidden_dim):
        import stagefwd as sf
        hidden, aux, _ = sf.stage_tensor_byte_sections(payload)
        rows = np.frombuffer(hidden, np.float32).reshape(-1, hidden_dim)
        out = self.s.continue_forward(req, rows)
        return sf.encode_stage_tensor_bytes(np.ascontiguousarray(out, np.float32).tobytes(), aux)

    def sample_tail_bytes(self, payload, hidden_dim):
        import stagefwd as sf
        rows = np.frombuffer(sf.stage_tensor_byte_sections(payload)[0], np.float32).reshape(-1, hidden_dim)
        return self.s.sample_tail(rows[-1])[:2]

    def verify_greedy(self, hidden, drafts):
        acc = 0
        while acc < len(drafts) and self.s.sample_tail(hidden[acc])[0] == int(drafts[acc]):
            acc += 1
        return acc, self.s.sample_tail(hidden[acc])[0]

    def session_len(self, req):
        s = self.s.sessions.get(req)
        return 0 if s is None else s["seq_len"]

    def rollback_kv(self, req, keep):
        self.s.rollback(req, keep)

    def clear_decode_session(self, req):
        self.s.sessions.pop(req, None)


def start_node(nd, backend, *layout):
    srv = socket.create_server(("127.0.0.1", 0))
    node = nd.StageNode(backend, "m", *layout, SPEC["hidden"], SPEC["vocab"])
    th = threading.Thread(target=nd.serve, args=(node, srv, 1), daemon=True)
    th.start()
    host, port = srv.getsockname()
    return nd.StageNodeClient(f"{host}:{port}", timeout=120), th, srv


def test_loopback_head_tail_pair(node):
    run_gateway_flow(node, OracleBackend(0, 1, True, False), OracleBackend(2, 3, False, True))


def run_gateway_flow(node, head_backend, tail_backend):
    """Head (layers 0-1) and tail (2-3) nodes on loopback sockets, driven as the gateway does; every
    token is checked against the single-process oracle."""
    head, th1, s1 = start_node(node, head_backend, "head", 0, 1, True, False)
    tail, th2, s2 = start_node(node, tail_backend, "tail", 2, 3, False, True)
    ref = so.OracleStage(so.synth_stage(so.ModelSpec(**SPEC), 0, 3, True, True), so.Layout("m", "f", 0, 3, True, True),
                         rope_theta=10000.0)
    try:
        assert head.request(node.request("info"))["info"] == {
            "protocol_version": 1, "model_id": "m", "stage_id": "head", "start_layer": 0, "end_layer": 1,
            "is_head": True, "is_tail": False, "spec_decode_v1": True}
        prompt = "hello stage"
        ids = node.simple_tokenize(prompt, SPEC["vocab"])
        assert head.request(node.request("tokenize", text=prompt))["token_ids"] == ids
        # BeginPrompt on the head, ContinueForward on the tail: the tail answers with its sample
        r = head.request(node.request("begin_prompt", request_id="g", prompt=prompt, max_tokens=None))
        t = r["tensor"]
        assert t["stage_trace"] == ["head"] and t["hidden_dim"] == SPEC["hidden"] and "tail_sample" not in r
        r = tail.request(node.request("continue_forward", tensor=t))
        assert "tensor" not in r
        toks, h = [], ref.begin_token_ids("g", ids)
        toks.append(ref.sample_tail(h[-1])[0])
        assert r["tail_sample"] == {"token_id": toks[0], "piece": node.decode_token(toks[0]), "is_eog": False}
        got = [r["tail_sample"]["token_id"]]
        for _ in range(3):  # decode steps: ContinueHeadTokens with the sampled token
            t = head.request(node.request("continue_head_tokens", request_id="g", token_ids=[got[-1]],
                                          max_tokens=None))["tensor"]
            got.append(tail.request(node.request("continue_forward", tensor=t))["tail_sample"]["token_id"])
            toks.append(ref.sample_tail(ref.begin_token_ids("g", [toks[-1]])[-1])[0])
        assert got == toks
        # SampleTail / SampleTailToken on a tensor of final hidden rows
        rows = ref.begin_token_ids("probe", ids)
        tens = node.stage_tensor("probe", SPEC["hidden"], rows.astype(np.float32).tobytes(), max_tokens=2)
        want = ref.sample_tail(rows[-1])[0]
        r = tail.request(node.request("sample_tail", tensor=tens))["sample"]
        assert r == {"request_id": "probe", "model_id": "m", "text": node.decode_token(want) * 2,
                     "token_ids": [want, want], "completion_tokens": 2}
        assert tail.request(node.request("sample_tail_token", tensor=tens))["sample"]["token_id"] == want
        # speculative verify: drafts = the true continuation (all accepted) then a wrong one
        n0 = len(ids) + 3
        ahead = [ref.sample_tail(ref.begin_token_ids("g", [toks[-1]])[-1])[0]]
        for _ in range(3):
            ahead.append(ref.sample_tail(ref.begin_token_ids("g", [ahead[-1]])[-1])[0])
        last, drafts = toks[-1], ahead[:3]
        t = head.request(node.request("continue_head_tokens", request_id="g", token_ids=[last] + drafts,
                                      max_tokens=None))["tensor"]
        v = tail.request(node.request("continue_forward_verify_k", request_id="g", tensor=t, last_token=last,
                                      draft_tokens=drafts, clear_memory=False))
        assert v["kind"] == "verified_batch" and v["accepted_count"] == 3
        assert v["accepted_token_ids"] == ahead[:4] and v["is_eog"] is False
        assert v["accepted_pieces"] == [node.decode_token(i) for i in ahead[:4]]
        # a draft that goes wrong at its second token: one accepted, the bonus is the true token
        assert head.request(node.request("rollback_kv", request_id="g", keep_count=n0)) == {"kind": "ack"}
        assert tail.request(node.request("rollback_kv", request_id="g", keep_count=n0)) == {"kind": "ack"}
        bad = [ahead[0], (ahead[1] + 1) % SPEC["vocab"], ahead[2]]
        t = head.request(node.request("continue_head_tokens", request_id="g", token_ids=[last] + bad,
                                      max_tokens=None))["tensor"]
        v = tail.request(node.request("continue_forward_verify_k", request_id="g", tensor=t, last_token=last,
                                      draft_tokens=bad, clear_memory=False))
        assert v["accepted_count"] == 1 and v["accepted_token_ids"] == [ahead[0], ahead[1]]
        # errors come back as StageNodeResponse::Error; ClearDecodeSession acks
        with pytest.raises(RuntimeError, match="Head stage should use begin_prompt"):
            head.request(node.request("continue_forward", tensor=t))
        assert tail.request(node.request("clear_decode_session", request_id="g")) == {"kind": "ack"}
    finally:
        head.close()
        tail.close()
        th1.join(timeout=30)
        th2.join(timeout=30)
        s1.close()
        s2.close()
