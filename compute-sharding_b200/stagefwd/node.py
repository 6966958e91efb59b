"""TCP stage node: the `StageNodeRequest` v1 protocol served by a stage backend.

The reference's gateway and orchestrator drive stage nodes over TCP
(crates/llama-stage-backend/src/lib.rs).  This module speaks the same protocol:

* framing (lib.rs:2308-2370): every message is a u32 little-endian length followed by that many
  bytes of MessagePack written by `rmp_serde::to_vec_named` (structs as maps with field names in
  declaration order, `Option` as nil, byte vectors as `bin`, unit enum variants as their names);
* requests (lib.rs:606-666) are internally tagged by `op`, responses (lib.rs:737-789) by `kind`,
  both in snake_case; `StageTensor` follows crates/stage-forward-lab/src/lib.rs:151-163;
* the handler (`handle_stage_node_request`, lib.rs:3837-3982) maps each request onto the stage
  API; one connection is served at a time (bin/llama_stage_tcp_node.rs:181-192); protocol
  version 1 (lib.rs:800).

The backend behind the node is the stage-forward backend (`StageForwardBackend` with
RealGemmaBackend semantics), not the llama backend: a text prompt without a tokenizer becomes
one id per byte modulo the vocabulary (simple_tokenize, real_forward.rs:1339-1344), and sampled
ids decode as single characters below 128 and "<id>" otherwise (decode_token, :282-292).
Any object with the CudaStageBackend methods used below can serve (the CPU tests use the oracle).

    python -m stagefwd.node --pack <stage>.index.json --model-id M --stage-id head \\
        --start 0 --end 20 --head [--tail] [--listen 127.0.0.1:0]

prints `listening=<host>:<port>` on stderr once the socket accepts connections (the handshake the
reference's spawner parses, lib.rs:4118-4184).
"""
from __future__ import annotations

import argparse
import socket
import struct
import sys

import msgpack

PROTOCOL_VERSION = 1
HIDDEN_STATE, PROMPT_INGRESS = "HiddenState", "PromptIngress"


# ---------------------------------------------------------------- wire format
def pack_message(obj) -> bytes:
    """One framed message: u32 LE length + MessagePack body."""
    body = msgpack.packb(obj, use_bin_type=True)
    return struct.pack("<I", len(body)) + body


def _read_exact(sock, n: int) -> bytes:
    buf = bytearray()
    while len(buf) < n:
        chunk = sock.recv(n - len(buf))
        if not chunk:
            raise ConnectionError("peer closed the connection")
        buf += chunk
    return bytes(buf)


def read_message(sock):
    """The next framed message (None when the peer closed between messages)."""
    head = sock.recv(4, socket.MSG_WAITALL)
    if not head:
        return None
    if len(head) < 4:
        head += _read_exact(sock, 4 - len(head))
    (n,) = struct.unpack("<I", head)
    if n == 0:
        raise ValueError("empty stage message")
    return msgpack.unpackb(_read_exact(sock, n), raw=False)


def stage_tensor(request_id: str, hidden_dim: int, data: bytes, stage_trace=(), kind: str = HIDDEN_STATE,
                 max_tokens=None, prompt_text=None) -> dict:
    """StageTensor (stage-forward-lab lib.rs:151-163), fields in declaration order."""
    return {"request_id": request_id, "kind": kind, "stage_trace": list(stage_trace), "hidden_dim": int(hidden_dim),
            "bytes": bytes(data), "prompt_text": prompt_text, "max_tokens": max_tokens, "continuation": None,
            "transient": None, "carry": None}


# Request fields per op (lib.rs:606-666), in declaration order after the tag.
REQUEST_FIELDS = {
    "info": (),
    "tokenize": ("text",),
    "begin_prompt": ("request_id", "prompt", "max_tokens"),
    "continue_head_tokens": ("request_id", "token_ids", "max_tokens"),
    "continue_forward": ("tensor",),
    "continue_forward_tokens": ("tensor", "token_ids", "clear_memory"),
    "sample_tail": ("tensor",),
    "sample_tail_token": ("tensor",),
    "clear_decode_session": ("request_id",),
    "continue_head_draft_k": ("request_id", "last_token", "draft_k", "max_tokens"),
    "continue_forward_verify_k": ("request_id", "tensor", "last_token", "draft_tokens", "clear_memory"),
    "rollback_kv": ("request_id", "keep_count"),
}
OPTIONAL_FIELDS = {"max_tokens"}


def request(op: str, **fields) -> dict:
    """A StageNodeRequest as the map rmp_serde writes: {"op": ..., fields in declaration order}."""
    if op not in REQUEST_FIELDS:
        raise ValueError(f"unknown stage request op {op!r}")
    out = {"op": op}
    for name in REQUEST_FIELDS[op]:
        if name not in fields and name not in OPTIONAL_FIELDS:
            raise ValueError(f"request {op} needs field {name!r}")
        out[name] = fields.get(name)
    return out


def check_request(msg) -> dict:
    """A decoded request with its op and required fields checked (the deserializer's rules)."""
    if not isinstance(msg, dict) or not isinstance(msg.get("op"), str):
        raise ValueError("stage request is not a map with an 'op' tag")
    op = msg["op"]
    if op not in REQUEST_FIELDS:
        raise ValueError(f"unknown variant `{op}`")
    for name in REQUEST_FIELDS[op]:
        if name not in msg and name not in OPTIONAL_FIELDS:
            raise ValueError(f"missing field `{name}`")
    return msg


def response(kind: str, **fields) -> dict:
    """A StageNodeResponse map (lib.rs:737-789); optional fields that are None are left out, as
    `skip_serializing_if = "Option::is_none"` does for Tensor and VerifiedBatch."""
    out = {"kind": kind}
    for k, v in fields.items():
        if v is None and kind in ("tensor", "verified_batch") and k in ("tensor", "tail_sample", "profile"):
            continue
        out[k] = v
    return out


def node_info(msg) -> dict:
    """StageNodeInfo with `spec_decode_v1` defaulting to false when absent (lib.rs:803-816)."""
    info = dict(msg)
    info.setdefault("spec_decode_v1", False)
    return info


# ---------------------------------------------------------------- hand-off payload rows
def _aux_split(aux: bytes | None):
    """(per-row per-layer inputs as bytes, layers, ple_dim) from an "rsa1" / "rpl1" aux section
    (real_forward.rs:1852-1990); ([], 0, 0) when there is none."""
    if not aux:
        return [], 0, 0
    if aux[:4] == b"rsa1":
        seq, layers, pdim, _ = struct.unpack_from("<IIII", aux, 4)
        off = 20
    elif aux[:4] == b"rpl1":
        seq, layers, pdim = struct.unpack_from("<III", aux, 4)
        off = 16
    else:
        raise ValueError("Invalid prompt-aux payload")
    w = layers * pdim * 4
    return [aux[off + i * w: off + (i + 1) * w] for i in range(seq)], layers, pdim


def _aux_join(rows, layers: int, pdim: int) -> bytes:
    """An "rsa1" section holding per-row per-layer inputs and no prefix hashes."""
    if not rows or layers * pdim == 0:
        return b""
    return b"rsa1" + struct.pack("<IIII", len(rows), layers, pdim, 0) + b"".join(rows)


def split_payload(payload: bytes, hidden_dim: int):
    """One single-row payload per hidden row, each with its row of per-layer inputs."""
    from . import encode_stage_tensor_bytes, stage_tensor_byte_sections
    hidden, aux, _ = stage_tensor_byte_sections(payload)
    w = hidden_dim * 4
    if len(hidden) % w or not hidden:
        raise ValueError(f"Hidden-state byte length {len(hidden)} is not a multiple of hidden_dim * 4 = {w}")
    ple, layers, pdim = _aux_split(aux)
    n = len(hidden) // w
    if ple and len(ple) != n:
        raise ValueError(f"prompt aux holds {len(ple)} rows for {n} hidden rows")
    return [encode_stage_tensor_bytes(hidden[i * w:(i + 1) * w], _aux_join(ple[i:i + 1], layers, pdim) or None)
            for i in range(n)]


def join_payloads(payloads, hidden_dim: int) -> bytes:
    """The rows of several payloads as one payload (per-layer inputs concatenated, hashes dropped)."""
    from . import encode_stage_tensor_bytes, stage_tensor_byte_sections
    hidden, ple, layers, pdim = [], [], 0, 0
    for p in payloads:
        h, aux, _ = stage_tensor_byte_sections(p)
        hidden.append(h)
        rows, layers_i, pdim_i = _aux_split(aux)
        ple += rows
        layers, pdim = max(layers, layers_i), max(pdim, pdim_i)
    return encode_stage_tensor_bytes(b"".join(hidden), _aux_join(ple, layers, pdim) or None)


# ---------------------------------------------------------------- the node
def simple_tokenize(text: str, vocab: int) -> list[int]:
    """simple_tokenize (real_forward.rs:1339-1344): one id per UTF-8 byte, modulo the vocabulary."""
    return [b % max(vocab, 1) for b in text.encode("utf-8")]


def decode_token(tok: int) -> str:
    """decode_token (real_forward.rs:282-292) without a vocabulary table."""
    return chr(tok) if tok < 128 else f"<{tok}>"


class StageNode:
    """handle_stage_node_request (lib.rs:3837-3982) over a stage backend."""

    def __init__(self, backend, model_id: str, stage_id: str, start_layer: int, end_layer: int, is_head: bool,
                 is_tail: bool, hidden_dim: int, vocab: int):
        self.b = backend
        self.model_id, self.stage_id = model_id, stage_id
        self.start_layer, self.end_layer = start_layer, end_layer
        self.is_head, self.is_tail = is_head, is_tail
        self.hidden_dim, self.vocab = hidden_dim, vocab

    # -- helpers
    def _tail_sample(self, payload: bytes) -> dict:
        tok, _ = self.b.sample_tail_bytes(payload, self.hidden_dim)
        return {"token_id": int(tok), "piece": decode_token(tok), "is_eog": False}

    def _out_tensor(self, request_id: str, payload: bytes, trace, max_tokens) -> dict:
        return stage_tensor(request_id, self.hidden_dim, payload, list(trace) + [self.stage_id], HIDDEN_STATE,
                            max_tokens)

    def _forward_response(self, request_id: str, payload: bytes, trace, max_tokens) -> dict:
        # a tail answers with the sampled token and no tensor (lib.rs:3855-3866)
        if self.is_tail:
            return response("tensor", tensor=None, tail_sample=self._tail_sample(payload), profile=None)
        return response("tensor", tensor=self._out_tensor(request_id, payload, trace, max_tokens), tail_sample=None,
                        profile=None)

    def _head_tokens(self, request_id: str, ids, max_tokens, append: bool) -> dict:
        if not self.is_head:
            raise ValueError("Only the head stage may accept prompt ingress")
        if len(ids) == 0:
            raise ValueError("Empty prompt")
        if append and len(ids) > 1 and self.b.session_len(request_id) > 0:
            # ContinueHeadTokens extends the session: single-token steps append (incremental decode
            # equals a rerun of the whole sequence, real_forward.rs:3129)
            payload = join_payloads([self.b.begin_token_ids_bytes(request_id, [t]) for t in ids], self.hidden_dim)
        else:
            payload = self.b.begin_token_ids_bytes(request_id, ids)
        return self._forward_response(request_id, payload, [], max_tokens)

    def _continue(self, tensor: dict, append: bool = False) -> bytes:
        if tensor.get("kind") != HIDDEN_STATE:
            raise ValueError("Stage forward requires hidden-state payloads")
        if int(tensor["hidden_dim"]) != self.hidden_dim:
            raise ValueError(f"payload hidden_dim {tensor['hidden_dim']}, stage hidden size {self.hidden_dim}")
        data, rid = bytes(tensor["bytes"]), tensor["request_id"]
        rows = split_payload(data, self.hidden_dim) if append else [data]
        if append and len(rows) > 1:  # extend the session row by row
            return join_payloads([self.b.continue_forward_bytes(rid, p, self.hidden_dim) for p in rows],
                                 self.hidden_dim)
        return self.b.continue_forward_bytes(rid, data, self.hidden_dim)

    # -- requests
    def handle(self, msg) -> dict:
        try:
            return self._handle(check_request(msg))
        except Exception as e:  # StageNodeResponse::Error (lib.rs:3976-3981)
            return response("error", message=str(e))

    def _handle(self, r: dict) -> dict:
        op = r["op"]
        if op == "info":
            return response("info", info={"protocol_version": PROTOCOL_VERSION, "model_id": self.model_id,
                                          "stage_id": self.stage_id, "start_layer": self.start_layer,
                                          "end_layer": self.end_layer, "is_head": self.is_head,
                                          "is_tail": self.is_tail, "spec_decode_v1": True})
        if op == "tokenize":
            return response("token_ids", token_ids=simple_tokenize(r["text"], self.vocab))
        if op == "begin_prompt":
            return self._head_tokens(r["request_id"], simple_tokenize(r["prompt"], self.vocab), r.get("max_tokens"),
                                     False)
        if op == "continue_head_tokens":
            return self._head_tokens(r["request_id"], [int(t) for t in r["token_ids"]], r.get("max_tokens"), True)
        if op in ("continue_forward", "continue_forward_tokens"):
            t = r["tensor"]
            if op == "continue_forward_tokens" and r["clear_memory"]:
                self.b.clear_decode_session(t["request_id"])
            out = self._continue(t)
            return self._forward_response(t["request_id"], out, t.get("stage_trace") or [], t.get("max_tokens"))
        if op == "sample_tail":
            t = r["tensor"]
            tok, _ = self.b.sample_tail_bytes(bytes(t["bytes"]), int(t["hidden_dim"]))
            n = max(int(t.get("max_tokens") or 1), 1)  # sample_hidden_state_with_trace (:946-958)
            ids = [int(tok)] * n
            return response("sample", sample={"request_id": t["request_id"], "model_id": self.model_id,
                                              "text": "".join(decode_token(i) for i in ids), "token_ids": ids,
                                              "completion_tokens": n})
        if op == "sample_tail_token":
            t = r["tensor"]
            return response("token_sample", sample=self._tail_sample(bytes(t["bytes"])))
        if op == "clear_decode_session":
            self.b.clear_decode_session(r["request_id"])
            return response("ack")
        if op == "continue_head_draft_k":
            raise ValueError("ContinueHeadDraftK is not implemented on this node (gateway-side drafting)")
        if op == "continue_forward_verify_k":
            return self._verify(r)
        if op == "rollback_kv":
            self.b.rollback_kv(r["request_id"], int(r["keep_count"]))
            return response("ack")
        raise ValueError(f"unknown variant `{op}`")

    def _verify(self, r: dict) -> dict:
        """verify_batch_at_tail (lib.rs:2022-2234): forward [last, d1..dk] at the tail, accept while
        the greedy token at row i equals d_{i+1}, bonus = the greedy token where that stops, keep
        n_pos + accepted + 1 positions."""
        import numpy as np
        if not self.is_tail:
            raise ValueError("ContinueForwardVerifyK needs the tail stage")
        t = r["tensor"]
        drafts = [int(x) for x in r["draft_tokens"]]
        if r["clear_memory"]:
            self.b.clear_decode_session(r["request_id"])
        n_pos = self.b.session_len(r["request_id"])
        out = self._continue(dict(t, request_id=r["request_id"]), append=True)
        from . import stage_tensor_byte_sections
        hidden = np.frombuffer(stage_tensor_byte_sections(out)[0], np.float32).reshape(-1, self.hidden_dim)
        if hidden.shape[0] != len(drafts) + 1:
            raise ValueError(f"verify payload has {hidden.shape[0]} rows for {len(drafts)} draft tokens")
        accepted, bonus = self.b.verify_greedy(hidden, np.asarray(drafts, np.uint32))
        self.b.rollback_kv(r["request_id"], n_pos + accepted + 1)
        ids = drafts[:accepted] + [int(bonus)]
        return response("verified_batch", accepted_count=accepted, accepted_token_ids=ids,
                        accepted_pieces=[decode_token(i) for i in ids], is_eog=False, profile=None)


def serve(node: StageNode, sock: socket.socket, max_connections=None):
    """Serve connections one at a time (bin/llama_stage_tcp_node.rs:181-192) until max_connections
    have been served (None: forever)."""
    served = 0
    while max_connections is None or served < max_connections:
        conn, _ = sock.accept()
        with conn:
            conn.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
            while True:
                try:
                    msg = read_message(conn)
                except (ConnectionError, ValueError, msgpack.ExtraData, msgpack.FormatError):
                    break
                if msg is None:
                    break
                conn.sendall(pack_message(node.handle(msg)))
        served += 1


class StageNodeClient:
    """TcpStageClient::request (lib.rs:2308-2370): one framed request, one framed response."""

    def __init__(self, addr: str, timeout: float | None = None):
        host, port = addr.rsplit(":", 1)
        self.sock = socket.create_connection((host, int(port)), timeout=timeout)
        self.sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)

    def request(self, req: dict) -> dict:
        self.sock.sendall(pack_message(req))
        resp = read_message(self.sock)
        if resp is None:
            raise ConnectionError("tcp stage returned empty response")
        if resp.get("kind") == "error":
            raise RuntimeError(f"tcp stage error: {resp.get('message')}")
        return resp

    def close(self):
        self.sock.close()


def main(argv=None):
    ap = argparse.ArgumentParser(description="Serve one stage over the StageNodeRequest v1 TCP protocol")
    ap.add_argument("--pack", help="<stage>-required.index.json of a packed stage")
    ap.add_argument("--gguf", help="a GGUF file: the layout's tensors are read from it directly")
    ap.add_argument("--model-id", required=True)
    ap.add_argument("--stage-id", required=True)
    ap.add_argument("--start", type=int, required=True)
    ap.add_argument("--end", type=int, required=True)
    ap.add_argument("--head", action="store_true")
    ap.add_argument("--tail", action="store_true")
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--max-ctx", type=int, default=4096)
    ap.add_argument("--listen", default="127.0.0.1:0")
    a = ap.parse_args(argv)
    from . import CudaStageBackend
    if bool(a.pack) == bool(a.gguf):
        ap.error("give exactly one of --pack or --gguf")
    be = CudaStageBackend(a.pack, gguf_path=a.gguf, device=a.device, max_ctx=a.max_ctx).load_layout(
        a.model_id, a.stage_id, a.start, a.end, a.head, a.tail)
    node = StageNode(be, a.model_id, a.stage_id, a.start, a.end, a.head, a.tail, be.hidden_dim, int(be.info.vocab))
    host, port = a.listen.rsplit(":", 1)
    sock = socket.create_server((host, int(port)))
    print(f"listening={sock.getsockname()[0]}:{sock.getsockname()[1]}", file=sys.stderr, flush=True)
    serve(node, sock)


if __name__ == "__main__":
    main()
