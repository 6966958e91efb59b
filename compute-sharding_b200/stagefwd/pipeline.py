"""Pipeline-parallel stage driver: one process per GPU, layer ranges per rank, hidden states
handed between ranks with torch.distributed send/recv (NCCL over NVLink on B200, gloo on CPU).

The reference splits layers with `suggest_even_stage_split` (crates/stage-forward-lab/src/
gguf.rs:307-329) and moves the f32 hidden state [T, hidden] head->tail over TCP
(crates/llama-stage-backend/src/lib.rs:1505-1562, :2308-2370); the gateway returns the tail's
sampled token to the head for the next step (lib.rs:3374-3490).  Here the same flow runs as
P2P messages: hidden rows travel rank r -> r+1 on one process group, sampled tokens travel
tail -> head on a second group so the two directions never queue behind each other.

The driver is generic over the per-rank compute (`StageCompute`): the CUDA stage on GPUs, or
any object with the same two methods (the CPU tests drive it with the oracle over gloo).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


def even_stage_split(total_layers: int, stages: int) -> list[tuple[int, int]]:
    """gguf.rs:307-329: the first `total % stages` stages take one extra layer."""
    if stages <= 0 or stages > total_layers:
        raise ValueError(f"cannot split {total_layers} layers into {stages} stages")
    base, rem = divmod(total_layers, stages)
    out, start = [], 0
    for i in range(stages):
        span = base + (1 if i < rem else 0)
        out.append((start, start + span - 1))
        start += span
    return out


def balanced_stage_split(total_layers: int, stages: int, tail_cost: float = 0.0) -> list[tuple[int, int]]:
    """Contiguous layer ranges that minimise the largest stage cost, every layer costing 1 and the
    tail stage carrying `tail_cost` more (its logits pass, in layers' worth).  With tail_cost 0 the
    result has the same stage sizes as even_stage_split, ordered so that earlier stages take the
    extra layers (gguf.rs:307-329).  The reference offers only the even split; this option exists for
    the tail's tied-embedding logits (1.34 GB per pass for the 262144 x 2560 table)."""
    if stages <= 0 or stages > total_layers:
        raise ValueError(f"cannot split {total_layers} layers into {stages} stages")
    if tail_cost <= 0:
        return even_stage_split(total_layers, stages)

    def fits(cap):  # greedy from the tail: the tail first, then as many layers per stage as fit
        sizes, left = [], total_layers
        for i in range(stages):
            budget = cap - (tail_cost if i == 0 else 0.0)
            rest = stages - i - 1  # stages still to fill need at least one layer each
            take = min(int(budget + 1e-9), left - rest)
            if take < 1:
                return None
            sizes.append(take)
            left -= take
        return sizes[::-1] if left == 0 else None

    lo, hi = 1.0, float(total_layers) + tail_cost
    best = fits(hi)
    for _ in range(60):  # bisection on the largest stage cost
        mid = (lo + hi) / 2
        got = fits(mid)
        if got is None:
            lo = mid
        else:
            hi, best = mid, got
    # the tail takes the most layers its share allows; the rest are split evenly over the other
    # stages (earlier stages take the extra layers, as the even split does)
    tail = min(int(hi - tail_cost + 1e-9), total_layers - (stages - 1))
    if stages > 1 and tail >= 1 and -(-(total_layers - tail) // (stages - 1)) <= hi + 1e-9:
        return even_stage_split(total_layers - tail, stages - 1) + [(total_layers - tail, total_layers - 1)]
    out, start = [], 0
    for n in best:
        out.append((start, start + n - 1))
        start += n
    return out


class StageCompute:
    """Per-rank compute interface used by the pipeline driver."""

    def forward(self, request_ids, seq_tokens, x, append: bool):  # x: int64/uint32 ids (head) or [T, H] rows
        raise NotImplementedError

    def sample(self, hidden):  # [n, H] -> int64 [n]
        raise NotImplementedError


class CudaCompute(StageCompute):
    """StageCompute over the CUDA stage (device tensors, current torch stream)."""

    def __init__(self, backend, hidden: int, max_rows: int, device):
        self.b = backend
        self.hidden = hidden
        self.out = torch.empty((max_rows, hidden), dtype=torch.float32, device=device)
        self.ids = torch.empty(max_rows, dtype=torch.int32, device=device)
        self.tok = torch.empty(max_rows, dtype=torch.int64, device=device)
        self.score = torch.empty(max_rows, dtype=torch.float32, device=device)

    def forward(self, request_ids, seq_tokens, x, append=True):
        T = int(sum(seq_tokens))
        out = self.out[:T]
        if x.dtype in (torch.int64, torch.int32):
            ids = self.ids[:T]
            ids.copy_(x.to(torch.int32))
            self.b.forward_dev(request_ids, seq_tokens, ids_dev=ids, out_dev=out, append=append)
        else:
            self.b.forward_dev(request_ids, seq_tokens, in_dev=x.contiguous(), out_dev=out, append=append)
        return out

    def sample(self, hidden):
        n = hidden.shape[0]
        self.b.sample_dev(hidden, self.tok[:n], self.score[:n])
        return self.tok[:n]


@dataclass
class PipeRanks:
    rank: int
    world: int
    fwd_group: object = None   # all ranks (hidden rows r -> r+1)
    back_group: object = None  # {0, world-1} (tokens tail -> head)

    @property
    def is_head(self):
        return self.rank == 0

    @property
    def is_tail(self):
        return self.rank == self.world - 1


def make_groups(rank: int, world: int) -> PipeRanks:
    pr = PipeRanks(rank, world)
    if world > 1:
        pr.fwd_group = dist.new_group(list(range(world)))
        pr.back_group = dist.new_group([0, world - 1])
    return pr


class Pipeline:
    """Drives one stage per rank through prefill and decode steps.

    Sends are non-blocking (isend on a private copy, completed at the end of a step or of a
    decode run): a rank never waits for its peer to post the matching receive, so the forward
    and backward message streams cannot deadlock against each other."""

    def __init__(self, compute: StageCompute, ranks: PipeRanks, hidden: int, device):
        self.c = compute
        self.r = ranks
        self.hidden = hidden
        self.device = device
        self._pending = []

    def _recv_rows(self, n):
        buf = torch.empty((n, self.hidden), dtype=torch.float32, device=self.device)
        dist.recv(buf, src=self.r.rank - 1, group=self.r.fwd_group)
        return buf

    def _isend(self, t, dst, group):
        t = t.contiguous().clone()
        self._pending.append((dist.isend(t, dst=dst, group=group), t))

    def _send_rows(self, rows):
        self._isend(rows, self.r.rank + 1, self.r.fwd_group)

    def flush(self):
        for w, _ in self._pending:
            w.wait()
        self._pending.clear()

    def step(self, request_ids, seq_tokens, tokens, append=True):
        """One pipeline pass.  Head gives `tokens` (int64 [sum]); returns the sampled tokens
        on the head (int64 [len(request_ids)], the last row of each sequence) and None elsewhere."""
        T = int(sum(seq_tokens))
        x = tokens if self.r.is_head else self._recv_rows(T)
        y = self.c.forward(request_ids, seq_tokens, x, append)
        if not self.r.is_tail:
            self._send_rows(y)
        nxt = None
        if self.r.is_tail:
            last = torch.tensor([sum(seq_tokens[: i + 1]) - 1 for i in range(len(seq_tokens))], device=y.device)
            nxt = self.c.sample(y.index_select(0, last)).to(torch.int64).clone()
            if self.r.world > 1:
                self._isend(nxt, 0, self.r.back_group)
        if self.r.is_head and self.r.world > 1:
            nxt = torch.empty(len(request_ids), dtype=torch.int64, device=self.device)
            dist.recv(nxt, src=self.r.world - 1, group=self.r.back_group)
        self.flush()
        return nxt

    def generate(self, request_id: str, prompt: torch.Tensor, n_steps: int):
        """Greedy generation of one sequence (the reference's generate loop,
        bin/real_two_stage_generate_bench.rs:232-290). Returns tokens on the head."""
        tok = self.step([request_id], [int(prompt.numel())], prompt, append=False)
        out = [tok]
        for _ in range(n_steps - 1):
            tok = self.step([request_id], [1], tok, append=True)
            out.append(tok)
        return torch.cat(out) if self.r.is_head else None

    def decode_microbatched(self, microbatches, tokens, n_steps: int):
        """Batched decode with microbatches in flight across stages.  `microbatches` is a list
        of request-id lists; `tokens[m]` holds the next input token of each sequence of
        microbatch m (head only).  On return the head's `tokens[m]` are the tokens sampled at
        the last step (the next inputs), whatever the number of ranks.  Sends and receives keep
        one order on every rank: the tail sends every step's samples, the head receives step
        s-1's samples before step s and the last step's after the loop."""
        M = len(microbatches)
        two_way = self.r.world > 1

        def recv_tokens(m):
            nxt = torch.empty(len(microbatches[m]), dtype=torch.int64, device=self.device)
            dist.recv(nxt, src=self.r.world - 1, group=self.r.back_group)
            tokens[m] = nxt

        for s in range(n_steps):
            for m in range(M):
                ids = microbatches[m]
                n = len(ids)
                if self.r.is_head:
                    if s > 0 and two_way:
                        recv_tokens(m)
                    x = tokens[m]
                else:
                    x = self._recv_rows(n)
                y = self.c.forward(ids, [1] * n, x, True)
                if not self.r.is_tail:
                    self._send_rows(y)
                else:
                    nxt = self.c.sample(y).to(torch.int64).clone()
                    if two_way:
                        self._isend(nxt, 0, self.r.back_group)
                    else:
                        tokens[m] = nxt
            if len(self._pending) > 4 * M:
                self._pending[0][0].wait()
                self._pending.pop(0)
        if self.r.is_head and two_way and n_steps > 0:
            for m in range(M):
                recv_tokens(m)
        self.flush()
        return tokens
