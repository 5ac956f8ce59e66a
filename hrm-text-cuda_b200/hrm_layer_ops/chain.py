"""The chained per-token layer-op pass, on device buffers or on host buffers.

One pass over T tokens runs the four kernels the HRM layer loop uses between
its GEMMs (src/lib.rs:1191-1200, 969, 828, 976-979, 998):

    h, n1  = embed_rms_norm(ids, table, scale, w1)     embedding gather + RMSNorm
    q, k   = rope_embed(q, k, offset, table)          in place, [B, 16, S, 128] or [B, S, 16, 128]
    r, n2  = add_rms_norm(h, o, w2)                   residual add + RMSNorm
    y      = swiglu_ffn(gate, up)

`run_device` queues the four launches on one stream.  `HostChain` takes
pinned host buffers and streams the pass through the GPU in chunks of tokens:
chunk i+1 is copied in while chunk i computes and chunk i-1 is copied out, on
three streams ordered by events, so PCIe traffic in both directions overlaps
the kernels.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional

import torch

from . import ops

CHAIN_KERNELS = ("embed_rms_norm", "rope_embed", "add_rms_norm", "swiglu_ffn")


@dataclass
class ChainWeights:
    table: torch.Tensor       # [vocab, hidden] bf16
    w1: torch.Tensor          # [hidden] bf16
    w2: torch.Tensor          # [hidden] bf16
    rope: torch.Tensor        # [positions, head_dim] fp32 (ops.rope_table)
    scale: float
    eps: float
    theta: float


def algorithmic_bytes_per_token(hidden: int, heads: int, head_dim: int, inter: int) -> Dict[str, int]:
    """Bytes each kernel must move per token, counted from its inputs and outputs
    (the gathered table row, not the table; weights and rope table excluded as
    L2-resident constants).  'minimal' is the whole pass with every
    intermediate kept on chip: ids + row + n1 + Q/K r/w + o + r + n2 + gate/up + y."""
    row, qk = 2 * hidden, 2 * heads * head_dim
    per = {
        "embed_rms_norm": 4 + row + row + row,   # id, table row, h, n1
        "rope_embed": 2 * qk + 2 * qk,           # Q, K read and written
        "add_rms_norm": 4 * row,                 # h, o read; r, n2 written
        "swiglu_ffn": 3 * 2 * inter,             # gate, up read; y written
    }
    per["op_sum"] = sum(per[k] for k in CHAIN_KERNELS)
    per["minimal"] = 4 + row + row + 4 * qk + row + row + row + 2 * 2 * inter + 2 * inter
    return per


def run_device(w: ChainWeights, ids, q, k, o, gate, up, h, n1, r, n2, y, offset: int = 0,
               stream: Optional[torch.cuda.Stream] = None, events: Optional[List] = None,
               token_major: bool = False) -> None:
    """Queues the four launches; `events` (5 CUDA events) brackets each kernel if given.

    q, k are [batch, heads, seq, head_dim] (the reference's layout) or, with
    token_major, [batch, seq, heads, head_dim]; token s is at position
    offset + s.
    """
    def mark(i):
        if events is not None:
            events[i].record(stream)

    mark(0)
    ops.embed_rms_norm(ids, w.table, w.scale, w.w1, w.eps, hidden_out=h, normed_out=n1, stream=stream)
    mark(1)
    if token_major:
        ops.rope_embed_token_major(q, k, offset, w.theta, w.rope, stream=stream)
    else:
        ops.rope_embed(q, k, offset, w.theta, w.rope, stream=stream)
    mark(2)
    ops.add_rms_norm(h, o, w.w2, w.eps, residual_out=r, normed_out=n2, stream=stream)
    mark(3)
    ops.swiglu_ffn(gate, up, out=y, stream=stream)
    mark(4)


class HostChain:
    """Runs the chain on pinned host tensors, streaming it through the GPU in chunks.

    Host inputs:  ids [T] int32, q, k bf16, o [T, hidden], gate, up [T, inter]
    Host outputs: q, k (rotated), h, n1, r, n2 [T, hidden], y [T, inter]
    (T = batch * seq; token t is position t % seq of sequence t // seq).

    Token-major q, k ([batch, seq, heads, head_dim]) let every tensor be cut
    into contiguous ranges of `chunk_tokens` tokens (a divisor of seq), each
    rotated at its own position offset; head-major q, k ([batch, heads, seq,
    head_dim]) are cut into whole sequences.  Two device slots of every
    per-chunk buffer alternate (double buffering).  A slot is refilled only
    after the copies out of it -- from this pass or the previous one -- have
    finished, so consecutive passes may overlap: one pass's last copies out
    run under the next pass's first copies in.
    """

    IN = ("ids", "q", "k", "o", "gate", "up")
    OUT = ("q", "k", "h", "n1", "r", "n2", "y")

    def __init__(self, weights: ChainWeights, batch: int, heads: int, seq: int, head_dim: int, hidden: int,
                 inter: int, chunk_tokens: Optional[int] = None, token_major: bool = True, device=None):
        self.w = weights
        self.B, self.heads, self.S, self.hd = batch, heads, seq, head_dim
        self.hidden, self.inter = hidden, inter
        self.token_major = token_major
        self.ct = (chunk_tokens or seq) if token_major else seq
        if seq % self.ct:
            raise ValueError("chunk_tokens must divide seq")
        self.device = torch.device(device if device is not None else "cuda")
        ct = self.ct
        bf = dict(dtype=torch.bfloat16, device=self.device)
        qk_shape = (1, ct, heads, head_dim) if token_major else (1, heads, seq, head_dim)
        self.slots = [dict(
            ids=torch.empty(ct, dtype=torch.int32, device=self.device),
            q=torch.empty(qk_shape, **bf), k=torch.empty(qk_shape, **bf),
            o=torch.empty((ct, hidden), **bf), gate=torch.empty((ct, inter), **bf),
            up=torch.empty((ct, inter), **bf), h=torch.empty((ct, hidden), **bf),
            n1=torch.empty((ct, hidden), **bf), r=torch.empty((ct, hidden), **bf),
            n2=torch.empty((ct, hidden), **bf), y=torch.empty((ct, inter), **bf)) for _ in range(2)]
        self.s_in = torch.cuda.Stream(self.device)
        self.s_cmp = torch.cuda.Stream(self.device)
        self.s_out = torch.cuda.Stream(self.device)
        self.slot_free = [None, None]  # per slot: event after the last copies out of it

    def bytes_per_pass(self, host_in: Dict[str, torch.Tensor], host_out: Dict[str, torch.Tensor]):
        return (sum(host_in[n].numel() * host_in[n].element_size() for n in self.IN),
                sum(host_out[n].numel() * host_out[n].element_size() for n in self.OUT))

    def _chunk(self, t: torch.Tensor, name: str, c: int) -> torch.Tensor:
        t0, t1 = c * self.ct, (c + 1) * self.ct
        if name in ("q", "k"):
            if self.token_major:
                return t.view(1, self.B * self.S, self.heads, self.hd)[:, t0:t1]
            return t[c:c + 1]
        return t[t0:t1]

    def run(self, host_in: Dict[str, torch.Tensor], host_out: Dict[str, torch.Tensor], offset: int = 0) -> int:
        """Queues the whole pass; returns the number of kernel launches queued."""
        n_chunks = self.B * self.S // self.ct
        launches = 0
        for c in range(n_chunks):
            slot = self.slots[c % 2]
            loaded, computed, drained = torch.cuda.Event(), torch.cuda.Event(), torch.cuda.Event()
            with torch.cuda.stream(self.s_in):
                if self.slot_free[c % 2] is not None:
                    self.s_in.wait_event(self.slot_free[c % 2])  # copies out of this slot are done
                for n in self.IN:
                    slot[n].copy_(self._chunk(host_in[n], n, c), non_blocking=True)
                loaded.record(self.s_in)
            self.s_cmp.wait_event(loaded)
            pos = offset + (c * self.ct) % self.S if self.token_major else offset
            run_device(self.w, slot["ids"], slot["q"], slot["k"], slot["o"], slot["gate"], slot["up"], slot["h"],
                       slot["n1"], slot["r"], slot["n2"], slot["y"], pos, stream=self.s_cmp,
                       token_major=self.token_major)
            launches += len(CHAIN_KERNELS)
            computed.record(self.s_cmp)
            with torch.cuda.stream(self.s_out):
                self.s_out.wait_event(computed)
                for n in self.OUT:
                    self._chunk(host_out[n], n, c).copy_(slot[n], non_blocking=True)
                drained.record(self.s_out)
            self.slot_free[c % 2] = drained
        torch.cuda.current_stream(self.device).wait_stream(self.s_out)
        return launches
