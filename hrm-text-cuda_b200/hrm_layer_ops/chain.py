"""The chained per-token layer-op pass, on device buffers or on host buffers.

One pass over T tokens runs the four kernels the HRM layer loop uses between
its GEMMs (src/lib.rs:1191-1200, 969, 828, 976-979, 998):

    h, n1  = embed_rms_norm(ids, table, scale, w1)     embedding gather + RMSNorm
    q, k   = rope_embed(q, k, offset, table)          in place, [B, 16, S, 128]
    r, n2  = add_rms_norm(h, o, w2)                   residual add + RMSNorm
    y      = swiglu_ffn(gate, up)

`run_device` queues the four launches on one stream.  `HostChain` takes
pinned host buffers and streams the pass through the GPU in chunks of whole
Q/K batches: chunk i+1 is copied in while chunk i computes and chunk i-1 is
copied out, on three streams ordered by events, so PCIe traffic in both
directions overlaps the kernels.
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
               stream: Optional[torch.cuda.Stream] = None, events: Optional[List] = None) -> None:
    """Queues the four launches; `events` (5 CUDA events) brackets each kernel if given."""
    def mark(i):
        if events is not None:
            events[i].record(stream)

    mark(0)
    ops.embed_rms_norm(ids, w.table, w.scale, w.w1, w.eps, hidden_out=h, normed_out=n1, stream=stream)
    mark(1)
    ops.rope_embed(q, k, offset, w.theta, w.rope, stream=stream)
    mark(2)
    ops.add_rms_norm(h, o, w.w2, w.eps, residual_out=r, normed_out=n2, stream=stream)
    mark(3)
    ops.swiglu_ffn(gate, up, out=y, stream=stream)
    mark(4)


class HostChain:
    """Runs the chain on pinned host tensors, chunked by Q/K batch.

    Host inputs:  ids [T] int32, q, k [B, heads, S, hd] bf16, o [T, hidden],
                  gate, up [T, inter]      (T = B * S; rows of batch b are b*S..)
    Host outputs: q, k (rotated, written back in place), h, n1, r, n2 [T, hidden],
                  y [T, inter].
    Device staging: two slots of every per-chunk buffer (double buffering).
    """

    def __init__(self, weights: ChainWeights, batch: int, heads: int, seq: int, head_dim: int, hidden: int,
                 inter: int, chunk_batches: int = 1, device=None):
        self.w = weights
        self.B, self.heads, self.S, self.hd = batch, heads, seq, head_dim
        self.hidden, self.inter = hidden, inter
        self.cb = chunk_batches
        if batch % chunk_batches:
            raise ValueError("batch must be a multiple of chunk_batches")
        self.device = torch.device(device if device is not None else "cuda")
        ct = chunk_batches * seq
        bf = dict(dtype=torch.bfloat16, device=self.device)
        self.slots = [dict(
            ids=torch.empty(ct, dtype=torch.int32, device=self.device),
            q=torch.empty((chunk_batches, heads, seq, head_dim), **bf),
            k=torch.empty((chunk_batches, heads, seq, head_dim), **bf),
            o=torch.empty((ct, hidden), **bf), gate=torch.empty((ct, inter), **bf),
            up=torch.empty((ct, inter), **bf), h=torch.empty((ct, hidden), **bf),
            n1=torch.empty((ct, hidden), **bf), r=torch.empty((ct, hidden), **bf),
            n2=torch.empty((ct, hidden), **bf), y=torch.empty((ct, inter), **bf)) for _ in range(2)]
        self.s_in = torch.cuda.Stream(self.device)
        self.s_cmp = torch.cuda.Stream(self.device)
        self.s_out = torch.cuda.Stream(self.device)

    IN = ("ids", "q", "k", "o", "gate", "up")
    OUT = ("q", "k", "h", "n1", "r", "n2", "y")

    def bytes_per_pass(self, host_in: Dict[str, torch.Tensor], host_out: Dict[str, torch.Tensor]):
        return (sum(host_in[n].numel() * host_in[n].element_size() for n in self.IN),
                sum(host_out[n].numel() * host_out[n].element_size() for n in self.OUT))

    def _chunk(self, t: torch.Tensor, name: str, c: int) -> torch.Tensor:
        if name in ("q", "k"):
            return t[c * self.cb:(c + 1) * self.cb]
        ct = self.cb * self.S
        return t[c * ct:(c + 1) * ct]

    def run(self, host_in: Dict[str, torch.Tensor], host_out: Dict[str, torch.Tensor], offset: int = 0) -> int:
        """Queues the whole pass; returns the number of kernel launches queued."""
        n_chunks = self.B // self.cb
        loaded = [torch.cuda.Event() for _ in range(n_chunks)]
        computed = [torch.cuda.Event() for _ in range(n_chunks)]
        drained = [torch.cuda.Event() for _ in range(n_chunks)]
        launches = 0
        for c in range(n_chunks):
            slot = self.slots[c % 2]
            with torch.cuda.stream(self.s_in):
                if c >= 2:
                    self.s_in.wait_event(drained[c - 2])  # slot free again
                for n in self.IN:
                    slot[n].copy_(self._chunk(host_in[n], n, c), non_blocking=True)
                loaded[c].record(self.s_in)
            self.s_cmp.wait_event(loaded[c])
            run_device(self.w, slot["ids"], slot["q"], slot["k"], slot["o"], slot["gate"], slot["up"], slot["h"],
                       slot["n1"], slot["r"], slot["n2"], slot["y"], offset, stream=self.s_cmp)
            launches += len(CHAIN_KERNELS)
            computed[c].record(self.s_cmp)
            with torch.cuda.stream(self.s_out):
                self.s_out.wait_event(computed[c])
                for n in self.OUT:
                    self._chunk(host_out[n], n, c).copy_(slot[n], non_blocking=True)
                drained[c].record(self.s_out)
        torch.cuda.current_stream(self.device).wait_stream(self.s_out)
        return launches
