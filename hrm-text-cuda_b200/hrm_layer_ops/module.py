"""The HRM layer loop's residual and norm schedule on the fused layer ops.

The reference runs, per transformer layer (src/lib.rs:955-1030):
    rms_norm(x) -> attention -> additive_inject(x, attn) -> rms_norm ->
    gate/up GEMMs -> swiglu_ffn -> down GEMM -> additive_inject -> memcpy;
per module (src/lib.rs:1036-1105) a memcpy of the output into a scratch input
before every later layer, and a final rms_norm + memcpy; and per cycle of the
recurrent loop (src/lib.rs:1215-1270) additive_inject(z_a, z_b) + memcpy as the
module's input.

transformer_module runs the same arithmetic as
    (x, n)  = add_rms_norm(z_a, z_b)        cycle injection + layer 0's pre-norm
    per layer i:
      attention(i, n, a)                    the caller's attention, writes a
      (x, n2) = add_rms_norm(x, a)          residual + FFN pre-norm, x in place
      gate_up(i, n2, g, u)                  the caller's two GEMMs
      swiglu_ffn(g, u, act)
      down(i, act, d)                       the caller's GEMM
      (x, n)  = add_rms_norm(x, d)          residual + the next layer's pre-norm
                                            (after the last layer: the module's
                                            final norm, written to `output`)
with no device copies.  Every value is the reference's bit for bit: each fused
call normalises the bf16-rounded sum, which is what the reference's rms_norm
reads back from additive_inject's output.

Per token and layer the residual stream moves 16 * hidden bytes here (two
fused calls of 8 * hidden) against 28 * hidden in the reference's order (two
norms, two adds, two copies), plus SwiGLU's 6 * intermediate in both.

recurrent_forward runs the loop around the modules (src/lib.rs:1189-1270):
z_H from the embedding, z_L broadcast from z_l_init, then per H-cycle
l_cycles x z_L = L(z_L + z_H) and z_H = H(z_H + z_L), with the reference's
KV-cache slot numbering.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional, Sequence

import torch

from .ops import add_rms_norm, broadcast_vec, embedding_lookup, swiglu_ffn

# attention(layer, normed [rows, H], out [rows, H])
AttentionFn = Callable[[int, torch.Tensor, torch.Tensor], None]
# gate_up(layer, normed [rows, H], gate [rows, I], up [rows, I])
GateUpFn = Callable[[int, torch.Tensor, torch.Tensor, torch.Tensor], None]
# down(layer, act [rows, I], out [rows, H])
DownFn = Callable[[int, torch.Tensor, torch.Tensor], None]


@dataclass
class ModuleNorms:
    """Optional RMSNorm weights ([hidden] bf16 each).  The reference's norms
    have no weight (src/kernels/rms_norm.cu); None everywhere reproduces it."""

    attn: Optional[Sequence[Optional[torch.Tensor]]] = None   # per layer, before attention
    ffn: Optional[Sequence[Optional[torch.Tensor]]] = None    # per layer, before the FFN
    final: Optional[torch.Tensor] = None                      # after the last layer

    def at(self, which: str, i: int) -> Optional[torch.Tensor]:
        seq = getattr(self, which)
        return None if seq is None else seq[i]


class ModuleScratch:
    """Device buffers of one module pass: the residual stream x, the normed
    activations n / n2, the attention output a, the FFN gate/up/act and the down
    projection d.  Allocated once per shape and reused across layers, modules
    and cycles (the reference's ScratchBuffers, src/lib.rs:86-112)."""

    def __init__(self, rows: int, hidden: int, intermediate: int, device, dtype=torch.bfloat16):
        def e(cols):
            return torch.empty((rows, cols), dtype=dtype, device=device)

        self.rows, self.hidden, self.intermediate = rows, hidden, intermediate
        self.x, self.n, self.n2, self.a, self.d = e(hidden), e(hidden), e(hidden), e(hidden), e(hidden)
        self.g, self.u, self.act = e(intermediate), e(intermediate), e(intermediate)


def transformer_module(z_a: torch.Tensor, z_b: torch.Tensor, output: torch.Tensor, n_layers: int,
                       attention: AttentionFn, gate_up: GateUpFn, down: DownFn, scratch: ModuleScratch, *,
                       eps: float = 1e-6, norms: Optional[ModuleNorms] = None, stream=None) -> torch.Tensor:
    """output = module(z_a + z_b): one pass of an H or L module.

    Replaces the injection at src/lib.rs:1220-1229 (L: z_L + z_H) or
    src/lib.rs:1248-1256 (H: z_H + z_L) followed by transformer_module
    (src/lib.rs:1036-1105).  `output` may be z_a itself (the recurrent loop
    writes z_L = L(z_L + z_H) in place): z_a and z_b are read only by the first
    call.  `output` must not alias z_b or a scratch buffer.
    """
    if n_layers < 1:
        raise ValueError("a module has at least one layer")
    rows, hidden = scratch.rows, scratch.hidden
    for name, t in (("z_a", z_a), ("z_b", z_b), ("output", output)):
        if t.numel() != rows * hidden:
            raise ValueError(f"{name} has {t.numel()} elements, the scratch expects {rows} x {hidden}")
    if output.data_ptr() == z_b.data_ptr():
        raise ValueError("output must not alias z_b")
    norms = norms or ModuleNorms()
    s = scratch
    x, n = s.x, s.n
    add_rms_norm(z_a.view(rows, hidden), z_b.view(rows, hidden), norms.at("attn", 0), eps,
                 residual_out=x, normed_out=n, stream=stream)
    for i in range(n_layers):
        attention(i, n, s.a)
        add_rms_norm(x, s.a, norms.at("ffn", i), eps, residual_out=x, normed_out=s.n2, stream=stream)
        gate_up(i, s.n2, s.g, s.u)
        swiglu_ffn(s.g, s.u, s.act, stream=stream)
        down(i, s.act, s.d)
        last = i == n_layers - 1
        w = norms.final if last else norms.at("attn", i + 1)
        add_rms_norm(x, s.d, w, eps, residual_out=x, normed_out=output.view(rows, hidden) if last else n,
                     stream=stream)
    return output


def module_bytes_per_token(hidden: int, intermediate: int, n_layers: int) -> int:
    """Algorithmic bytes per token of transformer_module's own kernels (bf16):
    the injection call (reads z_a, z_b, writes x, n: 8 * hidden), then per
    layer two fused calls (8 * hidden each) and SwiGLU (6 * intermediate)."""
    return 8 * hidden + n_layers * (16 * hidden + 6 * intermediate)


def reference_order_bytes_per_token(hidden: int, intermediate: int, n_layers: int) -> int:
    """The same pass in the reference's order (bf16): injection add (6H) and
    copy (4H); per layer two norms (4H each), two adds (6H each), the residual
    copy (4H) and SwiGLU (6I); a copy of the output before every later layer
    (4H); the final norm (4H) and its copy (4H)."""
    return (10 * hidden + n_layers * (24 * hidden + 6 * intermediate) + (n_layers - 1) * 4 * hidden
            + 8 * hidden)


# attention(layer, kv_slot, normed [rows, H], out [rows, H]) of recurrent_forward
SlotAttentionFn = Callable[[int, int, torch.Tensor, torch.Tensor], None]


@dataclass
class ModuleFns:
    """One module (H or L) for recurrent_forward: its layer count, the caller's
    attention (given the layer and the KV-cache slot) and FFN GEMMs, and
    optional norm weights."""

    n_layers: int
    attention: SlotAttentionFn
    gate_up: GateUpFn
    down: DownFn
    norms: Optional[ModuleNorms] = None


def recurrent_forward(input_ids: torch.Tensor, embed_table: torch.Tensor, embedding_scale: float,
                      z_l_init: torch.Tensor, h_cycles: int, l_cycles: int, l_module: ModuleFns,
                      h_module: ModuleFns, scratch: ModuleScratch, *, eps: float = 1e-6,
                      z_h: Optional[torch.Tensor] = None, z_l: Optional[torch.Tensor] = None, stream=None):
    """(z_H, z_L) after the HRM recurrent loop over `input_ids` (rows tokens).

    src/lib.rs:1189-1270: z_H = embedding_lookup(ids) * scale (1189-1200);
    z_L = broadcast(z_l_init) (1202-1203); then for each of h_cycles:
    l_cycles times z_L = L(z_L + z_H), then z_H = H(z_H + z_L), every module
    pass through transformer_module.  KV-cache slots are numbered as the
    reference's kv_slot_counter: each module pass takes the next n_layers slots,
    and its attention sees slot = base + layer.  The LM head, sampling and the
    cache itself stay with the caller.
    """
    rows, hidden = scratch.rows, scratch.hidden
    if input_ids.numel() != rows:
        raise ValueError(f"{input_ids.numel()} token ids for a scratch of {rows} rows")
    z_h = embedding_lookup(input_ids.reshape(-1), embed_table, embedding_scale, out=z_h, stream=stream)
    z_l = broadcast_vec(z_l_init.reshape(-1), rows, out=z_l, stream=stream)
    slot = 0

    def run(m: ModuleFns, z_a: torch.Tensor, z_b: torch.Tensor, base: int) -> None:
        transformer_module(z_a, z_b, z_a, m.n_layers, lambda i, n, o: m.attention(i, base + i, n, o), m.gate_up,
                           m.down, scratch, eps=eps, norms=m.norms, stream=stream)

    for _ in range(h_cycles):
        for _ in range(l_cycles):
            run(l_module, z_l, z_h, slot)
            slot += l_module.n_layers
        run(h_module, z_h, z_l, slot)
        slot += h_module.n_layers
    return z_h.view(rows, hidden), z_l.view(rows, hidden)
