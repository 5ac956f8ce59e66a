"""PyTorch-tensor front end of the C ABI (one function per hrm_* entry point).

Tensors supply device memory and the stream; every operator runs in
libhrm_ops.so.  Inputs must be contiguous CUDA tensors, all on one device; a
CPU tensor, or a tensor on another GPU, is an error, never a silent fallback.
The launch runs with that device current (the library sizes its grids from
the current device and launches there), by default on its current torch
stream.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from ._lib import call

_vp = ctypes.c_void_p


def _ptr(t: Optional[torch.Tensor]) -> Optional[ctypes.c_void_p]:
    return None if t is None else _vp(t.data_ptr())


def _stream(t: torch.Tensor, stream: Optional[torch.cuda.Stream]) -> ctypes.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream(t.device)
    return _vp(s.cuda_stream)


def _launch(name: str, tensors, stream: Optional[torch.cuda.Stream], *args) -> None:
    """Calls `name` with `args` and the stream, with the device of `tensors`
    current.  Every tensor (None entries skipped) must be on that one device,
    and so must an explicit stream: a pointer into another GPU's memory would
    reach the kernel as an illegal address."""
    ts = [t for t in tensors if t is not None]
    dev = ts[0].device
    for t in ts[1:]:
        if t.device != dev:
            raise ValueError(f"{name}: tensors on {dev} and {t.device}; every argument must be on one device")
    if stream is not None and stream.device != dev:
        raise ValueError(f"{name}: stream on {stream.device} but tensors on {dev}")
    with torch.cuda.device(dev):
        call(name, *args, _stream(ts[0], stream))


def _need(t: torch.Tensor, name: str, dtypes=(torch.bfloat16,)) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (there is no CPU implementation)")
    if t.dtype not in dtypes:
        raise TypeError(f"{name} has dtype {t.dtype}, expected one of {dtypes}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _ids(t: torch.Tensor, name: str) -> None:
    """Token ids: uint32 (the reference's type) or int32 read as uint32, so a
    negative int32 id is a huge uint32 and clamps to vocab - 1 like any id at
    or beyond the vocabulary (src/kernels/embedding_lookup.cu:35)."""
    _need(t, name, (torch.int32, torch.uint32))


def additive_inject(z_a: torch.Tensor, z_b: torch.Tensor, out: Optional[torch.Tensor] = None, *,
                    stream=None) -> torch.Tensor:
    """out = z_a + z_b (bf16, fp32 add, RNE).  src/lib.rs:378-399."""
    _need(z_a, "z_a"); _need(z_b, "z_b")
    if z_a.numel() != z_b.numel():
        raise ValueError("z_a and z_b differ in size")
    out = torch.empty_like(z_a) if out is None else out
    _need(out, "out")
    if out.numel() != z_a.numel():
        raise ValueError("out has the wrong size")
    _launch("hrm_additive_inject", (z_a, z_b, out), stream, _ptr(z_a), _ptr(z_b), _ptr(out), z_a.numel())
    return out


def swiglu_ffn(gate: torch.Tensor, up: torch.Tensor, out: Optional[torch.Tensor] = None, *,
               stream=None) -> torch.Tensor:
    """out = silu(gate) * up (bf16 I/O, fp32 math).  src/lib.rs:483-504."""
    _need(gate, "gate"); _need(up, "up")
    if gate.numel() != up.numel():
        raise ValueError("gate and up differ in size")
    out = torch.empty_like(gate) if out is None else out
    _need(out, "out")
    if out.numel() != gate.numel():
        raise ValueError("out has the wrong size")
    _launch("hrm_swiglu_ffn", (gate, up, out), stream, _ptr(gate), _ptr(up), _ptr(out), gate.numel())
    return out


def _rows(x: torch.Tensor) -> Tuple[int, int]:
    hidden = x.shape[-1] if x.dim() > 0 else 0
    return (x.numel() // hidden if hidden else 0), hidden


def rms_norm(x: torch.Tensor, weight: Optional[torch.Tensor] = None, eps: float = 1e-6,
             out: Optional[torch.Tensor] = None, *, stream=None) -> torch.Tensor:
    """RMSNorm over the last dim; bf16 or fp32 I/O (weight of the same dtype or None).

    src/lib.rs:401-422 (bf16, weight None is the reference's parameterless form).
    """
    _need(x, "x", (torch.bfloat16, torch.float32))
    rows, hidden = _rows(x)
    if weight is not None:
        _need(weight, "weight", (x.dtype,))
        if weight.numel() != hidden:
            raise ValueError("weight must have hidden_size elements")
    out = torch.empty_like(x) if out is None else out
    _need(out, "out", (x.dtype,))
    if out.numel() != x.numel():
        raise ValueError("out has the wrong size")
    fn = "hrm_rms_norm" if x.dtype == torch.bfloat16 else "hrm_rms_norm_f32"
    _launch(fn, (x, weight, out), stream, _ptr(x), _ptr(out), _ptr(weight), rows, hidden, eps)
    return out


def add_rms_norm(x: torch.Tensor, branch: torch.Tensor, weight: Optional[torch.Tensor] = None,
                 eps: float = 1e-6, residual_out: Optional[torch.Tensor] = None,
                 normed_out: Optional[torch.Tensor] = None, *, stream=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """(r, y) = (x + branch, rms_norm(x + branch) [* weight]) in one pass (bf16).

    Replaces additive_inject -> rms_norm (src/lib.rs:976-979).
    """
    _need(x, "x"); _need(branch, "branch")
    if x.shape != branch.shape:
        raise ValueError("x and branch differ in shape")
    rows, hidden = _rows(x)
    if weight is not None:
        _need(weight, "weight")
        if weight.numel() != hidden:
            raise ValueError("weight must have hidden_size elements")
    residual_out = torch.empty_like(x) if residual_out is None else residual_out
    normed_out = torch.empty_like(x) if normed_out is None else normed_out
    _need(residual_out, "residual_out"); _need(normed_out, "normed_out")
    if residual_out.numel() != x.numel() or normed_out.numel() != x.numel():
        raise ValueError("outputs have the wrong size")
    _launch("hrm_add_rms_norm", (x, branch, weight, residual_out, normed_out), stream, _ptr(x), _ptr(branch),
            _ptr(residual_out), _ptr(normed_out), _ptr(weight), rows, hidden, eps)
    return residual_out, normed_out


def rope_table(max_positions: int, head_dim: int, theta: float = 10000.0,
               device: Optional[torch.device] = None, out: Optional[torch.Tensor] = None, *,
               stream=None) -> torch.Tensor:
    """fp32 [max_positions, head_dim] table: cos in [:, :hd/2], sin in [:, hd/2:]."""
    if out is None:
        device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        out = torch.empty((max_positions, head_dim), dtype=torch.float32, device=device)
    _need(out, "out", (torch.float32,))
    if out.numel() != max_positions * head_dim:
        raise ValueError("out has the wrong size")
    _launch("hrm_rope_table_build", (out,), stream, _ptr(out), max_positions, head_dim, theta)
    return out


def rope_embed(q: torch.Tensor, k: torch.Tensor, position_offset: int = 0, theta: float = 10000.0,
               table: Optional[torch.Tensor] = None, *, stream=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """In-place rotate-half RoPE on q, k of shape [batch, heads, seq, head_dim].

    table=None evaluates angles in-kernel; otherwise a rope_table(...) with at
    least position_offset + seq rows.  src/lib.rs:424-458.
    """
    _need(q, "q"); _need(k, "k")
    if q.dim() != 4 or q.shape != k.shape:
        raise ValueError("q and k must both be [batch, heads, seq, head_dim]")
    b, h, s, d = q.shape
    positions = 0
    if table is not None:
        _need(table, "table", (torch.float32,))
        if table.dim() != 2 or table.shape[1] != d:
            raise ValueError("table must be [positions, head_dim]")
        positions = table.shape[0]
    _launch("hrm_rope_embed", (q, k, table), stream, _ptr(q), _ptr(k), b, h, s, d, position_offset, theta,
            _ptr(table), positions)
    return q, k


def rope_embed_token_major(q: torch.Tensor, k: torch.Tensor, position_offset: int = 0, theta: float = 10000.0,
                           table: Optional[torch.Tensor] = None, *, stream=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """In-place RoPE on token-major q, k of shape [batch, seq, heads, head_dim]."""
    _need(q, "q"); _need(k, "k")
    if q.dim() != 4 or q.shape != k.shape:
        raise ValueError("q and k must both be [batch, seq, heads, head_dim]")
    b, s, h, d = q.shape
    positions = 0
    if table is not None:
        _need(table, "table", (torch.float32,))
        if table.dim() != 2 or table.shape[1] != d:
            raise ValueError("table must be [positions, head_dim]")
        positions = table.shape[0]
    _launch("hrm_rope_embed_token_major", (q, k, table), stream, _ptr(q), _ptr(k), b, s, h, d, position_offset,
            theta, _ptr(table), positions)
    return q, k


def embedding_lookup(ids: torch.Tensor, table: torch.Tensor, embedding_scale: float,
                     out: Optional[torch.Tensor] = None, *, stream=None) -> torch.Tensor:
    """out[..., :] = table[clamp(ids)] * scale (bit-exact).  src/lib.rs:529-565."""
    _ids(ids, "ids"); _need(table, "table")
    if table.dim() != 2:
        raise ValueError("table must be [vocab, hidden]")
    vocab, hidden = table.shape
    out = torch.empty((*ids.shape, hidden), dtype=table.dtype, device=table.device) if out is None else out
    _need(out, "out")
    if out.numel() != ids.numel() * hidden:
        raise ValueError("out has the wrong size")
    _launch("hrm_embedding_lookup", (table, ids, out), stream, _ptr(ids), _ptr(table), _ptr(out), 1, ids.numel(),
            hidden, vocab, embedding_scale)
    return out


def embed_rms_norm(ids: torch.Tensor, table: torch.Tensor, embedding_scale: float,
                   weight: Optional[torch.Tensor] = None, eps: float = 1e-6, hidden_out: Optional[torch.Tensor] = None,
                   normed_out: Optional[torch.Tensor] = None, keep_hidden: bool = True,
                   *, stream=None) -> Tuple[Optional[torch.Tensor], torch.Tensor]:
    """(h, y) = (embedding_lookup(ids), rms_norm(h) [* weight]) in one pass.

    keep_hidden=False skips storing h (returns None for it).
    """
    _ids(ids, "ids"); _need(table, "table")
    vocab, hidden = table.shape
    shape = (*ids.shape, hidden)
    if hidden_out is None and keep_hidden:
        hidden_out = torch.empty(shape, dtype=table.dtype, device=table.device)
    normed_out = torch.empty(shape, dtype=table.dtype, device=table.device) if normed_out is None else normed_out
    if hidden_out is not None:
        _need(hidden_out, "hidden_out")
    _need(normed_out, "normed_out")
    if weight is not None:
        _need(weight, "weight")
        if weight.numel() != hidden:
            raise ValueError("weight must have hidden_size elements")
    _launch("hrm_embed_rms_norm", (table, ids, weight, hidden_out, normed_out), stream, _ptr(ids), _ptr(table),
            _ptr(hidden_out), _ptr(normed_out), _ptr(weight), ids.numel(), hidden, vocab, embedding_scale, eps)
    return hidden_out, normed_out


def split_gqkv_rope(gqkv: torch.Tensor, num_heads: int, position_offset: int = 0, theta: float = 10000.0,
                    table: Optional[torch.Tensor] = None, k_cache: Optional[torch.Tensor] = None,
                    v_cache: Optional[torch.Tensor] = None, cache_offset: int = 0, out=None, *, stream=None):
    """Split + RoPE + KV-cache write in one pass over gqkv [batch, seq, 4 * heads * head_dim].

    Returns (gate [b, s, h, d], q, k, v [b, h, s, d]); with k_cache / v_cache
    ([b, h, cache_len, d]) the rotated k and v are also written at rows
    cache_offset + s.  Replaces split_gqkv -> rope_embed -> kv_cache_update
    (src/lib.rs:798-857).
    """
    _need(gqkv, "gqkv")
    if gqkv.dim() != 3 or gqkv.shape[2] % (4 * num_heads):
        raise ValueError("gqkv must be [batch, seq, 4 * heads * head_dim]")
    b, s, w = gqkv.shape
    d = w // (4 * num_heads)
    if out is None:
        out = (torch.empty((b, s, num_heads, d), dtype=gqkv.dtype, device=gqkv.device),
               *(torch.empty((b, num_heads, s, d), dtype=gqkv.dtype, device=gqkv.device) for _ in range(3)))
    for t, n in zip(out, ("gate", "q", "k", "v")):
        _need(t, n)
    positions, cache_len = 0, 0
    if table is not None:
        _need(table, "table", (torch.float32,))
        positions = table.shape[0]
    if (k_cache is None) != (v_cache is None):
        raise ValueError("pass both k_cache and v_cache or neither")
    if k_cache is not None:
        _need(k_cache, "k_cache"); _need(v_cache, "v_cache")
        if k_cache.dim() != 4 or k_cache.shape != v_cache.shape or k_cache.shape[:2] != (b, num_heads):
            raise ValueError("caches must be [batch, heads, cache_len, head_dim]")
        cache_len = k_cache.shape[2]
    _launch("hrm_split_gqkv_rope", (gqkv, *out, table, k_cache, v_cache), stream, _ptr(gqkv),
            *(_ptr(t) for t in out), _ptr(k_cache), _ptr(v_cache), b, s, num_heads, d, position_offset, theta,
            _ptr(table), positions, cache_len, cache_offset)
    return out


def gated_attn_output(gate: torch.Tensor, attn_out: torch.Tensor, out: Optional[torch.Tensor] = None, *,
                      stream=None) -> torch.Tensor:
    """out = sigmoid(gate) * attn_out (bf16).  src/lib.rs:505-527."""
    _need(gate, "gate"); _need(attn_out, "attn_out")
    if gate.numel() != attn_out.numel():
        raise ValueError("gate and attn_out differ in size")
    out = torch.empty_like(attn_out) if out is None else out
    _need(out, "out")
    _launch("hrm_gated_attn_output", (gate, attn_out, out), stream, _ptr(gate), _ptr(attn_out), _ptr(out),
            gate.numel())
    return out


def apply_attn_gate(gate: torch.Tensor, attn_out: torch.Tensor, *, stream=None) -> torch.Tensor:
    """attn_out *= sigmoid(gate), in place.  src/lib.rs:607-630."""
    _need(gate, "gate"); _need(attn_out, "attn_out")
    if gate.numel() != attn_out.numel():
        raise ValueError("gate and attn_out differ in size")
    _launch("hrm_apply_attn_gate", (gate, attn_out), stream, _ptr(gate), _ptr(attn_out), gate.numel())
    return attn_out


def broadcast_vec(src: torch.Tensor, n_copies: int, out: Optional[torch.Tensor] = None, *,
                  stream=None) -> torch.Tensor:
    """out[r, :] = src for r < n_copies (bf16).  src/lib.rs:748-767."""
    _need(src, "src")
    out = torch.empty((n_copies, src.numel()), dtype=src.dtype, device=src.device) if out is None else out
    _need(out, "out")
    if out.numel() != n_copies * src.numel():
        raise ValueError("out has the wrong size")
    _launch("hrm_broadcast_vec", (src, out), stream, _ptr(out), _ptr(src), n_copies, src.numel())
    return out


def convert_to_bf16(raw: torch.Tensor, dtype: str, out: Optional[torch.Tensor] = None, *,
                    stream=None) -> torch.Tensor:
    """Checkpoint bytes (a CUDA uint8 tensor, any offset) of `dtype` ('f32', 'f16'
    or 'bf16') -> bf16, as the reference's raw_to_bf16 (src/lib.rs:1981-2008)."""
    from ._lib import DTYPES

    _need(raw, "raw", (torch.uint8,))
    size = 4 if dtype == "f32" else 2
    if raw.numel() % size:
        raise ValueError("raw byte count is not a multiple of the element size")
    n = raw.numel() // size
    out = torch.empty(n, dtype=torch.bfloat16, device=raw.device) if out is None else out
    _need(out, "out")
    if out.numel() != n:
        raise ValueError("out has the wrong size")
    _launch("hrm_convert_to_bf16", (raw, out), stream, _ptr(raw), DTYPES[dtype], _ptr(out), n)
    return out


def wait_timeouts(reset: bool = False) -> int:
    """Bounded device waits that ran out (0 in correct operation); reads device
    memory, so synchronize the streams that ran the library's kernels first."""
    n = ctypes.c_uint(0)
    call("hrm_wait_timeouts", ctypes.byref(n), int(reset))
    return int(n.value)
