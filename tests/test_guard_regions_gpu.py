"""Guard regions around every output (GPU): the write-bounds check.

Each output is a view into a larger buffer whose bytes around the view (and,
for the KV caches, the rows outside the written window) hold a sentinel:
bf16 0x7E57 (about 7e37, never produced from these inputs) or the f32 NaN
0x7FC0BEEF.  After the call, every guard element must still hold the sentinel
(nothing was written out of bounds) and no element of the output view may hold
it (every element was written).  Sizes cover the vector paths, their scalar
tails, the scalar fallbacks (odd widths, views shifted off 16-byte alignment)
and single elements.
"""

import math

import numpy as np
import pytest
import torch

import hrm_layer_ops as ops

pytestmark = pytest.mark.gpu

S16, S32 = 0x7E57, 0x7FC0BEEF
PAD = 4096


class Guarded:
    """A contiguous `shape` view `shift` elements past PAD sentinel elements,
    followed by PAD more; `fill` writes the view's initial contents."""

    def __init__(self, shape, dtype, device, shift=0, fill=None):
        n = math.prod(shape)
        self.n, self.lo = n, PAD + shift
        self.buf = torch.empty(self.lo + n + PAD, dtype=dtype, device=device)
        self.bits.fill_(self.sentinel)
        self.view = self.buf[self.lo:self.lo + n].view(shape)
        if fill is not None:
            self.view.copy_(fill)

    @property
    def bits(self):
        return self.buf.view(torch.int16 if self.buf.element_size() == 2 else torch.int32)

    @property
    def sentinel(self):
        return S16 if self.buf.element_size() == 2 else S32

    def check(self, what, written=True):
        b, s = self.bits, self.sentinel
        head, tail = b[:self.lo], b[self.lo + self.n:]
        assert bool((head == s).all()), f"{what}: write before the view"
        assert bool((tail == s).all()), f"{what}: write after the view"
        if written and self.n:
            missed = int((b[self.lo:self.lo + self.n] == s).sum())
            assert missed == 0, f"{what}: {missed} of {self.n} elements not written"


def rnd(shape, dtype=torch.bfloat16, std=1.0, seed=0, device="cuda"):
    g = torch.Generator(device=device).manual_seed(seed)
    return (torch.randn(shape, generator=g, device=device) * std).to(dtype)


def src(shape, device, shift=0, dtype=torch.bfloat16, std=1.0, seed=0):
    """An input with the same alignment shift as the outputs."""
    return Guarded(shape, dtype, device, shift, fill=rnd(shape, dtype, std, seed, device)).view


@pytest.mark.parametrize("n", [1, 7, 8, 9, 4097, 1000003])
@pytest.mark.parametrize("shift", [0, 1])
def test_elementwise(cuda, n, shift):
    a, b = src((n,), cuda, shift, seed=1), src((n,), cuda, shift, seed=2)
    for name, fn in (("additive_inject", lambda o: ops.additive_inject(a, b, out=o)),
                     ("swiglu_ffn", lambda o: ops.swiglu_ffn(a, b, out=o)),
                     ("gated_attn_output", lambda o: ops.gated_attn_output(a, b, out=o))):
        o = Guarded((n,), torch.bfloat16, cuda, shift)
        fn(o.view)
        o.check(name)
    g = Guarded((n,), torch.bfloat16, cuda, shift, fill=b)
    ops.apply_attn_gate(a, g.view)
    g.check("apply_attn_gate", written=False)


@pytest.mark.parametrize("copies,vec", [(1, 8), (5, 2048), (3, 7), (1000, 136), (2, 1)])
@pytest.mark.parametrize("shift", [0, 1])
def test_broadcast(cuda, copies, vec, shift):
    v = src((vec,), cuda, shift, seed=3)
    o = Guarded((copies, vec), torch.bfloat16, cuda, shift)
    ops.broadcast_vec(v, copies, out=o.view)
    o.check("broadcast_vec")


# ... plus launches of several waves of CTAs.
ROW_SHAPES = [(1, 8), (3, 2048), (17, 1536), (5, 200), (2, 6144), (1, 4), (9, 8200), (64, 4096), (1184, 8),
              (1500, 200), (4096, 2048), (2000, 4096), (4736, 2048), (4737, 1600)]


@pytest.mark.parametrize("rows,hidden", ROW_SHAPES)
@pytest.mark.parametrize("shift", [0, 1])
def test_row_ops(cuda, rows, hidden, shift):
    x, b = src((rows, hidden), cuda, shift, seed=4), src((rows, hidden), cuda, shift, seed=5)
    w = src((hidden,), cuda, shift, std=0.1, seed=6)
    y = Guarded((rows, hidden), torch.bfloat16, cuda, shift)
    ops.rms_norm(x, w, 1e-5, out=y.view)
    y.check("rms_norm")
    r, y = Guarded((rows, hidden), torch.bfloat16, cuda, shift), Guarded((rows, hidden), torch.bfloat16, cuda, shift)
    ops.add_rms_norm(x, b, w, 1e-5, residual_out=r.view, normed_out=y.view)
    r.check("add_rms_norm residual")
    y.check("add_rms_norm normed")
    xf = src((rows, hidden), cuda, shift, dtype=torch.float32, seed=7)
    wf = src((hidden,), cuda, shift, dtype=torch.float32, seed=8)
    yf = Guarded((rows, hidden), torch.float32, cuda, shift)
    ops.rms_norm(xf, wf, 1e-5, out=yf.view)
    yf.check("rms_norm f32")


@pytest.mark.parametrize("tokens,hidden", [(1, 8), (7, 2048), (300, 1536), (5, 200), (3, 6144), (64, 1600),
                                           (148, 2048), (1, 4096)])
@pytest.mark.parametrize("shift", [0, 1])
def test_embedding_ops(cuda, tokens, hidden, shift):
    vocab = 100
    table = src((vocab, hidden), cuda, shift, std=0.02, seed=9)
    ids = torch.randint(0, vocab + 5, (tokens,), device=cuda, dtype=torch.int32)  # some out of range
    o = Guarded((tokens, hidden), torch.bfloat16, cuda, shift)
    ops.embedding_lookup(ids, table, 45.25, out=o.view)
    o.check("embedding_lookup")
    h, y = Guarded((tokens, hidden), torch.bfloat16, cuda, shift), Guarded((tokens, hidden), torch.bfloat16, cuda, shift)
    ops.embed_rms_norm(ids, table, 45.25, None, 1e-5, hidden_out=h.view, normed_out=y.view)
    h.check("embed_rms_norm hidden")
    y.check("embed_rms_norm normed")


ROPE_SHAPES = [(1, 1, 1, 16, 0), (2, 3, 5, 64, 7), (1, 16, 33, 128, 0), (8, 16, 1, 128, 4095), (2, 2, 9, 6, 3),
               (1, 4, 300, 64, 9)]


@pytest.mark.parametrize("b,h,s,d,off", ROPE_SHAPES)
@pytest.mark.parametrize("shift", [0, 1])
@pytest.mark.parametrize("layout", ["head", "token"])
def test_rope(cuda, b, h, s, d, off, shift, layout):
    shape = (b, h, s, d) if layout == "head" else (b, s, h, d)
    fn = ops.rope_embed if layout == "head" else ops.rope_embed_token_major
    for table in (None, ops.rope_table(off + s, d)):
        q = Guarded(shape, torch.bfloat16, cuda, shift, fill=rnd(shape, seed=10))
        k = Guarded(shape, torch.bfloat16, cuda, shift, fill=rnd(shape, seed=11))
        fn(q.view, k.view, off, 10000.0, table)
        q.check("rope q", written=False)
        k.check("rope k", written=False)


@pytest.mark.parametrize("positions,d", [(1, 2), (33, 128), (4096, 64), (7, 6)])
def test_rope_table(cuda, positions, d):
    t = Guarded((positions, d), torch.float32, cuda, shift=0)
    ops.rope_table(positions, d, 10000.0, out=t.view)
    t.check("rope_table")


@pytest.mark.parametrize("b,s,h,d,cache_len,cache_off", [(1, 5, 2, 64, 16, 3), (2, 17, 16, 128, 64, 40),
                                                         (3, 1, 4, 128, 8, 7), (1, 4, 2, 6, 10, 2)])
@pytest.mark.parametrize("shift", [0, 1])
def test_split_gqkv_rope_and_cache_window(cuda, b, s, h, d, cache_len, cache_off, shift):
    gqkv = src((b, s, 4 * h * d), cuda, shift, seed=12)
    gate = Guarded((b, s, h, d), torch.bfloat16, cuda, shift)
    qkv = [Guarded((b, h, s, d), torch.bfloat16, cuda, shift) for _ in range(3)]
    kc, vc = (Guarded((b, h, cache_len, d), torch.bfloat16, cuda, shift) for _ in range(2))
    ops.split_gqkv_rope(gqkv, h, cache_off, 10000.0, None, kc.view, vc.view, cache_off,
                        out=(gate.view, *(t.view for t in qkv)))
    gate.check("gate")
    for name, t in zip("qkv", qkv):
        t.check(name)
    for name, c in (("k_cache", kc), ("v_cache", vc)):
        c.check(name, written=False)
        rows = c.view.view(torch.int16)
        inside = rows[:, :, cache_off:cache_off + s]
        outside = torch.cat([rows[:, :, :cache_off], rows[:, :, cache_off + s:]], dim=2)
        assert not bool((inside == S16).any()), f"{name}: window not fully written"
        assert bool((outside == S16).all()), f"{name}: rows outside the window written"


@pytest.mark.parametrize("dtype,size", [("f32", 4), ("f16", 2), ("bf16", 2)])
@pytest.mark.parametrize("n", [1, 7, 1001, 65536 + 3])
@pytest.mark.parametrize("byte_offset", [0, 1, 4])
def test_convert(cuda, dtype, size, n, byte_offset):
    rng = np.random.default_rng(n)
    raw = rng.integers(0, 256, n * size + byte_offset, dtype=np.uint8)
    if dtype != "bf16":  # keep the values finite and small so none converts to the sentinel
        vals = rng.standard_normal(n).astype(np.float32 if dtype == "f32" else np.float16)
        raw[byte_offset:] = np.frombuffer(vals.tobytes(), np.uint8)
    else:
        vals = rng.standard_normal(n).astype(np.float32)
        raw[byte_offset:] = np.frombuffer((vals.view(np.uint32) >> 16).astype(np.uint16).tobytes(), np.uint8)
    draw = torch.from_numpy(raw).to(cuda)[byte_offset:]
    o = Guarded((n,), torch.bfloat16, cuda, shift=byte_offset % 2)
    ops.convert_to_bf16(draw, dtype, out=o.view)
    o.check(f"convert {dtype}")
