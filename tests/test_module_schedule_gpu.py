"""The layer loop's fused residual/norm schedule (hrm_layer_ops.module), GPU.

transformer_module must give the reference's recurrent loop bit for bit:
* against the oracle running the reference's order of operations
  (src/lib.rs:955-1030 per layer, 1036-1105 per module, 1215-1270 per cycle)
  on the CPU, with exact stand-ins for attention and the FFN GEMMs (scalings
  by powers of two and column gathers, exact in bf16 on both sides);
* against this library's unfused operators in the reference's order on the GPU,
  with cuBLAS GEMMs as the attention and FFN stand-ins (the same GEMM calls on
  the same inputs on both sides).
The comparison with the reference's own kernels in the reference's order is in
test_reference_kernels_gpu.py.
"""

import numpy as np
import pytest
import torch

import hrm_layer_ops as ops
from hrm_layer_ops.module import ModuleFns, ModuleNorms, ModuleScratch, recurrent_forward, transformer_module
from helpers import assert_bits_equal, normal_bf16, to_dev, to_host

pytestmark = pytest.mark.gpu

EPS = 1e-5


# ----------------------------------------------------------- exact stand-ins
def _cols(hidden, inter):
    j = np.arange(inter)
    return j % hidden, (j * 7 + 3) % hidden


class ExactStandIns:
    """attention: a = n / 2; gate_up: g = n[:, j % H], u = -n[:, (7j+3) % H] / 4;
    down: d = 2 * act[:, :H].  Scalings by powers of two and gathers: the GPU
    and the oracle compute the same values."""

    def __init__(self, hidden, inter, device):
        ig, iu = _cols(hidden, inter)
        self.ig, self.iu = torch.from_numpy(ig).to(device), torch.from_numpy(iu).to(device)
        self.hidden = hidden

    def attention(self, i, n, out):
        torch.mul(n, 0.5, out=out)

    def gate_up(self, i, n, g, u):
        torch.index_select(n, 1, self.ig, out=g)
        torch.index_select(n, 1, self.iu, out=u)
        u.mul_(-0.25)

    def down(self, i, act, out):
        torch.mul(act[:, :self.hidden], 2.0, out=out)


def _host_standins(hidden, inter):
    """The same stand-ins on the CPU, in fp32 with RNE to bf16 as torch does."""
    from oracle import bf16_to_f32, f32_to_bf16

    ig, iu = _cols(hidden, inter)

    def attention(n):
        return f32_to_bf16(bf16_to_f32(n) * np.float32(0.5))

    def gate_up(n):
        f = bf16_to_f32(n)
        return n[:, ig].copy(), f32_to_bf16(f[:, iu] * np.float32(-0.25))

    def down(act):
        return f32_to_bf16(bf16_to_f32(act)[:, :hidden] * np.float32(2.0))

    return attention, gate_up, down


def _oracle_module(o, z_a, z_b, n_layers, sa, eps):
    """The reference's order on the CPU: injection + copy, per layer norm ->
    attention -> add -> norm -> FFN -> add -> copy, output copy before each
    later layer, final norm + copy."""
    attention, gate_up, down = sa
    inp = o.additive_inject(z_a, z_b)
    out = None
    for i in range(n_layers):
        x = inp if i == 0 else out.copy()
        n = o.rms_norm(x, None, eps)
        out = o.additive_inject(x, attention(n))
        n2 = o.rms_norm(out, None, eps)
        g, u = gate_up(n2)
        out = o.additive_inject(out, down(o.swiglu_ffn(g, u)))
    return o.rms_norm(out, None, eps)


def test_recurrent_loop_matches_oracle_in_reference_order(oracle, cuda):
    """2 H-cycles x 2 L-cycles over 3-layer modules, 64 rows, H 256, I 704."""
    rows, H, I, L = 64, 256, 704, 3
    rng = np.random.default_rng(21)
    z_h, z_l = normal_bf16(rng, (rows, H)), normal_bf16(rng, (rows, H))
    sa = ExactStandIns(H, I, cuda)
    scratch = ModuleScratch(rows, H, I, cuda)
    dh, dl = to_dev(z_h, cuda), to_dev(z_l, cuda)
    for _ in range(2):
        for _ in range(2):
            transformer_module(dl, dh, dl, L, sa.attention, sa.gate_up, sa.down, scratch, eps=EPS)
        transformer_module(dh, dl, dh, L, sa.attention, sa.gate_up, sa.down, scratch, eps=EPS)
    hs = _host_standins(H, I)
    for _ in range(2):
        for _ in range(2):
            z_l = _oracle_module(oracle, z_l, z_h, L, hs, EPS)
        z_h = _oracle_module(oracle, z_h, z_l, L, hs, EPS)
    assert_bits_equal(to_host(dl), z_l, "z_L")
    assert_bits_equal(to_host(dh), z_h, "z_H")


def test_recurrent_forward_matches_oracle_in_reference_order(oracle, cuda):
    """The whole loop of src/lib.rs:1189-1270 -- embedding into z_H, z_L
    broadcast from z_l_init, 2 H-cycles x 3 L-cycles of 2-layer modules -- equals
    the oracle running the reference's order, and the attention callbacks see
    the reference's KV-slot numbering (each module pass takes the next
    n_layers slots)."""
    rows, H, I, L, V = 48, 256, 704, 2, 100
    scale = 16.0
    rng = np.random.default_rng(23)
    ids = rng.integers(0, V + 3, rows, dtype=np.uint32)          # a few out of range: clamped
    table = normal_bf16(rng, (V, H), 0.5)
    z_l_init = normal_bf16(rng, H)
    sa = ExactStandIns(H, I, cuda)
    seen = []

    def attention(i, slot, n, out):
        seen.append(slot)
        sa.attention(i, n, out)

    m = ModuleFns(L, attention, sa.gate_up, sa.down)
    z_h, z_l = recurrent_forward(to_dev(ids, cuda), to_dev(table, cuda), scale, to_dev(z_l_init, cuda), 2, 3, m, m,
                                 ModuleScratch(rows, H, I, cuda), eps=EPS)
    hs = _host_standins(H, I)
    wh = oracle.embedding_lookup(ids, table, scale)
    wl = oracle.broadcast_vec(z_l_init, rows)
    for _ in range(2):
        for _ in range(3):
            wl = _oracle_module(oracle, wl, wh, L, hs, EPS)
        wh = _oracle_module(oracle, wh, wl, L, hs, EPS)
    assert_bits_equal(to_host(z_h), wh.reshape(rows, H), "z_H")
    assert_bits_equal(to_host(z_l), wl.reshape(rows, H), "z_L")
    assert seen == list(range(2 * (3 + 1) * L))


# --------------------------------------------------- GEMM stand-ins (cuBLAS)
class GemmStandIns:
    def __init__(self, n_layers, hidden, inter, device, seed):
        g = torch.Generator(device=device).manual_seed(seed)

        def w(k, n):
            return (torch.randn((k, n), generator=g, device=device) / k ** 0.5).to(torch.bfloat16)

        self.wa = [w(hidden, hidden) for _ in range(n_layers)]
        self.wg = [w(hidden, inter) for _ in range(n_layers)]
        self.wu = [w(hidden, inter) for _ in range(n_layers)]
        self.wd = [w(inter, hidden) for _ in range(n_layers)]

    def attention(self, i, n, out):
        torch.matmul(n, self.wa[i], out=out)

    def gate_up(self, i, n, g, u):
        torch.matmul(n, self.wg[i], out=g)
        torch.matmul(n, self.wu[i], out=u)

    def down(self, i, act, out):
        torch.matmul(act, self.wd[i], out=out)


def reference_order_module(k, z_a, z_b, out, n_layers, sa, bufs, eps):
    """The reference's transformer_module fed by its cycle injection, op for op,
    on the operator set `k` (additive_inject(a, b, out), rms_norm(x, y, eps),
    swiglu(g, u, out)); `bufs` holds its scratch buffers."""
    tmp1, tmp2, norm_buf, attn_out, norm2, g, u, act, down, res = bufs
    k.additive_inject(z_a, z_b, tmp1)               # lib.rs:1220-1229 / 1248-1256
    tmp2.copy_(tmp1)
    for i in range(n_layers):
        if i == 0:
            x = tmp2
        else:
            tmp1.copy_(out)                         # lib.rs:1068-1075
            x = tmp1
        k.rms_norm(x, norm_buf, eps)                # lib.rs:969
        sa.attention(i, norm_buf, attn_out)
        k.additive_inject(x, attn_out, out)         # lib.rs:976
        k.rms_norm(out, norm2, eps)                 # lib.rs:979
        sa.gate_up(i, norm2, g, u)
        k.swiglu(g, u, act)
        sa.down(i, act, down)
        k.additive_inject(out, down, res)           # lib.rs:1015-1028
        out.copy_(res)
    k.rms_norm(out, tmp1, eps)                      # lib.rs:1091-1104
    out.copy_(tmp1)


class OwnUnfused:
    @staticmethod
    def additive_inject(a, b, out):
        ops.additive_inject(a, b, out=out)

    @staticmethod
    def rms_norm(x, y, eps):
        ops.rms_norm(x, None, eps, out=y)

    @staticmethod
    def swiglu(g, u, out):
        ops.swiglu_ffn(g, u, out=out)


def make_bufs(rows, hidden, inter, device):
    e = lambda c: torch.empty((rows, c), dtype=torch.bfloat16, device=device)  # noqa: E731
    return (e(hidden), e(hidden), e(hidden), e(hidden), e(hidden), e(inter), e(inter), e(inter), e(hidden),
            e(hidden))


def run_both(k, rows, H, I, L, cuda, seed):
    """The recurrent loop (2 H-cycles x 2 L-cycles) in the reference's order on
    operator set k, and through transformer_module; returns both (z_H, z_L)."""
    g = torch.Generator(device=cuda).manual_seed(seed)
    z_h0 = torch.randn((rows, H), generator=g, device=cuda).to(torch.bfloat16)
    z_l0 = torch.randn((rows, H), generator=g, device=cuda).to(torch.bfloat16)
    mods = {"L": GemmStandIns(L, H, I, cuda, seed + 1), "H": GemmStandIns(L, H, I, cuda, seed + 2)}
    bufs = make_bufs(rows, H, I, cuda)
    rh, rl = z_h0.clone(), z_l0.clone()
    for _ in range(2):
        for _ in range(2):
            reference_order_module(k, rl, rh, rl, L, mods["L"], bufs, EPS)
        reference_order_module(k, rh, rl, rh, L, mods["H"], bufs, EPS)
    scratch = ModuleScratch(rows, H, I, cuda)
    fh, fl = z_h0.clone(), z_l0.clone()
    for _ in range(2):
        for _ in range(2):
            m = mods["L"]
            transformer_module(fl, fh, fl, L, m.attention, m.gate_up, m.down, scratch, eps=EPS)
        m = mods["H"]
        transformer_module(fh, fl, fh, L, m.attention, m.gate_up, m.down, scratch, eps=EPS)
    return (rh, rl), (fh, fl)


def test_recurrent_loop_matches_unfused_reference_order(cuda):
    """1024 rows, H 2048, I 5632, 2-layer modules, cuBLAS stand-ins."""
    (rh, rl), (fh, fl) = run_both(OwnUnfused, 1024, 2048, 5632, 2, cuda, seed=31)
    assert torch.equal(fl.view(torch.int16), rl.view(torch.int16))
    assert torch.equal(fh.view(torch.int16), rh.view(torch.int16))
    assert torch.isfinite(fh.float()).all()


def test_module_with_norm_weights_equals_unfused(cuda):
    """Weighted norms (an extension: the reference's have none): each fused call
    uses the weight of the norm it replaces."""
    rows, H, I, L = 256, 512, 1408, 3
    g = torch.Generator(device=cuda).manual_seed(41)

    def w():
        return (1 + 0.1 * torch.randn(H, generator=g, device=cuda)).to(torch.bfloat16)

    norms = ModuleNorms(attn=[w() for _ in range(L)], ffn=[w() for _ in range(L)], final=w())
    sa = GemmStandIns(L, H, I, cuda, 42)
    z_a = torch.randn((rows, H), generator=g, device=cuda).to(torch.bfloat16)
    z_b = torch.randn((rows, H), generator=g, device=cuda).to(torch.bfloat16)
    out = torch.empty_like(z_a)
    transformer_module(z_a, z_b, out, L, sa.attention, sa.gate_up, sa.down, ModuleScratch(rows, H, I, cuda),
                       eps=EPS, norms=norms)
    x = ops.additive_inject(z_a, z_b)
    for i in range(L):
        a = torch.empty_like(x)
        sa.attention(i, ops.rms_norm(x, norms.attn[i], EPS), a)
        x = ops.additive_inject(x, a)
        gg, uu = torch.empty((rows, I), dtype=torch.bfloat16, device=cuda), torch.empty(
            (rows, I), dtype=torch.bfloat16, device=cuda)
        sa.gate_up(i, ops.rms_norm(x, norms.ffn[i], EPS), gg, uu)
        d = torch.empty_like(x)
        sa.down(i, ops.swiglu_ffn(gg, uu), d)
        x = ops.additive_inject(x, d)
    assert torch.equal(out.view(torch.int16), ops.rms_norm(x, norms.final, EPS).view(torch.int16))


def test_module_argument_checks(cuda):
    s = ModuleScratch(8, 64, 128, cuda)
    z = torch.zeros((8, 64), dtype=torch.bfloat16, device=cuda)
    noop = lambda *a: None  # noqa: E731
    with pytest.raises(ValueError):
        transformer_module(z, z.clone(), z, 0, noop, noop, noop, s)
    with pytest.raises(ValueError):
        transformer_module(z, z.clone(), torch.zeros((8, 32), dtype=torch.bfloat16, device=cuda), 1, noop, noop,
                           noop, s)
    b = z.clone()
    with pytest.raises(ValueError):
        transformer_module(z, b, b, 1, noop, noop, noop, s)
