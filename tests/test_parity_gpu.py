"""GPU parity: every operator through the C ABI against the oracle.

Bars (written per test): bit-exact for the residual add, the embedding gather
and RMSNorm in all its forms (the kernels reproduce the reference's
reduction order); <= 2 bf16 ulp for SwiGLU (C-library expf in the oracle vs
the __expf intrinsic) and RoPE (C-library vs CUDA expf/logf/sincosf; ulp
measured at the rotated pair's magnitude).  Shapes cover the edge cases the
reference's launch code meets or mishandles: single rows, tails that are not
a multiple of the 8-element vector, hidden sizes that are not a multiple of
8, misaligned pointers (scalar paths), out-of-range ids, in-place calls,
special values, empty inputs and the fallback paths for large rows.
"""

import numpy as np
import pytest
import torch

import hrm_layer_ops as ops
from helpers import ULP_TOL, assert_bits_equal, normal_bf16, rope_pair_magnitude, to_dev, to_host
from oracle import f32_to_bf16, ulp_error

pytestmark = pytest.mark.gpu


def misaligned(t):
    """A view of t shifted by one element (2 bytes): not 16-byte aligned."""
    buf = torch.empty(t.numel() + 1, dtype=t.dtype, device=t.device)
    v = buf[1:].view(t.shape)
    v.copy_(t)
    return v


# ------------------------------------------------------------ additive add
@pytest.mark.parametrize("n", [1, 7, 8, 9, 4096, 65536 + 5, (1 << 20) + 3])
def test_additive_inject(oracle, rng, cuda, n):
    a, b = normal_bf16(rng, n, 3.0), normal_bf16(rng, n)
    out = ops.additive_inject(to_dev(a, cuda), to_dev(b, cuda))
    assert_bits_equal(to_host(out), oracle.additive_inject(a, b), "additive_inject")


def test_additive_inject_in_place_and_misaligned(oracle, rng, cuda):
    n = 10001
    a, b = normal_bf16(rng, n), normal_bf16(rng, n)
    want = oracle.additive_inject(a, b)
    da = to_dev(a, cuda)
    ops.additive_inject(da, to_dev(b, cuda), out=da)  # z_out aliases z_a exactly
    assert_bits_equal(to_host(da), want, "in place")
    ma, mb = misaligned(to_dev(a, cuda)), misaligned(to_dev(b, cuda))
    assert_bits_equal(to_host(ops.additive_inject(ma, mb, out=misaligned(torch.empty_like(ma)))), want, "misaligned")


# ------------------------------------------------------------------ swiglu
@pytest.mark.parametrize("n", [1, 4, 7, 8, 9, 1000003, 32 * 5632])
def test_swiglu(oracle, rng, cuda, n):
    g, u = normal_bf16(rng, n, 0.5), normal_bf16(rng, n, 0.5)
    out = to_host(ops.swiglu_ffn(to_dev(g, cuda), to_dev(u, cuda)))
    err = ulp_error(out, oracle.swiglu_ffn(g, u))
    assert err.max() <= ULP_TOL, f"max {err.max()} ulp"


def test_swiglu_special_values_in_place_misaligned(oracle, rng, cuda):
    g = np.array([0x0000, 0x8000, 0x7F80, 0xFF80, 0x7FC0, 0x4300, 0xC300, 0x0001, 0x42F0, 0xC2F0, 0x3F80],
                 np.uint16)  # 0, -0, inf, -inf, nan, 128, -128, denormal, 120, -120, 1
    u = f32_to_bf16(np.array([2.0, 2.0, 1.0, 1.0, 1.0, 1.0, 1.0, 1e30, 3.0, 3.0, -1.0], np.float32))
    want = oracle.swiglu_ffn(g, u)
    for dg, du in ((to_dev(g, cuda), to_dev(u, cuda)), (misaligned(to_dev(g, cuda)), misaligned(to_dev(u, cuda)))):
        err = ulp_error(to_host(ops.swiglu_ffn(dg, du)), want)
        assert err.max() <= ULP_TOL, f"max {err.max()} ulp"
    g2, u2 = normal_bf16(rng, 4099), normal_bf16(rng, 4099)
    dg = to_dev(g2, cuda)
    ops.swiglu_ffn(dg, to_dev(u2, cuda), out=dg)
    assert ulp_error(to_host(dg), oracle.swiglu_ffn(g2, u2)).max() <= ULP_TOL


# ----------------------------------------------------------------- rmsnorm
NORM_SHAPES = [(1, 4), (1, 8), (3, 24), (7, 1000), (2, 200), (64, 1536), (129, 2048), (5, 4096), (3, 6144),
               (2, 4100)]


@pytest.mark.parametrize("rows,hidden", NORM_SHAPES)
@pytest.mark.parametrize("with_weight", [False, True])
def test_rms_norm_bitexact(oracle, rng, cuda, rows, hidden, with_weight):
    x = normal_bf16(rng, (rows, hidden), 2.0)
    w = normal_bf16(rng, hidden, 0.1, 1.0) if with_weight else None
    y = ops.rms_norm(to_dev(x, cuda), None if w is None else to_dev(w, cuda), eps=1e-5)
    assert_bits_equal(to_host(y), oracle.rms_norm(x, w, eps=1e-5), f"rms_norm {rows}x{hidden}")


def test_rms_norm_reference_kat(cuda):
    """src/lib.rs:2247-2261: rows 1, hidden 4, x = [1, 2, 3, 4]."""
    x = torch.tensor([[1.0, 2.0, 3.0, 4.0]], dtype=torch.bfloat16, device=cuda)
    y = ops.rms_norm(x, eps=1e-6).float().cpu().numpy()
    rms = np.sqrt(30.0) / 2
    assert np.all(np.abs(y - np.array([1, 2, 3, 4]) / rms) < 0.01)


def test_rms_norm_misaligned_and_special_rows(oracle, rng, cuda):
    x = normal_bf16(rng, (6, 2048))
    x[1] = 0                         # all-zero row: y = 0
    x[2, :5] = [0x7F80, 0, 0, 0, 0]  # +inf in a row: ss = inf -> inv = 0, inf * 0 = nan
    x[3] = f32_to_bf16(np.full(2048, 1e30, np.float32))  # ss overflows fp32
    want = oracle.rms_norm(x, None, eps=1e-6)
    assert_bits_equal(to_host(ops.rms_norm(to_dev(x, cuda), eps=1e-6)), want, "special rows")
    dx = misaligned(to_dev(x, cuda))
    assert_bits_equal(to_host(ops.rms_norm(dx, eps=1e-6, out=misaligned(torch.empty_like(dx)))), want, "misaligned")


def test_rms_norm_empty(cuda):
    x = torch.empty((0, 2048), dtype=torch.bfloat16, device=cuda)
    assert ops.rms_norm(x).shape == (0, 2048)


@pytest.mark.parametrize("rows,hidden", [(1, 4), (33, 2048), (17, 1000), (4, 3000)])
def test_rms_norm_f32_bitexact(oracle, rng, cuda, rows, hidden):
    x = rng.standard_normal((rows, hidden)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(hidden)).astype(np.float32)
    y = ops.rms_norm(torch.from_numpy(x).to(cuda), torch.from_numpy(w).to(cuda), eps=1e-5).cpu().numpy()
    assert np.array_equal(y.view(np.uint32), oracle.rms_norm_f32(x, w, eps=1e-5).view(np.uint32))


# ------------------------------------------------------------ add + rmsnorm
@pytest.mark.parametrize("rows,hidden", [(1, 8), (3, 24), (65, 2048), (9, 1536), (4, 4096), (3, 5000), (2, 12)])
@pytest.mark.parametrize("with_weight", [False, True])
def test_add_rms_norm_bitexact(oracle, rng, cuda, rows, hidden, with_weight):
    x, b = normal_bf16(rng, (rows, hidden)), normal_bf16(rng, (rows, hidden))
    w = normal_bf16(rng, hidden, 0.1, 1.0) if with_weight else None
    r, y = ops.add_rms_norm(to_dev(x, cuda), to_dev(b, cuda), None if w is None else to_dev(w, cuda), eps=1e-5)
    wr, wy = oracle.add_rms_norm(x, b, w, eps=1e-5)
    assert_bits_equal(to_host(r), wr, "residual")
    assert_bits_equal(to_host(y), wy, "normed")


@pytest.mark.parametrize("hidden", [1536, 1544, 2048, 4096])
@pytest.mark.parametrize("weighted", [False, True])
def test_row_ops_decode_size_paths(oracle, rng, cuda, hidden, weighted):
    """Launches of at most one row per SM over rows of more than 192 chunks
    give each row a CTA of one warp per 32 chunks (warp 0 replays the
    summation from shared memory); narrower rows, and one row more than the
    SM count, keep the warp kernel.  Every op, both sides of both boundaries,
    bit-exact against the oracle."""
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    w = normal_bf16(rng, hidden, 0.1, 1.0) if weighted else None
    dw = None if w is None else to_dev(w, cuda)
    table = normal_bf16(rng, (700, hidden), 0.02)
    for rows in (1, 64, sms, sms + 1):
        x, b = normal_bf16(rng, (rows, hidden), 1.5), normal_bf16(rng, (rows, hidden))
        y = ops.rms_norm(to_dev(x, cuda), dw, eps=1e-5)
        assert_bits_equal(to_host(y), oracle.rms_norm(x, w, eps=1e-5), f"rms_norm {rows} x {hidden}")
        dx = to_dev(x, cuda)
        r, y = ops.add_rms_norm(dx, to_dev(b, cuda), dw, eps=1e-5, residual_out=dx)  # in place, as the layer loop
        wr, wy = oracle.add_rms_norm(x, b, w, eps=1e-5)
        assert_bits_equal(to_host(r), wr, f"add_rms_norm residual {rows} x {hidden}")
        assert_bits_equal(to_host(y), wy, f"add_rms_norm normed {rows} x {hidden}")
        ids = rng.integers(0, 705, rows, dtype=np.uint32)  # a few out of range: clamped
        h, y = ops.embed_rms_norm(to_dev(ids, cuda), to_dev(table, cuda), 45.254834, dw, eps=1e-5, keep_hidden=True)
        wh, wy = oracle.embed_rms_norm(ids, table, 45.254834, w, eps=1e-5)
        assert_bits_equal(to_host(h), wh, f"embed_rms_norm hidden {rows} x {hidden}")
        assert_bits_equal(to_host(y), wy, f"embed_rms_norm normed {rows} x {hidden}")


def test_add_rms_norm_residual_in_place(oracle, rng, cuda):
    x, b = normal_bf16(rng, (40, 2048)), normal_bf16(rng, (40, 2048))
    wr, wy = oracle.add_rms_norm(x, b, None, eps=1e-6)
    for alias in ("x", "branch"):
        dx, db = to_dev(x, cuda), to_dev(b, cuda)
        r, y = ops.add_rms_norm(dx, db, eps=1e-6, residual_out=dx if alias == "x" else db)
        assert_bits_equal(to_host(r), wr, f"residual aliasing {alias}")
        assert_bits_equal(to_host(y), wy, f"normed aliasing {alias}")


# --------------------------------------------------------------- embedding
@pytest.mark.parametrize("vocab,hidden,tokens", [(10, 8, 5), (100, 24, 33), (32000, 2048, 300), (77, 2052, 9),
                                                 (50, 5000, 4), (12, 6, 7)])
@pytest.mark.parametrize("scale", [1.0, 45.254834, 39.191835884530846])
def test_embedding_bitexact(oracle, rng, cuda, vocab, hidden, tokens, scale):
    table = normal_bf16(rng, (vocab, hidden), 0.02)
    ids = rng.integers(0, vocab, tokens, dtype=np.uint32)
    ids[0] = vocab - 1
    if tokens > 3:
        ids[1], ids[2] = vocab, 0xFFFFFFFF  # clamped to vocab - 1
    out = ops.embedding_lookup(to_dev(ids, cuda), to_dev(table, cuda), scale)
    assert_bits_equal(to_host(out), oracle.embedding_lookup(ids, table, scale), "embedding")


@pytest.mark.parametrize("hidden", [2048, 1536, 1600, 4096, 256])
@pytest.mark.parametrize("tokens", [1, 3, 8, 64, 148, 300])
def test_embedding_decode_row_split_bitexact(oracle, rng, cuda, hidden, tokens):
    """A gather of few tokens splits each row over up to 8 warps (32-chunk
    blocks p, p + split, ...); every split, including rows whose last block
    is partial (hidden 1600: 200 chunks), writes each element exactly once."""
    table = normal_bf16(rng, (3000, hidden), 0.02)
    ids = rng.integers(0, 3000, tokens, dtype=np.uint32)
    out = ops.embedding_lookup(to_dev(ids, cuda), to_dev(table, cuda), 45.254834)
    assert_bits_equal(to_host(out), oracle.embedding_lookup(ids, table, 45.254834), f"{tokens} x {hidden}")


def test_embedding_misaligned_table(oracle, rng, cuda):
    table = normal_bf16(rng, (40, 64), 0.02)
    ids = rng.integers(0, 40, 21, dtype=np.uint32)
    dt = misaligned(to_dev(table, cuda))
    out = ops.embedding_lookup(to_dev(ids, cuda), dt, 3.0)
    assert_bits_equal(to_host(out), oracle.embedding_lookup(ids, table, 3.0), "misaligned table")


@pytest.mark.parametrize("hidden", [8, 1536, 2048, 4104])
@pytest.mark.parametrize("keep_hidden", [True, False])
def test_embed_rms_norm_bitexact(oracle, rng, cuda, hidden, keep_hidden):
    table = normal_bf16(rng, (500, hidden), 0.02)
    w = normal_bf16(rng, hidden, 0.1, 1.0)
    ids = rng.integers(0, 520, 97, dtype=np.uint32)
    h, y = ops.embed_rms_norm(to_dev(ids, cuda), to_dev(table, cuda), 45.254834, to_dev(w, cuda), eps=1e-5,
                              keep_hidden=keep_hidden)
    wh, wy = oracle.embed_rms_norm(ids, table, 45.254834, w, eps=1e-5)
    assert_bits_equal(to_host(y), wy, "normed")
    if keep_hidden:
        assert_bits_equal(to_host(h), wh, "hidden")


# -------------------------------------------------------------------- rope
ROPE_CASES = [(2, 4, 300, 128, 0), (8, 16, 1, 128, 4095), (1, 12, 33, 128, 7), (3, 2, 77, 64, 3),
              (2, 3, 5, 32, 0), (1, 2, 9, 96, 11), (1, 1, 3, 130, 1), (2, 5, 17, 256, 100), (1, 3, 2, 2, 0)]


def check_rope(oracle, q, k, dq, dk, offset, theta):
    wq, wk = oracle.rope_embed(q, k, offset, theta)
    for got, want, name in ((to_host(dq), wq, "q"), (to_host(dk), wk, "k")):
        err = ulp_error(got, want, rope_pair_magnitude(want))
        assert err.max() <= ULP_TOL, f"{name}: max {err.max()} ulp"


@pytest.mark.parametrize("b,h,s,d,off", ROPE_CASES)
@pytest.mark.parametrize("use_table", [False, True])
def test_rope(oracle, rng, cuda, b, h, s, d, off, use_table):
    theta = 10000.0
    q, k = normal_bf16(rng, (b, h, s, d)), normal_bf16(rng, (b, h, s, d))
    dq, dk = to_dev(q, cuda), to_dev(k, cuda)
    table = ops.rope_table(off + s, d, theta) if use_table else None
    ops.rope_embed(dq, dk, off, theta, table)
    check_rope(oracle, q, k, dq, dk, off, theta)


def test_rope_table_and_in_kernel_angles_agree_bitwise(rng, cuda):
    q = to_dev(normal_bf16(rng, (2, 16, 512, 128)), cuda)
    k = to_dev(normal_bf16(rng, (2, 16, 512, 128)), cuda)
    q1, k1, q2, k2 = q.clone(), k.clone(), q.clone(), k.clone()
    ops.rope_embed(q1, k1, 1000, 10000.0, None)
    ops.rope_embed(q2, k2, 1000, 10000.0, ops.rope_table(1512, 128, 10000.0))
    assert torch.equal(q1.view(torch.int16), q2.view(torch.int16))
    assert torch.equal(k1.view(torch.int16), k2.view(torch.int16))


def test_rope_misaligned(oracle, rng, cuda):
    q, k = normal_bf16(rng, (1, 4, 20, 128)), normal_bf16(rng, (1, 4, 20, 128))
    dq, dk = misaligned(to_dev(q, cuda)), misaligned(to_dev(k, cuda))
    ops.rope_embed(dq, dk, 5, 10000.0, None)
    check_rope(oracle, q, k, dq, dk, 5, 10000.0)


def test_rope_table_close_to_oracle(oracle, cuda):
    """CUDA's and the C library's expf / sincosf may differ by an fp32 ulp or two;
    at angle ~4095 rad that is ~5e-4 of the angle."""
    t = ops.rope_table(4096, 128, 10000.0).cpu().numpy()
    want = oracle.rope_table(4096, 128, 10000.0)
    assert np.max(np.abs(t - want)) < 2e-3
    assert np.array_equal(t[0], want[0])  # position 0: cos 1, sin 0


def test_rope_table_range_error(cuda):
    q = torch.zeros((1, 1, 4, 128), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ops.HrmError):
        ops.rope_embed(q, q.clone(), 10, 10000.0, ops.rope_table(12, 128))


# -------------------------------------------------- split + RoPE + KV cache
SPLIT_CASES = [(2, 300, 4, 128, 0, True), (8, 1, 16, 128, 4095, True), (1, 33, 12, 128, 0, False),
               (1, 7, 3, 64, 5, True), (1, 5, 2, 96, 0, True), (1, 3, 2, 130, 2, False)]


@pytest.mark.parametrize("b,s,h,d,off,with_cache", SPLIT_CASES)
@pytest.mark.parametrize("use_table", [False, True])
def test_split_gqkv_rope(oracle, rng, cuda, b, s, h, d, off, with_cache, use_table):
    """Fused split + RoPE + cache write vs the oracle's split -> rope -> kv_cache_update:
    copies (gate, v, cache rows) bit-exact, rotated q/k <= 2 bf16 ulp at pair magnitude,
    cache rows outside [off, off + s) untouched."""
    gqkv = normal_bf16(rng, (b, s, 4 * h * d))
    cache_len = off + s + 3
    kc0, vc0 = normal_bf16(rng, (b, h, cache_len, d)), normal_bf16(rng, (b, h, cache_len, d))
    dkc, dvc = (to_dev(kc0, cuda), to_dev(vc0, cuda)) if with_cache else (None, None)
    table = ops.rope_table(off + s, d) if use_table else None
    gate, q, k, v = ops.split_gqkv_rope(to_dev(gqkv, cuda), h, off, 10000.0, table, dkc, dvc, cache_offset=off)
    wg, wq, wk, wv, wkc, wvc = oracle.split_gqkv_rope(gqkv, b, s, h, d, off, 10000.0, None, kc0, vc0, off)
    assert_bits_equal(to_host(gate), wg, "gate")
    assert_bits_equal(to_host(v), wv, "v")
    for got, want in ((to_host(q), wq), (to_host(k), wk)):
        assert ulp_error(got, want, rope_pair_magnitude(want)).max() <= ULP_TOL
    if with_cache:
        hk, hv = to_host(dkc), to_host(dvc)
        assert_bits_equal(hk[:, :, off:off + s], to_host(k), "k cache rows")
        assert_bits_equal(hv[:, :, off:off + s], to_host(v), "v cache rows")
        keep = np.ones(cache_len, bool)
        keep[off:off + s] = False
        assert_bits_equal(hk[:, :, keep], kc0[:, :, keep], "k cache untouched")
        assert_bits_equal(hv[:, :, keep], vc0[:, :, keep], "v cache untouched")


def test_split_gqkv_rope_errors(cuda):
    g = torch.zeros((1, 4, 4 * 2 * 128), dtype=torch.bfloat16, device=cuda)
    kc = torch.zeros((1, 2, 5, 128), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ops.HrmError):  # cache too short for offset 3 + seq 4
        ops.split_gqkv_rope(g, 2, 3, 10000.0, None, kc, kc.clone(), cache_offset=3)
    with pytest.raises(ValueError):
        ops.split_gqkv_rope(g, 2, 0, 10000.0, None, kc, None)


# ----------------------------------------- attention gate, broadcast, convert
@pytest.mark.parametrize("n", [1, 4, 9, 4099, 65536 * 3 + 5])
def test_gated_attn_output_and_in_place(oracle, rng, cuda, n):
    g, a = normal_bf16(rng, n, 2.0), normal_bf16(rng, n)
    want = oracle.gated_attn_output(g, a)
    out = to_host(ops.gated_attn_output(to_dev(g, cuda), to_dev(a, cuda)))
    assert ulp_error(out, want).max() <= ULP_TOL
    da = to_dev(a, cuda)
    ops.apply_attn_gate(to_dev(g, cuda), da)
    assert_bits_equal(to_host(da), out, "in place == out of place")


def test_gated_attn_output_reference_kat(cuda):
    """src/lib.rs:2283-2298: sigmoid(0) * 1 = 0.5."""
    y = ops.gated_attn_output(torch.zeros(4, dtype=torch.bfloat16, device=cuda),
                              torch.ones(4, dtype=torch.bfloat16, device=cuda)).float().cpu().numpy()
    assert np.all(np.abs(y - 0.5) < 0.01)


@pytest.mark.parametrize("n_copies,vec_len", [(1, 8), (7, 2048), (64, 1536), (5, 13), (3000, 2048)])
def test_broadcast_vec(oracle, rng, cuda, n_copies, vec_len):
    src = normal_bf16(rng, vec_len)
    assert_bits_equal(to_host(ops.broadcast_vec(to_dev(src, cuda), n_copies)), oracle.broadcast_vec(src, n_copies),
                      "broadcast")


def _raw(b: bytes, cuda, offset=0):
    buf = torch.zeros(len(b) + offset, dtype=torch.uint8, device=cuda)
    buf[offset:] = torch.frombuffer(bytearray(b), dtype=torch.uint8).to(cuda)
    return buf[offset:]


def test_convert_f16_exhaustive(oracle, cuda):
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    want = oracle.convert_to_bf16(h.tobytes(), "f16")
    for off in (0, 1, 2, 6):  # vector path (0) and byte-assembled paths
        got = to_host(ops.convert_to_bf16(_raw(h.tobytes(), cuda, off), "f16"))
        assert_bits_equal(got, want, f"f16 offset {off}")


def test_convert_f32(oracle, rng, cuda):
    x = np.concatenate([rng.standard_normal(1 << 20).astype(np.float32) * np.float32(1e3),
                        np.array([0x7FC00000, 0xFFC00001, 0x7F800001, 0xFFA5A5A5, 0x7FFFFFFF, 0x00000001, 0x3F808000,
                                  0x3F818000, 0x7F7FFFFF, 0x80000000, 0x7F800000], np.uint32).view(np.float32)])
    want = oracle.convert_to_bf16(x.tobytes(), "f32")
    for off in (0, 3):
        got = to_host(ops.convert_to_bf16(_raw(x.tobytes(), cuda, off), "f32"))
        assert_bits_equal(got, want, f"f32 offset {off}")
    b = normal_bf16(rng, 1001)
    assert_bits_equal(to_host(ops.convert_to_bf16(_raw(b.tobytes(), cuda), "bf16")), b, "bf16 copy")


@pytest.mark.parametrize("b,s,h,d,off", [(2, 300, 4, 128, 0), (64, 1, 16, 128, 4095), (1, 9, 3, 64, 5),
                                         (1, 5, 2, 96, 1), (1, 4, 2, 130, 0)])
@pytest.mark.parametrize("use_table", [False, True])
def test_rope_token_major_equals_head_major(rng, cuda, b, s, h, d, off, use_table):
    """[b, s, h, d] rotation == the [b, h, s, d] rotation of the transposed tensors, bit for bit."""
    q, k = normal_bf16(rng, (b, s, h, d)), normal_bf16(rng, (b, s, h, d))
    table = ops.rope_table(off + s, d) if use_table else None
    tq, tk = to_dev(q, cuda), to_dev(k, cuda)
    ops.rope_embed_token_major(tq, tk, off, 10000.0, table)
    hq = to_dev(np.ascontiguousarray(q.transpose(0, 2, 1, 3)), cuda)
    hk = to_dev(np.ascontiguousarray(k.transpose(0, 2, 1, 3)), cuda)
    ops.rope_embed(hq, hk, off, 10000.0, table)
    assert_bits_equal(to_host(tq), to_host(hq).transpose(0, 2, 1, 3), "q")
    assert_bits_equal(to_host(tk), to_host(hk).transpose(0, 2, 1, 3), "k")
