"""GPU parity at the full benchmark sizes (the five layer-op workloads).

Each workload is run once through the C ABI on seeded synthetic inputs of the
benchmark's shapes and distributions and compared with the oracle over the
whole output (the multithreaded oracle finishes each in seconds), with the
same bars as the small cases.  Size-independent properties are checked too:
the fused ops equal their unfused sequences, RoPE decode equals the matching
row of the prefill run, and the table and in-kernel angle paths agree.
"""

import numpy as np
import pytest
import torch

import hrm_layer_ops as ops
from helpers import ULP_TOL, assert_bits_equal, normal_bf16, rope_pair_magnitude, to_dev, to_host
from oracle import ulp_error

pytestmark = pytest.mark.gpu


def test_rms_norm_f32_4096x2048(oracle, cuda):
    """RMSNorm fp32 [4096 x 2048], w = 1 + 0.1 N(0,1), eps 1e-5, seed 0."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal((4096, 2048)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(2048)).astype(np.float32)
    y = ops.rms_norm(torch.from_numpy(x).to(cuda), torch.from_numpy(w).to(cuda), eps=1e-5).cpu().numpy()
    assert np.array_equal(y.view(np.uint32), oracle.rms_norm_f32(x, w, eps=1e-5).view(np.uint32))


@pytest.mark.parametrize("dtype,rows", [("bf16", 4096), ("bf16", 16384), ("f32", 4096), ("f32", 8192)])
def test_rms_norm_both_paths(oracle, cuda, dtype, rows):
    """Plain RMSNorm [rows x 2048] with a weight at the benchmark's row count
    and at 2-4x more (several waves of CTAs per SM), bit-exact."""
    rng = np.random.default_rng(rows)
    if dtype == "f32":
        x = rng.standard_normal((rows, 2048)).astype(np.float32)
        w = (1 + 0.1 * rng.standard_normal(2048)).astype(np.float32)
        y = ops.rms_norm(torch.from_numpy(x).to(cuda), torch.from_numpy(w).to(cuda), eps=1e-5).cpu().numpy()
        assert np.array_equal(y.view(np.uint32), oracle.rms_norm_f32(x, w, eps=1e-5).view(np.uint32))
    else:
        x, w = normal_bf16(rng, (rows, 2048), 1.5), normal_bf16(rng, 2048, 0.1, 1.0)
        y = ops.rms_norm(to_dev(x, cuda), to_dev(w, cuda), eps=1e-5)
        assert_bits_equal(to_host(y), oracle.rms_norm(x, w, eps=1e-5), f"bf16 {rows} rows")


@pytest.mark.parametrize("hidden", [2048, 1600])
@pytest.mark.parametrize("weighted", [True, False])
def test_rms_norm_one_wave_shape_boundary(oracle, cuda, hidden, weighted):
    """Plain bf16 RMSNorm over rows of 1544-2048 elements takes a one-wave shape
    (64 registers, 8-warp CTAs, 4 CTAs per SM) when the launch fits in one wave
    of it, and the 80-register 4-warp shape otherwise.  Both sides of the
    boundary (SMs x 32 rows), and launches with fewer than 8 rows per SM, are
    bit-exact against the oracle."""
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    edge = sms * 4 * 8
    rng = np.random.default_rng(hidden + weighted)
    w = normal_bf16(rng, hidden, 0.1, 1.0) if weighted else None
    for rows in (edge, edge + 1, edge + 8, sms * 8 - 1, sms + 3):
        x = normal_bf16(rng, (rows, hidden), 1.5)
        y = ops.rms_norm(to_dev(x, cuda), to_dev(w, cuda) if weighted else None, eps=1e-5)
        assert_bits_equal(to_host(y), oracle.rms_norm(x, w, eps=1e-5), f"{rows} x {hidden}")


@pytest.mark.parametrize("weighted", [True, False])
def test_rms_norm_f32_wave_boundaries(oracle, cuda, weighted):
    """fp32 RMSNorm over 2048-wide rows runs 16 warps per SM (4 CTAs of 4 warps
    at 119 registers), one row per warp (the HRM_RN_F32_TWO_ROWS build takes two
    rows per warp for launches of one to two waves).  Rows at one and two full
    waves (SMs x 16 and SMs x 32), just past each, and between them with a
    ragged last CTA are bit-exact against the oracle."""
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    one_wave = sms * 16
    rng = np.random.default_rng(7 + weighted)
    w = (1 + 0.1 * rng.standard_normal(2048)).astype(np.float32) if weighted else None
    for rows in (one_wave, one_wave + 1, one_wave + 5, sms * 24 + 3, 2 * one_wave, 2 * one_wave + 4):
        x = rng.standard_normal((rows, 2048)).astype(np.float32)
        dw = torch.from_numpy(w).to(cuda) if weighted else None
        y = ops.rms_norm(torch.from_numpy(x).to(cuda), dw, eps=1e-5).cpu().numpy()
        assert np.array_equal(y.view(np.uint32), oracle.rms_norm_f32(x, w, eps=1e-5).view(np.uint32)), rows


def test_add_rms_norm_16384x2048(oracle, cuda):
    """Fused residual add + RMSNorm bf16 [16384 x 2048], w = 1 + 0.1 N(0,1), eps 1e-5."""
    rng = np.random.default_rng(1)
    x, b = normal_bf16(rng, (16384, 2048)), normal_bf16(rng, (16384, 2048))
    w = normal_bf16(rng, 2048, 0.1, 1.0)
    dx, db, dw = to_dev(x, cuda), to_dev(b, cuda), to_dev(w, cuda)
    r, y = ops.add_rms_norm(dx, db, dw, eps=1e-5)
    wr, wy = oracle.add_rms_norm(x, b, w, eps=1e-5)
    assert_bits_equal(to_host(r), wr, "residual")
    assert_bits_equal(to_host(y), wy, "normed")
    # property: fused == additive_inject then rms_norm, on the device
    assert torch.equal(ops.rms_norm(ops.additive_inject(dx, db), dw, eps=1e-5).view(torch.int16),
                       y.view(torch.int16))


def test_rope_8x16x4096x128_prefill_and_decode(oracle, cuda):
    """RoPE on Q and K [8, 16, 4096, 128], theta 1e4, positions 0..4095, fp32 table;
    decode [8, 16, 1, 128] at offset 4095."""
    rng = np.random.default_rng(2)
    shape = (8, 16, 4096, 128)
    q, k = normal_bf16(rng, shape), normal_bf16(rng, shape)
    table = ops.rope_table(4096, 128, 10000.0)
    dq, dk = to_dev(q, cuda), to_dev(k, cuda)
    ops.rope_embed(dq, dk, 0, 10000.0, table)
    wq, wk = oracle.rope_embed(q, k, 0, 10000.0, oracle.rope_table(4096, 128, 10000.0))
    for got, want in ((to_host(dq), wq), (to_host(dk), wk)):
        assert ulp_error(got, want, rope_pair_magnitude(want)).max() <= ULP_TOL
    # decode at offset 4095 == row 4095 of the prefill, bit for bit
    sq, sk = to_dev(q[:, :, 4095:], cuda), to_dev(k[:, :, 4095:], cuda)
    ops.rope_embed(sq, sk, 4095, 10000.0, table)
    assert torch.equal(sq.view(torch.int16), dq[:, :, 4095:].view(torch.int16))
    assert torch.equal(sk.view(torch.int16), dk[:, :, 4095:].view(torch.int16))


def test_swiglu_32768x5632(oracle, cuda):
    """SwiGLU bf16 gate, up [32768 x 5632] ~ 0.5 N(0,1)."""
    rng = np.random.default_rng(3)
    g, u = normal_bf16(rng, (32768, 5632), 0.5), normal_bf16(rng, (32768, 5632), 0.5)
    out = to_host(ops.swiglu_ffn(to_dev(g, cuda), to_dev(u, cuda)))
    err = ulp_error(out, oracle.swiglu_ffn(g, u))
    assert err.max() <= ULP_TOL, f"max {err.max()} ulp"
    assert np.mean(err == 0) > 0.99


def test_chain_65536_tokens_and_decode(oracle, cuda):
    """Chained layer-op pass: embedding [32000 x 2048] ~ N(0, 0.02), ids U[0, 32000)
    -> RMSNorm -> RoPE on Q/K [tokens x 16 x 128] -> residual + RMSNorm ->
    SwiGLU [tokens x 5632]; 65536 tokens (as [16, 16, 4096, 128] Q/K), then the
    64-token decode shape ([64, 16, 1, 128] at offset 4095).  SwiGLU's inputs
    are generated on the device and checked on 2048 sampled rows (the full
    [32768 x 5632] SwiGLU is checked whole above)."""
    rng = np.random.default_rng(4)
    H, I = 2048, 5632
    scale, eps = float(np.float32(np.sqrt(2048.0))), 1e-5
    table = normal_bf16(rng, (32000, H), 0.02)
    w1, w2 = normal_bf16(rng, H, 0.1, 1.0), normal_bf16(rng, H, 0.1, 1.0)
    rope_tab = ops.rope_table(4096, 128, 10000.0)
    rope_tab_h = oracle.rope_table(4096, 128, 10000.0)
    dtable, dw1, dw2 = to_dev(table, cuda), to_dev(w1, cuda), to_dev(w2, cuda)
    for tokens, batch, seq, off in ((65536, 16, 4096, 0), (64, 64, 1, 4095)):
        ids = rng.integers(0, 32000, tokens, dtype=np.uint32)
        q, k = normal_bf16(rng, (batch, 16, seq, 128)), normal_bf16(rng, (batch, 16, seq, 128))
        o = normal_bf16(rng, (tokens, H))
        gen = torch.Generator(device=cuda).manual_seed(tokens)
        dg = (torch.randn((tokens, I), generator=gen, device=cuda) * 0.5).to(torch.bfloat16)
        du = (torch.randn((tokens, I), generator=gen, device=cuda) * 0.5).to(torch.bfloat16)
        dq, dk = to_dev(q, cuda), to_dev(k, cuda)
        h, n1 = ops.embed_rms_norm(to_dev(ids, cuda), dtable, scale, dw1, eps)
        ops.rope_embed(dq, dk, off, 10000.0, rope_tab)
        r, n2 = ops.add_rms_norm(h, to_dev(o, cuda), dw2, eps)
        out = ops.swiglu_ffn(dg, du)
        wh, wn1 = oracle.embed_rms_norm(ids, table, scale, w1, eps)
        wq, wk = oracle.rope_embed(q, k, off, 10000.0, rope_tab_h)
        wr, wn2 = oracle.add_rms_norm(wh, o, w2, eps)
        assert_bits_equal(to_host(h), wh, f"{tokens}: hidden")
        assert_bits_equal(to_host(n1), wn1, f"{tokens}: norm1")
        assert_bits_equal(to_host(r), wr, f"{tokens}: residual")
        assert_bits_equal(to_host(n2), wn2, f"{tokens}: norm2")
        for got, want in ((to_host(dq), wq), (to_host(dk), wk)):
            assert ulp_error(got, want, rope_pair_magnitude(want)).max() <= ULP_TOL
        rows = np.sort(rng.choice(tokens, min(tokens, 2048), replace=False))
        sel = torch.from_numpy(rows).to(cuda)
        g, u = to_host(dg[sel]), to_host(du[sel])
        assert ulp_error(to_host(out[sel]), oracle.swiglu_ffn(g, u)).max() <= ULP_TOL
    torch.cuda.synchronize()
    assert ops.wait_timeouts() == 0  # no bounded device wait ran out


def test_chain_at_the_reference_model_shapes(oracle, cuda):
    """The chained pass at the reference's default model shapes (hidden 1536,
    12 heads of 128, intermediate 4096, vocab 65536, scale sqrt(1536)) over
    16384 tokens, token-major Q/K [4, 4096, 12, 128]: every output against the
    oracle (SwiGLU on 2048 sampled rows)."""
    from hrm_layer_ops import chain

    rng = np.random.default_rng(6)
    H, HEADS, I, V, T, S = 1536, 12, 4096, 65536, 16384, 4096
    scale, eps = float(np.float32(np.sqrt(1536.0))), 1e-5
    table = normal_bf16(rng, (V, H), 0.02)
    w1, w2 = normal_bf16(rng, H, 0.1, 1.0), normal_bf16(rng, H, 0.1, 1.0)
    ids = rng.integers(0, V, T, dtype=np.uint32)
    q, k = normal_bf16(rng, (T // S, S, HEADS, 128)), normal_bf16(rng, (T // S, S, HEADS, 128))
    o = normal_bf16(rng, (T, H))
    gen = torch.Generator(device=cuda).manual_seed(6)
    dg = (torch.randn((T, I), generator=gen, device=cuda) * 0.5).to(torch.bfloat16)
    du = (torch.randn((T, I), generator=gen, device=cuda) * 0.5).to(torch.bfloat16)
    w = chain.ChainWeights(table=to_dev(table, cuda), w1=to_dev(w1, cuda), w2=to_dev(w2, cuda),
                           rope=ops.rope_table(S, 128), scale=scale, eps=eps, theta=10000.0)
    dq, dk = to_dev(q, cuda), to_dev(k, cuda)
    bf = dict(dtype=torch.bfloat16, device=cuda)
    h, n1, r, n2 = (torch.empty((T, H), **bf) for _ in range(4))
    y = torch.empty((T, I), **bf)
    chain.run_device(w, to_dev(ids, cuda), dq, dk, to_dev(o, cuda), dg, du, h, n1, r, n2, y, 0, token_major=True)
    wh, wn1 = oracle.embed_rms_norm(ids, table, scale, w1, eps)
    wr, wn2 = oracle.add_rms_norm(wh, o, w2, eps)
    assert_bits_equal(to_host(h), wh, "hidden")
    assert_bits_equal(to_host(n1), wn1, "norm1")
    assert_bits_equal(to_host(r), wr, "residual")
    assert_bits_equal(to_host(n2), wn2, "norm2")
    hq, hk = q.transpose(0, 2, 1, 3), k.transpose(0, 2, 1, 3)  # the oracle's [B, H, S, D]
    wq, wk = oracle.rope_embed(np.ascontiguousarray(hq), np.ascontiguousarray(hk), 0, 10000.0,
                               oracle.rope_table(S, 128, 10000.0))
    for got, want in ((to_host(dq).transpose(0, 2, 1, 3), wq), (to_host(dk).transpose(0, 2, 1, 3), wk)):
        assert ulp_error(np.ascontiguousarray(got), want, rope_pair_magnitude(want)).max() <= ULP_TOL
    rows = np.sort(rng.choice(T, 2048, replace=False))
    sel = torch.from_numpy(rows).to(cuda)
    assert ulp_error(to_host(y[sel]), oracle.swiglu_ffn(to_host(dg[sel]), to_host(du[sel]))).max() <= ULP_TOL
