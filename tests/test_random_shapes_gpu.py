"""GPU: randomized shapes, alignments and arguments for every operator, checked
against the oracle with the same bars as the fixed cases (bit-exact for the
add, gather, norms, gate copies and conversion; <= 2 bf16 ulp for SwiGLU, the
attention gate and RoPE).  Hypothesis runs derandomized, so a failing case is
reproduced by rerunning the test."""

import numpy as np
import pytest
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

import hrm_layer_ops as ops
from helpers import ULP_TOL, assert_bits_equal, max_ulp, normal_bf16, rope_pair_magnitude, to_dev, to_host
from oracle import Oracle

pytestmark = pytest.mark.gpu

SETTINGS = settings(max_examples=25, deadline=None, derandomize=True)
ORACLE = None


def oracle():
    global ORACLE
    if ORACLE is None:
        ORACLE = Oracle()
    return ORACLE


def dev(a, offset):
    """Device copy of a, starting `offset` elements into its allocation."""
    t = to_dev(a, torch.device("cuda", 0))
    if offset == 0:
        return t
    buf = torch.empty(t.numel() + offset, dtype=t.dtype, device=t.device)
    v = buf[offset:].view(t.shape)
    v.copy_(t)
    return v


@SETTINGS
@given(rows=st.integers(0, 300), hidden=st.integers(1, 5000), off=st.sampled_from([0, 1, 8]),
       weight=st.booleans(), eps=st.sampled_from([1e-6, 1e-5, 0.1]), seed=st.integers(0, 2**31))
def test_random_norms(rows, hidden, off, weight, eps, seed):
    rng = np.random.default_rng(seed)
    x, b = normal_bf16(rng, (rows, hidden), 2.0), normal_bf16(rng, (rows, hidden))
    w = normal_bf16(rng, hidden, 0.1, 1.0) if weight else None
    dw = None if w is None else dev(w, off)
    y = ops.rms_norm(dev(x, off), dw, eps)
    assert_bits_equal(to_host(y), oracle().rms_norm(x, w, eps), "rms_norm")
    r, n = ops.add_rms_norm(dev(x, off), dev(b, off), dw, eps)
    wr, wn = oracle().add_rms_norm(x, b, w, eps)
    assert_bits_equal(to_host(r), wr, "residual")
    assert_bits_equal(to_host(n), wn, "normed")


@SETTINGS
@given(tokens=st.integers(0, 200), hidden=st.integers(1, 3000), vocab=st.integers(1, 500),
       off=st.sampled_from([0, 1]), scale=st.floats(0.0625, 64.0, width=32), seed=st.integers(0, 2**31))
def test_random_gathers(tokens, hidden, vocab, off, scale, seed):
    rng = np.random.default_rng(seed)
    table = normal_bf16(rng, (vocab, hidden), 0.02)
    ids = rng.integers(0, vocab + 10, tokens, dtype=np.uint32)
    dt, di = dev(table, off), to_dev(ids, torch.device("cuda", 0))
    assert_bits_equal(to_host(ops.embedding_lookup(di, dt, scale)), oracle().embedding_lookup(ids, table, scale),
                      "embedding")
    h, n = ops.embed_rms_norm(di, dt, scale, None, 1e-5)
    wh, wn = oracle().embed_rms_norm(ids, table, scale, None, 1e-5)
    assert_bits_equal(to_host(h), wh, "hidden")
    assert_bits_equal(to_host(n), wn, "normed")


@SETTINGS
@given(n=st.integers(0, 100000), off=st.sampled_from([0, 1, 3, 8]), seed=st.integers(0, 2**31))
def test_random_elementwise(n, off, seed):
    rng = np.random.default_rng(seed)
    a, b = normal_bf16(rng, n, 3.0), normal_bf16(rng, n)
    assert_bits_equal(to_host(ops.additive_inject(dev(a, off), dev(b, off))), oracle().additive_inject(a, b), "add")
    assert max_ulp(to_host(ops.swiglu_ffn(dev(a, off), dev(b, off))), oracle().swiglu_ffn(a, b)) <= ULP_TOL
    assert max_ulp(to_host(ops.gated_attn_output(dev(a, off), dev(b, off))),
                   oracle().gated_attn_output(a, b)) <= ULP_TOL


@SETTINGS
@given(b=st.integers(1, 3), h=st.integers(1, 5), s=st.integers(1, 70), half=st.integers(1, 80),
       offset=st.integers(0, 5000), table=st.booleans(), token_major=st.booleans(), seed=st.integers(0, 2**31))
def test_random_rope(b, h, s, half, offset, table, token_major, seed):
    d = 2 * half
    rng = np.random.default_rng(seed)
    q, k = normal_bf16(rng, (b, h, s, d)), normal_bf16(rng, (b, h, s, d))
    tab = ops.rope_table(offset + s, d) if table else None
    if token_major:
        dq = to_dev(np.ascontiguousarray(q.transpose(0, 2, 1, 3)), torch.device("cuda", 0))
        dk = to_dev(np.ascontiguousarray(k.transpose(0, 2, 1, 3)), torch.device("cuda", 0))
        ops.rope_embed_token_major(dq, dk, offset, 10000.0, tab)
        gq, gk = to_host(dq).transpose(0, 2, 1, 3), to_host(dk).transpose(0, 2, 1, 3)
    else:
        dq, dk = dev(q, 0), dev(k, 0)
        ops.rope_embed(dq, dk, offset, 10000.0, tab)
        gq, gk = to_host(dq), to_host(dk)
    wq, wk = oracle().rope_embed(q, k, offset, 10000.0)
    for got, want in ((gq, wq), (gk, wk)):
        assert max_ulp(got, want, rope_pair_magnitude(want)) <= ULP_TOL


@SETTINGS
@given(b=st.integers(1, 2), s=st.integers(1, 40), h=st.integers(1, 4), half=st.sampled_from([8, 16, 32, 64, 3, 5]),
       offset=st.integers(0, 100), cache=st.booleans(), seed=st.integers(0, 2**31))
def test_random_split_rope(b, s, h, half, offset, cache, seed):
    d = 2 * half
    rng = np.random.default_rng(seed)
    g = normal_bf16(rng, (b, s, 4 * h * d))
    cl = offset + s + 1
    kc0, vc0 = normal_bf16(rng, (b, h, cl, d)), normal_bf16(rng, (b, h, cl, d))
    dkc, dvc = (dev(kc0, 0), dev(vc0, 0)) if cache else (None, None)
    gate, q, k, v = ops.split_gqkv_rope(dev(g, 0), h, offset, 10000.0, None, dkc, dvc, cache_offset=offset)
    wg, wq, wk, wv, wkc, wvc = oracle().split_gqkv_rope(g, b, s, h, d, offset, 10000.0, None, kc0, vc0, offset)
    assert_bits_equal(to_host(gate), wg, "gate")
    assert_bits_equal(to_host(v), wv, "v")
    for got, want in ((to_host(q), wq), (to_host(k), wk)):
        assert max_ulp(got, want, rope_pair_magnitude(want)) <= ULP_TOL
    if cache:
        assert_bits_equal(to_host(dvc), wvc, "v cache")


@SETTINGS
@given(n=st.integers(0, 50000), off=st.integers(0, 16), dtype=st.sampled_from(["f32", "f16", "bf16"]),
       seed=st.integers(0, 2**31))
def test_random_convert(n, off, dtype, seed):
    rng = np.random.default_rng(seed)
    size = 4 if dtype == "f32" else 2
    raw = rng.integers(0, 256, n * size, dtype=np.uint8).tobytes()  # every bit pattern, NaNs included
    buf = torch.zeros(len(raw) + off, dtype=torch.uint8, device=torch.device("cuda", 0))
    if raw:
        buf[off:] = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(buf.device)
    got = to_host(ops.convert_to_bf16(buf[off:], dtype))
    assert_bits_equal(got, oracle().convert_to_bf16(raw, dtype), dtype)
