"""CPU suite for the oracle: pins it to the reference before it checks anything.

* The reference's own known answers (src/lib.rs:2225-2279, restated in
  golden/reference_kats.json) at the reference's tolerance (0.01).
* Outputs of the reference's own kernels (compiled from its sources, run on a
  B200 by golden/make_golden.py --from-reference) on seeded inputs: bit-exact
  for the ops whose arithmetic the oracle reproduces exactly (residual add,
  embedding gather, RMSNorm including its reduction order), <= 2 bf16 ulp
  where only the transcendental library differs (SwiGLU's __expf, RoPE's
  expf/logf/sincosf).
* Derived known answers for the two ops the reference never tested.
"""

import glob
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN
from helpers import ULP_TOL, normal_bf16, rope_pair_magnitude
from oracle import bf16_to_f32, f32_to_bf16, ulp_error


def load_kats():
    with open(os.path.join(GOLDEN, "reference_kats.json")) as f:
        return json.load(f)


def test_reference_kat_additive_inject(oracle):
    k = load_kats()
    t = k["tests"]["additive_inject"]
    out = bf16_to_f32(oracle.additive_inject(f32_to_bf16(np.array(t["a"], np.float32)),
                                             f32_to_bf16(np.array(t["b"], np.float32))))
    assert np.all(np.abs(out - np.array(t["expected"])) < k["tolerance"])


def test_reference_kat_rms_norm(oracle):
    k = load_kats()
    t = k["tests"]["rms_norm"]
    x = np.array(t["x"], np.float32).reshape(t["rows"], t["hidden"])
    y = bf16_to_f32(oracle.rms_norm(f32_to_bf16(x), eps=1e-6))
    expected = x / (np.sqrt(30.0) / 2.0)
    assert np.all(np.abs(y - expected) < k["tolerance"])


def test_reference_kat_swiglu(oracle):
    k = load_kats()
    t = k["tests"]["swiglu_ffn"]
    y = bf16_to_f32(oracle.swiglu_ffn(f32_to_bf16(np.array(t["gate"], np.float32)),
                                      f32_to_bf16(np.array(t["up"], np.float32))))
    assert np.all(np.abs(y - np.array(t["expected"])) < k["tolerance"])


# ------------------------------------------------------------ bf16 rounding
def test_bf16_rounding_matches_c(oracle):
    rng = np.random.default_rng(7)
    x = np.concatenate([
        rng.standard_normal(10000).astype(np.float32) * 10.0,
        np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 3.4e38, -3.4e38, 1e-40, -1e-45,
                  1.00390625, 1.01171875, 1.0078125], np.float32),  # ties to even around 1.0
    ])
    import ctypes

    oracle.lib.ora_f32_to_bf16.argtypes = [ctypes.c_float]
    oracle.lib.ora_f32_to_bf16.restype = ctypes.c_uint16
    c = np.array([oracle.lib.ora_f32_to_bf16(float(v)) for v in x], np.uint16)
    assert np.array_equal(c, f32_to_bf16(x))
    assert f32_to_bf16(np.array([np.nan], np.float32))[0] == 0x7FFF
    # ties: 1 + 2^-8 rounds down to 1.0 (even), 1 + 3*2^-8 rounds up
    assert f32_to_bf16(np.array([1.00390625], np.float32))[0] == 0x3F80
    assert f32_to_bf16(np.array([1.01171875], np.float32))[0] == 0x3F82


# ------------------------------------------------- derived known answers
def test_rope_position_zero_is_identity(oracle, rng):
    q, k = normal_bf16(rng, (2, 3, 1, 128)), normal_bf16(rng, (2, 3, 1, 128))
    q2, k2 = oracle.rope_embed(q, k, offset=0)
    assert np.array_equal(q2, q) and np.array_equal(k2, k)


def test_rope_table_equals_formula(oracle, rng):
    q, k = normal_bf16(rng, (1, 2, 64, 128)), normal_bf16(rng, (1, 2, 64, 128))
    table = oracle.rope_table(100, 128)
    a = oracle.rope_embed(q, k, offset=17)
    b = oracle.rope_embed(q, k, offset=17, table=table)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


def test_rope_offset_equals_sliced_sequence(oracle, rng):
    """rope with (offset p, seq 1) equals row p of the full-sequence run."""
    q, k = normal_bf16(rng, (1, 2, 40, 64)), normal_bf16(rng, (1, 2, 40, 64))
    full_q, _ = oracle.rope_embed(q, k, offset=0)
    for p in (0, 1, 17, 39):
        one_q, _ = oracle.rope_embed(q[:, :, p:p + 1], k[:, :, p:p + 1], offset=p)
        assert np.array_equal(one_q[:, :, 0], full_q[:, :, p])


def test_rope_token_major_is_the_transposed_head_major(oracle, rng):
    """[B, S, H, D] rows rotate exactly as the same rows laid out [B, H, S, D]."""
    q = rng.integers(0, 1 << 16, (2, 40, 3, 64), dtype=np.uint16) & 0xBFFF  # finite values
    k = rng.integers(0, 1 << 16, (2, 40, 3, 64), dtype=np.uint16) & 0xBFFF
    for table in (None, oracle.rope_table(77, 64, 10000.0)):
        tq, tk = oracle.rope_embed_token_major(q, k, 37, 10000.0, table)
        hq, hk = oracle.rope_embed(q.transpose(0, 2, 1, 3), k.transpose(0, 2, 1, 3), 37, 10000.0, table)
        assert np.array_equal(tq, hq.transpose(0, 2, 1, 3)) and np.array_equal(tk, hk.transpose(0, 2, 1, 3))


def test_rope_preserves_pair_norm(oracle, rng):
    q, k = normal_bf16(rng, (1, 4, 256, 128)), normal_bf16(rng, (1, 4, 256, 128))
    q2, _ = oracle.rope_embed(q, k, offset=3000)
    a, b = bf16_to_f32(q).astype(np.float64), bf16_to_f32(q2).astype(np.float64)
    n0 = np.hypot(a[..., :64], a[..., 64:])
    n1 = np.hypot(b[..., :64], b[..., 64:])
    assert np.max(np.abs(n1 - n0) / np.maximum(n0, 1e-3)) < 2 * 2.0 ** -8


def test_embedding_scale_one_returns_rows_and_clamps(oracle, rng):
    table = normal_bf16(rng, (50, 24), 0.02)
    ids = np.array([0, 49, 50, 12345, 0xFFFFFFFF, 7], np.uint32)
    out = oracle.embedding_lookup(ids, table, 1.0)
    want = table[[0, 49, 49, 49, 49, 7]]
    assert np.array_equal(out, want)


def test_add_rms_norm_is_add_then_norm(oracle, rng):
    x, b = normal_bf16(rng, (9, 2048)), normal_bf16(rng, (9, 2048))
    w = normal_bf16(rng, 2048, 0.1, 1.0)
    r, y = oracle.add_rms_norm(x, b, w, eps=1e-5)
    assert np.array_equal(r, oracle.additive_inject(x, b))
    assert np.array_equal(y, oracle.rms_norm(r, w, eps=1e-5))


def test_embed_rms_norm_is_embed_then_norm(oracle, rng):
    table = normal_bf16(rng, (100, 256), 0.02)
    ids = rng.integers(0, 120, 33, dtype=np.uint32)
    h, y = oracle.embed_rms_norm(ids, table, 16.0, None, eps=1e-6)
    assert np.array_equal(h, oracle.embedding_lookup(ids, table, 16.0))
    assert np.array_equal(y, oracle.rms_norm(h, None, eps=1e-6))


def test_results_independent_of_thread_count(oracle, rng):
    x = normal_bf16(rng, (64, 2048))
    a = oracle.rms_norm(x, eps=1e-5)
    oracle.set_threads(1)
    try:
        b = oracle.rms_norm(x, eps=1e-5)
    finally:
        oracle.set_threads(os.cpu_count() or 1)
    assert np.array_equal(a, b)


def test_rms_norm_f32_close_to_float64(oracle, rng):
    x = rng.standard_normal((16, 2048)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(2048)).astype(np.float32)
    y = oracle.rms_norm_f32(x, w, eps=1e-5)
    xd = x.astype(np.float64)
    want = xd / np.sqrt((xd ** 2).mean(-1, keepdims=True) + 1e-5) * w
    assert np.max(np.abs(y - want) / np.abs(want).clip(1e-6)) < 1e-5


# ---------------------------------------- pinned to the reference's kernels
REF_FIXTURES = sorted(glob.glob(os.path.join(GOLDEN, "ref_kernels_*.npz")))


def test_reference_kernel_fixtures_present():
    names = {os.path.basename(p)[len("ref_kernels_"):-4] for p in REF_FIXTURES}
    assert {"rms_norm", "additive_inject", "swiglu_ffn", "embedding_lookup", "rope_embed",
            "rope_embed_decode"} <= names, "run tests/golden/make_golden.py --from-reference on a GPU"


@pytest.mark.parametrize("path", REF_FIXTURES, ids=lambda p: os.path.basename(p)[12:-4])
def test_oracle_matches_reference_kernels(oracle, path):
    d = np.load(path)
    name = os.path.basename(path)[len("ref_kernels_"):-4]
    if name.startswith("rms_norm"):
        got = oracle.rms_norm(d["x"], None, float(d["eps"]))
        assert np.array_equal(got, d["y"]), "rms_norm must be bit-exact (same reduction order)"
    elif name == "additive_inject":
        assert np.array_equal(oracle.additive_inject(d["a"], d["b"]), d["out"])
    elif name == "embedding_lookup":
        assert np.array_equal(oracle.embedding_lookup(d["ids"], d["table"], float(d["scale"])), d["out"])
    elif name == "swiglu_ffn":
        err = ulp_error(oracle.swiglu_ffn(d["gate"], d["up"]), d["out"])
        assert err.max() <= ULP_TOL, f"swiglu max {err.max()} ulp"
    else:
        q, k = oracle.rope_embed(d["q"], d["k"], int(d["offset"]), float(d["theta"]))
        for got, want in ((q, d["q_out"]), (k, d["k_out"])):
            err = ulp_error(got, want, rope_pair_magnitude(want))
            assert err.max() <= ULP_TOL, f"rope max {err.max()} ulp"



def test_reference_kat_gated_attn_output(oracle):
    k = load_kats()
    t = k["tests"]["gated_attn_output"]
    y = bf16_to_f32(oracle.gated_attn_output(f32_to_bf16(np.array(t["gate"], np.float32)),
                                             f32_to_bf16(np.array(t["attn"], np.float32))))
    assert np.all(np.abs(y - np.array(t["expected"])) < k["tolerance"])


def test_broadcast_vec(oracle, rng):
    src = normal_bf16(rng, 37)
    out = oracle.broadcast_vec(src, 5)
    assert out.shape == (5, 37) and all(np.array_equal(r, src) for r in out)


def test_convert_f16_exhaustive_matches_exact_widening(oracle):
    """Every f16 pattern: finite and infinite values equal numpy's exact f16 -> f32
    widening rounded to nearest even; NaNs keep sign and payload top bits, quiet."""
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    got = oracle.convert_to_bf16(h.tobytes(), "f16")
    f = h.view(np.float16).astype(np.float32)
    num = ~np.isnan(f)
    assert np.array_equal(got[num], f32_to_bf16(f[num]))
    nan = np.flatnonzero(~num)
    want = ((h[nan].astype(np.uint32) & 0x8000) | 0x7FC0 | ((h[nan].astype(np.uint32) & 0x3FF) >> 3)).astype(np.uint16)
    assert np.array_equal(got[nan], want)


def test_convert_f32_rounding_and_nan_rule(oracle, rng):
    x = rng.standard_normal(100000).astype(np.float32) * np.float32(1e3)
    specials = np.array([0x00000000, 0x80000000, 0x7F800000, 0xFF800000, 0x00000001, 0x807FFFFF,
                         0x3F808000, 0x3F818000, 0x3F808001, 0x7F7FFFFF, 0x7F7F8000, 0x7F7F7FFF],
                        np.uint32).view(np.float32)
    x = np.concatenate([x, specials])
    assert np.array_equal(oracle.convert_to_bf16(x.tobytes(), "f32"), f32_to_bf16(x))
    nans = np.array([0x7FC00000, 0xFFC00001, 0x7F800001, 0xFFA5A5A5, 0x7FFFFFFF], np.uint32)
    got = oracle.convert_to_bf16(nans.tobytes(), "f32")
    assert np.array_equal(got, ((nans >> 16) | 0x40).astype(np.uint16))
    raw = normal_bf16(rng, 1000)
    assert np.array_equal(oracle.convert_to_bf16(raw.tobytes(), "bf16"), raw)
