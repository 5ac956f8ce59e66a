"""GPU: RoPE pinned to the oracle in two separate parts.

The oracle's angles come from the C library (logf, expf, sinf, cosf), the
kernels' from CUDA's, so the two cos/sin tables differ slightly; rotating
with different tables mixes that difference into the rounding of every
output.  The two parts are therefore checked apart:

* rotation and rounding -- the oracle fed the device-built table rotates
  every element to the very same bf16 bits as the kernels (head-major and
  token-major, prefill and decode), i.e. 0 ulp at each element's own exponent;
* angles -- the device table differs from the oracle's table
  (rope_embed.cu:41-43 evaluated with glibc) by at most
  ANGLE_ULP fp32 ulp of the angle plus VALUE_ULP fp32 ulp of the value, per
  entry, at theta 1e4 and 1e6 over 65536 positions.
"""

import numpy as np
import pytest
import torch

import hrm_layer_ops as ops
from helpers import assert_bits_equal, normal_bf16, to_dev, to_host

pytestmark = pytest.mark.gpu

# Table bound, per entry: |dev - oracle| <= ANGLE_ULP * ulp32(angle) + VALUE_ULP * ulp32(value).
ANGLE_ULP, VALUE_ULP = 2.0, 2.0


def ulp32(x):
    a = np.abs(np.asarray(x, np.float64))
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -126)))
    return np.exp2(e - 23)


@pytest.mark.parametrize("layout", ["head", "token"])
@pytest.mark.parametrize("theta", [10000.0, 1e6])
def test_rotation_bit_exact_given_the_device_table(oracle, cuda, layout, theta):
    rng = np.random.default_rng(11)
    b, h, s, d = 2, 16, 4096, 128
    shape = (b, h, s, d) if layout == "head" else (b, s, h, d)
    q, k = normal_bf16(rng, shape), normal_bf16(rng, shape)
    table = ops.rope_table(s, d, theta)
    host_table = table.cpu().numpy()
    dq, dk = to_dev(q, cuda), to_dev(k, cuda)
    fn = ops.rope_embed if layout == "head" else ops.rope_embed_token_major
    ofn = oracle.rope_embed if layout == "head" else oracle.rope_embed_token_major
    fn(dq, dk, 0, theta, table)
    wq, wk = ofn(q, k, 0, theta, host_table)
    assert_bits_equal(to_host(dq), wq, "q, prefill")
    assert_bits_equal(to_host(dk), wk, "k, prefill")
    # decode: one position at offset 4095
    dshape = (b, h, 1, d) if layout == "head" else (b, 1, h, d)
    q1, k1 = normal_bf16(rng, dshape), normal_bf16(rng, dshape)
    dq1, dk1 = to_dev(q1, cuda), to_dev(k1, cuda)
    fn(dq1, dk1, 4095, theta, table)
    wq1, wk1 = ofn(q1, k1, 4095, theta, host_table)
    assert_bits_equal(to_host(dq1), wq1, "q, decode")
    assert_bits_equal(to_host(dk1), wk1, "k, decode")


@pytest.mark.parametrize("theta", [10000.0, 1e6])
def test_device_table_close_to_the_oracle_table(oracle, cuda, theta):
    positions, d = 65536, 128
    dev = ops.rope_table(positions, d, theta).cpu().numpy().astype(np.float64)
    ora = oracle.rope_table(positions, d, theta).astype(np.float64)
    half = d // 2
    # the oracle's fp32 angles, as rope_embed.cu:41 forms them
    i = np.arange(half, dtype=np.float32)
    inv = np.exp(np.float32(-2.0) * i * np.log(np.float32(theta)) / np.float32(d)).astype(np.float32)
    ang = (np.arange(positions, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float32)
    ang = np.concatenate([ang, ang], axis=1).astype(np.float64)
    bound = ANGLE_ULP * ulp32(ang) + VALUE_ULP * ulp32(ora)
    err = np.abs(dev - ora)
    worst = float((err / bound).max())
    print(f"theta {theta:g}: max |dev - oracle| / bound = {worst:.3f}; "
          f"max in angle ulps {float((err / ulp32(ang)).max()):.2f}; entries equal {np.mean(err == 0):.4f}")
    assert worst <= 1.0
