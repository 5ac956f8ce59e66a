"""GPU: the launch-resident RMSNorm path (one CTA per SM, every row of the
launch bulk-copied into shared memory at the start) against the oracle, bit
for bit, at the row counts around its limits.

The path takes launches of at least 8 rows per SM whose per-CTA share of rows
fits the SM's shared memory: bf16 rows of 2048 up to 56 per SM, fp32 rows of
2048 up to 28 per SM.  Just past either limit the warp-per-row grid takes the
launch; both sides of each limit are compared, with and without a weight, and
no bounded wait may have run out.
"""

import numpy as np
import pytest
import torch

import hrm_layer_ops as ops
from helpers import assert_bits_equal, normal_bf16, to_dev, to_host

pytestmark = pytest.mark.gpu


def sms():
    return torch.cuda.get_device_properties(0).multi_processor_count


def bf16_cases():
    g = sms()
    return [(8 * g - 1, 2048), (8 * g, 8), (8 * g + 1, 200), (1500, 1536), (4096, 2048), (2000, 4096),
            (56 * g, 2048), (56 * g + 1, 2048), (5003, 40)]


def f32_cases():
    g = sms()
    return [(8 * g, 4), (1500, 200), (4096, 2048), (28 * g, 2048), (28 * g + 1, 2048), (3001, 1020)]


@pytest.mark.parametrize("case", range(9))
@pytest.mark.parametrize("weighted", [True, False])
def test_resident_bf16_matches_oracle(oracle, cuda, case, weighted):
    rows, hidden = bf16_cases()[case]
    rng = np.random.default_rng(1000 + case)
    x = normal_bf16(rng, (rows, hidden), 1.5)
    w = normal_bf16(rng, hidden, 0.1, 1.0) if weighted else None
    ops.wait_timeouts(reset=True)
    y = ops.rms_norm(to_dev(x, cuda), None if w is None else to_dev(w, cuda), eps=1e-5)
    assert_bits_equal(to_host(y), oracle.rms_norm(x, w, eps=1e-5), f"bf16 [{rows} x {hidden}]")
    torch.cuda.synchronize()
    assert ops.wait_timeouts() == 0


@pytest.mark.parametrize("case", range(6))
@pytest.mark.parametrize("weighted", [True, False])
def test_resident_f32_matches_oracle(oracle, cuda, case, weighted):
    rows, hidden = f32_cases()[case]
    rng = np.random.default_rng(2000 + case)
    x = rng.standard_normal((rows, hidden)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(hidden)).astype(np.float32) if weighted else None
    ops.wait_timeouts(reset=True)
    y = ops.rms_norm(torch.from_numpy(x).to(cuda), None if w is None else torch.from_numpy(w).to(cuda), eps=1e-5)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), oracle.rms_norm_f32(x, w, eps=1e-5).view(np.uint32))
    torch.cuda.synchronize()
    assert ops.wait_timeouts() == 0


def test_resident_back_to_back_in_a_graph(oracle, cuda):
    """Dependent resident launches replayed from a CUDA graph (programmatic
    launches: each waits for the previous one's output) equal the oracle's chain."""
    rng = np.random.default_rng(7)
    x = normal_bf16(rng, (4096, 2048))
    w = normal_bf16(rng, 2048, 0.1, 1.0)
    dx, dw = to_dev(x, cuda), to_dev(w, cuda)
    bufs = [dx] + [torch.empty_like(dx) for _ in range(4)]
    s = torch.cuda.Stream(cuda)
    s.wait_stream(torch.cuda.current_stream(cuda))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(4):
            ops.rms_norm(bufs[i], dw, 1e-5, out=bufs[i + 1], stream=s)
    g.replay()
    torch.cuda.synchronize()
    want = x
    for _ in range(4):
        want = oracle.rms_norm(want, w, eps=1e-5)
    assert_bits_equal(to_host(bufs[4]), want, "4 chained resident launches")
