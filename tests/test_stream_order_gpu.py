"""Stream ordering of back-to-back launches (GPU).

Every kernel of the library is a programmatic dependent launch: the next
kernel in the stream may be scheduled while the previous one still runs, and
each kernel waits for its predecessor at entry.  These tests issue long
sequences of small dependent launches with no host synchronisation, where each
launch reads what the previous one wrote (read after write) and overwrites what
the previous one read (write after read), and compare the final state with the
same sequence run by the oracle, bit for bit.  Small tensors keep every kernel
short, so that neighbouring launches overlap as much as they can.
"""

import numpy as np
import pytest
import torch

import hrm_layer_ops as ops
from helpers import assert_bits_equal, normal_bf16, to_dev, to_host

pytestmark = pytest.mark.gpu

N = 64 * 512          # elements per elementwise tensor
ROWS, HIDDEN = 64, 512


def _oracle_elementwise(oracle, x, u, b, steps, negate_every=0):
    for i in range(steps):
        y = oracle.swiglu_ffn(x, u)
        x = oracle.additive_inject(y, b)
        if negate_every and i % negate_every == negate_every - 1:
            x = x ^ np.uint16(0x8000)
    return x


def test_elementwise_raw_and_war_chain(oracle, cuda):
    """200 x (y = swiglu(x, u); x = y + b): each launch reads the previous one's
    output and overwrites the buffer the previous one read."""
    rng = np.random.default_rng(11)
    x, u, b = normal_bf16(rng, N, 0.5), normal_bf16(rng, N, 0.5), normal_bf16(rng, N, 0.05)
    dx, du, db = to_dev(x, cuda), to_dev(u, cuda), to_dev(b, cuda)
    dy = torch.empty_like(dx)
    for _ in range(200):
        ops.swiglu_ffn(dx, du, out=dy)
        ops.additive_inject(dy, db, out=dx)
    assert_bits_equal(to_host(dx), _oracle_elementwise(oracle, x, u, b, 200), "x after 200 steps")


def test_interleaved_with_plain_torch_kernels(oracle, cuda):
    """Plain (non-programmatic) torch kernels between the library's launches:
    a negation every third step must be ordered on both sides."""
    rng = np.random.default_rng(12)
    x, u, b = normal_bf16(rng, N, 0.5), normal_bf16(rng, N, 0.5), normal_bf16(rng, N, 0.05)
    dx, du, db = to_dev(x, cuda), to_dev(u, cuda), to_dev(b, cuda)
    dy = torch.empty_like(dx)
    for i in range(120):
        ops.swiglu_ffn(dx, du, out=dy)
        ops.additive_inject(dy, db, out=dx)
        if i % 3 == 2:
            dx.neg_()
    assert_bits_equal(to_host(dx), _oracle_elementwise(oracle, x, u, b, 120, negate_every=3), "x")


def test_row_kernels_ping_pong(oracle, cuda):
    """(x', n') = add_rms_norm(x, n) alternating between two buffer pairs, 64
    steps: each launch writes the pair its predecessor read."""
    rng = np.random.default_rng(13)
    x, n = normal_bf16(rng, (ROWS, HIDDEN)), normal_bf16(rng, (ROWS, HIDDEN))
    w = normal_bf16(rng, HIDDEN, 0.1, 1.0)
    bufs = [(to_dev(x, cuda), to_dev(n, cuda)), (torch.empty((ROWS, HIDDEN), dtype=torch.bfloat16, device=cuda),
                                               torch.empty((ROWS, HIDDEN), dtype=torch.bfloat16, device=cuda))]
    dw = to_dev(w, cuda)
    for i in range(64):
        (sx, sn), (tx, tn) = bufs[i % 2], bufs[(i + 1) % 2]
        ops.add_rms_norm(sx, sn, dw, 1e-5, residual_out=tx, normed_out=tn)
    for _ in range(64):
        x, n = oracle.add_rms_norm(x, n, w, 1e-5)
    assert_bits_equal(to_host(bufs[0][0]), x, "residual")
    assert_bits_equal(to_host(bufs[0][1]), n, "normed")


def test_graph_replay_of_dependent_launches(oracle, cuda):
    """16 dependent steps captured in a CUDA graph and replayed 4 times equal
    64 steps of the oracle."""
    rng = np.random.default_rng(14)
    x, u, b = normal_bf16(rng, N, 0.5), normal_bf16(rng, N, 0.5), normal_bf16(rng, N, 0.05)
    dx, du, db = to_dev(x, cuda), to_dev(u, cuda), to_dev(b, cuda)
    dy = torch.empty_like(dx)
    x0 = dx.clone()
    s = torch.cuda.Stream(cuda)
    s.wait_stream(torch.cuda.current_stream(cuda))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for _ in range(16):
            ops.swiglu_ffn(dx, du, out=dy)
            ops.additive_inject(dy, db, out=dx)
    dx.copy_(x0)  # capture does not execute; start from x
    for _ in range(4):
        g.replay()
    torch.cuda.synchronize()
    assert_bits_equal(to_host(dx), _oracle_elementwise(oracle, x, u, b, 64), "x after 4 replays")
    del g


def test_two_streams_concurrently(oracle, cuda):
    """Two independent dependent-launch chains on two streams at once, joined
    by events: each equals its own oracle sequence."""
    rng = np.random.default_rng(15)
    xs = [normal_bf16(rng, N, 0.5) for _ in range(2)]
    u, b = normal_bf16(rng, N, 0.5), normal_bf16(rng, N, 0.05)
    du, db = to_dev(u, cuda), to_dev(b, cuda)
    streams = [torch.cuda.Stream(cuda) for _ in range(2)]
    dxs = [to_dev(x, cuda) for x in xs]
    dys = [torch.empty_like(dxs[0]) for _ in range(2)]
    torch.cuda.synchronize()
    for _ in range(100):
        for i, s in enumerate(streams):
            ops.swiglu_ffn(dxs[i], du, out=dys[i], stream=s)
            ops.additive_inject(dys[i], db, out=dxs[i], stream=s)
    for s in streams:
        torch.cuda.current_stream(cuda).wait_stream(s)
    for i in range(2):
        assert_bits_equal(to_host(dxs[i]), _oracle_elementwise(oracle, xs[i], u, b, 100), f"stream {i}")
