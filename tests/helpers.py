"""Helpers shared by the tests: seeded bf16 inputs and numpy <-> torch moves.

bf16 data lives in numpy as uint16 bit patterns and in torch as
torch.bfloat16 (moved through an int16 view, so bits are never re-rounded).
"""

import numpy as np

from oracle import f32_to_bf16

# The north star's bar for norm / rope / swiglu: max-abs error <= 2 bf16 ulp
# of the fp32-accumulated oracle.
ULP_TOL = 2.0


def normal_bf16(rng, shape, std=1.0, mean=0.0):
    x = rng.standard_normal(shape, dtype=np.float32)
    if std != 1.0:
        x *= np.float32(std)
    if mean != 0.0:
        x += np.float32(mean)
    return f32_to_bf16(x)


def to_dev(a, device):
    import torch

    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).to(device).view(torch.bfloat16)
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32).copy()).to(device)
    return torch.from_numpy(a.copy()).to(device)


def to_host(t):
    import torch

    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).cpu().numpy().view(np.uint16)
    return t.cpu().numpy()


def assert_bits_equal(got, want, what=""):
    got, want = np.asarray(got), np.asarray(want)
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    bad = np.flatnonzero(got.reshape(-1) != want.reshape(-1))
    assert bad.size == 0, (f"{what}: {bad.size} of {got.size} differ; first at {bad[0]}: "
                           f"{got.reshape(-1)[bad[0]]:#06x} != {want.reshape(-1)[bad[0]]:#06x}")


def rope_pair_magnitude(bits):
    """max(|x_i|, |x_{i+D/2}|) per element of a rotated [..., D] bf16 tensor.

    A rotation mixes the two members of a pair, so an angle that differs by a
    few fp32 ulp between two math libraries moves an output by about that
    angle times the pair's magnitude, even when the output itself is near
    zero.  RoPE's tolerance is therefore 2 bf16 ulp measured at the pair's
    magnitude (for the other ops it is measured at the value itself).
    """
    from oracle import bf16_to_f32

    v = np.abs(bf16_to_f32(bits))
    h = v.shape[-1] // 2
    m = np.maximum(v[..., :h], v[..., h:])
    return np.concatenate([m, m], axis=-1)


def max_ulp(got_bits, want_bits, magnitude=None):
    """Largest ulp error (see oracle.ulp_error); 0 for empty outputs."""
    from oracle import ulp_error

    err = ulp_error(got_bits, want_bits, magnitude)
    return float(err.max()) if err.size else 0.0
