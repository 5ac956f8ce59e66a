"""Counter-based synthetic inputs (hrm_layer_ops.synth): pinned values, the
shard property, host == device bit for bit, and the distributions."""

import numpy as np
import pytest
import torch

from hrm_layer_ops import synth


def test_splitmix64_published_first_output():
    # SplitMix64 from state 0: first output 0xE220A8397B1DCDAF.  With seed 0 and
    # tag 0 the key equals mix(0), so element 0 is mix(key ^ mix(0)) = mix(0).
    assert int(synth.bits_np(0, 0, 0, 1)[0]) == 0xE220A8397B1DCDAF


def test_pinned_values():
    assert [int(v) for v in synth.normal_bf16_np(0, synth.tag_of("q"), 0, 6)] == \
        [0x3F31, 0xC02C, 0xC018, 0x3D7A, 0xBF63, 0xBCAB]
    assert list(synth.ids_np(0, synth.tag_of("ids"), 0, 6, 32000)) == [12451, 28118, 15043, 17795, 21193, 14527]


def test_a_shard_is_a_slice_of_the_global_stream():
    full = synth.normal_bf16_np(5, 9, 0, 20000, 0.5)
    for a, b in ((0, 1), (7, 7001), (12345, 20000)):
        assert np.array_equal(synth.normal_bf16_np(5, 9, a, b - a, 0.5), full[a:b])
    ids = synth.ids_np(5, 9, 0, 20000, 77)
    assert np.array_equal(synth.ids_np(5, 9, 100, 900, 77), ids[100:1000])
    # different tags and seeds give different streams
    assert not np.array_equal(synth.normal_bf16_np(5, 10, 0, 64), full[:64])
    assert not np.array_equal(synth.normal_bf16_np(6, 9, 0, 64), synth.normal_bf16_np(5, 9, 0, 64))


def test_torch_cpu_equals_numpy():
    n = 200_003
    want = synth.normal_bf16_np(1, synth.tag_of("gate"), 4096, n, 0.5)
    got = synth.normal_bf16((n,), 1, synth.tag_of("gate"), 4096, 0.5, device="cpu")
    assert np.array_equal(got.view(torch.int16).numpy().view(np.uint16), want)
    ids = synth.ids(n, 1, synth.tag_of("ids"), 32000, 99, device="cpu").numpy().astype(np.uint32)
    assert np.array_equal(ids, synth.ids_np(1, synth.tag_of("ids"), 99, n, 32000))


def test_distributions():
    x = (synth.normal_bf16_np(2, 3, 0, 1 << 20, 0.1, 1.0).astype(np.uint32) << 16).view(np.float32)
    assert abs(x.mean() - 1.0) < 1e-3 and abs(x.std() - 0.1) < 1e-3
    # shape, before bf16 rounding: the mass within 1, 2 and 3 sigma
    z = synth.normal_f32_np(2, 5, 0, 1 << 20)
    for k, p in ((1, 0.6827), (2, 0.9545), (3, 0.9973)):
        assert abs(np.mean(np.abs(z) < k) - p) < 0.003
    ids = synth.ids_np(2, 4, 0, 1 << 20, 32000)
    assert ids.max() < 32000
    counts = np.bincount(ids, minlength=32000)
    assert counts.std() < 2 * np.sqrt(counts.mean())


@pytest.mark.gpu
def test_device_equals_host(cuda):
    """The CUDA path (int64 ops, float64 log / cos) equals numpy bit for bit on
    4M normals and 4M ids at an odd offset."""
    n, start = 1 << 22, (1 << 33) + 17
    got = synth.normal_bf16((n,), 3, synth.tag_of("up"), start, 0.5, device=cuda)
    want = synth.normal_bf16_np(3, synth.tag_of("up"), start, n, 0.5)
    assert np.array_equal(got.view(torch.int16).cpu().numpy().view(np.uint16), want)
    ids = synth.ids(n, 3, synth.tag_of("ids"), 32000, start, device=cuda).cpu().numpy().astype(np.uint32)
    assert np.array_equal(ids, synth.ids_np(3, synth.tag_of("ids"), start, n, 32000))


def test_oracle_generator_equals_numpy(oracle):
    """The oracle's C generator (the CPU reference arm's inputs) gives the same
    bits as the numpy path, so both arms of the benchmark see the same values."""
    n = 1 << 20
    for tag, start, std, mean in ((synth.tag_of("gate"), 12345, 0.5, 0.0),
                                  (synth.tag_of("norm1_weight"), 0, 0.1, 1.0), (7, 1 << 40, 1.0, 0.0)):
        got = oracle.fill_normal_bf16(np.empty(n, np.uint16), 0, tag, start, std, mean)
        assert np.array_equal(got, synth.normal_bf16_np(0, tag, start, n, std, mean))
    got = oracle.fill_ids(np.empty(n, np.uint32), 3, synth.tag_of("ids"), 32000, 999)
    assert np.array_equal(got, synth.ids_np(3, synth.tag_of("ids"), 999, n, 32000))
