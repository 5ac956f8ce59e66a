"""CPU suite for the C ABI boundary (no kernel is launched here).

* libhrm_ops.so loads and exports every function include/hrm_ops.h declares;
  the Python front end binds exactly that set.
* Argument validation happens on the host before anything is queued, so the
  error paths are testable without a GPU: every case below returns its
  status before any CUDA call.
* The front end refuses CPU tensors (there is no fallback implementation).
"""

import ctypes
import os
import re

import pytest

from conftest import PKG, ROOT

HEADER = os.path.join(ROOT, "include", "hrm_ops.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(hrm_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    import hrm_layer_ops

    return hrm_layer_ops.LIB


def test_header_declares_the_reference_wrappers():
    names = declared_functions()
    for op in ("hrm_additive_inject", "hrm_rms_norm", "hrm_rope_embed", "hrm_swiglu_ffn",
               "hrm_embedding_lookup", "hrm_add_rms_norm"):
        assert op in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_python_front_end_binds_every_declared_symbol():
    from hrm_layer_ops import _lib

    declared = set(declared_functions()) - {"hrm_status_string"}
    assert declared == set(_lib.SIGNATURES)


def declared_arity():
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for m in re.finditer(r"\b(hrm_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text):
        out[m.group(1)] = len([a for a in m.group(2).split(",") if a.strip() and a.strip() != "void"])
    return out


def test_python_bindings_match_header_arity():
    from hrm_layer_ops import _lib

    arity = declared_arity()
    for name, args in _lib.SIGNATURES.items():
        assert len(args) == arity[name], (name, len(args), arity[name])


def test_static_archive_and_cpp_host_built():
    for f in ("lib/libhrm_ops.a", "lib/libhrm_host.a", "build/test_layer_ops", "build/test_wait_timeout"):
        assert os.path.exists(os.path.join(PKG, f)), f


def test_abi_version_and_status_strings(lib):
    from hrm_layer_ops import _lib

    assert lib.hrm_abi_version() // 10000 == 1
    for code in (_lib.HRM_OK, _lib.HRM_ERR_NULL_POINTER, _lib.HRM_ERR_INVALID_SHAPE,
                 _lib.HRM_ERR_SIZE_OVERFLOW, _lib.HRM_ERR_ALIASING, _lib.HRM_ERR_TABLE_RANGE):
        assert lib.hrm_status_string(code).decode() not in ("", "unknown status")


# Fake device addresses: validation rejects every call below before it could
# dereference or launch anything.
A, B, C = 0x10000000, 0x20000000, 0x30000000
vp = ctypes.c_void_p


def test_validation_negative_and_zero_sizes(lib):
    from hrm_layer_ops import _lib

    assert lib.hrm_additive_inject(vp(A), vp(B), vp(C), -1, None) == _lib.HRM_ERR_INVALID_SHAPE
    assert lib.hrm_additive_inject(None, None, None, 0, None) == _lib.HRM_OK  # empty: nothing to do
    assert lib.hrm_swiglu_ffn(vp(A), vp(B), vp(C), -5, None) == _lib.HRM_ERR_INVALID_SHAPE
    assert lib.hrm_swiglu_ffn(None, None, None, 0, None) == _lib.HRM_OK
    assert lib.hrm_rms_norm(vp(A), vp(B), None, 4, 0, 1e-6, None) == _lib.HRM_ERR_INVALID_SHAPE
    assert lib.hrm_rms_norm(None, None, None, 0, 2048, 1e-6, None) == _lib.HRM_OK
    assert lib.hrm_rope_embed(vp(A), vp(B), 1, 1, 1, 127, 0, 1e4, None, 0, None) == _lib.HRM_ERR_INVALID_SHAPE
    assert lib.hrm_rope_embed(vp(A), vp(B), 1, 1, 1, 128, -1, 1e4, None, 0, None) == _lib.HRM_ERR_INVALID_SHAPE
    assert lib.hrm_rope_embed(None, None, 0, 16, 4096, 128, 0, 1e4, None, 0, None) == _lib.HRM_OK
    assert lib.hrm_embedding_lookup(vp(A), vp(B), vp(C), 1, 4, 2048, 0, 1.0, None) == _lib.HRM_ERR_INVALID_SHAPE
    assert lib.hrm_embedding_lookup(None, None, None, 0, 4, 2048, 10, 1.0, None) == _lib.HRM_OK
    assert lib.hrm_rope_table_build(vp(A), 16, 0, 1e4, None) == _lib.HRM_ERR_INVALID_SHAPE


def test_validation_null_pointers(lib):
    from hrm_layer_ops import _lib

    assert lib.hrm_wait_timeouts(None, 0) == _lib.HRM_ERR_NULL_POINTER

    assert lib.hrm_additive_inject(None, vp(B), vp(C), 8, None) == _lib.HRM_ERR_NULL_POINTER
    assert lib.hrm_rms_norm(vp(A), None, None, 1, 8, 1e-6, None) == _lib.HRM_ERR_NULL_POINTER
    assert lib.hrm_add_rms_norm(vp(A), vp(B), None, vp(C), None, 1, 8, 1e-6, None) == _lib.HRM_ERR_NULL_POINTER
    assert lib.hrm_rope_embed(None, vp(B), 1, 1, 1, 128, 0, 1e4, None, 0, None) == _lib.HRM_ERR_NULL_POINTER
    assert lib.hrm_embed_rms_norm(vp(A), vp(B), None, None, None, 1, 8, 4, 1.0, 1e-6,
                                  None) == _lib.HRM_ERR_NULL_POINTER


def test_validation_aliasing(lib):
    from hrm_layer_ops import _lib

    # out overlaps a by half a buffer (exact aliasing would be allowed).
    assert lib.hrm_additive_inject(vp(A), vp(B), vp(A + 8), 16, None) == _lib.HRM_ERR_ALIASING
    assert lib.hrm_swiglu_ffn(vp(A), vp(B), vp(B + 2), 16, None) == _lib.HRM_ERR_ALIASING
    # rms_norm in place is rejected (the two-pass fallback re-reads its input).
    assert lib.hrm_rms_norm(vp(A), vp(A), None, 2, 8, 1e-6, None) == _lib.HRM_ERR_ALIASING
    # normed_out overlapping the residual output.
    assert lib.hrm_add_rms_norm(vp(A), vp(B), vp(C), vp(C + 4), None, 2, 8, 1e-6, None) == _lib.HRM_ERR_ALIASING
    # q and k overlap.
    assert lib.hrm_rope_embed(vp(A), vp(A + 64), 1, 1, 2, 128, 0, 1e4, None, 0, None) == _lib.HRM_ERR_ALIASING


def test_validation_rope_table_range_and_overflow(lib):
    from hrm_layer_ops import _lib

    # 4096-row table cannot serve offset 4095 + seq 2.
    assert lib.hrm_rope_embed(vp(A), vp(B), 1, 1, 2, 128, 4095, 1e4, vp(C), 4096, None) == _lib.HRM_ERR_TABLE_RANGE
    assert lib.hrm_rope_embed(vp(A), vp(B), 1, 1, 2, 128, 2**31 - 1, 1e4, None, 0,
                              None) == _lib.HRM_ERR_SIZE_OVERFLOW
    assert lib.hrm_additive_inject(vp(A), vp(B), vp(C), 2**62, None) == _lib.HRM_ERR_SIZE_OVERFLOW
    # offsets near INT64_MAX are rejected without forming an overflowing sum
    big = 2**63 - 1
    assert lib.hrm_rope_embed(vp(A), vp(B), 1, 1, 2, 128, big, 1e4, None, 0, None) == _lib.HRM_ERR_SIZE_OVERFLOW
    assert lib.hrm_rope_embed(vp(A), vp(B), 1, 1, big, 128, 1, 1e4, None, 0, None) == _lib.HRM_ERR_SIZE_OVERFLOW
    D = 0x40000000
    split = lambda offset, cache_len, cache_offset: lib.hrm_split_gqkv_rope(  # noqa: E731
        vp(A), vp(B), vp(C), vp(C + D), vp(C + 2 * D), vp(C + 3 * D), vp(C + 4 * D), 1, 2, 1, 128, offset, 1e4,
        None, 0, cache_len, cache_offset, None)
    assert split(big, 0, 0) == _lib.HRM_ERR_SIZE_OVERFLOW
    assert split(0, 8, big) == _lib.HRM_ERR_INVALID_SHAPE  # cache_offset + seq would overflow
    assert split(0, 8, 7) == _lib.HRM_ERR_INVALID_SHAPE    # rows 7 and 8 of an 8-row cache
    assert split(0, 1, 0) == _lib.HRM_ERR_INVALID_SHAPE    # seq 2 > cache_len 1


def test_front_end_rejects_cpu_tensors():
    import torch

    import hrm_layer_ops

    x = torch.zeros(4, 8, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        hrm_layer_ops.rms_norm(x)
    with pytest.raises(ValueError, match="CUDA"):
        hrm_layer_ops.swiglu_ffn(x, x)


def test_front_end_refuses_tensors_on_two_devices():
    """Every tensor of a call (and an explicit stream) must be on one device:
    checked on the host before the library is called."""
    from types import SimpleNamespace

    import torch

    from hrm_layer_ops import ops

    t0 = SimpleNamespace(device=torch.device("cuda", 0))
    t1 = SimpleNamespace(device=torch.device("cuda", 1))
    with pytest.raises(ValueError, match="one device"):
        ops._launch("hrm_swiglu_ffn", (t0, None, t1), None)
    with pytest.raises(ValueError, match="stream on"):
        ops._launch("hrm_swiglu_ffn", (t0, t0), SimpleNamespace(device=torch.device("cuda", 1)))


def test_cpp_host_code_without_a_gpu():
    """The C++ host layer's own f32 -> bf16 (half's from_f32, NaN rule
    included) and its safetensors header parser on the fixture checkpoints."""
    import subprocess

    from conftest import GOLDEN

    exe = os.path.join(PKG, "build", "test_layer_ops")
    res = subprocess.run([exe, "--host-only", "--golden", GOLDEN], capture_output=True, text=True, timeout=60)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "all 2 host tests passed" in res.stdout
