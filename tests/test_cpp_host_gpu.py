"""GPU: the C++ host layer's known-answer tests (tests/cpp/test_layer_ops.cpp),
which restate the reference's own GPU tests (src/lib.rs:2225-2279) through
the HrmLayerOps methods that mirror the reference's wrappers, and check the
C++ layer-loop schedule (transformer_module) against the reference's order of
wrapper calls and device copies."""

import os
import subprocess

import pytest

from conftest import GOLDEN, PKG

pytestmark = pytest.mark.gpu


def test_cpp_host_known_answers():
    exe = os.path.join(PKG, "build", "test_layer_ops")
    assert os.path.exists(exe), "build with make -C hrm-text-cuda_b200"
    res = subprocess.run([exe, "--golden", GOLDEN], capture_output=True, text=True, timeout=120)
    print(res.stdout)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "all 14 tests passed" in res.stdout and "ok   test_bf16_from_f32" in res.stdout
    assert "ok   test_safetensors_header" in res.stdout and "ok   test_load_safetensors" in res.stdout


def test_bounded_mbarrier_wait_self_test():
    """tests/cpp/test_wait_timeout.cu: the deadline of the bulk-copy kernels'
    mbarrier waits -- waits that complete return at once; a barrier nothing
    completes returns false after 50 ms and is counted; the context stays usable."""
    exe = os.path.join(PKG, "build", "test_wait_timeout")
    assert os.path.exists(exe), "build with make -C hrm-text-cuda_b200"
    res = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    print(res.stdout)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "all wait tests passed" in res.stdout
