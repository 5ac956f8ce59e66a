"""GPU: checkpoint file -> bf16 device tensors (the on-disk format row).

hrm_layer_ops.checkpoint.load_safetensors reads the committed fixture
checkpoints (f32 / bf16 / f16 tensors, f32 tensors at byte offsets that are
not multiples of 4, NaN payloads, infinities, denormals and rounding ties)
and converts on the GPU.  Every device tensor must equal, bit for bit, the
oracle's restatement of the reference's raw_to_bf16 (src/lib.rs:1981-2008)
applied to the tensor's bytes in the file, with gate_up split at
intermediate x hidden elements as src/lib.rs:2072-2078 does -- for chunk
sizes that cut tensors at chunk ends and for whole-file chunks.  The C ABI
entry hrm_upload_to_bf16 is also checked on its own: pinned and pageable host
sources, staging buffers smaller than the tensor, and every dtype.
"""

import ctypes
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from helpers import to_host
from hrm_layer_ops import checkpoint as ck
from hrm_layer_ops._lib import DTYPES, HrmError, call

pytestmark = pytest.mark.gpu

LAYERS, HIDDEN, INTER = 2, 32, 48


def expected(oracle, raw, h, name, first=0, n=None):
    t = h.find(name)
    es = ck.DTYPE_SIZES[t.dtype]
    n = t.numel - first if n is None else n
    b0 = h.data_offset + t.begin + first * es
    return oracle.convert_to_bf16(raw[b0:b0 + n * es], t.dtype.lower())


@pytest.mark.parametrize("name", ["ckpt_tiny_attn.safetensors", "ckpt_tiny_flat.safetensors"])
@pytest.mark.parametrize("chunk", [64, 4096, 64 << 20])
def test_load_matches_raw_to_bf16(oracle, cuda, name, chunk):
    path = os.path.join(GOLDEN, name)
    raw = open(path, "rb").read()
    h = ck.read_header(path)
    w = ck.load_safetensors(path, LAYERS, HIDDEN, INTER, device=cuda, chunk_bytes=chunk, reader_threads=3)
    attn = "attn" in name
    a, m = (".attn", ".mlp") if attn else ("", "")
    split = INTER * HIDDEN
    for prefix, layers in (("model.H_module.layers", w.h_module), ("model.L_module.layers", w.l_module)):
        assert len(layers) == LAYERS
        for i, lw in enumerate(layers):
            p = f"{prefix}.{i}"
            gu = f"{p}{m}.gate_up_proj.weight"
            for got, want in ((lw.gqkv_proj, expected(oracle, raw, h, f"{p}{a}.gqkv_proj.weight")),
                              (lw.o_proj, expected(oracle, raw, h, f"{p}{a}.o_proj.weight")),
                              (lw.gate_proj, expected(oracle, raw, h, gu, 0, split)),
                              (lw.up_proj, expected(oracle, raw, h, gu, split)),
                              (lw.down_proj, expected(oracle, raw, h, f"{p}{m}.down_proj.weight"))):
                assert np.array_equal(to_host(got), want)
    assert np.array_equal(to_host(w.embed_tokens), expected(oracle, raw, h, "model.embed_tokens.weight"))
    lm = "lm_head.weight" if attn else "model.lm_head.weight"
    assert np.array_equal(to_host(w.lm_head), expected(oracle, raw, h, lm))
    assert np.array_equal(to_host(w.z_l_init), expected(oracle, raw, h, "model.z_L_init"))


def test_load_errors(cuda, tmp_path):
    path = os.path.join(GOLDEN, "ckpt_tiny_flat.safetensors")
    with pytest.raises(ValueError, match="missing tensor: model.H_module.layers.2.gqkv_proj.weight"):
        ck.load_safetensors(path, 3, HIDDEN, INTER, device=cuda)
    with pytest.raises(ValueError, match="fewer than intermediate x hidden"):
        ck.load_safetensors(path, LAYERS, HIDDEN, 4 * INTER, device=cuda)
    bad = tmp_path / "trunc.safetensors"
    bad.write_bytes(open(path, "rb").read()[:-2])
    with pytest.raises(ck.SafetensorsError) as e:
        ck.load_safetensors(str(bad), LAYERS, HIDDEN, INTER, device=cuda)
    assert e.value.kind == "MetadataIncompleteBuffer"


@pytest.mark.parametrize("dtype,size", [("f32", 4), ("f16", 2), ("bf16", 2)])
@pytest.mark.parametrize("pinned", [True, False])
@pytest.mark.parametrize("staging_bytes", [16, 1000, 1 << 20])
def test_upload_entry_point(oracle, cuda, dtype, size, pinned, staging_bytes):
    rng = np.random.default_rng(size + staging_bytes)
    n = 100_003
    raw = rng.integers(0, 256, n * size + 1, dtype=np.uint8)
    src = torch.from_numpy(raw)
    if pinned:
        src = src.pin_memory()
    src = src[1:]  # an odd host address
    dst = torch.empty(n, dtype=torch.bfloat16, device=cuda)
    staging = torch.empty(staging_bytes, dtype=torch.uint8, device=cuda)
    s = torch.cuda.current_stream(cuda)
    call("hrm_upload_to_bf16", ctypes.c_void_p(src.data_ptr()), DTYPES[dtype], ctypes.c_void_p(dst.data_ptr()), n,
         ctypes.c_void_p(staging.data_ptr()), staging_bytes, ctypes.c_void_p(s.cuda_stream))
    s.synchronize()
    assert np.array_equal(to_host(dst), oracle.convert_to_bf16(raw[1:].tobytes(), dtype))


def test_upload_rejects_bad_arguments(cuda):
    dst = torch.empty(64, dtype=torch.bfloat16, device=cuda)
    staging = torch.empty(64, dtype=torch.uint8, device=cuda)
    src = torch.zeros(256, dtype=torch.uint8).pin_memory()
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    with pytest.raises(HrmError) as e:
        call("hrm_upload_to_bf16", p(src), DTYPES["f32"], p(dst), 64, p(staging), 8, None)
    assert "invalid" in str(e.value) or e.value.status == 2
    with pytest.raises(HrmError):
        call("hrm_upload_to_bf16", p(src), 7, p(dst), 64, p(staging), 64, None)
    with pytest.raises(HrmError):  # staging overlapping dst
        call("hrm_upload_to_bf16", p(src), DTYPES["f32"], p(dst), 64, ctypes.c_void_p(dst.data_ptr() + 32), 64, None)
