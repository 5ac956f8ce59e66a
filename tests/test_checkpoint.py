"""CPU: safetensors headers (the checkpoint path's file format).

The Python front end (hrm_layer_ops.checkpoint) and the C++ host layer
(host/safetensors.cpp, through `test_layer_ops --parse`) restate the header
rules of the safetensors crate the reference loads checkpoints with
(Cargo.lock: 0.4.5).  Both parse the committed fixture checkpoints
(tests/golden/make_checkpoint.py) to the same tensors, which the safetensors
package, where installed, reads back to the same bytes; and both reject each
malformed header with the crate's error name.
"""

import json
import os
import struct
import subprocess

import numpy as np
import pytest

from conftest import GOLDEN, PKG
from hrm_layer_ops import checkpoint as ck

FIXTURES = ["ckpt_tiny_attn.safetensors", "ckpt_tiny_flat.safetensors"]
EXE = os.path.join(PKG, "build", "test_layer_ops")


def cpp_parse(path):
    res = subprocess.run([EXE, "--parse", path], capture_output=True, text=True, timeout=60)
    assert res.returncode == 0, res.stdout + res.stderr
    return res.stdout.split()


@pytest.mark.parametrize("name", FIXTURES)
def test_fixture_headers(name):
    path = os.path.join(GOLDEN, name)
    h = ck.read_header(path)
    size = os.path.getsize(path)
    assert h.data_offset % 8 == 0 and h.data_offset + h.tensors[-1].end == size
    assert all(a.end == b.begin for a, b in zip(h.tensors, h.tensors[1:]))
    assert cpp_parse(path) == ["ok", str(len(h.tensors)), str(h.data_offset)]
    if name == FIXTURES[0]:
        assert h.metadata == {"format": "pt", "note": "synthetic"}
        # odd offsets: f32 tensors that do not start on a 4-byte boundary
        assert any(t.dtype == "F32" and t.begin % 4 for t in h.tensors)
        assert {t.dtype for t in h.tensors} == {"F32", "BF16", "F16"}


@pytest.mark.parametrize("name", FIXTURES)
def test_fixture_reads_back_with_the_safetensors_package(name):
    st = pytest.importorskip("safetensors.torch")
    import torch

    path = os.path.join(GOLDEN, name)
    h = ck.read_header(path)
    raw = open(path, "rb").read()
    tensors = st.load_file(path)
    assert sorted(tensors) == sorted(t.name for t in h.tensors)
    names = {torch.float32: "F32", torch.bfloat16: "BF16", torch.float16: "F16"}
    for t in h.tensors:
        got = tensors[t.name]
        assert names[got.dtype] == t.dtype and tuple(got.shape) == t.shape
        want = raw[h.data_offset + t.begin:h.data_offset + t.end]
        assert got.contiguous().view(torch.uint8).numpy().tobytes() == want, t.name


def _file(tmp_path, header, data=b"", n=None, raw_header=None):
    text = raw_header if raw_header is not None else json.dumps(header).encode()
    p = tmp_path / "x.safetensors"
    p.write_bytes(struct.pack("<Q", len(text) if n is None else n) + text + data)
    return str(p)


def t(dtype, shape, b, e):
    return {"dtype": dtype, "shape": shape, "data_offsets": [b, e]}


CASES = [
    ("HeaderTooSmall", dict(raw=b"\x01\x00\x00")),
    ("HeaderTooLarge", dict(header={}, n=100_000_001)),
    ("InvalidHeaderLength", dict(header={"a": t("F32", [1], 0, 4)}, n=4096)),
    ("InvalidHeader", dict(raw_header=b'{"\xff":1}')),
    ("InvalidHeaderStart", dict(raw_header=b'[{"a":1}]')),
    ("InvalidHeaderDeserialization", dict(raw_header=b'{"a": {"dtype": "F32", "shape": [1]')),
    ("InvalidHeaderDeserialization", dict(header={"a": t("F128", [1], 0, 4)}, data=b"\0" * 4)),
    ("InvalidHeaderDeserialization", dict(header={"a": t("F32", [-1], 0, 4)}, data=b"\0" * 4)),
    ("InvalidHeaderDeserialization", dict(header={"a": {"dtype": "F32", "shape": [1]}}, data=b"\0" * 4)),
    ("InvalidHeaderDeserialization", dict(raw_header=b'{"a":{"dtype":"F32","shape":[1.0],"data_offsets":[0,4]}}',
                                          data=b"\0" * 4)),
    ("InvalidHeaderDeserialization", dict(header={"__metadata__": {"k": 1}})),
    ("InvalidHeaderDeserialization", dict(raw_header=b'{"a":{"dtype":"F32","shape":[1],"data_offsets":[0,4]},'
                                                     b'"a":{"dtype":"F32","shape":[1],"data_offsets":[0,4]}}',
                                          data=b"\0" * 4)),
    ("InvalidHeaderDeserialization", dict(raw_header=b'{"\\ud800":{"dtype":"F32","shape":[1],"data_offsets":[0,4]}}',
                                          data=b"\0" * 4)),
    ("InvalidOffset", dict(header={"a": t("F32", [1], 4, 8)}, data=b"\0" * 8)),
    ("InvalidOffset", dict(header={"a": t("F32", [1], 0, 4), "b": t("F32", [1], 2, 6)}, data=b"\0" * 8)),
    ("TensorInvalidInfo", dict(header={"a": t("F32", [2], 0, 4)}, data=b"\0" * 4)),
    ("ValidationOverflow", dict(header={"a": t("F32", [1 << 40, 1 << 40], 0, 4)}, data=b"\0" * 4)),
    ("MetadataIncompleteBuffer", dict(header={"a": t("F32", [1], 0, 4)}, data=b"\0" * 6)),
]


@pytest.mark.parametrize("kind,case", CASES, ids=[f"{i}-{c[0]}" for i, c in enumerate(CASES)])
def test_malformed_headers_rejected_alike(tmp_path, kind, case):
    if "raw" in case:
        p = tmp_path / "x.safetensors"
        p.write_bytes(case["raw"])
        path = str(p)
    else:
        path = _file(tmp_path, case.get("header"), case.get("data", b""), case.get("n"), case.get("raw_header"))
    with pytest.raises(ck.SafetensorsError) as e:
        ck.read_header(path)
    assert e.value.kind == kind
    assert cpp_parse(path) == ["error", kind]


@pytest.mark.parametrize("kind,case", [c for c in CASES if c[0] not in ("InvalidHeaderDeserialization",)])
def test_the_safetensors_package_rejects_them_too(tmp_path, kind, case):
    st = pytest.importorskip("safetensors")
    if "raw" in case:
        p = tmp_path / "x.safetensors"
        p.write_bytes(case["raw"])
        path = str(p)
    else:
        path = _file(tmp_path, case.get("header"), case.get("data", b""), case.get("n"), case.get("raw_header"))
    with pytest.raises(Exception):
        with st.safe_open(path, framework="np") as f:
            for k in f.keys():
                f.get_slice(k)


def test_valid_edge_cases(tmp_path):
    """Accepted alike: an empty header object, zero-size tensors, escaped
    names, a null __metadata__, extra fields and padding spaces."""
    hdr = {"__metadata__": None, "zéro": t("BF16", [0, 5], 0, 0),
           "w": dict(t("F16", [3], 0, 6), extra=[1, {"x": None}])}
    text = json.dumps(hdr).encode() + b"   "
    p = tmp_path / "ok.safetensors"
    p.write_bytes(struct.pack("<Q", len(text)) + text + np.arange(3, dtype="<f2").tobytes())
    h = ck.read_header(str(p))
    assert [x.name for x in h.tensors] == ["zéro", "w"] and h.metadata == {}
    assert cpp_parse(str(p)) == ["ok", "2", str(8 + len(text))]
    p.write_bytes(struct.pack("<Q", 2) + b"{}")
    assert ck.read_header(str(p)).tensors == [] and cpp_parse(str(p)) == ["ok", "0", "10"]
