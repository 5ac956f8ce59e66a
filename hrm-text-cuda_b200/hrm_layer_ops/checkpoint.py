"""safetensors checkpoint -> bf16 device tensors, converted on the GPU.

Replaces the reference's loader (src/lib.rs:2023-2125): it reads the whole
file, converts every tensor to bf16 on the host one element at a time
(raw_to_bf16, src/lib.rs:1981-2008), splits gate_up on the host
(src/lib.rs:2072-2078) and copies each tensor with htod_copy.  Here

* `read_header` parses and validates the header as the `safetensors` crate
  0.4.5 does (Cargo.lock; format and rules restated, raising
  SafetensorsError with the crate's error names);
* `load_safetensors` reads only the bytes of the tensors the model uses, in
  chunks of whole elements, into a ring of pinned host buffers with several
  reader threads, and uploads + converts each chunk's tensors on the GPU
  through the C ABI (hrm_upload_to_bf16, one device staging buffer), reading
  the next chunk while the GPU copies the previous one; gate_up's halves land
  straight in gate_proj and up_proj.

The returned structure mirrors the reference's ModelWeights (src/lib.rs:62-83).
"""

from __future__ import annotations

import ctypes
import json
import os
import struct
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import torch

from ._lib import DTYPES, call

MAX_HEADER = 100_000_000  # the crate's MAX_HEADER_SIZE
DTYPE_SIZES = {"BOOL": 1, "U8": 1, "I8": 1, "F8_E5M2": 1, "F8_E4M3": 1, "I16": 2, "U16": 2, "F16": 2, "BF16": 2,
               "I32": 4, "U32": 4, "F32": 4, "F64": 8, "I64": 8, "U64": 8}
ABI_DTYPE = {"BF16": DTYPES["bf16"], "F32": DTYPES["f32"], "F16": DTYPES["f16"]}


class SafetensorsError(ValueError):
    """A header the safetensors crate would reject; `kind` is the crate's
    SafeTensorError variant name (HeaderTooSmall, HeaderTooLarge,
    InvalidHeaderLength, InvalidHeader, InvalidHeaderStart,
    InvalidHeaderDeserialization, InvalidOffset, TensorInvalidInfo,
    ValidationOverflow, MetadataIncompleteBuffer)."""

    def __init__(self, kind: str, what: str):
        super().__init__(f"{kind}: {what}")
        self.kind = kind


@dataclass
class TensorInfo:
    name: str
    dtype: str
    shape: Tuple[int, ...]
    begin: int  # byte range within the data section
    end: int

    @property
    def numel(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n


@dataclass
class Header:
    header_len: int
    tensors: List[TensorInfo]  # in data-offset order
    metadata: Dict[str, str] = field(default_factory=dict)

    @property
    def data_offset(self) -> int:
        return 8 + self.header_len

    def find(self, name: str) -> Optional[TensorInfo]:
        for t in self.tensors:
            if t.name == name:
                return t
        return None


def _is_uint(v) -> bool:
    return isinstance(v, int) and not isinstance(v, bool) and 0 <= v < 1 << 64


def _object(pairs):
    """json object hook: no duplicate keys, and no lone surrogate escapes in a
    key or string value (strict JSON, as serde_json reads it)."""
    keys = [k for k, _ in pairs]
    if len(keys) != len(set(keys)):
        raise SafetensorsError("InvalidHeaderDeserialization", "duplicate key")
    try:
        for k, v in pairs:
            k.encode("utf-8")
            if isinstance(v, str):
                v.encode("utf-8")
            elif isinstance(v, list):
                for x in v:
                    if isinstance(x, str):
                        x.encode("utf-8")
    except UnicodeEncodeError as e:
        raise SafetensorsError("InvalidHeaderDeserialization", "lone surrogate") from e
    return dict(pairs)


def parse_header(prefix: bytes, file_len: int) -> Header:
    """Parses and validates a header; `prefix` is the file's first bytes (at
    least 8 + N of them, or the whole file if it is shorter)."""
    if file_len < 8 or len(prefix) < 8:
        raise SafetensorsError("HeaderTooSmall", "file shorter than the 8-byte header length")
    n = struct.unpack("<Q", prefix[:8])[0]
    if n > MAX_HEADER:
        raise SafetensorsError("HeaderTooLarge", f"header length {n} exceeds {MAX_HEADER}")
    if 8 + n > file_len or 8 + n > len(prefix):
        raise SafetensorsError("InvalidHeaderLength", f"header length {n} runs past the end of the file")
    try:
        text = bytes(prefix[8:8 + n]).decode("utf-8", errors="strict")
    except UnicodeDecodeError as e:
        raise SafetensorsError("InvalidHeader", "header is not UTF-8") from e
    if not text.startswith("{"):
        raise SafetensorsError("InvalidHeaderStart", "header does not start with '{'")

    def bad_const(c):
        raise SafetensorsError("InvalidHeaderDeserialization", f"non-JSON constant {c}")

    try:
        doc = json.loads(text, object_pairs_hook=_object, parse_constant=bad_const)
    except json.JSONDecodeError as e:
        raise SafetensorsError("InvalidHeaderDeserialization", str(e)) from e
    except RecursionError as e:
        raise SafetensorsError("InvalidHeaderDeserialization", "nested too deeply") from e
    if not isinstance(doc, dict):
        raise SafetensorsError("InvalidHeaderDeserialization", "header is not a JSON object")
    meta: Dict[str, str] = {}
    tensors: List[TensorInfo] = []
    for name, info in doc.items():
        if name == "__metadata__":
            if info is None:
                continue
            if not isinstance(info, dict) or not all(isinstance(v, str) for v in info.values()):
                raise SafetensorsError("InvalidHeaderDeserialization", "__metadata__ must map strings to strings")
            meta = dict(info)
            continue
        if not isinstance(info, dict) or not {"dtype", "shape", "data_offsets"} <= set(info):
            raise SafetensorsError("InvalidHeaderDeserialization", f"tensor {name!r}: missing fields")
        dtype, shape, offs = info["dtype"], info["shape"], info["data_offsets"]
        if not isinstance(dtype, str) or dtype not in DTYPE_SIZES:
            raise SafetensorsError("InvalidHeaderDeserialization", f"tensor {name!r}: unknown dtype {dtype!r}")
        if not isinstance(shape, list) or not all(_is_uint(d) for d in shape):
            raise SafetensorsError("InvalidHeaderDeserialization", f"tensor {name!r}: bad shape")
        if not isinstance(offs, list) or len(offs) != 2 or not all(_is_uint(o) for o in offs):
            raise SafetensorsError("InvalidHeaderDeserialization", f"tensor {name!r}: bad data_offsets")
        tensors.append(TensorInfo(name, dtype, tuple(shape), offs[0], offs[1]))
    tensors.sort(key=lambda t: (t.begin, t.end))  # stable, as the crate's sort_by
    start = 0
    for t in tensors:
        if t.begin != start or t.end < t.begin:
            raise SafetensorsError("InvalidOffset", f"tensor {t.name!r} has invalid offsets")
        start = t.end
        nel = 1
        for d in t.shape:
            nel *= d
            if nel >= 1 << 64:
                raise SafetensorsError("ValidationOverflow", f"tensor {t.name!r}: shape overflows")
        nbytes = nel * DTYPE_SIZES[t.dtype]
        if nbytes >= 1 << 64:
            raise SafetensorsError("ValidationOverflow", f"tensor {t.name!r}: byte size overflows")
        if t.end - t.begin != nbytes:
            raise SafetensorsError("TensorInvalidInfo", f"tensor {t.name!r}: {t.end - t.begin} bytes for {nbytes}")
    if start + 8 + n != file_len:
        raise SafetensorsError("MetadataIncompleteBuffer",
                               f"data section of {file_len - 8 - n} bytes, tensors cover {start}")
    return Header(n, tensors, meta)


def read_header(path: str) -> Header:
    with open(path, "rb") as f:
        file_len = os.fstat(f.fileno()).st_size
        head = f.read(8)
        if len(head) == 8:
            n = struct.unpack("<Q", head)[0]
            if n <= MAX_HEADER:
                head += f.read(min(n, file_len - 8))
    return parse_header(head, file_len)


# ------------------------------------------------------------------ loading
@dataclass
class LayerWeights:  # src/lib.rs:62-69
    gqkv_proj: torch.Tensor
    o_proj: torch.Tensor
    gate_proj: torch.Tensor
    up_proj: torch.Tensor
    down_proj: torch.Tensor


@dataclass
class ModelWeights:  # src/lib.rs:72-83
    h_module: List[LayerWeights]
    l_module: List[LayerWeights]
    embed_tokens: torch.Tensor
    lm_head: torch.Tensor
    z_l_init: torch.Tensor


@dataclass
class _Piece:
    off: int      # file offset
    nbytes: int   # whole elements
    esize: int
    dtype: int    # ABI dtype
    dst: int      # device address of the first destination element


def _plan_chunks(pieces: List[_Piece], cap: int) -> List[Tuple[int, int, List[_Piece]]]:
    """Groups file-contiguous pieces into chunks of at most cap bytes, cutting
    a piece at whole elements where it crosses a chunk's end."""
    chunks: List[Tuple[int, int, List[_Piece]]] = []
    for p in sorted(pieces, key=lambda p: p.off):
        off, left, dst = p.off, p.nbytes, p.dst
        while left > 0:
            if not chunks or chunks[-1][0] + chunks[-1][1] != off or cap - chunks[-1][1] < p.esize:
                chunks.append((off, 0, []))
            c0, cb, parts = chunks[-1]
            take = min(left, (cap - cb) // p.esize * p.esize)
            parts.append(_Piece(off, take, p.esize, p.dtype, dst))
            chunks[-1] = (c0, cb + take, parts)
            off, left, dst = off + take, left - take, dst + take // p.esize * 2
    return chunks


def load_safetensors(path: str, n_layers: int, hidden_size: int, intermediate_size: int,
                     device=None, chunk_bytes: int = 128 << 20, reader_threads: Optional[int] = None,
                     stream: Optional[torch.cuda.Stream] = None) -> ModelWeights:
    """The model's bf16 weights from one safetensors file, with the reference's
    tensor names and rules (see HrmLayerOps::load_safetensors in the C++ host
    layer): per module and layer gqkv_proj, o_proj, gate_up_proj split at
    intermediate x hidden elements, down_proj, under ".attn." / ".mlp." when
    "model.H_module.layers.0.attn.gqkv_proj.weight" exists; then
    model.embed_tokens.weight, lm_head.weight (else model.lm_head.weight) and
    model.z_L_init.  Returns once the weights are on the device.

    Raises SafetensorsError for an invalid header and ValueError for a missing
    tensor, a gate_up smaller than its gate half, or any tensor whose dtype is
    not BF16 / F32 / F16 (the reference converts every tensor and panics)."""
    if reader_threads is None:  # page-cache reads run at a few GB/s per thread
        # one per core, at most 16: a 4.7 GB f32 file loads at 38.8 GB/s with 16
        # threads and 128 MB chunks, 30.8 with 8 and 64 MB, 22.6 with 4 (16 cores)
        reader_threads = max(1, min(16, len(os.sched_getaffinity(0))))
    hdr = read_header(path)
    for t in hdr.tensors:
        if t.dtype not in ABI_DTYPE:
            raise ValueError(f"unsupported dtype {t.dtype} of tensor {t.name}")
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    pieces: List[_Piece] = []

    def tensor(name: str) -> TensorInfo:
        t = hdr.find(name)
        if t is None:  # src/lib.rs:2011-2020
            keys = [x.name for x in hdr.tensors if "layer" in x.name or "embed" in x.name or "lm_head" in x.name]
            raise ValueError(f"missing tensor: {name}. Available keys: {keys}")
        return t

    def take(t: TensorInfo, first: int, n: int) -> torch.Tensor:
        out = torch.empty(n, dtype=torch.bfloat16, device=device)
        es = DTYPE_SIZES[t.dtype]
        if n:
            pieces.append(_Piece(hdr.data_offset + t.begin + first * es, n * es, es, ABI_DTYPE[t.dtype],
                                 out.data_ptr()))
        return out

    def whole(name: str) -> torch.Tensor:
        t = tensor(name)
        return take(t, 0, t.numel)

    attn = hdr.find("model.H_module.layers.0.attn.gqkv_proj.weight") is not None  # src/lib.rs:2043-2044
    a, m = (".attn", ".mlp") if attn else ("", "")

    def module(prefix: str) -> List[LayerWeights]:
        layers = []
        for i in range(n_layers):
            p = f"{prefix}.{i}"
            gqkv, o = whole(f"{p}{a}.gqkv_proj.weight"), whole(f"{p}{a}.o_proj.weight")
            gu = tensor(f"{p}{m}.gate_up_proj.weight")
            split = intermediate_size * hidden_size  # src/lib.rs:2072-2078
            if gu.numel < split:
                raise ValueError(f"{gu.name}: {gu.numel} elements, fewer than intermediate x hidden")
            gate, up = take(gu, 0, split), take(gu, split, gu.numel - split)
            layers.append(LayerWeights(gqkv, o, gate, up, whole(f"{p}{m}.down_proj.weight")))
        return layers

    w = ModelWeights(module("model.H_module.layers"), module("model.L_module.layers"),
                     whole("model.embed_tokens.weight"),
                     whole("lm_head.weight" if hdr.find("lm_head.weight") else "model.lm_head.weight"),
                     whole("model.z_L_init"))
    _upload(path, _plan_chunks(pieces, max(64, chunk_bytes // 16 * 16)), device, chunk_bytes, reader_threads, stream)
    return w


def _upload(path, chunks, device, chunk_bytes, reader_threads, stream):
    if not chunks:
        return
    ring = 3
    cap = max(c[1] for c in chunks)
    host = [torch.empty(cap, dtype=torch.uint8, pin_memory=True) for _ in range(min(ring, len(chunks)))]
    staging_bytes = min(cap, 32 << 20) // 16 * 16 or 16
    staging = torch.empty(staging_bytes, dtype=torch.uint8, device=device)
    events: List[Optional[torch.cuda.Event]] = [None] * len(host)
    s = stream if stream is not None else torch.cuda.current_stream(device)
    fd = os.open(path, os.O_RDONLY)
    try:
        with ThreadPoolExecutor(max_workers=max(1, reader_threads)) as pool, torch.cuda.device(device):
            for ci, (off, nbytes, parts) in enumerate(chunks):
                r = ci % len(host)
                if events[r] is not None:
                    events[r].synchronize()  # the slot's copies are done
                view = memoryview(host[r].numpy())
                per = -(-nbytes // max(1, reader_threads))
                jobs = [pool.submit(_pread_into, fd, view[b0:min(nbytes, b0 + per)], off + b0)
                        for b0 in range(0, nbytes, per)]
                for j in jobs:
                    j.result()
                base = host[r].data_ptr()
                for p in parts:
                    call("hrm_upload_to_bf16", ctypes.c_void_p(base + p.off - off), p.dtype, ctypes.c_void_p(p.dst),
                         p.nbytes // p.esize, ctypes.c_void_p(staging.data_ptr()), staging_bytes,
                         ctypes.c_void_p(s.cuda_stream))
                ev = torch.cuda.Event()
                ev.record(s)
                events[r] = ev
    finally:
        # Also on an error: the pinned buffers go back to torch's allocator,
        # which does not know that copies queued through the C ABI read them.
        s.synchronize()
        os.close(fd)


def _pread_into(fd: int, view: memoryview, off: int) -> None:
    done = 0
    while done < len(view):
        got = os.preadv(fd, [view[done:]], off + done)
        if got <= 0:
            raise OSError(f"short read at offset {off + done}")
        done += got
