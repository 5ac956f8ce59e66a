"""Test-only Python access to the checker (never imported by the product).

* `Oracle`: numpy front end of liboracle.so, the CPU restatement of the
  reference kernels (hrm_oracle.c).  bf16 arrays are numpy uint16 bit patterns.
* `RefKernels`: the reference's own src/kernels/*.cu, compiled from source for
  sm_100a into _ref/libref_kernels.so (or, as the reference ships them, as
  compute_80 PTX that the driver compiles at load time, _ref/libref_kernels_ptx.so)
  and launched with the reference's launch configurations (ref_launch.cu);
  takes torch CUDA tensors.
* numpy helpers for bf16 conversion and ulp measurement used by the tests.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libref_kernels.so")
# The same kernels as the reference ships them: compute_80 PTX, compiled by the
# driver for the GPU when the library loads.
REF_LIB_PTX = os.path.join(HERE, "_ref", "libref_kernels_ptx.so")

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_f32 = ctypes.c_float


def build() -> None:
    """Builds liboracle.so (and _ref/ where the reference checkout exists)."""
    subprocess.run(["make", "-C", HERE, "-s"], check=True)


# ---------------------------------------------------------------- bf16 numpy
def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits (NaN -> 0x7fff)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FFF
    return r


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_ulp(x: np.ndarray) -> np.ndarray:
    """Spacing of bf16 values at |x| (7 stored mantissa bits); subnormal floor."""
    a = np.abs(np.asarray(x, dtype=np.float64))
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -126)))
    return np.exp2(e - 7)


def ulp_error(got_bits: np.ndarray, want_bits: np.ndarray, magnitude: np.ndarray | None = None) -> np.ndarray:
    """|got - want| in bf16 ulps measured at `magnitude` (default |want|).

    Identical bit patterns (including NaN and +-inf pairs) count as 0.
    """
    g = bf16_to_f32(got_bits).astype(np.float64)
    w = bf16_to_f32(want_bits).astype(np.float64)
    mag = np.abs(w) if magnitude is None else np.abs(magnitude)
    same = (np.asarray(got_bits) == np.asarray(want_bits)) | (np.isnan(g) & np.isnan(w))
    with np.errstate(invalid="ignore"):
        err = np.abs(g - w) / bf16_ulp(mag)
    err[same] = 0.0
    err[~same & ~np.isfinite(err)] = np.inf
    return err


# -------------------------------------------------------------------- oracle
class Oracle:
    SIGS = {
        "ora_additive_inject": [_p, _p, _p, _i64],
        "ora_swiglu_ffn": [_p, _p, _p, _i64],
        "ora_rms_norm": [_p, _p, _p, _i64, _i64, _f32],
        "ora_rms_norm_f32": [_p, _p, _p, _i64, _i64, _f32],
        "ora_add_rms_norm": [_p, _p, _p, _p, _p, _i64, _i64, _f32],
        "ora_embedding_lookup": [_p, _p, _p, _i64, _i64, _i64, _f32],
        "ora_embed_rms_norm": [_p, _p, _p, _p, _p, _i64, _i64, _i64, _f32, _f32],
        "ora_rope_table": [_p, _i64, _i64, _f32],
        "ora_rope_embed": [_p, _p, _i64, _i64, _i64, _i64, _i64, _f32, _p],
        "ora_split_gqkv": [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64],
        "ora_kv_cache_update": [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, ctypes.c_int],
        "ora_gated_attn_output": [_p, _p, _p, _i64],
        "ora_broadcast_vec": [_p, _p, _i64, _i64],
        "ora_convert_to_bf16": [_p, ctypes.c_int, _p, _i64],
        "ora_set_threads": [ctypes.c_int],
        "ora_rope_embed_token_major": [_p, _p, _i64, _i64, _i64, _i64, _i64, _f32, _p],
        "ora_fill_normal_bf16": [_p, _i64, ctypes.c_uint64, ctypes.c_uint64, _i64, ctypes.c_double,
                                 ctypes.c_double],
        "ora_fill_ids": [_p, _i64, ctypes.c_uint64, ctypes.c_uint64, _i64, ctypes.c_uint32],
    }

    def __init__(self, path: str = ORACLE_LIB):
        if not os.path.exists(path):
            build()
        self.lib = ctypes.CDLL(path)
        for name, args in self.SIGS.items():
            getattr(self.lib, name).argtypes = args
            getattr(self.lib, name).restype = None
        self.lib.ora_max_threads.restype = ctypes.c_int

    @staticmethod
    def _ptr(a):
        return None if a is None else a.ctypes.data_as(_p)

    @staticmethod
    def _c(a, dtype):
        return None if a is None else np.ascontiguousarray(a, dtype=dtype)

    def max_threads(self) -> int:
        return self.lib.ora_max_threads()

    def set_threads(self, n: int) -> None:
        self.lib.ora_set_threads(n)

    def additive_inject(self, a, b):
        a, b = self._c(a, np.uint16), self._c(b, np.uint16)
        out = np.empty_like(a)
        self.lib.ora_additive_inject(self._ptr(a), self._ptr(b), self._ptr(out), a.size)
        return out

    def swiglu_ffn(self, g, u):
        g, u = self._c(g, np.uint16), self._c(u, np.uint16)
        out = np.empty_like(g)
        self.lib.ora_swiglu_ffn(self._ptr(g), self._ptr(u), self._ptr(out), g.size)
        return out

    def rms_norm(self, x, w=None, eps=1e-6):
        x, w = self._c(x, np.uint16), self._c(w, np.uint16)
        hidden = x.shape[-1]
        y = np.empty_like(x)
        self.lib.ora_rms_norm(self._ptr(x), self._ptr(y), self._ptr(w), x.size // hidden, hidden, eps)
        return y

    def rms_norm_f32(self, x, w=None, eps=1e-6):
        x, w = self._c(x, np.float32), self._c(w, np.float32)
        hidden = x.shape[-1]
        y = np.empty_like(x)
        self.lib.ora_rms_norm_f32(self._ptr(x), self._ptr(y), self._ptr(w), x.size // hidden, hidden, eps)
        return y

    def add_rms_norm(self, x, b, w=None, eps=1e-6):
        x, b, w = self._c(x, np.uint16), self._c(b, np.uint16), self._c(w, np.uint16)
        hidden = x.shape[-1]
        r, y = np.empty_like(x), np.empty_like(x)
        self.lib.ora_add_rms_norm(self._ptr(x), self._ptr(b), self._ptr(r), self._ptr(y), self._ptr(w),
                                  x.size // hidden, hidden, eps)
        return r, y

    def embedding_lookup(self, ids, table, scale):
        ids, table = self._c(ids, np.uint32), self._c(table, np.uint16)
        vocab, hidden = table.shape
        out = np.empty((*ids.shape, hidden), dtype=np.uint16)
        self.lib.ora_embedding_lookup(self._ptr(ids), self._ptr(table), self._ptr(out), ids.size, hidden, vocab,
                                      scale)
        return out

    def embed_rms_norm(self, ids, table, scale, w=None, eps=1e-6):
        ids, table, w = self._c(ids, np.uint32), self._c(table, np.uint16), self._c(w, np.uint16)
        vocab, hidden = table.shape
        h = np.empty((*ids.shape, hidden), dtype=np.uint16)
        y = np.empty_like(h)
        self.lib.ora_embed_rms_norm(self._ptr(ids), self._ptr(table), self._ptr(h), self._ptr(y), self._ptr(w),
                                    ids.size, hidden, vocab, scale, eps)
        return h, y

    def rope_table(self, positions, head_dim, theta=10000.0):
        t = np.empty((positions, head_dim), dtype=np.float32)
        self.lib.ora_rope_table(self._ptr(t), positions, head_dim, theta)
        return t

    def rope_embed(self, q, k, offset=0, theta=10000.0, table=None):
        """Returns rotated copies of q, k ([B, H, S, D] uint16)."""
        q, k = (np.array(a, dtype=np.uint16, order="C", copy=True) for a in (q, k))
        table = self._c(table, np.float32)
        b, h, s, d = q.shape
        self.lib.ora_rope_embed(self._ptr(q), self._ptr(k), b, h, s, d, offset, theta, self._ptr(table))
        return q, k

    def rope_embed_token_major(self, q, k, offset=0, theta=10000.0, table=None):
        """Returns rotated copies of q, k ([B, S, H, D] uint16)."""
        q, k = (np.array(a, dtype=np.uint16, order="C", copy=True) for a in (q, k))
        table = self._c(table, np.float32)
        b, s, h, d = q.shape
        self.lib.ora_rope_embed_token_major(self._ptr(q), self._ptr(k), b, s, h, d, offset, theta,
                                            self._ptr(table))
        return q, k

    def fill_normal_bf16(self, out, seed, tag, start=0, std=1.0, mean=0.0):
        """Fills the contiguous uint16 array `out` with elements [start, start + out.size)
        of the counter-based (seed, tag) normal stream, as bf16 bits."""
        assert out.dtype == np.uint16 and out.flags.c_contiguous
        self.lib.ora_fill_normal_bf16(self._ptr(out), out.size, seed, tag, start, std, mean)
        return out

    def fill_ids(self, out, seed, tag, vocab, start=0):
        """Fills the contiguous uint32 array `out` with ids [start, start + out.size) of the stream."""
        assert out.dtype == np.uint32 and out.flags.c_contiguous
        self.lib.ora_fill_ids(self._ptr(out), out.size, seed, tag, start, vocab)
        return out


    def gated_attn_output(self, gate, attn):
        gate, attn = self._c(gate, np.uint16), self._c(attn, np.uint16)
        out = np.empty_like(attn)
        self.lib.ora_gated_attn_output(self._ptr(gate), self._ptr(attn), self._ptr(out), attn.size)
        return out

    def broadcast_vec(self, src, n_copies):
        src = self._c(src, np.uint16)
        out = np.empty((n_copies, src.size), np.uint16)
        self.lib.ora_broadcast_vec(self._ptr(out), self._ptr(src), n_copies, src.size)
        return out

    DTYPES = {"bf16": 0, "f32": 1, "f16": 2}

    def convert_to_bf16(self, raw: bytes, dtype: str):
        """raw little-endian bytes of a checkpoint tensor -> bf16 bits."""
        size = 4 if dtype == "f32" else 2
        buf = np.frombuffer(raw, np.uint8)
        n = buf.size // size
        out = np.empty(n, np.uint16)
        self.lib.ora_convert_to_bf16(buf.ctypes.data_as(_p), self.DTYPES[dtype], self._ptr(out), n)
        return out

    def split_gqkv(self, gqkv, batch, seq, heads, head_dim):
        gqkv = self._c(gqkv, np.uint16)
        gate = np.empty((batch, seq, heads, head_dim), np.uint16)
        q, k, v = (np.empty((batch, heads, seq, head_dim), np.uint16) for _ in range(3))
        self.lib.ora_split_gqkv(self._ptr(gqkv), self._ptr(gate), self._ptr(q), self._ptr(k), self._ptr(v), batch,
                                seq, heads, head_dim)
        return gate, q, k, v

    def kv_cache_update(self, k, v, k_cache, v_cache, cached_len, is_decode):
        """Writes into copies of the caches and returns them."""
        k, v = self._c(k, np.uint16), self._c(v, np.uint16)
        kc, vc = (np.array(a, np.uint16, order="C", copy=True) for a in (k_cache, v_cache))
        b, h, s, d = k.shape
        self.lib.ora_kv_cache_update(self._ptr(k), self._ptr(v), self._ptr(kc), self._ptr(vc), b, h, s, d,
                                     kc.shape[2], cached_len, int(is_decode))
        return kc, vc

    def split_gqkv_rope(self, gqkv, batch, seq, heads, head_dim, offset, theta=10000.0, table=None,
                        k_cache=None, v_cache=None, cache_offset=0):
        """The reference's attention prologue: split -> rope -> kv_cache_update."""
        gate, q, k, v = self.split_gqkv(gqkv, batch, seq, heads, head_dim)
        q, k = self.rope_embed(q, k, offset, theta, table)
        kc = vc = None
        if k_cache is not None:
            # the reference writes at s (prefill, offset 0) or cached_len + s (decode)
            kc, vc = self.kv_cache_update(k, v, k_cache, v_cache, cache_offset, True)
        return gate, q, k, v, kc, vc


# ------------------------------------------------- reference kernels (GPU)
class RefKernels:
    """The reference's kernels, built from its sources; torch CUDA tensors in."""

    SIGS = {
        "ref_additive_inject": [_p, _p, _p, _i64, _p],
        "ref_rms_norm": [_p, _p, _i64, _i64, _f32, _p],
        "ref_rope_embed": [_p, _p, _i64, _i64, _i64, _i64, _i64, _f32, _p],
        "ref_swiglu_ffn": [_p, _p, _p, _i64, _p],
        "ref_embedding_lookup": [_p, _p, _p, _i64, _i64, _i64, _i64, _f32, _p],
        "ref_split_gqkv": [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _p],
        "ref_kv_cache_update": [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, ctypes.c_int, _p],
        "ref_apply_attn_gate": [_p, _p, _i64, _p],
        "ref_gated_attn_output": [_p, _p, _p, _i64, _p],
        "ref_broadcast_vec": [_p, _p, _i64, _i64, _p],
    }

    def __init__(self, path: str = REF_LIB):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not built (needs the reference checkout at build time)")
        self.lib = ctypes.CDLL(path)
        for name, args in self.SIGS.items():
            getattr(self.lib, name).argtypes = args
            getattr(self.lib, name).restype = ctypes.c_int

    @staticmethod
    def available(path: str = REF_LIB) -> bool:
        return os.path.exists(path)

    def _run(self, name, *args):
        import torch

        st = _p(torch.cuda.current_stream().cuda_stream)
        rc = getattr(self.lib, name)(*args, st)
        if rc != 0:
            raise RuntimeError(f"{name}: cudaError {rc}")

    def additive_inject(self, a, b, out):
        self._run("ref_additive_inject", _p(a.data_ptr()), _p(b.data_ptr()), _p(out.data_ptr()), a.numel())

    def swiglu_ffn(self, g, u, out):
        self._run("ref_swiglu_ffn", _p(g.data_ptr()), _p(u.data_ptr()), _p(out.data_ptr()), g.numel())

    def rms_norm(self, x, y, eps):
        hidden = x.shape[-1]
        self._run("ref_rms_norm", _p(x.data_ptr()), _p(y.data_ptr()), x.numel() // hidden, hidden, eps)

    def rope_embed(self, q, k, offset, theta):
        b, h, s, d = q.shape
        self._run("ref_rope_embed", _p(q.data_ptr()), _p(k.data_ptr()), b, h, s, d, offset, theta)

    def embedding_lookup(self, ids, table, out, scale):
        vocab, hidden = table.shape
        self._run("ref_embedding_lookup", _p(ids.data_ptr()), _p(table.data_ptr()), _p(out.data_ptr()), 1,
                  ids.numel(), hidden, vocab, scale)

    def split_gqkv(self, gqkv, gate, q, k, v):
        b, h, s, d = q.shape
        self._run("ref_split_gqkv", _p(gqkv.data_ptr()), _p(gate.data_ptr()), _p(q.data_ptr()), _p(k.data_ptr()),
                  _p(v.data_ptr()), b, s, h, d)

    def kv_cache_update(self, k, v, k_cache, v_cache, cached_len, is_decode):
        b, h, s, d = k.shape
        self._run("ref_kv_cache_update", _p(k.data_ptr()), _p(v.data_ptr()), _p(k_cache.data_ptr()),
                  _p(v_cache.data_ptr()), b, h, s, d, k_cache.shape[2], cached_len, int(is_decode))

    def apply_attn_gate(self, gate, attn):
        self._run("ref_apply_attn_gate", _p(gate.data_ptr()), _p(attn.data_ptr()), attn.numel())

    def gated_attn_output(self, gate, attn, out):
        self._run("ref_gated_attn_output", _p(gate.data_ptr()), _p(attn.data_ptr()), _p(out.data_ptr()),
                  attn.numel())

    def broadcast_vec(self, dst, src):
        self._run("ref_broadcast_vec", _p(dst.data_ptr()), _p(src.data_ptr()), dst.shape[0], src.numel())
