"""Writes the synthetic safetensors checkpoints the loader tests read.

    python tests/golden/make_checkpoint.py

Two files of a tiny HRM model (2 layers per module, hidden 32, intermediate 48,
vocab 20), laid out in the safetensors format -- an 8-byte little-endian
header length, a JSON header padded with spaces to a multiple of 8 bytes, then
the tensors' bytes back to back:

* ckpt_tiny_attn.safetensors: the ".attn." / ".mlp." tensor names, lm_head at
  "lm_head.weight", tensors in f32, bf16 and f16 mixed, an unused bf16 tensor
  of odd length placed so that later f32 tensors start at byte offsets that
  are not multiples of 4, special values (NaN payloads, infinities,
  denormals, rounding ties) in the f32 and f16 tensors, a __metadata__ entry,
  and JSON keys written in an order unlike the data order;
* ckpt_tiny_flat.safetensors: the flat names, lm_head at
  "model.lm_head.weight", bf16 and f16.

The values come from a seeded numpy generator; the files are written here,
not by a safetensors library, so that the odd offsets are under control (the
tests also read them back with the safetensors package where it is
installed).
"""

import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LAYERS, HIDDEN, INTER, VOCAB = 2, 32, 48, 20


def f32_to_bf16_bits(x):
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def raw(dtype, values):
    """Little-endian bytes of `values` (float64 array) stored as dtype."""
    if dtype == "F32":
        return np.asarray(values, np.float32).astype("<f4").tobytes()
    if dtype == "F16":
        return np.asarray(values, np.float16).astype("<f2").tobytes()
    return f32_to_bf16_bits(np.asarray(values, np.float32)).astype("<u2").tobytes()


F32_SPECIALS = np.array([0x7F812345, 0xFFC00001, 0x7F800000, 0xFF800000, 0x00000001, 0x807FFFFF, 0x7F7FFFFF,
                         0x3F808000, 0x3F818000, 0x3F808001, 0x00000000, 0x80000000], np.uint32)
F16_SPECIALS = np.array([0x7C00, 0xFC00, 0xFE01, 0x7D55, 0x0001, 0x83FF, 0x7BFF, 0x8000], np.uint16)


def with_specials(dtype, data):
    b = bytearray(data)
    if dtype == "F32":
        b[:F32_SPECIALS.nbytes] = F32_SPECIALS.astype("<u4").tobytes()
    elif dtype == "F16":
        b[:F16_SPECIALS.nbytes] = F16_SPECIALS.astype("<u2").tobytes()
    return bytes(b)


def layer_tensors(prefix, attn):
    a, m = (".attn", ".mlp") if attn else ("", "")
    out = []
    for i in range(LAYERS):
        out += [(f"{prefix}.{i}{a}.gqkv_proj.weight", (4 * HIDDEN, HIDDEN)),
                (f"{prefix}.{i}{a}.o_proj.weight", (HIDDEN, HIDDEN)),
                (f"{prefix}.{i}{m}.gate_up_proj.weight", (2 * INTER, HIDDEN)),
                (f"{prefix}.{i}{m}.down_proj.weight", (HIDDEN, INTER))]
    return out


def write(path, entries, metadata, key_order_seed):
    """entries: (name, dtype, shape, bytes) in data order."""
    header, off = {}, 0
    for name, dtype, shape, data in entries:
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(data)]}
        off += len(data)
    keys = list(header)
    np.random.default_rng(key_order_seed).shuffle(keys)
    doc = {k: header[k] for k in keys}
    if metadata is not None:
        doc = {"__metadata__": metadata, **doc}
    text = json.dumps(doc, separators=(",", ":")).encode()
    text += b" " * (-len(text) % 8)
    with open(path, "wb") as f:
        f.write(len(text).to_bytes(8, "little"))
        f.write(text)
        for _, _, _, data in entries:
            f.write(data)


def main():
    rng = np.random.default_rng(2024)

    def values(shape, std):
        return rng.standard_normal(int(np.prod(shape))) * std

    # --- attn-prefix file: mixed dtypes, odd offsets, specials
    dtypes = ["F32", "BF16", "F16"]
    entries = [("model.extra.odd_bias", "BF16", (3,), raw("BF16", values((3,), 1.0)))]  # 6 bytes: f32 after it sits at 2 mod 4
    for j, (name, shape) in enumerate(layer_tensors("model.H_module.layers", True) +
                                      layer_tensors("model.L_module.layers", True)):
        dt = dtypes[j % 3]
        entries.append((name, dt, shape, with_specials(dt, raw(dt, values(shape, 0.02)))))
        if j == 4:  # another odd-length bf16 tensor shifts the offsets again
            entries.append(("model.extra.odd_scale", "BF16", (1,), raw("BF16", [0.5])))
    entries += [("model.embed_tokens.weight", "BF16", (VOCAB, HIDDEN), raw("BF16", values((VOCAB, HIDDEN), 0.02))),
                ("lm_head.weight", "F16", (VOCAB, HIDDEN), with_specials("F16", raw("F16", values((VOCAB, HIDDEN), 0.02)))),
                ("model.z_L_init", "F32", (HIDDEN,), with_specials("F32", raw("F32", values((HIDDEN,), 1.0))))]
    write(os.path.join(HERE, "ckpt_tiny_attn.safetensors"), entries, {"format": "pt", "note": "synthetic"}, 1)

    # --- flat-name file: bf16 and f16, lm_head under model.
    entries = []
    for j, (name, shape) in enumerate(layer_tensors("model.H_module.layers", False) +
                                      layer_tensors("model.L_module.layers", False)):
        dt = "F16" if j % 5 == 0 else "BF16"
        entries.append((name, dt, shape, raw(dt, values(shape, 0.02))))
    entries += [("model.z_L_init", "BF16", (HIDDEN,), raw("BF16", values((HIDDEN,), 1.0))),
                ("model.embed_tokens.weight", "BF16", (VOCAB, HIDDEN), raw("BF16", values((VOCAB, HIDDEN), 0.02))),
                ("model.lm_head.weight", "BF16", (VOCAB, HIDDEN), raw("BF16", values((VOCAB, HIDDEN), 0.02)))]
    write(os.path.join(HERE, "ckpt_tiny_flat.safetensors"), entries, None, 2)


if __name__ == "__main__":
    main()
