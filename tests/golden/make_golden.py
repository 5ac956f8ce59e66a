"""Writes the golden fixtures under tests/golden/.

1. reference_kats.json -- the reference's own known-answer GPU tests
   (src/lib.rs:2225-2279), restated as data: inputs, expected values and the
   tolerance the reference used (0.01).  The reference has no known answers
   for rope_embed or embedding_lookup; the derived known answers for those
   are stated in the tests.

2. ref_kernels_*.npz (`--from-reference`, needs a GPU and the reference
   kernels built from source into oracle/_ref/) -- seeded inputs and the
   outputs of the reference's own kernels, launched exactly as its wrappers
   launch them.  The CPU suite checks the oracle against these, which pins
   the oracle to the reference itself.

Run from the repo root:  python tests/golden/make_golden.py [--from-reference]
"""

import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

KATS = {
    "source": "ArjavDesa912/hrm-text-cuda src/lib.rs:2225-2279",
    "tolerance": 0.01,
    "tests": {
        # src/lib.rs:2227-2243
        "additive_inject": {"a": [1.0, 2.0, 3.0, 4.0], "b": [0.5, 1.5, 2.5, 3.5],
                            "expected": [1.5, 3.5, 5.5, 7.5]},
        # src/lib.rs:2247-2261: rows 1, hidden 4, expected x / (sqrt(30) / 2)
        "rms_norm": {"x": [1.0, 2.0, 3.0, 4.0], "rows": 1, "hidden": 4,
                     "expected_formula": "x / (sqrt(1 + 4 + 9 + 16) / 2)"},
        # src/lib.rs:2265-2279
        "swiglu_ffn": {"gate": [0.0, 0.0, 0.0, 0.0], "up": [2.0, 2.0, 2.0, 2.0],
                       "expected": [0.0, 0.0, 0.0, 0.0]},
        # src/lib.rs:2283-2298
        "gated_attn_output": {"gate": [0.0, 0.0, 0.0, 0.0], "attn": [1.0, 1.0, 1.0, 1.0],
                              "expected": [0.5, 0.5, 0.5, 0.5]},
    },
}

# Seeded cases run through the reference kernels (small enough for the CPU
# oracle in well under a second each).
REF_CASES = {
    "rms_norm": dict(rows=32, hidden=2048, eps=1e-5),
    "rms_norm_h1536": dict(rows=48, hidden=1536, eps=1e-6),
    "rms_norm_h200": dict(rows=8, hidden=200, eps=1e-6),
    "additive_inject": dict(n=16384 + 5),
    "swiglu_ffn": dict(n=65536 + 3),
    "embedding_lookup": dict(vocab=300, hidden=2048, tokens=130, scale=45.254834),
    "rope_embed": dict(batch=1, heads=4, seq=160, head_dim=128, offset=0, theta=10000.0),
    "rope_embed_decode": dict(batch=4, heads=16, seq=1, head_dim=128, offset=4095, theta=10000.0),
    "rope_embed_hd64": dict(batch=1, heads=2, seq=77, head_dim=64, offset=3, theta=500000.0),
}


def write_kats():
    with open(os.path.join(HERE, "reference_kats.json"), "w") as f:
        json.dump(KATS, f, indent=1)


def normal_bf16(rng, shape, std=1.0):
    sys.path.insert(0, ROOT)
    from oracle import f32_to_bf16

    return f32_to_bf16((rng.standard_normal(shape) * std).astype(np.float32))


def write_reference_outputs():
    import torch

    sys.path.insert(0, ROOT)
    from oracle import RefKernels

    ref = RefKernels()
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(1234)

    def T(a):
        return torch.from_numpy(a.view(np.int16).copy()).to(dev)

    def N(t):
        return t.cpu().numpy().view(np.uint16)

    for name, c in REF_CASES.items():
        if name.startswith("rms_norm"):
            x = normal_bf16(rng, (c["rows"], c["hidden"]))
            y = torch.empty_like(T(x))
            ref.rms_norm(T(x), y, c["eps"])
            out = dict(x=x, y=N(y), eps=np.float32(c["eps"]))
        elif name == "additive_inject":
            a, b = normal_bf16(rng, c["n"]), normal_bf16(rng, c["n"])
            o = torch.empty_like(T(a))
            ref.additive_inject(T(a), T(b), o)
            out = dict(a=a, b=b, out=N(o))
        elif name == "swiglu_ffn":
            g, u = normal_bf16(rng, c["n"], 0.5), normal_bf16(rng, c["n"], 0.5)
            g[:8] = np.array([0x0000, 0x8000, 0x7F80, 0xFF80, 0x7FC0, 0x4300, 0xC300, 0x0001], np.uint16)
            o = torch.empty_like(T(g))
            ref.swiglu_ffn(T(g), T(u), o)
            out = dict(gate=g, up=u, out=N(o))
        elif name == "embedding_lookup":
            table = normal_bf16(rng, (c["vocab"], c["hidden"]), 0.02)
            ids = rng.integers(0, c["vocab"], c["tokens"], dtype=np.uint32)
            ids[:3] = [c["vocab"] - 1, c["vocab"], 0xFFFFFFFF]  # last row and two clamped ids
            o = torch.empty((c["tokens"], c["hidden"]), dtype=torch.int16, device=dev)
            ref.embedding_lookup(torch.from_numpy(ids.view(np.int32)).to(dev), T(table), o, c["scale"])
            out = dict(ids=ids, table=table, out=N(o), scale=np.float32(c["scale"]))
        else:  # rope
            shape = (c["batch"], c["heads"], c["seq"], c["head_dim"])
            q, k = normal_bf16(rng, shape), normal_bf16(rng, shape)
            tq, tk = T(q), T(k)
            ref.rope_embed(tq, tk, c["offset"], c["theta"])
            out = dict(q=q, k=k, q_out=N(tq), k_out=N(tk), offset=np.int64(c["offset"]),
                       theta=np.float32(c["theta"]))
        torch.cuda.synchronize()
        np.savez_compressed(os.path.join(HERE, f"ref_kernels_{name}.npz"), **out)
        print("wrote", name)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--from-reference", action="store_true")
    args = ap.parse_args()
    write_kats()
    if args.from_reference:
        write_reference_outputs()
