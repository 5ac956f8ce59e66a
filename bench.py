#!/usr/bin/env python
"""Throughput benchmark of the sm_100a per-token layer operators.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload chain|add_rms_norm|rms_norm_f32|rms_norm|rope|swiglu|embedding|
                                split_rope|attn_gate|convert_f32|module]

Default workload ("chain"): the chained layer-op pass on 65536 tokens per GPU
-- embedding [32000 x 2048] ~ N(0, 0.02) gathered for ids ~ U[0, 32000) and
RMSNorm'd (fused), RoPE on token-major Q/K [16, 4096, 16, 128] (tokens x 16
heads x 128; --qk-layout head for the reference's [B, 16, S, 128]) with a fp32
cos/sin table,
residual add + RMSNorm [65536 x 2048], SwiGLU [65536 x 5632] ~ 0.5 N(0, 1);
norm weights 1 + 0.1 N(0, 1), eps 1e-5, scale sqrt(2048), theta 1e4.  Inputs
are synthetic, generated on the device by a counter-based generator keyed by
(seed, tensor, global index), so rank r holds global tokens [r T, (r + 1) T)
of one job-wide tensor set.  A step is one pass over the rank's 65536
tokens; rows (tokens) are independent, so N GPUs run N disjoint shards of an
N x 65536-token job with no collective on the data path (weak scaling).

The other workloads are the single layer-op configurations (their K timed
steps replayed from a CUDA graph) and `module`, one 4-layer pass of the
layer loop's residual / norm / SwiGLU schedule.

The metric is algorithmic HBM GB/s: the bytes the pass must move per token
(70,660 B: ids, gathered rows, n1, Q/K read+write, o, r, n2, gate/up, y --
every intermediate that has to reach HBM in the fused minimum) x tokens /
time.  Every step moves 4.6 GB, far more than the 126 MB L2, so no flush is
needed between steps.

One JSON line on rank 0 carries: value (device-resident, CUDA events, max
over ranks), e2e (pinned host buffers -> device -> host through the public
API, copies overlapped with the kernels), the roofline of the dominant
kernel (SwiGLU), per-kernel times, the 64-token decode-shape latency (CUDA
graph, median of 5), the clocks sampled during the timed region and the
oracle's multithreaded CPU throughput on a bounded sample.  Under torchrun,
every rank checks its peers' heartbeats before each collective.

--impl reference times the reference's path on the CPU (the oracle: a C
restatement of the reference kernels, all host threads) on the same metric.
"""

import argparse
import json
import os
import re
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "hrm-text-cuda_b200"))

METRIC = "fused layer-op HBM GB/s (% of B200 peak) and rows/s at 1/2/4/8 GPUs"
L2_BYTES = 126 * 1000 * 1000

# chain shape (per GPU)
HIDDEN, HEADS, HEAD_DIM, INTER, VOCAB = 2048, 16, 128, 5632, 32000
CHAIN_B, CHAIN_S = 16, 4096               # 16 sequences of 4096 tokens = 65536 tokens
DECODE_B = 64                             # decode shape: 64 tokens, seq 1, offset 4095
EPS, THETA = 1e-5, 10000.0
SEED = 0                                  # seed of the counter-based chain inputs
SCALE = 45.254833995939045                # (float)sqrt(2048)

# --dims: the benchmark's 1B-class shapes (the default), or the reference's own
# default model (HrmConfig, src/lib.rs:40-60: hidden 1536, 12 heads of 128,
# intermediate 4096, vocab 65536, embedding scale sqrt(1536)).
DIMS = {
    "bench": dict(HIDDEN=2048, HEADS=16, HEAD_DIM=128, INTER=5632, VOCAB=32000, SCALE=45.254833995939045),
    "hrm-text-1b": dict(HIDDEN=1536, HEADS=12, HEAD_DIM=128, INTER=4096, VOCAB=65536, SCALE=39.191835884530846),
}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="chain",
                    choices=["chain", "add_rms_norm", "rms_norm_f32", "rms_norm", "rope", "swiglu", "embedding",
                             "split_rope", "attn_gate", "convert_f32", "module", "load_checkpoint"])
    ap.add_argument("--tokens", type=int, default=CHAIN_B * CHAIN_S,
                    help="chain tokens per GPU (a multiple of 4096; default 65536)")
    ap.add_argument("--qk-layout", choices=["token", "head"], default="token",
                    help="chain Q/K layout: token-major [B, S, 16, 128] or head-major [B, 16, S, 128]")
    ap.add_argument("--chunk-tokens", type=int, default=4096, help="e2e pipeline chunk (token-major Q/K)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-oracle baseline leg")
    ap.add_argument("--ckpt", default=None, help="load_checkpoint: an existing safetensors file of the "
                    "reference model's shapes (default: a synthetic one written for the run)")
    ap.add_argument("--dims", choices=sorted(DIMS), default="bench",
                    help="chain / module shapes: the benchmark's (default) or the reference's default model")
    args = ap.parse_args()
    if args.dims != "bench" and args.workload not in ("chain", "module"):
        ap.error("--dims applies to the chain and module workloads")
    globals().update(DIMS[args.dims])
    return args


def chain_bytes_per_token(hidden, heads, head_dim, inter):
    """Bytes each chain kernel must move per token (the gathered table row, not
    the table; weights and the rope table are L2-resident constants).
    'minimal' is the whole pass with every intermediate kept on chip: ids + row
    + n1 + Q/K read and written + o + r + n2 + gate/up + y.  The library's
    hrm_layer_ops.chain.algorithmic_bytes_per_token states the same counts
    (a CPU test keeps the two equal); it is restated here so that the
    reference arm imports nothing of the library."""
    row, qk = 2 * hidden, 2 * heads * head_dim
    per = {
        "embed_rms_norm": 4 + row + row + row,   # id, table row, h, n1
        "rope_embed": 2 * qk + 2 * qk,           # Q, K read and written
        "add_rms_norm": 4 * row,                 # h, o read; r, n2 written
        "swiglu_ffn": 3 * 2 * inter,             # gate, up read; y written
    }
    per["op_sum"] = sum(per[k] for k in CHAIN_KERNEL_NAMES)
    per["minimal"] = 4 + row + row + 4 * qk + row + row + row + 2 * 2 * inter + 2 * inter
    return per


CHAIN_KERNEL_NAMES = ("embed_rms_norm", "rope_embed", "add_rms_norm", "swiglu_ffn")


def chain_qk_shape(tokens, token_major):
    batch = tokens // CHAIN_S
    return (batch, CHAIN_S, HEADS, HEAD_DIM) if token_major else (batch, HEADS, CHAIN_S, HEAD_DIM)


def chain_config(tokens, token_major, world):
    """The chain workload's `config`, the same dict on both arms."""
    per = chain_bytes_per_token(HIDDEN, HEADS, HEAD_DIM, INTER)
    return {"workload": "chain: embed+RMSNorm -> RoPE -> add+RMSNorm -> SwiGLU",
            "dims": "hrm-text-1b" if HIDDEN == 1536 else "bench",
            "tokens_per_gpu": tokens, "hidden": HIDDEN, "heads": HEADS, "head_dim": HEAD_DIM,
            "intermediate": INTER, "vocab": VOCAB, "qk_shape": list(chain_qk_shape(tokens, token_major)),
            "qk_layout": "token-major [B, S, heads, head_dim]" if token_major
            else "head-major [B, heads, S, head_dim]",
            "bytes_per_token_minimal": per["minimal"], "bytes_per_token_moved": per["op_sum"],
            "l2": f"inputs larger than L2 ({per['op_sum'] * tokens / 1e9:.1f} GB moved per step vs 126 MB L2); "
                  "no flush",
            "parallelism": f"{world} row shards, no collective"}


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def load_traffic(kernel, workload):
    """dram bytes per launch from the committed ncu summary, if one exists."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.txt")
    try:
        text = open(path).read()
    except OSError:
        return None
    m = re.search(rf"^{workload}\s+{kernel}\s+dram_bytes_per_launch=(\d+)", text, re.M)
    return int(m.group(1)) if m else None


# --------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons via NVML while running."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, torch_device):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            import torch

            uuid = str(torch.cuda.get_device_properties(torch_device).uuid)
            self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.nvml = pynvml
        except Exception as e:  # noqa: BLE001 - clocks are reported as unavailable
            self.nvml, self.error = None, f"{type(e).__name__}: {e}"

    def _run(self):
        n = self.nvml
        while not self._stop.is_set():
            try:
                self.samples.append(n.nvmlDeviceGetClockInfo(self.h, n.NVML_CLOCK_SM))
                get = getattr(n, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    n.nvmlDeviceGetCurrentClocksThrottleReasons
                bits = get(self.h)
                self.reasons |= {name for b, name in self.REASONS.items() if bits & b}
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(0.005)

    def __enter__(self):
        if self.nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        if self.nvml is None:
            return {"unavailable": self.error}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples)}


# ------------------------------------------------------------- workloads
def randn_bf16(shape, gen, device, std=1.0, mean=0.0):
    import torch

    x = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
    if std != 1.0:
        x.mul_(std)
    if mean != 0.0:
        x.add_(mean)
    return x.to(torch.bfloat16)


class Chain:
    """Chained pass on 65536 tokens per GPU (the default workload)."""

    name = "chain"
    dominant = "swiglu_ffn"
    data = ("synthetic, counter-based (splitmix64 + Box-Muller keyed by seed, tensor and global index), "
            "generated on the device; rank r holds global tokens [r*T, (r+1)*T)")

    def __init__(self, device, rank, world, tokens=CHAIN_B * CHAIN_S, token_major=True, chunk_tokens=4096):
        import torch

        from hrm_layer_ops import chain, ops

        if tokens % CHAIN_S or tokens <= 0:
            raise SystemExit(f"--tokens must be a positive multiple of {CHAIN_S}")
        self.torch, self.chain, self.ops, self.device = torch, chain, ops, device
        self.batch = tokens // CHAIN_S
        self.token_major, self.chunk_tokens = token_major, chunk_tokens
        T = tokens
        self.tokens = T
        # Counter-based inputs (hrm_layer_ops.synth): every element is keyed by
        # (seed, tensor, global index).  Weights are replicated (index from 0);
        # rank r holds global tokens [r T, (r + 1) T) of each activation, so the
        # N-GPU job is one global N x T-token tensor set, whatever N is.
        from hrm_layer_ops import synth

        def nb(name, shape, start=0, std=1.0, mean=0.0):
            return synth.normal_bf16(shape, SEED, synth.tag_of(name), start, std, mean, device)

        t0 = rank * T
        self.w = chain.ChainWeights(
            table=nb("embed_table", (VOCAB, HIDDEN), std=0.02), w1=nb("norm1_weight", (HIDDEN,), std=0.1, mean=1.0),
            w2=nb("norm2_weight", (HIDDEN,), std=0.1, mean=1.0), rope=ops.rope_table(CHAIN_S, HEAD_DIM, THETA, device),
            scale=SCALE, eps=EPS, theta=THETA)
        self.ids = synth.ids(T, SEED, synth.tag_of("ids"), VOCAB, t0, device)
        qk = chain_qk_shape(T, token_major)
        self.q = nb("q", qk, t0 * HEADS * HEAD_DIM)
        self.k = nb("k", qk, t0 * HEADS * HEAD_DIM)
        self.o = nb("attn_out", (T, HIDDEN), t0 * HIDDEN)
        self.gate = nb("gate", (T, INTER), t0 * INTER, std=0.5)
        self.up = nb("up", (T, INTER), t0 * INTER, std=0.5)
        e = torch.empty
        bf = dict(dtype=torch.bfloat16, device=device)
        self.h, self.n1, self.r, self.n2 = (e((T, HIDDEN), **bf) for _ in range(4))
        self.y = e((T, INTER), **bf)
        per = chain_bytes_per_token(HIDDEN, HEADS, HEAD_DIM, INTER)
        self.per_token = per
        self.bytes_per_step = per["minimal"] * T
        self.rows_per_step = T
        self.kernels = list(CHAIN_KERNEL_NAMES)
        self.kernel_bytes = {k: per[k] * T for k in self.kernels}
        self.footprint = per["op_sum"] * T
        self.config = chain_config(T, token_major, world)

    def step(self, stream=None, events=None):
        self.chain.run_device(self.w, self.ids, self.q, self.k, self.o, self.gate, self.up, self.h, self.n1,
                              self.r, self.n2, self.y, 0, stream=stream, events=events,
                              token_major=self.token_major)
        return len(self.kernels)

    # -- decode shape (64 tokens, offset 4095), launch-latency bound: CUDA graphs.
    # Returns (per chain inside a graph of `chains` chains: the device's time per
    # decode step when the caller captures many steps or layers, median and range
    # of 5 repetitions; per one-chain graph replayed alone, which the host's
    # graph-launch rate bounds, median and range).
    def decode_latency_us(self, iters=200, chains=50):
        torch = self.torch
        T = DECODE_B
        shape = (DECODE_B, 1, HEADS, HEAD_DIM) if self.token_major else (DECODE_B, HEADS, 1, HEAD_DIM)
        dq = self.q.reshape(-1)[:DECODE_B * HEADS * HEAD_DIM].reshape(shape).clone()
        dk = dq.clone()
        args = (self.ids[:T], dq, dk, self.o[:T], self.gate[:T], self.up[:T], self.h[:T], self.n1[:T],
                self.r[:T], self.n2[:T], self.y[:T])
        s = torch.cuda.Stream(self.device)
        with torch.cuda.stream(s):
            for _ in range(3):
                self.chain.run_device(self.w, *args, 4095, stream=s, token_major=self.token_major)
        s.synchronize()

        def per_chain(n_chains, replays):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for _ in range(n_chains):
                    self.chain.run_device(self.w, *args, 4095, stream=s, token_major=self.token_major)
            for _ in range(3):
                g.replay()
            torch.cuda.synchronize()
            reps = []
            for _ in range(5):
                t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                t0.record()
                for _ in range(replays):
                    g.replay()
                t1.record()
                torch.cuda.synchronize()
                reps.append(t0.elapsed_time(t1) * 1000.0 / (replays * n_chains))
            del g
            return statistics.median(reps), (min(reps), max(reps))

        return per_chain(chains, max(1, iters // chains)), per_chain(1, iters)

    # -- end to end: pinned host buffers through the public API
    def e2e(self, steps):
        torch = self.torch
        hc = self.chain.HostChain(self.w, self.batch, HEADS, CHAIN_S, HEAD_DIM, HIDDEN, INTER,
                                  chunk_tokens=self.chunk_tokens, token_major=self.token_major, device=self.device)
        pin = dict(pin_memory=True)
        host_in = {n: torch.empty(getattr(self, n).shape, dtype=getattr(self, n).dtype, **pin)
                   for n in hc.IN}
        for n in hc.IN:
            host_in[n].copy_(getattr(self, n))
        host_out = {n: torch.empty(getattr(self, n).shape, dtype=getattr(self, n).dtype, **pin)
                    for n in ("q", "k", "h", "n1", "r", "n2", "y")}
        h2d, d2h = hc.bytes_per_pass(host_in, host_out)
        hc.run(host_in, host_out)  # warm-up
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        launches = 0
        t0.record()
        for _ in range(steps):
            launches += hc.run(host_in, host_out)
        t1.record()
        torch.cuda.synchronize()
        ms = t0.elapsed_time(t1) / steps
        return ms, h2d, d2h, launches

    # -- the oracle on the same pass (rank 0's shard), a bounded number of passes
    def cpu_sample(self, min_seconds=8.0, max_reps=50):
        c = CpuChain(self.tokens, self.token_major)
        c.run_once()  # first touch of the outputs
        reps, t0 = 0, time.perf_counter()
        while True:
            c.run_once()
            reps += 1
            el = time.perf_counter() - t0
            if el >= min_seconds or reps >= max_reps:
                break
        sec = el / reps
        return {"gbs": c.bytes / sec / 1e9, "sec_per_sample": sec, "cores": c.cores,
                "sample": f"{reps} whole passes of the {c.tokens}-token chain (rank 0's inputs), "
                          f"oracle with {c.cores} OpenMP threads"}


def synth_tag(name):
    """The counter-based generator's 32-bit tensor tag (crc32 of the name)."""
    import zlib

    return zlib.crc32(name.encode())


class CpuChain:
    """The chained pass on the host cores through the oracle (a C restatement
    of the reference's kernels, all OpenMP threads): the same workload as the
    GPU arm -- `tokens` tokens of rank 0's counter-based inputs, in the same
    Q/K layout -- with every output buffer allocated once and RoPE in place,
    as the reference's kernels run.  Imports nothing of the library."""

    def __init__(self, tokens=CHAIN_B * CHAIN_S, token_major=True):
        import ctypes

        import numpy as np

        sys.path.insert(0, ROOT)
        from oracle import Oracle

        if tokens % CHAIN_S or tokens <= 0:
            raise SystemExit(f"--tokens must be a positive multiple of {CHAIN_S}")
        self.o = o = Oracle()
        # all the host cores this process may use (torchrun exports OMP_NUM_THREADS=1)
        o.set_threads(len(os.sched_getaffinity(0)))
        self.cores = o.max_threads()
        self.tokens = T = tokens
        self.token_major = token_major
        u16 = np.uint16

        def nb(name, shape, start=0, std=1.0, mean=0.0):
            return o.fill_normal_bf16(np.empty(shape, u16), SEED, synth_tag(name), start, std, mean)

        self.table = nb("embed_table", (VOCAB, HIDDEN), std=0.02)
        self.w1 = nb("norm1_weight", (HIDDEN,), std=0.1, mean=1.0)
        self.w2 = nb("norm2_weight", (HIDDEN,), std=0.1, mean=1.0)
        self.rope = o.rope_table(CHAIN_S, HEAD_DIM, THETA)
        self.ids = o.fill_ids(np.empty(T, np.uint32), SEED, synth_tag("ids"), VOCAB)
        self.qk_shape = chain_qk_shape(T, token_major)
        self.q, self.k = nb("q", self.qk_shape), nb("k", self.qk_shape)
        self.ob = nb("attn_out", (T, HIDDEN))
        self.g, self.u = nb("gate", (T, INTER), std=0.5), nb("up", (T, INTER), std=0.5)
        self.h, self.n1, self.r, self.n2 = (np.empty((T, HIDDEN), u16) for _ in range(4))
        self.y = np.empty((T, INTER), u16)
        self.bytes = chain_bytes_per_token(HIDDEN, HEADS, HEAD_DIM, INTER)["minimal"] * T
        p = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
        self._p = {n: p(getattr(self, n)) for n in ("table", "w1", "w2", "rope", "ids", "q", "k", "ob", "g", "u",
                                                     "h", "n1", "r", "n2", "y")}

    def run_once(self):
        lib, p, T = self.o.lib, self._p, self.tokens
        lib.ora_embed_rms_norm(p["ids"], p["table"], p["h"], p["n1"], p["w1"], T, HIDDEN, VOCAB, SCALE, EPS)
        B = T // CHAIN_S
        if self.token_major:
            lib.ora_rope_embed_token_major(p["q"], p["k"], B, CHAIN_S, HEADS, HEAD_DIM, 0, THETA, p["rope"])
        else:
            lib.ora_rope_embed(p["q"], p["k"], B, HEADS, CHAIN_S, HEAD_DIM, 0, THETA, p["rope"])
        lib.ora_add_rms_norm(p["h"], p["ob"], p["r"], p["n2"], p["w2"], T, HIDDEN, EPS)
        lib.ora_swiglu_ffn(p["g"], p["u"], p["y"], T * INTER)


def single_op_spec(name):
    """(config, algorithmic bytes per step, rows per step) of a single-op workload;
    shared by both arms, so that they report the same config and bytes."""
    if name == "add_rms_norm":        # [16384 x 2048] bf16, weight, eps 1e-5
        return {"workload": "fused residual add + RMSNorm bf16 [16384 x 2048]", "rows": 16384}, 16384 * HIDDEN * 8, 16384
    if name == "rms_norm_f32":        # [4096 x 2048] fp32, weight, eps 1e-5
        return {"workload": "RMSNorm fp32 [4096 x 2048]", "rows": 4096}, 4096 * HIDDEN * 8, 4096
    if name == "rms_norm":            # [4096 x 2048] bf16, weight, eps 1e-5
        return {"workload": "RMSNorm bf16 [4096 x 2048]", "rows": 4096}, 4096 * HIDDEN * 4, 4096
    if name == "rope":                # Q, K [8, 16, 4096, 128], table
        return ({"workload": "RoPE Q/K [8, 16, 4096, 128] bf16, fp32 table", "tokens": 8 * 4096},
                4 * 2 * 8 * HEADS * 4096 * HEAD_DIM, 8 * 4096)
    if name == "swiglu":              # gate, up [32768 x 5632]
        return {"workload": "SwiGLU bf16 [32768 x 5632]", "rows": 32768}, 32768 * INTER * 6, 32768
    if name == "embedding":           # table [32000 x 2048], 65536 ids
        return ({"workload": "embedding gather [32000 x 2048] table, 65536 ids", "tokens": 65536},
                65536 * (4 + 2 * 2 * HIDDEN), 65536)
    if name == "split_rope":          # gqkv [16, 4096, 4 x 16 x 128] -> gate, q, k, v + KV cache, table
        T = 16 * 4096
        return ({"workload": "split_gqkv + RoPE + KV-cache write, gqkv [16, 4096, 4 x 16 x 128] bf16", "tokens": T},
                T * (4 + 4 + 2) * HEADS * HEAD_DIM * 2, T)
    if name == "attn_gate":           # attn [65536 x 2048] *= sigmoid(gate), in place
        return {"workload": "attention gate in place [65536 x 2048] bf16", "rows": 65536}, 65536 * HIDDEN * 6, 65536
    if name == "convert_f32":         # 2^28 f32 checkpoint values -> bf16 (a 1 GB tensor)
        n = 1 << 28
        return {"workload": "checkpoint f32 -> bf16 conversion, 2^28 values", "elements": n}, n * 6, n
    raise ValueError(name)


def single_op_sets(bytes_per_step):
    """Input sets the GPU arm rotates so that their total exceeds 3x L2."""
    return max(1, -(-3 * L2_BYTES // bytes_per_step))


def single_op_l2_note(bytes_per_step):
    nbuf = single_op_sets(bytes_per_step)
    return (f"{nbuf} rotating input sets ({nbuf * bytes_per_step / 1e6:.0f} MB > 3x L2)"
            if nbuf > 1 else "inputs larger than L2; no flush")


class CpuSingleOp:
    """A single-op workload on the host cores through the oracle (a C
    restatement of the reference's kernels, all OpenMP threads): the GPU arm's
    shapes and byte count, seeded host inputs of the same distributions,
    outputs allocated once, in place where the reference's kernel is.  For
    split_rope it runs the reference's three steps (split_gqkv, rope_embed,
    kv_cache_update).  Imports nothing of the library."""

    def __init__(self, name):
        import ctypes

        import numpy as np

        sys.path.insert(0, ROOT)
        from oracle import Oracle

        self.name = name
        self.config, self.bytes, self.rows = single_op_spec(name)
        self.o = o = Oracle()
        o.set_threads(len(os.sched_getaffinity(0)))
        self.cores = o.max_threads()
        u16 = np.uint16
        tag = iter(range(1, 100))

        def nb(shape, std=1.0, mean=0.0):
            return o.fill_normal_bf16(np.empty(shape, u16), SEED + 7, next(tag), 0, std, mean)

        p = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
        lib = o.lib
        if name in ("rms_norm", "add_rms_norm"):
            R = self.rows
            x, w, y = nb((R, HIDDEN)), nb(HIDDEN, 0.1, 1.0), np.empty((R, HIDDEN), u16)
            if name == "rms_norm":
                self.run_once = lambda: lib.ora_rms_norm(p(x), p(y), p(w), R, HIDDEN, EPS)
            else:
                b, r = nb((R, HIDDEN)), np.empty((R, HIDDEN), u16)
                self.run_once = lambda: lib.ora_add_rms_norm(p(x), p(b), p(r), p(y), p(w), R, HIDDEN, EPS)
            self._keep = [x, w, y] + ([b, r] if name == "add_rms_norm" else [])
        elif name == "rms_norm_f32":
            rng = np.random.default_rng(SEED + 7)
            x = rng.standard_normal((4096, HIDDEN), dtype=np.float32)
            w = (1 + 0.1 * rng.standard_normal(HIDDEN, dtype=np.float32)).astype(np.float32)
            y = np.empty_like(x)
            self.run_once = lambda: lib.ora_rms_norm_f32(p(x), p(y), p(w), 4096, HIDDEN, EPS)
            self._keep = [x, w, y]
        elif name == "rope":
            q, k, tab = nb((8, HEADS, 4096, HEAD_DIM)), nb((8, HEADS, 4096, HEAD_DIM)), o.rope_table(4096, HEAD_DIM, THETA)
            self.run_once = lambda: lib.ora_rope_embed(p(q), p(k), 8, HEADS, 4096, HEAD_DIM, 0, THETA, p(tab))
            self._keep = [q, k, tab]
        elif name == "swiglu":
            g, u, y = nb((32768, INTER), 0.5), nb((32768, INTER), 0.5), np.empty((32768, INTER), u16)
            self.run_once = lambda: lib.ora_swiglu_ffn(p(g), p(u), p(y), 32768 * INTER)
            self._keep = [g, u, y]
        elif name == "embedding":
            tab, y = nb((VOCAB, HIDDEN), 0.02), np.empty((65536, HIDDEN), u16)
            ids = o.fill_ids(np.empty(65536, np.uint32), SEED + 7, next(tag), VOCAB)
            self.run_once = lambda: lib.ora_embedding_lookup(p(ids), p(tab), p(y), 65536, HIDDEN, VOCAB, SCALE)
            self._keep = [tab, y, ids]
        elif name == "attn_gate":
            g, a = nb((65536, HIDDEN)), nb((65536, HIDDEN))
            self.run_once = lambda: lib.ora_gated_attn_output(p(g), p(a), p(a), 65536 * HIDDEN)
            self._keep = [g, a]
        elif name == "convert_f32":
            n = self.rows
            src = np.random.default_rng(SEED + 7).standard_normal(n, dtype=np.float32)
            y = np.empty(n, u16)
            self.run_once = lambda: lib.ora_convert_to_bf16(p(src), 1, p(y), n)  # 1: f32
            self._keep = [src, y]
        elif name == "split_rope":
            B, S = 16, 4096
            gq = nb((B, S, 4 * HEADS * HEAD_DIM))
            gate = np.empty((B, S, HEADS, HEAD_DIM), u16)
            q, k, v, kc, vc = (np.empty((B, HEADS, S, HEAD_DIM), u16) for _ in range(5))
            tab = o.rope_table(S, HEAD_DIM, THETA)

            def run():
                lib.ora_split_gqkv(p(gq), p(gate), p(q), p(k), p(v), B, S, HEADS, HEAD_DIM)
                lib.ora_rope_embed(p(q), p(k), B, HEADS, S, HEAD_DIM, 0, THETA, p(tab))
                lib.ora_kv_cache_update(p(k), p(v), p(kc), p(vc), B, HEADS, S, HEAD_DIM, S, 0, 0)
            self.run_once = run
            self._keep = [gq, gate, q, k, v, kc, vc, tab]
        else:
            raise ValueError(name)

    def sample(self, min_seconds=5.0, max_reps=50):
        """GB/s over a bounded number of whole steps (at least min_seconds)."""
        self.run_once()  # first touch of the outputs
        reps, t0 = 0, time.perf_counter()
        while True:
            self.run_once()
            reps += 1
            el = time.perf_counter() - t0
            if el >= min_seconds or reps >= max_reps:
                break
        sec = el / reps
        return {"gbs": self.bytes / sec / 1e9, "sec_per_sample": sec, "cores": self.cores,
                "sample": f"{reps} whole steps of the {self.config['workload']} workload, oracle with "
                          f"{self.cores} OpenMP threads"}


class SingleOp:
    """One of the per-op workloads (the other layer-op configurations)."""

    def __init__(self, name, device, rank):
        import torch

        import hrm_layer_ops as ops

        self.torch, self.ops, self.device, self.name = torch, ops, device, name
        gen = torch.Generator(device=device).manual_seed(2000 + rank)
        bf = torch.bfloat16
        self.cfg, self.bytes_per_step, self.rows_per_step = single_op_spec(name)
        if name == "add_rms_norm":        # [16384 x 2048] bf16, weight, eps 1e-5
            R = 16384
            self.w = randn_bf16(HIDDEN, gen, device, 0.1, 1.0)
            mk = lambda: (randn_bf16((R, HIDDEN), gen, device), randn_bf16((R, HIDDEN), gen, device),
                          torch.empty((R, HIDDEN), dtype=bf, device=device),
                          torch.empty((R, HIDDEN), dtype=bf, device=device))
        elif name == "rms_norm_f32":      # [4096 x 2048] fp32, weight, eps 1e-5
            R = 4096
            self.w = torch.randn(HIDDEN, generator=gen, device=device) * 0.1 + 1
            mk = lambda: (torch.randn((R, HIDDEN), generator=gen, device=device),
                          torch.empty((R, HIDDEN), device=device))
        elif name == "rms_norm":          # [4096 x 2048] bf16, weight, eps 1e-5
            R = 4096
            self.w = randn_bf16(HIDDEN, gen, device, 0.1, 1.0)
            mk = lambda: (randn_bf16((R, HIDDEN), gen, device), torch.empty((R, HIDDEN), dtype=bf, device=device))
        elif name == "rope":              # Q, K [8, 16, 4096, 128], table
            shape = (8, HEADS, 4096, HEAD_DIM)
            self.table = ops.rope_table(4096, HEAD_DIM, THETA, device)
            mk = lambda: (randn_bf16(shape, gen, device), randn_bf16(shape, gen, device))
        elif name == "swiglu":            # gate, up [32768 x 5632]
            shape = (32768, INTER)
            mk = lambda: (randn_bf16(shape, gen, device, 0.5), randn_bf16(shape, gen, device, 0.5),
                          torch.empty(shape, dtype=bf, device=device))
        elif name == "embedding":         # table [32000 x 2048], 65536 ids
            T = 65536
            self.tab = randn_bf16((VOCAB, HIDDEN), gen, device, 0.02)
            mk = lambda: (torch.randint(0, VOCAB, (T,), generator=gen, device=device, dtype=torch.int32),
                          torch.empty((T, HIDDEN), dtype=bf, device=device))
        elif name == "split_rope":        # gqkv [16, 4096, 4 x 16 x 128] -> gate, q, k, v + KV cache, table
            B, S = 16, 4096
            T = B * S
            self.table = ops.rope_table(S, HEAD_DIM, THETA, device)
            mk = lambda: (randn_bf16((B, S, 4 * HEADS * HEAD_DIM), gen, device),
                          torch.empty((B, S, HEADS, HEAD_DIM), dtype=bf, device=device),
                          *(torch.empty((B, HEADS, S, HEAD_DIM), dtype=bf, device=device) for _ in range(5)))
        elif name == "attn_gate":         # attn [65536 x 2048] *= sigmoid(gate), in place
            shape = (65536, HIDDEN)
            mk = lambda: (randn_bf16(shape, gen, device), randn_bf16(shape, gen, device))
        elif name == "convert_f32":       # 2^28 f32 checkpoint values -> bf16 (a 1 GB tensor)
            n = 1 << 28
            mk = lambda: (torch.randn(n, generator=gen, device=device).view(torch.uint8),
                          torch.empty(n, dtype=bf, device=device))
        else:
            raise ValueError(name)
        # Rotate input sets so that their total exceeds 3x L2: no step finds its inputs in L2.
        nbuf = single_op_sets(self.bytes_per_step)
        self.bufs = [mk() for _ in range(nbuf)]
        self.i = 0
        self.kernels = [name]
        self.dominant = name
        self.kernel_bytes = {name: self.bytes_per_step}
        self.footprint = self.bytes_per_step
        self.cfg["l2"] = single_op_l2_note(self.bytes_per_step)
        self.config = self.cfg

    def step(self, stream=None, events=None):
        ops, b = self.ops, self.bufs[self.i % len(self.bufs)]
        self.i += 1
        if events is not None:
            events[0].record(stream)
        if self.name == "add_rms_norm":
            ops.add_rms_norm(b[0], b[1], self.w, EPS, residual_out=b[2], normed_out=b[3], stream=stream)
        elif self.name in ("rms_norm_f32", "rms_norm"):
            ops.rms_norm(b[0], self.w, EPS, out=b[1], stream=stream)
        elif self.name == "rope":
            ops.rope_embed(b[0], b[1], 0, THETA, self.table, stream=stream)
        elif self.name == "swiglu":
            ops.swiglu_ffn(b[0], b[1], out=b[2], stream=stream)
        elif self.name == "attn_gate":
            ops.apply_attn_gate(b[0], b[1], stream=stream)
        elif self.name == "convert_f32":
            ops.convert_to_bf16(b[0], "f32", out=b[1], stream=stream)
        elif self.name == "split_rope":
            ops.split_gqkv_rope(b[0], HEADS, 0, THETA, self.table, b[5], b[6], 0, out=b[1:5], stream=stream)
        else:
            ops.embedding_lookup(b[0], self.tab, SCALE, out=b[1], stream=stream)
        if events is not None:
            events[1].record(stream)
        return 1

    def e2e(self, steps):
        """Per step: H2D of the inputs from pinned host memory, the kernel, D2H of the outputs."""
        torch = self.torch
        b = self.bufs[0]
        n_in = {"add_rms_norm": 2, "rms_norm_f32": 1, "rms_norm": 1, "rope": 2, "swiglu": 2, "embedding": 1,
                "split_rope": 1, "attn_gate": 2, "convert_f32": 1}[self.name]
        outs = {"rope": [0, 1], "attn_gate": [1]}.get(self.name, list(range(n_in, len(b))))
        host = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in b]
        for h, t in zip(host, b):
            h.copy_(t)
        h2d = sum(host[i].numel() * host[i].element_size() for i in range(n_in))
        d2h = sum(host[i].numel() * host[i].element_size() for i in outs)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        launches = 0
        for it in range(steps + 1):  # iteration 0 is the warm-up
            if it == 1:
                torch.cuda.synchronize()
                t0.record()
            for i in range(n_in):
                b[i].copy_(host[i], non_blocking=True)
            self.i = 0
            n = self.step()
            launches += n if it else 0
            for i in outs:
                host[i].copy_(b[i], non_blocking=True)
        t1.record()
        torch.cuda.synchronize()
        return t0.elapsed_time(t1) / steps, h2d, d2h, launches

    def cpu_sample(self, min_seconds=5.0):
        """The oracle on the same workload's shapes (CpuSingleOp), a bounded sample."""
        return CpuSingleOp(self.name).sample(min_seconds)


# The reference model's shapes (HrmConfig defaults, src/lib.rs:40-60).
CKPT_LAYERS, CKPT_H, CKPT_I, CKPT_V = 16, 1536, 4096, 65536


def write_synthetic_checkpoint(path, dtype="F32"):
    """A safetensors file of the reference model's tensors (the names of
    src/lib.rs:2043-2112, attention / MLP prefixes), values 0.02 N(0, 1) from a
    16 MB seeded block repeated."""
    import json

    import numpy as np

    es = {"F32": 4, "BF16": 2, "F16": 2}[dtype]
    L, H, I, V = CKPT_LAYERS, CKPT_H, CKPT_I, CKPT_V
    shapes = []
    for mod in ("H", "L"):
        for i in range(L):
            p = f"model.{mod}_module.layers.{i}"
            shapes += [(f"{p}.attn.gqkv_proj.weight", (4 * H, H)), (f"{p}.attn.o_proj.weight", (H, H)),
                       (f"{p}.mlp.gate_up_proj.weight", (2 * I, H)), (f"{p}.mlp.down_proj.weight", (H, I))]
    shapes += [("model.embed_tokens.weight", (V, H)), ("lm_head.weight", (V, H)), ("model.z_L_init", (H,))]
    header, off = {}, 0
    for name, shape in shapes:
        n = int(np.prod(shape)) * es
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + n]}
        off += n
    text = json.dumps(header).encode()
    text += b" " * (-len(text) % 8)
    block = (np.random.default_rng(0).standard_normal(1 << 22) * 0.02).astype(
        {"F32": np.float32, "F16": np.float16, "BF16": np.float32}[dtype])
    if dtype == "BF16":
        block = (block.view(np.uint32) >> 16).astype(np.uint16)
    block = block.tobytes()
    with open(path, "wb") as f:
        f.write(len(text).to_bytes(8, "little"))
        f.write(text)
        left = off
        while left > 0:
            k = min(left, len(block))
            f.write(block[:k])
            left -= k


def checkpoint_config(dtype, file_bytes, pieces, bytes_per_step):
    """The load_checkpoint workload's `config`, the same dict on both arms."""
    return {"workload": "checkpoint file -> bf16 device tensors, HRM-Text-1B shapes "
                        f"({CKPT_LAYERS} layers x 2 modules, hidden {CKPT_H}, intermediate {CKPT_I}, "
                        f"vocab {CKPT_V})", "dtype_in_file": dtype, "file_bytes": file_bytes,
            "tensor_pieces": pieces,
            "l2": f"{bytes_per_step / 1e9:.1f} GB moved per step vs 126 MB L2; no flush"}


def temp_checkpoint(owner, dtype):
    """Writes the synthetic checkpoint into a fresh directory (in /dev/shm
    where there is one), removed at exit even after a failure; returns its path
    and sets owner.own_dir."""
    import atexit
    import tempfile

    base = "/dev/shm" if os.path.isdir("/dev/shm") else None
    owner.own_dir = tempfile.mkdtemp(prefix="hrm_ckpt_", dir=base)
    atexit.register(owner.close)
    path = os.path.join(owner.own_dir, "model.safetensors")
    write_synthetic_checkpoint(path, dtype)
    return path


class LoadCheckpoint:
    """Checkpoint file -> bf16 device tensors at the reference model's shapes
    (HrmConfig defaults, src/lib.rs:40-60: 16 layers per module, hidden 1536,
    intermediate 4096, vocab 65536; 1.18 B parameters).  A synthetic
    safetensors file is written once (f32 tensors, values ~ 0.02 N(0, 1)).

    value: the GPU conversion of the file's raw bytes already in HBM into the
    model's bf16 tensors (gate_up split), one launch per tensor piece, the
    step's launches replayed from a CUDA graph; bytes = raw read + bf16
    written.  e2e: the same bytes over the wall time of
    hrm_layer_ops.checkpoint.load_safetensors on the file (page-cached reads
    into pinned buffers, H2D, conversion on the GPU), plus a read-back of
    z_L_init; file_gbs is the file's bytes over that time."""

    name = "load_checkpoint"
    LAYERS, H, I, V = CKPT_LAYERS, CKPT_H, CKPT_I, CKPT_V

    def __init__(self, device, rank, path=None, dtype="F32"):
        import numpy as np
        import torch

        from hrm_layer_ops import checkpoint as ck
        import hrm_layer_ops as ops

        self.torch, self.ck, self.ops, self.device = torch, ck, ops, device
        self.own_dir = None
        if path is None:
            path = temp_checkpoint(self, dtype)  # removed at exit even if the run fails
        self.path = path
        self.hdr = ck.read_header(path)
        hdr = self.hdr
        # the raw data section resident in HBM, and the destination tensors
        size = os.path.getsize(path)
        raw = np.fromfile(path, dtype=np.uint8, offset=hdr.data_offset, count=size - hdr.data_offset)
        self.raw = torch.from_numpy(raw).to(device)
        del raw
        split = self.I * self.H
        self.pieces = []  # (byte offset in the data section, numel, dtype name, destination)
        for t in hdr.tensors:
            es = ck.DTYPE_SIZES[t.dtype]
            if t.name.endswith("gate_up_proj.weight"):  # split as src/lib.rs:2072-2078
                parts = [(t.begin, split), (t.begin + split * es, t.numel - split)]
            else:
                parts = [(t.begin, t.numel)]
            for b0, n in parts:
                self.pieces.append((b0, n, t.dtype.lower(), torch.empty(n, dtype=torch.bfloat16, device=device)))
        self.bytes_per_step = sum(n * (ck.DTYPE_SIZES[d.upper()] + 2) for _, n, d, _ in self.pieces)
        self.rows_per_step = sum(n for _, n, _, _ in self.pieces)
        self.file_bytes = size
        self.kernels = ["convert_to_bf16"]
        self.dominant = "convert_to_bf16"
        self.kernel_bytes = {"convert_to_bf16": self.bytes_per_step}
        self.footprint = self.bytes_per_step
        self.config = checkpoint_config(dtype, size, len(self.pieces), self.bytes_per_step)
        self.data = "synthetic safetensors file (f32, 0.02 N(0,1) tiled), written once per run"

    def cpu_sample(self, min_seconds=5.0, sample_bytes=512 << 20):
        """The reference's host conversion (raw_to_bf16, restated by the oracle,
        all host threads) over the first 512 MB of the file's data section."""
        import numpy as np

        sys.path.insert(0, ROOT)
        from oracle import Oracle

        o = Oracle()
        o.set_threads(len(os.sched_getaffinity(0)))
        d = self.hdr.tensors[0].dtype
        es = self.ck.DTYPE_SIZES[d]
        n = sample_bytes // es
        raw = np.fromfile(self.path, dtype=np.uint8, offset=self.hdr.data_offset, count=n * es).tobytes()
        o.convert_to_bf16(raw, d.lower())
        reps, t0 = 0, time.perf_counter()
        while True:
            o.convert_to_bf16(raw, d.lower())
            reps += 1
            el = time.perf_counter() - t0
            if el >= min_seconds:
                break
        sec = el / reps
        return {"gbs": n * (es + 2) / sec / 1e9, "cores": o.max_threads(),
                "sample": f"raw_to_bf16 of {n * es >> 20} MB of the file's {d} data on the host, {reps} reps, "
                          f"oracle with {o.max_threads()} OpenMP threads"}

    def close(self):
        import shutil

        if self.own_dir is not None:
            shutil.rmtree(self.own_dir, ignore_errors=True)
            self.own_dir = None

    def step(self, stream=None, events=None):
        if events is not None:
            events[0].record(stream)
        for b0, n, d, out in self.pieces:
            es = self.ck.DTYPE_SIZES[d.upper()]
            self.ops.convert_to_bf16(self.raw[b0:b0 + n * es], d, out=out, stream=stream)
        if events is not None:
            events[1].record(stream)
        return len(self.pieces)

    def e2e(self, steps):
        """Per step: the whole file -> device tensors through the public loader,
        then z_L_init read back.  Host wall time (file reads are host work)."""
        torch = self.torch
        ms = []
        w = None
        for it in range(steps + 1):  # iteration 0 is the warm-up
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            w = self.ck.load_safetensors(self.path, self.LAYERS, self.H, self.I, device=self.device)
            z = w.z_l_init.cpu()
            t1 = time.perf_counter()
            if it:
                ms.append((t1 - t0) * 1e3)
            del w
        mean = sum(ms) / len(ms)
        self.file_gbs = self.file_bytes / (mean / 1e3) / 1e9
        h2d = self.file_bytes - self.hdr.data_offset
        return mean, h2d, int(z.numel() * 2), steps * len(self.pieces)


class Module:
    """One pass of a 4-layer H/L module over 16384 tokens: the layer loop's
    residual / norm / SwiGLU schedule (hrm_layer_ops.module.transformer_module:
    injection + pre-norm, then per layer add+norm, SwiGLU, add+norm).  The
    attention and GEMM outputs are synthetic and pre-filled (their callbacks do
    nothing), so the step times exactly the library's 13 launches."""

    name = "module"
    LAYERS, TOKENS = 4, 16384

    def __init__(self, device, rank):
        import torch

        from hrm_layer_ops import module

        self.torch, self.module, self.device = torch, module, device
        gen = torch.Generator(device=device).manual_seed(3000 + rank)
        T, L = self.TOKENS, self.LAYERS
        self.sc = module.ModuleScratch(T, HIDDEN, INTER, device)
        for t in (self.sc.a, self.sc.d):
            t.copy_(randn_bf16(t.shape, gen, device))
        for t in (self.sc.g, self.sc.u):
            t.copy_(randn_bf16(t.shape, gen, device, 0.5))
        self.za, self.zb = randn_bf16((T, HIDDEN), gen, device), randn_bf16((T, HIDDEN), gen, device)
        self.out = torch.empty((T, HIDDEN), dtype=torch.bfloat16, device=device)
        per = module.module_bytes_per_token(HIDDEN, INTER, L)
        self.bytes_per_step, self.rows_per_step = per * T, T
        self.kernels = ["module_pass"]
        self.dominant = "module_pass"
        self.kernel_bytes = {"module_pass": self.bytes_per_step}
        self.footprint = self.bytes_per_step
        self.launches = 1 + 3 * L
        self.config = {"workload": f"layer-loop module pass, {L} layers x {T} tokens (H {HIDDEN}, I {INTER}): "
                                   "injection+norm, per layer add+norm / SwiGLU / add+norm",
                       "tokens": T, "layers": L, "bytes_per_token": per,
                       "bytes_per_token_reference_order": module.reference_order_bytes_per_token(HIDDEN, INTER, L),
                       "gemm_and_attention": "outputs pre-filled, not timed",
                       "roofline_scope": "the whole pass (13 launches)",
                       "l2": f"{per * T / 1e9:.1f} GB moved per step vs 126 MB L2; no flush"}

    @staticmethod
    def _noop(*_):
        return None

    def step(self, stream=None, events=None):
        if events is not None:
            events[0].record(stream)
        self.module.transformer_module(self.za, self.zb, self.out, self.LAYERS, self._noop, self._noop,
                                       self._noop, self.sc, eps=EPS, stream=stream)
        if events is not None:
            events[1].record(stream)
        return self.launches

    def e2e(self, steps):
        """Per step: z_a and z_b from pinned host memory, the pass, the output back."""
        torch = self.torch
        host = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in (self.za, self.zb, self.out)]
        host[0].copy_(self.za)
        host[1].copy_(self.zb)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        launches = 0
        for it in range(steps + 1):  # iteration 0 is the warm-up
            if it == 1:
                torch.cuda.synchronize()
                t0.record()
            self.za.copy_(host[0], non_blocking=True)
            self.zb.copy_(host[1], non_blocking=True)
            n = self.step()
            launches += n if it else 0
            host[2].copy_(self.out, non_blocking=True)
        t1.record()
        torch.cuda.synchronize()
        nb = self.za.numel() * 2
        return t0.elapsed_time(t1) / steps, 2 * nb, nb, launches


# ------------------------------------------------------------------ main
class ReferenceCheckpointLoad:
    """The reference's load_safetensors path (src/lib.rs:2023-2125) on the host:
    the whole file read into memory (std::fs::read), every tensor converted to
    bf16 on the host (raw_to_bf16, src/lib.rs:1981-2008, restated by the oracle
    with all host threads), gate_up split into two host copies
    (src/lib.rs:2072-2078), and each tensor copied to the GPU from pageable
    memory (cudarc's htod_copy; a torch copy here).  Imports nothing of the
    library."""

    def __init__(self, path=None, dtype="F32"):
        import numpy as np

        sys.path.insert(0, ROOT)
        from oracle import Oracle

        self.np = np
        self.o = Oracle()
        self.o.set_threads(len(os.sched_getaffinity(0)))
        self.cores = self.o.max_threads()
        self.own_dir = None
        self.path = path if path is not None else temp_checkpoint(self, dtype)
        self.dtype = dtype
        with open(self.path, "rb") as f:
            n = int.from_bytes(f.read(8), "little")
            self.header = {k: v for k, v in json.loads(f.read(n)).items() if k != "__metadata__"}
        self.base = 8 + n
        self.file_bytes = os.path.getsize(self.path)
        sizes = {"F32": 4, "F16": 2, "BF16": 2}
        self.bytes_per_step, self.pieces = 0, 0
        for name, t in self.header.items():
            numel = (t["data_offsets"][1] - t["data_offsets"][0]) // sizes[t["dtype"]]
            self.bytes_per_step += numel * (sizes[t["dtype"]] + 2)
            self.pieces += 2 if name.endswith("gate_up_proj.weight") else 1

    def run_once(self):
        import torch

        np = self.np
        with open(self.path, "rb") as f:
            data = f.read()
        split = CKPT_I * CKPT_H
        out = []
        for name, t in self.header.items():
            b0, b1 = self.base + t["data_offsets"][0], self.base + t["data_offsets"][1]
            host = self.o.convert_to_bf16(data[b0:b1], t["dtype"].lower())
            parts = [host[:split].copy(), host[split:].copy()] if name.endswith("gate_up_proj.weight") else [host]
            for h in parts:
                out.append(torch.from_numpy(h.view(np.int16)).to("cuda"))
        torch.cuda.synchronize()
        return out

    def close(self):
        import shutil

        if self.own_dir is not None:
            shutil.rmtree(self.own_dir, ignore_errors=True)
            self.own_dir = None


def reference_checkpoint_arm(args, world):
    c = ReferenceCheckpointLoad(args.ckpt)
    try:
        for _ in range(args.warmup):
            c.run_once()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            c.run_once()
        sec = (time.perf_counter() - t0) / args.steps
    finally:
        c.close()
    gbs = c.bytes_per_step / sec / 1e9
    sample = (f"whole loads of the {c.file_bytes / 1e9:.2f} GB synthetic checkpoint: file read, host conversion "
              f"(oracle, {c.cores} OpenMP threads), gate_up split, pageable copies to the GPU")
    line = {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1000, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (fp32 math)",
        "data": "synthetic safetensors file (f32, 0.02 N(0,1) tiled), written once per run",
        "config": checkpoint_config(c.dtype, c.file_bytes, c.pieces, c.bytes_per_step),
        "file_gbs": round(c.file_bytes / sec / 1e9, 3),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": c.cores, "nproc": os.cpu_count(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


SINGLE_OPS = ("add_rms_norm", "rms_norm_f32", "rms_norm", "rope", "swiglu", "embedding", "split_rope", "attn_gate",
              "convert_f32")


def reference_single_op_arm(args, world):
    """A single-op workload's reference path on the host cores: the oracle (all
    threads) over whole steps of the GPU arm's shapes, with its config and bytes."""
    c = CpuSingleOp(args.workload)
    for _ in range(args.warmup):
        c.run_once()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        c.run_once()
    sec = (time.perf_counter() - t0) / args.steps
    gbs = c.bytes / sec / 1e9
    sample = f"whole steps of the {c.config['workload']} workload, oracle with {c.cores} OpenMP threads"
    line = {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1000, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp32" if args.workload == "rms_norm_f32" else "bf16 (fp32 math)",
        "data": "synthetic, seeded, generated on the host by the oracle",
        "config": dict(c.config, l2=single_op_l2_note(c.bytes), parallelism=f"{world} row shards, no collective"),
        "rows_per_s": round(c.rows / sec, 1),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": c.cores, "nproc": os.cpu_count(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def reference_arm(args, world, rank):
    """The reference's path on the host cores: the oracle, all threads, over the
    whole pass of the GPU arm's workload (rank 0's shard of --tokens tokens).
    Imports nothing of the library (neither hrm_layer_ops nor libhrm_ops.so)."""
    if rank != 0:
        return
    if args.workload == "load_checkpoint":
        reference_checkpoint_arm(args, world)
        return
    if args.workload in SINGLE_OPS:
        reference_single_op_arm(args, world)
        return
    if args.workload != "chain":
        print(json.dumps({"impl": "reference", "unavailable": "reference arm implemented for the chain, the "
                                                                "single-op and load_checkpoint workloads"}))
        return
    token_major = args.qk_layout == "token"
    c = CpuChain(args.tokens, token_major)
    for _ in range(args.warmup):
        c.run_once()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        c.run_once()
    sec = (time.perf_counter() - t0) / args.steps
    gbs = c.bytes / sec / 1e9
    sample = (f"whole {c.tokens}-token passes of the chain (rank 0's counter-based inputs, "
              f"{'token' if token_major else 'head'}-major Q/K), oracle with {c.cores} OpenMP threads")
    line = {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1000, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (fp32 math)",
        "data": "synthetic, counter-based (splitmix64 + Box-Muller keyed by seed, tensor and global index), "
                "generated on the host by the oracle; the same values as the GPU arm's rank 0",
        "config": chain_config(c.tokens, token_major, world),
        "rows_per_s": round(c.tokens / sec, 1),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": c.cores, "nproc": os.cpu_count(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, world, rank)
        return

    import datetime

    import torch
    import torch.distributed as dist

    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    peers = None
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
        from hrm_layer_ops.shard import PeerMonitor

        peers = PeerMonitor.for_default_group("hrm/bench")
    try:
        run_ours(args, world, rank, device, peers)
    except BaseException as e:
        if peers is not None:  # tell the other ranks before they wait in a collective
            peers.fail(f"{type(e).__name__}: {e}")
        raise


def run_ours(args, world, rank, device, peers):
    """This library's arm: warm-up, K timed steps, extras, one JSON line on rank 0.
    Before each collective every rank checks its peers' heartbeats (host only),
    so a rank that failed is reported instead of waited for."""
    import torch
    import torch.distributed as dist

    def collective_point(phase):
        if peers is not None:
            peers.sync(phase, timeout_s=120)

    if args.workload == "chain":
        wl = Chain(device, rank, world, args.tokens, args.qk_layout == "token", args.chunk_tokens)
    elif args.workload == "module":
        wl = Module(device, rank)
    elif args.workload == "load_checkpoint":
        wl = LoadCheckpoint(device, rank, args.ckpt)
    else:
        wl = SingleOp(args.workload, device, rank)
    stream = torch.cuda.current_stream(device)

    for _ in range(args.warmup):
        wl.step(stream)
    torch.cuda.synchronize()

    # ---- timed region: K steps, per-kernel events on the launching stream.  A
    # single-op workload (one short kernel per step) has its K steps captured in
    # a CUDA graph first, so that host launch overhead is not what is timed; its
    # one kernel's time is then the step time.
    nk = len(wl.kernels)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(nk + 1)] for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches = 0
    graph = None
    if isinstance(wl, (SingleOp, LoadCheckpoint)):
        cap = torch.cuda.Stream(device)
        cap.wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=cap):
            for i in range(args.steps):
                launches += wl.step(cap)
        # One untimed replay first: the first launch of a new graph also uploads
        # it to the device (about 2 us per node here), which is not the steps' time.
        graph.replay()
        # ... then flush L2 by reading 256 MB (a read leaves only clean lines
        # behind, so no write-back of the flush lands in the timed region), so
        # that the timed replay's first steps do not find the warm-up replay's
        # last inputs there.
        flush = torch.ones(256 << 20, dtype=torch.uint8, device=device)
        torch.cuda.synchronize()
        flush.sum()
        del flush
        torch.cuda.synchronize()
        wl.config["launch"] = (f"CUDA graph of the {args.steps} timed steps, replayed once untimed (graph upload), "
                               "then once between the events")
    collective_point(1)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(device) as clocks:
        start.record(stream)
        if graph is not None:
            graph.replay()
        else:
            for i in range(args.steps):
                launches += wl.step(stream, evs[i])
        end.record(stream)
        torch.cuda.synchronize()
    collective_point(2)
    if world > 1:
        dist.barrier()
    ms_total = start.elapsed_time(end)
    if graph is not None:
        kern_ms = {wl.kernels[0]: ms_total / args.steps}
        del graph
    else:
        kern_ms = {k: sum(evs[i][j].elapsed_time(evs[i][j + 1]) for i in range(args.steps)) / args.steps
                   for j, k in enumerate(wl.kernels)}
    per_rank_ms = None
    if world > 1:
        t = torch.tensor([ms_total] + [kern_ms[k] for k in wl.kernels], device=device, dtype=torch.float64)
        every = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(every, t)
        per_rank_ms = [round(float(x[0]) / args.steps, 4) for x in every]
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t[0])
        kern_ms = {k: float(t[j + 1]) for j, k in enumerate(wl.kernels)}
    ms_step = ms_total / args.steps
    value_gbs = world * wl.bytes_per_step / (ms_step / 1e3) / 1e9
    rows_per_s = world * wl.rows_per_step / (ms_step / 1e3)

    # ---- extras: decode latency, end-to-end, CPU baseline
    decode = wl.decode_latency_us() if isinstance(wl, Chain) else None
    e2e = None
    if not args.no_e2e:
        e2e_steps = max(2, min(args.steps, 5))
        ms_e2e, h2d, d2h, _ = wl.e2e(e2e_steps)
        collective_point(3)
        if world > 1:
            t = torch.tensor([ms_e2e], device=device, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms_e2e = float(t[0])
        e2e = {"value": round(world * wl.bytes_per_step / (ms_e2e / 1e3) / 1e9, 3), "unit": "GB/s",
               "ms_per_step": round(ms_e2e, 3), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "path": ("pinned host buffers, H2D / kernels / D2H overlapped in chunks (public API)"
                        if isinstance(wl, Chain) else
                        "file (page cache) -> pinned ring -> H2D -> GPU conversion, hrm_layer_ops.checkpoint "
                        "(public API), host wall time" if isinstance(wl, LoadCheckpoint) else
                        "pinned host buffers, H2D -> kernels -> D2H on one stream (public API)")}
        if isinstance(wl, LoadCheckpoint):
            e2e["file_gbs"] = round(wl.file_gbs, 3)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu and isinstance(wl, (Chain, LoadCheckpoint, SingleOp)):
        c = wl.cpu_sample()
        cpu = {"value": round(c["gbs"], 3), "unit": "GB/s", "cores": c["cores"], "nproc": os.cpu_count(), "kind": "port",
               "sample": c["sample"]}

    collective_point(4)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        if isinstance(wl, LoadCheckpoint):
            wl.close()
        return

    peak, peak_kind = load_peaks()
    dom = wl.dominant
    dom_ms = kern_ms[dom]
    achieved = wl.kernel_bytes[dom] / (dom_ms / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": round(value_gbs, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32" if wl.name == "rms_norm_f32" else "bf16 (fp32 math)",
        "data": getattr(wl, "data", "synthetic (seeded, generated on device)"),
        "config": wl.config if isinstance(wl, Chain) else dict(wl.config, parallelism=f"{world} row shards, no collective"),
        "pct_of_peak": round(100 * value_gbs / (world * peak), 2), "rows_per_s": round(rows_per_s, 1),
        "effective_gbs": round(world * wl.footprint / (ms_step / 1e3) / 1e9, 3),
        "per_kernel": {k: {"us": round(kern_ms[k] * 1e3, 2),
                           "gbs": round(wl.kernel_bytes[k] / (kern_ms[k] / 1e3) / 1e9, 1)} for k in wl.kernels},
        "roofline": {"kernel": dom, "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "bytes_per_launch": wl.kernel_bytes[dom],
                     "traffic": load_traffic(dom, wl.name)},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
    }
    if per_rank_ms is not None:
        line["per_rank_ms_per_step"] = per_rank_ms  # each rank's own device time; value uses the max
    if decode is not None:
        (in_graph, in_range), (alone, alone_range) = decode
        # per 4-launch chain inside a graph of 50 chains (median of 5 repetitions)
        line["decode_64_tokens_us"] = round(in_graph, 2)
        line["decode_64_tokens_us_range"] = [round(v, 2) for v in in_range]
        # a one-chain graph replayed alone: bound by the host's graph-launch rate
        line["decode_64_tokens_graph_alone_us"] = round(alone, 2)
        line["decode_64_tokens_graph_alone_us_range"] = [round(v, 2) for v in alone_range]
    if e2e is not None:
        line["e2e"] = e2e
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    if isinstance(wl, LoadCheckpoint):
        wl.close()


if __name__ == "__main__":
    main()
