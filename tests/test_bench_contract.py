"""CPU: the benchmark's reference arm and its JSON line (no GPU needed).

`bench.py --impl reference` times the reference's path restated on the host
(the oracle) over whole passes of the GPU arm's workload and prints exactly
one JSON line with the metric, the CPU baseline and an e2e object; a
workload it does not cover prints an `unavailable` line and exits 0.  The arm
loads nothing of the library: neither the hrm_layer_ops package nor
libhrm_ops.so.
"""

import json
import os
import subprocess
import sys

import pytest

from conftest import ROOT


def run_bench(*args, timeout=600):
    env = dict(os.environ, OMP_NUM_THREADS="4")
    res = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                         timeout=timeout, env=env, cwd=ROOT)
    lines = [l for l in res.stdout.splitlines() if l.startswith("{")]
    return res, lines


def test_reference_arm_prints_one_contract_line():
    res, lines = run_bench("--impl", "reference", "--steps", "1", "--warmup", "3", "--tokens", "8192")
    assert res.returncode == 0, res.stderr[-2000:]
    assert len(lines) == 1, res.stdout[-2000:]
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 3
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["config"]["tokens_per_gpu"] == 8192 and d["config"]["qk_shape"] == [2, 4096, 16, 128]


def test_reference_arm_defaults_to_the_whole_gpu_workload():
    """Without --tokens both arms run the 65536-token pass, with the same config dict."""
    sys.path.insert(0, ROOT)
    import bench

    old = sys.argv
    try:
        sys.argv = ["bench.py", "--impl", "reference"]
        args = bench.parse_args()
    finally:
        sys.argv = old
    assert args.tokens == 65536 and args.qk_layout == "token"
    cfg = bench.chain_config(args.tokens, True, 1)
    assert cfg["tokens_per_gpu"] == 65536 and cfg["qk_shape"] == [16, 4096, 16, 128]


@pytest.mark.parametrize("workload", [["--tokens", "4096"], ["--workload", "rms_norm_f32"]])
def test_reference_arm_loads_nothing_of_the_library(workload):
    code = (
        "import sys, runpy\n"
        f"sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '3', *{workload!r}]\n"
        "runpy.run_path('bench.py', run_name='__main__')\n"
        "maps = open('/proc/self/maps').read()\n"
        "print('LOADED', [m for m in sys.modules if m.startswith('hrm_layer_ops')], 'libhrm_ops' in maps,"
        " 'liboracle' in maps)\n")
    env = dict(os.environ, OMP_NUM_THREADS="4")
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600, env=env,
                         cwd=ROOT)
    assert res.returncode == 0, res.stderr[-2000:]
    last = [l for l in res.stdout.splitlines() if l.startswith("LOADED")][-1]
    assert last == "LOADED [] False True", last


def test_bench_byte_counts_equal_the_library_s():
    sys.path.insert(0, ROOT)
    import bench
    from hrm_layer_ops.chain import CHAIN_KERNELS, algorithmic_bytes_per_token

    assert tuple(bench.CHAIN_KERNEL_NAMES) == tuple(CHAIN_KERNELS)
    for dims in ((2048, 16, 128, 5632), (1536, 12, 128, 4096), (64, 2, 16, 40)):
        assert bench.chain_bytes_per_token(*dims) == algorithmic_bytes_per_token(*dims)


def test_reference_arm_other_workload_is_unavailable():
    res, lines = run_bench("--impl", "reference", "--workload", "module", "--steps", "1", "--warmup", "3")
    assert res.returncode == 0, res.stderr[-2000:]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unavailable"]


def test_reference_arm_single_op_workload():
    """The CPU-runnable configuration (RMSNorm fp32 [4096 x 2048] + weight) through
    the oracle: one line with the GPU arm's config and byte count."""
    sys.path.insert(0, ROOT)
    import bench

    res, lines = run_bench("--impl", "reference", "--workload", "rms_norm_f32", "--steps", "2", "--warmup", "3")
    assert res.returncode == 0, res.stderr[-2000:]
    assert len(lines) == 1, res.stdout[-2000:]
    d = json.loads(lines[0])
    cfg, nbytes, rows = bench.single_op_spec("rms_norm_f32")
    assert d["impl"] == "reference" and d["value"] > 0 and d["dtype"] == "fp32"
    assert d["config"] == dict(cfg, l2=bench.single_op_l2_note(nbytes), parallelism="1 row shards, no collective")
    assert abs(d["rows_per_s"] * d["ms_per_step"] / 1e3 - rows) < 1 + 1e-3 * rows
    assert abs(d["value"] * d["ms_per_step"] * 1e6 - nbytes) < 1e-3 * nbytes


def test_warmup_below_three_is_refused():
    res, _ = run_bench("--warmup", "2", "--steps", "1", timeout=300)
    assert res.returncode != 0 and "warmup" in (res.stderr + res.stdout)


def test_reference_arm_at_the_reference_model_dims():
    res, lines = run_bench("--impl", "reference", "--dims", "hrm-text-1b", "--steps", "1", "--warmup", "3",
                           "--tokens", "4096")
    assert res.returncode == 0, res.stderr[-2000:]
    d = json.loads(lines[0])
    assert d["config"]["hidden"] == 1536 and d["config"]["intermediate"] == 4096


def test_dims_only_for_chain_and_module():
    res, _ = run_bench("--dims", "hrm-text-1b", "--workload", "swiglu", timeout=300)
    assert res.returncode != 0 and "--dims" in res.stderr


def test_reference_arm_under_torchrun_prints_on_rank_zero_only():
    """Launched as the multi-GPU bench is (torchrun, 2 ranks, 127.0.0.1), rank 0
    alone runs and prints its line (n_gpus = 2); the other rank exits 0."""
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, OMP_NUM_THREADS="4")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), os.path.join(ROOT, "bench.py"),
           "--impl", "reference", "--steps", "1", "--warmup", "3", "--tokens", "4096"]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [l for l in res.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, res.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0
