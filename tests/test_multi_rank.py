"""Multi-rank host logic on CPU: world_size-2 gloo process groups.

The sharded path has no data-path collective, so what needs testing is the
host logic: shard ranges, RoPE's sequence sharding through position_offset,
gathering shards for verification and the max-over-ranks timing reduction.
Each rank computes its shard with the oracle (CPU) and the gathered result
must equal the unsharded computation bit for bit.  A GPU variant
(test_multi_gpu.py) repeats this through the CUDA library on >= 2 GPUs.
"""

import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG, ROOT


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_row_range_partitions_exactly():
    from hrm_layer_ops.shard import row_range

    for total in (0, 1, 7, 8, 65536, 65537):
        for world in (1, 2, 3, 4, 8):
            spans = [row_range(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        row_range(10, 2, 2)


def test_rope_shard_modes():
    from hrm_layer_ops.shard import rope_shard

    s = rope_shard(batch=8, seq=4096, position_offset=0, world=4, rank=3)
    assert (s.b0, s.b1, s.s0, s.s1, s.position_offset) == (6, 8, 0, 4096, 0)
    s = rope_shard(batch=1, seq=100, position_offset=7, world=4, rank=2)
    assert (s.b0, s.b1, s.s0, s.s1, s.position_offset) == (0, 1, 50, 75, 57)


def _worker(rank, world, port, result_q):
    sys.path[:0] = [ROOT, PKG]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from hrm_layer_ops.shard import checksum, gather_rows, max_over_ranks, rope_shard, row_range
        from oracle import Oracle, f32_to_bf16

        o = Oracle()
        o.set_threads(1)
        rng = np.random.default_rng(5)  # same global inputs on every rank
        x = f32_to_bf16(rng.standard_normal((37, 256)).astype(np.float32))
        b = f32_to_bf16(rng.standard_normal((37, 256)).astype(np.float32))
        w = f32_to_bf16((1 + 0.1 * rng.standard_normal(256)).astype(np.float32))
        q = f32_to_bf16(rng.standard_normal((1, 2, 50, 64)).astype(np.float32))
        k = f32_to_bf16(rng.standard_normal((1, 2, 50, 64)).astype(np.float32))

        r0, r1 = row_range(37, world, rank)
        r, y = o.add_rms_norm(x[r0:r1], b[r0:r1], w, 1e-5)
        full_y = gather_rows(torch.from_numpy(y.view(np.int16)), 37).numpy().view(np.uint16)
        full_r = gather_rows(torch.from_numpy(r.view(np.int16)), 37).numpy().view(np.uint16)

        sh = rope_shard(1, 50, 3, world, rank)     # batch 1 < world: split along seq
        qs, _ = o.rope_embed(q[:, :, sh.s0:sh.s1], k[:, :, sh.s0:sh.s1], sh.position_offset)
        qs_t = torch.from_numpy(np.ascontiguousarray(qs.transpose(2, 0, 1, 3)).view(np.int16))  # seq-major rows
        full_q = gather_rows(qs_t, 50).numpy().view(np.uint16).transpose(1, 2, 0, 3)

        t_max = max_over_ranks(1.0 + rank)
        sums = [None] * world
        dist.all_gather_object(sums, checksum(torch.from_numpy(y.view(np.int16))))
        if rank == 0:
            wr, wy = o.add_rms_norm(x, b, w, 1e-5)
            wq, _ = o.rope_embed(q, k, 3)
            result_q.put(dict(y_ok=bool(np.array_equal(full_y, wy)), r_ok=bool(np.array_equal(full_r, wr)),
                              q_ok=bool(np.array_equal(full_q, wq)), t_max=t_max,
                              sums_ok=sums[0] == checksum(torch.from_numpy(wy[r0:r1].view(np.int16)))))
    finally:
        dist.destroy_process_group()


def test_gloo_world2_sharded_equals_unsharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = q.get(timeout=5)
    assert res == dict(y_ok=True, r_ok=True, q_ok=True, t_max=2.0, sums_ok=True), res


def _dying_worker(rank, world, port, result_q):
    """Rank 1 raises before the collective; rank 0 must get an error, not hang."""
    import datetime
    import time

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # a rank that dies between steps, with nothing in flight
    t0 = time.time()
    try:
        t = torch.ones(1)
        dist.all_reduce(t)
        result_q.put(("no error", time.time() - t0))
    except Exception as e:  # noqa: BLE001 - any error is the detection we want
        result_q.put((type(e).__name__, time.time() - t0))
    result_q.close()
    result_q.join_thread()  # flush before the hard exit
    os._exit(0)


def test_gloo_dead_rank_is_detected_within_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    assert procs[1].exitcode == 3
    kind, waited = q.get(timeout=5)
    assert kind != "no error" and waited < 60, (kind, waited)


def test_peer_monitor_declared_and_silent_failures():
    """In one process over a HashStore: a declared failure is reported at once;
    a missing heartbeat at the deadline."""
    import time

    from hrm_layer_ops.shard import PeerFailure, PeerMonitor

    st = dist.HashStore()
    m0, m1 = PeerMonitor(st, 0, 2), PeerMonitor(st, 1, 2)
    m1.beat(0)
    m0.sync(0, timeout_s=1)
    m1.fail("ValueError: injected")
    with pytest.raises(PeerFailure, match="injected") as e:
        m0.sync(1, timeout_s=30)
    assert e.value.ranks == [1]
    lone = PeerMonitor(dist.HashStore(), 0, 3)
    t0 = time.monotonic()
    with pytest.raises(PeerFailure, match="no heartbeat") as e:
        lone.sync(0, timeout_s=0.3)
    assert e.value.ranks == [1, 2] and time.monotonic() - t0 < 5


def _monitored_worker(rank, world, port, mode, result_q):
    """Step 0 completes on both ranks; then rank `mode`'s victim fails before
    step 1 (declared, silent, or the store-hosting rank 0 dies) and the
    survivor must raise PeerFailure before entering step 1's collective."""
    import datetime
    import time

    sys.path[:0] = [ROOT, PKG]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from hrm_layer_ops.shard import PeerFailure, PeerMonitor, max_over_ranks

    mon = PeerMonitor.for_default_group()
    mon.sync(0, timeout_s=30)
    max_over_ranks(float(rank))  # step 0's collective
    victim = 0 if mode == "host_dies" else 1
    if rank == victim:
        if mode == "declared":
            try:
                raise ValueError("injected failure in step 1")
            except ValueError as e:
                mon.fail(f"{type(e).__name__}: {e}")
        os._exit(3)
    t0 = time.monotonic()
    try:
        mon.sync(1, timeout_s=3)
        max_over_ranks(float(rank))
        result_q.put(("no failure", time.monotonic() - t0))
    except PeerFailure as e:
        result_q.put((e.reason, time.monotonic() - t0))
    result_q.close()
    result_q.join_thread()
    os._exit(0)


@pytest.mark.parametrize("mode", ["declared", "silent", "host_dies"])
def test_gloo_peer_failure_detected_before_the_collective(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_monitored_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    victim = 0 if mode == "host_dies" else 1
    assert procs[victim].exitcode == 3 and procs[1 - victim].exitcode == 0, [p.exitcode for p in procs]
    reason, waited = q.get(timeout=5)
    assert reason != "no failure"
    if mode == "declared":
        assert "injected failure" in reason and waited < 2.5, (reason, waited)
    else:
        assert waited < 10, (reason, waited)
