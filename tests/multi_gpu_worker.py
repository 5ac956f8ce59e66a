"""One rank of the multi-GPU sharding check (launched by test_multi_gpu.py via
torch.distributed.run, one process per GPU, NCCL).

Each rank computes its row shard of add_rms_norm and embed_rms_norm, and its
sequence shard of RoPE (position_offset = offset + s0), through the CUDA
library; the shards are all-gathered over NCCL and rank 0 compares them with
the same ops run unsharded on its own GPU.  Exit code 0 = identical.
"""

import datetime
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path[:0] = [ROOT, os.path.join(ROOT, "hrm-text-cuda_b200")]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import hrm_layer_ops as ops  # noqa: E402
from hrm_layer_ops.shard import gather_rows, max_over_ranks, rope_shard, row_range  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    g = torch.Generator(device=dev).manual_seed(99)  # identical global inputs on every rank
    R, H, V = 1000, 2048, 5000
    x = torch.randn((R, H), generator=g, device=dev).to(torch.bfloat16)
    b = torch.randn((R, H), generator=g, device=dev).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(H, generator=g, device=dev)).to(torch.bfloat16)
    table = (0.02 * torch.randn((V, H), generator=g, device=dev)).to(torch.bfloat16)
    ids = torch.randint(0, V, (R,), generator=g, device=dev, dtype=torch.int32)
    q = torch.randn((1, 16, 300, 128), generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn((1, 16, 300, 128), generator=g, device=dev).to(torch.bfloat16)

    r0, r1 = row_range(R, world, rank)
    r_s, y_s = ops.add_rms_norm(x[r0:r1], b[r0:r1], w, 1e-5)
    h_s, n_s = ops.embed_rms_norm(ids[r0:r1], table, 45.254834, w, 1e-5)
    sh = rope_shard(1, 300, 11, world, rank)
    qs, ks = q[:, :, sh.s0:sh.s1].contiguous(), k[:, :, sh.s0:sh.s1].contiguous()
    ops.rope_embed(qs, ks, sh.position_offset, 10000.0, None)

    full = {n: gather_rows(t, R) for n, t in (("r", r_s), ("y", y_s), ("h", h_s), ("n", n_s))}
    full_q = gather_rows(qs.permute(2, 0, 1, 3).contiguous(), 300).permute(1, 2, 0, 3)
    t = max_over_ranks(float(rank), dev)
    ok = True
    if rank == 0:
        r, y = ops.add_rms_norm(x, b, w, 1e-5)
        h, n = ops.embed_rms_norm(ids, table, 45.254834, w, 1e-5)
        ops.rope_embed(q, k, 11, 10000.0, None)
        for name, want in (("r", r), ("y", y), ("h", h), ("n", n), ("q", q)):
            got = full_q if name == "q" else full[name]
            same = torch.equal(got.view(torch.int16), want.view(torch.int16))
            print(f"{name}: {'identical' if same else 'DIFFERS'}")
            ok &= same
        ok &= t == float(world - 1)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


def dead_rank_main():
    """Failure detection over NCCL: both ranks run step 0 (a sharded
    add_rms_norm and the max-over-ranks all_reduce); rank 1 then leaves between
    steps, with nothing in flight, without a word; rank 0 runs step 1's kernels
    and must get PeerFailure from its heartbeat wait before it enters step 1's
    collective.  Launched as plain processes (not torch.distributed.run, whose
    agent would stop rank 0 as soon as rank 1 exits).  Prints 'detected: ...'."""
    import time

    from hrm_layer_ops.shard import PeerFailure, PeerMonitor

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=30), device_id=dev)
    mon = PeerMonitor.for_default_group()
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn((512, 2048), generator=g, device=dev).to(torch.bfloat16)
    b = torch.randn((512, 2048), generator=g, device=dev).to(torch.bfloat16)
    r0, r1 = row_range(512, world, rank)
    ops.add_rms_norm(x[r0:r1], b[r0:r1], None, 1e-5)
    torch.cuda.synchronize()
    mon.sync(0, timeout_s=30)
    max_over_ranks(1.0, dev)
    torch.cuda.synchronize()
    if rank == 1:
        os._exit(3)
    ops.add_rms_norm(x[r0:r1], b[r0:r1], None, 1e-5)
    torch.cuda.synchronize()
    t0 = time.monotonic()
    try:
        mon.sync(1, timeout_s=5)
        print("no failure detected", flush=True)
        os._exit(1)
    except PeerFailure as e:
        print(f"detected: {e} after {time.monotonic() - t0:.2f} s", flush=True)
        os._exit(0)


if __name__ == "__main__":
    if "--dead-rank" in sys.argv:
        dead_rank_main()
    else:
        main()
