"""Worker processes for the multi-rank sharding tests (spawned, not collected).

gloo_shard_worker is the CPU mirror of the sharded INT8 product: each rank
computes its N-shard with the oracle (per-tensor activation scale over the
whole input, as every rank of the GPU path does), the ranks all-gather the
[m, N/P] slices over gloo and concatenate them along N.

nccl_shard_worker runs the GPU path (mri_sharded_matmul_int8_from_f32) on
one GPU per rank with a communicator made from a unique id passed in by the
parent.
"""
import datetime
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
for p in (REPO, HERE, os.path.join(REPO, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def problem(m, n, k, seed):
    rng = np.random.default_rng(seed)
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    wq = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, size=n).astype(np.float32)
    return x, wq, ws


def gloo_shard_worker(rank, world, port, m, n, k, seed, results):
    import torch
    import torch.distributed as dist

    import oracle
    from conftest import load_mri

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        mri = load_mri()
        x, wq, ws = problem(m, n, k, seed)
        b, e = mri.shard_rows(n, world, rank)
        part = oracle.matmul_int8_from_f32(x, m, k, wq[b:e].reshape(-1), ws[b:e], e - b, k)
        parts = [torch.empty(m, e - b) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(part))
        results.put((rank, (b, e), torch.cat(parts, dim=1).numpy()))
    finally:
        dist.destroy_process_group()


def nccl_shard_worker(rank, world, results, uid, ms, n, k, seed, peer=0):
    """Runs the sharded product for every m in `ms` (same sequence on every
    rank) and reports {m: output}.  `peer` is the context's OPT_SHARD_PEER
    (0: small m gathered by NCCL, 1: over peer memory)."""
    import torch

    from conftest import load_mri

    try:
        mri = load_mri()
        torch.cuda.set_device(rank)
        ctx = mri.Context(rank)
        ctx.set_option(mri.OPT_SHARD_PEER, peer)
        comm = mri.Communicator(uid, world, rank, ctx=ctx, timeout_ms=60000)
        outs = {}
        for m in ms:
            x, wq, ws = problem(m, n, k, seed + m)
            w = mri.shard_quantized_matrix(wq.reshape(-1), ws, n, k, comm)
            out = mri.matmul_int8_from_f32_sharded(torch.from_numpy(x).cuda(rank), w, n, comm)
            comm.wait()
            outs[m] = out.cpu().numpy()
        results.put((rank, outs))
        comm.close()
    except Exception as e:  # noqa: BLE001 - reported to the parent
        results.put((rank, repr(e)))


def peer_timeout_worker(rank, world, results, uid, n, k, done):
    """Both ranks run one gathered product; then rank 0 runs a second one that
    rank 1 skips.  Rank 0's kernel must give up waiting for rank 1's arrivals
    (bounded wait) and report a timeout.  Rank 1 stays alive, with its buffers
    mapped and no work in flight, until rank 0 is done."""
    import torch

    from conftest import load_mri

    try:
        mri = load_mri()
        torch.cuda.set_device(rank)
        ctx = mri.Context(rank)
        ctx.set_option(mri.OPT_SHARD_PEER, 1)
        comm = mri.Communicator(uid, world, rank, ctx=ctx, timeout_ms=60000)
        x, wq, ws = problem(1, n, k, 5)
        w = mri.shard_quantized_matrix(wq.reshape(-1), ws, n, k, comm)
        xd = torch.from_numpy(x).cuda(rank)
        mri.matmul_int8_from_f32_sharded(xd, w, n, comm)
        comm.wait()
        if rank == 0:
            mri.matmul_int8_from_f32_sharded(xd, w, n, comm)
            try:
                comm.wait()
                results.put((rank, "no timeout"))
            except mri.DeviceTimeout:
                results.put((rank, "timeout"))
            done.set()
        else:
            done.wait(120)
            results.put((rank, "idle"))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        results.put((rank, repr(e)))
        done.set()
