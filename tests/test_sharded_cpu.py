"""Host side of the N-sharded INT8 product, on CPU.

The shard split (mri_shard_rows) and the all-gather-then-concatenate
assembly are checked with world_size-2 gloo ranks that compute their shards
with the oracle; the assembled [m, N] result must equal the unsharded oracle
product bit for bit (each output element depends only on its own weight row
and the per-tensor activation scale, ops/matmul/int8.rs:113-143).
"""
import multiprocessing as mp
import socket

import numpy as np
import pytest

import shard_workers


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("n,p", [(28672, 8), (8192, 4), (11008, 2), (16, 1), (6, 3)])
def test_shard_rows_partition(mri, n, p):
    spans = [mri.shard_rows(n, p, r) for r in range(p)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    assert all(spans[i][1] == spans[i + 1][0] for i in range(p - 1))
    assert len({e - b for b, e in spans}) == 1


def test_shard_rows_errors(mri):
    with pytest.raises(mri.InvalidShape):
        mri.shard_rows(11008, 3, 0)
    with pytest.raises(ValueError):
        mri.shard_rows(16, 2, 2)
    with pytest.raises(ValueError):
        mri.shard_rows(16, 0, 0)


def test_comm_entry_points_without_gpu(mri):
    import torch
    if torch.cuda.is_available():
        pytest.skip("CPU-only check")
    assert isinstance(mri.comm_available(), bool)
    with pytest.raises((mri.CudaError, mri.CommError)):
        mri.Communicator(bytes(128), 1, 0, ctx=None)


@pytest.mark.parametrize("m", [1, 5])
def test_gloo_two_ranks_assemble_unsharded_product(oracle, m):
    n, k, seed = 96, 64, 7
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=shard_workers.gloo_shard_worker, args=(r, 2, port, m, n, k, seed, results))
             for r in range(2)]
    for p in procs:
        p.start()
    got = [results.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x, wq, ws = shard_workers.problem(m, n, k, seed)
    want = oracle.matmul_int8_from_f32(x, m, k, wq.reshape(-1), ws, n, k)
    spans = sorted(s for _, s, _ in got)
    assert spans == [(0, n // 2), (n // 2, n)]
    for _, _, full in got:
        np.testing.assert_array_equal(full, want)
