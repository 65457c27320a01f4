"""N-sharded INT8 product on the GPU (mri_sharded_matmul_int8_from_f32).

Bar: bit-exact against the oracle's unsharded product (proj_int8_par,
forward_int8.rs:87-96).  Each output element comes from the same kernels on
the same weight row and the same per-tensor activation scale; the NCCL
all-gather moves f32 values unchanged.
"""
import multiprocessing as mp
import time

import numpy as np
import pytest
import torch

import shard_workers

pytestmark = pytest.mark.gpu


def oracle_product(oracle, x, wq, ws, n, k):
    """proj_int8_par (forward_int8.rs:87-96): quantize_symmetric over the
    whole input, then matmul_int8_parallel (parallel.rs:308-346)."""
    m = x.shape[0]
    aq, s = oracle.quantize_symmetric(x)
    return oracle.matmul_int8_parallel(aq, s, wq.reshape(-1), ws, n, k, m)


@pytest.fixture(scope="module")
def comm1(mri, gpu_ctx):
    if not mri.comm_available():
        pytest.fail("libnccl.so.2 not loadable on the GPU box")
    c = mri.Communicator(mri.Communicator.unique_id(), 1, 0, ctx=gpu_ctx, timeout_ms=30000)
    yield c
    c.close()


@pytest.mark.parametrize("m", [1, 3, 8, 300, 1100])
def test_single_rank_matches_unsharded(mri, gpu_ctx, comm1, oracle, m):
    n, k = 1024, 512
    x, wq, ws = shard_workers.problem(m, n, k, 11 + m)
    shard = mri.shard_quantized_matrix(wq.reshape(-1), ws, n, k, comm1)
    xd = torch.from_numpy(x).cuda()
    want = oracle_product(oracle, x, wq, ws, n, k)
    got = mri.matmul_int8_from_f32_sharded(xd, shard, n, comm1)
    comm1.wait()
    gpu_ctx.synchronize()
    np.testing.assert_array_equal(got.cpu().numpy().view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("p", [2, 4, 8])
@pytest.mark.parametrize("m", [1, 6, 600])
def test_emulated_shards_concatenate_to_unsharded(mri, gpu_ctx, oracle, p, m):
    """P shards computed one after another on one GPU and concatenated along
    N equal the unsharded product (the per-rank math of the sharded call)."""
    n, k = 2048, 1024
    x, wq, ws = shard_workers.problem(m, n, k, 5 * p + m)
    xd = torch.from_numpy(x).cuda()
    parts = []
    for r in range(p):
        b, e = mri.shard_rows(n, p, r)
        w = mri.QuantizedMatrix(wq.reshape(-1), ws, n, k, ctx=gpu_ctx, rows=(b, e))
        parts.append(mri.matmul_int8_from_f32(xd, w).cpu().numpy())
    got = np.concatenate(parts, axis=1)
    want = oracle_product(oracle, x, wq, ws, n, k)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("m", [1, 300])
@pytest.mark.parametrize("which", ["gate_up", "down"])
def test_emulated_70b_shards_match_oracle(mri, gpu_ctx, oracle, which, m):
    """The Llama-70B FFN projections (gate/up W [28672, 8192], down W [8192,
    28672]) cut into the 8 shards of an 8-GPU node, each shard's product
    computed on this GPU, concatenated along N: the oracle's unsharded
    product bit for bit."""
    n, k = (28672, 8192) if which == "gate_up" else (8192, 28672)
    p = 8
    rng = np.random.default_rng(70 + m)
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    wq = rng.integers(-127, 128, size=n * k, dtype=np.int8)
    ws = rng.uniform(0.001, 0.02, size=n).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    parts = []
    for r in range(p):
        b, e = mri.shard_rows(n, p, r)
        w = mri.QuantizedMatrix(wq, ws, n, k, ctx=gpu_ctx, rows=(b, e))
        parts.append(mri.matmul_int8_from_f32(xd, w).cpu().numpy())
        del w
    got = np.concatenate(parts, axis=1)
    want = oracle_product(oracle, x, wq, ws, n, k)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def test_sharded_argument_errors(mri, gpu_ctx, comm1):
    n, k = 64, 32
    x, wq, ws = shard_workers.problem(2, n, k, 1)
    w = mri.shard_quantized_matrix(wq.reshape(-1), ws, n, k, comm1)
    xd = torch.from_numpy(x).cuda()
    with pytest.raises(mri.ShapeMismatch):
        mri.matmul_int8_from_f32_sharded(xd[:, :16].contiguous(), w, n, comm1)
    with pytest.raises(mri.ShapeMismatch):
        mri.matmul_int8_from_f32_sharded(xd, w, 2 * n, comm1)


def test_comm_init_times_out_when_peer_never_joins(mri, gpu_ctx):
    """Rank 1 of 2 never joins: creation gives up after the deadline with
    DeviceTimeout and aborts the communicator (host-side wait; no kernel)."""
    t0 = time.time()
    with pytest.raises(mri.DeviceTimeout):
        mri.Communicator(mri.Communicator.unique_id(), 2, 0, ctx=gpu_ctx, timeout_ms=1500)
    assert time.time() - t0 < 30


def _run_two(target, args):
    """Spawns ranks 0 and 1 as target(rank, 2, results, *args[, event])."""
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    extra = (ctx.Event(),) if target is shard_workers.peer_timeout_worker else ()
    procs = [ctx.Process(target=target, args=(r, 2, results) + args + extra) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(results.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    return got


@pytest.mark.parametrize("path", ["peer", "nccl", "default"])
def test_two_ranks_match_unsharded(mri, gpu_ctx, oracle, path):
    """Two GPUs, OPT_SHARD_PEER = 1 ("peer": m = 1 and 4 gathered by the
    streaming GEMV's epilogue, m = 300 by the tensor-core GEMM's epilogue
    over peer memory), 0 ("nccl": the NCCL all-gather, chunked for m = 300)
    or 2 ("default": NCCL for m <= 8, the GEMM's peer gather for m = 300);
    every rank's result equals the oracle's unsharded product bit for bit."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    n, k, seed, ms = 4096, 2048, 3, (1, 4, 300, 1, 300)
    peer = {"peer": 1, "nccl": 0, "default": 2}[path]
    got = _run_two(shard_workers.nccl_shard_worker, (mri.Communicator.unique_id(), ms, n, k, seed, peer))
    for r in range(2):
        assert not isinstance(got[r], str), got[r]
        for m in ms:
            x, wq, ws = shard_workers.problem(m, n, k, seed + m)
            # proj_int8_par (forward_int8.rs:87-96): quantize_symmetric over
            # the whole input, then matmul_int8_parallel.
            aq, s = oracle.quantize_symmetric(x)
            want = oracle.matmul_int8_parallel(aq, s, wq.reshape(-1), ws, n, k, m)
            np.testing.assert_array_equal(got[r][m].view(np.uint32), want.view(np.uint32))


def test_peer_gather_wait_is_bounded(mri):
    """A rank that skips a call: the other rank's gather kernel stops waiting
    after its budget and the host sees DeviceTimeout (no GPU fault, no hang)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    got = _run_two(shard_workers.peer_timeout_worker, (mri.Communicator.unique_id(), 2048, 1024))
    assert got[0] == "timeout", got
    assert got[1] == "idle", got
