"""Data-parallel host logic on CPU: two gloo ranks, each with its shard.

Each rank takes its contiguous shard of one global batch (``shard_batch``),
computes GPT gradients on it with the oracle, and sums them over the process
group with ``GradSync`` in small buckets; the returned 1/world scale turns the
sum into the mean, as ``crossReplicaMean`` (Sources/Core/Distributed.swift:55-64)
and its lowering ``all_reduce(add)`` then ``× 1/n``
(Sources/StableHLO/Builder/MLIRBuilder.swift:923-929) do. The result must equal
the oracle's own all-reduce-mean of the shard gradients bit for bit, and the
full-batch gradient to float rounding.
"""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

CFG = dict(vocab=61, seq=16, layers=2, heads=2, dim=32)
WORLD = 2
BATCH = 4


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(oracle):
    cfg = oracle.gpt_config(CFG["vocab"], CFG["seq"], CFG["layers"], CFG["heads"], CFG["dim"])
    rng = np.random.default_rng(7)
    params = (rng.standard_normal(oracle.gpt_param_count(cfg)) * 0.05).astype(np.float32)
    tokens = rng.integers(0, CFG["vocab"], (BATCH, CFG["seq"] + 1)).astype(np.int32)
    return cfg, params, tokens


def _rank_main(rank, port, bucket_bytes, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(WORLD), LOCAL_RANK=str(rank))
    import torch
    import torch.distributed as dist

    from magma_b200 import dp
    from oracle import oracle

    try:
        r, w, _ = dp.init_from_env(backend="gloo", timeout_s=60)
        assert (r, w) == (rank, WORLD)
        cfg, params, tokens = _problem(oracle)
        shard = dp.shard_batch(torch.from_numpy(tokens), r, w).numpy()
        loss, grads = oracle.gpt_fwd_bwd(cfg, params, shard[:, :-1], shard[:, 1:])
        g = torch.from_numpy(grads.copy())
        scale = dp.GradSync(bucket_bytes=bucket_bytes)(g)
        # the segmented form (launch per finished range, then finish) sums the same
        g2 = torch.from_numpy(grads.copy())
        sync = dp.GradSync(bucket_bytes=bucket_bytes)
        k = g2.numel() // 3
        sync.launch(g2[k:])
        sync.launch(g2[:k])
        assert sync.finish() == scale and torch.equal(g2, g)
        out_q.put((rank, loss, grads, (g * scale).numpy(), scale))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent, which fails the test
        out_q.put((rank, repr(e), None, None, None))


@pytest.mark.parametrize("bucket_bytes", [256 << 20, 4096])
def test_gradsync_two_gloo_ranks_equals_oracle_mean(oracle, bucket_bytes):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, bucket_bytes, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(WORLD):
            rank, loss, local, synced, scale = q.get(timeout=240)
            assert local is not None, f"rank {rank} failed: {loss}"
            res[rank] = (loss, local, synced, scale)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    assert res[0][3] == res[1][3] == 1.0 / WORLD
    want = oracle.allreduce_mean([res[0][1], res[1][1]])
    for r in range(WORLD):
        assert np.array_equal(res[r][2], want), f"rank {r} differs from the oracle mean"

    cfg, params, tokens = _problem(oracle)
    full_loss, full = oracle.gpt_fwd_bwd(cfg, params, tokens[:, :-1], tokens[:, 1:])
    assert abs((res[0][0] + res[1][0]) / 2 - full_loss) < 1e-5 * abs(full_loss)
    err = np.linalg.norm(res[0][2] - full) / np.linalg.norm(full)
    assert err < 1e-5


def test_shard_batch_contiguous_split():
    import torch

    from magma_b200 import dp

    g = torch.arange(8 * 3).view(8, 3)
    parts = [dp.shard_batch(g, r, 4) for r in range(4)]
    assert torch.equal(torch.cat(parts), g)
    assert all(p.shape == (2, 3) for p in parts)


def test_gradsync_single_process_is_noop():
    import torch

    from magma_b200 import dp

    g = torch.ones(10)
    assert dp.GradSync()(g) == 1.0
    assert torch.equal(g, torch.ones(10))
