"""Data parallelism on two GPUs through the library's collectives (needs 2 GPUs).

Two ranks (one process per GPU, NCCL under the C ABI, NVLS off) train the same
small GPT from the same initial parameters on different token batches:

* replicated: the gradient of each finished backward segment is all-reduced
  (GradSync) and every rank runs the full Adam step with grad_scale 1/2 — the
  reference's crossReplicaMean (Sources/Core/Distributed.swift:59-64);
* sharded (ZeRO stage 1): the segments are reduce-scattered (ShardSync), each
  rank runs Adam on its half, the parameters are all-gathered.

After three steps both ranks of each mode hold identical parameters, and the
two modes agree to F32 rounding of the summation order (1e-6 of the norm).
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two GPUs")]

KW = dict(vocab=300, seq=128, layers=4, heads=2, dim=128, tied=True)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE="2", LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        import torch.distributed as dist

        from magma_b200 import dp
        from magma_b200.gpt import GPTConfig, GPTTrainer

        dp.init_from_env(backend="nccl", timeout_s=60)
        torch.cuda.set_device(rank)
        comm = dp.Comm.from_process_group(timeout_ms=60_000)
        g = torch.Generator().manual_seed(100 + rank)
        tok = torch.randint(0, KW["vocab"], (2, KW["seq"]), generator=g, dtype=torch.int32)
        tgt = torch.randint(0, KW["vocab"], (2, KW["seq"]), generator=g, dtype=torch.int32)
        out = {}
        for mode in ("replicated", "sharded"):
            tr = GPTTrainer(GPTConfig(**KW), 2, "bf16", lr=1e-3, seed=0, weight_decay=0.1,
                            grad_clip=0.5)
            tr.set_batch(tok, tgt)
            tr.capture()
            sync = dp.GradSync(comm=comm) if mode == "replicated" else dp.ShardSync(comm)
            for _ in range(3):
                scale = tr.run_fwd_bwd(sync=sync)
                if mode == "replicated":
                    tr.optimizer_step(grad_scale=scale)
                else:
                    tr.optimizer_step_sharded(sync)
            torch.cuda.synchronize()
            out[mode] = tr.params.cpu().numpy()
            out[mode + "_loss"] = float(tr.loss.item())
        comm.destroy()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, out))
    except Exception as e:  # reported to the parent
        import traceback

        q.put((rank, traceback.format_exc() + repr(e)))


def test_two_gpu_replicated_and_sharded_steps_agree():
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            rank, out = q.get(timeout=300)
            res[rank] = out
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, out in res.items():
        assert isinstance(out, dict), out
    a, b = res[0], res[1]
    # replicas stay in sync in both modes
    assert np.array_equal(a["replicated"], b["replicated"])
    assert np.array_equal(a["sharded"], b["sharded"])
    # the two modes agree to the summation order
    d = np.linalg.norm(a["sharded"].astype(np.float64) - a["replicated"])
    assert d <= 1e-6 * np.linalg.norm(a["replicated"].astype(np.float64)), d
    # and the step changed the parameters
    assert a["replicated_loss"] == pytest.approx(a["sharded_loss"], rel=1e-5)
