"""Collectives and events of the C ABI on one GPU (one rank).

With a single rank the reductions are identities, which checks the plumbing
(id, communicator, dtype and op mapping, stream ordering, teardown) through the
C ABI; the two-rank data-parallel behaviour is covered by the gloo CPU tests and
the multi-GPU bench. The bounded wait is checked on the host: a communicator
whose second rank never joins ends with MAGMA_DEADLINE_EXCEEDED.
"""
import ctypes as C
import subprocess
import sys
import textwrap

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _stream():
    return torch.cuda.current_stream().cuda_stream


def test_single_rank_collectives_and_events(cuda):
    from magma_b200 import lib

    uid = C.create_string_buffer(lib.COMM_ID_BYTES)
    lib.call("magma_comm_unique_id", uid, lib.COMM_ID_BYTES)
    comm = C.c_void_p()
    lib.call("magma_comm_init_rank", C.byref(comm), 1, 0, uid, 30000)
    try:
        n, r = C.c_int32(), C.c_int32()
        lib.call("magma_comm_size", comm, C.byref(n))
        lib.call("magma_comm_rank", comm, C.byref(r))
        assert (n.value, r.value) == (1, 0)
        lib.call("magma_comm_check", comm)
        x = torch.randn(1000, device="cuda")
        y = torch.empty_like(x)
        for op in (lib.REDUCE_SUM, lib.REDUCE_MAX, lib.REDUCE_MIN, lib.REDUCE_AVG):
            lib.call("magma_allreduce", x.data_ptr(), y.data_ptr(), x.numel(), lib.F32, op, comm,
                     _stream())
            torch.cuda.synchronize()
            assert torch.equal(x, y)
        xb = x.to(torch.bfloat16)
        lib.call("magma_allreduce", xb.data_ptr(), xb.data_ptr(), xb.numel(), lib.BF16,
                 lib.REDUCE_SUM, comm, _stream())
        z = torch.empty_like(x)
        lib.call("magma_reduce_scatter", x.data_ptr(), z.data_ptr(), x.numel(), lib.F32,
                 lib.REDUCE_SUM, comm, _stream())
        w = torch.empty_like(x)
        lib.call("magma_all_gather", z.data_ptr(), w.data_ptr(), z.numel(), lib.F32, comm,
                 _stream())
        # events: order a second stream after the first and time the work
        e0, e1 = C.c_void_p(), C.c_void_p()
        lib.call("magma_event_create", C.byref(e0), 1)
        lib.call("magma_event_create", C.byref(e1), 1)
        lib.call("magma_event_record", e0, _stream())
        big = torch.randn(1 << 24, device="cuda")
        big.mul_(2.0)
        lib.call("magma_event_record", e1, _stream())
        side = torch.cuda.Stream()
        lib.call("magma_stream_wait_event", side.cuda_stream, e1)
        with torch.cuda.stream(side):
            after = big.sum()
        lib.call("magma_event_synchronize", e1)
        done = C.c_int32()
        lib.call("magma_event_query", e1, C.byref(done))
        assert done.value == 1
        ms = C.c_float()
        lib.call("magma_event_elapsed_ms", e0, e1, C.byref(ms))
        assert ms.value > 0
        side.synchronize()
        assert torch.isfinite(after)
        torch.cuda.synchronize()
        assert torch.equal(w, x) and torch.equal(z, x)
        lib.call("magma_event_destroy", e0)
        lib.call("magma_event_destroy", e1)
        with pytest.raises(lib.MagmaError) as e:
            lib.call("magma_allreduce", x.data_ptr(), y.data_ptr(), x.numel(), lib.F32, 9, comm,
                     _stream())
        assert e.value.status == lib.INVALID_ARGUMENT
    finally:
        lib.call("magma_comm_destroy", comm)


def test_comm_init_waits_a_bounded_time_for_a_missing_rank(cuda, tmp_path):
    """Rank 0 of two, with rank 1 never started: the call returns
    DEADLINE_EXCEEDED after its timeout (run in a child process)."""
    code = textwrap.dedent("""
        import ctypes as C, sys, time
        sys.path.insert(0, %r)
        import torch
        torch.cuda.set_device(0)
        from magma_b200 import lib
        uid = C.create_string_buffer(lib.COMM_ID_BYTES)
        lib.call("magma_comm_unique_id", uid, lib.COMM_ID_BYTES)
        comm = C.c_void_p()
        t0 = time.time()
        try:
            lib.call("magma_comm_init_rank", C.byref(comm), 2, 0, uid, 1500)
            print("NO_ERROR")
        except lib.MagmaError as e:
            print("STATUS", e.status, round(time.time() - t0, 1))
    """) % str(__import__("pathlib").Path(__file__).resolve().parents[1])
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120,
                       env={**__import__("os").environ, "NCCL_NVLS_ENABLE": "0"})
    out = r.stdout.strip().splitlines()
    assert out and out[-1].startswith("STATUS"), (r.stdout, r.stderr[-2000:])
    from magma_b200 import lib

    status, secs = int(out[-1].split()[1]), float(out[-1].split()[2])
    assert status == lib.DEADLINE_EXCEEDED and secs < 30
