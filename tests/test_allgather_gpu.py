"""The row-sharded LM head with its logits all-gathered over NVLink peer stores
(arcllm_cuda_matvec_allgather, and its host-IO form): every rank's copy of the
logits equals the single-GPU matvec of the whole matrix bit for bit, the epoch-tagged words tell
consecutive launches apart, and a rank that never arrives ends the wait with
the device timeout flag (no hang, context still usable).

Multi-rank runs use one process per GPU (spawned), CUDA IPC for the exchange
buffers and gloo on the host only for the handle exchange; they are skipped
with fewer than two GPUs.  No test runs two waiting launches on one GPU.
"""
import ctypes as C
import datetime
import multiprocessing as mp
import socket

import numpy as np
import pytest

import arcllm_b200 as A

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from tests import gpu_util as G  # noqa: E402

K = 3584
NB = K // 256
RB = NB * A.Q6K_BLOCK_BYTES


def _plain(w_ptr, rows, x_ptr, sp):
    y = torch.empty(rows, dtype=torch.float32, device=torch.cuda.current_device())
    A.call("arcllm_cuda_matvec", A.GGML_Q6_K, w_ptr, rows, K, x_ptr, None, C.c_float(0.0), None, None,
           C.c_void_p(y.data_ptr()), sp)
    torch.cuda.synchronize()
    return y.cpu().numpy()


def _d2h(ptr, n):
    out = np.empty(n, np.float32)
    A.call("arcllm_cuda_memcpy_d2h", out.ctypes.data_as(C.c_void_p), C.c_void_p(ptr), 4 * n, None)
    A.call("arcllm_cuda_stream_synchronize", None)
    return out


def _device_error_bits():
    """Read and clear the device error word (the call's status is
    ARC_E_DEVICE_TIMEOUT when the timeout bit is set)."""
    bits = C.c_uint32(0)
    st = A.lib().arcllm_cuda_device_error(G.stream(), C.byref(bits))
    assert st in (0, 6), st
    assert (st == 6) == bool(bits.value & 1)
    return bits.value


def test_allgather_single_rank_equals_matvec():
    from arcllm_b200.rank_gather import RankGather
    rows, seed = 5000, 771
    sp = G.stream()
    w = G.empty_u8(rows * RB + 16)
    A.call("arcllm_cuda_fill_q6k", G.ptr(w), 0, rows * NB, seed, sp)
    x = G.empty_f32(K)
    A.call("arcllm_cuda_fill_normal_f32", G.ptr(x), 0, K, seed + 1, C.c_float(0.0), C.c_float(1.0), sp)
    ref = _plain(G.ptr(w), rows, G.ptr(x), sp)
    rg = RankGather(rows, 1, 0, lambda h: [h])
    try:
        for _ in range(3):  # epochs 1..3: the counter re-arms, the flag moves on
            rg.step(G.ptr(w), rows, K, G.ptr(x), 0, sp)
            torch.cuda.synchronize()
            got = _d2h(rg.logits_ptr, rows)
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
        assert _device_error_bits() == 0
    finally:
        rg.close()


def test_allgather_hostio_single_rank_equals_matvec():
    """arcllm_cuda_matvec_allgather_hostio: host x in, all logits in host memory.  A pinned y_host is
    written by the kernel's collect phase itself; a pageable one gets the gathered logits copied.  Both
    equal the plain matvec bit for bit, over consecutive epochs with a changing x."""
    from arcllm_b200.rank_gather import RankGather
    rows, seed = 5000, 774
    sp = G.stream()
    w = G.empty_u8(rows * RB + 16)
    A.call("arcllm_cuda_fill_q6k", G.ptr(w), 0, rows * NB, seed, sp)
    xd = G.empty_f32(K)
    xs = torch.empty(K, dtype=torch.float32).pin_memory()
    y_pinned = torch.full((rows,), float("nan"), dtype=torch.float32).pin_memory()
    y_pageable = np.full(rows, np.nan, np.float32)
    rg = RankGather(rows, 1, 0, lambda h: [h])
    try:
        for it in range(4):
            x = torch.from_numpy(np.random.default_rng(seed + it).standard_normal(K).astype(np.float32))
            xs.copy_(x)
            xref = G.empty_f32(K)
            xref.copy_(x.to(G.dev()))
            ref = _plain(G.ptr(w), rows, G.ptr(xref), sp)
            pinned = it % 2 == 0
            yh = C.c_void_p(y_pinned.data_ptr()) if pinned else y_pageable.ctypes.data_as(C.c_void_p)
            rg.step_hostio(G.ptr(w), rows, K, C.c_void_p(xs.data_ptr()), G.ptr(xd), 0, yh, sp)
            got = y_pinned.numpy() if pinned else y_pageable
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), "pinned" if pinned else "pageable"
        assert _device_error_bits() == 0
    finally:
        rg.close()


def test_allgather_wait_times_out_when_a_rank_never_arrives():
    """Rank 0 of two, with rank 1's buffer a local allocation that no kernel
    ever fills: rank 0's rows land in both buffers as epoch-1 words, the wait
    for rank 1's rows runs out after the 50 ms bound, the device error word
    reports it and the next launch works."""
    rows_total, rows, seed = 2048, 1024, 772
    sp = G.stream()
    w = G.empty_u8(rows * RB + 16)
    A.call("arcllm_cuda_fill_q6k", G.ptr(w), 0, rows * NB, seed, sp)
    x = G.empty_f32(K)
    A.call("arcllm_cuda_fill_normal_f32", G.ptr(x), 0, K, seed + 1, C.c_float(0.0), C.c_float(1.0), sp)
    ref = _plain(G.ptr(w), rows, G.ptr(x), sp)
    n = C.c_uint64(0)
    A.call("arcllm_cuda_allgather_buffer_bytes", rows_total, C.byref(n))
    bufs = [torch.zeros(n.value // 4 + 64, dtype=torch.float32, device=G.dev()) for _ in range(2)]
    ptrs = (C.c_void_p * 2)(*[(b.data_ptr() + 255) // 256 * 256 for b in bufs])
    assert _device_error_bits() == 0
    A.call("arcllm_cuda_matvec_allgather", A.GGML_Q6_K, G.ptr(w), rows, K, G.ptr(x), 0, rows_total, ptrs, 2, 0, 1,
           50000, sp)
    torch.cuda.synchronize()
    assert _device_error_bits() & 1, "the wait for rank 1's rows should have timed out"
    want = (np.uint64(1) << np.uint64(32)) | ref.view(np.uint32).astype(np.uint64)
    for p in ptrs:  # rank 0's rows were stored into both ranks' buffers before the wait
        words = _d2h(p, 2 * rows_total).view(np.uint64)
        assert np.array_equal(words[:rows], want)
        assert not words[rows:].any()  # rank 1 never stored its rows
    again = _plain(G.ptr(w), rows, G.ptr(x), sp)  # the context is still usable
    assert np.array_equal(again.view(np.uint32), ref.view(np.uint32))
    assert _device_error_bits() == 0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_worker(rank, world, port, rows_total, seed, q):
    try:
        import torch
        import torch.distributed as dist

        from arcllm_b200.rank_gather import RankGather
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        sp = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        dev = torch.device("cuda", rank)
        rows = rows_total // world
        row0 = rank * rows
        w = torch.empty(rows * RB + 16, dtype=torch.uint8, device=dev)
        A.call("arcllm_cuda_fill_q6k", C.c_void_p(w.data_ptr()), row0 * NB, rows * NB, seed, sp)
        x = torch.empty(K, dtype=torch.float32, device=dev)
        A.call("arcllm_cuda_fill_normal_f32", C.c_void_p(x.data_ptr()), 0, K, seed + 1, C.c_float(0.0),
               C.c_float(1.0), sp)
        wf = torch.empty(rows_total * RB + 16, dtype=torch.uint8, device=dev)
        A.call("arcllm_cuda_fill_q6k", C.c_void_p(wf.data_ptr()), 0, rows_total * NB, seed, sp)
        ref = _plain(C.c_void_p(wf.data_ptr()), rows_total, C.c_void_p(x.data_ptr()), sp)

        def exchange(h):
            out = [None] * world
            dist.all_gather_object(out, h)
            return out

        rg = RankGather(rows_total, world, rank, exchange, timeout_us=5000000)
        dist.barrier()
        ok = True
        for _ in range(4):
            rg.step(C.c_void_p(w.data_ptr()), rows, K, C.c_void_p(x.data_ptr()), row0, sp)
            torch.cuda.synchronize()
            got = _d2h(rg.logits_ptr, rows_total)
            ok = ok and np.array_equal(got.view(np.uint32), ref.view(np.uint32))
            dist.barrier()  # no rank starts the next epoch while another still reads these logits
        # the host-IO form: host x in, every rank's rows stored into this rank's pinned host logits
        xh = torch.empty(K, dtype=torch.float32).pin_memory()
        xh.copy_(x.cpu())
        yh = torch.full((rows_total,), float("nan"), dtype=torch.float32).pin_memory()
        xd = torch.empty(K, dtype=torch.float32, device=dev)
        for _ in range(2):
            rg.step_hostio(C.c_void_p(w.data_ptr()), rows, K, C.c_void_p(xh.data_ptr()), C.c_void_p(xd.data_ptr()),
                           row0, C.c_void_p(yh.data_ptr()), sp)
            ok = ok and np.array_equal(yh.numpy().view(np.uint32), ref.view(np.uint32))
            dist.barrier()
        bits = C.c_uint32(0)
        A.lib().arcllm_cuda_device_error(sp, C.byref(bits))
        dist.barrier()
        rg.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ok, bits.value, ""))
    except Exception as e:  # reported to the parent
        q.put((rank, False, -1, repr(e)))


@pytest.mark.parametrize("world", [2])
def test_allgather_ranks_on_separate_gpus(world):
    if torch.cuda.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_worker, args=(r, world, port, 6016, 773, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = sorted(q.get(timeout=300) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, ok, bits, msg in res:
        assert msg == "", "rank %d: %s" % (rank, msg)
        assert bits == 0, "rank %d device error %#x" % (rank, bits)
        assert ok, "rank %d logits differ from the single-GPU matvec" % rank


def test_stream_delay_waits_its_wall_clock_time():
    """The rendezvous delay of the multi-GPU bench: a 2 ms arcllm_cuda_stream_delay_us lasts at least
    2 ms by CUDA events on its stream and ends well within 10 ms."""
    s = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    A.call("arcllm_cuda_stream_delay_us", 10, C.c_void_p(s.cuda_stream))  # first launch loads the module
    a.record(s)
    A.call("arcllm_cuda_stream_delay_us", 2000, C.c_void_p(s.cuda_stream))
    b.record(s)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    assert 1.99 <= ms < 10.0, ms
