"""The output-row-sharded prefill GEMM whose split-K reduce kernel all-gathers
the result over NVLink peer stores (arcllm_cuda_gemm_bf16_allgather,
GemmGather): with one rank it equals arcllm_cuda_gemm_q4k_bf16 bit for bit over
several epochs; a rank that never arrives ends the flag wait with the device
timeout bit (no hang); on two GPUs every rank's gathered m x n_total result
equals the plain single-GPU GEMMs of both shards, bit for bit.

Multi-rank runs use one process per GPU (spawned), CUDA IPC for the buffers
and gloo on the host only for the handle exchange; skipped with fewer than two
GPUs.  No test runs two waiting launches on one GPU.
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
RB = (K // 256) * A.Q4K_BLOCK_BYTES
M = 96


def _x(dev, seed):
    xf = torch.empty(M * K, dtype=torch.float32, device=dev)
    A.call("arcllm_cuda_fill_normal_f32", C.c_void_p(xf.data_ptr()), 0, M * K, seed, C.c_float(0.0), C.c_float(1.0),
           C.c_void_p(torch.cuda.current_stream().cuda_stream))
    return xf.to(torch.bfloat16)


def _w(dev, row0, rows, seed):
    w = torch.empty(rows * RB + 16, dtype=torch.uint8, device=dev)
    A.call("arcllm_cuda_fill_q4k", C.c_void_p(w.data_ptr()), row0 * (K // 256), rows * (K // 256), seed,
           C.c_void_p(torch.cuda.current_stream().cuda_stream))
    return w


def _plain(w, rows, x):
    y = torch.empty(M * rows, dtype=torch.float32, device=x.device)
    A.call("arcllm_cuda_gemm_q4k_bf16", C.c_void_p(w.data_ptr()), rows, K, C.c_void_p(x.data_ptr()), M,
           C.c_void_p(y.data_ptr()), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return y.view(M, rows)


def _d2h(ptr, n):
    out = np.empty(n, np.float32)
    A.call("arcllm_cuda_memcpy_d2h", out.ctypes.data_as(C.c_void_p), C.c_void_p(ptr), 4 * n, None)
    A.call("arcllm_cuda_stream_synchronize", None)
    return out


def _error_bits():
    bits = C.c_uint32(0)
    st = A.lib().arcllm_cuda_device_error(G.stream(), C.byref(bits))
    assert st in (0, 6), st
    return bits.value


def test_gemm_allgather_single_rank_equals_gemm():
    from arcllm_b200.rank_gather import GemmGather
    n = 1024  # 8 column tiles: split K over the SMs, as a shard at 8+ GPUs would be
    x, w = _x(G.dev(), 901), _w(G.dev(), 0, n, 902)
    ref = _plain(w, n, x).cpu().numpy()
    gg = GemmGather(M, n, 1, 0, lambda h: [h])
    try:
        for _ in range(3):
            gg.step(A.GGML_Q4_K, C.c_void_p(w.data_ptr()), n, K, C.c_void_p(x.data_ptr()), 0, G.stream())
            torch.cuda.synchronize()
            got = _d2h(gg.y_ptr, M * n).reshape(M, n)
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
        assert _error_bits() == 0
    finally:
        gg.close()


def test_gemm_allgather_wait_times_out_when_a_rank_never_arrives():
    """Rank 0 of two with rank 1's buffer a local allocation no kernel signals:
    rank 0's columns land in both buffers, the flag wait runs out after 50 ms
    and sets the timeout bit, and the context stays usable."""
    n, n_total = 512, 1024
    x, w = _x(G.dev(), 903), _w(G.dev(), 0, n, 904)
    ref = _plain(w, n, x).cpu().numpy()
    nb = C.c_uint64(0)
    A.call("arcllm_cuda_gemm_allgather_buffer_bytes", M, n_total, C.byref(nb))
    bufs = [torch.zeros(nb.value // 4 + 64, dtype=torch.float32, device=G.dev()) for _ in range(2)]
    ptrs = (C.c_void_p * 2)(*[(b.data_ptr() + 255) // 256 * 256 for b in bufs])
    assert _error_bits() == 0
    A.call("arcllm_cuda_gemm_bf16_allgather", A.GGML_Q4_K, C.c_void_p(w.data_ptr()), n, K, C.c_void_p(x.data_ptr()),
           M, 0, n_total, ptrs, 2, 0, 1, 50000, G.stream())
    torch.cuda.synchronize()
    assert _error_bits() & 1, "the flag wait should have timed out"
    for p in ptrs:  # rank 0's columns were stored into both ranks' results before the wait
        got = _d2h(p, M * n_total).reshape(M, n_total)
        assert np.array_equal(got[:, :n].view(np.uint32), ref.view(np.uint32))
    again = _plain(w, n, x).cpu().numpy()  # the context is still usable
    assert np.array_equal(again.view(np.uint32), ref.view(np.uint32))
    assert _error_bits() == 0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_worker(rank, world, port, n_total, q):
    try:
        import torch
        import torch.distributed as dist

        from arcllm_b200.rank_gather import GemmGather
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        dev = torch.device("cuda", rank)
        sp = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        r0, rr = C.c_uint32(0), C.c_uint32(0)
        shards = []
        for r in range(world):
            A.call("arcllm_cuda_shard_rows", n_total, 128, world, r, C.byref(r0), C.byref(rr))
            shards.append((r0.value, rr.value))
        c0, n = shards[rank]
        x = _x(dev, 905)
        w = _w(dev, c0, n, 906)
        refs = [_plain(_w(dev, a, b, 906), b, x).cpu().numpy() for a, b in shards]

        def exchange(h):
            out = [None] * world
            dist.all_gather_object(out, h)
            return out

        gg = GemmGather(M, n_total, world, rank, exchange, timeout_us=5000000)
        dist.barrier()
        ok = True
        for _ in range(4):
            gg.step(A.GGML_Q4_K, C.c_void_p(w.data_ptr()), n, K, C.c_void_p(x.data_ptr()), c0, sp)
            torch.cuda.synchronize()
            got = _d2h(gg.y_ptr, M * n_total).reshape(M, n_total)
            for (a, b), ref in zip(shards, refs):
                ok = ok and np.array_equal(got[:, a:a + b].view(np.uint32), ref.view(np.uint32))
            dist.barrier()  # no rank starts the next epoch while another still reads this result
        bits = C.c_uint32(0)
        A.lib().arcllm_cuda_device_error(sp, C.byref(bits))
        dist.barrier()
        gg.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ok, bits.value, ""))
    except Exception as e:  # reported to the parent
        q.put((rank, False, -1, repr(e)))


@pytest.mark.parametrize("world", [2])
def test_gemm_allgather_ranks_on_separate_gpus(world):
    if torch.cuda.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_worker, args=(r, world, port, 2048, q)) for r in range(world)]
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
        assert ok, "rank %d: gathered result differs from the single-GPU shards" % rank
