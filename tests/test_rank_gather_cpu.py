"""Host side of the multi-GPU LM head (arcllm_b200/rank_gather.py) on CPU:
two and four gloo ranks in spawned processes build RankGather exactly as bench.py does
(handles swapped with all_gather_object), with the CUDA library replaced by a
stand-in whose "device memory" is POSIX shared memory, whose IPC handles name
those segments, and whose all-gather matvec follows the kernel's protocol
(store this rank's rows as 64-bit (epoch << 32 | fp32 bits) words into every
rank's buffer of the launch's parity, then read its own buffer's words until
all carry the epoch and copy their values into the logits).

Checked: the handle exchange and peer mapping, the buffer layout (the logits
after the words at a 256-byte boundary), the epoch parity that alternates the
two buffers, logits_ptr, and close().  The device kernel itself is covered by
tests/test_allgather_gpu.py.
"""
import ctypes as C
import datetime
import multiprocessing as mp
import socket
import time

import numpy as np
import pytest

ROWS_TOTAL = 1000  # 2 x 500 or 4 x 250 rows; logits at align256(8000) = 8192


class FakeLib:
    """The entry points RankGather uses, over shared-memory segments."""

    def __init__(self):
        from multiprocessing import shared_memory
        self._shm = shared_memory
        self.segments = {}  # address -> SharedMemory (own and opened)

    def _addr(self, shm):
        return C.addressof(C.c_char.from_buffer(shm.buf))

    def _logits_off(self, rows_total):
        return (8 * rows_total + 255) // 256 * 256

    def arcllm_cuda_allgather_buffer_bytes(self, rows_total, out):
        out._obj.value = self._logits_off(rows_total) + (4 * rows_total + 255) // 256 * 256
        return 0

    def arcllm_cuda_allgather_logits_offset(self, rows_total, out):
        out._obj.value = self._logits_off(rows_total)
        return 0

    def arcllm_cuda_malloc(self, nbytes, out):
        shm = self._shm.SharedMemory(create=True, size=int(nbytes))
        a = self._addr(shm)
        self.segments[a] = shm
        out._obj.value = a
        return 0

    def arcllm_cuda_memcpy_h2d(self, dst, src, nbytes, stream):
        C.memmove(dst.value, src.value, int(nbytes))
        return 0

    def arcllm_cuda_stream_synchronize(self, stream):
        return 0

    def arcllm_cuda_ipc_get_handle(self, ptr, handle):
        name = self.segments[ptr.value].name.encode()
        C.memmove(handle.value, name + b"\0" * (64 - len(name)), 64)
        return 0

    def arcllm_cuda_ipc_open_handle(self, handle, out):
        name = C.string_at(handle.value, 64).rstrip(b"\0").decode()
        shm = self._shm.SharedMemory(name=name)
        a = self._addr(shm)
        self.segments[a] = shm
        out._obj.value = a
        return 0

    def arcllm_cuda_ipc_close_handle(self, ptr):
        self.segments.pop(ptr.value).close()
        return 0

    def arcllm_cuda_free(self, ptr):
        shm = self.segments.pop(ptr.value)
        shm.close()
        shm.unlink()
        return 0

    def arcllm_cuda_matvec_allgather(self, ggml_type, w, rows, k, x, row0, rows_total, bufs, n_ranks, rank, epoch,
                                     timeout_us, stream):
        y = (np.arange(row0, row0 + rows, dtype=np.float32) + np.float32(1000 * epoch))
        words = (np.uint64(epoch) << np.uint64(32)) | y.view(np.uint32).astype(np.uint64)
        for r in range(n_ranks):  # tagged rows into every rank's buffer of this parity
            C.memmove(bufs[r] + 8 * row0, words.ctypes.data, 8 * rows)
        t0 = time.time()
        while True:  # every word of our own buffer carries the epoch
            got = np.frombuffer(C.string_at(bufs[rank], 8 * rows_total), np.uint64)
            if np.all((got >> np.uint64(32)) == np.uint64(epoch)):
                vals = (got & np.uint64(0xFFFFFFFF)).astype(np.uint32)
                C.memmove(bufs[rank] + self._logits_off(rows_total), vals.ctypes.data, 4 * rows_total)
                return 0
            if time.time() - t0 > timeout_us * 1e-6:
                return 6
            time.sleep(0.001)

    def call(self, name, *args):
        st = getattr(self, name)(*args)
        if st:
            raise RuntimeError("%s -> %d" % (name, st))
        return st


def _worker(rank, world, port, q):
    try:
        import torch.distributed as dist

        import arcllm_b200.rank_gather as RG
        fake = FakeLib()
        RG.call = fake.call
        RG.lib = lambda: fake
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))

        def exchange(h):
            out = [None] * world
            dist.all_gather_object(out, h)
            return out

        rg = RG.RankGather(ROWS_TOTAL, world, rank, exchange, timeout_us=20000000)
        rows = ROWS_TOTAL // world
        seen = []
        for e in range(1, 6):
            rg.step(None, rows, 256, None, rank * rows, None)
            got = np.frombuffer(C.string_at(rg.logits_ptr, 4 * ROWS_TOTAL), np.float32)
            want = np.arange(ROWS_TOTAL, dtype=np.float32) + np.float32(1000 * e)
            seen.append((rg.epoch, bool(np.array_equal(got, want)),
                         rg.logits_ptr == rg._own[e & 1].value + fake._logits_off(ROWS_TOTAL)))
            dist.barrier()  # nobody runs the next epoch while another still reads these logits
        dist.barrier()
        rg.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, seen, ""))
    except Exception as ex:  # reported to the parent
        q.put((rank, [], repr(ex)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world", [2, 4])
def test_rank_gather_host_protocol_gloo_ranks(world):
    pytest.importorskip("torch")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = sorted(q.get(timeout=120) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for rank, seen, msg in res:
        assert msg == "", "rank %d: %s" % (rank, msg)
        assert [s[0] for s in seen] == [1, 2, 3, 4, 5]
        assert all(s[1] for s in seen), "rank %d: gathered logits wrong" % rank
        assert all(s[2] for s in seen), "rank %d: logits_ptr not the buffer of the epoch's parity" % rank
