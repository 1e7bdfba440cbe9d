"""Host side of the tensor-parallel exchange (ExchangeBuffers in
arcllm_b200/rank_gather.py) and the exchange protocol, on CPU.

Two and four gloo ranks in spawned processes build ExchangeBuffers as the
tensor-parallel tests and bench.py do (handles swapped with
all_gather_object).  The CUDA library is replaced by a stand-in whose "device
memory" is POSIX shared memory and whose exchange follows the kernel's
protocol step by step (exchange.cu): sequence number = own counter + 1; the
slice stored into every rank's data region of that number's parity; the
number published in this rank's slot of every flag array; a wait until every
slot of its own array has reached it; the assembled vector copied out of its
own region.  The ranks run many exchanges back to back with no host barrier
in between, alternating slice layouts like the decode step (an 18944-word s,
a 3584-word hidden state, 4-word greedy records), so a rank that runs ahead
stores into its peers' buffers while they still copy out: every copied-out
vector must be exactly the one of its sequence number.  The device kernel
itself is covered by tests/test_tp_decode_gpu.py.
"""
import ctypes as C
import datetime
import multiprocessing as mp
import socket
import struct
import time

import numpy as np
import pytest

MAX_WORDS = 18944


class FakeLib:
    def __init__(self):
        from multiprocessing import shared_memory
        self._shm = shared_memory
        self.segments = {}

    def _addr(self, shm):
        return C.addressof(C.c_char.from_buffer(shm.buf))

    @staticmethod
    def _w(max_words):
        return (max_words + 3) & ~3

    def arcllm_cuda_exchange_buffer_bytes(self, max_words, out):
        out._obj.value = (2 * self._w(max_words) * 8 + 16 * 4 + 255) // 256 * 256
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

    def _begin(self, bufs, rank, max_words):
        """sequence number (counter + 1, every per-CTA counter advanced) and the region's word offset"""
        W = self._w(max_words)
        ctr = bufs[rank] + 16 * W
        seq = (struct.unpack("<I", C.string_at(ctr, 4))[0] + 1) & 0xFFFFFFFF
        C.memmove(ctr, struct.pack("<16I", *([seq] * 16)), 64)
        return seq, W * (seq & 1)

    @staticmethod
    def _store(bufs, n_ranks, region, at, words32, seq):
        tagged = (np.uint64(seq) << np.uint64(32)) | words32.astype(np.uint64)
        for q in range(n_ranks):  # into every rank's region of this parity
            C.memmove(bufs[q] + 8 * (region + at), tagged.ctypes.data, tagged.nbytes)

    @staticmethod
    def _collect(own, n, seq, timeout_us):
        """the n words at `own` once all carry seq (None on timeout)"""
        t0 = time.time()
        while True:
            w = np.frombuffer(C.string_at(own, 8 * n), np.uint64)
            if np.all((w >> np.uint64(32)) == np.uint64(seq)):
                return (w & np.uint64(0xFFFFFFFF)).astype(np.uint32)
            if time.time() - t0 > timeout_us * 1e-6:
                return None
            time.sleep(0.0002)

    def arcllm_cuda_exchange_gather(self, bufs, n_ranks, rank, max_words, src, n_local, off, dst, n_total,
                                    timeout_us, stream):
        seq, region = self._begin(bufs, rank, max_words)
        self._store(bufs, n_ranks, region, off, np.frombuffer(C.string_at(src, 4 * n_local), np.uint32), seq)
        vals = self._collect(bufs[rank] + 8 * region, n_total, seq, timeout_us)
        if vals is None:
            return 6
        C.memmove(dst, vals.ctypes.data, 4 * n_total)
        return 0

    def exchange_reduce(self, bufs, n_ranks, rank, max_words, src, n, residual, dst, timeout_us):
        """The reduce form: the whole vector into slot `rank`, then the slots summed in rank order."""
        seq, region = self._begin(bufs, rank, max_words)
        self._store(bufs, n_ranks, region, n * rank, np.frombuffer(C.string_at(src, 4 * n), np.uint32), seq)
        vals = self._collect(bufs[rank] + 8 * region, n * n_ranks, seq, timeout_us)
        if vals is None:
            return 6
        parts = vals.view(np.float32).reshape(n_ranks, n)
        t = parts[0].copy()
        for q in range(1, n_ranks):
            t = (t + parts[q]).astype(np.float32)
        out = (residual + t).astype(np.float32) if residual is not None else t
        C.memmove(dst, out.ctypes.data, 4 * n)
        return 0

    def call(self, name, *args):
        st = getattr(self, name)(*args)
        if st:
            raise RuntimeError("%s -> %d" % (name, st))
        return st


def _shard(n, world, rank, align=4):
    units = n // align
    base, extra = divmod(units, world)
    u0 = rank * base + min(rank, extra)
    return u0 * align, (base + (1 if rank < extra else 0)) * align


def _worker(rank, world, port, n_ex, q):
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

        ex = RG.ExchangeBuffers(MAX_WORDS, world, rank, exchange)
        bad = []
        for e in range(1, n_ex + 1):
            if e % 4 == 0:  # the all-reduce of the K-sharded down projection, between the gathers
                n = 3584
                part = (np.arange(n, dtype=np.float32) * np.float32(rank + 1) + np.float32(e)).astype(np.float32)
                res = np.full(n, 0.5, np.float32)
                out = np.zeros(n, np.float32)
                st = fake.exchange_reduce(ex.ptrs, world, rank, MAX_WORDS, part.ctypes.data, n, res, out.ctypes.data,
                                          20000000)
                want = np.zeros(n, np.float32)
                for r in range(world):
                    want = (want + (np.arange(n, dtype=np.float32) * np.float32(r + 1) + np.float32(e))).astype(
                        np.float32) if r else (np.arange(n, dtype=np.float32) * np.float32(r + 1) + np.float32(e))
                if st or not np.array_equal(out, (res + want).astype(np.float32)):
                    bad.append(e)
                continue
            n_total = (18944, 3584, 4 * world)[e % 3]
            if n_total == 4 * world:
                off, n_local = 4 * rank, 4
            else:
                off, n_local = _shard(n_total, world, rank)
            # the value of word i in exchange e, whoever stores it
            src = (np.arange(off, off + n_local, dtype=np.uint32) * 7 + np.uint32(e * 100003)).astype(np.uint32)
            dst = np.zeros(n_total, np.uint32)
            ex.gather(src.ctypes.data, n_local, off, dst.ctypes.data, n_total, None, timeout_us=20000000)
            want = (np.arange(n_total, dtype=np.uint32) * 7 + np.uint32(e * 100003)).astype(np.uint32)
            if not np.array_equal(dst, want):
                bad.append(e)
        dist.barrier()  # every rank's last exchange is done before the buffers go away
        ex.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, bad, ""))
    except Exception as exc:  # reported to the parent
        q.put((rank, None, repr(exc)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world", [2, 4])
def test_exchange_protocol_gloo_ranks_no_barriers(world):
    pytest.importorskip("torch")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 60, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = sorted(q.get(timeout=180) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for rank, bad, msg in res:
        assert msg == "", "rank %d: %s" % (rank, msg)
        assert bad == [], "rank %d: exchanges %s copied out a wrong vector" % (rank, bad)
