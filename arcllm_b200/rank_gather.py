"""Rank exchange buffers for the NVLink all-gather form of the LM-head matvec
(RankGather) and for the vector exchange of the tensor-parallel decode
(ExchangeBuffers).

One process per GPU.  Each rank allocates two exchange buffers (one per epoch
parity: the 64-bit epoch-tagged words of all rows, then the fp32 logits it
collects from them), shares CUDA IPC handles of them with the other ranks and
opens theirs, so that ``arcllm_cuda_matvec_allgather`` can store each rank's
rows into every rank's buffer with NVLink peer stores; each word carries its
own epoch, so the ranks need no separate flag handshake.  The handle
exchange itself is a host collective supplied by the caller
(``torch.distributed.all_gather_object`` in bench.py, a multiprocessing pipe in
the tests): the data path has no host collective and no NCCL call.

The reference runs its LM head on one device
(src/arcllm_v1_runtime.cpp:285-291); this is the row-sharded multi-GPU form of
that step.
"""
import ctypes as C

from . import GGML_Q6_K, call, lib

HANDLE_BYTES = 64  # cudaIpcMemHandle_t


class _ParityBuffers:
    """Two exchange buffers of `nbytes` per rank (one per epoch parity),
    zero-filled, shared with the other ranks through CUDA IPC handles
    (`exchange`: the caller's host all-gather of bytes) and mapped in this
    process; `_bufs[b]` is the rank-ordered array of device addresses of set b."""

    def _setup_buffers(self, nbytes, n_ranks, rank, exchange, what):
        if not (1 <= n_ranks <= 8 and 0 <= rank < n_ranks):
            raise ValueError("%s: 1 <= n_ranks <= 8 and 0 <= rank < n_ranks" % what)
        self.nbytes, self.n_ranks, self.rank = nbytes, n_ranks, rank
        self._own, self._opened, self._bufs = [], [], []
        zeros = (C.c_uint8 * self.nbytes)()
        handles = []
        for _ in range(2):
            own = C.c_void_p()
            call("arcllm_cuda_malloc", self.nbytes, C.byref(own))
            self._own.append(own)
            call("arcllm_cuda_memcpy_h2d", own, C.cast(zeros, C.c_void_p), self.nbytes, None)
            h = (C.c_uint8 * HANDLE_BYTES)()
            call("arcllm_cuda_ipc_get_handle", own, C.cast(h, C.c_void_p))
            handles.append(bytes(h))
        call("arcllm_cuda_stream_synchronize", None)
        everyone = exchange(handles[0] + handles[1])
        if len(everyone) != n_ranks:
            raise RuntimeError("%s: exchange returned %d entries for %d ranks" % (what, len(everyone), n_ranks))
        for b in range(2):
            ptrs = []
            for r, hb in enumerate(everyone):
                if r == rank:
                    ptrs.append(self._own[b].value)
                    continue
                p = C.c_void_p()
                raw = hb[b * HANDLE_BYTES:(b + 1) * HANDLE_BYTES]
                hbuf = (C.c_uint8 * HANDLE_BYTES).from_buffer_copy(raw)
                call("arcllm_cuda_ipc_open_handle", C.cast(hbuf, C.c_void_p), C.byref(p))
                self._opened.append(p)
                ptrs.append(p.value)
            self._bufs.append((C.c_void_p * n_ranks)(*ptrs))
        self.epoch = 0

    def close(self):
        """Unmap the peers' buffers and free this rank's.  Call only after every
        rank has finished its last step (a host barrier), so no peer still
        stores into this buffer."""
        for p in self._opened:
            call("arcllm_cuda_ipc_close_handle", p)
        self._opened = []
        for own in self._own:
            call("arcllm_cuda_free", own)
        self._own = []


class RankGather(_ParityBuffers):
    """Exchange buffers of `n_ranks` ranks for a `rows_total`-row result.

    exchange(handle_bytes) -> list of every rank's handle bytes, in rank order
    (the caller's host all-gather).  After construction, `step()` launches one
    all-gather matvec and `logits_ptr` holds all rows once it completes.

    Two buffers alternate by epoch parity: a peer that is already running the
    next launch stores into the other buffer, and it cannot get two launches
    ahead, because its launch completes only after this rank's next launch --
    stream-ordered after this rank's reads of the current logits -- has
    stored its rows.
    """

    def __init__(self, rows_total, n_ranks, rank, exchange, timeout_us=2000000):
        L = lib()
        self.rows_total, self.timeout_us = rows_total, timeout_us
        n = C.c_uint64(0)
        call("arcllm_cuda_allgather_buffer_bytes", rows_total, C.byref(n))
        self._setup_buffers(n.value, n_ranks, rank, exchange, "RankGather")
        off = C.c_uint64(0)
        call("arcllm_cuda_allgather_logits_offset", rows_total, C.byref(off))
        self._logits_off = off.value
        self.epoch = 0
        self._L = L

    @property
    def logits_ptr(self):
        """Device address of this rank's copy of all rows_total results of the
        last `step()` (after `step_hostio()` with a pinned y_host it holds only
        this rank's own rows: the others went straight to y_host)."""
        return self._own[self.epoch & 1].value + self._logits_off

    def step(self, w, rows, k, x, row0, stream, ggml_type=GGML_Q6_K):
        """One all-gather matvec of this rank's rows [row0, row0 + rows)."""
        self.epoch += 1
        st = self._L.arcllm_cuda_matvec_allgather(ggml_type, w, rows, k, x, row0, self.rows_total,
                                                  self._bufs[self.epoch & 1], self.n_ranks, self.rank, self.epoch,
                                                  self.timeout_us, stream)
        if st:
            from . import check
            check(st, "matvec_allgather")

    def step_hostio(self, w, rows, k, x_host, x_dev, row0, y_host, stream, ggml_type=GGML_Q6_K):
        """One all-gather matvec with host buffers: x_host (k floats) in, all
        rows_total logits in y_host (pinned and device-mapped: stored by the
        kernel itself) when it returns."""
        self.epoch += 1
        st = self._L.arcllm_cuda_matvec_allgather_hostio(ggml_type, w, rows, k, x_host, x_dev, row0, self.rows_total,
                                                         self._bufs[self.epoch & 1], self.n_ranks, self.rank,
                                                         self.epoch, self.timeout_us, y_host, stream)
        if st:
            from . import check
            check(st, "matvec_allgather_hostio")


class GemmGather(_ParityBuffers):
    """Buffers of the output-row-sharded prefill GEMM whose split-K reduce
    kernel all-gathers the result over NVLink (arcllm_cuda_gemm_bf16_allgather):
    after `step()`, `y_ptr` holds the whole m x n_total fp32 result on this
    rank.  Two buffer sets alternate by epoch parity, as in RankGather."""

    def __init__(self, m, n_total, n_ranks, rank, exchange, timeout_us=2000000):
        lib()
        self.m, self.n_total, self.timeout_us = m, n_total, timeout_us
        n = C.c_uint64(0)
        call("arcllm_cuda_gemm_allgather_buffer_bytes", m, n_total, C.byref(n))
        self._setup_buffers(n.value, n_ranks, rank, exchange, "GemmGather")

    @property
    def y_ptr(self):
        """Device address of this rank's copy of the last launch's m x n_total result."""
        return self._own[self.epoch & 1].value

    def step(self, ggml_type, w, n, k, x, c0, stream):
        """One GEMM of this rank's weight rows [c0, c0 + n) (w points at row c0)
        against x (m x k bf16), gathered into every rank's result."""
        self.epoch += 1
        call("arcllm_cuda_gemm_bf16_allgather", ggml_type, w, n, k, x, self.m, c0, self.n_total,
             self._bufs[self.epoch & 1], self.n_ranks, self.rank, self.epoch, self.timeout_us, stream)


class ExchangeBuffers:
    """One exchange buffer per rank for arcllm_cuda_exchange_gather and the
    tensor-parallel model (arcllm_cuda_model_set_tensor_parallel).

    Each rank allocates `arcllm_cuda_exchange_buffer_bytes(max_words)` bytes,
    zero-fills them, shares a CUDA IPC handle through `exchange` (the caller's
    host all-gather of bytes, as for RankGather) and maps the peers' buffers;
    `ptrs` is then the rank-ordered array of device addresses the C ABI takes.
    The sequence numbers and flags of the exchanges live inside the buffers,
    so nothing else needs to be carried between calls.
    """

    def __init__(self, max_words, n_ranks, rank, exchange):
        if not (1 <= n_ranks <= 8 and 0 <= rank < n_ranks):
            raise ValueError("ExchangeBuffers: 1 <= n_ranks <= 8 and 0 <= rank < n_ranks")
        L = lib()
        self.max_words, self.n_ranks, self.rank = max_words, n_ranks, rank
        n = C.c_uint64(0)
        call("arcllm_cuda_exchange_buffer_bytes", max_words, C.byref(n))
        self.nbytes = n.value
        own = C.c_void_p()
        call("arcllm_cuda_malloc", self.nbytes, C.byref(own))
        self._own, self._opened = own, []
        zeros = (C.c_uint8 * self.nbytes)()
        call("arcllm_cuda_memcpy_h2d", own, C.cast(zeros, C.c_void_p), self.nbytes, None)
        call("arcllm_cuda_stream_synchronize", None)
        h = (C.c_uint8 * HANDLE_BYTES)()
        call("arcllm_cuda_ipc_get_handle", own, C.cast(h, C.c_void_p))
        everyone = exchange(bytes(h))
        if len(everyone) != n_ranks:
            raise RuntimeError("ExchangeBuffers: exchange returned %d entries for %d ranks" % (len(everyone), n_ranks))
        ptrs = []
        for r, hb in enumerate(everyone):
            if r == rank:
                ptrs.append(own.value)
                continue
            p = C.c_void_p()
            hbuf = (C.c_uint8 * HANDLE_BYTES).from_buffer_copy(hb[:HANDLE_BYTES])
            call("arcllm_cuda_ipc_open_handle", C.cast(hbuf, C.c_void_p), C.byref(p))
            self._opened.append(p)
            ptrs.append(p.value)
        self.ptrs = (C.c_void_p * n_ranks)(*ptrs)
        self._L = L

    def gather(self, src, n_local, offset, dst, n_total, stream, timeout_us=2000000):
        """dst[0, n_total) = every rank's 32-bit-word slice at its offset."""
        call("arcllm_cuda_exchange_gather", self.ptrs, self.n_ranks, self.rank, self.max_words, src, n_local, offset,
             dst, n_total, timeout_us, stream)

    def close(self):
        """Unmap the peers' buffers and free this rank's.  Call only after
        every rank finished its last exchange (a host barrier)."""
        for p in self._opened:
            call("arcllm_cuda_ipc_close_handle", p)
        self._opened = []
        if self._own is not None:
            call("arcllm_cuda_free", self._own)
            self._own = None
