"""Collectives of the Gaussian-sharded multi-GPU mode.

Same functions and semantics as the reference's ``gsplat/distributed.py:25-272``:
integer all-gather / all-to-all and tensor-list all-gather / all-to-all that
concatenate the listed tensors column-wise so each exchange is one collective,
differentiable through ``torch.distributed.nn.functional`` when the data
requires grad. With ``world_size == 1`` every call returns its input unchanged.
The process group is NCCL on GPUs (one process per GPU); the same code runs on
``gloo`` for CPU tests.

The splat exchange of ``rasterization(distributed=True)`` uses either
``exchange_rows`` (one packed ``all_to_all_single`` per direction) or, by default
on one node, ``peer_exchange_rows``: kernels store the rows straight into the
other GPUs' memory (CUDA IPC mappings of per-rank arenas) and hand over with
system-scope flags, so no split size reaches the host.
"""

import math
from typing import Callable, List, Optional, Tuple, Union

import torch
import torch.distributed as dist
import torch.distributed.nn.functional as distF
from torch import Tensor


def all_gather_int32(world_size: int, value: Union[int, Tensor],
                     device: Optional[torch.device] = None) -> List:
    """Gathers one int32 from every rank (reference distributed.py:25-66)."""
    if world_size == 1:
        return [value]
    if isinstance(value, int):
        assert device is not None, "device is required for scalar input"
        value_tensor = torch.tensor(value, dtype=torch.int, device=device)
    else:
        value_tensor = value
    collected = torch.empty(world_size, dtype=value_tensor.dtype, device=value_tensor.device)
    dist.all_gather_into_tensor(collected, value_tensor.reshape(1))
    if isinstance(value, int):
        return collected.tolist()
    return list(collected.unbind())


def all_to_all_int32(world_size: int, values: List[Union[int, Tensor]],
                     device: Optional[torch.device] = None) -> List:
    """Exchanges one int32 with every rank (reference distributed.py:69-113)."""
    if world_size == 1:
        return values
    assert len(values) == world_size, "The length of values should be equal to world_size"
    if any(isinstance(v, int) for v in values):
        assert device is not None, "device is required for scalar input"
    values_tensor = [
        (torch.tensor(v, dtype=torch.int, device=device) if isinstance(v, int) else v).reshape(1)
        for v in values
    ]
    send = torch.cat(values_tensor)
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send)
    out = list(recv.unbind())
    return [o.item() if isinstance(v, int) else o for o, v in zip(out, values)]


def all_gather_tensor_list(world_size: int, tensor_list: List[Tensor]) -> List[Tensor]:
    """Gathers tensors sharing a first dimension from all ranks
    (reference distributed.py:116-179)."""
    if world_size == 1:
        return tensor_list
    N = len(tensor_list[0])
    for t in tensor_list:
        assert len(t) == N, "All tensors should have the same first dimension size"
    data = torch.cat([t.reshape(N, -1) for t in tensor_list], dim=-1)
    sizes = [t.numel() // N for t in tensor_list]
    if data.requires_grad:
        collected = distF.all_gather(data)
    else:
        collected = [torch.empty_like(data) for _ in range(world_size)]
        dist.all_gather(collected, data)
    collected = torch.cat(collected, dim=0)
    out = torch.split(collected, sizes, dim=-1)
    return [o.reshape(-1, *t.shape[1:]) for o, t in zip(out, tensor_list)]


def all_to_all_tensor_list(world_size: int, tensor_list: List[Tensor], splits: List,
                           output_splits: Optional[List] = None) -> List[Tensor]:
    """Splits rows of the listed tensors by ``splits`` and exchanges them with all
    ranks (reference distributed.py:182-272)."""
    if world_size == 1:
        return tensor_list
    N = len(tensor_list[0])
    for t in tensor_list:
        assert len(t) == N, "All tensors should have the same first dimension size"
    assert len(splits) == world_size, "The length of splits should be equal to world_size"
    data = torch.cat([t.reshape(N, -1) for t in tensor_list], dim=-1)
    sizes = [t.numel() // N for t in tensor_list]
    if output_splits is None:
        output_splits = all_to_all_int32(world_size, splits, device=data.device)
    out_splits = [int(s.item()) if isinstance(s, Tensor) else int(s) for s in output_splits]
    in_splits = [int(s.item()) if isinstance(s, Tensor) else int(s) for s in splits]
    # One all_to_all_single on a packed buffer (NCCL grouped send/recv under the
    # hood) instead of a list of per-rank chunks: no torch.cat of the received
    # pieces, and the same call works on gloo for CPU tests.
    collected = torch.empty((sum(out_splits), *data.shape[1:]), dtype=data.dtype, device=data.device)
    if data.requires_grad:
        collected = distF.all_to_all_single(collected, data, out_splits, in_splits)
    else:
        dist.all_to_all_single(collected, data, out_splits, in_splits)
    out = torch.split(collected, sizes, dim=-1)
    return [o.reshape(-1, *t.shape[1:]) for o, t in zip(out, tensor_list)]


def _words(t: Tensor) -> int:
    """4-byte words per row of a [rows, ...] tensor."""
    return math.prod(t.shape[1:]) * t.element_size() // 4


def _pack(tensors: List[Optional[Tensor]], words: List[int], rows: int, device,
          rows_device: Optional[Tensor] = None) -> Tensor:
    """[rows, sum(words)] int32 buffer with the tensors' rows side by side
    (None -> zeros): one gsb_pack_rows launch on CUDA. With ``rows_device`` (a
    device int64 count) only that many leading rows are filled."""
    buf = torch.empty((rows, sum(words)), dtype=torch.int32, device=device)
    if device.type == "cuda":
        import ctypes

        from .cuda._backend import call, stream_of

        srcs = (ctypes.c_void_p * len(words))(*[t.data_ptr() if t is not None else None for t in tensors])
        w = (ctypes.c_int * len(words))(*words)
        call("gsb_pack_rows", rows, rows_device.data_ptr() if rows_device is not None else None, len(words),
             srcs, w, buf.data_ptr(), stream_of(buf))
        return buf
    cols = [t[:rows].reshape(rows, -1).view(torch.int32) if t is not None else
            torch.zeros((rows, wj), dtype=torch.int32, device=device) for t, wj in zip(tensors, words)]
    return torch.cat(cols, dim=1) if cols else buf


def _unpack(buf: Tensor, like: List[Tuple], words: List[int]) -> List[Tensor]:
    """Splits a packed [rows, >= sum(words)] int32 buffer into new contiguous
    tensors of the given (dtype, trailing shape): one gsb_unpack_rows launch."""
    rows = buf.shape[0]
    outs = [torch.empty((rows, *shape), dtype=dtype, device=buf.device) for dtype, shape in like]
    if buf.is_cuda:
        import ctypes

        from .cuda._backend import call, stream_of

        dsts = (ctypes.c_void_p * len(outs))(*[o.data_ptr() for o in outs])
        w = (ctypes.c_int * len(words))(*words)
        call("gsb_unpack_rows", rows, None, buf.shape[1], buf.data_ptr(), len(outs), dsts, w, stream_of(buf))
        return outs
    off = 0
    for o, wj in zip(outs, words):
        o.view(torch.int32).reshape(rows, wj).copy_(buf[:, off:off + wj])
        off += wj
    return outs


class _ExchangeRows(torch.autograd.Function):
    """Row exchange of a list of float32 tensors (differentiable) and int32 /
    int64 tensors (not differentiable) with ONE all_to_all_single of a packed
    buffer each way; the backward sends the float gradients back with the splits
    swapped."""

    @staticmethod
    def forward(ctx, send_splits, recv_splits, n_float, packed, *tensors):
        ctx.set_materialize_grads(False)
        dev = tensors[0].device
        n = sum(send_splits)
        m = sum(recv_splits)
        words = [_words(t) for t in tensors]
        # the all-to-all wants exactly the sent rows (a pre-built buffer may
        # have spare capacity past them)
        buf = packed[:n] if packed is not None else _pack(list(tensors), words, n, dev)
        out = torch.empty((m, buf.shape[1]), dtype=buf.dtype, device=dev)
        dist.all_to_all_single(out, buf, recv_splits, send_splits)
        res = _unpack(out, [(t.dtype, t.shape[1:]) for t in tensors], words)
        ctx.splits = (send_splits, recv_splits)
        ctx.float_meta = [(t.shape, w) for t, w in zip(tensors[:n_float], words[:n_float])]
        ctx.n_inputs = len(tensors)
        ctx.mark_non_differentiable(*res[n_float:])
        return tuple(res)

    @staticmethod
    def backward(ctx, *grads):
        send_splits, recv_splits = ctx.splits
        nf = len(ctx.float_meta)
        words = [w for _, w in ctx.float_meta]
        g = [x.contiguous() if x is not None else None for x in grads[:nf]]
        dev = next((x.device for x in g if x is not None), None)
        if dev is None:
            return (None, None, None, None) + (None,) * ctx.n_inputs
        buf = _pack(g, words, sum(recv_splits), dev)
        n = sum(send_splits)
        back = torch.empty((n, buf.shape[1]), dtype=buf.dtype, device=dev)
        dist.all_to_all_single(back, buf, send_splits, recv_splits)
        # gradients have the inputs' full shapes; rows past the sent ones are
        # left unset (see exchange_rows)
        res = [torch.empty(shape, dtype=torch.float32, device=dev) for shape, _ in ctx.float_meta]
        if dev.type == "cuda":
            import ctypes

            from .cuda._backend import call, stream_of

            dsts = (ctypes.c_void_p * nf)(*[r.data_ptr() for r in res])
            w = (ctypes.c_int * nf)(*words)
            call("gsb_unpack_rows", n, None, back.shape[1], back.data_ptr(), nf, dsts, w, stream_of(back))
        else:
            for r, piece in zip(res, _unpack(back, [(torch.float32, shape[1:]) for shape, _ in ctx.float_meta],
                                             words)):
                r[:n] = piece
        return (None, None, None, None) + tuple(res) + (None,) * (ctx.n_inputs - nf)


def pack_rows(floats: List[Tensor], ints: List[Tensor], rows: int, rows_device: Optional[Tensor] = None) -> Tensor:
    """The send buffer of exchange_rows for these tensors, built ahead of time
    (for instance before the split sizes are read back from the device): the
    first ``rows`` rows, or the first ``*rows_device`` of them."""
    tensors = list(floats) + list(ints)
    return _pack(tensors, [_words(t) for t in tensors], rows, tensors[0].device, rows_device)


def exchange_rows(world_size: int, floats: List[Tensor], ints: List[Tensor], send_splits: List[int],
                  recv_splits: List[int], packed: Optional[Tensor] = None):
    """Sends rows [sum(send_splits[:r]), sum(send_splits[:r+1])) of every listed
    tensor to rank r and receives recv_splits[r] rows from it, with ONE
    all-to-all for all tensors (the float32 tensors keep their autograd graph;
    int32 / int64 tensors travel bit-cast inside the same buffer). The counts are
    host lists, so no collective or host read happens here besides the data
    exchange itself. Tensors may hold more rows than sum(send_splits) (buffers
    with spare capacity): only the leading rows are sent, and the gradient rows
    past them are left unset, for producers that never read those rows back.
    ``packed`` is a buffer from pack_rows for the same tensors, if already
    built. Returns (received floats, received ints)."""
    for t in floats:
        assert t.dtype == torch.float32
    for t in ints:
        assert t.dtype in (torch.int32, torch.int64)
    tensors = [t.contiguous() for t in floats] + [t.contiguous() for t in ints]
    out = _ExchangeRows.apply(list(send_splits), list(recv_splits), len(floats), packed, *tensors)
    return list(out[:len(floats)]), list(out[len(floats):])


def cli(fn: Callable, args, verbose: bool = False, backend: str = "nccl") -> bool:
    """Runs ``fn(local_rank, world_rank, world_size, args)`` in one process per GPU
    (reference distributed.py:287-375). Under torchrun / MPI launchers the ranks
    come from the environment; otherwise one process is spawned per visible GPU."""
    import os

    if "OMPI_COMM_WORLD_SIZE" in os.environ:
        local_rank = int(os.environ["OMPI_COMM_WORLD_LOCAL_RANK"])
        world_rank = int(os.environ["OMPI_COMM_WORLD_RANK"])
        world_size = int(os.environ["OMPI_COMM_WORLD_SIZE"])
        return _worker(local_rank, world_rank, world_size, fn, args, backend)
    if "WORLD_SIZE" in os.environ and "RANK" in os.environ:
        return _worker(int(os.environ.get("LOCAL_RANK", 0)), int(os.environ["RANK"]),
                       int(os.environ["WORLD_SIZE"]), fn, args, backend)
    world_size = torch.cuda.device_count() if backend == "nccl" else 1
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    if "MASTER_PORT" not in os.environ:
        import socket

        s = socket.socket()
        s.bind(("127.0.0.1", 0))
        os.environ["MASTER_PORT"] = str(s.getsockname()[1])
        s.close()
    torch.multiprocessing.spawn(_spawned, args=(world_size, fn, args, backend), nprocs=world_size,
                                join=True)
    return True


def _spawned(rank, world_size, fn, args, backend):
    _worker(rank, rank, world_size, fn, args, backend)


def _worker(local_rank, world_rank, world_size, fn, args, backend):
    import datetime

    if backend == "nccl":
        torch.cuda.set_device(local_rank)
    dist.init_process_group(backend=backend, rank=world_rank, world_size=world_size,
                            timeout=datetime.timedelta(seconds=120))
    try:
        fn(local_rank, world_rank, world_size, args)
    finally:
        dist.destroy_process_group()
    return True


# ---------------------------------------------------------------------------
# Peer-memory exchange (one node): the row exchange above without NCCL, host
# split sizes or a second copy of the rows. See gsb_peer_* in
# include/gsplat_b200.h for the device protocol.
# ---------------------------------------------------------------------------
def _align256(x: int) -> int:
    return (x + 255) // 256 * 256


def arena_bytes_needed(mailbox_bytes: int, recv_rows: int, grad_rows: int, row_words: int,
                       grad_words: int) -> int:
    """Bytes of a peer arena holding the mailbox, two receive buffers of
    recv_rows rows of row_words 4-byte words, and a gradient buffer of
    grad_rows rows of grad_words words, each region 256-byte aligned."""
    return (mailbox_bytes + 2 * _align256(max(1, recv_rows) * row_words * 4) +
            _align256(max(1, grad_rows) * grad_words * 4))


def arena_layout(arena_bytes: int, mailbox_bytes: int, grad_rows: int, row_words: int, grad_words: int):
    """Offsets inside an arena of arena_bytes (the same on every rank): the
    mailbox at 0, receive buffers 0 and 1 after it, the gradient buffer (room
    for grad_rows rows) at the end; the receive buffers take the rest. Returns
    recv_offset, recv_stride, grad_offset and the row capacities cap_recv,
    cap_grad."""
    grad_bytes = _align256(max(1, grad_rows) * grad_words * 4)
    recv_stride = (arena_bytes - mailbox_bytes - grad_bytes) // 2 // 256 * 256
    grad_offset = mailbox_bytes + 2 * recv_stride
    return {"recv_offset": mailbox_bytes, "recv_stride": recv_stride, "grad_offset": grad_offset,
            "cap_recv": recv_stride // (row_words * 4),
            "cap_grad": (arena_bytes - grad_offset) // (grad_words * 4)}


class PeerExchange:
    """The exchange arenas of this process group: one CUDA allocation per rank
    (mailbox, two receive buffers, gradient buffer), mapped by every rank
    through CUDA IPC. Created on first use and reallocated (collectively: every
    rank makes the same decision from the same gathered sizes) when a step
    needs more room.

    The gradient buffer has one slot per rank and no handshake of its own: a
    destination may write the gradients of exchange e into it once it holds
    the rows of e, because the source sent those rows after it had read the
    previous gradients. That holds when each backward runs after the forward
    of its exchange was issued following the previous backward
    (``claim_backward``); other orders take the collective path."""

    _instances = {}

    def __init__(self, device: torch.device):
        import ctypes

        from .cuda import _backend as B

        self.B = B
        self.ctypes = ctypes
        self.device = device
        self.rank = dist.get_rank()
        self.world = dist.get_world_size()
        assert self.world <= 8, "peer exchange: at most 8 GPUs (one node)"
        self.epoch = 0
        self.generation = 0  # arenas allocated so far (epochs restart with each)
        self.bwd_horizon = 0  # self.epoch when the last peer-path backward was issued
        self.arena_bytes = 0
        self.ptrs = None
        self.own = None
        self.err_host = ctypes.POINTER(ctypes.c_int)()
        self.err_dev = ctypes.c_void_p()
        with torch.cuda.device(device):
            B.call("gsb_peer_error_alloc", ctypes.byref(self.err_host), ctypes.byref(self.err_dev))
        self.group = B.GsbPeerGroup()
        self.layout = None
        self.disabled = False  # peer memory could not be set up on every rank: use the all-to-all

    @classmethod
    def get(cls, device: torch.device) -> "PeerExchange":
        key = (id(dist.group.WORLD), device.index)
        inst = cls._instances.get(key)
        if inst is None:
            inst = cls._instances[key] = cls(device)
        return inst

    def claim_backward(self, epoch: int, generation: int) -> bool:
        """Whether the gradients of exchange ``epoch`` (made in arena
        ``generation``) may go through the peer gradient buffer: only if that
        arena is still the current one and the exchange's forward was issued
        after the last peer-path backward. Backward passes in reverse or
        interleaved order (several distributed renders in one loss), a second
        backward through the same graph, or an arena reallocated since the
        forward return False: those gradients take the collective path
        (``_peer_grads_collective``). Every rank runs the same sequence of
        forwards and backwards, so every rank decides alike."""
        if generation != self.generation or epoch <= self.bwd_horizon:
            return False
        self.bwd_horizon = self.epoch
        return True

    def check(self):
        """Raises if a bounded wait of an exchange ran out (the error word is
        host-mapped: read without a device sync)."""
        code = self.err_host[0]
        if code:
            what = {1: "a destination did not consume the previous exchange",
                    2: "a source's rows did not arrive", 3: "gradients did not arrive"}.get(code, str(code))
            raise RuntimeError(f"peer exchange failed on rank {self.rank}: {what} (bounded wait ran out)")

    def _release(self):
        if self.ptrs is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier()
        with torch.cuda.device(self.device):
            for r, p in enumerate(self.ptrs):
                if r != self.rank:
                    self.B.call("gsb_peer_close", p)
            self.B.call("gsb_peer_free", self.own)
        self.ptrs = None

    def ensure(self, recv_rows: int, grad_rows: int, row_words: int, grad_words: int):
        """Arena layout for these capacities (the same numbers on every rank:
        receive rows and the largest rank's gradient rows, from gathered
        sizes), reallocated on every rank at once when the arena is too small."""
        mb = self.B.lib().gsb_peer_mailbox_bytes()
        need = arena_bytes_needed(mb, recv_rows, grad_rows, row_words, grad_words)
        if self.ptrs is None or need > self.arena_bytes or self.layout != (row_words, grad_words):
            self._release()
            size = int(need * 1.25)
            ctypes = self.ctypes
            handle = (ctypes.c_char * 64)()
            own = ctypes.c_void_p()
            ok = True
            try:
                with torch.cuda.device(self.device):
                    self.B.call("gsb_peer_alloc", size, ctypes.byref(own), handle)
            except RuntimeError:
                ok = False
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle) if ok else None)
            ptrs = []
            if all(h is not None for h in handles):
                with torch.cuda.device(self.device):
                    for r, h in enumerate(handles):
                        if r == self.rank:
                            ptrs.append(own.value)
                            continue
                        p = ctypes.c_void_p()
                        try:
                            self.B.call("gsb_peer_open", (ctypes.c_char * 64).from_buffer_copy(h),
                                        ctypes.byref(p))
                        except RuntimeError:
                            ok = False
                            break
                        ptrs.append(p.value)
            else:
                ok = False
            # every rank learns whether every rank could map every arena
            flags = [None] * self.world
            dist.all_gather_object(flags, ok)
            if not all(flags):
                with torch.cuda.device(self.device):
                    for r, p in enumerate(ptrs):
                        if r != self.rank:
                            self.B.call("gsb_peer_close", p)
                    if own.value:
                        self.B.call("gsb_peer_free", own.value)
                self.disabled = True
                return None
            self.own, self.ptrs, self.arena_bytes = own.value, ptrs, size
            self.layout = (row_words, grad_words)
            self.epoch = 0
            self.generation += 1
            self.bwd_horizon = 0
            dist.barrier()
        lay = arena_layout(self.arena_bytes, mb, grad_rows, row_words, grad_words)
        g = self.group
        for r in range(8):
            g.arena[r] = self.ptrs[r] if r < self.world else None
        g.recv_offset = lay["recv_offset"]
        g.recv_stride = lay["recv_stride"]
        g.grad_offset = lay["grad_offset"]
        g.rank = self.rank
        g.world = self.world
        g.error = self.err_dev.value
        self.cap_recv = lay["cap_recv"]
        self.cap_grad = lay["cap_grad"]
        return g


def _ptr_array(ctypes, tensors):
    return (ctypes.c_void_p * len(tensors))(*[t.data_ptr() if t is not None else None for t in tensors])


def _peer_grads_collective(route: Tensor, bounds: Tensor, world: int, float_meta: List[Tuple],
                           grads: List[Optional[Tensor]]) -> List[Tensor]:
    """The gradient leg of a peer exchange through one all_to_all_single, for
    the backward orders the peer gradient buffer cannot serve. ``route``
    (int64 [2 * world + 1]: prefix of the received counts by source, ...) and
    ``bounds`` (int64 [world + 1]: local rows [bounds[d], bounds[d + 1]) went to
    rank d) are the forward exchange's; ``grads`` are the gradients of the
    received float tensors (rows in source order, None -> zeros). Returns the
    gradients of the local float tensors (``float_meta``: full shape, words per
    row), rows past the sent ones left unset, like the peer path."""
    sizes = torch.cat([route[:world + 1].to(torch.int64), bounds.to(torch.int64)]).tolist()
    prefix, local = sizes[:world + 1], sizes[world + 1:]
    send = [prefix[s + 1] - prefix[s] for s in range(world)]  # rows received from s go back to s
    recv = [local[d + 1] - local[d] for d in range(world)]  # rows sent to d come back from d
    words = [wj for _, wj in float_meta]
    dev = route.device
    buf = _pack(list(grads), words, prefix[world], dev)
    back = torch.empty((sum(recv), buf.shape[1]), dtype=buf.dtype, device=dev)
    dist.all_to_all_single(back, buf, recv, send)
    # rows come back in destination order, which is the local row order
    pieces = _unpack(back, [(torch.float32, shape[1:]) for shape, _ in float_meta], words)
    res = []
    for (shape, _), piece in zip(float_meta, pieces):
        r = torch.empty(shape, dtype=torch.float32, device=dev)
        r[local[0]:local[0] + piece.shape[0]] = piece
        res.append(r)
    return res


class _PeerExchangeRows(torch.autograd.Function):
    """exchange_rows through peer memory: rows [bounds[d], bounds[d+1]) of the
    local packed tensors go to rank d; the received rows come back in source
    order, in tensors of ``cap_out`` rows of which the first ``*nnz_recv`` are
    set. Float tensors are differentiable; the backward returns the gradients of
    the local rows (rows past ``*nnz`` left unset, as exchange_rows does)."""

    @staticmethod
    def forward(ctx, px, cap_out, grad_rows, n_float, nnz, bounds, n_world, cams_per_rank, *tensors):
        ctx.set_materialize_grads(False)
        B, ctypes = px.B, px.ctypes
        words = [_words(t) for t in tensors]
        assert tensors[0].shape[0] <= grad_rows
        g = px.group  # laid out by px.ensure() for these sizes (peer_exchange_rows)
        px.epoch += 1
        epoch = px.epoch
        dev = tensors[0].device
        cap_in = tensors[0].shape[0]
        outs = [torch.empty((cap_out, *t.shape[1:]), dtype=t.dtype, device=dev) for t in tensors]
        route = torch.empty(2 * px.world + 1, dtype=torch.int64, device=dev)
        nnz_recv = torch.empty(1, dtype=torch.int64, device=dev)
        w = (ctypes.c_int * len(words))(*words)
        stream = B.stream_of(tensors[0])
        B.call("gsb_peer_send_rows", ctypes.byref(g), epoch, cap_in, nnz.data_ptr(), bounds.data_ptr(),
               n_world.data_ptr(), cams_per_rank, px.cap_recv, len(tensors), _ptr_array(ctypes, tensors), w,
               stream)
        B.call("gsb_peer_recv_rows", ctypes.byref(g), epoch, cap_out, route.data_ptr(), nnz_recv.data_ptr(),
               n_world.data_ptr(), cams_per_rank, px.cap_recv, len(outs), _ptr_array(ctypes, outs), w, stream)
        ctx.px, ctx.epoch, ctx.route, ctx.nnz, ctx.nnz_recv = px, epoch, route, nnz, nnz_recv
        ctx.generation, ctx.bounds = px.generation, bounds
        ctx.float_meta = [(t.shape, wj) for t, wj in zip(tensors[:n_float], words[:n_float])]
        ctx.n_inputs = len(tensors)
        ctx.cap_out = cap_out
        ctx.mark_non_differentiable(*outs[n_float:], nnz_recv)
        return tuple(outs) + (nnz_recv,)

    @staticmethod
    def backward(ctx, *grads):
        px = ctx.px
        B, ctypes = px.B, px.ctypes
        nf = len(ctx.float_meta)
        words = [wj for _, wj in ctx.float_meta]
        g_in = [x.contiguous() if x is not None else None for x in grads[:nf]]
        if not px.claim_backward(ctx.epoch, ctx.generation):
            res = _peer_grads_collective(ctx.route, ctx.bounds, px.world, ctx.float_meta, g_in)
            return (None,) * 8 + tuple(res) + (None,) * (ctx.n_inputs - nf)
        dev = ctx.route.device
        g = px.group
        w = (ctypes.c_int * nf)(*words)
        stream = B.stream_of(ctx.route)
        # every rank sends (zeros where a gradient is missing), so the sources'
        # waits always end
        B.call("gsb_peer_send_grads", ctypes.byref(g), ctx.epoch, ctx.cap_out, ctx.nnz_recv.data_ptr(),
               ctx.route.data_ptr(), px.cap_grad, nf, _ptr_array(ctypes, g_in), w, stream)
        res = [torch.empty(shape, dtype=torch.float32, device=dev) for shape, _ in ctx.float_meta]
        B.call("gsb_peer_recv_grads", ctypes.byref(g), ctx.epoch, res[0].shape[0], ctx.nnz.data_ptr(), nf,
               _ptr_array(ctypes, res), w, stream)
        return (None,) * 8 + tuple(res) + (None,) * (ctx.n_inputs - nf)


def peer_exchange_rows(floats: List[Tensor], ints: List[Tensor], nnz: Tensor, bounds: Tensor, n_world: Tensor,
                       n_world_host: List[int], cams_per_rank: int):
    """Sends local packed rows [bounds[d], bounds[d+1]) of every listed tensor
    to rank d (bounds, nnz, n_world: device int64) through peer memory. Returns
    (received floats, received ints, nnz_recv device int64 [1]); the received
    tensors have cams_per_rank * sum(n_world_host) rows, the first nnz_recv set,
    in source-rank order. Float tensors keep their autograd graph. Returns None
    (on every rank) when the peer arenas could not be set up everywhere; the
    caller then uses exchange_rows."""
    for t in floats:
        assert t.dtype == torch.float32
    for t in ints:
        assert t.dtype in (torch.int32, torch.int64)
    dev = floats[0].device
    px = PeerExchange.get(dev)
    px.check()
    world = len(n_world_host)
    cap_out = cams_per_rank * sum(n_world_host)
    # the packed rows of a rank: at most (all cameras) x (its Gaussians)
    grad_rows = world * cams_per_rank * max(n_world_host)
    tensors = [t.contiguous() for t in floats] + [t.contiguous() for t in ints]
    words = [_words(t) for t in tensors]
    if px.disabled or px.ensure(cap_out, grad_rows, sum(words), sum(words[:len(floats)])) is None:
        return None  # peer memory not available on every rank (decided together)
    out = _PeerExchangeRows.apply(px, cap_out, grad_rows, len(floats), nnz, bounds, n_world, cams_per_rank,
                                  *tensors)
    return list(out[:len(floats)]), list(out[len(floats):-1]), out[-1]


def peer_exchange_available(device: torch.device) -> bool:
    """Peer-memory exchange: every rank on this node with peer access to every
    other (one process per GPU, NCCL process group); GSB_PEER_EXCHANGE=0 turns it off."""
    import os

    if os.environ.get("GSB_PEER_EXCHANGE", "1") == "0":
        return False
    inst = PeerExchange._instances.get((id(dist.group.WORLD), device.index)) if dist.is_initialized() else None
    if inst is not None and inst.disabled:
        return False
    if device.type != "cuda" or not dist.is_initialized() or dist.get_world_size() > 8:
        return False
    return dist.get_backend() == "nccl"
