"""Collectives of the Gaussian-sharded multi-GPU mode.

Same functions and semantics as the reference's ``gsplat/distributed.py:25-272``:
integer all-gather / all-to-all and tensor-list all-gather / all-to-all that
concatenate the listed tensors column-wise so each exchange is one collective,
differentiable through ``torch.distributed.nn.functional`` when the data
requires grad. With ``world_size == 1`` every call returns its input unchanged.
The process group is NCCL on GPUs (one process per GPU); the same code runs on
``gloo`` for CPU tests.
"""

import math
from typing import Callable, List, Optional, Tuple, Union

import torch
import torch.distributed as dist
import torch.distributed.nn.functional as distF
from torch import Tensor


def _comm_device(t_device: torch.device) -> torch.device:
    return t_device


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
        call("gsb_unpack_rows", rows, buf.shape[1], buf.data_ptr(), len(outs), dsts, w, stream_of(buf))
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
            call("gsb_unpack_rows", n, back.shape[1], back.data_ptr(), nf, dsts, w, stream_of(back))
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
