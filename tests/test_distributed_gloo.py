"""Host logic of the Gaussian-sharded multi-GPU mode on CPU: the collectives of
gsplat_b200.distributed run on gloo with world size 2 (the reference's own test,
tests/_test_distributed.py, needs GPUs). Values and gradients are checked
against what each rank must receive.
"""

import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, fn, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        fn(rank, world)
        q.put((rank, None))
    except Exception:  # report to the parent
        q.put((rank, traceback.format_exc()))
    finally:
        dist.destroy_process_group()


def run(fn, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fn, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    errors = [e for _, e in results if e]
    assert not errors, errors[0]


def _collectives(rank, world):
    from gsplat_b200.distributed import (all_gather_int32, all_gather_tensor_list, all_to_all_int32,
                                         all_to_all_tensor_list)

    dev = torch.device("cpu")
    assert all_gather_int32(world, 10 + rank, device=dev) == [10, 11]
    assert all_to_all_int32(world, [rank * 10 + 1, rank * 10 + 2], device=dev) == [1 + rank, 11 + rank]
    a = torch.full((2, 3), float(rank))
    b = torch.full((2,), float(rank + 5))
    ga, gb = all_gather_tensor_list(world, [a, b])
    assert ga.shape == (4, 3) and gb.shape == (4,)
    assert ga[:2].eq(0).all() and ga[2:].eq(1).all() and gb[:2].eq(5).all() and gb[2:].eq(6).all()
    # uneven all-to-all with autograd: rank 0 sends 1 row to itself and 2 to rank 1,
    # rank 1 sends 3 rows to rank 0 and 1 to itself
    splits = [1, 2] if rank == 0 else [3, 1]
    n = sum(splits)
    x = (torch.arange(n, dtype=torch.float32) + 100 * rank).reshape(n, 1).repeat(1, 2)
    x.requires_grad_(True)
    y = torch.arange(n, dtype=torch.int64) + 1000 * rank
    out_x, out_y = all_to_all_tensor_list(world, [x, y], splits)
    if rank == 0:
        assert out_x[:, 0].tolist() == [0.0, 100.0, 101.0, 102.0]
        assert out_y.tolist() == [0, 1000, 1001, 1002]
    else:
        assert out_x[:, 0].tolist() == [1.0, 2.0, 103.0]
        assert out_y.tolist() == [1, 2, 1003]
    w = torch.arange(out_x.shape[0], dtype=torch.float32)[:, None] + 1.0
    (out_x * w).sum().backward()
    # each row's gradient is the weight of the position it landed at on its destination
    if rank == 0:
        assert x.grad[:, 0].tolist() == [1.0, 1.0, 2.0]
    else:
        assert x.grad[:, 0].tolist() == [2.0, 3.0, 4.0, 3.0]


def test_collectives_world2_gloo():
    run(_collectives)


def _single_rank_shortcuts(rank, world):
    from gsplat_b200.distributed import all_gather_tensor_list, all_to_all_tensor_list

    t = torch.ones(3, 2)
    assert all_gather_tensor_list(1, [t])[0] is t
    assert all_to_all_tensor_list(1, [t], [3])[0] is t


def test_world1_is_identity():
    run(_single_rank_shortcuts, world=1)


def _raising_rank(rank, world):
    """A rank that fails between steps: the other one sees its collective fail
    within the process-group timeout instead of hanging."""
    import datetime

    from gsplat_b200.distributed import all_gather_int32

    if rank == 1:
        raise RuntimeError("rank 1 leaves")
    try:
        dist.monitored_barrier(timeout=datetime.timedelta(seconds=5))
    except RuntimeError as e:
        assert "1" in str(e)
        return
    raise AssertionError("the surviving rank did not notice")


def test_failed_rank_is_detected_on_host():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, _raising_rank, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results[1] is not None and "rank 1 leaves" in results[1]
    assert results[0] is None, results[0]


def _exchange_rows(rank, world):
    from gsplat_b200.distributed import exchange_rows

    # rank 0 has 3 rows (1 to itself, 2 to rank 1); rank 1 has 2 rows (2 to rank 0)
    send = [1, 2] if rank == 0 else [2, 0]
    recv = [1, 2] if rank == 0 else [2, 0]
    n = sum(send)
    a = (torch.arange(n * 2, dtype=torch.float32).reshape(n, 2) + 100 * rank).requires_grad_(True)
    b = (torch.arange(n, dtype=torch.float32) + 0.5 + 100 * rank).requires_grad_(True)
    ids32 = torch.arange(n, dtype=torch.int32).reshape(n, 1).repeat(1, 2) + 1000 * rank
    ids64 = torch.arange(n, dtype=torch.int64) + (1 << 40) + rank
    (fa, fb), (i32, i64) = exchange_rows(world, [a, b], [ids32, ids64], send, recv)
    if rank == 0:
        assert fa[:, 0].tolist() == [0.0, 100.0, 102.0] and fb.tolist() == [0.5, 100.5, 101.5]
        assert i32[:, 0].tolist() == [0, 1000, 1001] and i64.tolist() == [1 << 40, (1 << 40) + 1, (1 << 40) + 2]
    else:
        assert fa[:, 0].tolist() == [2.0, 4.0] and fb.tolist() == [1.5, 2.5]
        assert i32[:, 1].tolist() == [1, 2] and i64.tolist() == [(1 << 40) + 1, (1 << 40) + 2]
    assert i32.dtype == torch.int32 and i64.dtype == torch.int64
    # gradients travel back: d(sum(w * fa) + sum(fb)) with w = row position + 1
    w = torch.arange(fa.shape[0], dtype=torch.float32)[:, None] + 1.0
    ((fa * w).sum() + (3 * fb).sum()).backward()
    if rank == 0:
        assert a.grad[:, 0].tolist() == [1.0, 1.0, 2.0] and b.grad.tolist() == [3.0, 3.0, 3.0]
    else:
        assert a.grad[:, 1].tolist() == [2.0, 3.0] and b.grad.tolist() == [3.0, 3.0]


def test_exchange_rows_world2_gloo():
    run(_exchange_rows)


def test_peer_arena_layout():
    """Arena layout of the peer-memory exchange (host arithmetic): every region
    fits, none overlaps, the capacities cover the requested rows, offsets are
    256-byte aligned, for arenas allocated with the 25% headroom and exactly."""
    from gsplat_b200.distributed import arena_bytes_needed, arena_layout

    mb = 4096
    for recv_rows, grad_rows, rw, gw in [(1, 1, 1, 1), (2_000_000, 2_000_000, 16, 10), (8_000_000, 8_000_000, 16, 10),
                                         (12345, 777, 13, 7), (0, 0, 3, 2)]:
        need = arena_bytes_needed(mb, recv_rows, grad_rows, rw, gw)
        for size in (need, int(need * 1.25)):
            lay = arena_layout(size, mb, grad_rows, rw, gw)
            assert lay["recv_offset"] == mb
            assert lay["recv_stride"] % 256 == 0 and lay["grad_offset"] % 256 == 0
            assert lay["cap_recv"] >= recv_rows and lay["cap_grad"] >= grad_rows
            # buffer 1 ends before the gradient buffer, which ends inside the arena
            assert mb + lay["recv_stride"] + lay["cap_recv"] * rw * 4 <= lay["grad_offset"]
            assert lay["grad_offset"] + lay["cap_grad"] * gw * 4 <= size


def test_peer_backward_order_decisions():
    """Which backward passes of the peer-memory exchange may use the peer
    gradient buffer (PeerExchange.claim_backward, host logic): in-order
    forward/backward pairs always; of reversed or interleaved backward passes
    (several distributed renders in one loss) only the first; a second backward
    through the same graph never; exchanges made in an arena reallocated since
    never. The others go through the collective path."""
    from gsplat_b200.distributed import PeerExchange

    px = PeerExchange.__new__(PeerExchange)  # host state only, no arena
    px.epoch, px.generation, px.bwd_horizon = 0, 1, 0

    def fwd():
        px.epoch += 1
        return px.epoch, px.generation

    def bwd(ex):
        return px.claim_backward(*ex)

    for _ in range(3):  # training steps in order
        assert bwd(fwd())
    e1, e2 = fwd(), fwd()  # two renders, one loss: autograd runs the later one first
    assert bwd(e2) and not bwd(e1)
    e1, e2 = fwd(), fwd()  # interleaved: the second backward may not reuse the buffer
    assert bwd(e1) and not bwd(e2)
    e1 = fwd()
    assert bwd(e1) and not bwd(e1)  # retain_graph=True and a second backward
    e1 = fwd()
    fwd()  # a forward-only exchange in between changes nothing
    assert bwd(e1)
    e1 = fwd()
    px.epoch, px.generation, px.bwd_horizon = 0, px.generation + 1, 0  # arena reallocated (ensure)
    e2 = fwd()
    assert not bwd(e1) and bwd(e2)
    assert bwd(fwd())


def _peer_grads_collective(rank, world):
    """The collective gradient leg of the peer exchange returns, for every local
    row, the gradient its destination computed: the same as the backward of
    exchange_rows over the same rows. Receive tensors carry spare capacity rows
    (as the peer path's do) and one gradient is missing (zeros)."""
    from gsplat_b200.distributed import _peer_grads_collective, _words, exchange_rows

    torch.manual_seed(3 + rank)
    send = [2, 3] if rank == 0 else [4, 0]  # local rows to rank 0, rank 1
    n = sum(send)
    cap_in = n + 2  # spare rows past the sent ones, never read back
    a = torch.randn(cap_in, 3, requires_grad=True)
    b = torch.randn(cap_in, requires_grad=True)
    c = torch.randn(cap_in, 2, requires_grad=True)
    recv_t = torch.empty(world, dtype=torch.int64)
    dist.all_to_all_single(recv_t, torch.tensor(send, dtype=torch.int64))
    recv = recv_t.tolist()
    (fa, fb, fc), _ = exchange_rows(world, [a, b, c], [], send, recv)
    m = sum(recv)
    ga, gb = torch.randn(m, 3), torch.randn(m)
    ((fa * ga).sum() + (fb * gb).sum() + 0 * fc.sum()).backward()
    # the peer path's view of the same exchange
    prefix = [0]
    for r in recv:
        prefix.append(prefix[-1] + r)
    route = torch.tensor(prefix + [0] * world, dtype=torch.int64)
    bounds = torch.tensor([0, send[0], n], dtype=torch.int64)
    cap_out = m + 5
    pad = lambda g: torch.cat([g, torch.full((cap_out - m, *g.shape[1:]), float("nan"))])
    meta = [(t.shape, _words(t)) for t in (a, b, c)]
    res = _peer_grads_collective(route, bounds, world, meta, [pad(ga), pad(gb), None])
    assert [r.shape for r in res] == [a.shape, b.shape, c.shape]
    assert torch.equal(res[0][:n], a.grad[:n]) and torch.equal(res[1][:n], b.grad[:n])
    assert torch.equal(res[2][:n], torch.zeros(n, 2))


def test_peer_grads_collective_world2_gloo():
    run(_peer_grads_collective)


def test_trim_local_meta_exact_rows_and_means2d_grad():
    """Distributed packed mode keeps the projection's capacity rows on the
    device until the sizes are read; rasterization() then trims the local
    entries of meta to the splat count (rendering._trim_local_meta). meta's
    means2d is exact-size and its .grad, after retain_grad() and backward(), is
    the gradient of those rows, accumulated over repeated backward passes,
    like the reference's exact-size means2d."""
    from gsplat_b200.rendering import _trim_local_meta

    cap, n = 10, 6
    x = torch.randn(cap, 2, requires_grad=True)
    means2d = x * 3.0  # the projection output (capacity rows, non-leaf)
    meta = {"batch_ids": torch.zeros(cap, dtype=torch.int64), "camera_ids": torch.zeros(cap, dtype=torch.int64),
            "gaussian_ids": torch.arange(cap), "radii": torch.ones(cap, 2, dtype=torch.int32),
            "means2d": means2d, "depths": torch.rand(cap), "conics": torch.rand(cap, 3),
            "opacities": torch.rand(cap)}
    _trim_local_meta(meta, n)
    for k, t in meta.items():
        assert t.shape[0] == n, k
    m = meta["means2d"]
    m.retain_grad()  # what a strategy does before backward
    assert torch.equal(m, means2d[:n].detach())
    w = torch.arange(cap * 2, dtype=torch.float32).reshape(cap, 2)
    loss = (means2d[:n] * w[:n]).sum()  # the exchange reads only the set rows
    loss.backward(retain_graph=True)
    assert torch.equal(m.grad, w[:n])
    loss.backward()
    assert torch.equal(m.grad, 2 * w[:n])
    # without autograd (a forward under no_grad) there is nothing to fill
    meta = {"means2d": torch.randn(cap, 2)}
    _trim_local_meta(meta, n)
    assert meta["means2d"].shape == (n, 2) and not meta["means2d"].requires_grad


def _peer_availability(rank, world):
    from gsplat_b200.distributed import peer_exchange_available

    # peer memory needs CUDA devices and an NCCL group: a gloo group or a CPU
    # device answers no, and the library then takes the all-to-all path
    assert not peer_exchange_available(torch.device("cpu"))
    assert not peer_exchange_available(torch.device("cuda", rank))
    os.environ["GSB_PEER_EXCHANGE"] = "0"
    assert not peer_exchange_available(torch.device("cuda", rank))


def test_peer_exchange_not_offered_without_nccl_world2_gloo():
    run(_peer_availability)


def test_peer_exchange_error_codes_are_reported():
    """A bounded wait that ran out leaves a code in the host-mapped error word;
    PeerExchange.check() raises with the rank and what did not arrive."""
    import ctypes

    from gsplat_b200.distributed import PeerExchange

    px = PeerExchange.__new__(PeerExchange)
    px.rank = 1
    word = ctypes.c_int(0)
    px.err_host = ctypes.pointer(word)
    px.check()  # no error recorded
    for code, text in ((1, "did not consume"), (2, "rows did not arrive"), (3, "gradients did not arrive")):
        word.value = code
        with pytest.raises(RuntimeError, match=f"rank 1: .*{text}"):
            px.check()


def _cli_fn(local_rank, world_rank, world_size, path):
    import torch.distributed as d

    t = torch.tensor([world_rank + 1])
    d.all_reduce(t)
    with open(f"{path}.{world_rank}", "w") as f:
        f.write(f"{local_rank} {world_rank} {world_size} {int(t)}")


def test_cli_launcher_gloo(tmp_path):
    """distributed.cli (reference distributed.py:287-375): spawned ranks when no
    launcher environment is set, and the ranks a torchrun-style environment names."""
    import subprocess
    import sys

    from gsplat_b200.distributed import cli

    path = str(tmp_path / "spawned")
    assert cli(_cli_fn, path, backend="gloo") is True
    assert open(path + ".0").read() == "0 0 1 1"

    path = str(tmp_path / "env")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = ("import sys; sys.path.insert(0, %r); from gsplat_b200.distributed import cli; "
            "from tests.test_distributed_gloo import _cli_fn; cli(_cli_fn, %r, backend='gloo')") % (root, path)
    port = str(_free_port())
    procs = [subprocess.Popen([sys.executable, "-c", code], cwd=root,
                              env=dict(os.environ, RANK=str(r), LOCAL_RANK=str(r), WORLD_SIZE="2",
                                       MASTER_ADDR="127.0.0.1", MASTER_PORT=port))
             for r in range(2)]
    assert [p.wait(timeout=120) for p in procs] == [0, 0]
    assert open(path + ".0").read() == "0 0 2 3" and open(path + ".1").read() == "1 1 2 3"
