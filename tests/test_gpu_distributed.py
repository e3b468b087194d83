"""Gaussian-sharded rasterization on two GPUs (NCCL, one process per GPU)
against a single-process render of the gathered scene: every rank renders its
own camera from all Gaussians through the packed all-to-all exchange; images and
the gradients of the rank's own Gaussians must match the single-GPU pipeline
(reference tests/_test_distributed.py runs the same comparison). Skipped with
fewer than two GPUs."""

import os
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu


def _scene(rank, dev, N=20000, C=1):
    g = torch.Generator().manual_seed(50 + rank)
    means = torch.empty(N, 3)
    means[:, 0].uniform_(-3, 3, generator=g)
    means[:, 1].uniform_(-3, 3, generator=g)
    means[:, 2].uniform_(3, 9, generator=g)
    means[:, 0] += 3.0 * (rank - 0.5)  # the two shards overlap in the middle
    quats = torch.randn(N, 4, generator=g)
    quats = quats / quats.norm(dim=-1, keepdim=True)
    scales = torch.exp(torch.randn(N, 3, generator=g) * 0.4 - 3.0)
    opac = torch.sigmoid(torch.randn(N, generator=g))
    sh = torch.randn(N, 16, 3, generator=g) * 0.1
    sh[:, 0] += 0.5
    # the rank's C cameras: small sideways and vertical offsets around its shard
    vm = torch.eye(4)[None].repeat(C, 1, 1)
    for c in range(C):
        vm[c, 0, 3] = -1.5 * (rank - 0.5) + 0.4 * c
        vm[c, 1, 3] = -0.3 * c
    K = torch.tensor([[260.0, 0.0, 160.0], [0.0, 260.0, 120.0], [0.0, 0.0, 1.0]])[None].repeat(C, 1, 1)
    return [t.to(dev) for t in (means, quats, scales, opac, sh, vm, K)]


def _worker(rank, world, store_path, q, C=1):
    import datetime

    import torch.distributed as dist

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        # file rendezvous: no TCP port that another process on the box could hold
        dist.init_process_group("nccl", init_method=f"file://{store_path}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        import gsplat_b200

        W, H = 320, 240
        mine = _scene(rank, dev, C=C)
        params = [t.clone().requires_grad_(True) for t in mine[:5]]
        vm, K = mine[5], mine[6]
        G = torch.randn((C, H, W, 3), generator=torch.Generator().manual_seed(7 + rank)).to(dev)
        # several exchanges (both receive buffers of the peer path), one of them
        # forward-only, must all give the same result
        grads_seen = []
        for it in range(3):
            for p in params:
                p.grad = None
            rc, ra, _ = gsplat_b200.rasterization(*params, vm, K, W, H, sh_degree=3, packed=True,
                                                  distributed=True)
            if it == 1:
                with torch.no_grad():
                    gsplat_b200.rasterization(*params, vm, K, W, H, sh_degree=3, packed=True, distributed=True)
            (rc * G).sum().backward()
            grads_seen.append([p.grad.clone() for p in params])
        for gs in grads_seen[1:]:
            for a, b in zip(gs, grads_seen[0]):
                # the rasterizer's float atomics may add in another order
                torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-5)

        # single-process reference: all Gaussians, every rank's cameras, summed loss
        scenes = [_scene(r, dev, C=C) for r in range(world)]
        full = [torch.cat([s[i] for s in scenes]).requires_grad_(True) for i in range(5)]
        loss = 0.0
        ref_img = None
        for r in range(world):
            Gr = torch.randn((C, H, W, 3), generator=torch.Generator().manual_seed(7 + r)).to(dev)
            img, _, _ = gsplat_b200.rasterization(*full, scenes[r][5], scenes[r][6], W, H, sh_degree=3,
                                                  packed=True)
            loss = loss + (img * Gr).sum()
            if r == rank:
                ref_img = img.detach()
        loss.backward()
        torch.testing.assert_close(rc.detach(), ref_img, rtol=1e-4, atol=1e-5)
        n = mine[0].shape[0]
        for p, f in zip(params, full):
            torch.testing.assert_close(p.grad, f.grad[rank * n:(rank + 1) * n], rtol=2e-3, atol=1e-5)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, None))
    except Exception:  # report to the parent
        q.put((rank, traceback.format_exc()))


@pytest.mark.parametrize("peer", ["1", "0"])
@pytest.mark.parametrize("cams", [1, 3])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_distributed_packed_matches_single_gpu(tmp_path, peer, cams, world, monkeypatch):
    """peer "1": the peer-memory exchange; "0": the NCCL all-to-all path; `cams`
    cameras per rank (config 4 has 4 per rank at 8 GPUs); 1 (a process group of
    one: the distributed path against the plain one), 2, 4 or 8 ranks."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    monkeypatch.setenv("GSB_PEER_EXCHANGE", peer)
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    store = str(tmp_path / "rendezvous")
    procs = [ctx.Process(target=_worker, args=(r, world, store, q, cams)) for r in range(world)]
    for p in procs:
        p.start()
    import queue

    results = []
    for _ in procs:
        try:
            results.append(q.get(timeout=300))
        except queue.Empty:
            break
        if results[-1][1]:
            break  # a failed rank: its peer may now wait in a collective
    for p in procs:
        p.join(timeout=90)
        if p.is_alive():
            p.kill()
    errors = [f"rank {r}: {e}" for r, e in results if e]
    assert not errors, errors[0]
    assert len(results) == len(procs), "a rank neither finished nor reported an error"
