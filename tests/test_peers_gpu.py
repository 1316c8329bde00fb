"""GPU tests of b2g_gemm_peers (a GEMM whose epilogue also writes D into peer copies) and of
the CUDA IPC helpers that give one-process-per-GPU callers those copies.

The cross-process test runs two processes on device 0: each computes its M-row panel and
pushes it into the other's full D through an IPC mapping. The two kernels never wait for each
other, so they may share one GPU."""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

import b2g
from helpers import inputs, to_dev, to_host

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


@pytest.mark.parametrize("npeer", [0, 1, 3, 7])
@pytest.mark.parametrize("M,N,K", [(512, 512, 256), (300, 136, 1000), (2048, 1024, 64)])
def test_gemm_peers_writes_every_copy(npeer, M, N, K):
    A, B, bias = inputs(M, N, K, seed=npeer + M)
    dA, dB = to_dev(torch, A), to_dev(torch, B)
    D = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    # copies with a wider pitch than N would need the same ldd as D: keep them contiguous too
    copies = [torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
              for _ in range(npeer)]
    b2g.gemm_peers(dA, dB, D, [c.data_ptr() for c in copies])
    b2g.sync_status()
    ref = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    b2g.gemm(dA, dB, ref)
    b2g.sync_status()
    r = to_host(ref)
    assert np.array_equal(to_host(D), r)
    for c in copies:
        assert np.array_equal(to_host(c), r)


def test_gemm_peers_rejects_what_it_cannot_push():
    A, B, _ = inputs(64, 60, 64)
    dA, dB = to_dev(torch, A), to_dev(torch, B)
    D = torch.empty((64, 60), dtype=torch.float16, device="cuda")
    other = torch.empty_like(D)
    with pytest.raises(b2g.B2GError) as e:
        b2g.gemm_peers(dA, dB, D, [other.data_ptr()])   # N % 8 != 0
    assert e.value.code == b2g.ERR_ALIGN
    b2g.gemm_peers(dA, dB, D, [])                       # no copies: plain GEMM, any N
    b2g.sync_status()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _ipc_worker(rank, world, port, q):
    import sys

    sys.path[:0] = [os.path.join(ROOT, "ada-tensor-core-gemm_b200"), HERE,
                    os.path.join(ROOT, "oracle")]
    try:
        import torch
        import torch.distributed as dist

        import b2g
        from helpers import inputs, to_dev, to_host

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        torch.cuda.set_device(0)
        M, N, K = 1024, 768, 512
        A, B, _ = inputs(M, N, K, seed=21)
        r0, r1 = b2g.panel_rows(M, world, rank)
        dA, dB = to_dev(torch, A[r0:r1]), to_dev(torch, B)
        full = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
        torch.cuda.synchronize()
        handles = [None] * world
        dist.all_gather_object(handles, b2g.ipc_handle(full))
        bases, peers = [], []
        for p in range(world):
            if p == rank:
                continue
            h, off = handles[p]
            base = b2g.ipc_open(h)
            bases.append(base)
            peers.append(base + off + r0 * N * 2)
        b2g.gemm_peers(dA, dB, full[r0:r1], peers)
        b2g.sync_status()
        dist.barrier()  # every rank's pushes have completed
        # expected: every panel computed locally, as its owner computed it
        want = []
        for p in range(world):
            p0, p1 = b2g.panel_rows(M, world, p)
            ref = torch.empty((p1 - p0, N), dtype=torch.float16, device="cuda")
            b2g.gemm(to_dev(torch, A[p0:p1]), dB, ref)
            want.append(to_host(ref))
        b2g.sync_status()
        ok = bool(np.array_equal(to_host(full), np.concatenate(want)))
        dist.barrier()  # nobody still reads a mapping
        for base in bases:
            b2g.ipc_close(base)
        dist.destroy_process_group()
        q.put((rank, ok, ""))
    except Exception as e:  # noqa: BLE001
        q.put((rank, False, repr(e)))


def test_ipc_fused_allgather_two_processes():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ipc_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = []
    try:
        for _ in procs:
            results.append(q.get(timeout=180))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for rank, ok, err in sorted(results):
        assert ok, f"rank {rank}: {err or 'gathered D differs'}"
