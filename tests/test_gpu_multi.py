"""Column-sharded swiglu on two GPUs (one process per GPU), against the single-GPU operator:
NCCL all-gather with 1 or 2 row chunks, and the fused kernel that stores into both ranks'
buffers over NVLink. Skipped when fewer than two GPUs are visible."""
import math
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    import datetime

    import torch.distributed as dist

    import tritonllmcompiler_b200 as T
    from tritonllmcompiler_b200 import sharded as S

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        m, k, n = 1000, 1024, 2048
        g = torch.Generator(device="cuda").manual_seed(5)
        x = torch.randn(m, k, generator=g, device="cuda").half()
        w1 = (torch.randn(k, n, generator=g, device="cuda") / math.sqrt(k)).half()
        w3 = (torch.randn(k, n, generator=g, device="cuda") / math.sqrt(k)).half()
        n0, n1 = S.column_range(n, rank, world)
        w1l, w3l = w1[:, n0:n1].contiguous(), w3[:, n0:n1].contiguous()
        full = T.swiglu(x, w1, w3)
        if mode.startswith("peers"):
            peers = S.PeerBuffers((m, n), x.dtype, x.device, slots=int(mode[-1]))
            ok = True
            for _ in range(3):  # the slots are reused across calls
                peers.local.fill_(float("nan"))
                torch.cuda.synchronize()
                dist.barrier()
                out = S.swiglu_column_sharded(x, w1l, w3l, peers=peers)
                torch.cuda.synchronize()
                ok = ok and bool(torch.equal(out, full))
            dist.barrier()
            peers.close()
        else:
            out = S.swiglu_column_sharded(x, w1l, w3l, chunks=int(mode))
            torch.cuda.synchronize()
            ok = bool(torch.equal(out, full))
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["1", "2", "peers1", "peers2"])
def test_swiglu_column_sharded_two_gpus(cuda_device, mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res == {0: True, 1: True}
