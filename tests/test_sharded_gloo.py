"""Multi-rank host logic of the sharded operators on CPU ranks (gloo, world_size 2).

The per-rank compute function is injected (the CPU oracle), so the partitioning, the NCCL/gloo
all-gather and the column re-assembly are checked without a GPU.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tritonllmcompiler_b200 import sharded as S


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _oracle_swiglu(x, w1, w3):
    from oracle import ops_oracle as O

    return torch.from_numpy(O.swiglu(x.float().numpy(), w1.float().numpy(), w3.float().numpy())).half()


def _worker(rank, world, port, chunks, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(7)
        m, k, n = 24, 32, 48
        x = torch.randn(m, k, generator=g).half()
        w1 = (torch.randn(k, n, generator=g) / 6).half()
        w3 = (torch.randn(k, n, generator=g) / 6).half()
        n0, n1 = S.column_range(n, rank, world)
        out = S.swiglu_column_sharded(x, w1[:, n0:n1].contiguous(), w3[:, n0:n1].contiguous(),
                                      chunks=chunks, op=_oracle_swiglu)
        full = _oracle_swiglu(x, w1, w3)
        result_q.put((rank, bool(torch.equal(out, full))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("chunks", [1, 3])
def test_swiglu_column_sharded_gloo(chunks):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, chunks, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res == {0: True, 1: True}


def _rank_that_fails(rank, world, port, result_q):
    """Rank 1 raises before the collective; rank 0 must end with an error, not hang."""
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        if rank == 1:
            raise RuntimeError("injected failure on rank 1")
        t = torch.zeros(4)
        try:
            dist.all_reduce(t)
            result_q.put((rank, "completed"))
        except Exception as e:  # gloo reports the peer that went away / timed out
            result_q.put((rank, "error:" + type(e).__name__))
    except RuntimeError:
        result_q.put((rank, "raised"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_failed_rank_surfaces_as_error_not_hang():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_that_fails, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert res[1] == "raised"
    assert res[0].startswith("error:")


def test_head_and_column_ranges():
    assert [S.head_range(64, r, 8) for r in (0, 7)] == [(0, 8), (56, 64)]
    with pytest.raises(ValueError):
        S.head_range(6, 0, 4)
    assert S.column_range(14336, 3, 8) == (5376, 7168)
    with pytest.raises(ValueError):
        S.column_range(100, 0, 8)


def test_partition_sequences_balances_tokens():
    rng = np.random.default_rng(4)
    lens = rng.integers(1024, 32769, size=256).tolist()
    for world in (2, 4, 8):
        parts = S.partition_sequences(lens, world, "tokens")
        assert sorted(i for p in parts for i in p) == list(range(256))
        loads = [sum(lens[i] for i in p) for p in parts]
        assert max(loads) - min(loads) <= max(lens)  # LPT bound
        cnt = S.partition_sequences(lens, world, "count")
        assert [len(p) for p in cnt] == [256 // world] * world
        cnt_loads = [sum(lens[i] for i in p) for p in cnt]
        assert max(loads) <= max(cnt_loads)


def test_localize_blocks_matches_global_view():
    from oracle import ops_oracle as O

    g = torch.Generator().manual_seed(9)
    bs, h, d = 16, 2, 32
    lens = [40, 3, 70, 16]
    nb = [(n + bs - 1) // bs for n in lens]
    pool = sum(nb) + 4
    perm = torch.randperm(pool, generator=g)
    bt = torch.zeros(4, max(nb) + 1, dtype=torch.int32)
    pos = 0
    for i, n in enumerate(nb):
        bt[i, :n] = perm[pos:pos + n].to(torch.int32)
        pos += n
    kc = torch.randn(pool, bs, h, d, generator=g).half()
    vc = torch.randn(pool, bs, h, d, generator=g).half()
    q = torch.randn(4, h, 1, d, generator=g).half()
    cl = torch.tensor(lens, dtype=torch.int32)
    full = O.paged_attention(q.float().numpy(), kc.float().numpy(), vc.float().numpy(), bt.numpy(),
                             cl.numpy(), block_size=bs)
    for part in S.partition_sequences(lens, 2):
        ids, lbt, lcl = S.localize_blocks(bt, cl, part, bs)
        local = O.paged_attention(q[part].float().numpy(), kc[ids].float().numpy(),
                                  vc[ids].float().numpy(), lbt.numpy(), lcl.numpy(), block_size=bs)
        assert np.array_equal(local, full[part])


def test_ipc_handles_are_opened_once_and_closed_by_the_last_user(monkeypatch):
    """Small tensors of one rank can share an allocation (the caching allocator sub-allocates),
    so their IPC handles can be equal: the mapping is opened once and closed only when its last
    user releases it. Checked with a stand-in for the library's IPC calls (no GPU)."""
    import ctypes

    from tritonllmcompiler_b200 import _lib

    calls = []

    class FakeLib:
        def tllm_ipc_open(self, handle, offset, ptr, base):
            calls.append(("open", handle))
            ctypes.cast(base, ctypes.POINTER(ctypes.c_void_p))[0] = 0x10000
            return 0

        def tllm_ipc_close(self, base):
            calls.append(("close", base))
            return 0

    monkeypatch.setattr(_lib, "load", lambda: FakeLib())
    h1, h2 = b"A" * 64, b"B" * 64
    p, h = S._ipc_open(h1, 256)
    assert p == 0x10000 + 256 and h == h1
    assert S._ipc_open(h1, 512)[0] == 0x10000 + 512  # same allocation: no second open
    S._ipc_open(h2, 0)
    assert [c[0] for c in calls] == ["open", "open"]
    S._ipc_release(h1)
    assert [c[0] for c in calls] == ["open", "open"]  # one user of h1 left
    S._ipc_release(h1)
    S._ipc_release(h2)
    assert [c[0] for c in calls] == ["open", "open", "close", "close"]
    assert not S._IPC_OPEN
