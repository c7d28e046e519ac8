"""Sharded operators on 2, 4 and 8 GPUs (one process per GPU), against the single-GPU
operators on the same inputs. Skipped when fewer GPUs are visible than the case needs.

Per world size, one group of processes runs every mode:
* swiglu column-sharded, the all-gather fused into the GEMM epilogue with the in-kernel peer
  handshake: automatic kernel, forced one-CTA and CTA-pair kernels (128-byte and 256-byte row
  stores), one and two output slots,
  a column slice that is not a multiple of 128 (one-CTA kernel), several calls in a row with
  the output poisoned in between -- bit-identical to ``swiglu`` on one GPU;
* swiglu column-sharded with the output stored once through an NVLink multicast address
  (torch symmetric memory), where the devices offer multicast -- bit-identical;
* swiglu column-sharded with the NCCL all-gather (1 and 2 row chunks) -- bit-identical;
* flash_attention head-sharded -- bit-identical to the full problem's heads;
* paged_attention batch-sharded over a token-balanced partition with rank-local block pools
  -- within the operator tolerance of the full problem's sequences (the split-KV plan
  depends on the batch, so the summation order may differ).
"""
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


def _multicast_ok():
    from torch._C._distributed_c10d import _SymmetricMemory

    return bool(_SymmetricMemory.has_multicast_support(torch._C._autograd.DeviceType.CUDA,
                                                       torch.cuda.current_device()))


def _swiglu_modes(rank, world, T, S, dist):
    res = {}
    for (m, k, n_loc) in [(1000, 1024, 256), (300, 512, 136)]:
        n = n_loc * world
        g = torch.Generator(device="cuda").manual_seed(5 + n_loc)
        x = torch.randn(m, k, generator=g, device="cuda").half()
        w1 = (torch.randn(k, n, generator=g, device="cuda") / math.sqrt(k)).half()
        w3 = (torch.randn(k, n, generator=g, device="cuda") / math.sqrt(k)).half()
        n0, n1 = S.column_range(n, rank, world)
        w1l, w3l = w1[:, n0:n1].contiguous(), w3[:, n0:n1].contiguous()
        full = T.swiglu(x, w1, w3)
        variants = [0, 1, 2, 3] if n_loc % 128 == 0 else [0, 1]
        for slots in (1, 2):
            for variant in variants:
                peers = S.PeerBuffers((m, n), x.dtype, x.device, slots=slots)
                ok = True
                for _ in range(3):  # the slots are reused across calls
                    peers.local.fill_(float("nan"))
                    torch.cuda.synchronize()
                    dist.barrier()
                    out = S.swiglu_column_sharded(x, w1l, w3l, peers=peers, variant=variant)
                    torch.cuda.synchronize()
                    ok = ok and bool(torch.equal(out, full))
                # back to back with no host barrier or synchronisation: each call's output is
                # copied on this rank's stream before the next call may overwrite it
                outs = []
                for _ in range(4):
                    out = S.swiglu_column_sharded(x, w1l, w3l, peers=peers, variant=variant)
                    outs.append(out.clone())
                torch.cuda.synchronize()
                ok = ok and all(bool(torch.equal(o, full)) for o in outs)
                dist.barrier()
                peers.close()
                res[f"peers m{m} nloc{n_loc} slots{slots} variant{variant}"] = ok
        if _multicast_ok():
            # Output stored once through an NVLink multicast address (CTA-pair kernel; the
            # 136-column slice runs the one-CTA kernel with per-destination stores).
            for slots in (1, 2):
                peers = S.PeerBuffers((m, n), x.dtype, x.device, slots=slots, multicast=True)
                ok = True
                for _ in range(3):
                    peers.local.fill_(float("nan"))
                    torch.cuda.synchronize()
                    dist.barrier()
                    out = S.swiglu_column_sharded(x, w1l, w3l, peers=peers)
                    torch.cuda.synchronize()
                    ok = ok and bool(torch.equal(out, full))
                outs = []
                for _ in range(4):
                    out = S.swiglu_column_sharded(x, w1l, w3l, peers=peers)
                    outs.append(out.clone())
                torch.cuda.synchronize()
                ok = ok and all(bool(torch.equal(o, full)) for o in outs)
                dist.barrier()
                peers.close()
                res[f"multicast m{m} nloc{n_loc} slots{slots}"] = ok
        for chunks in (1, 2):
            out = S.swiglu_column_sharded(x, w1l, w3l, chunks=chunks)
            torch.cuda.synchronize()
            res[f"nccl m{m} nloc{n_loc} chunks{chunks}"] = bool(torch.equal(out, full))
    from tritonllmcompiler_b200 import _lib

    res["no device errors"] = _lib.debug_status() == 0
    return res


def _flash_mode(rank, world, T, S):
    b, h, s, d = 2, 4 * world, 384, 128
    g = torch.Generator(device="cuda").manual_seed(11)
    q, k, v = (torch.randn(b, h, s, d, generator=g, device="cuda").half() for _ in range(3))
    full = T.flash_attention(q, k, v, causal=True)
    h0, h1 = S.head_range(h, rank, world)
    loc = S.flash_attention_head_sharded(q[:, h0:h1].contiguous(), k[:, h0:h1].contiguous(),
                                         v[:, h0:h1].contiguous(), causal=True)
    torch.cuda.synchronize()
    return {"flash head-sharded": bool(torch.equal(loc, full[:, h0:h1]))}


def _paged_mode(rank, world, T, S):
    from tests import _golden as G

    bsz, h, d, bs = 6 * world, 8, 128, 16
    g = torch.Generator().manual_seed(13)
    lens = torch.randint(1, 3000, (bsz,), generator=g, dtype=torch.int32)
    nb = [(int(n) + bs - 1) // bs for n in lens]
    pool = sum(nb)
    perm = torch.randperm(pool, generator=g)
    bt = torch.zeros(bsz, max(nb), dtype=torch.int32)
    pos = 0
    for i, n in enumerate(nb):
        bt[i, :n] = perm[pos:pos + n].to(torch.int32)
        pos += n
    gd = torch.Generator(device="cuda").manual_seed(13)
    kc = torch.randn(pool, bs, h, d, generator=gd, device="cuda").half()
    vc = torch.randn(pool, bs, h, d, generator=gd, device="cuda").half()
    q = torch.randn(bsz, h, 1, d, generator=gd, device="cuda").half()
    full = T.paged_attention(q, kc, vc, bt.cuda(), lens.cuda(), block_size=bs)
    seqs = S.partition_sequences(lens.tolist(), world, "tokens")[rank]
    ids, lbt, llen = S.localize_blocks(bt, lens, seqs, bs)
    idx = ids.cuda()
    sel = torch.tensor(seqs, dtype=torch.int64, device="cuda")
    loc = T.paged_attention(q[sel].contiguous(), kc[idx].contiguous(), vc[idx].contiguous(),
                            lbt.cuda(), llen.cuda(), block_size=bs)
    torch.cuda.synchronize()
    ok = bool(torch.allclose(loc.float(), full[sel].float(), **G.tol(torch.float16)))
    return {"paged batch-sharded": ok and len(seqs) > 0}


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    import tritonllmcompiler_b200 as T
    from tritonllmcompiler_b200 import sharded as S

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        res = {}
        res.update(_swiglu_modes(rank, world, T, S, dist))
        res.update(_flash_mode(rank, world, T, S))
        res.update(_paged_mode(rank, world, T, S))
        q.put((rank, res))
        dist.barrier()
    except Exception as e:  # reported to the parent; the others time out in their collective
        q.put((rank, {"exception": repr(e)}))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_operators(cuda_device, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0
    bad = {(r, k): v for r, d in res.items() for k, v in d.items() if v is not True}
    assert not bad, bad


def _worker_missing_peer(rank, world, port, q):
    import datetime
    import time

    import torch.distributed as dist

    from tritonllmcompiler_b200 import _lib
    from tritonllmcompiler_b200 import sharded as S

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        import tritonllmcompiler_b200 as T

        m, k, n_loc = 512, 256, 256
        n = n_loc * world
        g = torch.Generator(device="cuda").manual_seed(3)
        x = torch.randn(m, k, generator=g, device="cuda").half()
        w1 = (torch.randn(k, n, generator=g, device="cuda") / math.sqrt(k)).half()
        w3 = (torch.randn(k, n, generator=g, device="cuda") / math.sqrt(k)).half()
        n0, n1 = S.column_range(n, rank, world)
        w1l, w3l = w1[:, n0:n1].contiguous(), w3[:, n0:n1].contiguous()
        full = T.swiglu(x, w1, w3)
        peers = S.PeerBuffers((m, n), x.dtype, x.device)
        out = S.swiglu_column_sharded(x, w1l, w3l, peers=peers)
        torch.cuda.synchronize()
        res = {"healthy call": bool(torch.equal(out, full)), "status clean": _lib.debug_status() == 0}
        dist.barrier()
        if rank == 0:
            # Rank 1 skips this call: rank 0's kernel must give up on its peer (bounded waits)
            # and report it, not hang.
            t0 = time.time()
            S.swiglu_column_sharded(x, w1l, w3l, peers=peers)
            torch.cuda.synchronize()
            res["gave up within 30 s"] = time.time() - t0 < 30
            res["timeout reported"] = (_lib.debug_status() & 0xF00) == 0x100
            res["context still usable"] = bool(torch.equal(T.swiglu(x, w1, w3), full))
        dist.barrier()
        peers.close()
        q.put((rank, res))
        dist.barrier()
    except Exception as e:
        q.put((rank, {"exception": repr(e)}))
        raise
    finally:
        dist.destroy_process_group()


def test_peer_that_never_launches_is_reported(cuda_device):
    """A rank that skips a column-sharded call (the failure is made on the host) leaves its
    peer's kernel waiting on flags that nobody sets: the waits are bounded, the kernel returns,
    the timeout is reported through the device status word and the context keeps working."""
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker_missing_peer, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    bad = {(r, k): v for r, d in res.items() for k, v in d.items() if v is not True}
    assert not bad, bad
    assert "timeout reported" in res[0]
