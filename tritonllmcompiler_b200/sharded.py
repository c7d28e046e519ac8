"""Multi-GPU partitioning of the four-op hot path (one process per GPU, torch.distributed).

The reference is single-GPU only. Across the GPUs of one node the operators shard as:

* flash_attention over heads: rank r owns heads [r*H/g, (r+1)*H/g) of q/k/v/o; no
  communication (``head_range``, ``flash_attention_head_sharded``).
* paged_attention over sequences: each rank owns whole sequences, their block-table rows and
  only their physical blocks, re-indexed into a rank-local pool; no communication
  (``partition_sequences``, ``localize_blocks``). Sequences are balanced by token count
  (greedy longest-first) because context lengths vary widely.
* swiglu over output columns: rank r holds x and the column slices w1[:, Nr], w3[:, Nr] and
  computes out[:, Nr] (``swiglu_column_sharded``). With ``PeerBuffers`` (the default in the
  benchmark) the GEMM epilogue stores each output tile straight into every rank's [M, N]
  buffer over NVLink, so there is no separate all-gather pass, and the kernel synchronises
  with its peers itself through flag words in every rank's memory (no host barrier, no NCCL
  call per step); without them the slices are all-gathered with NCCL and permuted into
  [M, N] (row chunks let the gather of chunk c overlap the GEMM of chunk c+1).

The per-rank compute function is a parameter only so the partitioning and gather logic can
be exercised on CPU ranks (gloo); the default is the CUDA operator.
"""
from __future__ import annotations

import ctypes
from typing import Callable, Sequence

import torch
import torch.distributed as dist


def head_range(num_heads: int, rank: int, world: int) -> tuple[int, int]:
    """Heads [h0, h1) owned by `rank`; num_heads must divide evenly."""
    if num_heads % world:
        raise ValueError(f"{num_heads} heads do not split over {world} ranks")
    per = num_heads // world
    return rank * per, (rank + 1) * per


def flash_attention_head_sharded(q_local, k_local, v_local, *, causal=False, sm_scale=None,
                                 op: Callable | None = None):
    """Attention over this rank's heads (inputs and output stay sharded)."""
    if op is None:
        from tritonllmcompiler_b200.ops.flash_attention import flash_attention as op
    return op(q_local, k_local, v_local, causal=causal, sm_scale=sm_scale)


def partition_sequences(context_lens: Sequence[int], world: int, scheme: str = "tokens") -> list[list[int]]:
    """Assigns sequence indices to ranks.

    scheme="count": contiguous runs of ceil(B/world) sequences.
    scheme="tokens": greedy longest-first onto the rank with the fewest tokens so far
    (ties broken by rank), each rank's list sorted ascending.
    """
    lens = [int(x) for x in context_lens]
    b = len(lens)
    if scheme == "count":
        per = -(-b // world) if b else 0
        return [list(range(r * per, min(b, (r + 1) * per))) for r in range(world)]
    if scheme != "tokens":
        raise ValueError(f"unknown scheme {scheme!r}")
    load = [0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(b), key=lambda i: (-lens[i], i)):
        r = min(range(world), key=lambda r: (load[r], r))
        out[r].append(i)
        load[r] += lens[i]
    return [sorted(x) for x in out]


def localize_blocks(block_tables: torch.Tensor, context_lens: torch.Tensor, seq_ids: Sequence[int],
                    block_size: int):
    """Rank-local view of a paged KV cache for the sequences `seq_ids`.

    Returns (global_block_ids, local_tables, local_lens): the physical blocks the sequences
    use (in first-use order; gather k_cache[global_block_ids] to build the local pool), the
    block tables re-indexed into that local pool (padding entries 0), and their lengths.
    Only the first ceil(len/block_size) entries of a row are read, as the reference does.
    """
    bt = block_tables.cpu()
    cl = context_lens.cpu()
    ids: list[int] = []
    remap: dict[int, int] = {}
    rows = []
    width = 1
    for s in seq_ids:
        n = (int(cl[s]) + block_size - 1) // block_size
        n = min(n, bt.shape[1])
        row = []
        for j in range(n):
            g = int(bt[s, j])
            if g not in remap:
                remap[g] = len(ids)
                ids.append(g)
            row.append(remap[g])
        rows.append(row)
        width = max(width, len(row))
    local = torch.zeros(len(seq_ids), width, dtype=torch.int32)
    for i, row in enumerate(rows):
        if row:
            local[i, :len(row)] = torch.tensor(row, dtype=torch.int32)
    lens = torch.tensor([int(cl[s]) for s in seq_ids], dtype=torch.int32)
    return torch.tensor(ids, dtype=torch.int64), local, lens


def column_range(n: int, rank: int, world: int, align: int = 8) -> tuple[int, int]:
    """Output columns [n0, n1) of `rank`; each slice is a multiple of `align` columns."""
    if n % (world * align):
        raise ValueError(f"N={n} does not split into {world} slices of a multiple of {align}")
    per = n // world
    return rank * per, (rank + 1) * per


# IPC mappings opened by this process: allocation handle -> [base pointer, users]. Small
# tensors of one rank can share an allocation (the caching allocator sub-allocates), so a
# handle is opened once and closed when its last user is done.
_IPC_OPEN: dict[bytes, list] = {}


def _ipc_open(handle: bytes, offset: int) -> tuple[int, bytes]:
    from tritonllmcompiler_b200 import _lib

    ent = _IPC_OPEN.get(handle)
    if ent is None:
        ptr, base = ctypes.c_void_p(), ctypes.c_void_p()
        _lib.check(_lib.load().tllm_ipc_open(handle, 0, ctypes.byref(ptr), ctypes.byref(base)))
        ent = _IPC_OPEN[handle] = [base.value, 0]
    ent[1] += 1
    return ent[0] + offset, handle


def _ipc_release(handle: bytes) -> None:
    from tritonllmcompiler_b200 import _lib

    ent = _IPC_OPEN.get(handle)
    if ent is None:
        return
    ent[1] -= 1
    if ent[1] == 0:
        del _IPC_OPEN[handle]
        _lib.load().tllm_ipc_close(ent[0])


class PeerBuffers:
    """[rows, cols] output buffers on every rank, each mapped into every rank's process
    (CUDA IPC), used in ``slots`` alternating copies, plus the flag words through which the
    column-sharded kernel synchronises with its peers.

    ``ptrs[slot][r]`` is rank r's buffer of that slot as seen from this process;
    ``locals[slot]`` is this rank's own tensor. A call stores into a peer only after the
    peer's own call has begun, and ends only once every peer's stores into this rank have
    landed, so a call's output is complete when its launch ends and stays valid until this
    rank's next call with the same slot (the call after next with two slots). Every rank
    must make every call. Create once per output shape (opening IPC handles is slow) and
    ``close()`` on every rank before the process group goes away.

    With ``multicast=True`` the output buffers are torch symmetric memory bound to an NVLink
    multicast object (``mc[slot]`` is its address): the CTA-pair kernel then stores each
    output block once and the NVSwitch writes it into every rank's buffer, so a rank sends its
    own slice over NVLink once instead of once per peer. Raises if the devices offer no
    multicast.
    """

    FLAG_WORDS = 16  # TLLM_SWIGLU_PEER_FLAG_WORDS

    def __init__(self, shape, dtype, device, group=None, slots: int = 2, multicast: bool = False):
        assert slots in (1, 2)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        assert self.world <= 8, "the column-sharded kernel writes at most 8 destinations"
        self.slots = slots
        self.calls = 0
        self.device = torch.device(device)
        self._handles: list[bytes] = []
        self._symm: list = []
        self.mc: list[int] = []
        with torch.cuda.device(self.device):
            self.flags = torch.zeros(self.FLAG_WORDS, dtype=torch.int32, device=self.device)
            self.done = torch.zeros(1, dtype=torch.int32, device=self.device)
            if multicast:
                import torch.distributed._symmetric_memory as symm

                name = (group if group is not None else dist.group.WORLD).group_name
                self.locals = []
                self.ptrs: list[list[int]] = []
                for _ in range(slots):
                    t = symm.empty(shape, dtype=dtype, device=self.device)
                    h = symm.rendezvous(t, name)
                    if not h.multicast_ptr:
                        raise RuntimeError("PeerBuffers: no NVLink multicast on these devices")
                    self._symm.append(h)
                    self.locals.append(t)
                    self.ptrs.append([int(p) for p in h.buffer_ptrs])
                    self.mc.append(int(h.multicast_ptr))
            else:
                self.locals = [torch.empty(shape, dtype=dtype, device=self.device)
                               for _ in range(slots)]
            torch.cuda.synchronize()  # zeroed before any peer can write a flag
        if not multicast:
            self.ptrs = [self._share(t) for t in self.locals]
        self._arrs = [(ctypes.c_void_p * self.world)(*p) for p in self.ptrs]
        self._flag_arr = (ctypes.c_void_p * self.world)(*self._share(self.flags))

    def _share(self, t: torch.Tensor) -> list[int]:
        """Every rank's tensor `t` (same role) as a pointer in this process."""
        from tritonllmcompiler_b200 import _lib

        lib = _lib.load()
        handle = (ctypes.c_char * 64)()
        offset = ctypes.c_uint64(0)
        with torch.cuda.device(self.device):
            _lib.check(lib.tllm_ipc_get_handle(t.data_ptr(), handle, ctypes.byref(offset)))
        infos = [None] * self.world
        dist.all_gather_object(infos, (bytes(handle), offset.value), group=self.group)
        ptrs = []
        with torch.cuda.device(self.device):
            for r, (hb, off) in enumerate(infos):
                if r == self.rank:
                    ptrs.append(t.data_ptr())
                    continue
                p, h = _ipc_open(hb, off)
                ptrs.append(p)
                self._handles.append(h)
        return ptrs

    @property
    def local(self) -> torch.Tensor:
        """This rank's buffer of the slot the next call writes."""
        return self.locals[self.calls % self.slots]

    def close(self):
        """Collective (every rank): releases the peers' mappings; multicast buffers are freed
        once every rank's device work is done."""
        with torch.cuda.device(self.device):
            if self._symm:
                torch.cuda.synchronize()
                dist.barrier(group=self.group)
                self._symm, self.mc, self.locals, self.ptrs = [], [], [], []
            for h in self._handles:
                _ipc_release(h)
        self._handles = []


def _swiglu_into_peers(x, w1_local, w3_local, peers: PeerBuffers, variant: int = 0):
    from tritonllmcompiler_b200 import _lib

    m, k = x.shape
    n_loc = w1_local.shape[1]
    slot = peers.calls % peers.slots
    out = peers.locals[slot]
    assert out.shape == (m, n_loc * peers.world) and out.dtype == x.dtype
    assert x.stride(1) == 1 and w1_local.stride(1) == 1 and w3_local.stride(1) == 1
    epoch = peers.calls % 0xFFFFFFFF + 1  # 1 .. 2^32 - 1, then 1 again; never 0 (the initial flags)
    with torch.cuda.device(x.device):
        if peers.mc:
            assert variant == 0, "the multicast path picks its kernel itself"
            _lib.check(_lib.load().tllm_swiglu_colshard_multicast(
                x.data_ptr(), w1_local.data_ptr(), w3_local.data_ptr(), peers._arrs[slot],
                peers.mc[slot], peers._flag_arr, peers.world, peers.rank, peers.done.data_ptr(),
                epoch, m, n_loc, k, x.stride(0), w1_local.stride(0), w3_local.stride(0),
                out.stride(0), _lib.DTYPE_CODES[x.dtype], _lib.stream_of(x)))
            peers.calls += 1
            return out
        _lib.check(_lib.load().tllm_swiglu_colshard_peers(
            x.data_ptr(), w1_local.data_ptr(), w3_local.data_ptr(), peers._arrs[slot],
            peers._flag_arr, peers.world, peers.rank, peers.done.data_ptr(), epoch, m, n_loc, k,
            x.stride(0), w1_local.stride(0), w3_local.stride(0), out.stride(0),
            _lib.DTYPE_CODES[x.dtype], variant, _lib.stream_of(x)))
    peers.calls += 1
    return out


def swiglu_column_sharded(x: torch.Tensor, w1_local: torch.Tensor, w3_local: torch.Tensor,
                          group=None, *, chunks: int = 1, op: Callable | None = None,
                          out: torch.Tensor | None = None,
                          peers: PeerBuffers | None = None, variant: int = 0) -> torch.Tensor:
    """out = silu(x @ w1) * (x @ w3) with w1/w3 column-sharded over the process group.

    Every rank passes the full x [M, K] and its column slices [K, N/g]; every rank returns
    the full [M, N] output. With ``peers`` (CUDA, one node) the kernel writes every rank's
    output directly and this rank's buffer of the slot just written is returned (``variant``
    picks the kernel: 0 automatic, 1 one CTA per tile, 2 CTA pairs). Otherwise the slices are
    all-gathered;
    with chunks > 1 the rows are processed in `chunks` blocks and the all-gather of block c
    runs on a side stream (CUDA) while block c+1 computes.
    """
    if peers is not None:
        return _swiglu_into_peers(x, w1_local, w3_local, peers, variant)
    if op is None:
        from tritonllmcompiler_b200.ops.swiglu import swiglu as op
    world = dist.get_world_size(group)
    m = x.shape[0]
    n_loc = w1_local.shape[1]
    n = n_loc * world
    if out is None:
        out = torch.empty((m, n), dtype=x.dtype, device=x.device)
    bounds = [(m * c) // chunks for c in range(chunks + 1)]
    cuda = x.is_cuda
    comm = torch.cuda.Stream(device=x.device) if (cuda and chunks > 1) else None
    pending = []
    for c in range(chunks):
        r0, r1 = bounds[c], bounds[c + 1]
        if r1 == r0:
            continue
        part = op(x[r0:r1], w1_local, w3_local)
        gathered = torch.empty((world, r1 - r0, n_loc), dtype=x.dtype, device=x.device)
        if comm is not None:
            comm.wait_stream(torch.cuda.current_stream(x.device))
            with torch.cuda.stream(comm):
                dist.all_gather_into_tensor(gathered.view(-1), part.contiguous().view(-1), group=group)
                out[r0:r1].view(r1 - r0, world, n_loc).copy_(gathered.permute(1, 0, 2))
            part.record_stream(comm)
            gathered.record_stream(comm)
            pending.append(gathered)
        else:
            dist.all_gather_into_tensor(gathered.view(-1), part.contiguous().view(-1), group=group)
            out[r0:r1].view(r1 - r0, world, n_loc).copy_(gathered.permute(1, 0, 2))
    if comm is not None:
        torch.cuda.current_stream(x.device).wait_stream(comm)
    return out
