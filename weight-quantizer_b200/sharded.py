"""Row-sharded (column-parallel) dequant-GEMM across the GPUs of one node.

ptqkit splits the output rows of a layer across OpenMP threads
(src/ptqkit/csrc/dequant_gemm.cpp:196-205). Here the same split is taken across
GPUs, one process per GPU: rank r owns rows [r*Mp, (r+1)*Mp) of the packed
codes and of the scale/zero tables (Mp = ceil(M / world); the last shard is
padded with rows whose output is dropped), while x and the channel scale are
replicated. Per-tensor granularity (one scale for all rows) is replicated on
every rank. When the whole y is needed on every rank there are two exchanges:

* ``exchange="p2p"``: every rank maps the other ranks' full
  y buffers [B, world*Mp] once (CUDA IPC over NVLink) and the dequant-GEMM's
  epilogue stores each finished value into all of them, so the exchange
  overlaps the computation. y alternates between two buffers, so a
  one-element NCCL all-reduce after each call is the only ordering needed:
  when any rank starts call i+2 (which rewrites the buffer of call i), every
  rank has passed call i+1's all-reduce and therefore finished whatever it
  did with call i's y before call i+1. A returned y stays valid until the
  second following forward with the same batch size.
* ``exchange="nvls"``: the full y buffers are PyTorch symmetric memory and
  the epilogue stores each value once through the NVLink switch address that
  reaches every rank's buffer (NVLS), so each GPU sends its rows once instead
  of once per peer; falls back to peer stores where the switch address is not
  available. Same ordering as p2p.
* ``exchange="auto"`` (default): nvls, or p2p if symmetric memory cannot be
  set up on this system. The ranks agree on the choice (a MIN all-reduce of
  each rank's setup outcome, once after the local allocation and once after
  the collective rendezvous), so a setup that fails on one rank alone sends
  every rank to p2p instead of leaving the ranks in different collectives.
* ``exchange="nccl"``: the kernel writes the local shard, one NCCL all-gather
  collects [world, B, Mp] and a permute kernel lays it out as [B, M].
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _kernels
from .quant import QuantizedWeight


def shard_rows(M: int, world: int) -> tuple[int, list[tuple[int, int]]]:
    """Padded shard height Mp and the [r0, r1) row range of every rank."""
    if world < 1:
        raise ValueError("world size must be positive")
    mp = (M + world - 1) // world
    ranges = [(min(r * mp, M), min((r + 1) * mp, M)) for r in range(world)]
    return mp, ranges


def shard_weight(qw: QuantizedWeight, rank: int, world: int) -> QuantizedWeight:
    """Rows of ``qw`` owned by ``rank``, padded to the common shard height with
    zero codes (their outputs are discarded after the gather)."""
    mp, ranges = shard_rows(qw.out_features, world)
    r0, r1 = ranges[rank]
    rows = r1 - r0

    def take(t: torch.Tensor) -> torch.Tensor:
        part = t[r0:r1]
        if rows == mp:
            return part.contiguous()
        pad = torch.zeros((mp - rows,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        if t.dtype.is_floating_point and t is qw.scales:
            pad.fill_(1.0)
        return torch.cat((part, pad), dim=0).contiguous()

    per_row = int(qw.scales.shape[0]) == qw.out_features and qw.out_features > 1
    return QuantizedWeight(
        codes=take(qw.codes),
        scales=take(qw.scales) if per_row else qw.scales.contiguous(),
        zeros=take(qw.zeros) if per_row else qw.zeros.contiguous(),
        bits=qw.bits,
        group_size=qw.group_size,
        in_features=qw.in_features,
        out_features=mp,
        symmetric=qw.symmetric,
        packed=qw.packed,
        granularity=qw.granularity,
        channel_scale=qw.channel_scale,
    )


def all_ranks_agree(ok: bool, group: dist.ProcessGroup | None, device: torch.device) -> bool:
    """True on every rank iff ``ok`` is true on every rank (MIN all-reduce)."""
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    return bool(int(flag.item()) == 1)


_SETUP_ERRORS = (RuntimeError, AttributeError, ImportError, ValueError, NotImplementedError)


def choose_collectively(setup_local, setup_collective, group: dist.ProcessGroup | None,  # type: ignore[no-untyped-def]
                        device: torch.device) -> bool:
    """Run a two-phase setup and agree on its outcome across ranks.

    ``setup_local()`` may fail on any rank alone (an allocation); it returns a
    state handed to ``setup_collective(state)``, which every rank enters only
    if every rank's local phase succeeded (it may itself be a collective).
    Returns True on every rank iff both phases succeeded on every rank; the
    ranks always take the same collective calls in the same order."""
    state = None
    try:
        state = setup_local()
        ok = True
    except _SETUP_ERRORS:
        ok = False
    if not all_ranks_agree(ok, group, device):
        return False
    try:
        setup_collective(state)
        ok = True
    except _SETUP_ERRORS:
        ok = False
    return all_ranks_agree(ok, group, device)


def gather_shards(y_local: torch.Tensor, out: torch.Tensor, group: dist.ProcessGroup | None = None) -> None:
    """All-gather every rank's [B, Mp] shard into ``out`` [world, B, Mp]."""
    dist.all_gather_into_tensor(out.view(-1), y_local.contiguous().view(-1), group=group)


class RowParallelDequantLinear:
    """One rank's part of a row-sharded quantized linear layer (no bias)."""

    def __init__(self, shard: QuantizedWeight, out_features: int, rank: int, world: int,
                 group: dist.ProcessGroup | None = None, exchange: str = "auto") -> None:
        mp, _ = shard_rows(out_features, world)
        if shard.out_features != mp:
            raise ValueError("shard height does not match the row split")
        if shard.codes.device.type != "cuda":
            raise ValueError("the shard must live on a CUDA device")
        self.shard = shard
        self.out_features = out_features
        self.rank = rank
        self.world = world
        self.group = group
        self.mp = mp
        if exchange not in ("auto", "p2p", "nvls", "nccl"):
            raise ValueError("exchange must be 'auto', 'p2p', 'nvls' or 'nccl'")
        self.exchange = exchange
        self._bufs: dict[int, tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = {}
        # batch -> two (full y, output pointers (own first), opened (ptr, offset) list) sets
        self._peer: dict[int, list[tuple[torch.Tensor, list[int], list[tuple[int, int]]]]] = {}
        # batch -> two (full y, output pointers (own first), switch address or 0, handle) sets
        self._nvls: dict[int, list[tuple[torch.Tensor, list[int], int, object]]] = {}
        self._calls: dict[int, int] = {}
        self._sync: torch.Tensor | None = None

    def _buffers(self, batch: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        if batch not in self._bufs:
            dev = self.shard.codes.device
            local = torch.empty((batch, self.mp), dtype=torch.float32, device=dev)
            gathered = torch.empty((self.world, batch, self.mp), dtype=torch.float32, device=dev)
            full = torch.empty((batch, self.world * self.mp), dtype=torch.float32, device=dev)
            self._bufs[batch] = (local, gathered, full)
        return self._bufs[batch]

    def forward_local(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """This rank's [B, Mp] shard of y."""
        s = self.shard
        return _kernels.dequant_gemm(x, s.codes, s.scales, s.zeros, s.channel_scale, s.group_size, s.bits, out=out)

    def _sync_word(self) -> torch.Tensor:
        if self._sync is None:
            self._sync = torch.zeros(1, dtype=torch.float32, device=self.shard.codes.device)
        return self._sync

    def _peer_buffers(self, batch: int) -> list[tuple[torch.Tensor, list[int], list[tuple[int, int]]]]:
        """Two full y [B, world*Mp] buffers on this rank, each with the pointers
        at which this rank's columns start in every rank's copy (own first)."""
        if batch not in self._peer:
            dev = self.shard.codes.device
            sets = []
            for _ in range(2):
                full = torch.empty((batch, self.world * self.mp), dtype=torch.float32, device=dev)
                handles: list[tuple[bytes, int] | None] = [None] * self.world
                dist.all_gather_object(handles, _kernels.ipc_handle(full), group=self.group)
                col = self.rank * self.mp * 4
                outs = [full.data_ptr() + col]
                opened: list[tuple[int, int]] = []
                for r in range(self.world):
                    if r == self.rank:
                        continue
                    h = handles[r]
                    assert h is not None
                    ptr = _kernels.ipc_open(h[0], h[1])
                    opened.append((ptr, h[1]))
                    outs.append(ptr + col)
                sets.append((full, outs, opened))
            self._peer[batch] = sets
        return self._peer[batch]

    def _nvls_alloc(self, batch: int) -> list[torch.Tensor]:
        """This rank's two full y buffers in symmetric memory (local; may fail
        on one rank alone, e.g. out of memory)."""
        from torch.distributed import _symmetric_memory as symm_mem

        dev = self.shard.codes.device
        return [symm_mem.empty((batch, self.world * self.mp), dtype=torch.float32, device=dev) for _ in range(2)]

    def _nvls_bind(self, batch: int, fulls: list[torch.Tensor]) -> None:
        """Collective: binds both buffers across the ranks and records this
        rank's column pointers in every rank's copy and the NVLink-switch
        address (0 when the system has none)."""
        from torch.distributed import _symmetric_memory as symm_mem

        group = self.group if self.group is not None else dist.group.WORLD
        col = self.rank * self.mp * 4
        sets = []
        for full in fulls:
            handle = symm_mem.rendezvous(full, group)
            ptrs = [int(p) for p in handle.buffer_ptrs]
            outs = [ptrs[self.rank] + col] + [ptrs[r] + col for r in range(self.world) if r != self.rank]
            switch = int(getattr(handle, "multicast_ptr", 0) or 0)
            sets.append((full, outs, switch + col if switch else 0, handle))
        self._nvls[batch] = sets

    def _nvls_buffers(self, batch: int) -> list[tuple[torch.Tensor, list[int], int, object]]:
        """Two full y buffers in symmetric memory, with this rank's column
        pointers in every rank's copy and the NVLink-switch address (0 when the
        system has none)."""
        if batch not in self._nvls:
            self._nvls_bind(batch, self._nvls_alloc(batch))
        return self._nvls[batch]

    def close(self) -> None:
        """Unmaps the peers' y buffers (every rank calls it; the mappings also
        end with the process)."""
        for sets in self._peer.values():
            for _, _, opened in sets:
                for ptr, off in opened:
                    _kernels.ipc_close(ptr, off)
        self._peer.clear()
        self._nvls.clear()

    def forward(self, x: torch.Tensor, gather: bool = True) -> torch.Tensor:
        """y [B, M] on every rank (gather=True), else this rank's [B, Mp] shard."""
        batch = int(x.shape[0])
        if gather and self.world > 1 and self.exchange == "auto":
            ok = choose_collectively(lambda: self._nvls_alloc(batch), lambda fulls: self._nvls_bind(batch, fulls),
                                     self.group, self.shard.codes.device)
            if not ok:
                self._nvls.pop(batch, None)   # drop a half-built set
            self.exchange = "nvls" if ok else "p2p"
        if gather and self.world > 1 and self.exchange in ("nvls", "p2p"):
            k = self._calls.get(batch, 0)
            self._calls[batch] = k + 1
            s = self.shard
            if self.exchange == "nvls":
                full, outs, switch, _ = self._nvls_buffers(batch)[k & 1]
            else:
                full, outs, _ = self._peer_buffers(batch)[k & 1]
                switch = 0
            _kernels.dequant_gemm_multi(x, s.codes, s.scales, s.zeros, s.channel_scale, s.group_size, s.bits,
                                        outs, self.world * self.mp, y_all=switch)
            dist.all_reduce(self._sync_word(), group=self.group)   # every rank's rows are in every y
            return full[:, : self.out_features]
        local, gathered, full = self._buffers(batch)
        self.forward_local(x, out=local)
        if not gather:
            return local
        if self.world == 1:
            return local[:, : self.out_features]
        gather_shards(local, gathered, self.group)
        _kernels.gather_permute(gathered, self.world, out=full)
        return full[:, : self.out_features]
