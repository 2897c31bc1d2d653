"""Row-sharded (column-parallel) dequant-GEMM: host logic on CPU ranks (gloo).

The sharded layer splits output rows across ranks the way ptqkit's CPU kernel
splits them across OpenMP threads (src/ptqkit/csrc/dequant_gemm.cpp:196-205)
and all-gathers y. Here each gloo rank computes its shard with the oracle, the
shards are gathered with the same collective call the GPU path uses, and the
result must equal the unsharded oracle output bit for bit (rows are
independent). A rank that never joins must make the others fail with an error
within the process group's timeout, never hang.
"""

from __future__ import annotations

import importlib
import os
import socket
import time
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_rows_cover_every_row_once() -> None:
    sharded = importlib.import_module("weight-quantizer_b200.sharded")
    for M in (1, 7, 128, 1000, 28672):
        for world in (1, 2, 3, 4, 8):
            mp_, ranges = sharded.shard_rows(M, world)
            assert mp_ == -(-M // world)
            covered = [r for (a, b) in ranges for r in range(a, b)]
            assert covered == list(range(M))
            assert all(b - a <= mp_ for a, b in ranges)


def _quantized_cpu(seed: int, M: int, K: int, group: int | None, bits: int = 4):  # type: ignore[no-untyped-def]
    wq = importlib.import_module("weight-quantizer_b200")
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(M, K, generator=g) * 0.02
    r = oracle.quantize_stored(w.numpy(), bits, True, group)
    qw = wq.QuantizedWeight(
        codes=torch.from_numpy(r["q"]), scales=torch.from_numpy(r["scales"]), zeros=torch.from_numpy(r["zeros"]),
        bits=bits, group_size=int(r["group_size"]), in_features=K, out_features=M, symmetric=True,
        packed=bits == 4, granularity="group" if group else "channel")
    x = torch.randn(5, K, generator=g)
    return qw, x


def _oracle_y(qw, x: torch.Tensor) -> np.ndarray:  # type: ignore[no-untyped-def]
    return oracle.dequant_gemm(x.numpy(), qw.codes.numpy(), qw.scales.numpy(), qw.zeros.numpy(), None,
                               qw.group_size, qw.bits, 1)


def _gather_worker(rank: int, world: int, port: int, M: int, K: int, group: int | None, out_dir: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    sharded = importlib.import_module("weight-quantizer_b200.sharded")
    qw, x = _quantized_cpu(1, M, K, group)
    shard = sharded.shard_weight(qw, rank, world)
    y_local = torch.from_numpy(_oracle_y(shard, x))
    mp_, _ = sharded.shard_rows(M, world)
    gathered = torch.empty(world, x.shape[0], mp_)
    sharded.gather_shards(y_local, gathered)
    full = gathered.permute(1, 0, 2).reshape(x.shape[0], world * mp_)[:, :M]
    np.save(os.path.join(out_dir, f"y{rank}.npy"), full.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,M,group", [(2, 96, 32), (3, 100, None), (2, 7, 16)])
def test_sharded_gather_equals_unsharded(tmp_path, world: int, M: int, group: int | None) -> None:
    K = 64
    mp.spawn(_gather_worker, args=(world, _port(), M, K, group, str(tmp_path)), nprocs=world, join=True)
    qw, x = _quantized_cpu(1, M, K, group)
    expect = _oracle_y(qw, x)
    for r in range(world):
        got = np.load(tmp_path / f"y{r}.npy")
        assert np.array_equal(got.view(np.int32), expect.view(np.int32)), r


def _absent_peer_worker(rank: int, port: int, out_dir: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=4))
    sharded = importlib.import_module("weight-quantizer_b200.sharded")
    if rank == 1:
        time.sleep(12)  # alive, but never joins the collective
        return
    t0 = time.time()
    outcome = "completed"
    try:
        sharded.gather_shards(torch.ones(2, 3), torch.empty(2, 2, 3))
    except Exception as e:  # noqa: BLE001 - the collective's error type depends on the backend
        outcome = f"raised {type(e).__name__}"
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(f"{outcome} {time.time() - t0:.1f}")


def test_rank_that_never_joins_fails_the_collective(tmp_path) -> None:
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=_absent_peer_worker, args=(r, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    for p in procs:
        if p.is_alive():
            p.kill()
    text = (tmp_path / "rank0.txt").read_text().split()
    assert text[0] == "raised", text
    assert float(text[-1]) < 30.0


def _choose_worker(rank: int, world: int, port: int, fail: str, out_dir: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    sharded = importlib.import_module("weight-quantizer_b200.sharded")
    calls: list[str] = []

    def setup_local() -> str:
        calls.append("local")
        if fail == f"local{rank}":
            raise RuntimeError("out of memory (injected on this rank)")
        return "buffers"

    def setup_collective(state: str) -> None:
        assert state == "buffers"
        calls.append("collective")
        dist.barrier()   # the collective phase is a collective
        if fail == f"collective{rank}":
            raise RuntimeError("rendezvous failed (injected on this rank)")

    ok = sharded.choose_collectively(setup_local, setup_collective, None, torch.device("cpu"))
    dist.barrier()   # every rank is still in step after the choice
    with open(os.path.join(out_dir, f"r{rank}.txt"), "w") as f:
        f.write(f"{int(ok)} {','.join(calls)}")
    dist.destroy_process_group()


@pytest.mark.parametrize("fail", ["none", "local1", "local0", "collective1"])
def test_exchange_choice_is_collective(tmp_path, fail: str) -> None:
    """A setup failure on one rank alone sends every rank to the same choice,
    with every rank taking the same collectives (no rank left waiting)."""
    world = 3
    mp.spawn(_choose_worker, args=(world, _port(), fail, str(tmp_path)), nprocs=world, join=True)
    results = [(tmp_path / f"r{r}.txt").read_text().split() for r in range(world)]
    oks = {res[0] for res in results}
    assert oks == {"1" if fail == "none" else "0"}, results
    if fail.startswith("local"):
        assert all(res[1] == "local" for res in results), results   # nobody entered the rendezvous
