"""Row-sharded dequant-GEMM on GPUs: the permute kernel, the one-rank layer, and
(with two or more GPUs) the NCCL and peer-store exchanges compared with the
unsharded layer, at batches that run each kernel's multi-output epilogue
(1: the batch-1/2 decode kernel, 8: the batch 3-32 kernel, 64 and 1024: the
tcgen05 kernel's 64- and 192-wide tiles)."""

from __future__ import annotations

import importlib
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import assert_close_y

pytestmark = pytest.mark.gpu


def test_gather_permute_kernel(wq, cuda) -> None:
    g = torch.Generator().manual_seed(3)
    for P, B, Mp in [(1, 3, 5), (2, 7, 33), (8, 4, 3584), (3, 1, 1)]:
        src = torch.randn(P, B, Mp, generator=g).to(cuda)
        got = wq._kernels.gather_permute(src, P)
        assert torch.equal(got, src.permute(1, 0, 2).reshape(B, P * Mp))


def test_row_parallel_single_rank(wq, cuda) -> None:
    sharded = importlib.import_module("weight-quantizer_b200.sharded")
    g = torch.Generator().manual_seed(4)
    w = torch.randn(1000, 2048, generator=g) * 0.02
    qw = wq.quantize_weight(w, wq.QuantConfig(bits=4, symmetric=True, group_size=128))
    lin = sharded.RowParallelDequantLinear(sharded.shard_weight(qw, 0, 1), 1000, 0, 1)
    for b in (1, 40):
        x = torch.randn(b, 2048, generator=g).to(cuda)
        assert torch.equal(lin.forward(x), wq.dequant_gemm(x, qw, impl="kernel"))


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _nccl_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=120))
    wq = importlib.import_module("weight-quantizer_b200")
    sharded = importlib.import_module("weight-quantizer_b200.sharded")
    g = torch.Generator().manual_seed(5)
    M, K = 3001, 4096
    w = torch.randn(M, K, generator=g) * 0.02
    cfg = wq.QuantConfig(bits=4, symmetric=True, group_size=128)
    mp_, ranges = sharded.shard_rows(M, world)
    r0, r1 = ranges[rank]
    part = wq.quantize_weight(w[r0:r1].to(dev), cfg)
    full_rows = wq.QuantizedWeight(codes=part.codes, scales=part.scales, zeros=part.zeros, bits=4, group_size=128,
                                   in_features=K, out_features=r1 - r0, symmetric=True, packed=True,
                                   granularity="group")
    pad = mp_ - (r1 - r0)
    shard = full_rows if pad == 0 else wq.QuantizedWeight(
        codes=torch.cat((full_rows.codes, torch.zeros(pad, K // 2, dtype=torch.uint8, device=dev))),
        scales=torch.cat((full_rows.scales, torch.ones(pad, K // 128, device=dev))),
        zeros=torch.cat((full_rows.zeros, torch.zeros(pad, K // 128, device=dev))),
        bits=4, group_size=128, in_features=K, out_features=mp_, symmetric=True, packed=True, granularity="group")
    lin = sharded.RowParallelDequantLinear(shard, M, rank, world, exchange="nccl")
    p2p = sharded.RowParallelDequantLinear(shard, M, rank, world, exchange="p2p")
    nvls = sharded.RowParallelDequantLinear(shard, M, rank, world, exchange="nvls")
    for b in (1, 8, 64, 1024):
        x = torch.randn(b, K, generator=g).to(dev)
        y = lin.forward(x)
        np.save(os.path.join(out_dir, f"y{rank}_b{b}.npy"), y.cpu().numpy())
        for rep in range(2):   # the second call reuses the mapped peer buffers
            y2 = p2p.forward(x)
            np.save(os.path.join(out_dir, f"p2p{rank}_b{b}_{rep}.npy"), y2.cpu().numpy())
            y3 = nvls.forward(x)
            np.save(os.path.join(out_dir, f"nvls{rank}_b{b}_{rep}.npy"), y3.cpu().numpy())
    torch.cuda.synchronize()
    dist.barrier()
    p2p.close()
    nvls.close()
    dist.barrier()
    dist.destroy_process_group()


def test_row_parallel_nccl_matches_unsharded(wq, cuda, tmp_path) -> None:
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    mp.spawn(_nccl_worker, args=(world, _port(), str(tmp_path)), nprocs=world, join=True)
    g = torch.Generator().manual_seed(5)
    M, K = 3001, 4096
    w = torch.randn(M, K, generator=g) * 0.02
    qw = wq.quantize_weight(w.to(cuda), wq.QuantConfig(bits=4, symmetric=True, group_size=128))
    for b in (1, 8, 64, 1024):
        x = torch.randn(b, K, generator=g).to(cuda)
        expect = wq.dequant_gemm(x, qw, impl="kernel").cpu().numpy()
        for r in range(world):
            got = np.load(tmp_path / f"y{r}_b{b}.npy")
            assert_close_y(got, expect, f"rank {r} b{b}")
            # the peer-store exchange delivers the same values bit for bit
            for rep in range(2):
                assert np.array_equal(np.load(tmp_path / f"p2p{r}_b{b}_{rep}.npy"), got), (r, b, rep)
                assert np.array_equal(np.load(tmp_path / f"nvls{r}_b{b}_{rep}.npy"), got), ("nvls", r, b, rep)
