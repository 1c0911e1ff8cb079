"""Batch-sharded data parallelism, host side, on CPU: world_size-2 `gloo`
ranks check that GradAllReduce averages every parameter gradient (complex
ones through their real view) exactly like one process over the global
batch, and that a rank failure surfaces as an error instead of a hang."""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from prospective_rqf_b200.train import GradAllReduce


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class Tiny(torch.nn.Module):
    """Complex and real parameters, like the encoder (W complex, readout real)."""

    def __init__(self):
        super().__init__()
        g = torch.Generator().manual_seed(0)
        self.W = torch.nn.Parameter(torch.complex(torch.randn(4, 3, generator=g),
                                                  torch.randn(4, 3, generator=g)))
        self.lin = torch.nn.Linear(8, 2)
        with torch.no_grad():
            self.lin.weight.copy_(torch.randn(2, 8, generator=g))
            self.lin.bias.copy_(torch.randn(2, generator=g))

    def forward(self, x):  # x (N, 3) complex
        h = x @ self.W.t()
        return self.lin(torch.cat([h.real, h.imag], dim=-1))


def _loss(model, x, y):
    return torch.nn.functional.cross_entropy(model(x), y, reduction="mean")


def _data(n):
    g = torch.Generator().manual_seed(1)
    x = torch.complex(torch.randn(n, 3, generator=g), torch.randn(n, 3, generator=g))
    y = torch.randint(0, 2, (n,), generator=g)
    return x, y


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        model = Tiny()
        x, y = _data(8)
        shard = slice(rank * 4, rank * 4 + 4)
        _loss(model, x[shard], y[shard]).backward()
        GradAllReduce(model.parameters())()
        out[rank] = [p.grad.clone() for p in model.parameters()]
    finally:
        dist.destroy_process_group()


def test_grad_allreduce_matches_global_batch():
    world = 2
    port = _free_port()
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(world, port, out), nprocs=world, join=True)
    ref = Tiny()
    x, y = _data(8)
    _loss(ref, x, y).backward()  # mean over the global batch = average of shard means
    for r in range(world):
        for got, want in zip(out[r], [p.grad for p in ref.parameters()]):
            torch.testing.assert_close(got, want, rtol=1e-6, atol=1e-6)


def _failing_worker(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        raise RuntimeError("rank 1 fails before the collective")
    model = Tiny()
    x, y = _data(4)
    _loss(model, x, y).backward()
    GradAllReduce(model.parameters())()  # the peer never joins: must error, not hang


def test_rank_failure_surfaces_as_error():
    port = _free_port()
    with pytest.raises(Exception):
        mp.spawn(_failing_worker, args=(2, port), nprocs=2, join=True)
