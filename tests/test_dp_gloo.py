"""The data-parallel runner's host logic with 2 CPU ranks over gloo: partitioning,
the all-gather back into input order, and a rank that fails mid-step (the other
rank's collective ends with an error after the process group's short timeout
instead of hanging)."""

from __future__ import annotations

import os
import queue
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from latefuse_b200.dp import DataParallelEmbedder, all_gather_rows, packed_cost, partition_rows, partition_tokens

H = 8


class RowEcho:
    """Stands in for an embedder: row i -> [sum of its ids, tenant number, ...]."""

    def embed_tokens(self, ids, mask, tenants, **kw):
        out = torch.zeros(ids.shape[0], H)
        out[:, 0] = (ids * mask).sum(1).float()
        out[:, 1] = torch.tensor([float(t.split("_")[1]) for t in tenants])
        return out


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q, ready):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    # both ranks have started (spawning and importing torch can take seconds on a
    # loaded machine) before the short-timeout rendezvous begins
    ready.wait(timeout=120)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    try:
        g = torch.Generator().manual_seed(0)
        ids = torch.randint(5, 100, (7, 12), generator=g)
        lengths = torch.tensor([12, 3, 7, 12, 1, 9, 5])
        mask = (torch.arange(12).unsqueeze(0) < lengths.unsqueeze(1)).long()
        tenants = [f"t_{i % 3}" for i in range(7)]
        if mode == "ok":
            out = DataParallelEmbedder(RowEcho()).embed_tokens(ids, mask, tenants)
            want = RowEcho().embed_tokens(ids, mask, tenants)
            q.put((rank, bool(torch.equal(out, want))))
        else:
            if rank == 1:
                raise RuntimeError("injected failure before the collective")
            try:
                all_gather_rows(torch.ones(3, H), [3, 3])
                q.put((rank, "no error"))
            except Exception as exc:  # the peer never joins: the collective must fail, not hang
                q.put((rank, type(exc).__name__))
    except RuntimeError as exc:
        q.put((rank, f"raised: {exc}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ready = ctx.Barrier(2)
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q, ready)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(2):  # one result per rank, read before joining
            r, v = q.get(timeout=120)
            results[r] = v
    except queue.Empty:
        pass
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


def test_partition_balances_rows_then_tokens():
    parts = partition_rows([512, 32, 300, 512, 40, 200, 100, 90], 3)
    assert sorted(i for p in parts for i in p) == list(range(8))
    assert sorted(len(p) for p in parts) == [2, 3, 3]
    loads = [sum([512, 32, 300, 512, 40, 200, 100, 90][i] for i in p) for p in parts]
    assert max(loads) - min(loads) <= 512
    assert partition_rows([5], 4) == [[0], [], [], []]


def test_partition_tokens_balances_the_packed_cost():
    """512 rows of lengths U[32, 512] over 8 ranks (the 8-GPU bge-m3 batch): every
    row placed once, each rank's share of the packed cost within 1% of the mean,
    row counts free to differ."""
    g = torch.Generator().manual_seed(0)
    lengths = torch.randint(32, 513, (512,), generator=g).tolist()
    parts = partition_tokens(lengths, 8)
    assert sorted(i for p in parts for i in p) == list(range(512))
    assert all(p == sorted(p) for p in parts)
    loads = [sum(packed_cost(lengths[i]) for i in p) for p in parts]
    mean = sum(loads) / 8
    assert max(loads) / mean < 1.01, loads
    assert partition_tokens([7], 3) == [[0], [], []]
    assert partition_tokens([], 2) == [[], []]


def test_two_rank_gather_restores_input_order():
    assert _run("ok") == {0: True, 1: True}


def test_failed_rank_surfaces_as_an_error_not_a_hang():
    res = _run("fail")
    assert res[1].startswith("raised")
    assert res[0] != "no error" and res[0]  # rank 0's collective ended with an exception
