"""Multi-rank host logic on CPU: world_size-2 gloo process groups.

The GPU kernel is replaced by the CPU oracle here (the host logic under test
is the row split, the per-shard column-major scale slabs, the gather used for
checking, the max-over-ranks timing reduction and failure propagation).
"""

import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import reference as ora
from thingy_b200.shard import init_from_env, max_over_ranks, shard_rows
from thingy_b200.workloads import WORKLOADS, make_inputs


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _env(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))


def _sharded_worker(rank, world, port, M, out_q):
    _env(rank, world, port)
    init_from_env("gloo", timeout_s=60)
    w = WORKLOADS["g128_sharded_262144x8192"]
    full = make_inputs(w, M, device="cpu", seed=0)  # every rank sees the same global batch
    sh = shard_rows(M, world, rank)
    x = full["x"][sh.start:sh.stop]
    q, s, _, _ = ora.rms_norm_fp8(x, full["weight"], w.eps, group_size=128)
    slab = s.t().contiguous()  # this rank's [G, M_r] column-major slab
    rows = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(rows, torch.tensor([sh.rows]))
    rows = [int(r) for r in rows]
    mr = max(rows)  # gloo gathers equal sizes: pad to the largest shard, trim after
    qs = [torch.zeros(mr, x.shape[1], dtype=torch.uint8) for _ in rows]
    ss = [torch.zeros(slab.shape[0], mr) for _ in rows]
    dist.all_gather(qs, torch.nn.functional.pad(q, (0, 0, 0, mr - sh.rows)))
    dist.all_gather(ss, torch.nn.functional.pad(slab, (0, mr - sh.rows)))
    t = max_over_ranks(1.0 + rank)
    if rank == 0:
        q_all = torch.cat([a[:r] for a, r in zip(qs, rows)], 0)
        s_all = torch.cat([a[:, :r] for a, r in zip(ss, rows)], 1)
        q_ref, s_ref, _, _ = ora.rms_norm_fp8(full["x"], full["weight"], w.eps, group_size=128)
        out_q.put((torch.equal(q_all, q_ref), torch.equal(s_all, s_ref.t().contiguous()), t))
    dist.destroy_process_group()


def test_row_sharded_scales_follow_their_rows():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_worker, args=(r, 2, port, 37, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    q_ok, s_ok, t = q.get(timeout=5)
    assert q_ok and s_ok
    assert t == 2.0  # max over ranks of (1 + rank)


def _failing_worker(rank, world, port, out_q):
    _env(rank, world, port)
    init_from_env("gloo", timeout_s=5)
    if rank == 1:
        raise SystemExit(3)  # this rank dies before the collective
    t0 = time.monotonic()
    try:
        max_over_ranks(1.0)
        out_q.put(("no error", time.monotonic() - t0))
    except Exception as e:  # the survivor must get an error, not hang
        out_q.put((type(e).__name__, time.monotonic() - t0))


def test_dead_rank_surfaces_as_an_error_not_a_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    assert procs[1].exitcode == 3
    kind, waited = q.get(timeout=5)
    assert kind != "no error"
    assert waited < 60
