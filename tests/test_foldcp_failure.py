"""Failure detection of the Fold-CP ranks, on the host (gloo CPU ranks, no GPU involved).

A rank that fails must not leave the others waiting for ever: with the short process-group
timeout the launch API passes through (``FoldCPConfig`` users create the default group; here
``timeout=5 s``), the surviving ranks' next collective of the band exchange ends with an error
within a bounded time, and every process exits. Two failures are made on the host:

* a rank that leaves between two trunk steps (its process exits before the second step);
* a rank that never joins (it never creates the process group).

The reference has no failure detection beyond its NCCL init timeout
(opendde runner/inference.py:55,197-199); these tests pin the bound for this build's path.
"""
import os
import queue
import socket
import time

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

C_Z, C_S, HEADS, N = 16, 32, 4, 10
PG_TIMEOUT_S = 5
BOUND_S = 60  # every surviving rank must have failed (not hung) within this


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, scenario, results):
    import sys
    from datetime import timedelta
    sys.path.insert(0, os.path.dirname(__file__))
    sys.path.insert(0, os.path.dirname(os.path.dirname(__file__)))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    t0 = time.time()
    if scenario == "never_joins" and rank == world - 1:
        results.put((rank, "left", 0.0))
        return
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=PG_TIMEOUT_S))
        from foldcp_support import OracleBandOps
        from opendde_b200.distributed.foldcp import (FoldCPConfig, FoldCPProcessMesh,
                                                      distributed_pairformer_stack_single_bridge_update)
        from opendde_b200.model import PairformerStack
        from opendde_b200.utils import make_inputs, seeded_init_

        mesh = FoldCPProcessMesh.create(FoldCPConfig.from_runtime_args(mode="distributed", size_cp=world,
                                                                        mesh=f"1x{world}"))
        st = PairformerStack(n_blocks=1, n_heads=HEADS, c_z=C_Z, c_s=C_S)
        seeded_init_(st, seed=0)
        s, z, mask = make_inputs(N, c_z=C_Z, c_s=C_S, seed=1)
        with torch.no_grad():
            for step in range(2):
                if scenario == "leaves" and rank == world - 1 and step == 1:
                    results.put((rank, "left", time.time() - t0))
                    results.close()
                    results.join_thread()   # the message is out before the process dies
                    os._exit(3)  # the process dies between two steps, without any cleanup
                s, z = distributed_pairformer_stack_single_bridge_update(st, s, z, mesh, pair_mask=mask,
                                                                         ops=OracleBandOps())
        results.put((rank, "done", time.time() - t0))
    except Exception as e:  # noqa: BLE001 - the failure under test
        results.put((rank, f"error: {type(e).__name__}", time.time() - t0))


def _run(scenario, world):
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, scenario, results)) for r in range(world)]
    t0 = time.time()
    for p in procs:
        p.start()
    out = {}
    while len(out) < world and time.time() - t0 < BOUND_S + 30:
        try:
            rank, what, dt = results.get(timeout=1.0)
            out[rank] = (what, dt)
        except queue.Empty:
            pass
    for p in procs:
        p.join(timeout=max(1.0, BOUND_S + 30 - (time.time() - t0)))
    alive = [p.pid for p in procs if p.is_alive()]
    for p in procs:
        if p.is_alive():
            p.kill()
    return out, alive


def test_rank_leaving_between_steps_fails_the_others_within_the_timeout():
    world = 3
    out, alive = _run("leaves", world)
    assert not alive, f"processes still waiting: {alive}"
    assert out.get(world - 1, ("?",))[0] == "left", out
    for r in range(world - 1):
        what, dt = out[r]
        assert what.startswith("error"), f"rank {r}: {what}"
        assert dt < BOUND_S, f"rank {r} took {dt:.1f} s to fail"


def test_rank_that_never_joins_fails_the_others_within_the_timeout():
    world = 2
    out, alive = _run("never_joins", world)
    assert not alive, f"processes still waiting: {alive}"
    what, dt = out[0]
    assert what.startswith("error"), what
    assert dt < BOUND_S, f"rank 0 took {dt:.1f} s to fail"
