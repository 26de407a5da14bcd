"""Data-parallel path on CPU: two gloo ranks split the sequences round-robin,
decode their share with the oracle (tiny model) and reduce the statistics the
way bench.py does; the union of their outputs equals a single-process run.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ssd.engine import dp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_models():
    from oracle.model import OracleModel, weights_from_hf
    from ssd import synthetic as S

    base = S.build_base_model("tiny", 0, torch.float32, "cpu")
    w, conf = weights_from_hf(base, np.float64)
    target = OracleModel(w, conf, list(range(conf["layers"])))
    return target


def _prompts():
    from ssd import synthetic as S

    return [S.make_prompt(10 + i, 6 + i, 128)[0].tolist() for i in range(5)]


def _decode(target, prompts):
    from oracle.engine import speculative_generate

    return [speculative_generate(target, target, dict(depth=3, branch=[2, 2, 1]), p, 6)["tokens"] for p in prompts]


def _worker(rank: int, world: int, port: int, q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        prompts = _prompts()
        mine = dp.shard(list(range(len(prompts))), rank, world)
        target = _oracle_models()
        outs = _decode(target, [prompts[i] for i in mine])
        n_tok = sum(len(o) for o in outs)
        total = dp.all_sum(n_tok, world)
        slowest = dp.all_max(float(rank + 1), world)
        dp.barrier(world)
        gathered = dp.gather_lists(list(zip(mine, outs)), world)
        q.put((rank, total, slowest, gathered))
    finally:
        dist.destroy_process_group()


def test_shard_round_robin():
    items = list(range(8))
    assert dp.shard(items, 0, 1) == items
    parts = [dp.shard(items, r, 4) for r in range(4)]
    assert parts[1] == [1, 5] and sorted(sum(parts, [])) == items
    with pytest.raises(ValueError):
        dp.shard(items, 2, 2)
    assert dp.all_max(3.0, 1) == 3.0 and dp.all_sum(2.0, 1) == 2.0


def test_two_gloo_ranks_match_single_process():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = _decode(_oracle_models(), _prompts())
    for rank, total, slowest, gathered in results:
        assert total == sum(len(o) for o in ref)
        assert slowest == float(world)
        merged = {i: o for part in gathered for i, o in part}
        assert [merged[i] for i in range(len(ref))] == ref


def _leaving_worker(rank: int, world: int, port: int, q) -> None:
    """Step 1 on both ranks; then rank 1 leaves between steps (exits without
    joining the next collective) and rank 0's next reduction must fail on the
    host within the short process-group timeout instead of waiting for good."""
    import time
    from datetime import timedelta

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    first = dp.all_sum(1.0, world)
    if rank == 1:
        q.put((rank, first, None, 0.0))
        q.close()
        q.join_thread()  # flush the queue before leaving without any clean-up
        os._exit(0)
    t0 = time.time()
    try:
        dp.all_sum(1.0, world)
        err = None
    except Exception as exc:  # gloo reports the departed peer or the timeout
        err = type(exc).__name__
    q.put((rank, first, err, time.time() - t0))
    q.close()
    q.join_thread()
    os._exit(0)


def test_departed_rank_surfaces_as_an_error_on_the_next_collective():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        rank, first, err, dt = q.get(timeout=120)
        got[rank] = (first, err, dt)
    for p in procs:
        p.join(timeout=60)
    assert got[0][0] == got[1][0] == 2.0
    assert got[0][1] is not None, "rank 0's collective returned although its peer had left"
    assert got[0][2] < 60.0
