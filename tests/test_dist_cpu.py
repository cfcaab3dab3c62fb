"""Multi-rank host logic on CPU: world_size-2 gloo ranks shard the attention
heads and the GEMM columns with no collective in the step, then gather results
for verification, the way bench.py does over NCCL on the GPUs."""
import os
import socket

import numpy as np
import pytest

from beacon_b200.shard import column_shard, even_shard, gqa_shard, head_shard


def test_even_shard_covers_every_unit_once():
    for total in (0, 1, 7, 256, 4096):
        for world in (1, 2, 3, 4, 8):
            seen = []
            for r in range(world):
                s, c = even_shard(total, world, r)
                seen.extend(range(s, s + c))
            assert seen == list(range(total))
    assert head_shard(8, 32, 8, 3) == (96, 32)
    assert column_shard(4096, 8, 7) == (3584, 512)
    assert gqa_shard(1, 64, 8, 8, 5) == (5, 1)
    with pytest.raises(ValueError):
        even_shard(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    import oracle as O
    from beacon_b200.shard import gather_checksums, gather_rows, head_shard

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, H, S, D = 2, 4, 32, 16
        qa = O.normal((B, H, S, D), 2)
        ka = O.normal((B, H, S, D), 2, offset=qa.size)
        va = O.normal((B, H, S, D), 2, offset=2 * qa.size)
        start, count = head_shard(B, H, world, rank)
        sl = lambda a: np.ascontiguousarray(a.reshape(B * H, 1, S, D)[start:start + count].reshape(1, count, S, D))
        o, _ = O.attention_fwd(sl(qa), sl(ka), sl(va))           # this rank's heads only
        full = gather_rows(torch.from_numpy(o.reshape(count, S, D)), world)
        sums = gather_checksums(torch.from_numpy(o), world)
        if rank == 0:
            ref, _ = O.attention_fwd(qa, ka, va)
            q.put((O.rel_err(full.numpy().reshape(B, H, S, D), ref), float(sums[:, 0].sum()),
                   float(ref.astype(np.float64).sum())))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_gather():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    err, gathered_sum, ref_sum = q.get(timeout=5)
    assert err == 0.0
    assert abs(gathered_sum - ref_sum) <= 1e-6 * max(1.0, abs(ref_sum))


def _worker_units(rank, world, port, q):
    import torch
    import torch.distributed as dist

    from beacon_b200.shard import even_shard, gather_units, unit_generator

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        total = 10
        start, count = even_shard(total, world, rank)
        # each rank generates only its units, from (seed, unit): the global tensor is the
        # same whatever the world size
        local = torch.stack([torch.randn(3, 4, generator=unit_generator(7, u, "cpu")) for u in
                             range(start, start + count)])
        wanted = [0, 4, 9]
        got = gather_units(local, start, total, wanted, world)
        if rank == 0:
            ref = torch.stack([torch.randn(3, 4, generator=unit_generator(7, u, "cpu")) for u in wanted])
            q.put(bool(torch.equal(got, ref)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_gather_sampled_units_from_their_owners():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_units, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) is True


def test_bench_cpulist_parsing():
    import importlib.util
    import pathlib
    spec = importlib.util.spec_from_file_location("bench_mod", pathlib.Path(__file__).resolve().parents[1] / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    assert bench.parse_cpulist("0-3,8,10-11") == {0, 1, 2, 3, 8, 10, 11}
    assert bench.parse_cpulist("5\n") == {5}
    assert bench.parse_cpulist("") == set()
    before = os.sched_getaffinity(0)
    assert bench.bind_host_threads(0) is None  # no GPU here: the threads stay where they are
    assert os.sched_getaffinity(0) == before
