"""Multi-rank host logic on the CPU with gloo (world size 2 and 3): batch sharding, the
logits gather in global image order, and a rank that fails before the collective.

The per-rank "forward pass" is the CPU oracle on a tiny ViT, so the gathered logits can be
checked against one whole-batch oracle run; on GPUs the same helpers run over NCCL with the
CUDA library computing each shard (bench.py).
"""

from __future__ import annotations

import datetime
import os
import pathlib
import socket
import sys
import traceback

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = pathlib.Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, total, mode, results):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "cu-vit_b200"))
    try:
        import torch
        import torch.distributed as dist

        import oracle
        from cuvit.replicas import gather_logits, shard
        from cuvit.vit import VitConfig, random_weights, tensor_specs

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=20))
        config = VitConfig(16, 4, 3, 16, 2, 2, 32, 5)
        weights = random_weights(config, 9, std=0.3)
        images = np.random.default_rng(4).standard_normal(
            total * config.image_elements()).astype(np.float32)
        start, count = shard(total, world, rank)
        per_image = config.image_elements()
        mine = images[start * per_image:(start + count) * per_image]
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 failed before the gather")
        logits = torch.from_numpy(
            oracle.vit_forward(config, weights, tensor_specs(config), mine, threads=1))
        counts = [shard(total, world, r)[1] for r in range(world)]
        gathered = gather_logits(logits, world, rank, counts)
        if rank == 0:
            want = oracle.vit_forward(config, weights, tensor_specs(config), images, threads=2)
            results[rank] = ("ok", bool(np.array_equal(gathered.numpy(), want)))
        else:
            results[rank] = ("ok", gathered is None)
        dist.destroy_process_group()
    except Exception as error:  # reported to the parent, which decides pass/fail
        results[rank] = ("error", f"{type(error).__name__}: {error}\n{traceback.format_exc()}")


def _run(world, total, mode):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, world, port, total, mode, results))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
        return dict(results)


def test_shard_covers_the_batch_in_order():
    from cuvit.replicas import shard

    for total in (0, 1, 7, 256, 1024, 1027):
        for world in (1, 2, 3, 8):
            spans = [shard(total, world, r) for r in range(world)]
            assert spans[0][0] == 0
            for (s0, c0), (s1, _) in zip(spans, spans[1:]):
                assert s0 + c0 == s1
            assert sum(c for _, c in spans) == total
            assert max(c for _, c in spans) - min(c for _, c in spans) <= 1
    with pytest.raises(ValueError):
        shard(8, 2, 2)


def test_c_library_shards_like_the_host_helper():
    """cuvit_shard -- the partition the C ABI's multi-GPU entry points use (replicas and the
    NCCL gather's rank order) -- equals the Python helper, and concatenating the parts in
    index order restores the global image order; bad partitions are rejected."""
    from cuvit.errors import InvalidArgument
    from cuvit.replicas import shard, shard_c

    for total in (0, 1, 5, 7, 256, 1024, 1025):
        for parts in (1, 2, 3, 4, 8):
            order = []
            for index in range(parts):
                first, count = shard_c(total, parts, index)
                assert (first, count) == shard(total, parts, index)
                order.extend(range(first, first + count))
            assert order == list(range(total))
    for bad in ((5, 0, 0), (5, 2, 2), (5, 2, -1), (-1, 2, 0)):
        with pytest.raises(InvalidArgument):
            shard_c(*bad)


def test_cpu_lists_and_device_locality_from_sysfs(tmp_path):
    """Each rank binds to its GPU's NUMA-local CPUs (bench.py, N > 1); the topology comes from
    the PCI device's local_cpulist in sysfs, here a fake tree."""
    from cuvit.replicas import device_local_cpus, parse_cpulist

    assert parse_cpulist("0-3,8,10-11\n") == [0, 1, 2, 3, 8, 10, 11]
    assert parse_cpulist("") == []
    entry = tmp_path / "0000:1b:00.0"
    entry.mkdir()
    (entry / "local_cpulist").write_text("56-111,168-223\n")
    cpus = device_local_cpus(0, 0x1B, 0, root=str(tmp_path))
    assert cpus[0] == 56 and cpus[-1] == 223 and len(cpus) == 112
    assert device_local_cpus(0, 0x2C, 0, root=str(tmp_path)) is None


def test_gpus_on_one_node_take_disjoint_cpu_shares():
    from cuvit.replicas import cpu_share

    node0, node1 = list(range(0, 16)), list(range(16, 32))
    local = {g: (node0 if g < 4 else node1) for g in range(8)}
    shares = [cpu_share(g, local, set(range(32))) for g in range(8)]
    assert shares[0] == [0, 1, 2, 3] and shares[3] == [12, 13, 14, 15]
    assert shares[4] == [16, 17, 18, 19] and shares[7] == [28, 29, 30, 31]
    assert len({c for share in shares for c in share}) == 32
    # fewer allowed CPUs than GPUs: every GPU keeps at least the allowed local ones
    assert cpu_share(1, local, {0, 1}) in ([0], [1], [0, 1])
    # one GPU per node keeps the node
    assert cpu_share(0, {0: node0, 1: node1}, set(range(32))) == node0


@pytest.mark.parametrize("world,total", [(2, 6), (3, 7)])
def test_gathered_logits_equal_one_whole_batch(world, total):
    results = _run(world, total, "ok")
    assert len(results) == world, results
    for rank, (status, value) in sorted(results.items()):
        assert status == "ok", value
        assert value is True, f"rank {rank}"


def test_a_failed_rank_surfaces_as_an_error_not_a_hang():
    results = _run(2, 4, "fail")
    assert results.get(1, ("", ""))[0] == "error"
    # rank 0 either errors out of the gather (peer gone / timeout) -- it must not report ok
    status, _ = results.get(0, ("missing", ""))
    assert status in ("error", "missing")
