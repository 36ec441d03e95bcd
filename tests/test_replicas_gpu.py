"""The multi-GPU entry points of the C ABI on GPUs: one process driving several replicas
(cuvit_replicas_*), and the NCCL logits gather of one process per GPU (cuvit_comm_*,
cuvit_gather_logits). Images never interact, so every sharded result must equal one
whole-batch pass of a single model bitwise. With one GPU the replicas share it (two models on
device 0); the two-process NCCL test needs two GPUs and skips otherwise."""

from __future__ import annotations

import multiprocessing
import pathlib
import sys

import numpy as np
import pytest

import make_golden as mg
from cuvit import VisionTransformer
from cuvit.replicas import Comm, Replicas
from cuvit.vit import PRECISION_BF16, random_weights
from helpers import to_device, to_host

pytestmark = pytest.mark.gpu

ROOT = pathlib.Path(__file__).resolve().parents[1]


def small_case():
    _, config, _, std, _, _ = next(c for c in mg.VIT_CASES if c[0] == "vit hd64")
    return config, random_weights(config, 909, std=std)


def whole_batch(config, weights, images, batch, cuda):
    model = VisionTransformer(config, weights, max_batch=batch, precision=PRECISION_BF16)
    logits = cuda.full((batch, config.classes), float("nan"), device="cuda")
    model.forward(to_device(images), logits, batch)
    cuda.cuda.synchronize()
    model.close()
    return to_host(logits)


def test_replicas_on_one_device_match_a_single_model(cuda):
    """Two replicas (both on device 0, each with its own host thread and stream): the host
    and the device-resident forms give the single model's logits, in global image order, for
    batches that split evenly, unevenly and leave a replica idle."""
    config, weights = small_case()
    replicas = Replicas(config, weights, max_batch_per_device=4, precision=PRECISION_BF16,
                        devices=[0, 0])
    assert replicas.device_count() == 2
    for batch in (8, 5, 1):
        images = mg.vit_images(config, batch, 60 + batch)
        want = whole_batch(config, weights, images, batch, cuda)
        np.testing.assert_array_equal(replicas.forward_host(images), want, err_msg=str(batch))
        d_logits = cuda.full((batch, config.classes), float("nan"), device="cuda")
        replicas.forward(to_device(images), 0, d_logits, 0, batch)
        np.testing.assert_array_equal(to_host(d_logits), want, err_msg=f"device {batch}")
    from cuvit.errors import InvalidArgument

    with pytest.raises(InvalidArgument):
        replicas.forward_host(mg.vit_images(config, 9, 1))
    replicas.close()


def test_single_rank_gather_is_a_copy(cuda):
    comm = Comm(Comm.unique_id(), 1, 0, 0)
    local = cuda.arange(12, dtype=cuda.float32, device="cuda").reshape(3, 4)
    gathered = cuda.full((3, 4), float("nan"), device="cuda")
    comm.gather_logits(local, gathered, 3, 4)
    cuda.cuda.synchronize()
    assert cuda.equal(local, gathered)
    comm.close()


def _gather_rank(rank, world, unique, total, results):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "cu-vit_b200"))
    sys.path.insert(0, str(ROOT / "tests"))
    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    try:
        import torch

        import make_golden as mg_child
        from cuvit import VisionTransformer as Model
        from cuvit.replicas import Comm as ChildComm, shard_c
        from cuvit.vit import PRECISION_BF16 as BF16, random_weights as weights_for

        torch.cuda.set_device(rank)
        _, config, _, std, _, _ = next(c for c in mg_child.VIT_CASES if c[0] == "vit hd64")
        weights = weights_for(config, 909, std=std)
        images = mg_child.vit_images(config, total, 77)
        first, count = shard_c(total, world, rank)
        per_image = config.image_elements()
        model = Model(config, weights, max_batch=count, precision=BF16, device=rank)
        mine = torch.from_numpy(images[first * per_image:(first + count) * per_image]).cuda()
        local = torch.zeros(count, config.classes, device="cuda")
        model.forward(mine, local, count)
        comm = ChildComm(unique, world, rank, rank)
        gathered = torch.full((world * count, config.classes), float("nan"), device="cuda")
        comm.gather_logits(local, gathered if rank == 0 else None, count, config.classes, 0)
        torch.cuda.synchronize()
        if rank == 0:
            results[rank] = gathered.cpu().numpy()
        else:
            results[rank] = "ok"
        comm.close()
        model.close()
    except Exception as error:  # reported to the parent
        results[rank] = f"error: {error!r}"


def test_nccl_gather_over_two_gpus(cuda):
    """One process per GPU (spawned), each running its shard through its own model, the
    logits gathered to rank 0 by cuvit_gather_logits: equal to one whole-batch pass."""
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world, total = 2, 6
    context = multiprocessing.get_context("spawn")
    manager = context.Manager()
    results = manager.dict()
    unique = Comm.unique_id()
    processes = [context.Process(target=_gather_rank, args=(r, world, unique, total, results))
                 for r in range(world)]
    for p in processes:
        p.start()
    for p in processes:
        p.join(timeout=240)
    for p in processes:
        if p.is_alive():
            p.kill()
    assert results.get(1) == "ok", results.get(1)
    got = results.get(0)
    assert not isinstance(got, str), got
    config, weights = small_case()
    want = whole_batch(config, weights, mg.vit_images(config, total, 77), total, cuda)
    np.testing.assert_array_equal(got, want)


def test_replicas_over_two_gpus(cuda):
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    config, weights = small_case()
    replicas = Replicas(config, weights, max_batch_per_device=4, precision=PRECISION_BF16,
                        devices=[0, 1])
    images = mg.vit_images(config, 7, 88)
    want = whole_batch(config, weights, images, 7, cuda)
    np.testing.assert_array_equal(replicas.forward_host(images), want)
    d_logits = cuda.full((7, config.classes), float("nan"), device="cuda")
    replicas.forward(to_device(images), 0, d_logits, 0, 7)
    np.testing.assert_array_equal(to_host(d_logits), want)
    replicas.close()
