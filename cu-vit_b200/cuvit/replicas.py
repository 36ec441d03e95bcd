"""Data-parallel replicas: one process per GPU, the batch sharded by image, weights
replicated, and the logits gathered to rank 0 -- the only collective of the path (images never
interact, so nothing is exchanged per layer).

The helpers work on any torch.distributed backend (NCCL on GPUs, gloo on CPU for tests).
"""

from __future__ import annotations

import os

SYSFS_PCI_DEVICES = "/sys/bus/pci/devices"


def parse_cpulist(text: str) -> list[int]:
    """CPUs of a Linux cpulist string ("0-7,16-23", "3", "")."""
    cpus: list[int] = []
    for part in text.strip().split(","):
        if not part:
            continue
        first, _, last = part.partition("-")
        cpus.extend(range(int(first), int(last or first) + 1))
    return cpus


def device_local_cpus(domain: int, bus: int, device: int,
                      root: str = SYSFS_PCI_DEVICES) -> list[int] | None:
    """The CPUs Linux lists as local to a PCI device (its NUMA node's cores), or None where
    sysfs has no such entry."""
    path = os.path.join(root, f"{domain:04x}:{bus:02x}:{device:02x}.0", "local_cpulist")
    try:
        with open(path) as handle:
            return parse_cpulist(handle.read())
    except (OSError, ValueError):
        return None


def cpu_share(gpu: int, local: dict[int, list[int]], allowed: set[int]) -> list[int]:
    """This GPU's CPUs: those local to it (and allowed), split evenly in device order among
    the GPUs with the same local CPUs, so one process per GPU gets a disjoint share."""
    mine = sorted(set(local[gpu]) & allowed)
    peers = [g for g in sorted(local) if local[g] == local[gpu]]
    if len(peers) > 1 and mine:
        index = peers.index(gpu)
        share = mine[index * len(mine) // len(peers):(index + 1) * len(mine) // len(peers)]
        if share:
            return share
    return mine


def bind_to_gpu_cpus(gpu: int, root: str = SYSFS_PCI_DEVICES) -> list[int] | None:
    """Restricts the calling process to its share of the CPUs local to CUDA device `gpu`
    (cpu_share, within the CPUs it may already use), so host memory it allocates afterwards
    -- pinned staging buffers above all -- sits on the GPU's NUMA node, and host threads of
    the processes of GPUs on one node (the BF16 model's image rounding) do not contend for
    the same cores. Returns the CPUs bound, or None (nothing changed) where the topology is
    unknown or shares no CPU with the current affinity."""
    import torch

    local: dict[int, list[int]] = {}
    for device in range(torch.cuda.device_count()):
        props = torch.cuda.get_device_properties(device)
        cpus = device_local_cpus(props.pci_domain_id, props.pci_bus_id, props.pci_device_id,
                                 root)
        if cpus:
            local[device] = cpus
    if gpu not in local:
        return None
    share = cpu_share(gpu, local, os.sched_getaffinity(0))
    if not share:
        return None
    os.sched_setaffinity(0, share)
    return share


def shard(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous slice [start, start + count) of `total` images owned by `rank`; the first
    total % world ranks take one extra image. Global image b lives on the rank whose slice
    contains b, so gathering in rank order restores the global order."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if total < 0:
        raise ValueError("total cannot be negative")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def gather_logits(local, world: int, rank: int, counts: list[int] | None = None):
    """Gathers every rank's [count, classes] logits to rank 0 in rank order.

    counts: per-rank row counts (defaults to equal shards). Returns the concatenated tensor
    on rank 0 and None elsewhere. Every rank must call it, in the same order as its other
    collectives.
    """
    import torch
    import torch.distributed as dist

    if world == 1:
        return local
    counts = counts or [local.shape[0]] * world
    rows = max(counts)
    padded = local
    if local.shape[0] < rows:  # gather needs equal shapes
        padded = torch.zeros((rows,) + tuple(local.shape[1:]), dtype=local.dtype,
                             device=local.device)
        padded[: local.shape[0]] = local
    buffers = [torch.empty_like(padded) for _ in range(world)] if rank == 0 else None
    dist.gather(padded, buffers, dst=0)
    if rank != 0:
        return None
    return torch.cat([buffers[r][: counts[r]] for r in range(world)])
