"""Data-parallel replicas: the batch sharded by image, weights replicated, and the logits
gathered to one place -- the only exchange of the path (images never interact, so nothing is
exchanged per layer).

Two layers:
  * the C ABI's multi-GPU entry points (no torch): `shard_c` (cuvit_shard), `Comm` (an NCCL
    communicator for one process per GPU, with `gather_logits` to a root rank) and `Replicas`
    (one process driving several GPUs, one host thread per device);
  * torch.distributed helpers for the host side of a multi-process job (CPU affinity, and a
    gloo/NCCL logits gather used by the CPU tests of the sharding logic).
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

from . import _lib
from .errors import check

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


# ---- the C ABI ------------------------------------------------------------------------------

def _ptr(value) -> ctypes.c_void_p:
    if value is None:
        return ctypes.c_void_p(0)
    if hasattr(value, "data_ptr"):
        return ctypes.c_void_p(value.data_ptr())
    if isinstance(value, np.ndarray):
        return ctypes.c_void_p(value.ctypes.data)
    return ctypes.c_void_p(int(value))


def _stream(stream) -> ctypes.c_void_p:
    if stream is None:
        return ctypes.c_void_p(0)
    if hasattr(stream, "cuda_stream"):
        return ctypes.c_void_p(stream.cuda_stream)
    return ctypes.c_void_p(int(stream))


def shard_c(total: int, parts: int, index: int) -> tuple[int, int]:
    """cuvit_shard: (first, count) of part `index` -- the C library's own partition, which
    the multi-GPU entry points use."""
    first, count = ctypes.c_int(0), ctypes.c_int(0)
    check(_lib.library().cuvit_shard(total, parts, index, ctypes.byref(first),
                                     ctypes.byref(count)))
    return first.value, count.value


class Comm:
    """An NCCL communicator through the C ABI (one process per GPU). Rank 0 calls
    `unique_id()` and hands the bytes to every rank by any host channel."""

    ID_BYTES = 128

    @staticmethod
    def unique_id() -> bytes:
        buffer = ctypes.create_string_buffer(Comm.ID_BYTES)
        check(_lib.library().cuvit_comm_unique_id(buffer, Comm.ID_BYTES))
        return buffer.raw

    def __init__(self, unique_id: bytes, world: int, rank: int, device: int):
        if len(unique_id) != Comm.ID_BYTES:
            raise ValueError(f"a unique id has {Comm.ID_BYTES} bytes")
        handle = ctypes.c_void_p(0)
        buffer = ctypes.create_string_buffer(unique_id, Comm.ID_BYTES)
        check(_lib.library().cuvit_comm_create(buffer, world, rank, device,
                                               ctypes.byref(handle)))
        self._handle = handle
        self.world, self.rank, self.device = world, rank, device

    def gather_logits(self, local, gathered, rows: int, classes: int, root: int = 0,
                      stream=None) -> None:
        """cuvit_gather_logits: every rank's [rows, classes] device logits into `gathered`
        (device, root only) in rank order."""
        check(_lib.library().cuvit_gather_logits(self._handle, _ptr(local), _ptr(gathered),
                                                 rows, classes, root, _stream(stream)))

    def close(self) -> None:
        if getattr(self, "_handle", None):
            check(_lib.library().cuvit_comm_destroy(self._handle))
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown
            pass


class Replicas:
    """One process, several GPUs (cuvit_replicas_*): a model per device, one host thread per
    device, shards in cuvit_shard order."""

    def __init__(self, config, weights, max_batch_per_device: int, precision: int,
                 devices: list[int]):
        from .vit import host_tensors

        self.config = config
        arrays = host_tensors(config, weights)
        pointers = (ctypes.c_void_p * len(arrays))(*[a.ctypes.data for a in arrays])
        c_devices = (ctypes.c_int * len(devices))(*devices)
        c_config = config.to_c()
        handle = ctypes.c_void_p(0)
        check(_lib.library().cuvit_replicas_create(ctypes.byref(c_config), pointers,
                                                   len(arrays), max_batch_per_device,
                                                   precision, c_devices, len(devices),
                                                   ctypes.byref(handle)))
        self._handle = handle
        self.devices = list(devices)

    def device_count(self) -> int:
        return _lib.library().cuvit_replicas_device_count(self._handle)

    def forward_host(self, images: np.ndarray) -> np.ndarray:
        """Host images in, host logits [batch, classes] out (synchronous)."""
        images = np.ascontiguousarray(images, dtype=np.float32).reshape(-1)
        per_image = self.config.image_elements()
        if images.size % per_image:
            raise ValueError("image buffer is not a whole number of images")
        batch = images.size // per_image
        logits = np.empty((batch, self.config.classes), np.float32)
        check(_lib.library().cuvit_replicas_forward_host(self._handle, _ptr(images),
                                                         _ptr(logits), batch))
        return logits

    def forward(self, images, images_device: int, logits, logits_device: int,
                batch: int) -> None:
        """Device-resident images and logits (synchronous)."""
        check(_lib.library().cuvit_replicas_forward(self._handle, _ptr(images), images_device,
                                                    _ptr(logits), logits_device, batch))

    def close(self) -> None:
        if getattr(self, "_handle", None):
            check(_lib.library().cuvit_replicas_destroy(self._handle))
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown
            pass
