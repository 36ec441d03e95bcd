"""Reader and writer of Cu-Vit's .cvw v1 weight files.

Layout (little-endian, as documented at src/runtime/weights.cpp:13-24 of the reference):
  magic u32 "CVIT", version u32 = 1, entry_count u32, reserved u32
  entry_count x { name_length u32, name, type u32 (1 = float32), rank u32,
                  extents i64[rank], offset u64, bytes u64 }
  payloads, each starting on a 64-byte boundary; offsets are absolute.
The format has to match byte for byte so that files written here load in the reference and
the other way round; the code is this package's own.
"""

from __future__ import annotations

import pathlib
import struct

import numpy as np

MAGIC = 0x54495643
VERSION = 1
FLOAT32 = 1
ALIGNMENT = 64
MAX_RANK = 4


def _align(value: int) -> int:
    return (value + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT


class WeightFileWriter:
    """reference: WeightFileWriter (include/cuvit/weights.hpp:78-92)."""

    def __init__(self) -> None:
        self._entries: list[tuple[str, tuple[int, ...], np.ndarray]] = []

    def add(self, name: str, extents, data) -> None:
        if not name:
            raise ValueError("A weight tensor needs a name")
        extents = tuple(int(e) for e in extents)
        if not extents or len(extents) > MAX_RANK:
            raise ValueError(f"Tensor '{name}' has an unsupported rank")
        if any(e < 0 for e in extents):
            raise ValueError(f"Tensor '{name}' has a negative extent")
        if any(existing == name for existing, _, _ in self._entries):
            raise ValueError(f"Tensor '{name}' was added twice")
        array = np.ascontiguousarray(np.asarray(data, dtype=np.float32)).reshape(-1)
        if array.size != int(np.prod(extents)):
            raise ValueError(f"Tensor '{name}' data does not match its extents")
        self._entries.append((name, extents, array))

    def __len__(self) -> int:
        return len(self._entries)

    def write(self, path) -> None:
        table = 16
        for name, extents, _ in self._entries:
            table += 4 + len(name.encode()) + 8 + 8 * len(extents) + 16
        offsets = []
        cursor = _align(table)
        for _, _, array in self._entries:
            offsets.append(cursor)
            cursor = _align(cursor + array.nbytes)
        out = bytearray(struct.pack("<IIII", MAGIC, VERSION, len(self._entries), 0))
        for (name, extents, array), offset in zip(self._entries, offsets):
            encoded = name.encode()
            out += struct.pack("<I", len(encoded)) + encoded
            out += struct.pack("<II", FLOAT32, len(extents))
            out += struct.pack(f"<{len(extents)}q", *extents)
            out += struct.pack("<QQ", offset, array.nbytes)
        for (_, _, array), offset in zip(self._entries, offsets):
            out += b"\0" * (offset - len(out))
            out += array.astype("<f4").tobytes()
        pathlib.Path(path).write_bytes(bytes(out))


class WeightFile:
    """reference: WeightFile (include/cuvit/weights.hpp:45-74), read into host memory."""

    def __init__(self, entries: dict[str, tuple[tuple[int, ...], np.ndarray]]):
        self._entries = entries

    @classmethod
    def load(cls, path) -> "WeightFile":
        blob = pathlib.Path(path).read_bytes()
        if len(blob) < 16:
            raise RuntimeError("Weight file ends inside a header field")
        magic, version, count, _ = struct.unpack_from("<IIII", blob, 0)
        if magic != MAGIC:
            raise RuntimeError(f"Not a Cu-Vit weight file: {path}")
        if version != VERSION:
            raise RuntimeError(f"Weight file {path} has version {version}, but this build "
                               f"reads version {VERSION}")
        cursor = 16
        entries: dict[str, tuple[tuple[int, ...], np.ndarray]] = {}
        for _ in range(count):
            (length,) = struct.unpack_from("<I", blob, cursor)
            cursor += 4
            name = blob[cursor:cursor + length].decode()
            cursor += length
            dtype, rank = struct.unpack_from("<II", blob, cursor)
            cursor += 8
            if dtype != FLOAT32:
                raise RuntimeError(f"Tensor '{name}' has unsupported data type {dtype}")
            if rank == 0 or rank > MAX_RANK:
                raise RuntimeError(f"Tensor '{name}' has rank {rank}, outside 1..{MAX_RANK}")
            extents = struct.unpack_from(f"<{rank}q", blob, cursor)
            cursor += 8 * rank
            offset, nbytes = struct.unpack_from("<QQ", blob, cursor)
            cursor += 16
            if nbytes != int(np.prod(extents)) * 4:
                raise RuntimeError(f"Tensor '{name}' declares {nbytes} bytes but its shape "
                                   f"{list(extents)} needs {int(np.prod(extents)) * 4}")
            if offset + nbytes > len(blob):
                raise RuntimeError(f"Tensor '{name}' lies outside the file")
            if name in entries:
                raise RuntimeError(f"Weight file contains two tensors named '{name}'")
            data = np.frombuffer(blob, dtype="<f4", count=nbytes // 4, offset=offset)
            entries[name] = (tuple(extents), data.astype(np.float32))
        return cls(entries)

    def __len__(self) -> int:
        return len(self._entries)

    def __contains__(self, name: str) -> bool:
        return name in self._entries

    def names(self) -> list[str]:
        return list(self._entries)

    def float_data(self, name: str, extents) -> np.ndarray:
        if name not in self._entries:
            raise RuntimeError(f"Weight file has no tensor named '{name}'")
        found, data = self._entries[name]
        if tuple(found) != tuple(extents):
            raise RuntimeError(f"Tensor '{name}' has shape {list(found)}, but {list(extents)} "
                               "was expected")
        return data
