"""Writes VPK archives in the layout the reference's packer produces
(TVFS.PackDirectory, src/vendor/StdApp/StdApp.VFS.pas:434-560): a 52-byte
header ("VPK0", version 1, entry count, data start, 32 reserved bytes), 544-byte
directory entries (260 UTF-16 path units, offset, size, CRC-32, flags), then
the entries' bytes back to back.  Paths are stored normalised (lower case,
'/'), as PackDirectory does.  Used by the tests to build archives on the fly."""
from __future__ import annotations

import json
import struct
import zlib

import numpy as np


def pack(entries: dict[str, bytes], version: int = 1, magic: bytes = b"VPK0") -> bytes:
    names = list(entries)
    header = 52
    dir_size = 544 * len(names)
    data_start = header + dir_size
    out = bytearray()
    out += struct.pack("<4sIIQ32s", magic, version, len(names), data_start, b"\0" * 32)
    off = data_start
    for n in names:
        path = n.replace("\\", "/").lower().encode("utf-16-le")[: 259 * 2]
        data = entries[n]
        out += path + b"\0" * (520 - len(path))
        out += struct.pack("<QQII", off, len(data), zlib.crc32(data) & 0xFFFFFFFF, 0)
        off += len(data)
    for n in names:
        out += entries[n]
    return bytes(out)


def model_archive(tensors: list[tuple[str, str, np.ndarray, list[int]]], root: str = "E4B") -> bytes:
    """tensors: (name, dtype string, raw bytes as a uint8 array, shape).  Builds
    manifest.json + weights.bin as TWeightStore expects them (16-byte aligned
    offsets, like the reference's packer)."""
    blob = bytearray()
    man = []
    for name, dt, raw, shape in tensors:
        while len(blob) % 16:
            blob += b"\0"
        man.append({"name": name, "source_dtype": "BF16" if dt == "Q4_0" else dt, "output_dtype": dt,
                    "offset": len(blob), "size": int(raw.nbytes), "shape": list(shape)})
        blob += raw.tobytes()
    manifest = json.dumps({"format": "gemma4-test", "tensors": man}).encode()
    return pack({f"{root}/manifest.json": manifest, f"{root}/weights.bin": bytes(blob)})
