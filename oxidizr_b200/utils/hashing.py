"""Bit-compatible re-implementation of the hashes the upstream resume check uses.

Upstream hashes with Rust's ``std::collections::hash_map::DefaultHasher::new()``,
which is SipHash-1-3 with both keys zero (``config.rs:495-518``).  The bytes
fed to the hasher follow Rust's ``Hash`` impls:

* ``String``/``str``: the UTF-8 bytes followed by one ``0xff`` byte;
* ``Vec<u8>``: the length as a native-endian ``usize`` (8 bytes, little endian
  on x86-64) followed by the bytes;
* ``u64``: 8 little-endian bytes.

SipHash itself is the published algorithm of Aumasson & Bernstein (2012); the
round counts are parameters so the implementation can be checked against the
paper's SipHash-2-4 test vector.
"""
from __future__ import annotations

import os
import struct

_MASK = 0xFFFFFFFFFFFFFFFF


def _rotl(x: int, b: int) -> int:
    return ((x << b) | (x >> (64 - b))) & _MASK


def siphash(data: bytes, k0: int = 0, k1: int = 0, c_rounds: int = 1, d_rounds: int = 3) -> int:
    v0 = k0 ^ 0x736F6D6570736575
    v1 = k1 ^ 0x646F72616E646F6D
    v2 = k0 ^ 0x6C7967656E657261
    v3 = k1 ^ 0x7465646279746573

    def sipround():
        nonlocal v0, v1, v2, v3
        v0 = (v0 + v1) & _MASK
        v1 = _rotl(v1, 13)
        v1 ^= v0
        v0 = _rotl(v0, 32)
        v2 = (v2 + v3) & _MASK
        v3 = _rotl(v3, 16)
        v3 ^= v2
        v0 = (v0 + v3) & _MASK
        v3 = _rotl(v3, 21)
        v3 ^= v0
        v2 = (v2 + v1) & _MASK
        v1 = _rotl(v1, 17)
        v1 ^= v2
        v2 = _rotl(v2, 32)

    n = len(data)
    full = n - (n % 8)
    for off in range(0, full, 8):
        m = struct.unpack_from("<Q", data, off)[0]
        v3 ^= m
        for _ in range(c_rounds):
            sipround()
        v0 ^= m
    tail = data[full:] + b"\x00" * (7 - (n % 8))
    b = ((n & 0xFF) << 56) | int.from_bytes(tail, "little")
    v3 ^= b
    for _ in range(c_rounds):
        sipround()
    v0 ^= b
    v2 ^= 0xFF
    for _ in range(d_rounds):
        sipround()
    return (v0 ^ v1 ^ v2 ^ v3) & _MASK


def rust_default_hash_str(s: str) -> int:
    return siphash(s.encode("utf-8") + b"\xff")


def compute_model_config_hash(model_cfg) -> str:
    """``compute_model_config_hash`` (config.rs:495-501)."""
    from ..config import model_config_json
    return f"{rust_default_hash_str(model_config_json(model_cfg)):016x}"


def compute_file_hash(path: str) -> str:
    """``compute_file_hash`` (config.rs:504-518): first MiB + file size."""
    size = os.path.getsize(path)
    with open(path, "rb") as fh:
        buf = fh.read(min(1024 * 1024, size))
    data = struct.pack("<Q", len(buf)) + buf + struct.pack("<Q", size)
    return f"{siphash(data):016x}"
