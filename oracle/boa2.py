"""BOA2 container restatement (TEST INFRASTRUCTURE: the checker for the
library's C++ container code).

Layout, as written by compress_v2 (portability_solved_cpp/boa.cpp:538-581)
and read by read_boa2 (boa.cpp:190-277):

    "BOA2" | u32 version=1 | u32 flags (bit0 warm start) | u64 total_size |
    u32 chunk_len | u32 n_chunks | u32 last_chunk_len | u8 fp_len | fp bytes |
    payload (each chunk's 32-bit LE words, chunk order) |
    "IDX2" | first_bytes[n] | uvarint(stream_bytes)[n] | u32 CRC-32
The Python BoaFile writer (boa.py:107-131, :226-311) writes the same layout
with flags 0 and a 16-byte fingerprint, blake2s(model class name).
The CRC-32 (reflected, polynomial 0xEDB88320, boa.cpp:85-107) covers
"IDX2"...end of the lengths.  The reader also accepts "IDX1" (uvarint
delta-offsets then lengths, boa.cpp:240-250).
"""
from __future__ import annotations

import struct
import zlib


def uvarint(x: int) -> bytes:  # boa.cpp:158-165
    out = bytearray()
    while True:
        b = x & 0x7F
        x >>= 7
        out.append(b | (0x80 if x else 0))
        if not x:
            return bytes(out)


def read_uvarint(buf: bytes, pos: int):  # boa.cpp:167-176
    x = shift = 0
    while True:
        b = buf[pos]
        pos += 1
        x |= (b & 0x7F) << shift
        if not b & 0x80:
            return x, pos
        shift += 7


def build(total_size, chunk_len, first_bytes, streams, warm_start=False, interleave_batch=0,
          fingerprint=None) -> bytes:
    n = len(streams)
    last = total_size - (n - 1) * chunk_len if n > 1 else total_size
    flags = 1 if warm_start else 0
    head = b"BOA2" + struct.pack("<IIQIII", 1, flags, total_size, chunk_len, n, last)
    if fingerprint is not None:  # boa.py:120-121
        head += bytes([len(fingerprint)]) + bytes(fingerprint)
    else:
        head += bytes([4]) + struct.pack("<I", interleave_batch) if warm_start else bytes([0])
    payload = b"".join(bytes(s) for s in streams)
    idx = b"IDX2" + bytes(first_bytes) + b"".join(uvarint(len(bytes(s))) for s in streams)
    return head + payload + idx + struct.pack("<I", zlib.crc32(idx) & 0xFFFFFFFF)


def parse(buf: bytes) -> dict:
    if len(buf) < 32:
        raise ValueError("Invalid BOA2 file")
    if buf[:4] != b"BOA2":
        raise ValueError("Bad BOA2 magic")
    version, flags, total, chunk_len, n, last = struct.unpack_from("<IIQIII", buf, 4)
    if version != 1:
        raise ValueError("Unsupported BOA2 version")
    p = 32
    fp_len = buf[p]
    p += 1
    interleave = struct.unpack_from("<I", buf, p)[0] if (flags & 1) and fp_len >= 4 else 0
    p += fp_len
    payload_start = p
    idx_pos, ver = -1, 0
    for i in range(len(buf) - 5, -1, -1):  # backward scan as boa.cpp:220-225
        if buf[i:i + 3] == b"IDX" and buf[i + 3] in (ord("1"), ord("2")):
            idx_pos, ver = i, buf[i + 3] - ord("0")
            break
    if idx_pos < 0:
        raise ValueError("IDX not found")
    crc = struct.unpack_from("<I", buf, len(buf) - 4)[0]
    if crc != (zlib.crc32(buf[idx_pos:len(buf) - 4]) & 0xFFFFFFFF):
        raise ValueError("Bad BOA2 CRC")
    q = idx_pos + 4
    first = list(buf[q:q + n])
    q += n
    offsets, lengths = [], []
    if ver == 1:
        prev = 0
        for _ in range(n):
            dlt, q = read_uvarint(buf, q)
            prev += dlt
            offsets.append(prev)
        for _ in range(n):
            ln, q = read_uvarint(buf, q)
            lengths.append(ln)
    else:
        off = 0
        for _ in range(n):
            ln, q = read_uvarint(buf, q)
            lengths.append(ln)
            offsets.append(off)
            off += ln
    payload = buf[payload_start:idx_pos]
    streams = []
    for o, ln in zip(offsets, lengths):
        if o + ln > len(payload):
            raise ValueError("BOA2 payload out of range")
        streams.append(payload[o:o + ln])
    return dict(total_size=total, chunk_len=chunk_len, n_chunks=n, last_chunk_len=last, flags=flags,
                interleave_batch=interleave, first_bytes=first, streams=streams, index_version=ver)
