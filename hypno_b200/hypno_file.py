"""The `.hypno` container (crates/hypno/src/format.rs, loader.rs) in Python:
an image writer laid out like the reference converter (sft_convert.rs:139-285)
and a manifest reader used by tests.

Layout: 16-byte header (b"HYPN", version 1 u32, metadata count u32, tensor
count u32), metadata entries (u32 key length, key, u32 value length, value),
the tensor table (u32 name length, name, u32 ndim, ndim x u64 shape, u32
dtype, u64 offset, u64 length), zero padding to a 64-byte boundary, then
each payload at a 64-byte-aligned offset.  Tensors are written in byte-wise
name order (the converter's BTreeMap).  The format has to be the same as the
reference's so an image written here loads in the reference and vice versa.
"""
import struct

import numpy as np

MAGIC = b"HYPN"
VERSION = 1
ALIGNMENT = 64

DT_FP32, DT_FP16, DT_Q8_0, DT_Q4_0 = 0, 1, 2, 3


def data_bytes(dtype, n_elems):
    """DType::data_bytes (dtype.rs:57-70)."""
    if dtype == DT_FP32:
        return n_elems * 4
    if dtype == DT_FP16:
        return n_elems * 2
    blocks = -(-n_elems // 32)
    return blocks * (34 if dtype == DT_Q8_0 else 18)


def effective_dtype(target, n_elems):
    """sft_convert::effective_dtype (sft_convert.rs:11-17): tensors of at most
    4096 elements stay FP32 when quantizing."""
    if n_elems <= 4096 and target not in (DT_FP32, DT_FP16):
        return DT_FP32
    return target


def rust_f64_display(x):
    """Formats a float the way Rust's `f64::to_string` does (shortest
    round-trip digits, no exponent), as the converter writes rms_norm_eps and
    rope_theta (sft_convert.rs:96-97)."""
    s = np.format_float_positional(float(x), trim="-", unique=True)
    return s


def _align(x):
    return (x + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT


def layout(metadata, entries):
    """Header bytes, payload offsets and total size of an image.

    entries: list of (name, shape tuple, dtype code, payload length).
    Returns (header bytes, {name: offset}, total size, sorted entries)."""
    entries = sorted(entries, key=lambda t: t[0].encode())
    head = bytearray(MAGIC + struct.pack("<III", VERSION, len(metadata), len(entries)))
    for k, v in metadata:
        kb, vb = k.encode(), v.encode()
        head += struct.pack("<I", len(kb)) + kb + struct.pack("<I", len(vb)) + vb
    table_size = sum(4 + len(n.encode()) + 4 + 8 * len(s) + 4 + 8 + 8 for n, s, _, _ in entries)
    cur = _align(len(head) + table_size)
    offsets = {}
    for name, _, _, ln in entries:
        offsets[name] = cur
        cur = _align(cur + ln)
    for name, shape, dt, ln in entries:
        nb = name.encode()
        head += struct.pack("<I", len(nb)) + nb + struct.pack("<I", len(shape))
        for d in shape:
            head += struct.pack("<Q", int(d))
        head += struct.pack("<IQQ", dt, offsets[name], ln)
    return bytes(head), offsets, cur, entries


def empty_image(metadata, entries):
    """A zero-filled image with the header and table of `entries` written;
    returns (image, {name: offset}) for the caller to fill payloads in place."""
    head, offsets, total, _ = layout(metadata, entries)
    img = np.zeros(total, dtype=np.uint8)
    img[: len(head)] = np.frombuffer(head, dtype=np.uint8)
    return img, offsets


def write_image(metadata, tensors):
    """Builds a .hypno image.

    metadata: list of (key, value) strings, written in the given order.
    tensors: list of (name, shape tuple, dtype code, payload bytes-like); the
    payload length is the stored data_len (sft_convert.rs:162-168 computes it
    from the shape; callers pass exactly that many bytes).
    Returns a numpy uint8 array holding the whole image.
    """
    payloads = {}
    entries = []
    for name, shape, dt, payload in tensors:
        p = payload.view(np.uint8).reshape(-1) if isinstance(payload, np.ndarray) else np.frombuffer(payload, dtype=np.uint8)
        payloads[name] = p
        entries.append((name, tuple(shape), dt, p.size))
    img, offsets = empty_image(metadata, entries)
    for name, p in payloads.items():
        img[offsets[name]: offsets[name] + p.size] = p
    return img


class Manifest:
    """Parsed header, metadata and tensor table of an image (loader.rs:39-133)."""

    def __init__(self, buf):
        b = memoryview(np.ascontiguousarray(buf).view(np.uint8).reshape(-1)).cast("B")
        if len(b) < 16:
            raise ValueError(f"buffer too short: needed 16 bytes, got {len(b)}")
        if bytes(b[:4]) != MAGIC:
            raise ValueError("invalid magic bytes")
        ver, nkv, nt = struct.unpack_from("<III", b, 4)
        if ver != VERSION:
            raise ValueError(f"unsupported format version {ver} (expected 1)")
        cur = 16
        self.metadata = {}
        for _ in range(nkv):
            (kl,) = struct.unpack_from("<I", b, cur)
            k = bytes(b[cur + 4: cur + 4 + kl]).decode()
            cur += 4 + kl
            (vl,) = struct.unpack_from("<I", b, cur)
            v = bytes(b[cur + 4: cur + 4 + vl]).decode()
            cur += 4 + vl
            self.metadata.setdefault(k, v)
        self.tensors = {}
        for _ in range(nt):
            (nl,) = struct.unpack_from("<I", b, cur)
            name = bytes(b[cur + 4: cur + 4 + nl]).decode()
            cur += 4 + nl
            (nd,) = struct.unpack_from("<I", b, cur)
            cur += 4
            shape = struct.unpack_from("<" + "Q" * nd, b, cur)
            cur += 8 * nd
            dt, off, ln = struct.unpack_from("<IQQ", b, cur)
            cur += 20
            if off > len(b) or off + ln > len(b):
                raise ValueError(f"invalid tensor offset {off}: out of file bounds ({len(b)})")
            self.tensors.setdefault(name, (tuple(shape), dt, off, ln))
        self._buf = b

    def tensor_bytes(self, name):
        shape, dt, off, ln = self.tensors[name]
        return self._buf[off: off + ln], dt
