"""The framing of cuVS index files: every scalar and array is one NumPy
``.npy`` version-1.0 record (RAFT's numpy serializer), little endian, after a
4-byte dtype prefix of the dataset.

Follows python/mlxvs/cuvs/_serialize.py:11-105, whose files cuVS's own
``brute_force.load`` reads: the dtype strings, the header dictionary without
a trailing comma, and the padding of the record preamble to a multiple of 64
bytes with 1 to 64 spaces before the newline are kept byte for byte.
"""

import ast
import struct

import numpy as np

MAGIC = b"\x93NUMPY"

# RAFT's dtype strings (one-byte types have no byte order; bool is written as
# an unsigned byte)
_DESCR = {
    np.dtype(np.float32): "<f4",
    np.dtype(np.float64): "<f8",
    np.dtype(np.float16): "<e2",
    np.dtype(np.int8): "|i1",
    np.dtype(np.uint8): "|u1",
    np.dtype(np.bool_): "|u1",
    np.dtype(np.int32): "<i4",
    np.dtype(np.uint32): "<u4",
    np.dtype(np.int64): "<i8",
    np.dtype(np.uint64): "<u8",
}
_FROM_DESCR = {
    "<f4": np.float32,
    "<f8": np.float64,
    "<e2": np.float16,
    "<f2": np.float16,
    "|i1": np.int8,
    "|u1": np.uint8,
    "|b1": np.bool_,
    "<i4": np.int32,
    "<u4": np.uint32,
    "<i8": np.int64,
    "<u8": np.uint64,
}


def _header(dtype, shape):
    if len(shape) == 0:
        dims = "()"
    elif len(shape) == 1:
        dims = f"({int(shape[0])},)"
    else:
        dims = "(" + ", ".join(str(int(s)) for s in shape) + ")"
    text = f"{{'descr': '{_DESCR[np.dtype(dtype)]}', 'fortran_order': False, 'shape': {dims}}}"
    # magic, 2 version bytes, 2 length bytes, the text, the newline
    used = len(MAGIC) + 4 + len(text) + 1
    spaces = 64 - used % 64
    return (MAGIC + b"\x01\x00" + struct.pack("<H", len(text) + spaces + 1)
            + text.encode() + b" " * spaces + b"\n")


def write_scalar(f, value, dtype):
    f.write(_header(dtype, ()))
    f.write(np.array(value, dtype=dtype).tobytes())


def write_array(f, a):
    a = np.ascontiguousarray(a)
    f.write(_header(a.dtype, a.shape))
    f.write(a.tobytes())


def _read_header(f):
    head = f.read(10)
    if len(head) < 10 or head[:6] != MAGIC:
        raise ValueError("not a cuVS index file: missing a NumPy record")
    (size,) = struct.unpack("<H", head[8:10])
    fields = ast.literal_eval(f.read(size).decode("latin1").strip())
    if fields.get("fortran_order"):
        raise ValueError("Fortran-ordered arrays are not supported")
    if fields["descr"] not in _FROM_DESCR:
        raise ValueError(f"unknown dtype {fields['descr']!r} in a cuVS index file")
    return np.dtype(_FROM_DESCR[fields["descr"]]), tuple(fields["shape"])


def read_scalar(f):
    dtype, shape = _read_header(f)
    if shape:
        raise ValueError(f"expected a scalar, found shape {shape}")
    raw = f.read(dtype.itemsize)
    if len(raw) != dtype.itemsize:
        raise ValueError("truncated cuVS index file")
    return np.frombuffer(raw, dtype=dtype)[0].item()


def read_array(f):
    dtype, shape = _read_header(f)
    count = int(np.prod(shape)) if shape else 1
    raw = f.read(count * dtype.itemsize)
    if len(raw) != count * dtype.itemsize:
        raise ValueError("truncated cuVS index file")
    return np.frombuffer(raw, dtype=dtype).reshape(shape)


def dtype_prefix(dtype, version):
    """The 4-byte dtype prefix of an index file (NUL padded); half is "<f2"
    in files of format version 6 and later, "<e2" before."""
    s = _DESCR[np.dtype(dtype)]
    if s == "<e2" and version >= 6:
        s = "<f2"
    return s.encode().ljust(4, b"\0")


def read_prefix(f):
    s = f.read(4).rstrip(b"\0").decode("latin1")
    if s not in _FROM_DESCR:
        raise ValueError(f"unknown dtype prefix {s!r}")
    return np.dtype(_FROM_DESCR[s])
