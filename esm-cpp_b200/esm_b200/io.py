"""Weight files: HF safetensors (FP32) and GGUF v3 with the reference's
Q8_ESM tensor type.

Formats follow the reference's loaders so the two engines read and write the
same artefacts:
  * safetensors: 8-byte little-endian header length, JSON header
    {name: {dtype, shape, data_offsets}}, raw data (io/safetensors.cpp).
  * GGUF v3 (io/gguf.cpp, model.cpp:174-298, 562-725): metadata KV section,
    tensor infos with shapes in [in, out] order, data aligned to
    general.alignment (32).  Q8_ESM (type 100) stores [N*K int8][N fp32
    scales] for a weight of logical shape [N, K]; its wire shape is [K, N].
"""
from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

GGUF_MAGIC = 0x46554747
GGUF_VERSION = 3
GGML_F32, GGML_F16, GGML_Q8_ESM = 0, 1, 100

_ST_DTYPES = {"F32": np.float32, "F16": np.float16, "I32": np.int32, "I64": np.int64,
              "I8": np.int8, "U8": np.uint8, "F64": np.float64}
_ST_NAMES = {np.dtype(v): k for k, v in _ST_DTYPES.items()}


# ------------------------------------------------------------- safetensors
def read_safetensors(path) -> dict[str, np.ndarray]:
    data = Path(path).read_bytes()
    (n,) = struct.unpack_from("<Q", data, 0)
    header = json.loads(data[8:8 + n])
    base = 8 + n
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        b, e = info["data_offsets"]
        arr = np.frombuffer(data, dtype=_ST_DTYPES[info["dtype"]], count=(e - b) // np.dtype(_ST_DTYPES[info["dtype"]]).itemsize, offset=base + b)
        out[name] = arr.reshape(info["shape"]).copy()
    return out


def write_safetensors(path, tensors: dict[str, np.ndarray]) -> None:
    header, blobs, off = {}, [], 0
    for name, arr in tensors.items():
        arr = np.ascontiguousarray(arr)
        raw = arr.tobytes()
        header[name] = {"dtype": _ST_NAMES[arr.dtype], "shape": list(arr.shape),
                        "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for b in blobs:
            f.write(b)


# -------------------------------------------------------------------- GGUF
def _read_str(buf, p):
    (n,) = struct.unpack_from("<Q", buf, p)
    p += 8
    return buf[p:p + n].decode(), p + n


_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 10: "<Q", 11: "<q", 12: "<d"}


def _read_value(buf, p, t):
    if t in _SCALAR:
        fmt = _SCALAR[t]
        (v,) = struct.unpack_from(fmt, buf, p)
        return v, p + struct.calcsize(fmt)
    if t == 7:
        return buf[p] != 0, p + 1
    if t == 8:
        return _read_str(buf, p)
    if t == 9:
        (et,) = struct.unpack_from("<I", buf, p)
        (cnt,) = struct.unpack_from("<Q", buf, p + 4)
        p += 12
        vals = []
        for _ in range(cnt):
            v, p = _read_value(buf, p, et)
            vals.append(v)
        return vals, p
    raise ValueError(f"gguf: unknown metadata type {t}")


def read_gguf(path):
    """Returns (metadata dict, tensors dict).  F32 tensors come back in their
    logical row-major shape (wire shape reversed); Q8_ESM tensors come back
    as a (int8 [N, K], float32 [N]) pair."""
    buf = Path(path).read_bytes()
    magic, version = struct.unpack_from("<II", buf, 0)
    if magic != GGUF_MAGIC:
        raise ValueError(f"gguf: bad magic in {path}")
    if version != GGUF_VERSION:
        raise ValueError(f"gguf: version {version} not supported (need v3)")
    n_tensors, n_meta = struct.unpack_from("<QQ", buf, 8)
    p = 24
    meta = {}
    for _ in range(n_meta):
        k, p = _read_str(buf, p)
        (t,) = struct.unpack_from("<I", buf, p)
        v, p = _read_value(buf, p + 4, t)
        meta[k] = v
    infos = []
    for _ in range(n_tensors):
        name, p = _read_str(buf, p)
        (nd,) = struct.unpack_from("<I", buf, p)
        shape = list(struct.unpack_from(f"<{nd}Q", buf, p + 4))
        p += 4 + 8 * nd
        t, off = struct.unpack_from("<IQ", buf, p)
        p += 12
        infos.append((name, shape, t, off))
    align = int(meta.get("general.alignment", 32))
    data0 = (p + align - 1) // align * align
    tensors = {}
    for name, shape, t, off in infos:
        o = data0 + off
        if t == GGML_F32:
            n = int(np.prod(shape)) if shape else 1
            arr = np.frombuffer(buf, np.float32, n, o).reshape(shape[::-1]).copy()
            tensors[name] = arr
        elif t == GGML_Q8_ESM:
            K, N = shape
            q = np.frombuffer(buf, np.int8, N * K, o).reshape(N, K).copy()
            s = np.frombuffer(buf, np.float32, N, o + N * K).copy()
            tensors[name] = (q, s)
        elif t == GGML_F16:
            n = int(np.prod(shape))
            tensors[name] = np.frombuffer(buf, np.float16, n, o).reshape(shape[::-1]).astype(np.float32)
        else:
            raise ValueError(f"gguf: unknown tensor type {t} for {name}")
    return meta, tensors


def _meta_bytes(k, v):
    out = struct.pack("<Q", len(k.encode())) + k.encode()
    if isinstance(v, bool):
        return out + struct.pack("<IB", 7, int(v))
    if isinstance(v, int):
        return out + struct.pack("<Iq", 11, v)
    if isinstance(v, float):
        return out + struct.pack("<Id", 12, v)
    if isinstance(v, str):
        b = v.encode()
        return out + struct.pack("<IQ", 8, len(b)) + b
    raise TypeError(f"unsupported metadata value for {k}")


def write_gguf(path, meta: dict, tensors: list) -> None:
    """tensors: list of (name, value) with value an FP32 ndarray (logical
    row-major shape) or an (int8 [N, K], float32 [N]) Q8_ESM pair."""
    align = int(meta.get("general.alignment", 32))
    infos, blobs, cur = [], [], 0
    for name, val in tensors:
        if isinstance(val, tuple):
            q, s = val
            N, K = q.shape
            raw = np.ascontiguousarray(q, np.int8).tobytes() + np.ascontiguousarray(s, np.float32).tobytes()
            shape, t = [K, N], GGML_Q8_ESM
        else:
            a = np.ascontiguousarray(val, np.float32)
            raw = a.tobytes()
            shape, t = list(a.shape[::-1]), GGML_F32
        infos.append((name, shape, t, cur))
        pad = (align - len(raw) % align) % align
        blobs.append(raw + b"\0" * pad)
        cur += len(raw) + pad
    head = struct.pack("<IIQQ", GGUF_MAGIC, GGUF_VERSION, len(tensors), len(meta))
    for k, v in meta.items():
        head += _meta_bytes(k, v)
    for name, shape, t, off in infos:
        nb = name.encode()
        head += struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(shape))
        head += struct.pack(f"<{len(shape)}Q", *shape) + struct.pack("<IQ", t, off)
    head += b"\0" * ((align - len(head) % align) % align)
    with open(path, "wb") as f:
        f.write(head)
        for b in blobs:
            f.write(b)
