"""helix-substrate model files (safetensors) in and out of this library.

A compressed module `prefix` is stored as the tensors
    prefix.codebook            float [k] (scalar VQ) or [k, vdim] (vector VQ)
    prefix.indices             integer [out_f, in_f] (scalar) or [out_f, in_f / vdim]
    prefix.sidecar_positions   int64 flat positions row * in_f + col   (optional)
    prefix.sidecar_values      float TARGET weights at those positions (optional)
(the layout the reference's tools/convert_hxq_to_gguf.py:237-295 reads).  In
that format a sidecar value replaces the decoded weight, the last entry of
a repeated position winning; hxq.c instead adds (row, col, delta)
corrections in array order (src/hxq.c:343-346).  `module_tensor` converts
each target into the delta that makes hxq.c's fp32 add land exactly on it,
so decompressing the module with this library gives the weights the file
describes, bit for bit.

Two containers are read, both directly (neither the safetensors nor the
gguf package is needed):
  * safetensors: 8-byte little-endian header length, a JSON header of
    {name: {dtype, shape, data_offsets}}, then the raw little-endian data;
  * GGUF (version 2 or 3), as the reference's converter writes in its
    "compressed" mode (tools/convert_hxq_to_gguf.py:611-633): codebook F32,
    indices I8 (the uint8 index bytes), sidecar positions I64 and values
    F32.  Names longer than 63 characters were abbreviated there
    (convert_hxq_to_gguf.py:32-72), so the sidecar parts may be called
    `.sc_pos` / `.sc_val`; a name cut short with a hash suffix no longer
    ends in its part and is not grouped.
"""
from __future__ import annotations

import json
import struct

import numpy as np

from .synth import HXQ_SCALAR_VQ, HXQ_VQ2D_12BIT, pack12

_DTYPES = {
    "F64": np.float64, "F32": np.float32, "F16": np.float16,
    "I64": np.int64, "I32": np.int32, "I16": np.int16, "I8": np.int8,
    "U64": np.uint64, "U32": np.uint32, "U16": np.uint16, "U8": np.uint8, "BOOL": np.bool_,
}
_NAMES = {np.dtype(v).str: k for k, v in _DTYPES.items()}
PARTS = ("codebook", "indices", "sidecar_positions", "sidecar_values")
_SUFFIXES = {"codebook": "codebook", "indices": "indices", "sidecar_positions": "sidecar_positions",
             "sidecar_values": "sidecar_values", "sc_pos": "sidecar_positions", "sc_val": "sidecar_values"}

# GGUF tensor types this reader takes (ggml type ids) and metadata value types
_GGML = {0: np.float32, 1: np.float16, 24: np.int8, 25: np.int16, 26: np.int32, 27: np.int64, 28: np.float64}
_GGML_BF16 = 30
_GGML_IDS = {np.dtype(v).str: k for k, v in _GGML.items()}
_GGUF_SCALAR = {0: "<u1", 1: "<i1", 2: "<u2", 3: "<i2", 4: "<u4", 5: "<i4", 6: "<f4", 7: "<u1",
                10: "<u8", 11: "<i8", 12: "<f8"}
_GGUF_STRING, _GGUF_ARRAY = 8, 9


def _bf16_to_f32(raw: np.ndarray) -> np.ndarray:
    return (raw.astype(np.uint32) << 16).view(np.float32)


def read_safetensors(path: str) -> dict[str, np.ndarray]:
    """All tensors of a safetensors file (BF16 widened to float32)."""
    with open(path, "rb") as f:
        blob = f.read()
    if len(blob) < 8:
        raise ValueError(f"{path}: not a safetensors file")
    (n,) = struct.unpack("<Q", blob[:8])
    if 8 + n > len(blob):
        raise ValueError(f"{path}: header length {n} past the end of the file")
    header = json.loads(blob[8:8 + n].decode("utf-8"))
    data = memoryview(blob)[8 + n:]
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        dt, shape = info["dtype"], tuple(info["shape"])
        b0, b1 = info["data_offsets"]
        if not (0 <= b0 <= b1 <= len(data)):
            raise ValueError(f"{path}: {name}: data offsets {b0}..{b1} outside the data")
        if dt == "BF16":
            arr = _bf16_to_f32(np.frombuffer(data[b0:b1], dtype="<u2"))
        elif dt in _DTYPES:
            arr = np.frombuffer(data[b0:b1], dtype=np.dtype(_DTYPES[dt]).newbyteorder("<")).astype(_DTYPES[dt])
        else:
            raise ValueError(f"{path}: {name}: unsupported dtype {dt}")
        if arr.size != int(np.prod(shape, dtype=np.int64)):
            raise ValueError(f"{path}: {name}: {arr.size} elements for shape {shape}")
        out[name] = arr.reshape(shape)
    return out


def write_safetensors(path: str, tensors: dict[str, np.ndarray], metadata: dict | None = None) -> None:
    """Write tensors (numpy arrays of the dtypes above) as a safetensors file."""
    header, chunks, off = {}, [], 0
    for name in sorted(tensors):
        a = np.ascontiguousarray(tensors[name])
        dt = _NAMES.get(a.dtype.newbyteorder("<").str if a.dtype.byteorder != "|" else a.dtype.str)
        if dt is None:
            raise ValueError(f"{name}: unsupported dtype {a.dtype}")
        raw = a.astype(a.dtype.newbyteorder("<"), copy=False).tobytes()
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(raw)]}
        chunks.append(raw)
        off += len(raw)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(header, separators=(",", ":")).encode("utf-8")
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for c in chunks:
            f.write(c)


class _Reader:
    def __init__(self, blob: bytes, path: str):
        self.b, self.o, self.path = blob, 0, path

    def take(self, n: int) -> bytes:
        if self.o + n > len(self.b):
            raise ValueError(f"{self.path}: truncated GGUF file")
        v = self.b[self.o:self.o + n]
        self.o += n
        return v

    def u(self, fmt: str):
        return struct.unpack(fmt, self.take(struct.calcsize(fmt)))[0]

    def string(self) -> str:
        return self.take(self.u("<Q")).decode("utf-8")

    def value(self, vt: int):
        if vt == _GGUF_STRING:
            return self.string()
        if vt == _GGUF_ARRAY:
            et, n = self.u("<I"), self.u("<Q")
            return [self.value(et) for _ in range(n)]
        if vt not in _GGUF_SCALAR:
            raise ValueError(f"{self.path}: unknown GGUF metadata type {vt}")
        v = np.frombuffer(self.take(np.dtype(_GGUF_SCALAR[vt]).itemsize), dtype=_GGUF_SCALAR[vt])[0]
        return bool(v) if vt == 7 else v.item()


def read_gguf(path: str) -> tuple[dict[str, np.ndarray], dict]:
    """(tensors, metadata) of a GGUF file.  Tensor shapes are given outermost
    first (numpy order; GGUF lists the innermost dimension first)."""
    with open(path, "rb") as f:
        blob = f.read()
    r = _Reader(blob, path)
    if r.take(4) != b"GGUF":
        raise ValueError(f"{path}: not a GGUF file")
    version = r.u("<I")
    if version not in (2, 3):
        raise ValueError(f"{path}: GGUF version {version} not supported")
    n_tensors, n_kv = r.u("<Q"), r.u("<Q")
    meta = {}
    for _ in range(n_kv):
        key = r.string()
        meta[key] = r.value(r.u("<I"))
    infos = []
    for _ in range(n_tensors):
        name = r.string()
        dims = [r.u("<Q") for _ in range(r.u("<I"))]
        infos.append((name, tuple(reversed(dims)), r.u("<I"), r.u("<Q")))
    align = int(meta.get("general.alignment", 32))
    base = (r.o + align - 1) // align * align
    out = {}
    for name, shape, gt, off in infos:
        n = int(np.prod(shape, dtype=np.int64))
        if gt == _GGML_BF16:
            dt, size = np.dtype("<u2"), 2
        elif gt in _GGML:
            dt = np.dtype(_GGML[gt]).newbyteorder("<")
            size = dt.itemsize
        else:
            raise ValueError(f"{path}: {name}: GGML type {gt} not supported")
        b0 = base + off
        if b0 + n * size > len(blob):
            raise ValueError(f"{path}: {name}: data past the end of the file")
        arr = np.frombuffer(blob, dtype=dt, count=n, offset=b0)
        arr = _bf16_to_f32(arr) if gt == _GGML_BF16 else arr.astype(dt.newbyteorder("="))
        out[name] = arr.reshape(shape)
    return out, meta


def write_gguf(path: str, tensors: dict[str, np.ndarray], metadata: dict[str, str] | None = None,
               alignment: int = 32) -> None:
    """Write tensors (float32/16/64, int8/16/32/64) as a GGUF version 3 file
    with string metadata."""
    def gstr(x: str) -> bytes:
        e = x.encode("utf-8")
        return struct.pack("<Q", len(e)) + e

    meta = dict(metadata or {})
    head = [b"GGUF", struct.pack("<IQQ", 3, len(tensors), len(meta) + (alignment != 32))]
    for k, v in meta.items():
        head += [gstr(k), struct.pack("<I", _GGUF_STRING), gstr(str(v))]
    if alignment != 32:
        head += [gstr("general.alignment"), struct.pack("<II", 4, alignment)]
    datas, off = [], 0
    for name in sorted(tensors):
        a = np.ascontiguousarray(tensors[name])
        gt = _GGML_IDS.get(a.dtype.newbyteorder("<").str if a.dtype.byteorder != "|" else a.dtype.str)
        if gt is None:
            raise ValueError(f"{name}: dtype {a.dtype} has no GGML type here")
        dims = list(reversed(a.shape)) or [1]
        head += [gstr(name), struct.pack("<I", len(dims)), struct.pack(f"<{len(dims)}Q", *dims),
                 struct.pack("<IQ", gt, off)]
        raw = a.astype(a.dtype.newbyteorder("<"), copy=False).tobytes()
        pad = -len(raw) % alignment
        datas.append(raw + b"\0" * pad)
        off += len(raw) + pad
    h = b"".join(head)
    h += b"\0" * (-len(h) % alignment)
    with open(path, "wb") as f:
        f.write(h)
        for d in datas:
            f.write(d)


def read_tensors(path: str) -> dict[str, np.ndarray]:
    """All tensors of a safetensors or GGUF file (told apart by the magic)."""
    with open(path, "rb") as f:
        magic = f.read(4)
    return read_gguf(path)[0] if magic == b"GGUF" else read_safetensors(path)


def hxq_modules(names) -> dict[str, dict[str, str]]:
    """{prefix: {part: tensor name}} for every prefix with a codebook and indices."""
    mods: dict[str, dict[str, str]] = {}
    for name in names:
        stem, _, last = name.rpartition(".")
        part = _SUFFIXES.get(last)
        if stem and part:
            mods.setdefault(stem, {})[part] = name
    return {p: m for p, m in mods.items() if "codebook" in m and "indices" in m}


def _same(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    return a.view(np.uint32) == b.view(np.uint32)


def _exact_deltas(base: np.ndarray, target: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """(d, reached): float32 d with float32(base + d) == target bit for bit
    where `reached` (hxq.c adds d to the codebook value in fp32).
    fl(target - base) is exact when the two are within a factor of two
    (Sterbenz); otherwise the subtraction's rounding can miss by an ulp and
    a few neighbouring floats of d are tried.  A target far below the
    codebook value's ulp (or -0.0) is not reachable by one add."""
    base = np.asarray(base, dtype=np.float32)
    target = np.asarray(target, dtype=np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        d = target - base
        miss = ~_same(base + d, target)
        lo, hi = d.copy(), d.copy()
        for _ in range(4):
            if not miss.any():
                break
            lo = np.nextafter(lo, np.float32(-np.inf))
            hi = np.nextafter(hi, np.float32(np.inf))
            for c in (lo, hi):
                hit = miss & _same(base + c, target)
                d = np.where(hit, c, d)
                miss &= ~hit
    return d.astype(np.float32), ~miss


def module_tensor(parts: dict[str, np.ndarray]) -> dict:
    """One helix-substrate module as a tensor dict for hxq_b200.Tensor.load:
    scalar VQ (8-bit indices, up to 256 codewords) or 2D VQ with vdim 2
    (12-bit packed pairs, up to 4096 codewords); the sidecar as (row, col, delta) entries whose fp32
    adds, in array order, reproduce the file's target weights bit for bit.
    A target that one add to its codebook value cannot reach becomes two
    entries at its position, -value then target (value + -value is +0.0
    exactly, and 0.0 + target is target); a -0.0 target decodes as +0.0.
    The confidence hxq.c reports for the module is the L2 norm of these
    deltas."""
    cb = np.asarray(parts["codebook"], dtype=np.float32)
    idx = np.asarray(parts["indices"])
    if idx.dtype == np.int8:               # uint8 index bytes stored as GGML I8
        idx = idx.view(np.uint8)
    if idx.ndim != 2:
        raise ValueError("indices must be [out_features, in_features / vector_dim]")
    k = cb.shape[0]
    vdim = 1 if cb.ndim == 1 else cb.shape[1]
    out_f, in_f = idx.shape[0], idx.shape[1] * vdim
    if idx.size and (int(idx.min()) < 0 or int(idx.max()) >= k):
        raise ValueError("an index is outside the codebook")
    if vdim not in (1, 2):
        raise ValueError(f"vector dimension {vdim} is not an hxq.c format")
    # hxq.c takes codebooks of exactly 256 (8-bit indices) or 4096 (12-bit)
    # entries (src/hxq.c:46); a shorter one is padded with zero codewords
    # that no index selects
    kk = 256 if vdim == 1 else 4096
    if k > kk:
        raise ValueError(f"{k} codewords of dimension {vdim}: hxq.c holds at most {kk}")
    flat_cb = np.zeros(kk * vdim, np.float32)
    flat_cb[:cb.size] = cb.reshape(-1)
    if vdim == 1:
        d = dict(mode=HXQ_SCALAR_VQ, out_f=out_f, in_f=in_f, k=kk, vdim=1, codebook=flat_cb,
                 indices=np.ascontiguousarray(idx.astype(np.uint8).reshape(-1)))
        dense = flat_cb[idx.reshape(-1).astype(np.int64)]
    else:
        pairs = idx.astype(np.uint16).reshape(-1)
        d = dict(mode=HXQ_VQ2D_12BIT, out_f=out_f, in_f=in_f, k=kk, vdim=2, codebook=flat_cb,
                 packed=pack12(pairs, out_f, in_f))
        dense = cb[pairs.astype(np.int64)].reshape(-1)
    pos = parts.get("sidecar_positions")
    val = parts.get("sidecar_values")
    if pos is None or len(pos) == 0:
        d.update(rows=np.zeros(0, np.uint32), cols=np.zeros(0, np.uint32), vals=np.zeros(0, np.float32))
        return d
    pos = np.asarray(pos, dtype=np.int64).reshape(-1)
    val = np.asarray(val, dtype=np.float32).reshape(-1)
    if pos.shape != val.shape:
        raise ValueError("sidecar positions and values differ in length")
    if (pos < 0).any() or (pos >= out_f * in_f).any():
        raise ValueError("a sidecar position is outside the tensor")
    # replace semantics: the last entry of a repeated position wins
    rev = pos[::-1]
    _, first_in_rev = np.unique(rev, return_index=True)
    keep = np.sort(len(pos) - 1 - first_in_rev)
    pos, val = pos[keep], val[keep]
    base = dense[pos]
    delta, reached = _exact_deltas(base, val)
    far = np.flatnonzero(~reached)
    if far.size:                      # two adds at each unreachable position
        at = np.repeat(np.arange(len(pos)), np.where(reached, 1, 2))
        second = np.zeros(len(at), bool)
        second[np.cumsum(np.where(reached, 1, 2)) - 1] = ~reached
        vals = np.where(second, val[at], np.where(reached[at], delta[at], -base[at])).astype(np.float32)
        pos = pos[at]
    else:
        vals = delta
    d.update(rows=(pos // in_f).astype(np.uint32), cols=(pos % in_f).astype(np.uint32), vals=vals)
    return d


def load_modules(path: str) -> dict[str, dict]:
    """{prefix: tensor dict} for every compressed module of a safetensors or
    GGUF file."""
    tensors = read_tensors(path)
    out = {}
    for prefix, names in hxq_modules(tensors.keys()).items():
        out[prefix] = module_tensor({part: tensors[name] for part, name in names.items()})
    return out
