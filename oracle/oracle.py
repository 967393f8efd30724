"""ctypes access to the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Loads oracle/liboracle.so (this repository's C restatement of the
reference algorithm, hxq_oracle.c) and, when it was built here,
oracle/_ref/libhxqref.so (the reference library itself compiled from its
own sources with renamed symbols).  Only tests, the smoke check and the
benchmark's CPU-baseline leg use this module; the product never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libhxqref.so")
REF_LLOYD_SO = os.path.join(HERE, "_ref", "libhxqref_lloyd.so")
REF_PQ_SO = os.path.join(HERE, "_ref", "libpqref.so")

P = C.c_void_p


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE, "oracle"], check=True)


def _p(a):
    return None if a is None else a.ctypes.data


class Oracle:
    """The C restatement (hxq_oracle.c)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build()
        L = self.L = C.CDLL(path)
        L.orc_decompress.restype = C.c_int
        L.orc_decompress.argtypes = [C.c_int, P, C.c_uint32, C.c_uint32, P, C.c_size_t, C.c_uint32,
                                     C.c_uint32, P, P, C.c_uint32, P, P, P, C.c_uint32, P, P]
        L.orc_affine_matmul_rows.restype = None
        L.orc_affine_matmul_rows.argtypes = [P, P, P, P, P, P, C.c_uint32, C.c_uint32, C.c_uint32,
                                             C.c_uint32, C.c_uint32]
        L.orc_affine_decompress.restype = None
        L.orc_affine_decompress.argtypes = [P, P, P, P, C.c_uint32, C.c_uint32, C.c_uint32]
        L.orc_sidecar_l2_exact.restype = C.c_double
        L.orc_sidecar_l2_exact.argtypes = [P, P, P, C.c_uint32, C.c_uint32, C.c_uint32]
        L.orc_dense_matmul_rows.restype = None
        L.orc_dense_matmul_rows.argtypes = [P, P, P, P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]
        L.orc_dense_matmul_rows_f64.restype = None
        L.orc_dense_matmul_rows_f64.argtypes = [P, P, P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]
        L.orc_pack12.restype = None
        L.orc_pack12.argtypes = [C.c_uint16, C.c_uint16, P]
        L.orc_unpack12.restype = None
        L.orc_unpack12.argtypes = [P, P, P]
        L.orc_pack_rows12.restype = C.c_size_t
        L.orc_pack_rows12.argtypes = [P, C.c_uint32, C.c_uint32, P]
        L.orc_lloyd_assign.restype = None
        L.orc_lloyd_assign.argtypes = [P, P, P, C.c_size_t, C.c_int, C.c_int]
        L.orc_lloyd_reassign.restype = C.c_int
        L.orc_lloyd_reassign.argtypes = [P, P, P, C.c_size_t, C.c_int, C.c_int]
        L.orc_pq_apply.restype = None
        L.orc_pq_apply.argtypes = [P, P, C.c_size_t, C.c_uint32, C.c_int, P]

    def decompress(self, d: dict, out: np.ndarray | None = None, k: int | None = None,
                   vdim: int | None = None, idx_len: int | None = None):
        """Returns (err, weights[out_f*in_f] fp32, confidence or None)."""
        n = d["out_f"] * d["in_f"]
        if out is None:
            out = np.zeros(n, np.float32)
        mode = d["mode"]
        if mode == 3:
            idx = np.ascontiguousarray(d["codes"], np.uint8)
            cb = None
            s, o, gs = d["scales"], d["offsets"], d["gs"]
        else:
            idx = np.ascontiguousarray(d["packed"] if mode == 2 else d["indices"], np.uint8)
            cb = np.ascontiguousarray(d["codebook"], np.float32)
            s = o = None
            gs = 0
        rows = d.get("rows")
        nnz = 0 if rows is None else len(rows)
        l2 = np.zeros(1, np.float32)
        err = self.L.orc_decompress(
            mode, _p(cb), k if k is not None else d.get("k", 0), vdim if vdim is not None else d.get("vdim", 0),
            _p(idx), idx.size if idx_len is None else idx_len, d["out_f"], d["in_f"], _p(s), _p(o), gs,
            _p(rows) if nnz else None, _p(d.get("cols")) if nnz else None, _p(d.get("vals")) if nnz else None,
            nnz, _p(out), _p(l2))
        return err, out, (float(l2[0]) if err == 0 else None)

    def l2_exact(self, d: dict) -> float:
        rows = d.get("rows")
        if rows is None or len(rows) == 0:
            return 0.0
        return float(self.L.orc_sidecar_l2_exact(_p(rows), _p(d["cols"]), _p(d["vals"]), len(rows),
                                                 d["out_f"], d["in_f"]))

    def affine_matmul(self, x: np.ndarray, d: dict, bias=None, n0: int = 0, n1: int | None = None):
        x = np.ascontiguousarray(x, np.float32)
        N = x.shape[0]
        n1 = N if n1 is None else n1
        out = np.zeros((N, d["out_f"]), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self.L.orc_affine_matmul_rows(_p(x), _p(d["codes"]), _p(d["scales"]), _p(d["offsets"]), _p(b),
                                      _p(out), n0, n1, d["in_f"], d["out_f"], d["gs"])
        return out[n0:n1]

    def affine_decompress(self, d: dict) -> np.ndarray:
        out = np.zeros(d["out_f"] * d["in_f"], np.float32)
        self.L.orc_affine_decompress(_p(d["codes"]), _p(d["scales"]), _p(d["offsets"]), _p(out),
                                     d["out_f"], d["in_f"], d["gs"])
        return out

    def dense_matmul(self, x: np.ndarray, W: np.ndarray, bias=None, n0: int = 0, n1: int | None = None):
        x = np.ascontiguousarray(x, np.float32)
        W = np.ascontiguousarray(W, np.float32)
        N, in_f = x.shape
        out_f = W.size // in_f
        n1 = N if n1 is None else n1
        out = np.zeros((N, out_f), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self.L.orc_dense_matmul_rows(_p(x), _p(W), _p(b), _p(out), n0, n1, in_f, out_f)
        return out[n0:n1]

    def dense_matmul_f64(self, x: np.ndarray, W: np.ndarray, n0: int = 0, n1: int | None = None):
        x = np.ascontiguousarray(x, np.float32)
        W = np.ascontiguousarray(W, np.float32)
        N, in_f = x.shape
        out_f = W.size // in_f
        n1 = N if n1 is None else n1
        out = np.zeros((n1 - n0, out_f), np.float64)
        self.L.orc_dense_matmul_rows_f64(_p(x), _p(W), _p(out), n0, n1, in_f, out_f)
        return out

    def lloyd_assign(self, w: np.ndarray, cb: np.ndarray, k: int, d: int) -> np.ndarray:
        w = np.ascontiguousarray(w, np.float32)
        cb = np.ascontiguousarray(cb, np.float32)
        n = w.size // d
        idx = np.zeros(n, np.uint8)
        self.L.orc_lloyd_assign(_p(w), _p(cb), _p(idx), n, k, d)
        return idx

    def lloyd_reassign(self, w: np.ndarray, cb: np.ndarray, k: int, d: int):
        """(indices, updated codebook, dead count)."""
        w = np.ascontiguousarray(w, np.float32)
        cb = np.array(cb, np.float32, copy=True)
        n = w.size // d
        idx = np.zeros(n, np.uint8)
        dead = self.L.orc_lloyd_reassign(_p(w), _p(cb), _p(idx), n, k, d)
        return idx, cb, dead

    def pq_apply(self, values: np.ndarray, Q: np.ndarray, head_dim: int, rotate: bool) -> np.ndarray:
        """head @ Q^T (rotate) or head @ Q, for every head_dim-vector."""
        out = np.array(values, np.float32, copy=True).reshape(-1)
        Q = np.ascontiguousarray(Q, np.float32)
        tmp = np.zeros(head_dim, np.float32)
        self.L.orc_pq_apply(_p(out), _p(Q), out.size // head_dim, head_dim, 1 if rotate else 0, _p(tmp))
        return out

    def pack12(self, a: int, b: int) -> bytes:
        buf = np.zeros(3, np.uint8)
        self.L.orc_pack12(a, b, _p(buf))
        return bytes(buf)

    def unpack12(self, three: bytes):
        buf = np.frombuffer(three, np.uint8).copy()
        a = np.zeros(1, np.uint16)
        b = np.zeros(1, np.uint16)
        self.L.orc_unpack12(_p(buf), _p(a), _p(b))
        return int(a[0]), int(b[0])

    def pack_rows12(self, idx: np.ndarray, out_f: int, in_f: int) -> np.ndarray:
        idx = np.ascontiguousarray(idx, np.uint16)
        n = self.L.orc_pack_rows12(_p(idx), out_f, in_f, None)
        out = np.zeros(n, np.uint8)
        self.L.orc_pack_rows12(_p(idx), out_f, in_f, _p(out))
        return out


class _RefTensor(C.Structure):
    _fields_ = [
        ("codebook", P), ("k", C.c_uint32), ("vector_dim", C.c_uint32),
        ("indices_raw", P), ("indices_len", C.c_size_t),
        ("sidecar_rows", P), ("sidecar_cols", P), ("sidecar_vals", P), ("sidecar_nnz", C.c_uint32),
        ("out_features", C.c_uint32), ("in_features", C.c_uint32), ("mode", C.c_int),
        ("affine_scales", P), ("affine_offsets", P), ("affine_group_size", C.c_uint32),
        ("sidecar_l2_norm", C.c_float),
    ]


class _RefBuf(C.Structure):
    _fields_ = [("data", P), ("capacity", C.c_size_t), ("high_water", C.c_size_t)]


class _RefResult(C.Structure):
    _fields_ = [("weights", P), ("confidence", C.c_float), ("out_features", C.c_uint32),
                ("in_features", C.c_uint32)]


def container_dense(parts: dict) -> np.ndarray:
    """Dense fp32 weights of one helix-substrate module as the reference's
    converter defines them (tools/convert_hxq_to_gguf.py:268-295,
    dequant_hxq_tensor): codebook lookup (a 2-D codebook gives a pair per
    index), then every sidecar value REPLACES the weight at its flat
    position, in array order, so the last of repeated positions wins.
    Pinned to fixtures made by that function itself
    (tests/golden/make_container_golden.py)."""
    cb = np.asarray(parts["codebook"], dtype=np.float32)
    idx = np.asarray(parts["indices"])
    idx = (idx.view(np.uint8) if idx.dtype == np.int8 else idx).astype(np.int64)
    W = (cb[idx] if cb.ndim == 1 else cb[idx].reshape(idx.shape[0], -1)).reshape(-1).copy()
    pos = parts.get("sidecar_positions")
    if pos is not None:
        for q, v in zip(np.asarray(pos).reshape(-1), np.asarray(parts["sidecar_values"], np.float32).reshape(-1)):
            W[int(q)] = v
    return W


def ref_available(path: str = REF_SO) -> bool:
    return os.path.exists(path)


class Reference:
    """The reference library compiled from its own sources (oracle/_ref)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = self.L = C.CDLL(path)
        TP = C.POINTER(_RefTensor)
        for name, res, args in [
            ("ref_hxq_tensor_init", C.c_int, [TP]),
            ("ref_hxq_tensor_free", None, [TP]),
            ("ref_hxq_tensor_load_codebook", C.c_int, [TP, P, C.c_uint32, C.c_uint32]),
            ("ref_hxq_tensor_load_indices_8bit", C.c_int, [TP, P, C.c_uint32, C.c_uint32]),
            ("ref_hxq_tensor_load_indices_12bit", C.c_int, [TP, P, C.c_size_t, C.c_uint32, C.c_uint32]),
            ("ref_hxq_tensor_load_sidecar", C.c_int, [TP, P, P, P, C.c_uint32]),
            ("ref_hxq_tensor_load_affine", C.c_int, [TP, P, P, P, C.c_uint32, C.c_uint32, C.c_uint32]),
            ("ref_hxq_tensor_decompress", C.c_int, [TP, P]),
            ("ref_hxq_shared_buffer_init", C.c_int, [C.POINTER(_RefBuf), C.c_size_t]),
            ("ref_hxq_shared_buffer_free", None, [C.POINTER(_RefBuf)]),
            ("ref_hxq_dequant", C.c_int, [TP, C.POINTER(_RefBuf), C.c_int, C.POINTER(_RefResult)]),
            ("ref_hxq_affine_group_matmul_ref", None, [P, P, P, P, P, P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]),
            ("ref_hxq_affine_decompress_ref", None, [P, P, P, P, C.c_uint32, C.c_uint32, C.c_uint32]),
        ]:
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args

    def tensor(self, d: dict, idx_len: int | None = None, k: int | None = None, vdim: int | None = None):
        """Build a reference hxq_tensor_t from a synth dict (caller frees)."""
        t = _RefTensor()
        L = self.L
        L.ref_hxq_tensor_init(C.byref(t))
        keep = []
        if d["mode"] == 3:
            arrs = [np.ascontiguousarray(d["codes"], np.uint8), np.ascontiguousarray(d["scales"], np.float32),
                    np.ascontiguousarray(d["offsets"], np.float32)]
            keep += arrs
            err = L.ref_hxq_tensor_load_affine(C.byref(t), *[a.ctypes.data for a in arrs], d["out_f"], d["in_f"], d["gs"])
            assert err == 0, err
        else:
            cb = np.ascontiguousarray(d["codebook"], np.float32)
            err = L.ref_hxq_tensor_load_codebook(C.byref(t), cb.ctypes.data, k or d["k"], vdim or d["vdim"])
            assert err == 0, err
            if d["mode"] == 0:
                idx = np.ascontiguousarray(d["indices"], np.uint8)
                err = L.ref_hxq_tensor_load_indices_8bit(C.byref(t), idx.ctypes.data, d["out_f"], d["in_f"])
            else:
                idx = np.ascontiguousarray(d["packed"], np.uint8)
                err = L.ref_hxq_tensor_load_indices_12bit(C.byref(t), idx.ctypes.data,
                                                          idx.size if idx_len is None else idx_len,
                                                          d["out_f"], d["in_f"])
            assert err == 0, err
        rows = d.get("rows")
        if rows is not None and len(rows):
            arrs = [np.ascontiguousarray(rows, np.uint32), np.ascontiguousarray(d["cols"], np.uint32),
                    np.ascontiguousarray(d["vals"], np.float32)]
            err = L.ref_hxq_tensor_load_sidecar(C.byref(t), *[a.ctypes.data for a in arrs], len(rows))
            assert err == 0, err
        return t

    def decompress(self, d: dict, out: np.ndarray | None = None, **kw):
        """(err, weights, confidence) from ref hxq_tensor_decompress."""
        t = self.tensor(d, **kw)
        n = d["out_f"] * d["in_f"]
        if out is None:
            out = np.zeros(n, np.float32)
        err = self.L.ref_hxq_tensor_decompress(C.byref(t), out.ctypes.data)
        conf = t.sidecar_l2_norm
        self.L.ref_hxq_tensor_free(C.byref(t))
        return err, out, (float(conf) if err == 0 else None)

    def affine_matmul(self, x: np.ndarray, d: dict, bias=None) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros((x.shape[0], d["out_f"]), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self.L.ref_hxq_affine_group_matmul_ref(x.ctypes.data, d["codes"].ctypes.data, d["scales"].ctypes.data,
                                               d["offsets"].ctypes.data, None if b is None else b.ctypes.data,
                                               out.ctypes.data, x.shape[0], d["in_f"], d["out_f"], d["gs"])
        return out


class ReferenceLloyd:
    """The reference's Lloyd library compiled from its own source (oracle/_ref)."""

    def __init__(self, path: str = REF_LLOYD_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = self.L = C.CDLL(path)
        L.ref_hxq_lloyd_reassign.restype = C.c_int
        L.ref_hxq_lloyd_reassign.argtypes = [P, P, P, C.c_size_t, C.c_int, C.c_int, P]
        L.ref_hxq_lloyd_assign_only.restype = C.c_int
        L.ref_hxq_lloyd_assign_only.argtypes = [P, P, P, C.c_size_t, C.c_int, C.c_int]

    def reassign(self, w: np.ndarray, cb: np.ndarray, k: int, d: int):
        """(return code, indices, updated codebook, dead count)."""
        w = np.ascontiguousarray(w, np.float32)
        cb = np.array(cb, np.float32, copy=True)
        n = w.size // d
        idx = np.zeros(n, np.uint8)
        dead = C.c_int(-1)
        rc = self.L.ref_hxq_lloyd_reassign(_p(w), _p(cb), _p(idx), n, k, d, C.addressof(dead))
        return rc, idx, cb, dead.value

    def assign(self, w: np.ndarray, cb: np.ndarray, k: int, d: int):
        w = np.ascontiguousarray(w, np.float32)
        cb = np.ascontiguousarray(cb, np.float32)
        idx = np.zeros(w.size // d, np.uint8)
        rc = self.L.ref_hxq_lloyd_assign_only(_p(w), _p(cb), _p(idx), w.size // d, k, d)
        return rc, idx


class ReferencePolarQuant:
    """The reference's PolarQuant library compiled from its own source (oracle/_ref)."""

    def __init__(self, path: str = REF_PQ_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = self.L = C.CDLL(path)
        for name, res, args in [
            ("ref_pq_generate_rotation", C.c_int, [C.c_uint32, C.c_uint32, P]),
            ("ref_pq_rotate", C.c_int, [P, P, C.c_uint32, C.c_uint32]),
            ("ref_pq_unrotate", C.c_int, [P, P, C.c_uint32, C.c_uint32]),
        ]:
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args

    def rotation(self, dim: int, seed: int) -> np.ndarray:
        Q = np.zeros(dim * dim, np.float32)
        assert self.L.ref_pq_generate_rotation(dim, seed, _p(Q)) == 0
        return Q.reshape(dim, dim)

    def apply(self, values: np.ndarray, Q: np.ndarray, head_dim: int, rotate: bool) -> np.ndarray:
        out = np.array(values, np.float32, copy=True).reshape(-1)
        Q = np.ascontiguousarray(Q, np.float32)
        fn = self.L.ref_pq_rotate if rotate else self.L.ref_pq_unrotate
        assert fn(_p(out), _p(Q), out.size // head_dim, head_dim) == 0
        return out
