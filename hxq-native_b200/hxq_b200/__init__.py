"""ctypes binding of libhxq.so, the B200 implementation of the HXQ codec.

The shared library exports the reference C API (include/hxq.h,
include/hxq_affine.h) and the additive CUDA API (include/hxq_cuda.h).  This
module declares every entry point with its C signature and offers small
numpy-friendly helpers; it does no computation of its own.  Loading fails
loudly when the library has not been built (`make -C hxq-native_b200`).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.dirname(_HERE)
REPO_DIR = os.path.dirname(PKG_DIR)
# HXQ_LIB names another build of the library (e.g. one made with different
# EXTRA flags); by default the one `make -C hxq-native_b200` puts in lib/.
LIB_PATH = os.environ.get("HXQ_LIB") or os.path.join(PKG_DIR, "lib", "libhxq.so")
INCLUDE_DIR = os.path.join(REPO_DIR, "include")

# -- status codes (include/hxq.h, include/hxq_cuda.h) ------------------------
HXQ_OK = 0
HXQ_ERR_NULL_PTR = 1
HXQ_ERR_INVALID_K = 2
HXQ_ERR_INVALID_DIM = 3
HXQ_ERR_ALLOC_FAILED = 4
HXQ_ERR_INDEX_OOB = 5
HXQ_ERR_PACK_FORMAT = 6
HXQ_ERR_SIDECAR_OOB = 7
HXQ_ERR_CUDA = 32
HXQ_ERR_BACKEND_UNAVAILABLE = 33
HXQ_ERR_INVALID_ARG = 34
HXQ_ERR_NCCL = 35

HXQ_SCALAR_VQ, HXQ_VQ2D_8BIT, HXQ_VQ2D_12BIT, HXQ_AFFINE_G128 = 0, 1, 2, 3
HXQ_BACKEND_AUTO, HXQ_BACKEND_CPU, HXQ_BACKEND_CUDA, HXQ_BACKEND_METAL, HXQ_BACKEND_VULKAN = range(5)
HXQ_OUT_F32, HXQ_OUT_BF16 = 0, 1
HXQ_IMAGE_STREAMED, HXQ_IMAGE_MATMUL = 1, 2
HXQ_AFFINE_PATH_AUTO, HXQ_AFFINE_PATH_GEMV, HXQ_AFFINE_PATH_TC_GEMV, HXQ_AFFINE_PATH_GEMM = 0, 1, 2, 3
MAX_BATCH = 64

P = C.c_void_p
u8p = C.POINTER(C.c_uint8)
u16p = C.POINTER(C.c_uint16)
u32p = C.POINTER(C.c_uint32)
f32p = C.POINTER(C.c_float)


class HxqTensor(C.Structure):
    """hxq_tensor_t, 96 bytes (include/hxq.h)."""
    _fields_ = [
        ("codebook", f32p), ("k", C.c_uint32), ("vector_dim", C.c_uint32),
        ("indices_raw", u8p), ("indices_len", C.c_size_t),
        ("sidecar_rows", u32p), ("sidecar_cols", u32p), ("sidecar_vals", f32p),
        ("sidecar_nnz", C.c_uint32),
        ("out_features", C.c_uint32), ("in_features", C.c_uint32),
        ("mode", C.c_int),
        ("affine_scales", f32p), ("affine_offsets", f32p),
        ("affine_group_size", C.c_uint32),
        ("sidecar_l2_norm", C.c_float),
    ]


class SharedBuffer(C.Structure):
    """hxq_shared_buffer_t, 24 bytes."""
    _fields_ = [("data", P), ("capacity", C.c_size_t), ("high_water", C.c_size_t)]


class Result(C.Structure):
    """hxq_result_t, 24 bytes."""
    _fields_ = [("weights", P), ("confidence", C.c_float),
                ("out_features", C.c_uint32), ("in_features", C.c_uint32)]


class AffineTensor(C.Structure):
    """hxq_affine_tensor_t, 48 bytes; device pointers for the GPU API."""
    _fields_ = [("indices", P), ("scales", P), ("offsets", P), ("bias", P),
                ("out_features", C.c_uint32), ("in_features", C.c_uint32),
                ("group_size", C.c_uint32)]


TP = C.POINTER(HxqTensor)
BP = C.POINTER(SharedBuffer)

# name -> (restype, argtypes)
SIGNATURES = {
    # include/hxq.h
    "hxq_tensor_init": (C.c_int, [TP]),
    "hxq_tensor_load_codebook": (C.c_int, [TP, P, C.c_uint32, C.c_uint32]),
    "hxq_tensor_load_indices_8bit": (C.c_int, [TP, P, C.c_uint32, C.c_uint32]),
    "hxq_tensor_load_indices_12bit": (C.c_int, [TP, P, C.c_size_t, C.c_uint32, C.c_uint32]),
    "hxq_tensor_load_affine": (C.c_int, [TP, P, P, P, C.c_uint32, C.c_uint32, C.c_uint32]),
    "hxq_tensor_load_sidecar": (C.c_int, [TP, P, P, P, C.c_uint32]),
    "hxq_tensor_decompress": (C.c_int, [TP, P]),
    "hxq_tensor_decompress_shared": (C.c_int, [TP, BP, C.POINTER(P)]),
    "hxq_tensor_free": (None, [TP]),
    "hxq_shared_buffer_init": (C.c_int, [BP, C.c_size_t]),
    "hxq_shared_buffer_free": (None, [BP]),
    "hxq_dequant": (C.c_int, [TP, BP, C.c_int, C.POINTER(Result)]),
    # include/hxq_affine.h
    "hxq_affine_group_matmul_ref": (None, [P, P, P, P, P, P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]),
    "hxq_affine_decompress_ref": (None, [P, P, P, P, C.c_uint32, C.c_uint32, C.c_uint32]),
    "hxq_affine_group_matmul": (C.c_int, [P, C.POINTER(AffineTensor), P, C.c_uint32]),
    "hxq_affine_matmul_flat": (C.c_int, [P, P, P, P, P, P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]),
    # include/hxq_cuda.h
    "hxq_error_string": (C.c_char_p, [C.c_int]),
    "hxq_b200_version": (C.c_char_p, []),
    "hxq_cuda_device_count": (C.c_int, []),
    "hxq_cuda_arena_init": (C.c_int, [BP, C.c_size_t]),
    "hxq_cuda_buffer_is_device": (C.c_int, [BP]),
    "hxq_cuda_decompress": (C.c_int, [TP, P, C.c_int]),
    "hxq_dequant_bf16": (C.c_int, [TP, BP, C.POINTER(Result)]),
    "hxq_cuda_tensor_invalidate": (None, [TP]),
    "hxq_cuda_image_create": (C.c_int, [TP, C.c_uint32, C.c_uint32, C.POINTER(P)]),
    "hxq_cuda_image_destroy": (None, [P]),
    "hxq_cuda_image_numel": (C.c_size_t, [P]),
    "hxq_cuda_image_device_bytes": (C.c_size_t, [P]),
    "hxq_cuda_image_sidecar_sumsq": (C.c_double, [P]),
    "hxq_cuda_image_reference_confidence": (C.c_float, [P]),
    "hxq_cuda_image_tensor_confidence": (C.c_float, [P]),
    "hxq_cuda_decompress_images": (C.c_int, [C.POINTER(P), C.c_uint32, P, C.POINTER(C.c_size_t), C.c_int, P, P, P]),
    "hxq_cuda_stream_synchronize": (C.c_int, [P]),
    "hxq_cuda_decompress_images_noalloc": (C.c_int, [C.POINTER(P), C.c_uint32, P, C.POINTER(C.c_size_t), C.c_int, P, P, P]),
    "hxq_cuda_image_create_streamed": (C.c_int, [TP, C.c_uint32, C.c_uint32, C.POINTER(P)]),
    "hxq_cuda_image_block_bytes": (C.c_size_t, [P]),
    "hxq_cuda_image_upload": (C.c_int, [P, P, P]),
    "hxq_cuda_launch_count": (C.c_ulonglong, []),
    "hxq_cuda_decompress_scalar": (C.c_int, [P, P, P, C.c_uint32, C.c_uint32]),
    "hxq_cuda_decompress_vq2d_12bit": (C.c_int, [P, P, P, C.c_uint32, C.c_uint32]),
    "hxq_cuda_apply_sidecar": (C.c_float, [P, P, P, P, C.c_uint32, C.c_uint32]),
    "hxq_affine_group_matmul_bf16": (C.c_int, [P, C.POINTER(AffineTensor), P, C.c_uint32, P]),
    "hxq_affine_group_matmul_bf16_path": (C.c_int, [P, C.POINTER(AffineTensor), P, C.c_uint32, C.c_int, P]),
    "hxq_affine_group_matmul_bf16_auto_path": (C.c_int, [P, C.POINTER(AffineTensor), C.c_uint32]),
    "hxq_affine_group_matmul_async": (C.c_int, [P, C.POINTER(AffineTensor), P, C.c_uint32, P]),
    "hxq_cuda_affine_device_status": (C.c_int, []),
    "hxq_cuda_vq_matmul": (C.c_int, [P, P, C.c_uint32, P, C.c_uint32, P]),
    "hxq_cuda_image_create_ex": (C.c_int, [TP, C.c_uint32, C.c_uint32, C.c_uint32, C.POINTER(P)]),
    "hxq_cuda_vq_matmul_multi": (C.c_int, [P, P, C.c_uint32, C.POINTER(P), C.c_uint32, C.c_uint32, P]),
    "hxq_affine_group_matmul_bf16_multi": (C.c_int, [P, C.POINTER(AffineTensor), C.POINTER(P), C.c_uint32,
                                                     C.c_uint32, C.c_uint32, P]),
    "hxq_cuda_vq_matmul_batch": (C.c_int, [C.c_uint32, C.POINTER(P), C.POINTER(P), C.POINTER(P), C.c_uint32,
                                           C.POINTER(C.c_uint32), C.c_uint32, P]),
    "hxq_affine_group_matmul_bf16_batch": (C.c_int, [C.c_uint32, C.POINTER(AffineTensor), C.POINTER(P), C.POINTER(P),
                                                     C.c_uint32, C.POINTER(C.c_uint32), C.c_uint32, P]),
    "hxq_cuda_ipc_alloc": (C.c_int, [C.c_size_t, C.POINTER(P), P]),
    "hxq_cuda_ipc_open": (C.c_int, [P, C.POINTER(P)]),
    "hxq_cuda_ipc_close": (C.c_int, [P]),
    "hxq_cuda_ipc_free": (C.c_int, [P]),
    "hxq_cuda_peer_signal": (C.c_int, [C.POINTER(P), C.c_uint32, C.c_uint32, P, P]),
    "hxq_cuda_peer_wait": (C.c_int, [P, C.c_uint32, P, P, P]),
    "hxq_cuda_image_has_matmul_tables": (C.c_int, [P]),
    "hxq_cuda_vq_matmul_path": (C.c_int, [P, P, C.c_uint32, P, C.c_uint32, C.c_int, P]),
    # Lloyd's algorithm (hxq_lloyd.h, hxq_cuda.h)
    "hxq_lloyd_reassign": (C.c_int, [P, P, P, C.c_size_t, C.c_int, C.c_int, P]),
    "hxq_lloyd_assign_only": (C.c_int, [P, P, P, C.c_size_t, C.c_int, C.c_int]),
    "hxq_cuda_lloyd_assign": (C.c_int, [P, P, P, C.c_size_t, C.c_int, C.c_int, P]),
    "hxq_cuda_lloyd_reassign": (C.c_int, [P, P, P, C.c_size_t, C.c_int, C.c_int, P, P]),
    # PolarQuant (polarquant.h, hxq_cuda.h)
    "pq_generate_rotation": (C.c_int, [C.c_uint32, C.c_uint32, P]),
    "pq_rotate": (C.c_int, [P, P, C.c_uint32, C.c_uint32]),
    "pq_unrotate": (C.c_int, [P, P, C.c_uint32, C.c_uint32]),
    "pq_infer_head_geometry": (C.c_int, [C.c_uint32, C.c_uint32, P, P]),
    "pq_layer_init": (C.c_int, [P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]),
    "pq_layer_rotate": (C.c_int, [P, P]),
    "pq_layer_unrotate": (C.c_int, [P, P]),
    "pq_layer_free": (None, [P]),
    "hxq_cuda_pq_rotate": (C.c_int, [P, P, C.c_uint64, C.c_uint32, P]),
    "hxq_cuda_pq_unrotate": (C.c_int, [P, P, C.c_uint64, C.c_uint32, P]),
}


class PqLayer(C.Structure):
    """pq_layer_t (polarquant.h)."""
    _fields_ = [("Q", C.POINTER(C.c_float)), ("head_dim", C.c_uint32), ("n_heads", C.c_uint32),
                ("seed", C.c_uint32), ("initialized", C.c_int)]


def load(path: str = LIB_PATH) -> C.CDLL:
    """Load libhxq.so and declare every signature.  Raises if it is missing."""
    if not os.path.exists(path):
        raise RuntimeError(f"libhxq.so not built: {path} missing (run `make -C hxq-native_b200`)")
    lib = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_LIB = None


def lib() -> C.CDLL:
    global _LIB
    if _LIB is None:
        _LIB = load()
    return _LIB


def ptr(a) -> int | None:
    """Address of a numpy array, a torch tensor or an int (None stays None)."""
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    return a.data_ptr()  # torch tensor


def check(err: int, what: str = "") -> None:
    if err != HXQ_OK:
        msg = lib().hxq_error_string(err).decode()
        raise RuntimeError(f"{what}: hxq error {err} ({msg})")


class Tensor:
    """Owns an hxq_tensor_t and loads numpy arrays through the C loaders."""

    def __init__(self):
        self.t = HxqTensor()
        check(lib().hxq_tensor_init(C.byref(self.t)), "init")

    @property
    def ref(self):
        return C.byref(self.t)

    def load_codebook(self, cb: np.ndarray, k: int, vdim: int) -> int:
        cb = np.ascontiguousarray(cb, dtype=np.float32)
        return lib().hxq_tensor_load_codebook(self.ref, cb.ctypes.data, k, vdim)

    def load_indices_8bit(self, idx: np.ndarray, out_f: int, in_f: int) -> int:
        idx = np.ascontiguousarray(idx, dtype=np.uint8)
        return lib().hxq_tensor_load_indices_8bit(self.ref, idx.ctypes.data, out_f, in_f)

    def load_indices_12bit(self, packed: np.ndarray, out_f: int, in_f: int, length: int | None = None) -> int:
        packed = np.ascontiguousarray(packed, dtype=np.uint8)
        n = packed.size if length is None else length
        return lib().hxq_tensor_load_indices_12bit(self.ref, packed.ctypes.data, n, out_f, in_f)

    def load_sidecar(self, rows, cols, vals) -> int:
        rows = np.ascontiguousarray(rows, dtype=np.uint32)
        cols = np.ascontiguousarray(cols, dtype=np.uint32)
        vals = np.ascontiguousarray(vals, dtype=np.float32)
        return lib().hxq_tensor_load_sidecar(self.ref, rows.ctypes.data, cols.ctypes.data,
                                             vals.ctypes.data, rows.size)

    def load_affine(self, idx, scales, offsets, out_f, in_f, gs) -> int:
        idx = np.ascontiguousarray(idx, dtype=np.uint8)
        scales = np.ascontiguousarray(scales, dtype=np.float32)
        offsets = np.ascontiguousarray(offsets, dtype=np.float32)
        return lib().hxq_tensor_load_affine(self.ref, idx.ctypes.data, scales.ctypes.data,
                                            offsets.ctypes.data, out_f, in_f, gs)

    def load(self, d: dict) -> "Tensor":
        """Load a synthetic tensor dict produced by hxq_b200.synth."""
        if d["mode"] == HXQ_AFFINE_G128:
            check(self.load_affine(d["codes"], d["scales"], d["offsets"], d["out_f"], d["in_f"], d["gs"]), "affine")
        else:
            check(self.load_codebook(d["codebook"], d["k"], d["vdim"]), "codebook")
            if d["mode"] == HXQ_SCALAR_VQ:
                check(self.load_indices_8bit(d["indices"], d["out_f"], d["in_f"]), "idx8")
            else:
                check(self.load_indices_12bit(d["packed"], d["out_f"], d["in_f"]), "idx12")
        if d.get("rows") is not None and len(d["rows"]):
            check(self.load_sidecar(d["rows"], d["cols"], d["vals"]), "sidecar")
        return self

    @property
    def confidence(self) -> float:
        return self.t.sidecar_l2_norm

    def free(self):
        if self.t is not None:
            lib().hxq_tensor_free(self.ref)
            self.t = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class _DeviceView:
    def __init__(self, dptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr,
                                         "data": (int(dptr), False), "version": 2}


def device_view(torch, dptr: int, n: int, dtype=np.float32):
    """A torch CUDA tensor aliasing n elements at a raw device pointer
    (e.g. hxq_result_t.weights of a device arena)."""
    typestr = np.dtype(dtype).newbyteorder("<").str
    return torch.as_tensor(_DeviceView(dptr, n, typestr), device="cuda")


def header_functions(include_dir: str = INCLUDE_DIR) -> list[str]:
    """Names of the functions declared (non-inline) in include/*.h."""
    import re
    names = []
    for fn in sorted(os.listdir(include_dir)):
        if not fn.endswith(".h"):
            continue
        src = open(os.path.join(include_dir, fn)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"static inline[^{]*\{.*?\n\}", "", src, flags=re.S)
        for m in re.finditer(r"\b((?:hxq|pq)_[a-z0-9_]+)\s*\(", src):
            name = m.group(1)
            start = src.rfind("\n", 0, m.start()) + 1
            line = src[start:m.start()]
            if "#define" in line:
                continue
            if name not in names:
                names.append(name)
    return names
