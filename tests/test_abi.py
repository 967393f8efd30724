"""The drop-in boundary: libhxq.so loads, exports every function include/*.h
declares, keeps the reference struct layouts, and returns the reference's
status codes on the host-checked error paths.  No GPU needed."""
import ctypes as C
import os
import subprocess
import tempfile

import numpy as np
import pytest

from conftest import REPO


def test_library_exports_every_declared_function(H, L):
    names = H.header_functions()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    # every declared function has a ctypes signature in the binding
    assert not [n for n in names if n not in H.SIGNATURES]


def test_reference_symbols_present(L):
    # the reference's exported C symbols (hxq.h:111-333, hxq_affine.h:60-117,
    # hxq_affine_cuda.cu:252, hxq_cuda.cu:209-288)
    for n in ["hxq_tensor_init", "hxq_tensor_load_codebook", "hxq_tensor_load_indices_8bit",
              "hxq_tensor_load_indices_12bit", "hxq_tensor_load_affine", "hxq_tensor_load_sidecar",
              "hxq_tensor_decompress", "hxq_tensor_decompress_shared", "hxq_tensor_free",
              "hxq_shared_buffer_init", "hxq_shared_buffer_free", "hxq_dequant",
              "hxq_affine_group_matmul_ref", "hxq_affine_decompress_ref", "hxq_affine_group_matmul",
              "hxq_affine_matmul_flat", "hxq_cuda_decompress_scalar",
              "hxq_cuda_decompress_vq2d_12bit", "hxq_cuda_apply_sidecar"]:
        assert hasattr(L, n), n


def test_struct_layout_ctypes(H):
    assert C.sizeof(H.HxqTensor) == 96
    assert H.HxqTensor.mode.offset == 68
    assert H.HxqTensor.sidecar_l2_norm.offset == 92
    assert C.sizeof(H.SharedBuffer) == 24
    assert C.sizeof(H.Result) == 24
    assert C.sizeof(H.AffineTensor) == 48


@pytest.mark.parametrize("std", ["c99", "c11", "c++17"])
def test_headers_compile_with_layout_pins(std):
    src = r'''
#include "hxq.h"
#include "hxq_affine.h"
#include "hxq_cuda.h"
#include <stddef.h>
int main(void) {
    hxq_tensor_t t; hxq_shared_buffer_t b; hxq_result_t r; hxq_affine_tensor_t a;
    (void)t; (void)b; (void)r; (void)a;
    return (sizeof(hxq_tensor_t) == 96 && offsetof(hxq_tensor_t, sidecar_l2_norm) == 92 &&
            HXQ_BACKEND_CUDA == 2 && HXQ_VQ2D_12BIT == 2 && HXQ_ERR_PACK_FORMAT == 6) ? 0 : 1;
}
'''
    with tempfile.TemporaryDirectory() as d:
        ext = ".cpp" if "++" in std else ".c"
        path = os.path.join(d, "t" + ext)
        open(path, "w").write(src)
        cc = "g++" if "++" in std else "gcc"
        exe = os.path.join(d, "t")
        subprocess.run([cc, f"-std={std}", "-Wall", "-Werror", "-I", os.path.join(REPO, "include"),
                        path, "-o", exe], check=True)
        assert subprocess.run([exe]).returncode == 0


def test_loader_error_codes(H, L):
    t = H.Tensor()
    cb = np.zeros(4096 * 2, np.float32)
    assert L.hxq_tensor_init(None) == H.HXQ_ERR_NULL_PTR
    assert L.hxq_tensor_load_codebook(None, cb.ctypes.data, 256, 1) == H.HXQ_ERR_NULL_PTR
    assert L.hxq_tensor_load_codebook(t.ref, None, 256, 1) == H.HXQ_ERR_NULL_PTR
    for k in (0, 255, 512, 1024):
        assert t.load_codebook(cb, k, 1) == H.HXQ_ERR_INVALID_K
    for vdim in (0, 3):
        assert t.load_codebook(cb, 256, vdim) == H.HXQ_ERR_INVALID_DIM
    assert t.load_affine(np.zeros(8, np.uint8), np.ones(2, np.float32), np.zeros(2, np.float32), 2, 4, 0) \
        == H.HXQ_ERR_INVALID_DIM
    assert t.load_affine(np.zeros(8, np.uint8), np.ones(2, np.float32), np.zeros(2, np.float32), 2, 4, 3) \
        == H.HXQ_ERR_INVALID_DIM
    assert L.hxq_tensor_load_sidecar(None, None, None, None, 0) == H.HXQ_ERR_NULL_PTR
    assert L.hxq_tensor_load_sidecar(t.ref, None, None, None, 3) == H.HXQ_ERR_NULL_PTR


def test_decompress_error_codes(H, L):
    t = H.Tensor()
    out = np.zeros(16, np.float32)
    # nothing loaded
    assert L.hxq_tensor_decompress(t.ref, out.ctypes.data) == H.HXQ_ERR_NULL_PTR
    assert L.hxq_tensor_decompress(None, out.ctypes.data) == H.HXQ_ERR_NULL_PTR
    assert L.hxq_tensor_decompress(t.ref, None) == H.HXQ_ERR_NULL_PTR
    assert t.load_indices_8bit(np.zeros(16, np.uint8), 4, 4) == 0
    assert L.hxq_tensor_decompress(t.ref, out.ctypes.data) == H.HXQ_ERR_NULL_PTR  # no codebook
    assert t.load_codebook(np.zeros(256, np.float32), 256, 1) == 0
    t.t.mode = H.HXQ_VQ2D_8BIT  # declared, not implemented (src/hxq.c:376-377)
    assert L.hxq_tensor_decompress(t.ref, out.ctypes.data) == H.HXQ_ERR_INVALID_DIM
    t.t.mode = 7
    assert L.hxq_tensor_decompress(t.ref, out.ctypes.data) == H.HXQ_ERR_INVALID_DIM


def test_dequant_backend_policy(H, L):
    t = H.Tensor()
    assert t.load_codebook(np.arange(256, dtype=np.float32), 256, 1) == 0
    assert t.load_indices_8bit(np.arange(6, dtype=np.uint8), 2, 3) == 0
    buf = H.SharedBuffer()
    assert L.hxq_shared_buffer_init(C.byref(buf), 4) == 0
    r = H.Result()
    assert L.hxq_dequant(None, C.byref(buf), 0, C.byref(r)) == H.HXQ_ERR_NULL_PTR
    assert L.hxq_dequant(t.ref, C.byref(buf), H.HXQ_BACKEND_METAL, C.byref(r)) == H.HXQ_ERR_BACKEND_UNAVAILABLE
    assert L.hxq_dequant(t.ref, C.byref(buf), H.HXQ_BACKEND_VULKAN, C.byref(r)) == H.HXQ_ERR_BACKEND_UNAVAILABLE
    assert L.hxq_cuda_buffer_is_device(C.byref(buf)) == 0
    for backend in (H.HXQ_BACKEND_AUTO, H.HXQ_BACKEND_CPU):  # host buffer -> CPU backend
        assert L.hxq_dequant(t.ref, C.byref(buf), backend, C.byref(r)) == 0
        w = np.ctypeslib.as_array(C.cast(r.weights, C.POINTER(C.c_float)), shape=(6,))
        assert list(w) == [0, 1, 2, 3, 4, 5]
    assert buf.capacity == 6 and buf.high_water == 6
    L.hxq_shared_buffer_free(C.byref(buf))
    assert buf.data is None and buf.capacity == 0


def test_error_strings(H, L):
    for code in list(range(8)) + [32, 33, 34, 35]:
        assert L.hxq_error_string(code)
    assert b"sm_100a" in L.hxq_b200_version()


def test_cuda_entry_points_without_gpu(H, L):
    """Without a device the CUDA backend reports it; it never computes on the CPU."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert L.hxq_cuda_device_count() == 0
    t = H.Tensor()
    assert t.load_codebook(np.zeros(256, np.float32), 256, 1) == 0
    assert t.load_indices_8bit(np.zeros(4, np.uint8), 2, 2) == 0
    buf = H.SharedBuffer()
    assert L.hxq_shared_buffer_init(C.byref(buf), 4) == 0
    r = H.Result()
    assert L.hxq_dequant(t.ref, C.byref(buf), H.HXQ_BACKEND_CUDA, C.byref(r)) == H.HXQ_ERR_BACKEND_UNAVAILABLE
    assert L.hxq_cuda_arena_init(C.byref(H.SharedBuffer()), 16) == H.HXQ_ERR_BACKEND_UNAVAILABLE
    img = C.c_void_p()
    assert L.hxq_cuda_image_create(t.ref, 0, 2, C.byref(img)) == H.HXQ_ERR_BACKEND_UNAVAILABLE
    assert L.hxq_affine_matmul_flat(None, None, None, None, None, None, 1, 128, 1, 128) == -1
    assert L.hxq_cuda_vq_matmul(None, None, 1, None, 1, None) == H.HXQ_ERR_NULL_PTR
    L.hxq_shared_buffer_free(C.byref(buf))
