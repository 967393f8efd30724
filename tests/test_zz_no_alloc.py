"""The decompress entry point that allocates nothing
(hxq_cuda_decompress_images_noalloc), for callers that cannot let a library
call cudaMalloc (engines that pre-plan all of HBM, latency-critical serving
loops).  It must give exactly what the regular batched entry point gives,
call after call, while its scratch lives in one fixed array shared by all
calls.  Collected last on purpose (file name), so a failure here cannot stop
the rest of the suite; it also passes when run alone in a fresh process.
"""
import ctypes as C
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from hxq_b200 import synth

pytestmark = pytest.mark.gpu


def _image(H, L, d):
    t = H.Tensor().load(d)
    img = C.c_void_p()
    assert L.hxq_cuda_image_create(t.ref, 0, d["out_f"], C.byref(img)) == 0
    return t, img


def _run(torch, L, fn, imgs, offs, total, dtype, n):
    elem_t = torch.float32 if dtype == 0 else torch.bfloat16
    out = torch.full((total,), float("nan"), dtype=elem_t, device="cuda")
    sumsq = torch.full((n,), -1.0, dtype=torch.float64, device="cuda")
    conf = torch.full((n,), -1.0, dtype=torch.float32, device="cuda")
    arr = (C.c_void_p * n)(*[i.value for i in imgs])
    offs_c = (C.c_size_t * n)(*offs)
    torch.cuda.synchronize()
    err = fn(arr, n, out.data_ptr(), offs_c, dtype, sumsq.data_ptr(), conf.data_ptr(), None)
    return err, out, sumsq, conf


def test_noalloc_matches_regular_entry_point_twice(H, L, cuda):
    torch = cuda
    ds = [synth.vq12(512, 2048, 41), synth.vq12(128, 1024, 42, k=256), synth.scalar(300, 600, 43, frac=0.01),
          synth.vq12(2048, 4096, 44), synth.scalar(7, 5, 45, frac=0.3)]
    pairs = [_image(H, L, d) for d in ds]
    imgs = [img for _, img in pairs]
    sizes = [d["out_f"] * d["in_f"] for d in ds]
    offs, pos = [], 0
    for n_el in sizes:
        offs.append(pos)
        pos += (n_el + 7) // 8 * 8
    for dtype in (H.HXQ_OUT_F32, H.HXQ_OUT_BF16):
        err, ref_out, ref_ss, ref_cf = _run(torch, L, L.hxq_cuda_decompress_images, imgs, offs, pos, dtype, len(ds))
        assert err == 0 and L.hxq_cuda_stream_synchronize(None) == 0
        ref_bits = ref_out.view(torch.int16 if dtype else torch.int32).cpu().numpy()
        for call in range(2):  # the shared scratch keeps the last call's contents
            err, out, ss, cf = _run(torch, L, L.hxq_cuda_decompress_images_noalloc, imgs, offs, pos, dtype, len(ds))
            assert err == 0, (dtype, call, err)
            bits = out.view(torch.int16 if dtype else torch.int32).cpu().numpy()
            for i, n_el in enumerate(sizes):  # compare each image's slot (padding stays NaN in both)
                assert np.array_equal(bits[offs[i]: offs[i] + n_el], ref_bits[offs[i]: offs[i] + n_el]), (dtype, call, i)
            assert np.array_equal(ss.cpu().numpy(), ref_ss.cpu().numpy())
            assert np.array_equal(cf.cpu().numpy(), ref_cf.cpu().numpy())
    for img in imgs:
        L.hxq_cuda_image_destroy(img)


def test_noalloc_rejects_beyond_its_fixed_scratch(H, L, cuda):
    torch = cuda
    # one 4096 x 4096 matrix is 8192 chunks = 512 units; 17 copies need 8704
    # units, more than the 8192 the fixed scratch holds
    d = synth.vq12(4096, 4096, 46, frac=0.0)
    t, img = _image(H, L, d)
    n = 17
    arr = (C.c_void_p * n)(*([img.value] * n))
    offs = (C.c_size_t * n)(*([0] * n))
    out = torch.empty(4096 * 4096, dtype=torch.float32, device="cuda")
    assert L.hxq_cuda_decompress_images_noalloc(arr, n, out.data_ptr(), offs, H.HXQ_OUT_F32, None, None,
                                                None) == H.HXQ_ERR_INVALID_ARG
    # 16 copies (8192 units) is exactly the limit and runs
    assert L.hxq_cuda_decompress_images_noalloc(arr, 16, out.data_ptr(), offs, H.HXQ_OUT_F32, None, None,
                                                None) == 0
    # an unaligned output slot is refused up front as well
    assert L.hxq_cuda_decompress_images_noalloc(arr, 1, out.data_ptr() + 4, offs, H.HXQ_OUT_F32, None, None,
                                                None) == H.HXQ_ERR_INVALID_ARG
    L.hxq_cuda_image_destroy(img)


# Run in a fresh process: after one warm-up call (which looks up the array's
# address and loads the kernels), calls on a stream the library has never
# seen must leave the device's free memory unchanged.  The regular entry
# point would cudaMalloc reduction scratch for that new stream.
_NO_ALLOC_PROBE = textwrap.dedent("""
    import ctypes as C, sys
    import torch
    sys.path[:0] = [REPO, PKG]
    import hxq_b200 as H
    from hxq_b200 import synth
    torch.cuda.init()
    L = H.lib()
    ds = [synth.vq12(512, 2048, 51), synth.scalar(256, 512, 52, frac=0.01)]
    ts = [H.Tensor().load(d) for d in ds]
    imgs = []
    for t, d in zip(ts, ds):
        img = C.c_void_p()
        assert L.hxq_cuda_image_create(t.ref, 0, d["out_f"], C.byref(img)) == 0
        imgs.append(img)
    offs = [0, 512 * 2048]
    out = torch.empty(512 * 2048 + 256 * 512, dtype=torch.float32, device="cuda")
    ss = torch.empty(2, dtype=torch.float64, device="cuda")
    cf = torch.empty(2, dtype=torch.float32, device="cuda")
    arr = (C.c_void_p * 2)(*[i.value for i in imgs])
    offs_c = (C.c_size_t * 2)(*offs)
    def call(stream):
        return L.hxq_cuda_decompress_images_noalloc(arr, 2, out.data_ptr(), offs_c, 0, ss.data_ptr(),
                                                    cf.data_ptr(), stream.cuda_stream)
    warm = torch.cuda.Stream()
    assert call(warm) == 0
    torch.cuda.synchronize()
    same = 0
    for trial in range(3):
        fresh = torch.cuda.Stream()
        before = torch.cuda.mem_get_info()[0]
        for _ in range(3):
            assert call(fresh) == 0
        torch.cuda.synchronize()
        after = torch.cuda.mem_get_info()[0]
        print("free bytes", before, after)
        same += before == after
    print("NOALLOC_OK" if same >= 1 else "NOALLOC_CHANGED")
""")


def test_noalloc_allocates_no_device_memory(H, cuda):
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    pkg = os.path.join(repo, "hxq-native_b200")
    code = "REPO = %r\nPKG = %r\n" % (repo, pkg) + _NO_ALLOC_PROBE
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "NOALLOC_OK" in r.stdout, r.stdout
