"""Fused VQ-dequant matmul on the GPU against the oracle.

The reference library has no fused VQ matmul; its result is defined as the
reference decompress (hxq.c, restated bit-exactly by the oracle) followed by
the naive ordered fp32 matmul of test/test_affine.c:51-65 (oracle
dense_matmul).  Errors are normalised per output by sum_i |x_i * w_i|, the
natural scale of an fp32 dot product's rounding error:
  * GEMV (few tokens): exact fp32 weights, tolerance 1e-5 (fp32 paths);
  * tcgen05 GEMM: weights rounded to bf16, tolerance 2^-9 + 1e-5 (inside
    the 1e-2 allowed for bf16 paths), and 1e-4 against a float64 product
    with the kernel's own weights bf16(W) -- which pins the layout.
All calls go through the C ABI of libhxq.so.
"""
import ctypes as C

import numpy as np
import pytest

from hxq_b200 import synth

pytestmark = pytest.mark.gpu
TOL = 1e-5
GEMM_TOL = 2.0 ** -9 + 1e-5


def _scale(x, W):
    return np.abs(x.astype(np.float64)) @ np.abs(W.astype(np.float64)).T


def _check(y, y_ref, scale, tol):
    err = np.abs(y.astype(np.float64) - y_ref.astype(np.float64)) / np.maximum(scale, 1e-30)
    assert float(err.max()) <= tol, float(err.max())


def _image(H, L, t, r0, r1, matmul=True):
    img = C.c_void_p()
    flags = H.HXQ_IMAGE_MATMUL if matmul else 0
    assert L.hxq_cuda_image_create_ex(t.ref, r0, r1, flags, C.byref(img)) == 0
    return img


def _run(torch, L, img, xh, rows, path=None, ldy=None, col0=0):
    N = xh.shape[0]
    ldy = rows if ldy is None else ldy
    xd = torch.from_numpy(np.ascontiguousarray(xh.view(np.int16))).cuda()
    y = torch.full((N, ldy), float("nan"), dtype=torch.float32, device="cuda")
    yp = y.data_ptr() + 4 * col0
    torch.cuda.synchronize()
    if path is None:
        assert L.hxq_cuda_vq_matmul(img, xd.data_ptr(), N, yp, ldy, None) == 0
    else:
        assert L.hxq_cuda_vq_matmul_path(img, xd.data_ptr(), N, yp, ldy, path, None) == 0
    torch.cuda.synchronize()
    return y.cpu().numpy()


def _with_dups_and_oob(d, seed):
    """Append repeated coordinates (summed in array order) and entries the
    reference skips (row >= out_f or col >= in_f)."""
    rng = np.random.default_rng(seed)
    n = len(d["rows"])
    pick = rng.integers(0, n, size=min(n, 8))
    rows = np.concatenate([d["rows"], d["rows"][pick], np.array([d["out_f"], 0], np.uint32)])
    cols = np.concatenate([d["cols"], d["cols"][pick], np.array([0, d["in_f"]], np.uint32)])
    vals = np.concatenate([d["vals"], (rng.standard_normal(len(pick)) * 0.01).astype(np.float32),
                           np.array([5.0, 5.0], np.float32)])
    d = dict(d)
    d["rows"], d["cols"], d["vals"] = rows.astype(np.uint32), cols.astype(np.uint32), vals.astype(np.float32)
    return d


def _case(oracle, out_f, in_f, N, seed, frac=0.005, dups=False):
    d = synth.vq12(out_f, in_f, seed, frac=frac)
    if dups:
        d = _with_dups_and_oob(d, seed)
    err, w, _ = oracle.decompress(d)
    assert err == 0
    W = w.reshape(out_f, in_f)
    xh, x = synth.activations(N, in_f, seed + 1)
    return d, W, xh, x


@pytest.mark.parametrize("out_f,in_f,N", [(256, 512, 1), (256, 512, 2), (300, 1024, 3), (37, 64, 4),
                                          (100, 192, 16), (4096, 4096, 1), (11008, 4096, 1), (4096, 11008, 2),
                                          (513, 2048, 8), (64, 4096, 5)])
def test_gemv_vs_oracle(H, L, oracle, cuda, out_f, in_f, N):
    d, W, xh, x = _case(oracle, out_f, in_f, N, out_f * 3 + in_f + N, dups=True)
    t = H.Tensor().load(d)
    img = _image(H, L, t, 0, out_f)
    try:
        y = _run(cuda, L, img, xh, out_f, path=0)
    finally:
        L.hxq_cuda_image_destroy(img)
    _check(y, oracle.dense_matmul(x, W), _scale(x, W), TOL)


@pytest.mark.parametrize("out_f,in_f,N", [(256, 512, 5), (129, 128, 16), (300, 1024, 33), (4096, 4096, 16),
                                          (1024, 2048, 100), (256, 384, 257), (11008, 4096, 16),
                                          (4096, 11008, 16), (200, 256, 2), (1024, 4096, 256), (513, 2048, 24)])
def test_gemm_vs_oracle(H, L, oracle, cuda, out_f, in_f, N):
    """The tcgen05 GEMM (path 1): token tiles of 16 to 256 (256 with the A
    tiles in shared memory), ragged rows and tiles, split K
    (1024 x 4096 at 256 tokens: 256-token tiles in 16 splits), repeated and
    out-of-range sidecar entries."""
    d, W, xh, x = _case(oracle, out_f, in_f, N, out_f * 7 + in_f + N, dups=True)
    t = H.Tensor().load(d)
    img = _image(H, L, t, 0, out_f)
    try:
        y = _run(cuda, L, img, xh, out_f, path=1)
    finally:
        L.hxq_cuda_image_destroy(img)
    assert L.hxq_cuda_affine_device_status() == 0
    sc = _scale(x, W)
    _check(y, oracle.dense_matmul(x, W), sc, GEMM_TOL)
    # the kernel's own weights: one rounding of the fp32 (sidecar-corrected) weight
    Wb = synth.bf16_to_f32(synth.bf16_round(W)).reshape(out_f, in_f)
    _check(y, oracle.dense_matmul_f64(x, Wb), sc, 1e-4)


def test_gemm_last_wave_split(H, L, oracle, cuda):
    """2400 x 2048 at 2000 tokens: 152 tiles of 128 x 256 on 148 SMs; the
    last 4 (ragged rows and tokens) are split along K into 4 ranges added in
    order by the last arriving CTA.  Sampled token rows cover whole and split
    tiles; repeated and out-of-range sidecar entries; the same result on
    every run."""
    out_f, in_f, N = 2400, 2048, 2000
    d = synth.vq12(out_f, in_f, 2402)
    d = _with_dups_and_oob(d, 2402)
    err, w, _ = oracle.decompress(d)
    assert err == 0
    W = w.reshape(out_f, in_f)
    xh, x = synth.activations(N, in_f, 2403)
    t = H.Tensor().load(d)
    img = _image(H, L, t, 0, out_f)
    try:
        y = _run(cuda, L, img, xh, out_f, path=1)
        y2 = _run(cuda, L, img, xh, out_f, path=1)
    finally:
        L.hxq_cuda_image_destroy(img)
    assert L.hxq_cuda_affine_device_status() == 0
    assert np.array_equal(y, y2)
    Wb = synth.bf16_to_f32(synth.bf16_round(W)).reshape(out_f, in_f)
    rows = [0, 1000, 1791, 1792, 1900, 1999]
    xs = x[rows]
    sc = _scale(xs, W)
    _check(y[rows], oracle.dense_matmul(xs, W), sc, GEMM_TOL)
    _check(y[rows], oracle.dense_matmul_f64(xs, Wb), sc, 1e-4)


@pytest.mark.parametrize("out_f,in_f,N", [(256, 512, 1), (256, 512, 2), (300, 1024, 3), (17, 128, 7), (4096, 4096, 1),
                                          (11008, 4096, 1), (4096, 11008, 2), (513, 2048, 8), (64, 4096, 5),
                                          (256, 512, 9), (300, 1024, 12), (17, 128, 16), (4096, 4096, 16),
                                          (4096, 11008, 8), (300, 11008, 12), (4096, 11008, 13), (77, 9856, 12)])
def test_tc_gemv_vs_oracle(H, L, oracle, cuda, out_f, in_f, N):
    """The tensor-core GEMV (path 2), one and two 8-token tiles: ragged row
    blocks, index rows that are not a multiple of 128 bytes (128: 96-byte
    rows; 11008: 8256), a partial last stage, repeated and out-of-range
    sidecar entries; within the bf16-weight bound of the oracle, and within
    1e-4 of a float64 product with the kernel's own weights (bf16 of each
    final weight).  Activations too wide for the staging (11008 from 8
    tokens, 9856 at 12) run as two K parts of whole 128-column windows, the
    second one shorter where the windows are odd (9856: 4992, 4864), whose
    partial products a second kernel adds."""
    d, W, xh, x = _case(oracle, out_f, in_f, N, out_f * 11 + in_f + N, dups=True)
    t = H.Tensor().load(d)
    img = _image(H, L, t, 0, out_f)
    try:
        y = _run(cuda, L, img, xh, out_f, path=2)
    finally:
        L.hxq_cuda_image_destroy(img)
    assert L.hxq_cuda_affine_device_status() == 0
    sc = _scale(x, W)
    _check(y, oracle.dense_matmul(x, W), sc, GEMM_TOL)
    Wb = synth.bf16_to_f32(synth.bf16_round(W)).reshape(out_f, in_f)
    _check(y, oracle.dense_matmul_f64(x, Wb), sc, 1e-4)


def test_c5_prefill_2048_sampled(H, L, oracle, cuda):
    """The prefill batch of the fused-matmul sweep on a 4096 x 4096 layer
    matrix; outputs checked for a seeded sample of tokens."""
    d, W, xh, x = _case(oracle, 4096, 4096, 2048, synth.SEED_C5)
    t = H.Tensor().load(d)
    img = _image(H, L, t, 0, 4096)
    try:
        y = _run(cuda, L, img, xh, 4096)          # default path: GEMM
    finally:
        L.hxq_cuda_image_destroy(img)
    assert L.hxq_cuda_affine_device_status() == 0
    for n in sorted({0, 1, 777, 1024, 2046, 2047}):
        ref = oracle.dense_matmul(x, W, n0=n, n1=n + 1)
        _check(y[n:n + 1], ref, _scale(x[n:n + 1], W), GEMM_TOL)


def test_default_path_choice(H, L, oracle, cuda):
    """With matmul tables, up to 16 tokens take the tensor-core GEMV and more
    the GEMM; without tables, the exact GEMV: each bit-identical to its
    explicit path."""
    d, W, xh, x = _case(oracle, 512, 1024, 17, 99)
    t = H.Tensor().load(d)
    img = _image(H, L, t, 0, 512)
    plain = _image(H, L, t, 0, 512, matmul=False)
    try:
        for n, path in ((4, 2), (8, 2), (9, 2), (16, 2), (17, 1)):
            y_default = _run(cuda, L, img, xh[:n], 512)
            y_path = _run(cuda, L, img, xh[:n], 512, path=path)
            assert np.array_equal(y_default.view(np.uint32), y_path.view(np.uint32)), n
        y_default = _run(cuda, L, plain, xh[:4], 512)
        y_gemv = _run(cuda, L, plain, xh[:4], 512, path=0)
        assert np.array_equal(y_default.view(np.uint32), y_gemv.view(np.uint32))
    finally:
        L.hxq_cuda_image_destroy(img)
        L.hxq_cuda_image_destroy(plain)


@pytest.mark.parametrize("path", [0, 1, 2])
def test_row_shards_into_column_slices(H, L, oracle, cuda, path):
    """An image of rows [r0, r1) writes output columns r0..r1 of a wider
    [N, ldy] matrix (the column-sharded layout); nothing else is touched."""
    out_f, in_f, N = 1000, 1024, 6
    d, W, xh, x = _case(oracle, out_f, in_f, N, 4242, dups=True)
    t = H.Tensor().load(d)
    ref = oracle.dense_matmul(x, W)
    sc = _scale(x, W)
    tol = TOL if path == 0 else GEMM_TOL
    for r0, r1 in ((0, 250), (250, 600), (600, 1000), (999, 1000)):
        img = _image(H, L, t, r0, r1)
        try:
            y = _run(cuda, L, img, xh, r1 - r0, path=path, ldy=out_f + 3, col0=r0)
        finally:
            L.hxq_cuda_image_destroy(img)
        assert np.isnan(y[:, :r0]).all() and np.isnan(y[:, r1:]).all()
        _check(y[:, r0:r1], ref[:, r0:r1], sc[:, r0:r1], tol)
    assert L.hxq_cuda_affine_device_status() == 0


@pytest.mark.parametrize("path", [0, 1, 2])
def test_dense_sidecar_rows(H, L, oracle, cuda, path):
    """Rows with many patches in one K step (more than the four a converter
    prefetches), repeated coordinates summed in array order, and a row whose
    every weight is corrected."""
    out_f, in_f, N = 256, 1024, 8
    d = synth.vq12(out_f, in_f, 31, frac=0.002)
    rng = np.random.default_rng(3)
    extra_r = np.concatenate([np.full(40, 5), np.full(in_f, 130), np.full(12, 255)]).astype(np.uint32)
    extra_c = np.concatenate([np.arange(40) * 3, np.arange(in_f), rng.integers(0, 64, 12)]).astype(np.uint32)
    extra_v = (rng.standard_normal(len(extra_r)) * 0.01).astype(np.float32)
    d["rows"] = np.concatenate([d["rows"], extra_r, extra_r[:40]])
    d["cols"] = np.concatenate([d["cols"], extra_c, extra_c[:40]])
    d["vals"] = np.concatenate([d["vals"], extra_v, extra_v[:40] * np.float32(-0.5)])
    err, w, _ = oracle.decompress(d)
    assert err == 0
    W = w.reshape(out_f, in_f)
    xh, x = synth.activations(N, in_f, 8)
    t = H.Tensor().load(d)
    img = _image(H, L, t, 0, out_f)
    try:
        assert L.hxq_cuda_image_has_matmul_tables(img) == 1
        y = _run(cuda, L, img, xh, out_f, path=path)
    finally:
        L.hxq_cuda_image_destroy(img)
    sc = _scale(x, W)
    _check(y, oracle.dense_matmul(x, W), sc, TOL if path == 0 else GEMM_TOL)
    if path != 0:
        Wb = synth.bf16_to_f32(synth.bf16_round(W)).reshape(out_f, in_f)
        _check(y, oracle.dense_matmul_f64(x, Wb), sc, 1e-4)


def test_no_sidecar_and_zero_tokens(H, L, oracle, cuda):
    d, W, xh, x = _case(oracle, 128, 256, 3, 7, frac=0.0)
    assert len(d["rows"]) == 0
    t = H.Tensor().load(d)
    img = _image(H, L, t, 0, 128)
    try:
        for path in (0, 1, 2):
            _check(_run(cuda, L, img, xh, 128, path=path), oracle.dense_matmul(x, W), _scale(x, W),
                   TOL if path == 0 else GEMM_TOL)
        y = cuda.full((1, 128), 7.0, device="cuda")
        xd = cuda.zeros((1, 256), dtype=cuda.int16, device="cuda")
        assert L.hxq_cuda_vq_matmul(img, xd.data_ptr(), 0, y.data_ptr(), 128, None) == 0
        cuda.cuda.synchronize()
        assert bool((y == 7.0).all())
    finally:
        L.hxq_cuda_image_destroy(img)


def test_invalid_images_and_arguments(H, L, cuda):
    xd = cuda.zeros((4, 4096), dtype=cuda.int16, device="cuda")
    y = cuda.zeros((4, 4096), dtype=cuda.float32, device="cuda")
    cases = [synth.scalar(64, 128, 1),          # not 12-bit VQ
             synth.vq12(64, 128, 2, k=256),     # k != 4096
             synth.vq12(64, 96, 3)]             # in_f % 64 != 0
    for d in cases:
        t = H.Tensor().load(d)
        img = _image(H, L, t, 0, d["out_f"])
        try:
            assert L.hxq_cuda_vq_matmul(img, xd.data_ptr(), 1, y.data_ptr(), 4096, None) == H.HXQ_ERR_INVALID_ARG
        finally:
            L.hxq_cuda_image_destroy(img)
    d = synth.vq12(64, 192, 4)                  # in_f % 128 != 0: no matmul tables, GEMV only
    t = H.Tensor().load(d)
    img = _image(H, L, t, 0, 64)
    plain = _image(H, L, H.Tensor().load(synth.vq12(64, 256, 5)), 0, 64, matmul=False)
    try:
        assert L.hxq_cuda_image_has_matmul_tables(img) == 0
        assert L.hxq_cuda_image_has_matmul_tables(plain) == 0
        assert L.hxq_cuda_vq_matmul_path(img, xd.data_ptr(), 8, y.data_ptr(), 64, 1, None) == H.HXQ_ERR_INVALID_ARG
        assert L.hxq_cuda_vq_matmul_path(plain, xd.data_ptr(), 8, y.data_ptr(), 64, 1, None) == H.HXQ_ERR_INVALID_ARG
        assert L.hxq_cuda_vq_matmul_path(plain, xd.data_ptr(), 4, y.data_ptr(), 64, 2, None) == H.HXQ_ERR_INVALID_ARG
        assert L.hxq_cuda_vq_matmul_path(plain, xd.data_ptr(), 4, y.data_ptr(), 64, 3, None) == H.HXQ_ERR_INVALID_ARG
        assert L.hxq_cuda_vq_matmul(plain, xd.data_ptr(), 8, y.data_ptr(), 64, None) == 0   # takes the GEMV
        assert L.hxq_cuda_vq_matmul(img, xd.data_ptr(), 8, y.data_ptr(), 63, None) == H.HXQ_ERR_INVALID_ARG
        assert L.hxq_cuda_vq_matmul(img, xd.data_ptr() + 2, 1, y.data_ptr(), 64, None) == H.HXQ_ERR_INVALID_ARG
        assert L.hxq_cuda_vq_matmul(img, None, 1, y.data_ptr(), 64, None) == H.HXQ_ERR_NULL_PTR
        assert L.hxq_cuda_vq_matmul(img, xd.data_ptr(), 8, y.data_ptr(), 64, None) == 0
    finally:
        L.hxq_cuda_image_destroy(img)
        L.hxq_cuda_image_destroy(plain)
    cuda.cuda.synchronize()
    bad = C.c_void_p()
    assert L.hxq_cuda_image_create_ex(t.ref, 0, 64, 8, C.byref(bad)) == H.HXQ_ERR_INVALID_ARG


@pytest.mark.parametrize("N", [1, 3, 5, 8, 16])
def test_batch_of_layer_projections(H, L, oracle, cuda, N):
    """A layer's projections (row shards of 7B shapes) in one batch call, two
    outputs each at a column offset: bit-identical to one call per image on
    the same path.  From 3 tokens the 11008-wide matrix's activations leave
    one CTA per SM, so the batch splits into two tensor-core launches; from
    8 to 13 tokens that matrix runs as two K parts sharing the first launch,
    added by a part-sum kernel; at 16 it would need three, so it takes the
    GEMM."""
    torch = cuda
    shapes = [(512, 4096), (256, 4096), (384, 4096), (512, 4096), (1376, 4096), (1376, 4096), (512, 11008)]
    imgs, xs, refs, outs = [], [], [], []
    try:
        for i, (O, I) in enumerate(shapes):
            d = _with_dups_and_oob(synth.vq12(O, I, 300 + i), 300 + i)
            t = H.Tensor().load(d)
            img = _image(H, L, t, 0, O)
            imgs.append((img, t))
            xh, _ = synth.activations(N, I, 400 + i)
            x = torch.from_numpy(np.ascontiguousarray(xh.view(np.int16))).cuda()
            ref = torch.empty((N, O), dtype=torch.float32, device="cuda")
            # the batch takes the tensor-core GEMV up to 16 tokens where it fits
            if N > 16 or L.hxq_cuda_vq_matmul_path(img, x.data_ptr(), N, ref.data_ptr(), O, 2, None) != 0:
                assert L.hxq_cuda_vq_matmul(img, x.data_ptr(), N, ref.data_ptr(), O, None) == 0
            xs.append(x); refs.append(ref)
            outs.append([torch.full((N, O + 32), float("nan"), dtype=torch.float32, device="cuda") for _ in range(2)])
        n = len(shapes)
        IM = (C.c_void_p * n)(*[im.value for im, _ in imgs])
        X = (C.c_void_p * n)(*[x.data_ptr() for x in xs])
        Y = (C.c_void_p * (2 * n))(*[o.data_ptr() + 4 * 16 for pair in outs for o in pair])
        LD = (C.c_uint32 * n)(*[O + 32 for O, _ in shapes])
        assert L.hxq_cuda_vq_matmul_batch(n, IM, X, Y, 2, LD, N, None) == 0
        torch.cuda.synchronize()
        for (O, _), ref, pair in zip(shapes, refs, outs):
            for o in pair:
                assert torch.equal(o[:, 16:16 + O].contiguous().view(torch.int32), ref.view(torch.int32))
                assert bool(torch.isnan(o[:, :16]).all()) and bool(torch.isnan(o[:, 16 + O:]).all())
        assert L.hxq_cuda_affine_device_status() == 0
    finally:
        for im, _ in imgs:
            L.hxq_cuda_image_destroy(im)


def test_batch_chained_gemms(H, L, oracle, cuda):
    """A prefill batch whose GEMMs are unsplit (4096 x 256 images at 2048
    tokens: 256 tiles each), so each one after the first is chained to the
    one before it: every output bit-identical to one call per image."""
    torch = cuda
    N, shapes = 2048, [(4096, 256)] * 3
    imgs, xs, refs, outs = [], [], [], []
    try:
        for i, (O, I) in enumerate(shapes):
            d = _with_dups_and_oob(synth.vq12(O, I, 900 + i), 900 + i)
            t = H.Tensor().load(d)
            img = _image(H, L, t, 0, O)
            imgs.append((img, t))
            xh, _ = synth.activations(N, I, 950 + i)
            x = torch.from_numpy(np.ascontiguousarray(xh.view(np.int16))).cuda()
            ref = torch.empty((N, O), dtype=torch.float32, device="cuda")
            assert L.hxq_cuda_vq_matmul(img, x.data_ptr(), N, ref.data_ptr(), O, None) == 0
            xs.append(x); refs.append(ref)
            outs.append(torch.full((N, O), float("nan"), dtype=torch.float32, device="cuda"))
        n = len(shapes)
        IM = (C.c_void_p * n)(*[im.value for im, _ in imgs])
        X = (C.c_void_p * n)(*[x.data_ptr() for x in xs])
        Y = (C.c_void_p * n)(*[o.data_ptr() for o in outs])
        LD = (C.c_uint32 * n)(*[O for O, _ in shapes])
        for _ in range(2):
            assert L.hxq_cuda_vq_matmul_batch(n, IM, X, Y, 1, LD, N, None) == 0
            total = sum(o.sum() for o in outs)   # reads every output after the batch
            torch.cuda.synchronize()
            assert torch.isfinite(total)
            for ref, o in zip(refs, outs):
                assert torch.equal(o.view(torch.int32), ref.view(torch.int32))
            for o in outs:
                o.fill_(float("nan"))
        assert L.hxq_cuda_affine_device_status() == 0
    finally:
        for im, _ in imgs:
            L.hxq_cuda_image_destroy(im)


def test_batch_chain_breaks_at_other_kernels(H, L, oracle, cuda):
    """Prefill batch of GEMM images with an image without matmul tables
    between them (it takes the exact GEMV): the chain of GEMMs breaks there,
    so the GEMM after the GEMV waits for it; every output bit-identical to
    one call per image, over several repetitions."""
    torch = cuda
    N = 2048
    specs = [(4096, 256, True), (4096, 256, True), (512, 256, False), (4096, 256, True), (4096, 256, True)]
    imgs, xs, refs, outs = [], [], [], []
    try:
        for i, (O, I, mm) in enumerate(specs):
            d = _with_dups_and_oob(synth.vq12(O, I, 1200 + i), 1200 + i)
            t = H.Tensor().load(d)
            img = _image(H, L, t, 0, O, matmul=mm)
            imgs.append((img, t))
            xh, _ = synth.activations(N, I, 1300 + i)
            x = torch.from_numpy(np.ascontiguousarray(xh.view(np.int16))).cuda()
            ref = torch.empty((N, O), dtype=torch.float32, device="cuda")
            assert L.hxq_cuda_vq_matmul(img, x.data_ptr(), N, ref.data_ptr(), O, None) == 0
            xs.append(x); refs.append(ref)
            outs.append(torch.full((N, O), float("nan"), dtype=torch.float32, device="cuda"))
        n = len(specs)
        IM = (C.c_void_p * n)(*[im.value for im, _ in imgs])
        X = (C.c_void_p * n)(*[x.data_ptr() for x in xs])
        Y = (C.c_void_p * n)(*[o.data_ptr() for o in outs])
        LD = (C.c_uint32 * n)(*[O for O, _, _ in specs])
        for _ in range(3):
            assert L.hxq_cuda_vq_matmul_batch(n, IM, X, Y, 1, LD, N, None) == 0
            torch.cuda.synchronize()
            for ref, o in zip(refs, outs):
                assert torch.equal(o.view(torch.int32), ref.view(torch.int32))
            for o in outs:
                o.fill_(float("nan"))
        assert L.hxq_cuda_affine_device_status() == 0
    finally:
        for im, _ in imgs:
            L.hxq_cuda_image_destroy(im)


def test_vq_gemm_and_gemv_repeatable(H, L, cuda):
    """VQ GEMM (16 and 2048 tokens) and tensor-core GEMV (1, 8 and 16
    tokens; at 8 the 11008-wide matrix in two K parts) on two 7B-shaped
    images, repeated: every run bit-identical to the first (their TMA stages
    are refilled only after the reads of the previous fill are ordered; the
    parts are added in order)."""
    torch = cuda
    from hxq_b200.sharded import ColumnSplitLayer
    mats = [dict(name="q", O=4096, I=4096, vq=synth.vq12(4096, 4096, 7200)),
            dict(name="down", O=4096, I=11008, vq=synth.vq12(4096, 11008, 7201))]
    layer = ColumnSplitLayer(mats, "vq12", max_tokens=2048, rank=0, world=1, torch=torch, lib=L)
    stream = torch.cuda.Stream()
    for N in (1, 8, 16, 2048):
        xs = {I: torch.from_numpy(synth.activations(N, I, 7300 + I)[0].view(np.int16)).cuda() for I in (4096, 11008)}
        ref = None
        for _ in range(8):
            layer.forward(xs, N, stream)
            stream.synchronize()
            outs = [y.clone() for y in layer.outputs(N)]
            if ref is None:
                ref = outs
                continue
            for a, b in zip(outs, ref):
                assert torch.equal(a.view(torch.int32), b.view(torch.int32)), N
    assert L.hxq_cuda_affine_device_status() == 0
    layer.close()
