"""Affine group-quantized matmul on the GPU against the reference.

Tolerance (stated by the north star: rel 1e-5 for fp32 paths, 1e-2 for bf16
paths) is applied per output as |y - y_ref| / sum_i |x_i * w_i|: the
natural scale of an fp32 dot product's rounding error (a plain relative
error is ill-posed for outputs near zero).  The fp32-activation entry points
and the bf16 GEMV (one token) are held to 1e-5; the tcgen05 dequant-GEMM
(bf16, from 2 tokens) to its bf16-weight bound 2^-9 (and to 1e-5 against a
float64 product with the same bf16 weights).
"""
import ctypes as C

import numpy as np
import pytest

from conftest import golden_names, load_golden
from hxq_b200 import synth

pytestmark = pytest.mark.gpu
TOL = 1e-5
# bf16 activations from 2 tokens on take the tcgen05 dequant-GEMM, which
# rounds each dequantized weight to bf16: |error| <= 2^-9 sum|x_i w_i| (plus
# fp32 accumulation), inside the north star's 1e-2 for bf16 paths.
GEMM_TOL = 2.0 ** -9 + 1e-5


def _tol_bf16(N, d):
    gemm = N >= 2 and d["in_f"] % 128 == 0 and d["gs"] % 64 == 0
    return GEMM_TOL if gemm else TOL


def _tol_path(H, L, dev, xd, N):
    """Tolerance of the kernel the automatic choice takes for these operands:
    the bf16-weight GEMM's bound, else the exact GEMVs' 1e-5."""
    t = dev.tensor(H)
    p = L.hxq_affine_group_matmul_bf16_auto_path(xd.data_ptr(), C.byref(t), N)
    assert p in (H.HXQ_AFFINE_PATH_GEMV, H.HXQ_AFFINE_PATH_TC_GEMV, H.HXQ_AFFINE_PATH_GEMM)
    return GEMM_TOL if p == H.HXQ_AFFINE_PATH_GEMM else TOL


def _scale(oracle, x, d):
    W = oracle.affine_decompress(d).reshape(d["out_f"], d["in_f"]).astype(np.float64)
    return np.abs(x.astype(np.float64)) @ np.abs(W).T


def _check(y, y_ref, scale, tol=TOL):
    err = np.abs(y.astype(np.float64) - y_ref.astype(np.float64)) / np.maximum(scale, 1e-30)
    assert float(err.max()) <= tol, float(err.max())


class Dev:
    def __init__(self, torch, d, bias=None):
        self.torch = torch
        self.codes = torch.from_numpy(np.ascontiguousarray(d["codes"])).cuda()
        self.scales = torch.from_numpy(np.ascontiguousarray(d["scales"])).cuda()
        self.offsets = torch.from_numpy(np.ascontiguousarray(d["offsets"])).cuda()
        self.bias = None if bias is None else torch.from_numpy(np.ascontiguousarray(bias)).cuda()
        self.d = d

    def tensor(self, H):
        return H.AffineTensor(self.codes.data_ptr(), self.scales.data_ptr(), self.offsets.data_ptr(),
                              None if self.bias is None else self.bias.data_ptr(),
                              self.d["out_f"], self.d["in_f"], self.d["gs"])


def _run_f32(torch, H, L, dev, x, api="struct"):
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    y = torch.full((x.shape[0], dev.d["out_f"]), float("nan"), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    if api == "struct":
        t = dev.tensor(H)
        assert L.hxq_affine_group_matmul(xd.data_ptr(), C.byref(t), y.data_ptr(), x.shape[0]) == 0
    else:
        d = dev.d
        assert L.hxq_affine_matmul_flat(xd.data_ptr(), dev.codes.data_ptr(), dev.scales.data_ptr(),
                                        dev.offsets.data_ptr(), None if dev.bias is None else dev.bias.data_ptr(),
                                        y.data_ptr(), x.shape[0], d["in_f"], d["out_f"], d["gs"]) == 0
    torch.cuda.synchronize()
    return y.cpu().numpy()


def _run_bf16(torch, H, L, dev, xh, path=None):
    """bf16 matmul through the automatic entry point, or with `path` forced."""
    xd = torch.from_numpy(np.ascontiguousarray(xh.view(np.int16))).cuda()
    y = torch.full((xh.shape[0], dev.d["out_f"]), float("nan"), dtype=torch.float32, device="cuda")
    t = dev.tensor(H)
    torch.cuda.synchronize()
    if path is None:
        assert L.hxq_affine_group_matmul_bf16(xd.data_ptr(), C.byref(t), y.data_ptr(), xh.shape[0], None) == 0
    else:
        assert L.hxq_affine_group_matmul_bf16_path(xd.data_ptr(), C.byref(t), y.data_ptr(), xh.shape[0], path,
                                                   None) == 0
    torch.cuda.synchronize()
    return y.cpu().numpy()


@pytest.mark.parametrize("name", golden_names("affine_mm"))
@pytest.mark.parametrize("api", ["struct", "flat"])
def test_golden(H, L, oracle, cuda, name, api):
    g = load_golden(name)
    dev = Dev(cuda, g, g.get("bias"))
    y = _run_f32(cuda, H, L, dev, g["x"], api)
    _check(y, g["expect_y"], _scale(oracle, g["x"], g))


@pytest.mark.parametrize("N", [1, 2, 5, 8, 16, 64])
def test_c3_4096_small_batches(H, L, oracle, cuda, N):
    d = synth.affine(4096, 4096, 128, synth.SEED_C3, bias=(N == 5))
    xh, x = synth.activations(N, 4096, synth.SEED_C3 + N)
    dev = Dev(cuda, d, d["bias"])
    ref = oracle.affine_matmul(x, d, bias=d["bias"])
    sc = _scale(oracle, x, d)
    xd = cuda.from_numpy(np.ascontiguousarray(xh.view(np.int16))).cuda()
    tol = _tol_path(H, L, dev, xd, N)
    assert (tol == TOL) == (N <= 8)           # up to 8 tokens: an exact-product GEMV
    _check(_run_bf16(cuda, H, L, dev, xh), ref, sc, tol)
    _check(_run_f32(cuda, H, L, dev, x), ref, sc)
    assert L.hxq_cuda_affine_device_status() == 0


@pytest.mark.parametrize("N", [512, 4096])
def test_c3_4096_large_batches_sampled(H, L, oracle, cuda, N):
    d = synth.affine(4096, 4096, 128, synth.SEED_C3)
    xh, x = synth.activations(N, 4096, synth.SEED_C3 + N)
    dev = Dev(cuda, d)
    yb = _run_bf16(cuda, H, L, dev, xh)
    yf = _run_f32(cuda, H, L, dev, x)
    rows = sorted({0, 1, N // 3, N // 2, N - 2, N - 1})
    for n in rows:
        ref = oracle.affine_matmul(x, d, n0=n, n1=n + 1)
        sc = _scale(oracle, x[n:n + 1], d)
        _check(yb[n:n + 1], ref, sc, GEMM_TOL)
        _check(yf[n:n + 1], ref, sc)
    assert L.hxq_cuda_affine_device_status() == 0


@pytest.mark.parametrize("O,I,gs,N", [(33, 96, 32, 3), (40, 120, 24, 2), (17, 256, 128, 9), (64, 1024, 256, 1)])
def test_odd_shapes(H, L, oracle, cuda, O, I, gs, N):
    d = synth.affine(O, I, gs, O + I, bias=True)
    xh, x = synth.activations(N, I, gs)
    dev = Dev(cuda, d, d["bias"])
    ref = oracle.affine_matmul(x, d, bias=d["bias"])
    sc = _scale(oracle, x, d)
    _check(_run_f32(cuda, H, L, dev, x), ref, sc)
    _check(_run_bf16(cuda, H, L, dev, xh), ref, sc, _tol_bf16(N, d))


@pytest.mark.parametrize("O,I,gs,N", [(200, 256, 128, 17), (128, 512, 64, 100), (300, 1024, 256, 300),
                                      (64, 11008, 128, 40), (129, 128, 128, 16), (256, 384, 128, 257),
                                      (4096, 4096, 128, 2), (1024, 2048, 128, 8), (11008, 4096, 128, 33)])
def test_tcgen05_gemm_shapes(H, L, oracle, cuda, O, I, gs, N):
    """Ragged output rows, ragged token tiles (BN = 32, 128, 256), group
    sizes 64..256, K not a power of two, with bias."""
    d = synth.affine(O, I, gs, O * 7 + I + N, bias=True)
    xh, x = synth.activations(N, I, O + N)
    dev = Dev(cuda, d, d["bias"])
    ref = oracle.affine_matmul(x, d, bias=d["bias"])
    sc = _scale(oracle, x, d)
    y = _run_bf16(cuda, H, L, dev, xh, path=H.HXQ_AFFINE_PATH_GEMM)
    assert L.hxq_cuda_affine_device_status() == 0
    _check(y, ref, sc, GEMM_TOL)
    # layout check: the same contraction in float64 with the kernel's own
    # weights, bf16(fp32(code*scale + offset)) (one rounding to fp32, as the
    # kernel's fma); what remains is fp32 tensor-core accumulation over K
    ng = I // gs
    q = d["codes"].reshape(O, I).astype(np.float64)
    s64 = np.repeat(d["scales"].reshape(O, ng).astype(np.float64), gs, axis=1)
    f64 = np.repeat(d["offsets"].reshape(O, ng).astype(np.float64), gs, axis=1)
    W32 = (q * s64 + f64).astype(np.float32)
    Wb = synth.bf16_to_f32(synth.bf16_round(W32)).astype(np.float64).reshape(O, I)
    yd = x.astype(np.float64) @ Wb.T + d["bias"].astype(np.float64)
    _check(y, yd, sc, 1e-4)


def test_gemm_last_wave_split(H, L, oracle, cuda):
    """2400 x 2048 at 2000 tokens: 19 x 8 = 152 tiles of 128 x 256 on 148
    SMs, so the last 4 tiles (row tiles 15-18, the last ragged in rows, of the
    last, ragged token tile) are split along K into 4 ranges whose partial
    sums the last arriving CTA adds in order.  Sampled token rows cover whole
    tiles and split ones; the result is the same on every run."""
    O, I, gs, N = 2400, 2048, 128, 2000
    d = synth.affine(O, I, gs, 2400, bias=True)
    xh, x = synth.activations(N, I, 2401)
    dev = Dev(cuda, d, d["bias"])
    y = _run_bf16(cuda, H, L, dev, xh, path=H.HXQ_AFFINE_PATH_GEMM)
    y2 = _run_bf16(cuda, H, L, dev, xh, path=H.HXQ_AFFINE_PATH_GEMM)
    assert L.hxq_cuda_affine_device_status() == 0
    assert np.array_equal(y, y2)
    ng = I // gs
    q = d["codes"].reshape(O, I).astype(np.float64)
    s64 = np.repeat(d["scales"].reshape(O, ng).astype(np.float64), gs, axis=1)
    f64 = np.repeat(d["offsets"].reshape(O, ng).astype(np.float64), gs, axis=1)
    Wb = synth.bf16_to_f32(synth.bf16_round((q * s64 + f64).astype(np.float32))).astype(np.float64).reshape(O, I)
    for n in (0, 1000, 1791, 1792, 1900, 1999):
        ref = oracle.affine_matmul(x, d, bias=d["bias"], n0=n, n1=n + 1)
        sc = _scale(oracle, x[n:n + 1], d)
        _check(y[n:n + 1], ref, sc, GEMM_TOL)
        yd = x[n:n + 1].astype(np.float64) @ Wb.T + d["bias"].astype(np.float64)
        _check(y[n:n + 1], yd, sc, 1e-4)


@pytest.mark.parametrize("shape", [(2048, 2048), (11008, 2048), (2048, 11008)])
def test_reference_shapes_6bit_codes(H, L, oracle, cuda, shape):
    # test/test_affine_cuda.cu:194-272 shapes at N=1 with 6-bit codes
    O, I = shape
    d = synth.affine(O, I, 128, O * 3 + I)
    d["codes"] = (np.random.default_rng(O + I).integers(0, 64, O * I)).astype(np.uint8)
    _, x = synth.activations(1, I, O)
    dev = Dev(cuda, d)
    y = _run_f32(cuda, H, L, dev, x)
    ref = oracle.affine_matmul(x, d)
    assert np.max(np.abs(y - ref)) < 1e-3
    _check(y, ref, _scale(oracle, x, d))


def test_bias_only(H, L, oracle, cuda):
    # test/test_affine_cuda.cu:276-338: zero codes and x, output = bias
    d = dict(codes=np.zeros(64 * 128, np.uint8), scales=np.ones(64, np.float32), offsets=np.zeros(64, np.float32),
             out_f=64, in_f=128, gs=128)
    bias = (np.arange(64, dtype=np.float32) + 1) * 10
    dev = Dev(cuda, d, bias)
    y = _run_f32(cuda, H, L, dev, np.zeros((1, 128), np.float32))
    assert np.max(np.abs(y[0] - bias)) < 1e-5


def test_invalid_arguments(H, L, cuda):
    d = synth.affine(8, 128, 128, 1)
    dev = Dev(cuda, d)
    t = dev.tensor(H)
    t.group_size = 0
    x = cuda.zeros(128, device="cuda")
    y = cuda.zeros(8, device="cuda")
    assert L.hxq_affine_group_matmul(x.data_ptr(), C.byref(t), y.data_ptr(), 1) == -1
    t.group_size = 96  # does not divide 128
    assert L.hxq_affine_group_matmul(x.data_ptr(), C.byref(t), y.data_ptr(), 1) == -1
    assert L.hxq_affine_group_matmul(x.data_ptr(), None, y.data_ptr(), 1) == -1


@pytest.mark.parametrize("O,I,gs,N", [(1, 128, 64, 1), (17, 128, 64, 3), (100, 768, 256, 8), (4096, 4096, 128, 1),
                                      (4096, 4096, 128, 16), (513, 2048, 256, 9), (11008, 4096, 128, 2),
                                      (4096, 11008, 128, 4), (33, 11008, 128, 1), (256, 4096, 512, 12)])
def test_tc_gemv_vs_oracle(H, L, oracle, cuda, O, I, gs, N):
    """The tensor-core GEMV (forced): ragged row blocks (1, 17, 100, 513
    rows), K not a multiple of the 512-code stage, group sizes 64..512,
    1..16 tokens (one and two 8-token tiles), bias on odd token counts."""
    d = synth.affine(O, I, gs, O * 5 + I + N, bias=(N % 2 == 1))
    xh, x = synth.activations(N, I, O + 3 * N)
    dev = Dev(cuda, d, d["bias"])
    y = _run_bf16(cuda, H, L, dev, xh, path=H.HXQ_AFFINE_PATH_TC_GEMV)
    assert L.hxq_cuda_affine_device_status() == 0
    _check(y, oracle.affine_matmul(x, d, bias=d["bias"]), _scale(oracle, x, d))


def test_tc_gemv_byte_codes_and_token_scales(H, L, oracle, cuda):
    """Every byte value as a code (widened exactly), and tokens of very
    different sizes (2^-120 .. 2^40, an all-zero token, values 2^-30 below
    the token's largest): each token's power-of-two staging scale keeps the
    products exact."""
    O, I, gs, N = 96, 1024, 128, 6
    d = synth.affine(O, I, gs, 77)
    d["codes"] = np.random.default_rng(5).integers(0, 256, O * I).astype(np.uint8)
    _, x = synth.activations(N, I, 78)
    x = x * np.array([1.0, 2.0 ** -60, 2.0 ** 40, 0.0, 1.0, 2.0 ** -120], np.float32)[:, None]
    x[4, ::7] *= np.float32(2.0 ** -30)
    xh = synth.bf16_round(x.astype(np.float32)).reshape(N, I)
    x = synth.bf16_to_f32(xh).reshape(N, I)
    dev = Dev(cuda, d)
    ref = oracle.affine_matmul(x, d)
    sc = _scale(oracle, x, d)
    for path in (H.HXQ_AFFINE_PATH_TC_GEMV, H.HXQ_AFFINE_PATH_AUTO):
        y = _run_bf16(cuda, H, L, dev, xh, path=path)
        _check(y, ref, sc)
        assert not np.any(y[3])                 # the zero token: exactly zero
    assert L.hxq_cuda_affine_device_status() == 0


def test_path_selection(H, L, cuda):
    d = synth.affine(256, 4096, 128, 3)
    dev = Dev(cuda, d)
    t = dev.tensor(H)
    x = cuda.zeros(64 * 4096, dtype=cuda.int16, device="cuda")
    y = cuda.zeros(64 * 256, dtype=cuda.float32, device="cuda")
    auto = L.hxq_affine_group_matmul_bf16_auto_path
    assert auto(x.data_ptr(), C.byref(t), 1) == H.HXQ_AFFINE_PATH_TC_GEMV
    assert auto(x.data_ptr(), C.byref(t), 8) == H.HXQ_AFFINE_PATH_TC_GEMV
    assert auto(x.data_ptr(), C.byref(t), 9) == H.HXQ_AFFINE_PATH_GEMM
    assert auto(x.data_ptr() + 2, C.byref(t), 4) == H.HXQ_AFFINE_PATH_GEMV     # unaligned activations
    assert auto(x.data_ptr(), None, 4) == -1
    run = L.hxq_affine_group_matmul_bf16_path
    assert run(x.data_ptr(), C.byref(t), y.data_ptr(), 17, H.HXQ_AFFINE_PATH_TC_GEMV, None) == -1
    assert run(x.data_ptr(), C.byref(t), y.data_ptr(), 4, 9, None) == -1
    for p in (H.HXQ_AFFINE_PATH_GEMV, H.HXQ_AFFINE_PATH_TC_GEMV, H.HXQ_AFFINE_PATH_GEMM):
        assert run(x.data_ptr(), C.byref(t), y.data_ptr(), 4, p, None) == 0
    cuda.cuda.synchronize()
    assert L.hxq_cuda_affine_device_status() == 0


@pytest.mark.parametrize("N", [1, 5, 16])
def test_batch_of_layer_projections(H, L, cuda, N):
    """A layer's projections in one batch call (shared launches), two
    outputs each at a column offset: bit-identical to one call per matrix on
    the same path (up to 16 tokens the batch takes the tensor-core GEMV for
    every matrix it suits, one call only up to 8)."""
    torch = cuda
    shapes = [(512, 4096), (256, 4096), (256, 4096), (512, 4096), (1376, 4096), (1376, 4096), (512, 11008)]
    devs, xs, refs, outs, ts = [], [], [], [], []
    for i, (O, I) in enumerate(shapes):
        d = synth.affine(O, I, 128, 100 + i, bias=(i % 2 == 0))
        dev = Dev(torch, d, d["bias"])
        xh, _ = synth.activations(N, I, 200 + i)
        x = torch.from_numpy(np.ascontiguousarray(xh.view(np.int16))).cuda()
        ref = torch.empty((N, O), dtype=torch.float32, device="cuda")
        t = dev.tensor(H)
        if N > 16 or L.hxq_affine_group_matmul_bf16_path(x.data_ptr(), C.byref(t), ref.data_ptr(), N,
                                                         H.HXQ_AFFINE_PATH_TC_GEMV, None) != 0:
            assert L.hxq_affine_group_matmul_bf16(x.data_ptr(), C.byref(t), ref.data_ptr(), N, None) == 0
        devs.append(dev); xs.append(x); refs.append(ref); ts.append(dev.tensor(H))
        outs.append([torch.full((N, O + 64), float("nan"), dtype=torch.float32, device="cuda") for _ in range(2)])
    n = len(shapes)
    T = (H.AffineTensor * n)(*ts)
    X = (C.c_void_p * n)(*[x.data_ptr() for x in xs])
    Y = (C.c_void_p * (2 * n))(*[o.data_ptr() + 4 * 32 for pair in outs for o in pair])
    LD = (C.c_uint32 * n)(*[O + 64 for O, _ in shapes])
    assert L.hxq_affine_group_matmul_bf16_batch(n, T, X, Y, 2, LD, N, None) == 0
    torch.cuda.synchronize()
    for (O, _), ref, pair in zip(shapes, refs, outs):
        for o in pair:
            assert torch.equal(o[:, 32:32 + O].contiguous().view(torch.int32), ref.view(torch.int32))
            assert bool(torch.isnan(o[:, :32]).all()) and bool(torch.isnan(o[:, 32 + O:]).all())
    assert L.hxq_cuda_affine_device_status() == 0


def test_batch_chained_gemms(H, L, cuda):
    """A prefill batch whose GEMMs are unsplit (4096 x 256 at 2048 tokens:
    256 tiles each), so each one after the first is chained to the one
    before it and overlaps its last wave: every output bit-identical to one
    call per matrix, and the batch's outputs complete before the next
    kernel on the stream reads them."""
    torch = cuda
    N, shapes = 2048, [(4096, 256)] * 3
    devs, xs, refs, outs, ts = [], [], [], [], []
    for i, (O, I) in enumerate(shapes):
        d = synth.affine(O, I, 128, 700 + i, bias=(i == 1))
        dev = Dev(torch, d, d["bias"])
        xh, _ = synth.activations(N, I, 800 + i)
        x = torch.from_numpy(np.ascontiguousarray(xh.view(np.int16))).cuda()
        ref = torch.empty((N, O), dtype=torch.float32, device="cuda")
        t = dev.tensor(H)
        assert L.hxq_affine_group_matmul_bf16(x.data_ptr(), C.byref(t), ref.data_ptr(), N, None) == 0
        devs.append(dev); xs.append(x); refs.append(ref); ts.append(t)
        outs.append(torch.full((N, O), float("nan"), dtype=torch.float32, device="cuda"))
    n = len(shapes)
    T = (H.AffineTensor * n)(*ts)
    X = (C.c_void_p * n)(*[x.data_ptr() for x in xs])
    Y = (C.c_void_p * n)(*[o.data_ptr() for o in outs])
    LD = (C.c_uint32 * n)(*[O for O, _ in shapes])
    for _ in range(2):
        assert L.hxq_affine_group_matmul_bf16_batch(n, T, X, Y, 1, LD, N, None) == 0
        total = sum(o.sum() for o in outs)   # a kernel that reads every output after the batch
        torch.cuda.synchronize()
        assert torch.isfinite(total)
        for ref, o in zip(refs, outs):
            assert torch.equal(o.view(torch.int32), ref.view(torch.int32))
        for o in outs:
            o.fill_(float("nan"))
    assert L.hxq_cuda_affine_device_status() == 0


def test_batch_chain_breaks_at_other_kernels(H, L, cuda):
    """Prefill batch of GEMM matrices with one between them that the GEMM
    does not take (group size 32: the CUDA-core GEMV): the chain of GEMMs
    breaks there; every output bit-identical to one call per matrix."""
    torch = cuda
    N = 2048
    specs = [(4096, 256, 128), (4096, 256, 128), (512, 256, 32), (4096, 256, 128), (4096, 256, 128)]
    devs, xs, refs, outs, ts = [], [], [], [], []
    for i, (O, I, gs) in enumerate(specs):
        d = synth.affine(O, I, gs, 1400 + i)
        dev = Dev(torch, d)
        xh, _ = synth.activations(N, I, 1500 + i)
        x = torch.from_numpy(np.ascontiguousarray(xh.view(np.int16))).cuda()
        ref = torch.empty((N, O), dtype=torch.float32, device="cuda")
        t = dev.tensor(H)
        assert L.hxq_affine_group_matmul_bf16(x.data_ptr(), C.byref(t), ref.data_ptr(), N, None) == 0
        devs.append(dev); xs.append(x); refs.append(ref); ts.append(t)
        outs.append(torch.full((N, O), float("nan"), dtype=torch.float32, device="cuda"))
    n = len(specs)
    T = (H.AffineTensor * n)(*ts)
    X = (C.c_void_p * n)(*[x.data_ptr() for x in xs])
    Y = (C.c_void_p * n)(*[o.data_ptr() for o in outs])
    LD = (C.c_uint32 * n)(*[O for O, _, _ in specs])
    for _ in range(3):
        assert L.hxq_affine_group_matmul_bf16_batch(n, T, X, Y, 1, LD, N, None) == 0
        torch.cuda.synchronize()
        for ref, o in zip(refs, outs):
            assert torch.equal(o.view(torch.int32), ref.view(torch.int32))
        for o in outs:
            o.fill_(float("nan"))
    assert L.hxq_cuda_affine_device_status() == 0


def test_gemm_batch_repeatable(H, L, cuda):
    """The tcgen05 GEMMs of a 7B layer's shard (2048 / 5504 rows, as one of
    two GPUs holds them) at 2048 tokens, repeated: every run bit-identical to
    the first.  (A shared-memory stage refilled by TMA while reads of it were
    still in flight once made a few rows differ from run to run.)"""
    torch = cuda
    from hxq_b200.sharded import ColumnSplitLayer
    N = 2048
    mats = [dict(name=n, O=O, I=I, affine=synth.affine(O, I, 128, 7000 + p))
            for p, (n, O, I) in enumerate(synth.LLAMA7B_PROJ)]
    xs = {I: torch.from_numpy(synth.activations(N, I, 7100 + I)[0].view(np.int16)).cuda() for I in (4096, 11008)}
    layer = ColumnSplitLayer(mats, "affine", max_tokens=N, rank=0, world=2, torch=torch, lib=L)
    stream = torch.cuda.Stream()
    ref = None
    for _ in range(12):
        layer.forward(xs, N, stream, assembly="local")
        stream.synchronize()
        outs = [y.clone() for y in layer.local_outputs(N)]
        if ref is None:
            ref = outs
            continue
        for j, (a, b) in enumerate(zip(outs, ref)):
            assert torch.equal(a.view(torch.int32), b.view(torch.int32)), mats[j]["name"]
    assert L.hxq_cuda_affine_device_status() == 0
    layer.close()
