"""CUDA decompress path against the reference: golden vectors produced by the
reference library, and the oracle on seeded inputs at the benchmark sizes.

Bar: weights bit-exact (fp32) or equal to round-to-nearest-even of the
reference's fp32 value (bf16); status codes identical.  Confidence, on
every API (hxq_dequant, hxq_tensor_decompress, and the d_conf output of the
batched hxq_cuda_decompress_images): the reference's value, the float
running sum in array order (src/hxq.c:335-349), bit for bit -- which is
inside the 1e-5 relative bar against the reference's float accumulation.
The batched API's d_sumsq output (GPU fused fp64 reduction) is held to
1e-9 relative of the exactly computed sum of squares, and the reference's
own running sum to its a-priori rounding bound against that exact value,
so the two definitions are tied together.
All calls go through the C ABI of libhxq.so.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import golden_names, load_golden
from hxq_b200 import synth
from hxq_b200.shard import slice_rows as shard_rows_dict

pytestmark = pytest.mark.gpu

CONF_REL_EXACT = 1e-6   # vs the sum computed in double
CONF_REL_REF = 1e-5     # vs the reference's float accumulation
SUMSQ_REL = 1e-9        # fp64 GPU sum of squares vs the exact sum


def _dev(torch, host: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(host)).cuda()


def _check_conf(got, ref_conf, exact=None):
    """Every API: the reference's value, bit for bit (so within 1e-5)."""
    assert abs(float(got) - float(ref_conf)) <= CONF_REL_REF * abs(float(ref_conf)), (got, ref_conf)
    assert np.float32(got) == np.float32(ref_conf), (got, ref_conf)


def _check_sumsq(got, exact, ref_conf=None, nnz=0):
    """d_sumsq: the exact sum of squares; the reference's running sum stays
    within its rounding bound of it."""
    ex2 = exact * exact
    assert abs(float(got) - ex2) <= 1e-300 + SUMSQ_REL * ex2, (got, ex2)
    if ref_conf is not None and exact > 0.0:
        bound = 0.5 * max(nnz - 1, 0) * 2.0 ** -24 * exact + 2.0 ** -23 * exact
        assert abs(ref_conf - exact) <= bound, (ref_conf, exact, bound)


def _check_conf_exact(got, exact, ref_conf=None, nnz=0):
    """Fused GPU reduction: the exact value; and the reference within its bound."""
    if exact == 0.0:
        assert got == 0.0
        return
    assert abs(got - exact) <= CONF_REL_EXACT * exact, (got, exact)
    if ref_conf is not None:
        bound = 0.5 * max(nnz - 1, 0) * 2.0 ** -24 * exact + 2.0 ** -23 * exact
        assert abs(ref_conf - exact) <= bound, (ref_conf, exact, bound)


def _bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def _golden_tensor(H, g):
    t = H.Tensor()
    if g["mode"] == 3:
        assert t.load_affine(g["codes"], g["scales"], g["offsets"], g["out_f"], g["in_f"], g["gs"]) == 0
    else:
        assert t.load_codebook(g["codebook"], g.get("call_k") or g["k"], g["vdim"]) == 0
        if g["mode"] == 0:
            assert t.load_indices_8bit(g["indices"], g["out_f"], g["in_f"]) == 0
        else:
            assert t.load_indices_12bit(g["packed"], g["out_f"], g["in_f"], length=g.get("call_idx_len")) == 0
    if g.get("rows") is not None and len(g["rows"]):
        assert t.load_sidecar(g["rows"], g["cols"], g["vals"]) == 0
    return t


@pytest.mark.parametrize("name", [n for n in golden_names() if not n.startswith("affine_mm")])
def test_golden_fp32_device_output(H, L, oracle, cuda, name):
    torch = cuda
    g = load_golden(name)
    t = _golden_tensor(H, g)
    t.t.sidecar_l2_norm = -1.0
    out = _dev(torch, g["out_init"])
    torch.cuda.synchronize()
    err = L.hxq_tensor_decompress(t.ref, out.data_ptr())
    assert err == g["expect_err"]
    if err != 0:
        assert t.confidence == -1.0
        return
    w = out.cpu().numpy()
    assert np.array_equal(_bits(w), _bits(g["expect_w"]))
    _check_conf(t.confidence, float(g["expect_conf"]), oracle.l2_exact(g))


@pytest.mark.parametrize("name", ["vq12_64x256", "vq12_odd_6x10", "vq12_dups_16x64", "vq12_k256_32x128",
                                  "scalar_64x96", "scalar_dups_9x13", "affine_dq_16x256"])
def test_golden_bf16_device_output(H, L, cuda, name):
    torch = cuda
    g = load_golden(name)
    t = _golden_tensor(H, g)
    n = g["out_f"] * g["in_f"]
    out = torch.zeros(n, dtype=torch.bfloat16, device="cuda")
    assert L.hxq_cuda_decompress(t.ref, out.data_ptr(), H.HXQ_OUT_BF16) == 0
    got = out.view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(got, synth.bf16_round(g["expect_w"]))


def test_c1_full_vq12_2048(H, L, oracle, cuda):
    torch = cuda
    d = synth.vq12(2048, 2048, synth.SEED_C1)
    err, w_ref, conf_ref = oracle.decompress(d)
    assert err == 0
    t = H.Tensor().load(d)
    out = torch.empty(2048 * 2048, dtype=torch.float32, device="cuda")
    for _ in range(2):  # second call reuses the cached device image and scratch
        out.fill_(float("nan"))
        torch.cuda.synchronize()
        assert L.hxq_tensor_decompress(t.ref, out.data_ptr()) == 0
        assert np.array_equal(_bits(out.cpu().numpy()), _bits(w_ref))
        _check_conf(t.confidence, conf_ref, oracle.l2_exact(d))
    first = t.confidence
    assert L.hxq_tensor_decompress(t.ref, out.data_ptr()) == 0
    assert t.confidence == first  # deterministic reduction


def test_c2_scalar_arena_fp32_and_bf16(H, L, oracle, cuda):
    d = synth.scalar(4096, 4096, synth.SEED_C2)
    small = synth.scalar(64, 128, 5, frac=0.01)
    err, w_ref, conf_ref = oracle.decompress(d)
    t, ts = H.Tensor().load(d), H.Tensor().load(small)
    arena = H.SharedBuffer()
    assert L.hxq_cuda_arena_init(C.byref(arena), 1024) == 0
    assert L.hxq_cuda_buffer_is_device(C.byref(arena)) == 1
    r = H.Result()
    # reused arena: small tensor, big tensor (grows), small again
    for tt, dd in ((ts, small), (t, d), (ts, small)):
        for backend in (H.HXQ_BACKEND_CUDA, H.HXQ_BACKEND_AUTO):
            assert L.hxq_dequant(tt.ref, C.byref(arena), backend, C.byref(r)) == 0
            n = dd["out_f"] * dd["in_f"]
            host = np.empty(n, np.float32)
            assert r.out_features == dd["out_f"] and r.in_features == dd["in_f"]
            _copy_d2h(cuda, r.weights, host)
            e2, w2, c2 = oracle.decompress(dd)
            assert np.array_equal(_bits(host), _bits(w2))
            _check_conf(r.confidence, c2, oracle.l2_exact(dd))
    assert arena.high_water == 4096 * 4096 and arena.capacity >= 4096 * 4096
    # bf16 into the same arena
    assert L.hxq_dequant_bf16(t.ref, C.byref(arena), C.byref(r)) == 0
    got = np.empty(4096 * 4096, np.uint16)
    _copy_d2h(cuda, r.weights, got)
    assert np.array_equal(got, synth.bf16_round(w_ref))
    _check_conf(r.confidence, conf_ref, oracle.l2_exact(d))
    # CPU backend refuses a device arena
    assert L.hxq_dequant(t.ref, C.byref(arena), H.HXQ_BACKEND_CPU, C.byref(r)) == H.HXQ_ERR_INVALID_ARG
    L.hxq_shared_buffer_free(C.byref(arena))
    assert arena.capacity == 0 and L.hxq_cuda_buffer_is_device(C.byref(arena)) == 0


def _copy_d2h(torch, dptr, host: np.ndarray):
    """Copy n elements at a raw device pointer into a numpy array."""
    from hxq_b200 import device_view
    torch.cuda.synchronize()
    host[:] = device_view(torch, dptr, host.size, host.dtype).cpu().numpy()


def test_dequant_cuda_backend_host_buffer(H, L, oracle, cuda):
    d = synth.vq12(512, 1024, 77)
    t = H.Tensor().load(d)
    buf = H.SharedBuffer()
    assert L.hxq_shared_buffer_init(C.byref(buf), 16) == 0
    r = H.Result()
    assert L.hxq_dequant(t.ref, C.byref(buf), H.HXQ_BACKEND_CUDA, C.byref(r)) == 0
    w = np.ctypeslib.as_array(C.cast(r.weights, C.POINTER(C.c_float)), shape=(512 * 1024,)).copy()
    err, w_ref, conf = oracle.decompress(d)
    assert np.array_equal(_bits(w), _bits(w_ref))
    _check_conf(r.confidence, conf, oracle.l2_exact(d))
    assert buf.high_water == 512 * 1024
    L.hxq_shared_buffer_free(C.byref(buf))


@pytest.mark.parametrize("name", ["vq12_odd_6x10", "vq12_ragged_5x7", "vq12_64x256", "scalar_64x96"])
def test_dequant_cuda_backend_host_buffer_golden(H, L, cuda, name):
    """HXQ_BACKEND_CUDA into a host buffer: columns the 12-bit decoder never
    writes (odd pair counts) keep the buffer's contents, as in hxq.c; other
    shapes are written in full."""
    g = load_golden(name)
    t = _golden_tensor(H, g)
    n = g["out_f"] * g["in_f"]
    buf = H.SharedBuffer()
    assert L.hxq_shared_buffer_init(C.byref(buf), n) == 0
    host = np.ctypeslib.as_array(C.cast(buf.data, C.POINTER(C.c_float)), shape=(n,))
    host[:] = g["out_init"]
    r = H.Result()
    assert L.hxq_dequant(t.ref, C.byref(buf), H.HXQ_BACKEND_CUDA, C.byref(r)) == g["expect_err"]
    if g["expect_err"] == 0:
        w = np.ctypeslib.as_array(C.cast(r.weights, C.POINTER(C.c_float)), shape=(n,)).copy()
        assert np.array_equal(_bits(w), _bits(g["expect_w"]))
        _check_conf(r.confidence, float(g["expect_conf"]))
    L.hxq_shared_buffer_free(C.byref(buf))


def _image(H, L, t, r0, r1):
    img = C.c_void_p()
    assert L.hxq_cuda_image_create(t.ref, r0, r1, C.byref(img)) == 0
    return img


def test_batched_images_mixed_kinds(H, L, oracle, cuda):
    torch = cuda
    ds = [synth.vq12(256, 512, 1), synth.scalar(100, 300, 2, frac=0.02), synth.vq12(64, 1024, 3, k=256),
          synth.vq12(37, 30, 4, frac=0.05),   # in_f % 4 != 0: generic kernel
          synth.vq12(128, 4096, 5), synth.scalar(7, 5, 6, frac=0.3)]
    ts = [H.Tensor().load(d) for d in ds]
    imgs = [_image(H, L, t, 0, d["out_f"]) for t, d in zip(ts, ds)]
    sizes = [d["out_f"] * d["in_f"] for d in ds]
    offs = np.zeros(len(ds), np.uint64)
    pos = 0
    for i, n in enumerate(sizes):
        offs[i] = pos
        pos += (n + 63) // 64 * 64 + 4  # +4 floats: the next slot is only 16-B aligned
    out = torch.full((pos,), float("nan"), dtype=torch.float32, device="cuda")
    sumsq = torch.zeros(len(ds), dtype=torch.float64, device="cuda")
    conf = torch.zeros(len(ds), dtype=torch.float32, device="cuda")
    arr = (C.c_void_p * len(ds))(*[i.value for i in imgs])
    offs_c = (C.c_size_t * len(ds))(*[int(o) for o in offs])
    torch.cuda.synchronize()
    assert L.hxq_cuda_decompress_images(arr, len(ds), out.data_ptr(), offs_c, H.HXQ_OUT_F32,
                                        sumsq.data_ptr(), conf.data_ptr(), None) == 0
    assert L.hxq_cuda_stream_synchronize(None) == 0
    host = out.cpu().numpy()
    ss, cf = sumsq.cpu().numpy(), conf.cpu().numpy()
    for i, d in enumerate(ds):
        init = np.full(sizes[i], np.nan, np.float32)
        err, w_ref, c_ref = oracle.decompress(d, out=init)
        got = host[int(offs[i]): int(offs[i]) + sizes[i]]
        assert np.array_equal(_bits(got), _bits(w_ref)), i
        exact = oracle.l2_exact(d)
        _check_sumsq(ss[i], exact, c_ref, len(d["rows"]))
        assert abs(L.hxq_cuda_image_sidecar_sumsq(imgs[i]) - exact * exact) <= 1e-9 * max(exact * exact, 1e-30)
        assert np.float32(L.hxq_cuda_image_reference_confidence(imgs[i])) == np.float32(c_ref)
        assert np.float32(L.hxq_cuda_image_tensor_confidence(imgs[i])) == np.float32(c_ref)
        _check_conf(float(cf[i]), c_ref)
    for im in imgs:
        L.hxq_cuda_image_destroy(im)


def test_exact_sums_optional_and_deterministic(H, L, oracle, cuda):
    """Two 4096 x 4096 12-bit images (units handed out by the counter) and a
    small scalar one (one CTA per unit, no counter): without a sum-of-squares
    output the call is one launch and still stores every confidence; with
    one, a second kernel adds each image's unit sums in a fixed order, so two
    calls give the same bits; the weights are the same either way."""
    torch = cuda
    ds = [synth.vq12(4096, 4096, 61), synth.vq12(4096, 4096, 62), synth.scalar(64, 256, 63, frac=0.02)]
    ts = [H.Tensor().load(d) for d in ds]
    imgs = [_image(H, L, t, 0, d["out_f"]) for t, d in zip(ts, ds)]
    sizes = [d["out_f"] * d["in_f"] for d in ds]
    offs, pos = [], 0
    for n in sizes:
        offs.append(pos)
        pos += (n + 63) // 64 * 64
    arr = (C.c_void_p * len(ds))(*[i.value for i in imgs])
    offs_c = (C.c_size_t * len(ds))(*offs)
    refs = [oracle.decompress(d) for d in ds]

    def run(with_sums):
        out = torch.full((pos,), float("nan"), dtype=torch.float32, device="cuda")
        ss = torch.full((len(ds),), -1.0, dtype=torch.float64, device="cuda")
        cf = torch.full((len(ds),), -1.0, dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        n0 = L.hxq_cuda_launch_count()
        assert L.hxq_cuda_decompress_images(arr, len(ds), out.data_ptr(), offs_c, H.HXQ_OUT_F32,
                                            ss.data_ptr() if with_sums else None, cf.data_ptr(), None) == 0
        launches = L.hxq_cuda_launch_count() - n0
        assert L.hxq_cuda_stream_synchronize(None) == 0
        return out.cpu().numpy(), ss.cpu().numpy(), cf.cpu().numpy(), launches

    out0, ss0, cf0, l0 = run(False)
    out1, ss1, cf1, l1 = run(True)
    _, ss2, _, _ = run(True)
    # one launch per kind (12-bit and scalar), and each followed by its sums
    assert (l0, l1) == (2, 4), (l0, l1)
    assert np.array_equal(_bits(out0), _bits(out1))
    assert np.array_equal(ss1.view(np.uint64), ss2.view(np.uint64))
    assert np.all(ss0 == -1.0)
    for i, d in enumerate(ds):
        err, w_ref, c_ref = refs[i]
        assert err == 0
        assert np.array_equal(_bits(out0[offs[i]: offs[i] + sizes[i]]), _bits(w_ref)), i
        _check_conf(float(cf0[i]), c_ref)
        _check_conf(float(cf1[i]), c_ref)
        _check_sumsq(ss1[i], oracle.l2_exact(d), c_ref, len(d["rows"]))
    for im in imgs:
        L.hxq_cuda_image_destroy(im)


def test_row_shards_reassemble(H, L, oracle, cuda):
    torch = cuda
    d = synth.vq12(1376 * 3, 4096, 9)  # 11008/8-style ragged row count per shard
    t = H.Tensor().load(d)
    bounds = [0, 1376, 2752, d["out_f"]]
    imgs = [_image(H, L, t, bounds[i], bounds[i + 1]) for i in range(3)]
    out = torch.empty(d["out_f"] * d["in_f"], dtype=torch.float32, device="cuda")
    sumsq = torch.zeros(3, dtype=torch.float64, device="cuda")
    conf = torch.zeros(3, dtype=torch.float32, device="cuda")
    arr = (C.c_void_p * 3)(*[i.value for i in imgs])
    offs = (C.c_size_t * 3)(*[b * d["in_f"] for b in bounds[:3]])
    assert L.hxq_cuda_decompress_images(arr, 3, out.data_ptr(), offs, 0, sumsq.data_ptr(), conf.data_ptr(),
                                        None) == 0
    assert L.hxq_cuda_stream_synchronize(None) == 0
    err, w_ref, c_ref = oracle.decompress(d)
    assert np.array_equal(_bits(out.cpu().numpy()), _bits(w_ref))
    total = float(sumsq.sum().item())
    _check_conf_exact(float(np.sqrt(total)), oracle.l2_exact(d), c_ref, len(d["rows"]))
    # each shard reports the reference's value for its own rows, and carries
    # the whole matrix's reference value
    cf = conf.cpu().numpy()
    for i in range(3):
        part = shard_rows_dict(d, bounds[i], bounds[i + 1])
        _check_conf(float(cf[i]), oracle.decompress(part)[2])
        _check_conf(L.hxq_cuda_image_tensor_confidence(imgs[i]), c_ref)
    for im in imgs:
        L.hxq_cuda_image_destroy(im)


def test_unaligned_output_uses_generic_path(H, L, oracle, cuda):
    torch = cuda
    for d in (synth.vq12(33, 64, 11, frac=0.05), synth.scalar(40, 50, 12, frac=0.05)):
        t = H.Tensor().load(d)
        n = d["out_f"] * d["in_f"]
        buf = torch.zeros(n + 1, dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        assert L.hxq_tensor_decompress(t.ref, buf.data_ptr() + 4) == 0
        err, w_ref, c_ref = oracle.decompress(d)
        assert np.array_equal(_bits(buf.cpu().numpy()[1:]), _bits(w_ref))
        _check_conf(t.confidence, c_ref, oracle.l2_exact(d))


def test_index_oob_reported_and_cleared(H, L, oracle, cuda):
    torch = cuda
    g = load_golden("vq12_oob_8x64")
    t = _golden_tensor(H, g)
    out = torch.zeros(8 * 64, dtype=torch.float32, device="cuda")
    t.t.sidecar_l2_norm = 3.0
    assert L.hxq_tensor_decompress(t.ref, out.data_ptr()) == H.HXQ_ERR_INDEX_OOB
    assert t.confidence == 3.0
    d = synth.vq12(8, 64, 3)
    t2 = H.Tensor().load(d)
    assert L.hxq_tensor_decompress(t2.ref, out.data_ptr()) == 0  # error word was cleared
    assert np.array_equal(_bits(out.cpu().numpy()), _bits(oracle.decompress(d)[1]))


def test_reload_invalidates_device_copy(H, L, oracle, cuda):
    torch = cuda
    a, b = synth.vq12(64, 128, 21), synth.vq12(64, 128, 22)
    t = H.Tensor().load(a)
    out = torch.empty(64 * 128, dtype=torch.float32, device="cuda")
    assert L.hxq_tensor_decompress(t.ref, out.data_ptr()) == 0
    assert t.load_indices_12bit(b["packed"], 64, 128) == 0
    assert t.load_codebook(b["codebook"], 4096, 2) == 0
    assert t.load_sidecar(b["rows"], b["cols"], b["vals"]) == 0
    assert L.hxq_tensor_decompress(t.ref, out.data_ptr()) == 0
    assert np.array_equal(_bits(out.cpu().numpy()), _bits(oracle.decompress(b)[1]))


def test_reference_gpu_launchers(H, L, oracle, cuda):
    torch = cuda
    d = synth.vq12(96, 256, 31, frac=0.01)
    dn = dict(d, rows=None)
    cb, pk = _dev(torch, d["codebook"]), _dev(torch, d["packed"])
    out = torch.empty(96 * 256, dtype=torch.float32, device="cuda")
    assert L.hxq_cuda_decompress_vq2d_12bit(cb.data_ptr(), pk.data_ptr(), out.data_ptr(), 96, 256) == 0
    torch.cuda.synchronize()
    assert np.array_equal(_bits(out.cpu().numpy()), _bits(oracle.decompress(dn)[1]))
    r, c, v = _dev(torch, d["rows"]), _dev(torch, d["cols"]), _dev(torch, d["vals"])
    conf = L.hxq_cuda_apply_sidecar(r.data_ptr(), c.data_ptr(), v.data_ptr(), out.data_ptr(), 256, len(d["rows"]))
    err, w_ref, c_ref = oracle.decompress(d)
    assert np.array_equal(_bits(out.cpu().numpy()), _bits(w_ref))
    _check_conf_exact(conf, oracle.l2_exact(d), c_ref, len(d["rows"]))
    s = synth.scalar(50, 70, 32)
    sn = dict(s, rows=None)
    cb2, ix = _dev(torch, s["codebook"]), _dev(torch, s["indices"])
    out2 = torch.empty(50 * 70, dtype=torch.float32, device="cuda")
    assert L.hxq_cuda_decompress_scalar(cb2.data_ptr(), ix.data_ptr(), out2.data_ptr(), 50, 70) == 0
    torch.cuda.synchronize()
    assert np.array_equal(_bits(out2.cpu().numpy()), _bits(oracle.decompress(sn)[1]))


def test_llama7b_layer0_batch(H, L, oracle, cuda):
    """One 7B layer (q,k,v,o,gate,up,down) in one launch, each bit-exact."""
    torch = cuda
    ds = [synth.vq12(o, i, synth.llama7b_seed(0, p)) for p, (_, o, i) in enumerate(synth.LLAMA7B_PROJ)]
    ts = [H.Tensor().load(d) for d in ds]
    imgs = [_image(H, L, t, 0, d["out_f"]) for t, d in zip(ts, ds)]
    sizes = [d["out_f"] * d["in_f"] for d in ds]
    offs = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.uint64)
    out = torch.empty(int(sum(sizes)), dtype=torch.float32, device="cuda")
    conf = torch.zeros(7, dtype=torch.float32, device="cuda")
    sumsq = torch.zeros(7, dtype=torch.float64, device="cuda")
    arr = (C.c_void_p * 7)(*[i.value for i in imgs])
    offs_c = (C.c_size_t * 7)(*[int(o) for o in offs])
    assert L.hxq_cuda_decompress_images(arr, 7, out.data_ptr(), offs_c, 0, sumsq.data_ptr(), conf.data_ptr(),
                                        None) == 0
    assert L.hxq_cuda_stream_synchronize(None) == 0
    cf = conf.cpu().numpy()
    ss = sumsq.cpu().numpy()
    for i, d in enumerate(ds):
        err, w_ref, c_ref = oracle.decompress(d)
        got = out[int(offs[i]): int(offs[i]) + sizes[i]].cpu().numpy()
        assert np.array_equal(_bits(got), _bits(w_ref)), i
        # the confidence the batched API returns is the reference's (1e-5 bar,
        # met bit for bit); the fp64 sum of squares is the exact one
        _check_conf(float(cf[i]), c_ref)
        _check_sumsq(ss[i], oracle.l2_exact(d), c_ref, len(d["rows"]))
        assert np.float32(L.hxq_cuda_image_reference_confidence(imgs[i])) == np.float32(c_ref)
    for im in imgs:
        L.hxq_cuda_image_destroy(im)
