"""Lloyd's algorithm and PolarQuant rotation (reference src/hxq_lloyd.c,
src/polarquant.c) against the reference compiled from its own sources
(oracle/_ref) and the oracle restatement.

Bars:
- Lloyd indices: bit-exact.
- Dead counts: equal.
- Updated codebooks: within one fp32 ulp. The reference sums in double in
  an order that depends on its thread count; here the sums are
  order-independent fixed-point ones.
- Rotation matrix: bit-exact to the reference, and within 1e-4 of numpy's
  float64 QR of the same RandomState draws (the reference's own
  verification tolerance).
- GPU rotate/unrotate: bit-exact to the reference's sequential fp32 sums.
"""
import ctypes as C

import numpy as np
import pytest

from oracle.oracle import REF_LLOYD_SO, REF_PQ_SO, ReferenceLloyd, ReferencePolarQuant, ref_available


def _randf(seed, n):
    """The reference tests' generator (test/test_lloyd.c:35-38): an LCG and
    float(state >> 16) / 32768 - 1 in fp32; n draws from one stream."""
    hi = np.empty(n, np.uint32)
    s = seed
    for i in range(n):
        s = (s * 1103515245 + 12345) & 0xFFFFFFFF
        hi[i] = s >> 16
    return (hi.astype(np.float32) / np.float32(32768.0) - np.float32(1.0)).astype(np.float32)


def _rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


def _ulps(a, b):
    ai = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    bi = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    ai = np.where(ai < 0, -(ai & 0x7FFFFFFF), ai)
    bi = np.where(bi < 0, -(bi & 0x7FFFFFFF), bi)
    return np.abs(ai - bi)


needs_ref = pytest.mark.skipif(not (ref_available(REF_LLOYD_SO) and ref_available(REF_PQ_SO)),
                               reason="oracle/_ref not built (no reference tree)")


# ---- CPU: host API, oracle pins ---------------------------------------------

@needs_ref
@pytest.mark.parametrize("dim,seed", [(1, 0), (8, 42), (8, 99), (32, 7), (64, 47), (100, 3), (128, 42), (256, 1)])
def test_rotation_matches_reference_bit_for_bit(H, L, dim, seed):
    Q = np.zeros(dim * dim, np.float32)
    assert L.pq_generate_rotation(dim, seed, Q.ctypes.data) == 0
    ref = ReferencePolarQuant().rotation(dim, seed).reshape(-1)
    assert np.array_equal(Q.view(np.uint32), ref.view(np.uint32))


@needs_ref
@pytest.mark.parametrize("dim,seed", [(8, 42), (64, 5), (128, 42)])
def test_reference_rotation_matches_numpy_qr(dim, seed):
    """The algorithm the reference states: numpy RandomState(seed).randn(dim,
    dim), QR, columns signed so that R's diagonal is positive."""
    h = np.random.RandomState(seed).randn(dim, dim)
    q, r = np.linalg.qr(h)
    q = q * np.sign(np.diag(r))[None, :]
    ref = ReferencePolarQuant().rotation(dim, seed)
    assert np.abs(ref - q).max() < 1e-4
    assert np.abs(ref @ ref.T - np.eye(dim)).max() < 1e-4


@needs_ref
@pytest.mark.parametrize("hd", [32, 64, 96, 128])
def test_oracle_rotation_matches_reference(oracle, hd):
    rp = ReferencePolarQuant()
    Q = rp.rotation(hd, 11)
    x = _rng(hd).standard_normal(37 * hd).astype(np.float32)
    for rot in (True, False):
        assert np.array_equal(oracle.pq_apply(x, Q, hd, rot).view(np.uint32), rp.apply(x, Q, hd, rot).view(np.uint32))


def test_pq_host_api_and_errors(H, L):
    nh, hd = C.c_uint32(), C.c_uint32()
    g = L.pq_infer_head_geometry
    assert g(256, 4, C.byref(nh), C.byref(hd)) == 0 and (nh.value, hd.value) == (4, 64)
    assert g(1024, 0, C.byref(nh), C.byref(hd)) == 0 and (nh.value, hd.value) == (8, 128)
    assert g(192, 0, C.byref(nh), C.byref(hd)) == 0 and (nh.value, hd.value) == (3, 64)
    assert g(17, 0, C.byref(nh), C.byref(hd)) == 4            # PQ_ERR_NOT_DIVISIBLE
    assert g(100, 3, C.byref(nh), C.byref(hd)) == 4
    assert g(100, 0, None, C.byref(hd)) == 1
    assert L.pq_generate_rotation(32, 42, None) == 1           # PQ_ERR_NULL_PTR
    dummy = np.zeros(4, np.float32)
    assert L.pq_generate_rotation(0, 42, dummy.ctypes.data) == 2   # PQ_ERR_INVALID_DIM
    assert L.pq_generate_rotation(2048, 42, dummy.ctypes.data) == 2
    Q = np.eye(32, dtype=np.float32)
    assert L.pq_rotate(None, Q.ctypes.data, 1, 32) == 1
    assert L.pq_rotate(dummy.ctypes.data, None, 1, 32) == 1
    assert L.pq_unrotate(dummy.ctypes.data, Q.ctypes.data, 0, 32) == 2
    layer = H.PqLayer()
    assert L.pq_layer_init(C.byref(layer), 16, 2, 42, 5) == 0
    assert layer.initialized == 1 and layer.seed == 47
    Qs = np.zeros(256, np.float32)
    assert L.pq_generate_rotation(16, 47, Qs.ctypes.data) == 0
    assert np.array_equal(np.ctypeslib.as_array(layer.Q, (256,)).view(np.uint32), Qs.view(np.uint32))
    L.pq_layer_free(C.byref(layer))
    assert not layer.Q and layer.initialized == 0
    assert L.pq_layer_rotate(C.byref(layer), dummy.ctypes.data) == 1


@needs_ref
@pytest.mark.parametrize("n,k,d", [(500, 32, 1), (500, 32, 2), (777, 7, 4), (300, 256, 8), (10, 4, 2)])
def test_oracle_lloyd_matches_reference(oracle, n, k, d):
    rl = ReferenceLloyd()
    w = _rng(n + k).standard_normal(n * d).astype(np.float32)
    cb = _rng(k + d).standard_normal(k * d).astype(np.float32)
    rc, ridx = rl.assign(w, cb, k, d)
    assert rc == 0 and np.array_equal(oracle.lloyd_assign(w, cb, k, d), ridx)
    rc, ri, rcb, rdead = rl.reassign(w, cb, k, d)
    oi, ocb, odead = oracle.lloyd_reassign(w, cb, k, d)
    assert rc == 0 and np.array_equal(oi, ri) and odead == rdead
    assert np.array_equal(ocb.view(np.uint32), rcb.view(np.uint32))   # single-threaded reference: same order


def test_lloyd_host_validation(L):
    w = np.zeros(4, np.float32)
    cb = np.zeros(4, np.float32)
    idx = np.zeros(2, np.uint8)
    nd = C.c_int(-7)
    r = L.hxq_lloyd_reassign
    assert r(None, cb.ctypes.data, idx.ctypes.data, 2, 2, 2, C.byref(nd)) == -1
    assert r(w.ctypes.data, None, idx.ctypes.data, 2, 2, 2, C.byref(nd)) == -1
    assert r(w.ctypes.data, cb.ctypes.data, None, 2, 2, 2, C.byref(nd)) == -1
    assert r(w.ctypes.data, cb.ctypes.data, idx.ctypes.data, 2, 0, 2, C.byref(nd)) == -2
    assert r(w.ctypes.data, cb.ctypes.data, idx.ctypes.data, 2, 257, 2, C.byref(nd)) == -2
    assert r(w.ctypes.data, cb.ctypes.data, idx.ctypes.data, 2, 4, 3, C.byref(nd)) == -3
    assert r(w.ctypes.data, cb.ctypes.data, idx.ctypes.data, 0, 4, 2, C.byref(nd)) == 0 and nd.value == 0
    assert L.hxq_lloyd_assign_only(w.ctypes.data, cb.ctypes.data, idx.ctypes.data, 2, 4, 5) == -3


# ---- GPU --------------------------------------------------------------------

@pytest.mark.gpu
@needs_ref
@pytest.mark.parametrize("n,k,d", [(1, 1, 1), (500, 32, 1), (1000, 16, 2), (4097, 256, 2), (333, 7, 4), (2000, 256, 8),
                                   (590000, 256, 2), (295000, 256, 4)])
def test_gpu_lloyd_matches_reference(H, L, cuda, n, k, d):
    """Device API against the reference: indices bit-exact, dead counts
    equal, codebooks within one ulp; the reference tests' production shapes
    (590K x 256 x 2, 295K x 256 x 4, test/test_lloyd.c:214-275) included."""
    torch = cuda
    rl = ReferenceLloyd()
    if n >= 100000:   # the reference's benchmark inputs: seed 999 (d = 2) / 777 (d = 4), weights then codebook
        r = _randf(999 if d == 2 else 777, n * d + k * d)
        w, cb = r[:n * d].copy(), r[n * d:].copy()
    else:
        w = _rng(n * 3 + k).standard_normal(n * d).astype(np.float32)
        cb = _rng(k * 5 + d).standard_normal(k * d).astype(np.float32) * np.float32(0.7)
    dw = torch.from_numpy(w).cuda()
    dcb = torch.from_numpy(cb.copy()).cuda()
    didx = torch.zeros(n, dtype=torch.uint8, device="cuda")
    rc, ridx = rl.assign(w, cb, k, d)
    assert L.hxq_cuda_lloyd_assign(dw.data_ptr(), dcb.data_ptr(), didx.data_ptr(), n, k, d, None) == 0
    torch.cuda.synchronize()
    assert np.array_equal(didx.cpu().numpy(), ridx)
    dnd = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    assert L.hxq_cuda_lloyd_reassign(dw.data_ptr(), dcb.data_ptr(), didx.data_ptr(), n, k, d, dnd.data_ptr(),
                                     None) == 0
    torch.cuda.synchronize()
    rc, ri, rcb, rdead = rl.reassign(w, cb, k, d)
    assert rc == 0
    assert np.array_equal(didx.cpu().numpy(), ri)
    assert int(dnd.item()) == rdead
    assert int(_ulps(dcb.cpu().numpy(), rcb).max()) <= 1
    # run-to-run reproducible (order-independent sums)
    dcb2 = torch.from_numpy(cb.copy()).cuda()
    assert L.hxq_cuda_lloyd_reassign(dw.data_ptr(), dcb2.data_ptr(), didx.data_ptr(), n, k, d, None, None) == 0
    assert torch.equal(dcb2.view(torch.int32), dcb.view(torch.int32))


@pytest.mark.gpu
@needs_ref
def test_gpu_lloyd_dead_reinit_kat(H, L, cuda):
    """test/test_lloyd.c:174-210: ten points near (1,1), three far
    centroids; all three die and move to the farthest member x 1.001."""
    n, k, d = 10, 4, 2
    w = np.array([[1.0 + i * 0.01, 1.0] for i in range(n)], np.float32).reshape(-1)
    cb = np.array([1, 1, 100, 100, -100, -100, 200, 200], np.float32)
    idx = np.zeros(n, np.uint8)
    nd = C.c_int(-1)
    got = cb.copy()
    assert L.hxq_lloyd_reassign(w.ctypes.data, got.ctypes.data, idx.ctypes.data, n, k, d, C.byref(nd)) == 0
    rc, ri, rcb, rdead = ReferenceLloyd().reassign(w, cb, k, d)
    assert nd.value == rdead == 3
    assert np.array_equal(idx, ri)
    assert int(_ulps(got, rcb).max()) <= 1
    near = [float(((got[j * 2:j * 2 + 2] - 1.0) ** 2).sum()) < 1.0 for j in range(1, k)]
    assert all(near)


@pytest.mark.gpu
@needs_ref
@pytest.mark.parametrize("hd,nvec", [(128, 1), (128, 33), (128, 4099), (64, 65), (64, 1000), (32, 129), (96, 50),
                                     (256, 17), (48, 3)])
def test_gpu_rotation_bit_exact(H, L, cuda, hd, nvec):
    """Device rotate/unrotate against the reference's pq_rotate/pq_unrotate:
    tiled kernel (32/64/128, ragged last tile) and the generic one."""
    torch = cuda
    rp = ReferencePolarQuant()
    Q = rp.rotation(hd, 42 + hd)
    x = _rng(hd * 7 + nvec).standard_normal(nvec * hd).astype(np.float32)
    dQ = torch.from_numpy(Q.reshape(-1).copy()).cuda()
    for rot in (True, False):
        dv = torch.from_numpy(x.copy()).cuda()
        fn = L.hxq_cuda_pq_rotate if rot else L.hxq_cuda_pq_unrotate
        assert fn(dv.data_ptr(), dQ.data_ptr(), nvec, hd, None) == 0
        torch.cuda.synchronize()
        assert np.array_equal(dv.cpu().numpy().view(np.uint32), rp.apply(x, Q, hd, rot).view(np.uint32)), rot


@pytest.mark.gpu
@needs_ref
def test_gpu_rotation_host_api_and_roundtrip(H, L, cuda):
    """pq_rotate / pq_unrotate / pq_layer_* through host pointers: equal to
    the reference; rotate then unrotate returns the input within 1e-4
    (test/test_polarquant.c:180-218)."""
    rp = ReferencePolarQuant()
    hd, nh = 128, 8
    x = _rng(5).standard_normal(nh * hd).astype(np.float32)
    Q = np.zeros(hd * hd, np.float32)
    assert L.pq_generate_rotation(hd, 42, Q.ctypes.data) == 0
    v = x.copy()
    assert L.pq_rotate(v.ctypes.data, Q.ctypes.data, nh, hd) == 0
    assert np.array_equal(v.view(np.uint32), rp.apply(x, Q.reshape(hd, hd), hd, True).view(np.uint32))
    assert L.pq_unrotate(v.ctypes.data, Q.ctypes.data, nh, hd) == 0
    assert np.abs(v - x).max() < 1e-4
    layer = H.PqLayer()
    assert L.pq_layer_init(C.byref(layer), hd, nh, 42, 0) == 0
    w = x.copy()
    assert L.pq_layer_rotate(C.byref(layer), w.ctypes.data) == 0
    assert L.pq_layer_unrotate(C.byref(layer), w.ctypes.data) == 0
    cos = float(np.dot(w, x) / (np.linalg.norm(w) * np.linalg.norm(x)))
    assert cos > 0.9999
    L.pq_layer_free(C.byref(layer))
