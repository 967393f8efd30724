"""The library's own CPU backend (HXQ_BACKEND_CPU / host buffers) against the
reference's golden vectors and the oracle: bit-exact weights, identical
confidence and status codes.  Also the host-side helpers (packing, seeds)."""
import ctypes as C

import numpy as np
import pytest

from conftest import golden_names, load_golden
from hxq_b200 import synth


def _load(H, g, idx_len=None, k=None):
    t = H.Tensor()
    if g["mode"] == 3:
        assert t.load_affine(g["codes"], g["scales"], g["offsets"], g["out_f"], g["in_f"], g["gs"]) == 0
    else:
        assert t.load_codebook(g["codebook"], k or g["k"], g["vdim"]) == 0
        if g["mode"] == 0:
            assert t.load_indices_8bit(g["indices"], g["out_f"], g["in_f"]) == 0
        else:
            assert t.load_indices_12bit(g["packed"], g["out_f"], g["in_f"], length=idx_len) == 0
    if g.get("rows") is not None and len(g["rows"]):
        assert t.load_sidecar(g["rows"], g["cols"], g["vals"]) == 0
    return t


@pytest.mark.parametrize("name", [n for n in golden_names() if not n.startswith("affine_mm")])
def test_cpu_backend_matches_reference_golden(H, L, name):
    g = load_golden(name)
    t = _load(H, g, idx_len=g.get("call_idx_len"), k=g.get("call_k"))
    t.t.sidecar_l2_norm = -1.0
    out = g["out_init"].copy()
    err = L.hxq_tensor_decompress(t.ref, out.ctypes.data)
    assert err == g["expect_err"]
    if err == 0:
        assert np.array_equal(out.view(np.uint32), g["expect_w"].view(np.uint32))
        assert np.float32(t.confidence) == g["expect_conf"]
    else:
        assert t.confidence == -1.0  # untouched on error


@pytest.mark.parametrize("name", golden_names("affine_mm"))
def test_cpu_affine_ref_matches_reference_golden(H, L, name):
    g = load_golden(name)
    x = np.ascontiguousarray(g["x"], np.float32)
    y = np.zeros((x.shape[0], g["out_f"]), np.float32)
    b = g.get("bias")
    L.hxq_affine_group_matmul_ref(x.ctypes.data, g["codes"].ctypes.data, g["scales"].ctypes.data,
                                  g["offsets"].ctypes.data, None if b is None else b.ctypes.data,
                                  y.ctypes.data, x.shape[0], g["in_f"], g["out_f"], g["gs"])
    assert np.array_equal(y.view(np.uint32), g["expect_y"].view(np.uint32))


@pytest.mark.parametrize("seed", range(4))
def test_cpu_backend_vs_oracle_random(H, L, oracle, seed):
    rng = np.random.default_rng(100 + seed)
    for d in (synth.vq12(int(rng.integers(1, 64)), 4 * int(rng.integers(1, 64)), seed),
              synth.scalar(int(rng.integers(1, 64)), int(rng.integers(1, 200)), seed, frac=0.05)):
        t = H.Tensor().load(d)
        out = np.zeros(d["out_f"] * d["in_f"], np.float32)
        assert L.hxq_tensor_decompress(t.ref, out.ctypes.data) == 0
        err, w, conf = oracle.decompress(d)
        assert err == 0 and np.array_equal(out.view(np.uint32), w.view(np.uint32))
        assert t.confidence == conf


def test_shared_buffer_kat(H, L):
    # test_hxq.c:190-235: two tensors through one buffer, high_water 16
    buf = H.SharedBuffer()
    assert L.hxq_shared_buffer_init(C.byref(buf), 16) == 0 and buf.capacity == 16
    cb = np.arange(256, dtype=np.float32)
    t1, t2 = H.Tensor(), H.Tensor()
    assert t1.load_codebook(cb, 256, 1) == 0 and t1.load_indices_8bit(np.arange(4, dtype=np.uint8), 2, 2) == 0
    assert t2.load_codebook(cb, 256, 1) == 0
    assert t2.load_indices_8bit(np.arange(10, 170, 10, dtype=np.uint8), 4, 4) == 0
    out = C.c_void_p()
    assert L.hxq_tensor_decompress_shared(t1.ref, C.byref(buf), C.byref(out)) == 0
    assert C.cast(out, C.POINTER(C.c_float))[0] == 0.0
    assert L.hxq_tensor_decompress_shared(t2.ref, C.byref(buf), C.byref(out)) == 0
    assert C.cast(out, C.POINTER(C.c_float))[0] == 10.0
    assert buf.high_water == 16
    # growth beyond capacity
    t3 = H.Tensor()
    assert t3.load_codebook(cb, 256, 1) == 0 and t3.load_indices_8bit(np.zeros(40, np.uint8), 5, 8) == 0
    assert L.hxq_tensor_decompress_shared(t3.ref, C.byref(buf), C.byref(out)) == 0
    assert buf.capacity == 40 and buf.high_water == 40
    L.hxq_shared_buffer_free(C.byref(buf))


def test_sidecar_nnz_zero_keeps_arrays(H, L):
    # src/hxq.c:140-143: nnz == 0 clears the count, keeps the arrays
    t = H.Tensor()
    assert t.load_codebook(np.arange(256, dtype=np.float32), 256, 1) == 0
    assert t.load_indices_8bit(np.arange(4, dtype=np.uint8), 2, 2) == 0
    assert t.load_sidecar([0], [0], [1.0]) == 0
    rows_ptr = C.cast(t.t.sidecar_rows, C.c_void_p).value
    assert L.hxq_tensor_load_sidecar(t.ref, None, None, None, 0) == 0
    assert t.t.sidecar_nnz == 0 and C.cast(t.t.sidecar_rows, C.c_void_p).value == rows_ptr
    out = np.zeros(4, np.float32)
    assert L.hxq_tensor_decompress(t.ref, out.ctypes.data) == 0
    assert list(out) == [0, 1, 2, 3] and t.confidence == 0.0


def test_vq12_vdim1_rejected(H, L):
    # the reference reads past a dim-1 codebook here; this library refuses
    t = H.Tensor()
    assert t.load_codebook(np.zeros(4096, np.float32), 4096, 1) == 0
    assert t.load_indices_12bit(np.zeros(6, np.uint8), 2, 4) == 0
    out = np.zeros(8, np.float32)
    assert L.hxq_tensor_decompress(t.ref, out.ctypes.data) == 3


def test_free_zeroes_descriptor(H, L):
    d = synth.vq12(4, 8, 1, frac=0.2)
    t = H.Tensor().load(d)
    L.hxq_tensor_free(t.ref)
    assert bytes(t.t) == bytes(96)


def test_pack12_matches_oracle(oracle):
    rng = np.random.default_rng(7)
    for out_f, in_f in [(3, 8), (2, 6), (5, 10), (4, 4), (1, 2), (7, 7)]:
        idx = rng.integers(0, 4096, out_f * (in_f // 2)).astype(np.uint16)
        p = synth.pack12(idx, out_f, in_f)
        assert np.array_equal(p, oracle.pack_rows12(idx, out_f, in_f))
        assert np.array_equal(synth.unpack12(p, out_f, in_f), idx)


def test_synth_is_deterministic():
    a, b = synth.vq12(32, 64, 5), synth.vq12(32, 64, 5)
    for k in ("codebook", "packed", "rows", "cols", "vals"):
        assert np.array_equal(a[k], b[k])
    d = synth.vq12(2048, 2048, synth.SEED_C1)
    assert len(d["rows"]) == 20971 and len(d["packed"]) == 3145728
    assert np.all(np.diff(d["rows"].astype(np.int64) * 2048 + d["cols"]) > 0)  # unique, row-major
    s = synth.scalar(4096, 4096, synth.SEED_C2)
    assert len(s["rows"]) == 16777 and np.all(np.diff(s["codebook"]) >= 0)
