"""Pins the oracle (oracle/hxq_oracle.c) before anything is compared with it:
  * the reference's own known-answer tests (test/test_hxq.c,
    test/test_affine.c), restated with the same inputs and expectations;
  * golden vectors produced by the reference library itself
    (tests/golden, made by tests/golden/make_golden.py);
  * a seeded differential run against the reference library compiled
    here from its own sources (oracle/_ref), when that build exists.
"""
import math

import numpy as np
import pytest

from conftest import golden_names, load_golden
from hxq_b200 import synth


def _dict12(cb, packed, out_f, in_f, k=4096, rows=None, cols=None, vals=None):
    return dict(mode=2, out_f=out_f, in_f=in_f, k=k, vdim=2, codebook=np.asarray(cb, np.float32),
                packed=np.asarray(packed, np.uint8), rows=rows, cols=cols, vals=vals)


def _dict8(cb, idx, out_f, in_f, rows=None, cols=None, vals=None):
    return dict(mode=0, out_f=out_f, in_f=in_f, k=256, vdim=1, codebook=np.asarray(cb, np.float32),
                indices=np.asarray(idx, np.uint8), rows=rows, cols=cols, vals=vals)


def _sc(rows, cols, vals):
    return (np.asarray(rows, np.uint32), np.asarray(cols, np.uint32), np.asarray(vals, np.float32))


# ---- test/test_hxq.c known answers ----------------------------------------

def test_kat_pack_unpack_all_values(oracle):
    # test_hxq.c:92-130: 0xABC/0x123, zero pair, max pair, all 4096 values
    assert oracle.unpack12(oracle.pack12(0xABC, 0x123)) == (0xABC, 0x123)
    assert oracle.unpack12(oracle.pack12(0, 0)) == (0, 0)
    assert oracle.unpack12(oracle.pack12(4095, 4095)) == (4095, 4095)
    for v in range(4096):
        assert oracle.unpack12(oracle.pack12(v, 4095 - v)) == (v, 4095 - v)
    # byte layout of the code (include/hxq.h:250-251)
    assert oracle.pack12(0xABC, 0x123) == bytes([0xAB, 0xC1, 0x23])


def test_kat_scalar_4x4(oracle):
    # test_hxq.c:40-88
    cb = np.arange(256, dtype=np.float32) * np.float32(0.01)
    idx = [0, 1, 2, 3, 10, 20, 30, 40, 100, 150, 200, 250, 255, 128, 64, 32]
    err, w, conf = oracle.decompress(_dict8(cb, idx, 4, 4))
    assert err == 0
    np.testing.assert_allclose(w[:4], [0.0, 0.01, 0.02, 0.03], atol=1e-6)
    np.testing.assert_allclose(w[12:], [2.55, 1.28, 0.64, 0.32], atol=1e-6)
    assert conf == 0.0


def test_kat_sidecar_2x2(oracle):
    # test_hxq.c:134-186
    cb = np.zeros(256, np.float32)
    cb[:4] = [1, 2, 3, 4]
    d = _dict8(cb, [0, 1, 2, 3], 2, 2, *_sc([0, 1], [1, 0], [0.5, -0.3]))
    err, w, conf = oracle.decompress(d)
    assert err == 0
    np.testing.assert_allclose(w, [1.0, 2.5, 2.7, 4.0], atol=1e-6)
    assert abs(conf - math.sqrt(0.5 * 0.5 + 0.3 * 0.3)) < 1e-5


def test_kat_vq12_2x4(oracle):
    # test_hxq.c:239-281 (codebook i*0.001, i*0.001+0.5; indices 100,200 / 300,400)
    i = np.arange(4096, dtype=np.float32)
    cb = np.empty(8192, np.float32)
    cb[0::2] = i * np.float32(0.001)
    cb[1::2] = i * np.float32(0.001) + np.float32(0.5)
    packed = oracle.pack12(100, 200) + oracle.pack12(300, 400)
    err, w, _ = oracle.decompress(_dict12(cb, np.frombuffer(packed, np.uint8), 2, 4))
    assert err == 0
    np.testing.assert_allclose(w[:4], [0.1, 0.6, 0.2, 0.7], atol=1e-4)
    np.testing.assert_allclose(w[4:], [0.3, 0.8, 0.4, 0.9], atol=1e-4)


def test_kat_meta_2x3(oracle):
    # test_hxq.c:285-326
    cb = np.arange(256, dtype=np.float32)
    d = _dict8(cb, [10, 20, 30, 40, 50, 60], 2, 3, *_sc([1], [2], [0.7]))
    err, w, conf = oracle.decompress(d)
    assert err == 0 and w[0] == 10.0
    assert abs(w[5] - 60.7) < 1e-6 and abs(conf - 0.7) < 1e-5


# ---- test/test_affine.c known answers --------------------------------------

def _aff(codes, scales, offsets, out_f, in_f, gs):
    return dict(mode=3, codes=np.asarray(codes, np.uint8), scales=np.asarray(scales, np.float32),
                offsets=np.asarray(offsets, np.float32), out_f=out_f, in_f=in_f, gs=gs, rows=None)


def test_kat_affine_small(oracle):
    # :69-98, :102-128, :218-236, :399-427
    y = oracle.affine_matmul(np.ones((1, 4), np.float32), _aff(range(8), [2, 0.5], [1, -1], 2, 4, 4))
    np.testing.assert_allclose(y[0], [16, 7], atol=1e-5)
    y = oracle.affine_matmul(np.ones((1, 8), np.float32), _aff([1] * 4 + [2] * 4, [1, 3], [0, 0], 1, 8, 4))
    np.testing.assert_allclose(y[0], [28], atol=1e-5)
    y = oracle.affine_matmul(np.zeros((1, 2), np.float32), _aff([0] * 4, [1, 1], [0, 0], 2, 2, 2),
                             bias=np.array([10, -5], np.float32))
    np.testing.assert_allclose(y[0], [10, -5], atol=1e-6)
    y = oracle.affine_matmul(np.ones((1, 4), np.float32), _aff([1] * 4 + [2] * 4, [1, 1], [0, 0], 2, 4, 4),
                             bias=np.array([100, 200], np.float32))
    np.testing.assert_allclose(y[0], [104, 208], atol=1e-5)


def test_kat_affine_zero_and_max_codes(oracle):
    # :240-276 zero codes, :280-302 max code 63
    offs = (np.arange(8, dtype=np.float32) + 1) * np.float32(0.5)
    y = oracle.affine_matmul(np.ones((1, 8), np.float32), _aff([0] * 32, [1] * 8, offs, 4, 8, 4))
    for o in range(4):
        assert abs(y[0, o] - (offs[2 * o] * 4 + offs[2 * o + 1] * 4)) < 1e-4
    y = oracle.affine_matmul(np.ones((1, 4), np.float32), _aff([63] * 8, [0.1, 0.2], [0, 0], 2, 4, 4))
    np.testing.assert_allclose(y[0], [4 * 63 * 0.1, 4 * 63 * 0.2], atol=1e-4)


def test_kat_affine_decompress(oracle):
    # :306-331 and :431-462 (same values through the dequant path)
    d = _aff([0, 10, 20, 30, 5, 15, 25, 63], [0.5, 2.0], [1.0, -3.0], 2, 4, 4)
    W = oracle.affine_decompress(d)
    np.testing.assert_allclose(W, [1, 6, 11, 16, 7, 27, 47, 123], atol=1e-6)
    err, W2, conf = oracle.decompress(d)
    assert err == 0 and conf == 0.0 and np.array_equal(W, W2)


@pytest.mark.parametrize("N,OUT,IN,tol", [(1, 16, 128, 1e-4), (4, 32, 256, 1e-3)])
def test_kat_affine_fused_vs_dense(oracle, N, OUT, IN, tol):
    # :132-214: fused == decompress + naive matmul (6-bit codes, LCG data)
    rng = np.random.default_rng(OUT)
    d = _aff(rng.integers(0, 64, OUT * IN), rng.uniform(-0.05, 0.05, OUT * IN // 128),
             rng.uniform(-0.005, 0.005, OUT * IN // 128), OUT, IN, 128)
    x = rng.uniform(-0.5, 0.5, (N, IN)).astype(np.float32)
    fused = oracle.affine_matmul(x, d)
    dense = oracle.dense_matmul(x, oracle.affine_decompress(d))
    assert np.max(np.abs(fused - dense)) < tol


# ---- golden vectors from the reference library -----------------------------

@pytest.mark.parametrize("name", [n for n in golden_names() if not n.startswith("affine_mm")])
def test_oracle_matches_reference_golden(oracle, name):
    g = load_golden(name)
    kw = {k[5:]: v for k, v in g.items() if k.startswith("call_")}
    k = kw.get("k")
    err, w, conf = oracle.decompress(g, out=g["out_init"].copy(), idx_len=kw.get("idx_len"), k=k)
    assert err == g["expect_err"]
    if err == 0:
        assert np.array_equal(w.view(np.uint32), g["expect_w"].view(np.uint32))
        assert np.float32(conf) == g["expect_conf"]


@pytest.mark.parametrize("name", golden_names("affine_mm"))
def test_oracle_affine_matches_reference_golden(oracle, name):
    g = load_golden(name)
    y = oracle.affine_matmul(g["x"], g, bias=g.get("bias"))
    assert np.array_equal(y.view(np.uint32), g["expect_y"].view(np.uint32))


# ---- differential run against the reference built here ---------------------

def _ref_or_skip():
    from oracle.oracle import Reference, ref_available
    if not ref_available():
        pytest.skip("oracle/_ref not built (needs the reference tree)")
    return Reference()


@pytest.mark.parametrize("seed", range(6))
def test_oracle_vs_reference_random(oracle, seed):
    ref = _ref_or_skip()
    rng = np.random.default_rng(seed)
    out_f, in_f = int(rng.integers(1, 40)), int(rng.integers(1, 90))
    for d in (synth.vq12(out_f, in_f, seed, frac=0.1), synth.scalar(out_f, in_f, seed, frac=0.1),
              synth.affine(out_f, 32 * int(rng.integers(1, 4)), 32, seed)):
        init = rng.standard_normal(d["out_f"] * d["in_f"]).astype(np.float32)
        e1, w1, c1 = oracle.decompress(d, out=init.copy())
        e2, w2, c2 = ref.decompress(d, out=init.copy())
        assert e1 == e2
        assert np.array_equal(w1.view(np.uint32), w2.view(np.uint32))
        assert c1 == c2


def test_oracle_vs_reference_c1_full(oracle):
    ref = _ref_or_skip()
    d = synth.vq12(2048, 2048, synth.SEED_C1)
    e1, w1, c1 = oracle.decompress(d)
    e2, w2, c2 = ref.decompress(d)
    assert e1 == e2 == 0 and np.array_equal(w1.view(np.uint32), w2.view(np.uint32)) and c1 == c2


def test_oracle_vs_reference_affine_random(oracle):
    ref = _ref_or_skip()
    for seed, (O, I, gs, N) in enumerate([(64, 256, 128, 5), (33, 384, 64, 2), (256, 512, 128, 1)]):
        d = synth.affine(O, I, gs, seed, bias=True)
        _, x = synth.activations(N, I, seed)
        assert np.array_equal(oracle.affine_matmul(x, d, bias=d["bias"]).view(np.uint32),
                              ref.affine_matmul(x, d, bias=d["bias"]).view(np.uint32))
