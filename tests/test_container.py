"""The helix-substrate container adapter (hxq_b200.container): safetensors
and GGUF files read without their packages, HXQ modules grouped by suffix,
and the file's REPLACE sidecar targets turned into hxq.c ADD deltas.  The
bar is bit-exact: decompressing a converted module (oracle, the library's
CPU backend, and on the GPU the device path) gives exactly the weights the
file defines (codebook lookup, then each sidecar value replacing its
position, the last of repeated positions winning --
tools/convert_hxq_to_gguf.py:268-295)."""
import os
import struct

import numpy as np
import pytest

from conftest import golden_names, load_golden
from hxq_b200 import container as CT
from oracle.oracle import container_dense


def _rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


def _module(seed, out_f, in_f, vdim, k, nnz, spread=1.0, dup=0):
    """Parts of one module as helix-substrate stores it.  Targets are the
    decoded value plus noise (spread scales it up to far-off values that
    need the ulp search); `dup` repeats some positions with new values."""
    rng = _rng(seed)
    if vdim == 1:
        cb = rng.standard_normal(k).astype(np.float32) * 0.05
        idx = rng.integers(0, k, size=(out_f, in_f)).astype(np.uint8 if k <= 256 else np.int16)
        base = cb[idx.astype(np.int64)].reshape(-1)
    else:
        cb = rng.standard_normal((k, vdim)).astype(np.float32) * 0.05
        idx = rng.integers(0, k, size=(out_f, in_f // vdim)).astype(np.int16)
        base = cb[idx.astype(np.int64)].reshape(-1)
    parts = {"codebook": cb, "indices": idx}
    if nnz:
        pos = rng.choice(out_f * in_f, size=nnz, replace=False).astype(np.int64)
        if dup:
            pos = np.concatenate([pos, rng.choice(pos, size=dup)])
        noise = rng.standard_normal(len(pos)).astype(np.float32) * np.float32(0.01 * spread)
        vals = (base[pos] + noise).astype(np.float32)
        # a few targets of a very different size (1e3x, 1e-3x) and exact zeros
        vals[:3] *= np.float32(1e3)
        vals[3:6] *= np.float32(1e-3)
        vals[6:8] = 0.0
        parts["sidecar_positions"] = pos
        parts["sidecar_values"] = vals
    return parts


def _decode_all(H, L, oracle, d):
    ref_err, w_orc, _ = oracle.decompress(d)
    assert ref_err == 0
    t = H.Tensor().load(d)
    w_lib = np.zeros(d["out_f"] * d["in_f"], np.float32)
    assert L.hxq_tensor_decompress(t.ref, w_lib.ctypes.data) == 0
    return w_orc, w_lib


def test_safetensors_roundtrip(tmp_path):
    rng = _rng(1)
    ts = {"a.f32": rng.standard_normal((3, 5)).astype(np.float32),
          "a.i64": rng.integers(-9, 9, 7).astype(np.int64),
          "a.u8": rng.integers(0, 255, (2, 2, 2)).astype(np.uint8),
          "a.i8": rng.integers(-128, 127, 9).astype(np.int8),
          "a.f16": rng.standard_normal(4).astype(np.float16),
          "empty": np.zeros((0, 4), np.float32)}
    p = str(tmp_path / "m.safetensors")
    CT.write_safetensors(p, ts, metadata={"format": "pt"})
    back = CT.read_safetensors(p)
    assert set(back) == set(ts)
    for k, v in ts.items():
        assert back[k].dtype == v.dtype and back[k].shape == v.shape
        assert np.array_equal(back[k], v)
    with open(p, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
    assert n % 8 == 0


def test_safetensors_bf16_and_bad_files(tmp_path):
    import json
    w = np.array([1.0, -2.5, 3.140625, 0.0], np.float32)
    raw = (w.view(np.uint32) >> 16).astype("<u2").tobytes()
    h = json.dumps({"w": {"dtype": "BF16", "shape": [2, 2], "data_offsets": [0, len(raw)]}}).encode()
    p = str(tmp_path / "b.safetensors")
    with open(p, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + raw)
    got = CT.read_safetensors(p)["w"]
    assert got.dtype == np.float32 and np.array_equal(got.reshape(-1), w)
    # header that claims more data than the file holds
    h2 = json.dumps({"w": {"dtype": "F32", "shape": [4], "data_offsets": [0, 64]}}).encode()
    with open(p, "wb") as f:
        f.write(struct.pack("<Q", len(h2)) + h2 + raw)
    with pytest.raises(ValueError):
        CT.read_safetensors(p)
    with open(p, "wb") as f:
        f.write(struct.pack("<Q", 1 << 40))
    with pytest.raises(ValueError):
        CT.read_safetensors(p)


@pytest.mark.parametrize("alignment", [32, 64])
def test_gguf_roundtrip(tmp_path, alignment):
    rng = _rng(2)
    ts = {"blk.0.attn_q.codebook": rng.standard_normal(256).astype(np.float32),
          "blk.0.attn_q.indices": rng.integers(-128, 127, (6, 10)).astype(np.int8),
          "blk.0.attn_q.sc_pos": rng.integers(0, 60, 5).astype(np.int64),
          "blk.0.attn_q.sc_val": rng.standard_normal(5).astype(np.float32),
          "x.f16": rng.standard_normal((3, 3)).astype(np.float16),
          "x.i32": rng.integers(0, 5, (2, 3, 4)).astype(np.int32)}
    p = str(tmp_path / "m.gguf")
    CT.write_gguf(p, ts, metadata={"general.architecture": "llama"}, alignment=alignment)
    back, meta = CT.read_gguf(p)
    assert meta["general.architecture"] == "llama"
    if alignment != 32:
        assert meta["general.alignment"] == alignment
    for k, v in ts.items():
        assert back[k].dtype == v.dtype and back[k].shape == v.shape
        assert np.array_equal(back[k], v)
    assert set(CT.read_tensors(p)) == set(ts)
    with open(p, "r+b") as f:
        f.write(b"GGXX")
    with pytest.raises(ValueError):
        CT.read_gguf(p)


def test_module_grouping():
    names = ["m.l0.q.codebook", "m.l0.q.indices", "m.l0.q.sidecar_positions", "m.l0.q.sidecar_values",
             "m.l1.k.codebook", "m.l1.k.indices", "m.l1.k.sc_pos", "m.l1.k.sc_val",
             "m.l2.v.codebook",                      # no indices: not a module
             "m.norm.weight", "st.attn.gup_ada.0.indi.a1b2c3"]
    mods = CT.hxq_modules(names)
    assert set(mods) == {"m.l0.q", "m.l1.k"}
    assert mods["m.l1.k"]["sidecar_positions"] == "m.l1.k.sc_pos"
    assert set(mods["m.l0.q"]) == set(CT.PARTS)


@pytest.mark.parametrize("vdim,k,out_f,in_f,nnz,dup", [
    (1, 256, 24, 40, 50, 7),     # scalar VQ, uint8 indices
    (1, 100, 7, 9, 10, 0),       # scalar VQ, short codebook, odd sizes
    (2, 4096, 16, 64, 60, 9),    # 2D VQ, 12-bit
    (2, 4096, 5, 10, 12, 3),     # 2D VQ, odd number of pairs per row
    (2, 300, 8, 12, 0, 0),       # 2D VQ without sidecar
])
def test_safetensors_modules_decode_bit_exact(tmp_path, H, L, oracle, vdim, k, out_f, in_f, nnz, dup):
    parts = _module(10 + vdim + out_f, out_f, in_f, vdim, k, nnz, dup=dup)
    p = str(tmp_path / "model.safetensors")
    CT.write_safetensors(p, {f"model.layers.0.mlp.proj.{n}": a for n, a in parts.items()}
                         | {"model.norm.weight": np.ones(in_f, np.float32)})
    mods = CT.load_modules(p)
    assert list(mods) == ["model.layers.0.mlp.proj"]
    d = mods["model.layers.0.mlp.proj"]
    assert d["mode"] == (0 if vdim == 1 else 2)
    assert len(np.unique(d["rows"].astype(np.int64) * in_f + d["cols"])) == \
        (len(np.unique(parts["sidecar_positions"])) if nnz else 0)
    want = container_dense(parts)
    w_orc, w_lib = _decode_all(H, L, oracle, d)
    assert np.array_equal(w_orc.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(w_lib.view(np.uint32), want.view(np.uint32))


def test_gguf_compressed_scalar_module_decodes_bit_exact(tmp_path, H, L, oracle):
    parts = _module(33, 32, 48, 1, 256, 80, spread=4.0, dup=11)
    st = {"blk.3.ffn_down.codebook": parts["codebook"],
          "blk.3.ffn_down.indices": parts["indices"].astype(np.int8),   # as the converter stores them
          "blk.3.ffn_down.sc_pos": parts["sidecar_positions"],
          "blk.3.ffn_down.sc_val": parts["sidecar_values"]}
    p = str(tmp_path / "model.gguf")
    CT.write_gguf(p, st)
    d = CT.load_modules(p)["blk.3.ffn_down"]
    want = container_dense(parts)
    w_orc, w_lib = _decode_all(H, L, oracle, d)
    assert np.array_equal(w_orc.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(w_lib.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("name", golden_names("container_"))
def test_reference_converter_fixtures(H, L, oracle, name):
    """Fixtures made by the reference converter's own dequant_hxq_tensor
    (tools/convert_hxq_to_gguf.py:268-295): the oracle's restatement equals
    it, and the module converted to hxq.c ADD deltas decodes to exactly it
    on the oracle and on the library's CPU backend."""
    g = load_golden(name)
    parts = {k: g[k] for k in ("codebook", "indices", "sidecar_positions", "sidecar_values")}
    want = g["expect"]
    assert np.array_equal(container_dense(parts).view(np.uint32), want.view(np.uint32))
    d = CT.module_tensor(parts)
    assert (d["out_f"], d["in_f"]) == (g["out_f"], g["in_f"])
    w_orc, w_lib = _decode_all(H, L, oracle, d)
    assert np.array_equal(w_orc.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(w_lib.view(np.uint32), want.view(np.uint32))


def test_exact_deltas():
    rng = _rng(5)
    base = rng.standard_normal(20000).astype(np.float32)
    target = np.concatenate([base[:5000] * np.float32(1.0000001),
                             rng.standard_normal(5000).astype(np.float32) * np.float32(30.0),
                             rng.standard_normal(5000).astype(np.float32) * np.float32(1e-4),
                             np.zeros(5000, np.float32)])
    d, reached = CT._exact_deltas(base, target)
    assert d.dtype == np.float32
    # near the codebook value (Sterbenz), or zero: always one add; large
    # targets almost always (unless target - base crosses into a coarser binade)
    assert reached[:5000].all() and reached[15000:].all()
    assert reached[5000:10000].mean() > 0.9
    assert np.array_equal((base + d)[reached].view(np.uint32), target[reached].view(np.uint32))
    # tiny targets under a unit-size codebook value mostly need the two-add form
    assert (~reached[10000:15000]).sum() > 1000


def test_two_add_entries_in_array_order(H, L, oracle):
    cb = np.array([1.0, -3.0, 0.5, 1e3], np.float32)
    idx = np.array([[0, 1, 2, 3], [3, 2, 1, 0]], np.uint8)
    tgt = np.array([1e-7, 2.0, 1.5e-9, -7.25, 0.0, 1e-30], np.float32)
    pos = np.array([0, 1, 2, 3, 4, 7], np.int64)
    parts = {"codebook": cb, "indices": idx, "sidecar_positions": pos, "sidecar_values": tgt}
    d = CT.module_tensor(parts)
    assert len(d["rows"]) > len(pos)
    want = container_dense(parts)
    w_orc, w_lib = _decode_all(H, L, oracle, d)
    assert np.array_equal(w_orc.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(w_lib.view(np.uint32), want.view(np.uint32))


def test_bad_modules_raise():
    cb = np.zeros(4, np.float32)
    with pytest.raises(ValueError):          # index outside the codebook
        CT.module_tensor({"codebook": cb, "indices": np.full((2, 2), 4, np.uint8)})
    with pytest.raises(ValueError):          # sidecar position outside the tensor
        CT.module_tensor({"codebook": cb, "indices": np.zeros((2, 2), np.uint8),
                          "sidecar_positions": np.array([4]), "sidecar_values": np.array([1.0], np.float32)})
    with pytest.raises(ValueError):          # vector dimension 3
        CT.module_tensor({"codebook": np.zeros((4, 3), np.float32), "indices": np.zeros((2, 2), np.int16)})
    with pytest.raises(ValueError):          # 1-D indices
        CT.module_tensor({"codebook": cb, "indices": np.zeros(4, np.uint8)})


@pytest.mark.gpu
@pytest.mark.parametrize("world", [1, 3])
def test_gpu_layers_from_a_model_file(tmp_path, H, L, oracle, cuda, world):
    """A converted model file on the device path, whole and as row shards:
    the dequantized weights equal the file's own weights bit for bit, and
    the fused VQ matmul of the 12-bit module (the tensor-core GEMV: each
    weight rounded to bf16) is within 2^-9 + 1e-5 of sum |x w| of the
    oracle's exact fp32 GEMV of those weights, and within 1e-4 of a float64
    product with the bf16 weights."""
    torch = cuda
    from hxq_b200 import synth
    from hxq_b200.torch_ops import load_linears
    mods = {"m.q": _module(71, 256, 512, 2, 4096, 400, dup=30),
            "m.o": _module(72, 96, 160, 1, 256, 120, dup=10)}
    p = str(tmp_path / "m.safetensors")
    CT.write_safetensors(p, {f"{m}.{n}": a for m, parts in mods.items() for n, a in parts.items()})
    wants = {m: container_dense(parts).reshape(parts["indices"].shape[0], -1) for m, parts in mods.items()}
    for rank in range(world):
        layers = load_linears(p, (rank, world))
        assert set(layers) == set(mods)
        for name, lin in layers.items():
            want = wants[name][lin.row_begin:lin.row_begin + lin.out_features]
            w = lin.weight(torch.float32).cpu().numpy()
            assert np.array_equal(w.view(np.uint32), want.view(np.uint32)), (name, rank)
        q = layers["m.q"]
        assert q.fused
        xh, xf = synth.activations(2, 512, 73)
        x = torch.from_numpy(xh.view(np.int16)).cuda().view(torch.bfloat16)
        y = q(x).cpu().numpy().astype(np.float64)
        Wq = wants["m.q"][q.row_begin:q.row_begin + q.out_features]
        ref = oracle.dense_matmul(xf, Wq).astype(np.float64)
        scale = np.abs(xf.astype(np.float64)) @ np.abs(Wq.astype(np.float64)).T
        assert float((np.abs(y - ref) / np.maximum(scale, 1e-30)).max()) <= 2.0 ** -9 + 1e-5
        Wb = synth.bf16_to_f32(synth.bf16_round(Wq)).astype(np.float64)
        ref64 = xf.astype(np.float64) @ Wb.T
        assert float((np.abs(y - ref64) / np.maximum(scale, 1e-30)).max()) <= 1e-4
    assert os.path.exists(p)
