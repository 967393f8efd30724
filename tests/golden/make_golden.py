"""Generate tests/golden/*.npz: seeded inputs and the outputs the reference
library itself produces for them.

The reference (hxq-native src/hxq.c and src/hxq_affine.c) is compiled from
its own sources by `make -C oracle ref` into oracle/_ref/libhxqref.so; this
script runs it and stores inputs + outputs, so parity tests on machines
without the reference tree still compare against the reference's answers.

    make -C oracle ref && python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "hxq-native_b200"))

from hxq_b200 import synth  # noqa: E402
from oracle.oracle import Reference  # noqa: E402


def _save(name: str, d: dict, **extra) -> None:
    arrays = {}
    meta = {}
    for k, v in list(d.items()) + list(extra.items()):
        if v is None:
            continue
        if isinstance(v, np.ndarray):
            arrays[k] = v
        else:
            meta[k] = v
    for k, v in meta.items():
        arrays["meta_" + k] = np.asarray(v)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrays)


def decompress_case(ref: Reference, name: str, d: dict, out_init: np.ndarray | None = None,
                    **kw) -> None:
    n = d["out_f"] * d["in_f"]
    init = np.zeros(n, np.float32) if out_init is None else out_init.astype(np.float32)
    err, w, conf = ref.decompress(d, out=init.copy(), **kw)
    extra = dict(out_init=init, expect_err=int(err), expect_w=w,
                 expect_conf=np.float32(conf if conf is not None else np.nan))
    for key in ("idx_len", "k", "vdim"):
        if key in kw and kw[key] is not None:
            extra["call_" + key] = int(kw[key])
    _save(name, d, **extra)


def main() -> None:
    ref = Reference()
    # ordinary 12-bit tensor, 0.5% sidecar
    decompress_case(ref, "vq12_64x256", synth.vq12(64, 256, 101))
    # rows with an odd pair count, heavy sidecar
    decompress_case(ref, "vq12_odd_6x10", synth.vq12(6, 10, 102, frac=0.3))
    # in_f = 7: the last column of every row is never written by the decoder
    d = synth.vq12(5, 7, 103, frac=0.4)
    decompress_case(ref, "vq12_ragged_5x7", d, out_init=np.arange(35, dtype=np.float32) * 0.5)
    # duplicates, out-of-range and unsorted sidecar entries
    d = synth.vq12(16, 64, 104, frac=0.05)
    rng = np.random.default_rng(104)
    extra_r = np.array([3, 3, 3, 16, 2, 100, 7, 0], np.uint32)
    extra_c = np.array([5, 5, 5, 1, 64, 3, 63, 0], np.uint32)
    extra_v = rng.standard_normal(8).astype(np.float32)
    order = rng.permutation(len(d["rows"]) + 8)
    d["rows"] = np.concatenate([d["rows"], extra_r])[order]
    d["cols"] = np.concatenate([d["cols"], extra_c])[order]
    d["vals"] = np.concatenate([d["vals"], extra_v])[order]
    decompress_case(ref, "vq12_dups_16x64", d)
    # k = 256 codebook with 12-bit indices (all in range)
    decompress_case(ref, "vq12_k256_32x128", synth.vq12(32, 128, 105, k=256))
    # k = 256 with one index >= k: INDEX_OOB
    d = synth.vq12(8, 64, 106, k=256)
    idx = d["idx"].copy()
    idx[37] = 300
    d["idx"] = idx
    d["packed"] = synth.pack12(idx, 8, 64)
    decompress_case(ref, "vq12_oob_8x64", d)
    # short packed stream: PACK_FORMAT; and an OOB index before the shortfall
    d = synth.vq12(8, 64, 107)
    decompress_case(ref, "vq12_short_8x64", d, idx_len=len(d["packed"]) - 5)
    d = synth.vq12(8, 64, 108, k=256)
    idx = d["idx"].copy()
    idx[3] = 4000
    d["idx"] = idx
    d["packed"] = synth.pack12(idx, 8, 64)
    decompress_case(ref, "vq12_short_oob_8x64", d, idx_len=len(d["packed"]) - 5)
    # scalar k=256
    decompress_case(ref, "scalar_64x96", synth.scalar(64, 96, 109, frac=0.01))
    d = synth.scalar(9, 13, 110, frac=0.1)  # ragged size, duplicates appended
    d["rows"] = np.concatenate([d["rows"], np.array([4, 4, 8], np.uint32)])
    d["cols"] = np.concatenate([d["cols"], np.array([7, 7, 12], np.uint32)])
    d["vals"] = np.concatenate([d["vals"], np.array([0.25, -0.125, 1.5], np.float32)])
    decompress_case(ref, "scalar_dups_9x13", d)
    # affine dense dequant through hxq_tensor_decompress, with a sidecar
    d = synth.affine(16, 256, 128, 111)
    rr, cc, vv = synth.sidecar(np.random.default_rng(111), 16, 256, 0.02, 0.01)
    d.update(rows=rr, cols=cc, vals=vv)
    decompress_case(ref, "affine_dq_16x256", d)
    # fused affine matmul, several batches, gs 128 and 32, with/without bias
    for name, (O, I, gs, N, bias, seed) in {
        "affine_mm_64x256_n1": (64, 256, 128, 1, False, 112),
        "affine_mm_64x256_n3_bias": (64, 256, 128, 3, True, 113),
        "affine_mm_48x512_n8_g32": (48, 512, 32, 8, True, 114),
    }.items():
        d = synth.affine(O, I, gs, seed, bias=bias)
        _, x = synth.activations(N, I, seed + 1000)
        y = ref.affine_matmul(x, d, bias=d["bias"])
        _save(name, d, x=x, expect_y=y)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
