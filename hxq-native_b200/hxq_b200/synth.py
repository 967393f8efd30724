"""Seeded synthetic HXQ tensors with the shapes and value distributions of
the benchmark workloads (no real checkpoints are available).

  vq12:    k=4096 x dim-2 fp32 codebook ~N(0, 0.02); indices uniform in
           [0, 4096) packed two per 3 bytes, rows of ceil((in_f/2)/2)
           triples; sidecar at floor(frac * out_f * in_f) unique uniformly
           random coordinates sorted row-major, deltas ~N(0, 0.005).
  scalar:  k=256 fp32 codebook ~N(0, 0.02) sorted ascending; uint8 indices
           uniform; sidecar 0.1%, deltas ~N(0, 0.002).
  affine:  4-bit codes uniform in [0, 16) stored one per byte; per-group
           scale ~U(0.001, 0.01), zero point z uniform in [0, 16) and
           offset = -z * scale (fp32); activations bf16 = RNE(N(0, 1) fp32).

Everything is drawn from numpy's PCG64 with an explicit seed, so tests,
benchmarks and fixtures regenerate identical inputs.
"""
from __future__ import annotations

import numpy as np

from . import HXQ_AFFINE_G128, HXQ_SCALAR_VQ, HXQ_VQ2D_12BIT


def _rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def _u16(rng: np.random.Generator, n: int) -> np.ndarray:
    raw = rng.bit_generator.random_raw((n + 3) // 4)
    return raw.view(np.uint16)[:n].copy()


def _bytes(rng: np.random.Generator, n: int) -> np.ndarray:
    raw = rng.bit_generator.random_raw((n + 7) // 8)
    return raw.view(np.uint8)[:n].copy()


def pack12(idx: np.ndarray, out_f: int, in_f: int) -> np.ndarray:
    """Pack out_f*(in_f//2) 12-bit indices into the row layout the decoder
    reads: per row ceil(pairs/2) triples, an odd last pair padded with 0."""
    ppr = in_f // 2
    idx = np.asarray(idx, dtype=np.uint16).reshape(out_f, ppr)
    if ppr % 2:
        idx = np.concatenate([idx, np.zeros((out_f, 1), np.uint16)], axis=1)
    a = idx[:, 0::2].astype(np.uint32)
    b = idx[:, 1::2].astype(np.uint32)
    out = np.empty(a.shape + (3,), np.uint8)
    out[..., 0] = (a >> 4) & 0xFF
    out[..., 1] = ((a & 0xF) << 4) | (b >> 8)
    out[..., 2] = b & 0xFF
    return out.reshape(-1)


def unpack12(packed: np.ndarray, out_f: int, in_f: int) -> np.ndarray:
    """Inverse of pack12 (padding dropped)."""
    ppr = in_f // 2
    tpr = (ppr + 1) // 2
    t = np.asarray(packed, dtype=np.uint8)[: out_f * tpr * 3].reshape(out_f, tpr, 3).astype(np.uint16)
    a = (t[..., 0] << 4) | (t[..., 1] >> 4)
    b = ((t[..., 1] & 0xF) << 8) | t[..., 2]
    both = np.stack([a, b], axis=-1).reshape(out_f, 2 * tpr)
    return both[:, :ppr].reshape(-1)


def sidecar(rng: np.random.Generator, out_f: int, in_f: int, frac: float, std: float,
            nnz: int | None = None):
    n = out_f * in_f
    if nnz is None:
        nnz = int(np.floor(frac * n))
    nnz = min(nnz, n)
    if nnz == 0:
        z = np.zeros(0, np.uint32)
        return z, z.copy(), np.zeros(0, np.float32)
    pos = np.sort(rng.choice(n, size=nnz, replace=False)).astype(np.uint64)
    rows = (pos // in_f).astype(np.uint32)
    cols = (pos % in_f).astype(np.uint32)
    vals = (rng.standard_normal(nnz, dtype=np.float32) * np.float32(std)).astype(np.float32)
    return rows, cols, vals


def vq12(out_f: int, in_f: int, seed: int, frac: float = 0.005, delta_std: float = 0.005,
         cb_std: float = 0.02, k: int = 4096, nnz: int | None = None) -> dict:
    rng = _rng(seed)
    cb = (rng.standard_normal(k * 2, dtype=np.float32) * np.float32(cb_std)).astype(np.float32)
    n_idx = out_f * (in_f // 2)
    idx = _u16(rng, n_idx) & np.uint16(0xFFF)
    if k < 4096:
        idx = (idx % np.uint16(k)).astype(np.uint16)
    packed = pack12(idx, out_f, in_f)
    rows, cols, vals = sidecar(rng, out_f, in_f, frac, delta_std, nnz)
    return dict(mode=HXQ_VQ2D_12BIT, out_f=out_f, in_f=in_f, k=k, vdim=2, codebook=cb,
                idx=idx, packed=packed, rows=rows, cols=cols, vals=vals)


def scalar(out_f: int, in_f: int, seed: int, frac: float = 0.001, delta_std: float = 0.002,
           cb_std: float = 0.02, nnz: int | None = None) -> dict:
    rng = _rng(seed)
    cb = np.sort(rng.standard_normal(256, dtype=np.float32) * np.float32(cb_std)).astype(np.float32)
    indices = _bytes(rng, out_f * in_f)
    rows, cols, vals = sidecar(rng, out_f, in_f, frac, delta_std, nnz)
    return dict(mode=HXQ_SCALAR_VQ, out_f=out_f, in_f=in_f, k=256, vdim=1, codebook=cb,
                indices=indices, rows=rows, cols=cols, vals=vals)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (nearest-even) and return the bf16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def affine(out_f: int, in_f: int, gs: int, seed: int, bias: bool = False) -> dict:
    rng = _rng(seed)
    ng = in_f // gs
    codes = (_bytes(rng, out_f * in_f) & np.uint8(15)).astype(np.uint8)
    scales = (rng.random(out_f * ng, dtype=np.float32) * np.float32(0.009) + np.float32(0.001)).astype(np.float32)
    zero = (_bytes(rng, out_f * ng) & np.uint8(15)).astype(np.float32)
    offsets = (np.float32(-1.0) * zero * scales).astype(np.float32)
    b = (rng.standard_normal(out_f, dtype=np.float32) * np.float32(0.1)).astype(np.float32) if bias else None
    return dict(mode=HXQ_AFFINE_G128, out_f=out_f, in_f=in_f, gs=gs, codes=codes, scales=scales,
                offsets=offsets, zero=zero.astype(np.uint8), bias=b, rows=None)


def activations(n: int, in_f: int, seed: int):
    """bf16 activations ~N(0,1): (bf16 bit patterns, the same values as fp32)."""
    rng = _rng(seed)
    x = rng.standard_normal(n * in_f, dtype=np.float32).reshape(n, in_f)
    h = bf16_round(x).reshape(n, in_f)
    return h, bf16_to_f32(h).reshape(n, in_f)


# Seeds of the benchmark workloads.
SEED_BASE = 0x485851
SEED_C1 = SEED_BASE + 1
SEED_C2 = SEED_BASE + 2
SEED_C3 = SEED_BASE + 3
SEED_C4 = SEED_BASE + 4
SEED_C5 = SEED_BASE + 5

LLAMA7B_PROJ = (("q", 4096, 4096), ("k", 4096, 4096), ("v", 4096, 4096), ("o", 4096, 4096),
                ("gate", 11008, 4096), ("up", 11008, 4096), ("down", 4096, 11008))


def llama7b_seed(layer: int, proj: int) -> int:
    return SEED_C4 + 7 * layer + proj
