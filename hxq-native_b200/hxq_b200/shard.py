"""Row sharding of HXQ tensors by out_features.

Rank r of N owns rows [r*O/N, (r+1)*O/N) of every matrix.  Every output row
is independent, so each rank decompresses its rows alone (the driver that
does so is hxq_b200.sharded).  These helpers cut a host-side tensor (the
dict layout of hxq_b200.synth) to a row range with the same rules
hxq_cuda_image_create applies to a loaded tensor.
"""
from __future__ import annotations

import numpy as np


def shard_rows(out_f: int, rank: int, world: int) -> tuple[int, int]:
    return out_f * rank // world, out_f * (rank + 1) // world


def slice_rows(d: dict, r0: int, r1: int) -> dict:
    """Rows [r0, r1) of a scalar or 12-bit tensor, as a tensor of r1 - r0 rows.

    Index bytes: 12-bit rows hold ceil((in_f/2)/2) byte triples each and
    follow each other, so a row range is one contiguous byte range; scalar
    rows are in_f bytes.  Sidecar: entries the reference would apply (row <
    out_f, col < in_f) whose row falls in the range, rebased, in their
    original order."""
    in_f = d["in_f"]
    out = dict(d)
    out["out_f"] = r1 - r0
    if d["mode"] == 2:
        rb = ((in_f // 2) + 1) // 2 * 3
        out["packed"] = np.ascontiguousarray(d["packed"][r0 * rb: r1 * rb])
        if "idx" in d:
            ppr = in_f // 2
            out["idx"] = np.ascontiguousarray(d["idx"][r0 * ppr: r1 * ppr])
    elif d["mode"] == 0:
        out["indices"] = np.ascontiguousarray(d["indices"][r0 * in_f: r1 * in_f])
    else:
        raise ValueError("row slicing covers the VQ modes")
    rows = d.get("rows")
    if rows is not None and len(rows):
        rows = np.asarray(rows, np.uint32)
        cols = np.asarray(d["cols"], np.uint32)
        keep = (rows < d["out_f"]) & (cols < in_f) & (rows >= r0) & (rows < r1)
        out["rows"] = (rows[keep] - np.uint32(r0)).astype(np.uint32)
        out["cols"] = cols[keep]
        out["vals"] = np.asarray(d["vals"], np.float32)[keep]
    return out
