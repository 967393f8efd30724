"""Generate tests/golden/container_*.npz: helix-substrate modules and the
dense weights the reference's own converter makes of them.

The function is `dequant_hxq_tensor` of the reference's
tools/convert_hxq_to_gguf.py (lines 268-295: codebook lookup, then each
sidecar value REPLACES the weight at its flat position, in array order).
That module imports the safetensors and gguf packages at its top, which are
not installed here, so this script reads the file, takes the function's
source with `ast` and runs it unchanged with torch.  Run in a container that
has the reference tree:

    python tests/golden/make_container_golden.py [reference tree]

(default: $HXQ_REFERENCE_TREE, else a directory named `reference` beside
this repository).  The fixtures are small and committed; the tests read
only them.
"""
import ast
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def reference_function(tree_dir: str):
    path = os.path.join(tree_dir, "tools", "convert_hxq_to_gguf.py")
    src = open(path).read()
    mod = ast.parse(src)
    fn = next(n for n in mod.body if isinstance(n, ast.FunctionDef) and n.name == "dequant_hxq_tensor")
    ns = {"torch": torch, "np": np}
    exec(compile(ast.Module(body=[fn], type_ignores=[]), path, "exec"), ns)
    return ns["dequant_hxq_tensor"], fn.lineno


def module(seed, out_f, in_f, vdim, k, nnz, dup):
    """One module as helix-substrate stores it: codebook [k] or [k, 2],
    indices [out_f, in_f / vdim], int64 flat sidecar positions, fp32 target
    values (some far from the codebook value, some zero), `dup` repeated
    positions with new values."""
    rng = np.random.Generator(np.random.PCG64(seed))
    if vdim == 1:
        cb = (rng.standard_normal(k) * 0.05).astype(np.float32)
        idx = rng.integers(0, k, size=(out_f, in_f)).astype(np.uint8 if k <= 256 else np.int16)
    else:
        cb = (rng.standard_normal((k, vdim)) * 0.05).astype(np.float32)
        idx = rng.integers(0, k, size=(out_f, in_f // vdim)).astype(np.int16)
    base = cb[idx.astype(np.int64)].reshape(-1)
    pos = rng.choice(out_f * in_f, size=nnz, replace=False).astype(np.int64)
    pos = np.concatenate([pos, rng.choice(pos, size=dup)])
    vals = (base[pos] + rng.standard_normal(len(pos)).astype(np.float32) * np.float32(0.01)).astype(np.float32)
    vals[:3] *= np.float32(1e3)
    vals[3:6] *= np.float32(1e-3)
    vals[6:8] = 0.0
    return {"codebook": cb, "indices": idx, "sidecar_positions": pos, "sidecar_values": vals}


CASES = {
    "container_scalar_k256_24x40": (11, 24, 40, 1, 256, 60, 7),
    "container_scalar_k100_9x10": (12, 9, 10, 1, 100, 12, 3),
    "container_vq2d_k4096_16x64": (13, 16, 64, 2, 4096, 50, 9),
    "container_vq2d_k300_6x10": (14, 6, 10, 2, 300, 10, 2),
}


def main():
    tree = sys.argv[1] if len(sys.argv) > 1 else (
        os.environ.get("HXQ_REFERENCE_TREE") or os.path.join(os.path.dirname(REPO), "reference"))
    fn, line = reference_function(tree)
    for name, (seed, out_f, in_f, vdim, k, nnz, dup) in CASES.items():
        parts = module(seed, out_f, in_f, vdim, k, nnz, dup)
        W = fn(torch.from_numpy(parts["codebook"]),
               torch.from_numpy(parts["indices"].astype(np.int64)),
               torch.from_numpy(parts["sidecar_positions"]),
               torch.from_numpy(parts["sidecar_values"]), out_f, in_f)
        np.savez(os.path.join(HERE, name + ".npz"), expect=W.numpy().astype(np.float32).reshape(-1),
                 meta_out_f=out_f, meta_in_f=in_f, meta_source_line=line, **parts)
        print("wrote", name)


if __name__ == "__main__":
    main()
