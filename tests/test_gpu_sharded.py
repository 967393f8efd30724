"""The model-level driver (hxq_b200.sharded) on one GPU against the oracle.

Ranks of a row-sharded model are emulated on one device by building one
ShardedDecompress per (rank, world) pair with explicit rank/world (no
process group, no collective): every shard must decompress bit-exactly to
its rows of the oracle's whole-matrix result, every shard must report the
reference's confidence for the whole matrix, and the shards' fp64 sums of
squares, added in rank order, must give the exact confidence.  The
column-split fused matmul is checked on one rank (local assembly) against
the oracle's decompress + ordered matmul, and its shards at world 2 against
the whole-matrix product.
"""
import numpy as np
import pytest

from hxq_b200 import synth

pytestmark = pytest.mark.gpu
GEMM_TOL = 2.0 ** -9 + 1e-5


def _bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def _layers():
    # two layers of ragged shapes: row counts that do not split evenly, a
    # scalar matrix, a 12-bit matrix with k = 256, duplicate sidecar rows
    return [[synth.vq12(301, 256, 1, frac=0.02), synth.scalar(77, 96, 2, frac=0.03)],
            [synth.vq12(130, 512, 3, k=256, frac=0.01), synth.vq12(64, 1024, 4, frac=0.05)]]


@pytest.mark.parametrize("world", [1, 3])
def test_sharded_decompress_emulated_ranks(H, L, oracle, cuda, world):
    torch = cuda
    from hxq_b200.sharded import ShardedDecompress, combine_sumsq
    layers = _layers()
    models = [ShardedDecompress(layers, rank=r, world=world, torch=torch, lib=L) for r in range(world)]
    stream = torch.cuda.Stream()
    for li, layer in enumerate(layers):
        for p, d in enumerate(layer):
            err, w_ref, c_ref = oracle.decompress(d)
            assert err == 0
            W = w_ref.reshape(d["out_f"], d["in_f"])
            parts, sumsq = [], []
            for m in models:
                m.decompress_group(m.group_of(li), stream.cuda_stream)
                stream.synchronize()
                assert L.hxq_cuda_stream_synchronize(None) == 0
                parts.append(m.output_view(li, p).cpu().numpy())
                k = sum(len(layers[q]) for q in range(li)) + p
                sumsq.append(float(m.sumsq[k].item()))
                # the reference's value for the whole matrix, on every shard
                assert np.float32(m.reference_confidences()[k]) == np.float32(c_ref)
                if world == 1:
                    assert np.float32(m.conf[k].item()) == np.float32(c_ref)
            assert np.array_equal(_bits(np.concatenate(parts)), _bits(W)), (li, p)
            exact = oracle.l2_exact(d)
            assert abs(combine_sumsq(sumsq) - exact) <= 1e-6 * max(exact, 1e-30)
    for m in models:
        assert m.numel() == sum(mm["numel"] for lm in m.meta for mm in lm)
        m.close()
    assert sum(m.n_matrices for m in models) == 4 * world


def test_sharded_stream_step_and_restore(H, L, oracle, cuda):
    """stream_step: images copied from pinned host memory every step (copy
    stream) and decompressed on the compute stream; restore_pool points the
    images back at the resident pool."""
    torch = cuda
    from hxq_b200.sharded import ShardedDecompress
    layers = _layers()
    m = ShardedDecompress(layers, rank=0, world=1, torch=torch, lib=L)
    copy_s, comp_s = torch.cuda.Stream(), torch.cuda.Stream()
    host_conf = torch.empty(m.n_matrices, dtype=torch.float32, pin_memory=True)
    for _ in range(2):
        m.stream_step(copy_s, comp_s, host_conf)
    comp_s.synchronize()
    assert L.hxq_cuda_stream_synchronize(None) == 0
    last = len(layers) - 1
    for p, d in enumerate(layers[last]):
        err, w_ref, c_ref = oracle.decompress(d)
        got = m.output_view(last, p).cpu().numpy().ravel()
        assert np.array_equal(_bits(got), _bits(w_ref)), p
    refs = [oracle.decompress(d)[2] for layer in layers for d in layer]
    assert np.array_equal(_bits(host_conf.numpy()), _bits(np.array(refs, np.float32)))
    m.restore_pool()
    stream = torch.cuda.Stream()
    m.step(stream.cuda_stream)
    stream.synchronize()
    for p, d in enumerate(layers[last]):
        got = m.output_view(last, p).cpu().numpy().ravel()
        assert np.array_equal(_bits(got), _bits(oracle.decompress(d)[1])), p
    m.close()


def _mats(seed=7):
    mats = []
    for j, (O, I) in enumerate(((256, 512), (384, 512), (256, 1024))):
        mats.append(dict(name=f"m{j}", O=O, I=I, vq=synth.vq12(O, I, seed + j, frac=0.01),
                         affine=synth.affine(O, I, 128, seed + 100 + j)))
    return mats


@pytest.mark.parametrize("fmt", ["vq12", "affine"])
@pytest.mark.parametrize("N", [1, 3])
def test_column_split_layer_local_and_shards(H, L, oracle, cuda, fmt, N):
    torch = cuda
    from hxq_b200.sharded import ColumnSplitLayer
    mats = _mats()
    xs_h = {I: synth.activations(N, I, 50 + I) for I in (512, 1024)}
    xs = {I: torch.from_numpy(h.view(np.int16)).cuda() for I, (h, _) in xs_h.items()}
    stream = torch.cuda.Stream()
    whole = ColumnSplitLayer(mats, fmt, max_tokens=N, rank=0, world=1, torch=torch, lib=L)
    whole.forward(xs, N, stream)
    shards = [ColumnSplitLayer(mats, fmt, max_tokens=N, rank=r, world=2, torch=torch, lib=L) for r in range(2)]
    for s in shards:
        s.forward(xs, N, stream, assembly="local")
    stream.synchronize()
    if fmt == "vq12":
        assert L.hxq_cuda_affine_device_status() == 0
    outs = [y.cpu().numpy() for y in whole.outputs(N)]
    for j, m in enumerate(mats):
        x = xs_h[m["I"]][1]
        if fmt == "vq12":
            err, w, _ = oracle.decompress(m["vq"])
            W = w.reshape(m["O"], m["I"])
        else:
            W = oracle.affine_decompress(m["affine"]).reshape(m["O"], m["I"])
        y_ref = oracle.dense_matmul(x, W)
        scale = np.abs(x.astype(np.float64)) @ np.abs(W.astype(np.float64)).T
        err_n = np.abs(outs[j].astype(np.float64) - y_ref) / np.maximum(scale, 1e-30)
        assert float(err_n.max()) <= GEMM_TOL, (fmt, N, j, float(err_n.max()))
        # the two row shards are the whole matrix's columns, bit for bit
        cat = np.concatenate([s.local_outputs(N)[j].cpu().numpy() for s in shards], axis=1)
        assert np.array_equal(_bits(cat), _bits(outs[j])), (fmt, N, j)
    for layer in [whole] + shards:
        layer.close()
