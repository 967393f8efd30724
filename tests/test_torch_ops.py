"""The PyTorch binding (hxq_b200.torch_ops): operators registered with
fake (meta) implementations on CPU; on the GPU, results equal the C ABI's,
bit for bit, and the operators capture into CUDA graphs."""
import ctypes as C

import numpy as np
import pytest

from hxq_b200 import synth


def test_ops_registered_and_fake_shapes():
    import torch
    from torch._subclasses.fake_tensor import FakeTensorMode

    import hxq_b200.torch_ops  # noqa: F401  (registers torch.ops.hxq.*)
    for name in ("dequant", "vq_matmul", "affine_matmul"):
        assert hasattr(torch.ops.hxq, name)
    with FakeTensorMode():
        x = torch.empty((3, 5, 256), dtype=torch.bfloat16, device="cuda")
        y = torch.ops.hxq.vq_matmul(x, 1234, 96)
        assert y.shape == (3, 5, 96) and y.dtype == torch.float32
        codes = torch.empty((64, 256), dtype=torch.uint8, device="cuda")
        s = torch.empty((64, 2), dtype=torch.float32, device="cuda")
        y = torch.ops.hxq.affine_matmul(x, codes, s, s, None, 128)
        assert y.shape == (3, 5, 64)
        w = torch.ops.hxq.dequant(1234, 96, 256, torch.bfloat16)
        assert w.shape == (96, 256) and w.dtype == torch.bfloat16


@pytest.mark.gpu
def test_linear_and_ops_match_the_c_abi(H, L, cuda):
    torch = cuda
    from hxq_b200.torch_ops import HxqLinear
    d = synth.vq12(384, 1024, 17)
    lin = HxqLinear(d, 128, 384)
    assert lin.fused and lin.out_features == 256
    xh, _ = synth.activations(6, 1024, 18)
    x = torch.from_numpy(xh.view(np.int16)).cuda().view(torch.bfloat16).view(2, 3, 1024)
    y = lin(x)
    ref = torch.empty((6, 256), dtype=torch.float32, device="cuda")
    assert L.hxq_cuda_vq_matmul(lin.image, x.data_ptr(), 6, ref.data_ptr(), 256, None) == 0
    torch.cuda.synchronize()
    assert y.shape == (2, 3, 256)
    assert torch.equal(y.reshape(6, 256).view(torch.int32), ref.view(torch.int32))
    # weights: the decompress path, as hxq_cuda_decompress_images
    w = lin.weight(torch.float32)
    w_ref = torch.empty(256 * 1024, dtype=torch.float32, device="cuda")
    imgs = (C.c_void_p * 1)(lin.image)
    offs = (C.c_size_t * 1)(0)
    assert L.hxq_cuda_decompress_images(imgs, 1, w_ref.data_ptr(), offs, H.HXQ_OUT_F32, None, None, None) == 0
    assert L.hxq_cuda_stream_synchronize(None) == 0
    assert torch.equal(w.reshape(-1).view(torch.int32), w_ref.view(torch.int32))
    assert lin.confidence >= 0.0
    # captured into a CUDA graph on a side stream
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        y2 = lin(x)
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        y3 = lin(x)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y3.view(torch.int32), y.view(torch.int32)) and torch.equal(y2, y)


@pytest.mark.gpu
def test_affine_op_matches_the_c_abi(H, L, cuda):
    torch = cuda
    import hxq_b200.torch_ops  # noqa: F401
    d = synth.affine(192, 512, 128, 5, bias=True)
    codes = torch.from_numpy(d["codes"].reshape(192, 512)).cuda()
    sc = torch.from_numpy(d["scales"].reshape(192, 4)).cuda()
    of = torch.from_numpy(d["offsets"].reshape(192, 4)).cuda()
    b = torch.from_numpy(d["bias"]).cuda()
    for N in (1, 7):
        xh, _ = synth.activations(N, 512, 9)
        x = torch.from_numpy(xh.view(np.int16)).cuda().view(torch.bfloat16)
        y = torch.ops.hxq.affine_matmul(x, codes, sc, of, b, 128)
        ref = torch.empty((N, 192), dtype=torch.float32, device="cuda")
        t = H.AffineTensor(codes.data_ptr(), sc.data_ptr(), of.data_ptr(), b.data_ptr(), 192, 512, 128)
        assert L.hxq_affine_group_matmul_bf16(x.data_ptr(), C.byref(t), ref.data_ptr(), N, None) == 0
        torch.cuda.synchronize()
        assert torch.equal(y.view(torch.int32), ref.view(torch.int32))
