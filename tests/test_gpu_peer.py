"""Outputs stored into several buffers (the shape a node-local output split
uses: every rank's buffer, local or peer-mapped) and the step flags, on one
GPU.  Several outputs must be bit-identical to the single-output call at the
given column offsets; a signal/wait round must complete with status 0; a
wait on a flag nothing sets must run out (about two seconds) and report it
through the status word, leaving the context usable."""
import ctypes as C
import time

import numpy as np
import pytest

from hxq_b200 import synth

pytestmark = pytest.mark.gpu


def _ptrs(*ts):
    return (C.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


@pytest.mark.parametrize("N", [1, 3, 40])
def test_vq_matmul_multi_outputs(H, L, cuda, N):
    torch = cuda
    out_f, in_f = 600, 1024
    d = synth.vq12(out_f, in_f, 5 + N)
    t = H.Tensor().load(d)
    r0, r1 = 200, 600
    img = C.c_void_p()
    assert L.hxq_cuda_image_create_ex(t.ref, r0, r1, H.HXQ_IMAGE_MATMUL, C.byref(img)) == 0
    try:
        xh, _ = synth.activations(N, in_f, 7)
        x = torch.from_numpy(xh.view(np.int16)).cuda()
        ref = torch.full((N, r1 - r0), float("nan"), device="cuda")
        assert L.hxq_cuda_vq_matmul(img, x.data_ptr(), N, ref.data_ptr(), r1 - r0, None) == 0
        outs = [torch.full((N, out_f), float("nan"), device="cuda") for _ in range(3)]
        ys = (C.c_void_p * 3)(*[o.data_ptr() + 4 * r0 for o in outs])
        assert L.hxq_cuda_vq_matmul_multi(img, x.data_ptr(), N, ys, 3, out_f, None) == 0
        torch.cuda.synchronize()
        for o in outs:
            assert torch.equal(o[:, r0:r1].contiguous().view(torch.int32), ref.view(torch.int32))
            assert bool(torch.isnan(o[:, :r0]).all())
        assert L.hxq_cuda_affine_device_status() == 0
        assert L.hxq_cuda_vq_matmul_multi(img, x.data_ptr(), N, ys, 9, out_f, None) == H.HXQ_ERR_INVALID_ARG
    finally:
        L.hxq_cuda_image_destroy(img)


@pytest.mark.parametrize("N", [1, 5, 300])
def test_affine_matmul_multi_outputs(H, L, cuda, N):
    torch = cuda
    O, I, gs = 384, 512, 128
    d = synth.affine(O, I, gs, 9 + N, bias=True)
    codes = torch.from_numpy(d["codes"]).cuda()
    sc = torch.from_numpy(d["scales"]).cuda()
    of = torch.from_numpy(d["offsets"]).cuda()
    bias = torch.from_numpy(d["bias"]).cuda()
    at = H.AffineTensor(codes.data_ptr(), sc.data_ptr(), of.data_ptr(), bias.data_ptr(), O, I, gs)
    xh, _ = synth.activations(N, I, 3)
    x = torch.from_numpy(xh.view(np.int16)).cuda()
    ref = torch.empty((N, O), device="cuda")
    assert L.hxq_affine_group_matmul_bf16(x.data_ptr(), C.byref(at), ref.data_ptr(), N, None) == 0
    ld = O + 100
    outs = [torch.full((N, ld), float("nan"), device="cuda") for _ in range(2)]
    ys = (C.c_void_p * 2)(*[o.data_ptr() + 4 * 50 for o in outs])
    assert L.hxq_affine_group_matmul_bf16_multi(x.data_ptr(), C.byref(at), ys, 2, ld, N, None) == 0
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o[:, 50:50 + O].contiguous().view(torch.int32), ref.view(torch.int32))
        assert bool(torch.isnan(o[:, :50]).all()) and bool(torch.isnan(o[:, 50 + O:]).all())
    assert L.hxq_cuda_affine_device_status() == 0


def test_signal_then_wait_one_rank(H, L, cuda):
    torch = cuda
    flags = torch.zeros(8, dtype=torch.int32, device="cuda")
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    peers = (C.c_void_p * 1)(flags.data_ptr())
    for step in range(1, 4):
        assert L.hxq_cuda_peer_signal(peers, 1, 0, counter.data_ptr(), None) == 0
        assert L.hxq_cuda_peer_wait(flags.data_ptr(), 1, counter.data_ptr(), status.data_ptr(), None) == 0
        torch.cuda.synchronize()
        assert int(counter.item()) == step and int(flags[0].item()) == step
    assert int(status.item()) == 0


def test_wait_runs_out_on_a_flag_nothing_sets(H, L, cuda):
    """Two ranks' slots, only this rank signals: the wait gives up after its
    bound, sets the status word and returns; the context stays usable."""
    torch = cuda
    flags = torch.zeros(8, dtype=torch.int32, device="cuda")
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    other = torch.zeros(8, dtype=torch.int32, device="cuda")     # stands in for the absent peer
    peers = (C.c_void_p * 2)(flags.data_ptr(), other.data_ptr())
    assert L.hxq_cuda_peer_signal(peers, 2, 0, counter.data_ptr(), None) == 0
    t0 = time.time()
    assert L.hxq_cuda_peer_wait(flags.data_ptr(), 2, counter.data_ptr(), status.data_ptr(), None) == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 1
    assert time.time() - t0 < 30
    y = torch.ones(4, device="cuda") * 2     # the context still works
    assert float(y.sum().item()) == 8.0
    assert L.hxq_cuda_peer_wait(flags.data_ptr(), 0, counter.data_ptr(), status.data_ptr(), None) == H.HXQ_ERR_INVALID_ARG
