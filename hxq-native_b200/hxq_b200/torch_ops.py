"""PyTorch binding of the HXQ CUDA path: custom operators over the C ABI of
libhxq.so and a linear layer whose weight stays compressed on the GPU.

This is the framework glue the reference describes (README "Integration
Paths": a framework calls hxq_dequant and then its own matmul), plus the
fused paths of this library:

    torch.ops.hxq.dequant(image, rows, in_features, dtype)   -> weights
    torch.ops.hxq.vq_matmul(x_bf16, image, rows)             -> x @ W.T (fp32)
    torch.ops.hxq.affine_matmul(x_bf16, codes, scales, offsets, bias, gs)

`image` is the integer handle of an hxq_cuda_image_t (see HxqLinear).  Every
operator runs on the caller's current CUDA stream, allocates its output
with PyTorch's allocator, and has a fake (meta) implementation for shape
propagation.  There is no CPU implementation: without the CUDA library the
operators raise.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import (HXQ_IMAGE_MATMUL, HXQ_OUT_BF16, HXQ_OUT_F32, AffineTensor, Tensor, check, lib)

_DT = {torch.float32: HXQ_OUT_F32, torch.bfloat16: HXQ_OUT_BF16}


def _stream() -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


@torch.library.custom_op("hxq::dequant", mutates_args=())
def dequant(image: int, rows: int, in_features: int, dtype: torch.dtype) -> torch.Tensor:
    """Decompressed weights [rows, in_features] of an image (codebook +
    sidecar, the reference's decode), fp32 or bf16."""
    if dtype not in _DT:
        raise ValueError("dtype must be torch.float32 or torch.bfloat16")
    L = lib()
    out = torch.empty((rows, in_features), dtype=dtype, device="cuda")
    imgs = (C.c_void_p * 1)(image)
    offs = (C.c_size_t * 1)(0)
    check(L.hxq_cuda_decompress_images(imgs, 1, out.data_ptr(), offs, _DT[dtype], None, None, _stream()),
          "hxq_cuda_decompress_images")
    return out


@dequant.register_fake
def _(image, rows, in_features, dtype):
    return torch.empty((rows, in_features), dtype=dtype, device="cuda")


@torch.library.custom_op("hxq::vq_matmul", mutates_args=())
def vq_matmul(x: torch.Tensor, image: int, rows: int) -> torch.Tensor:
    """x [..., in_features] (bf16, CUDA) times the image's weights
    transposed: [..., rows] fp32, without dense weights in memory."""
    if x.dtype != torch.bfloat16 or not x.is_cuda:
        raise ValueError("x must be a bf16 CUDA tensor")
    xc = x.contiguous()
    n = xc.numel() // xc.shape[-1] if xc.dim() else 1
    y = torch.empty((*x.shape[:-1], rows), dtype=torch.float32, device=x.device)
    check(lib().hxq_cuda_vq_matmul(image, xc.data_ptr(), n, y.data_ptr(), rows, _stream()), "hxq_cuda_vq_matmul")
    return y


@vq_matmul.register_fake
def _(x, image, rows):
    return x.new_empty((*x.shape[:-1], rows), dtype=torch.float32)


@torch.library.custom_op("hxq::affine_matmul", mutates_args=())
def affine_matmul(x: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor, offsets: torch.Tensor,
                  bias: torch.Tensor | None, group_size: int) -> torch.Tensor:
    """x [..., in_features] (bf16, CUDA) times the affine group-quantized
    weights (codes uint8 [out, in], scales/offsets fp32 [out, in/gs])
    transposed, plus bias: [..., out] fp32."""
    if x.dtype != torch.bfloat16 or not x.is_cuda:
        raise ValueError("x must be a bf16 CUDA tensor")
    out_f, in_f = codes.shape
    xc = x.contiguous()
    n = xc.numel() // in_f
    y = torch.empty((*x.shape[:-1], out_f), dtype=torch.float32, device=x.device)
    t = AffineTensor(codes.data_ptr(), scales.data_ptr(), offsets.data_ptr(),
                     None if bias is None else bias.data_ptr(), out_f, in_f, group_size)
    if lib().hxq_affine_group_matmul_bf16(xc.data_ptr(), C.byref(t), y.data_ptr(), n, _stream()) != 0:
        raise RuntimeError("hxq_affine_group_matmul_bf16 failed")
    return y


@affine_matmul.register_fake
def _(x, codes, scales, offsets, bias, group_size):
    return x.new_empty((*x.shape[:-1], codes.shape[0]), dtype=torch.float32)


class HxqLinear(torch.nn.Module):
    """A linear layer (no bias) whose weight is an HXQ tensor kept compressed
    on the GPU: 12-bit 2D-VQ tensors run the fused VQ matmul, other modes
    decompress through the device path and use torch.matmul.  `tensor` is a
    dict as accepted by hxq_b200.Tensor.load (or a loaded Tensor);
    [row_begin, row_end) selects the output features this module holds
    (a tensor-parallel shard)."""

    def __init__(self, tensor, row_begin: int = 0, row_end: int | None = None):
        super().__init__()
        self._t = tensor if isinstance(tensor, Tensor) else Tensor().load(tensor)
        desc = self._t.t
        self.in_features = int(desc.in_features)
        self.row_begin = row_begin
        self.out_features = (int(desc.out_features) if row_end is None else row_end) - row_begin
        self._img = C.c_void_p()
        L = lib()
        check(L.hxq_cuda_image_create_ex(self._t.ref, row_begin, row_begin + self.out_features,
                                         HXQ_IMAGE_MATMUL, C.byref(self._img)), "hxq_cuda_image_create_ex")
        self.fused = int(desc.mode) == 2 and int(desc.k) == 4096 and self.in_features % 64 == 0

    @property
    def image(self) -> int:
        return int(self._img.value)

    @property
    def confidence(self) -> float:
        """The sidecar L2 of the module's rows, as the reference computes it."""
        return float(lib().hxq_cuda_image_reference_confidence(self._img))

    def weight(self, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        return dequant(self.image, self.out_features, self.in_features, dtype)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.fused:
            return vq_matmul(x.to(torch.bfloat16), self.image, self.out_features)
        return torch.matmul(x.float(), self.weight(torch.float32).t())

    def __del__(self):
        img = getattr(self, "_img", None)
        if img is not None and img.value:
            try:
                lib().hxq_cuda_image_destroy(img)
            except Exception:
                pass
            self._img = C.c_void_p()


def load_linears(path: str, shard: tuple[int, int] = (0, 1)) -> dict[str, HxqLinear]:
    """HxqLinear layers for every compressed module of a helix-substrate
    safetensors or GGUF file (hxq_b200.container), keyed by module prefix.
    shard=(rank, world) keeps this rank's contiguous share of each module's
    output features: rows [rank*O//world, (rank+1)*O//world)."""
    from .container import load_modules
    rank, world = shard
    if not 0 <= rank < world:
        raise ValueError("shard must be (rank, world) with 0 <= rank < world")
    out = {}
    for name, d in load_modules(path).items():
        O = d["out_f"]
        out[name] = HxqLinear(d, rank * O // world, (rank + 1) * O // world)
    return out
