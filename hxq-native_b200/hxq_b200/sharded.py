"""Model-level multi-GPU driver: whole weight matrices sharded by
out_features over the GPUs of one node, one process per GPU.

The reference library has no multi-GPU code; this is the driver the
B200 build adds around its C ABI (libhxq.so), with torch.distributed for
process-group plumbing and NCCL.

Decompress (`ShardedDecompress`): rank r of N owns rows
[r*O/N, (r+1)*O/N) of every matrix (`shard.shard_rows`), builds device
images of exactly those rows (`hxq_cuda_image_create_streamed` with a row
range, uploaded once into one device pool) and decompresses them where the
weights are consumed, so there is no collective on this path.  Launches
cover groups of layers (as many layers as ranks, at most 8), so every launch
carries about one layer's weights whatever N is; one device arena holds one
group and is reused by all groups, as the reference reuses its shared
buffer.  Each matrix reports two confidences: the reference's own value for
the whole matrix (hxq.c's fp32 running sum, carried by every shard's image)
and the exact value from the shards' fp64 sums of squares, added in rank
order.

Fused matmul (`ColumnSplitLayer`): output features are split the same way;
every rank multiplies the full activations by its rows (tensor-core GEMV or
tcgen05 GEMM inside libhxq) and the output shards are assembled either by an
NCCL all-gather into [ranks * tokens, rows] (a permute gives [tokens, O]) or
inside the matmul epilogues: every rank's [tokens, O] output buffer is mapped
into every other rank (CUDA IPC) and each output element is stored into all
of them over NVLink, then one flag kernel tells the peers and one bounded
wait kernel waits for theirs.  Two output buffers alternate by step parity,
so a rank never overwrites outputs a peer may still read.
"""
from __future__ import annotations

import ctypes as C
from typing import Callable, Sequence

import numpy as np

from .shard import shard_rows

MAX_LAYERS_PER_LAUNCH = 8
_ALIGN = 256


def _align(x: int) -> int:
    return (x + _ALIGN - 1) // _ALIGN * _ALIGN


def launch_groups(n_layers: int, world: int, max_layers: int = MAX_LAYERS_PER_LAUNCH) -> list[list[int]]:
    """Layers per decompress launch: as many layers as ranks (at most
    max_layers), so a rank's launch holds about one full layer's weights."""
    per = max(1, min(max_layers, world, n_layers))
    return [list(range(g, min(g + per, n_layers))) for g in range(0, n_layers, per)]


def packed_offsets(numels: Sequence[int]) -> tuple[list[int], int]:
    """Element offsets of consecutive outputs and their total."""
    offs, pos = [], 0
    for n in numels:
        offs.append(pos)
        pos += int(n)
    return offs, pos


def combine_sumsq(per_rank: Sequence[float]) -> float:
    """Exact confidence of a row-sharded matrix: sqrt of the shards' sums of
    squared sidecar deltas added in rank order (deterministic), as fp32."""
    total = 0.0
    for s in per_rank:
        total += float(s)
    return float(np.float32(np.sqrt(total)))


def assemble_gathered(gathered, world: int, tokens: int, rows: int):
    """[ranks * tokens, rows] from an all-gather of equal row shards ->
    [tokens, ranks * rows] (works on torch tensors and numpy arrays)."""
    g = gathered.reshape(world, tokens, rows)
    if hasattr(g, "permute"):
        return g.permute(1, 0, 2).reshape(tokens, world * rows)
    return g.transpose(1, 0, 2).reshape(tokens, world * rows)


def _rank_world(rank, world):
    if rank is not None and world is not None:
        return rank, world
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


# ---------------------------------------------------------------------------
# Row-sharded decompress

class ShardedDecompress:
    """This rank's row shards of a model's VQ matrices, resident in HBM.

    layers: a sequence of layers, each a sequence of matrices; a matrix is a
        host dict in the hxq_b200.synth layout (scalar or 12-bit VQ) or a
        zero-argument callable returning one (so only one full matrix needs
        to be on the host at a time).  Every rank passes the same matrices.
    Each image keeps its pinned host block too, so `stream_step` can time
    weights that live on the host and cross PCIe each step.
    """

    def __init__(self, layers: Sequence[Sequence[dict | Callable[[], dict]]], *, rank: int | None = None,
                 world: int | None = None, torch=None, lib=None, log: Callable[[str], None] | None = None):
        import hxq_b200 as H
        if torch is None:
            import torch as _torch
            torch = _torch
        self.H, self.L, self.torch = H, (lib or H.lib()), torch
        self.rank, self.world = _rank_world(rank, world)
        L = self.L
        self.imgs: list[list[C.c_void_p]] = []
        self.meta: list[list[dict]] = []
        for li, layer in enumerate(layers):
            imgs, meta = [], []
            for m in layer:
                d = m() if callable(m) else m
                out_f, in_f = int(d["out_f"]), int(d["in_f"])
                r0, r1 = shard_rows(out_f, self.rank, self.world)
                t = H.Tensor().load(d)
                img = C.c_void_p()
                H.check(L.hxq_cuda_image_create_streamed(t.ref, r0, r1, C.byref(img)), "image")
                t.free()
                rows = np.asarray(d.get("rows") if d.get("rows") is not None else [], np.int64)
                cols = np.asarray(d.get("cols") if d.get("cols") is not None else [], np.int64)
                nnz = int(np.count_nonzero((rows >= r0) & (rows < r1) & (cols < in_f))) if rows.size else 0
                imgs.append(img)
                meta.append(dict(row_begin=r0, rows=r1 - r0, out_f=out_f, in_f=in_f, nnz=nnz,
                                 numel=(r1 - r0) * in_f, block=int(L.hxq_cuda_image_block_bytes(img)),
                                 mode=int(d["mode"])))
                del d
            self.imgs.append(imgs)
            self.meta.append(meta)
            if log and li == 0:
                log(f"[rank {self.rank}] layer 0 images built")
        self.n_layers = len(self.imgs)
        self.n_matrices = sum(len(li) for li in self.imgs)

        # device residency: every image block uploaded once into one pool
        self.pool_bytes = sum(_align(m["block"]) for lm in self.meta for m in lm)
        self.pool = torch.empty(max(self.pool_bytes, _ALIGN), dtype=torch.uint8, device="cuda")
        off = 0
        for li, lm in zip(self.imgs, self.meta):
            for img, m in zip(li, lm):
                H.check(L.hxq_cuda_image_upload(img, self.pool.data_ptr() + off, None), "upload")
                off += _align(m["block"])
        torch.cuda.synchronize()

        # launch groups over one shared arena
        self.groups = launch_groups(self.n_layers, self.world)
        self._g_imgs, self._g_offs, g_numel = [], [], []
        for grp in self.groups:
            gi = [img for layer in grp for img in self.imgs[layer]]
            offs, total = packed_offsets([m["numel"] for layer in grp for m in self.meta[layer]])
            self._g_imgs.append((C.c_void_p * len(gi))(*[i.value for i in gi]))
            self._g_offs.append((C.c_size_t * len(offs))(*offs))
            g_numel.append(total)
        self.arena = H.SharedBuffer()
        H.check(L.hxq_cuda_arena_init(C.byref(self.arena), max(g_numel) if g_numel else 1), "arena")
        self._first = [sum(len(self.imgs[layer]) for layer in range(grp[0])) for grp in self.groups]
        # per-layer views (one layer per launch) for stream_step
        self._l_arrs = [(C.c_void_p * len(li))(*[i.value for i in li]) for li in self.imgs]
        self._l_offs = []
        for lm in self.meta:
            offs, _ = packed_offsets([m["numel"] for m in lm])
            self._l_offs.append((C.c_size_t * len(offs))(*offs))
        self._l_first = [int(v) for v in np.cumsum([0] + [len(li) for li in self.imgs])[:-1]]
        self.conf = torch.zeros(self.n_matrices, dtype=torch.float32, device="cuda")
        self.sumsq = torch.zeros(self.n_matrices, dtype=torch.float64, device="cuda")
        self._stage = None

    # -- sizes -------------------------------------------------------------
    def numel(self) -> int:
        """Weights this rank decompresses per step."""
        return sum(m["numel"] for lm in self.meta for m in lm)

    def algorithmic_bytes(self, cb_bytes: int = 4096 * 2 * 4, out_elem: int = 4) -> int:
        """Index bytes + codebook + 12 B per in-range sidecar entry (the
        reference's COO: row, col, value) + output, over this rank's shards."""
        tot = 0
        for lm in self.meta:
            for m in lm:
                idx = m["numel"] * 3 // 4 if m["mode"] == 2 else m["numel"]
                tot += idx + cb_bytes + 12 * m["nnz"] + out_elem * m["numel"]
        return tot

    def host_block_bytes(self) -> int:
        """Bytes one streamed step copies host -> device."""
        return sum(_align(m["block"]) for lm in self.meta for m in lm)

    # -- decompress ----------------------------------------------------------
    def decompress_group(self, gi: int, stream_ptr) -> None:
        """Decompress the shards of launch group gi into the arena (one
        launch), writing their conf / sumsq entries (stream-ordered)."""
        first = self._first[gi]
        n = sum(len(self.imgs[layer]) for layer in self.groups[gi])
        e = self.L.hxq_cuda_decompress_images(self._g_imgs[gi], n, self.arena.data, self._g_offs[gi], 0,
                                              self.sumsq.data_ptr() + 8 * first,
                                              self.conf.data_ptr() + 4 * first, stream_ptr)
        self.H.check(e, "hxq_cuda_decompress_images")

    def step(self, stream_ptr) -> None:
        """Decompress every shard from the device pool into the arena, one
        launch per group (the arena then holds the last group)."""
        for gi in range(len(self.groups)):
            self.decompress_group(gi, stream_ptr)

    def group_of(self, layer: int) -> int:
        return next(gi for gi, grp in enumerate(self.groups) if layer in grp)

    def output_view(self, layer: int, p: int):
        """fp32 [rows, in_features] view of matrix p of `layer` in the arena,
        valid while the arena holds that layer's group (after
        decompress_group(group_of(layer)) and before the next launch)."""
        gi = self.group_of(layer)
        k = sum(len(self.imgs[q]) for q in self.groups[gi] if q < layer) + p
        m = self.meta[layer][p]
        off = self._g_offs[gi][k]
        return self.H.device_view(self.torch, self.arena.data + 4 * off, m["numel"]).view(m["rows"], m["in_f"])

    def launches_per_step(self) -> int:
        return len(self.groups)

    def stream_step(self, copy_s, comp_s, host_conf=None) -> None:
        """One step with the weights on the host: every layer's images are
        copied from pinned host memory (copy stream) while the previous
        layer decompresses (compute stream); optionally the confidences are
        copied back into `host_conf` (pinned) at the end."""
        torch, H, L = self.torch, self.H, self.L
        if self._stage is None:
            layer_bytes = [sum(_align(m["block"]) for m in lm) for lm in self.meta]
            self._stage = [torch.empty(max(layer_bytes), dtype=torch.uint8, device="cuda") for _ in range(2)]
            self._up = [torch.cuda.Event() for _ in range(2)]
            self._done = [torch.cuda.Event() for _ in range(2)]
        for layer in range(self.n_layers):
            s = layer % 2
            copy_s.wait_event(self._done[s])
            off = 0
            for img, m in zip(self.imgs[layer], self.meta[layer]):
                H.check(L.hxq_cuda_image_upload(img, self._stage[s].data_ptr() + off,
                                                C.c_void_p(copy_s.cuda_stream)), "upload")
                off += _align(m["block"])
            self._up[s].record(copy_s)
            comp_s.wait_event(self._up[s])
            first = self._l_first[layer]
            e = L.hxq_cuda_decompress_images(self._l_arrs[layer], len(self.imgs[layer]), self.arena.data,
                                             self._l_offs[layer], 0, self.sumsq.data_ptr() + 8 * first,
                                             self.conf.data_ptr() + 4 * first, C.c_void_p(comp_s.cuda_stream))
            H.check(e, "hxq_cuda_decompress_images")
            self._done[s].record(comp_s)
        if host_conf is not None:
            with torch.cuda.stream(comp_s):
                host_conf.copy_(self.conf, non_blocking=True)

    def restore_pool(self) -> None:
        """Point every image back at its block in the resident pool (after
        stream_step moved them to the staging buffers)."""
        off = 0
        for li, lm in zip(self.imgs, self.meta):
            for img, m in zip(li, lm):
                self.H.check(self.L.hxq_cuda_image_upload(img, self.pool.data_ptr() + off, None), "upload")
                off += _align(m["block"])
        self.torch.cuda.synchronize()

    # -- confidences ---------------------------------------------------------
    def reference_confidences(self) -> list[float]:
        """Per matrix, in layer order: the reference's confidence for the
        whole matrix (hxq.c's fp32 running sum over all rows), which every
        shard's image carries; no communication."""
        return [float(self.L.hxq_cuda_image_tensor_confidence(img)) for li in self.imgs for img in li]

    def exact_confidences(self) -> list[float]:
        """Per matrix: sqrt of the shards' GPU sums of squares, gathered from
        every rank and added in rank order (a collective when world > 1:
        every rank must call it)."""
        torch = self.torch
        mine = self.sumsq.detach().clone()
        if self.world > 1:
            import torch.distributed as dist
            parts = [torch.empty_like(mine) for _ in range(self.world)]
            dist.all_gather(parts, mine)
        else:
            parts = [mine]
        host = [p.cpu().numpy() for p in parts]
        return [combine_sumsq([h[i] for h in host]) for i in range(self.n_matrices)]

    def close(self) -> None:
        if getattr(self, "imgs", None) is None:
            return
        for li in self.imgs:
            for img in li:
                self.L.hxq_cuda_image_destroy(img)
        self.L.hxq_shared_buffer_free(C.byref(self.arena))
        self.imgs = None


# ---------------------------------------------------------------------------
# Column-split fused matmul

class ColumnSplitLayer:
    """A layer's matrices with output features split over the ranks, in one
    weight format.

    mats: sequence of dicts with "name", "O", "I" and either "vq" (a host
        dict of the full 12-bit matrix, k = 4096) or "affine" (a host dict
        of the full affine matrix: codes [O*I] uint8, scales/offsets
        [O*I/gs], gs).  Every rank passes the same matrices and keeps only
        its rows.
    fmt: "vq12" or "affine".
    p2p: also map every rank's output buffers into every other rank, so
        forward() can assemble with "p2p" (a collective at construction
        when world > 1: every rank must pass the same value).
    max_tokens: the largest token count forward() will see (sizes the p2p
        output buffers).
    Assembly, chosen per forward(): "local" (one rank), "nccl" (all-gather
    of the output shards) or "p2p" (stores into every rank's mapped output
    buffer inside the matmul epilogues).
    """

    def __init__(self, mats: Sequence[dict], fmt: str, *, p2p: bool = False, max_tokens: int = 1,
                 rank: int | None = None, world: int | None = None, torch=None, lib=None):
        import hxq_b200 as H
        if torch is None:
            import torch as _torch
            torch = _torch
        if fmt not in ("vq12", "affine"):
            raise ValueError("fmt must be vq12 or affine")
        self.H, self.L, self.torch = H, (lib or H.lib()), torch
        self.rank, self.world = _rank_world(rank, world)
        self.fmt, self.max_tokens = fmt, int(max_tokens)
        self.default_assembly = "local" if self.world == 1 else ("p2p" if p2p else "nccl")
        L = self.L
        self.mats = []
        self.weight_bytes = 0
        for m in mats:
            O, I = int(m["O"]), int(m["I"])
            r0, r1 = shard_rows(O, self.rank, self.world)
            e = dict(name=m.get("name", ""), O=O, I=I, r0=r0, rows=r1 - r0)
            if fmt == "vq12":
                d = m["vq"]
                t = H.Tensor().load(d)
                img = C.c_void_p()
                H.check(L.hxq_cuda_image_create_ex(t.ref, r0, r1, H.HXQ_IMAGE_MATMUL, C.byref(img)), "image")
                t.free()
                e["img"] = img
                nnz = int(np.count_nonzero((d["rows"] >= r0) & (d["rows"] < r1) & (d["cols"] < I)))
                self.weight_bytes += (r1 - r0) * I * 3 // 4 + 4096 * 2 * 4 + 12 * nnz
            else:
                a = m["affine"]
                gs = int(a.get("gs", 128))
                ng = I // gs
                codes = torch.from_numpy(np.ascontiguousarray(a["codes"].reshape(O, I)[r0:r1])).cuda()
                scales = torch.from_numpy(np.ascontiguousarray(a["scales"].reshape(O, ng)[r0:r1])).cuda()
                offs = torch.from_numpy(np.ascontiguousarray(a["offsets"].reshape(O, ng)[r0:r1])).cuda()
                e["aff"] = H.AffineTensor(codes.data_ptr(), scales.data_ptr(), offs.data_ptr(), None, r1 - r0, I, gs)
                e["keep"] = (codes, scales, offs)
                self.weight_bytes += (r1 - r0) * I + 2 * (r1 - r0) * ng * 4
            self.mats.append(e)
        n = len(self.mats)
        self._aff = (H.AffineTensor * n)(*[e["aff"] for e in self.mats]) if fmt == "affine" else None
        self._imgs = (C.c_void_p * n)(*[e["img"].value for e in self.mats]) if fmt == "vq12" else None
        self._local: dict[int, list] = {}
        self._gathered: dict[int, list] = {}
        self.p2p = self._open_p2p() if (p2p and self.world > 1) else None

    # -- p2p output buffers ---------------------------------------------------
    def _open_p2p(self) -> dict:
        import torch.distributed as dist
        H, L, world, rank = self.H, self.L, self.world, self.rank
        handle = lambda: (C.c_char * 64)()  # noqa: E731
        own, hnd = [], []
        for e in self.mats:
            for _ in range(2):
                ptr, h = C.c_void_p(), handle()
                H.check(L.hxq_cuda_ipc_alloc(self.max_tokens * e["O"] * 4, C.byref(ptr), h), "ipc alloc")
                own.append(ptr)
                hnd.append(bytes(h))
        fptr, fh = C.c_void_p(), handle()
        H.check(L.hxq_cuda_ipc_alloc(256, C.byref(fptr), fh), "ipc alloc")
        all_h = [None] * world
        dist.all_gather_object(all_h, (hnd, bytes(fh)))
        opened = []
        bufs = [[None] * world for _ in range(2 * len(self.mats))]   # [matrix*2 + parity][rank]
        flag_ptrs = [None] * world
        for pr in range(world):
            for j in range(2 * len(self.mats)):
                if pr == rank:
                    bufs[j][pr] = own[j].value
                else:
                    dp = C.c_void_p()
                    H.check(L.hxq_cuda_ipc_open((C.c_char * 64).from_buffer_copy(all_h[pr][0][j]), C.byref(dp)),
                            "ipc open")
                    opened.append(dp)
                    bufs[j][pr] = dp.value
            if pr == rank:
                flag_ptrs[pr] = fptr.value
            else:
                dp = C.c_void_p()
                H.check(L.hxq_cuda_ipc_open((C.c_char * 64).from_buffer_copy(all_h[pr][1]), C.byref(dp)), "ipc open")
                opened.append(dp)
                flag_ptrs[pr] = dp.value
        torch = self.torch
        p = dict(own=own, fptr=fptr, opened=opened, bufs=bufs, flags=(C.c_void_p * world)(*flag_ptrs),
                 counter=torch.zeros(1, dtype=torch.int32, device="cuda"),
                 status=torch.zeros(1, dtype=torch.int32, device="cuda"))
        torch.cuda.synchronize()
        dist.barrier()
        return p

    # -- forward ----------------------------------------------------------------
    def _batch(self, xs_ptrs, outs_per_matrix, ldys, N, stream_ptr):
        n = len(self.mats)
        n_out = len(outs_per_matrix[0])
        X = (C.c_void_p * n)(*xs_ptrs)
        Y = (C.c_void_p * (n * n_out))(*[p for outs in outs_per_matrix for p in outs])
        LD = (C.c_uint32 * n)(*ldys)
        if self.fmt == "vq12":
            self.H.check(self.L.hxq_cuda_vq_matmul_batch(n, self._imgs, X, Y, n_out, LD, N, stream_ptr),
                         "vq matmul batch")
        elif self.L.hxq_affine_group_matmul_bf16_batch(n, self._aff, X, Y, n_out, LD, N, stream_ptr) != 0:
            raise RuntimeError("affine matmul batch failed")

    def local_outputs(self, N: int) -> list:
        """This rank's output shards [N, rows] (nccl / local assembly)."""
        if N not in self._local:
            torch = self.torch
            self._local[N] = [torch.empty((N, e["rows"]), dtype=torch.float32, device="cuda") for e in self.mats]
            self._gathered[N] = [torch.empty((self.world * N, e["rows"]), dtype=torch.float32, device="cuda")
                                 for e in self.mats]
        return self._local[N]

    def _assembly(self, assembly):
        a = assembly or self.default_assembly
        if self.world == 1:
            a = "local"
        if a not in ("local", "nccl", "p2p") or (a == "p2p" and self.p2p is None):
            raise ValueError(f"assembly {a!r} not available")
        return a

    def forward(self, xs: dict, N: int, stream, step: int = 0, assembly: str | None = None) -> None:
        """y_j = x W_j^T for every matrix j, assembled on every rank.
        xs maps in_features -> bf16 activations [N, in_features] (CUDA).
        stream: a torch.cuda.Stream; step: the step index (p2p buffers
        alternate by its parity).  Outputs: `outputs(N, step, assembly)`."""
        if N > self.max_tokens:
            raise ValueError("more tokens than max_tokens")
        assembly = self._assembly(assembly)
        sp = C.c_void_p(stream.cuda_stream)
        x_ptrs = [xs[e["I"]].data_ptr() for e in self.mats]
        if assembly == "p2p":
            p = self.p2p
            outs = [[b + 4 * e["r0"] for b in p["bufs"][2 * j + (step & 1)]] for j, e in enumerate(self.mats)]
            self._batch(x_ptrs, outs, [e["O"] for e in self.mats], N, sp)
            self.H.check(self.L.hxq_cuda_peer_signal(p["flags"], self.world, self.rank, p["counter"].data_ptr(), sp),
                         "peer signal")
            self.H.check(self.L.hxq_cuda_peer_wait(p["flags"][self.rank], self.world, p["counter"].data_ptr(),
                                                   p["status"].data_ptr(), sp), "peer wait")
            return
        ys = self.local_outputs(N)
        self._batch(x_ptrs, [[y.data_ptr()] for y in ys], [e["rows"] for e in self.mats], N, sp)
        if assembly == "nccl":
            import torch.distributed as dist
            with self.torch.cuda.stream(stream):
                for y, g in zip(ys, self._gathered[N]):
                    dist.all_gather_into_tensor(g, y)

    def outputs(self, N: int, step: int = 0, assembly: str | None = None) -> list:
        """The assembled outputs [N, O] of the last forward with that
        assembly (views, or permuted copies for nccl)."""
        torch, H = self.torch, self.H
        assembly = self._assembly(assembly)
        if assembly == "p2p":
            return [H.device_view(torch, self.p2p["own"][2 * j + (step & 1)].value, N * e["O"]).view(N, e["O"])
                    for j, e in enumerate(self.mats)]
        if assembly == "local":
            return self.local_outputs(N)
        return [assemble_gathered(g, self.world, N, e["rows"]) for g, e in zip(self._gathered[N], self.mats)]

    def gathered_raw(self, N: int) -> list:
        """[ranks * N, rows] all-gather buffers (nccl assembly)."""
        return self._gathered.get(N, [])

    def peer_wait_status(self) -> int:
        return int(self.p2p["status"].item()) if self.p2p else 0

    def close(self) -> None:
        if getattr(self, "mats", None) is None:
            return
        if self.p2p is not None:
            import torch.distributed as dist
            self.torch.cuda.synchronize()
            dist.barrier()
            for dp in self.p2p["opened"]:
                self.L.hxq_cuda_ipc_close(dp)
            self.torch.cuda.synchronize()
            dist.barrier()
            for ptr in self.p2p["own"] + [self.p2p["fptr"]]:
                self.L.hxq_cuda_ipc_free(ptr)
            self.p2p = None
        for e in self.mats:
            if "img" in e:
                self.L.hxq_cuda_image_destroy(e["img"])
        self.mats = None
