#!/usr/bin/env python
"""HXQ on B200: decompress throughput of a 7B Llama-shaped model.

Workload (default, `llama7b`): 32 layers x {q,k,v,o 4096x4096, gate/up
11008x4096, down 4096x11008} = 224 matrices, 6,476,005,376 weights, every
matrix 12-bit 2D-VQ (k=4096 x dim 2 codebook ~N(0,0.02), uniform indices,
0.5% sidecar, deltas ~N(0,0.005)), seeded synthetic data.  Each rank owns
rows [r*O/N, (r+1)*O/N) of every matrix (no collective on this path) and
decompresses a whole layer per launch into one reusable device arena.

A step = decompress all 224 matrices once (each rank its row shards; the
driver is the library's hxq_b200.sharded.ShardedDecompress).
  value:      compressed images already resident in HBM, CUDA-graph replay.
  e2e:        through the public C API with host buffers: every step uploads
              each matrix's compressed image from pinned host memory
              (overlapped with the previous layer's decompress) and reads the
              224 confidences back.
  e2e_dropin: the reference's own entry point, hxq_dequant(HXQ_BACKEND_CUDA),
              called once per matrix into a device arena (N=1).
  aux:        one short measurement of each other configuration (c1, c2,
              c3 at one token, c5 one-token layer), N=1.
Inputs per step (5.3 GB compressed, 25.9 GB written) exceed the 126 MB L2,
so no L2 flush is needed between steps.

`--impl reference` times the reference C library (hxq.c built from source,
oracle/_ref) on the host cores over the same 32 layers: every step
decompresses all 224 matrices with all host threads (threads over row
slices, each with its own reused shared buffer).
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import sys
import threading
import time

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(HERE, "hxq-native_b200")
for p in (HERE, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402

from hxq_b200.shard import slice_rows  # noqa: E402

METRIC = "dequant weights/s (7B-shaped 12-bit 2D-VQ decompress, sidecar + confidence fused)"
UNIT = "weights/s"
SIDECAR_FRAC = 0.005
LAYERS = 32
CB_BYTES = 4096 * 2 * 4


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def measured_peaks() -> tuple[float, str]:
    path = os.path.join(HERE, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def algorithmic_bytes(rows: int, in_f: int, nnz: int) -> int:
    """Index bytes + codebook + 12 B per sidecar entry (row, col, value) + fp32 output."""
    return rows * in_f * 3 // 4 + CB_BYTES + 12 * nnz + 4 * rows * in_f


def measured_tensor_peak() -> float:
    """Dense bf16 TFLOP/s measured on this pool (burst), else the fallback."""
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"])
    except Exception:
        return 1590.0


N1_LAYER_ALGO_BYTES = 973653900  # one layer launch at N=1 (algorithmic_bytes summed)


def profiled_traffic(bytes_per_launch: float, world: int):
    """DRAM bytes per launch from the committed ncu summary of one layer launch
    at N=1 (dram__bytes_read.sum + dram__bytes_write.sum); for a row shard the
    traffic scales with the shard's algorithmic bytes."""
    path = os.path.join(HERE, "profiles", "vq_fast_kernel_llama7b_layer_n1.md")
    try:
        for line in open(path):
            if line.startswith("dram_bytes_per_launch:"):
                n1 = float(line.split(":")[1])
                return n1 if world == 1 else n1 * bytes_per_launch / N1_LAYER_ALGO_BYTES
    except OSError:
        pass
    return None


# ---------------------------------------------------------------------------
# synthetic matrices (generated on the GPU, sliced, handed to the C loaders)

def gen_matrix(torch, seed: int, out_f: int, in_f: int) -> dict:
    """One matrix drawn on the device from `seed` (codebook ~N(0,0.02),
    uniform packed index bytes = uniform 12-bit indices, floor(0.5%) unique
    sidecar positions sorted row-major, deltas ~N(0,0.005)), returned on the
    host in the hxq_b200.synth dict layout."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    cb = (torch.randn(8192, generator=g, device="cuda") * 0.02).float()
    nbytes = out_f * in_f * 3 // 4
    packed = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, generator=g, device="cuda")
    n = out_f * in_f
    nnz = int(SIDECAR_FRAC * n)
    pos = torch.randperm(n, generator=g, device="cuda")[:nnz].sort().values
    vals = (torch.randn(nnz, generator=g, device="cuda") * 0.005).float()
    return dict(mode=2, out_f=out_f, in_f=in_f, k=4096, vdim=2, codebook=cb.cpu().numpy(),
                packed=packed.cpu().numpy(),
                rows=(pos // in_f).to(torch.int32).cpu().numpy().astype(np.uint32),
                cols=(pos % in_f).to(torch.int32).cpu().numpy().astype(np.uint32),
                vals=vals.cpu().numpy())


# ---------------------------------------------------------------------------
# clocks

class ClockSampler:
    """SM clock and clock-event reasons sampled through NVML every 5 ms while
    the timed region runs (read-only queries)."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self.ok = False
        self.stop_flag = threading.Event()

    def start(self):
        try:
            import pynvml as N
            N.nvmlInit()
            h = N.nvmlDeviceGetHandleByUUID(self.uuid) if self.uuid else N.nvmlDeviceGetHandleByIndex(0)
            self.max_mhz = float(N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM))
            get_reasons = getattr(N, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                N.nvmlDeviceGetCurrentClocksThrottleReasons

            def loop():
                while not self.stop_flag.is_set():
                    try:
                        self.samples.append((float(N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM)),
                                             int(get_reasons(h))))
                    except Exception:
                        pass
                    time.sleep(0.005)
            self.thread = threading.Thread(target=loop, daemon=True)
            self.thread.start()
            self.ok = True
        except Exception as e:  # no NVML: report it instead of guessing
            self.err = str(e)

    def stop(self) -> dict:
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        self.stop_flag.set()
        self.thread.join(timeout=2)
        sm = [c for c, _ in self.samples]
        reasons = sorted({name for _, r in self.samples for bit, name in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(sm), "source": "nvml 5 ms"}


# ---------------------------------------------------------------------------
# CPU baseline: the reference library on the host cores

def cpu_reference_runner(matrices, threads: int | None = None):
    """Returns (run_once() -> seconds, cores, kind, weights) for the given
    matrices (host dicts, or zero-argument callables returning one) on
    `threads` host threads (default: all).  Each job runs the unchanged
    reference function hxq_dequant (CPU) on a slice of rows into the calling
    thread's own shared buffer, reused across jobs as the reference reuses
    one buffer for a whole model."""
    from concurrent.futures import ThreadPoolExecutor

    from oracle.oracle import Oracle, Reference, ref_available
    cores = threads or os.cpu_count() or 1
    kind = "reference" if ref_available() else "port"
    local = threading.local()
    if kind == "reference":
        from oracle.oracle import _RefBuf, _RefResult
        ref = Reference()
        Lr = ref.L
    else:
        orc = Oracle()
    jobs, weights = [], 0
    for m in matrices:
        d = m() if callable(m) else m
        o = d["out_f"]
        weights += o * d["in_f"]
        step = max(1, o // max(1, cores // 2))
        for r0 in range(0, o, step):
            sl = slice_rows(d, r0, min(o, r0 + step))
            jobs.append(ref.tensor(sl) if kind == "reference" else sl)
        del d
    keep = []  # every thread's buffer stays alive with the runner

    if kind == "reference":
        def work(t):
            if getattr(local, "buf", None) is None:
                local.buf, local.res = _RefBuf(), _RefResult()
                Lr.ref_hxq_shared_buffer_init(C.byref(local.buf), 0)
                keep.append(local.buf)
            err = Lr.ref_hxq_dequant(C.byref(t), C.byref(local.buf), 1, C.byref(local.res))
            assert err == 0, err
    else:
        def work(sl):
            n = sl["out_f"] * sl["in_f"]
            if getattr(local, "buf", None) is None or local.buf.size < n:
                local.buf = np.zeros(n, np.float32)
                keep.append(local.buf)
            err, _, _ = orc.decompress(sl, out=local.buf[:n])
            assert err == 0
    pool = ThreadPoolExecutor(max_workers=cores)

    def run_once() -> float:
        t0 = time.perf_counter()
        list(pool.map(work, jobs))
        return time.perf_counter() - t0
    return run_once, cores, kind, weights


def layer_matrices(torch, layer: int = 0, lazy: bool = False):
    """The seven matrices of one 7B layer (q, k, v, o, gate, up, down), or
    zero-argument callables that generate them."""
    from hxq_b200 import synth
    out = []
    for p, (_, o, i) in enumerate(synth.LLAMA7B_PROJ):
        def f(s=synth.llama7b_seed(layer, p), o=o, i=i):
            return gen_matrix(torch, s, o, i)
        out.append(f if lazy else f())
    return out


def run_reference_arm(args):
    """The reference C library (hxq.c compiled from its sources, oracle/_ref)
    on all host threads over the same workload as our arm: every step
    decompresses all 224 matrices of the 32 layers (row slices per thread,
    one reused shared buffer per thread)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # the reference arm runs on rank 0 only
    import torch
    torch.cuda.set_device(0)
    nl = args.layers
    mats = [m for layer in range(nl) for m in layer_matrices(torch, layer, lazy=True)]
    t0 = time.time()
    run_once, cores, kind, weights = cpu_reference_runner(mats)
    log(f"[reference] {len(mats)} matrices loaded in {time.time() - t0:.1f}s")
    for _ in range(args.warmup):
        run_once()
    times = [run_once() for _ in range(args.steps)]
    total = sum(times)
    value = weights * args.steps / total
    sample = (f"all {nl} layers of the 7B workload ({len(mats)} matrices, {weights} weights) per step, "
              f"{cores} host threads")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": "llama7b-vq12-decompress", "layers": nl,
                                        "matrices": len(mats), "weights": weights},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ---------------------------------------------------------------------------
# auxiliary workloads: single-tensor decompress (c1, c2) and the affine sweep (c3)

def _graph_time(torch, stream, launch, n_launch: int, warmup: int) -> float:
    """Capture n_launch calls of launch(i) in a CUDA graph, replay it after
    warm-up, return the device time of one replay in ms (CUDA events)."""
    with torch.cuda.stream(stream):
        for i in range(min(n_launch, 8)):
            launch(i)
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(n_launch):
            launch(i)
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            g.replay()
    stream.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        g.replay()
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    del g
    return ms


def _decompress_case(torch, H, L, name: str, d: dict, dtype: int, algo_bytes: int, stream, args) -> dict:
    """Replicas of one tensor (inputs + outputs > 4x L2) decompressed one per
    launch, cycling, in a CUDA graph of --steps x 10 launches."""
    n = d["out_f"] * d["in_f"]
    elem = 4 if dtype == 0 else 2
    reps = max(2, int(np.ceil(4 * 126e6 / (algo_bytes))))
    t = H.Tensor().load(d)
    imgs = []
    for _ in range(reps):
        img = C.c_void_p()
        H.check(L.hxq_cuda_image_create(t.ref, 0, d["out_f"], C.byref(img)), "image")
        imgs.append(img)
    slot = (n + 63) // 64 * 64
    out = torch.empty(slot * reps * elem, dtype=torch.uint8, device="cuda")
    conf = torch.zeros(reps, dtype=torch.float32, device="cuda")
    arrs = [(C.c_void_p * 1)(img.value) for img in imgs]
    zero = (C.c_size_t * 1)(0)

    def launch(i):
        r = i % reps
        e = L.hxq_cuda_decompress_images(arrs[r], 1, out.data_ptr() + r * slot * elem, zero, dtype, None,
                                         conf.data_ptr() + 4 * r, stream.cuda_stream)
        if e != 0:
            raise RuntimeError(f"decompress failed {e}")
    n_launch = args.steps * 10
    ms = _graph_time(torch, stream, launch, n_launch, args.warmup)
    H.check(L.hxq_cuda_stream_synchronize(C.c_void_p(stream.cuda_stream)), name)
    per = ms / n_launch
    # drop-in API, synchronous, device arena
    arena = H.SharedBuffer()
    H.check(L.hxq_cuda_arena_init(C.byref(arena), n), "arena")
    r = H.Result()
    lat = []
    fn = L.hxq_dequant if dtype == 0 else None
    for i in range(30):
        t0 = time.perf_counter()
        if dtype == 0:
            H.check(fn(t.ref, C.byref(arena), H.HXQ_BACKEND_CUDA, C.byref(r)), "dequant")
        else:
            H.check(L.hxq_dequant_bf16(t.ref, C.byref(arena), C.byref(r)), "dequant_bf16")
        lat.append(time.perf_counter() - t0)
    L.hxq_shared_buffer_free(C.byref(arena))
    for img in imgs:
        L.hxq_cuda_image_destroy(img)
    peak, kind = measured_peaks()
    gbs = algo_bytes / (per / 1e3) / 1e9
    return {"case": name, "dtype": "f32" if dtype == 0 else "bf16", "weights": n,
            "us_per_launch": per * 1e3, "weights_per_s": n / (per / 1e3),
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                         "bytes_per_launch": algo_bytes, "peak_source": kind},
            "replicas": reps, "launches": n_launch,
            "dequant_api_sync_us_median": 1e6 * statistics.median(lat[5:])}


def _affine_case(torch, H, L, N: int, stream, args) -> dict:
    from hxq_b200 import synth
    O = I = 4096
    gs = 128
    d = synth.affine(O, I, gs, synth.SEED_C3)
    xh, _ = synth.activations(N, I, synth.SEED_C3 + N)
    code_bytes = O * I
    io_bytes = code_bytes + 2 * O * (I // gs) * 4 + 2 * N * I + 4 * N * O
    reps = max(2, int(np.ceil(4 * 126e6 / io_bytes))) if N <= 64 else 2
    codes = [torch.from_numpy(d["codes"]).cuda() for _ in range(reps)]
    sc = torch.from_numpy(d["scales"]).cuda()
    of = torch.from_numpy(d["offsets"]).cuda()
    x = torch.from_numpy(xh.view(np.int16)).cuda()
    y = torch.empty(N * O, dtype=torch.float32, device="cuda")
    ts = [H.AffineTensor(c.data_ptr(), sc.data_ptr(), of.data_ptr(), None, O, I, gs) for c in codes]

    def launch(i):
        if L.hxq_affine_group_matmul_bf16(x.data_ptr(), C.byref(ts[i % reps]), y.data_ptr(), N,
                                          stream.cuda_stream) != 0:
            raise RuntimeError("affine matmul failed")
    n_launch = max(4, args.steps * (10 if N <= 64 else 2))
    ms = _graph_time(torch, stream, launch, n_launch, args.warmup)
    per_s = ms / n_launch / 1e3
    flops = 2.0 * N * O * I
    tf_peak = measured_tensor_peak()
    hbm, _ = measured_peaks()
    gbs = io_bytes / per_s / 1e9
    tfl = flops / per_s / 1e12
    return {"case": f"affine 4096x4096 g128 N={N}", "us_per_call": per_s * 1e6, "tflops": tfl,
            "gbs": gbs, "hbm_frac": gbs / hbm, "tensor_frac": tfl / tf_peak, "bytes_per_call": io_bytes,
            "replicas": reps}


def run_aux_workload(args):
    import torch

    import hxq_b200 as H
    from hxq_b200 import synth
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    L = H.lib()
    stream = torch.cuda.Stream()
    results = []
    if args.workload == "c1":
        d = synth.vq12(2048, 2048, synth.SEED_C1)
        nnz = len(d["rows"])
        results.append(_decompress_case(torch, H, L, "c1 12-bit 2048x2048", d, 0,
                                        2048 * 2048 * 3 // 4 + CB_BYTES + 12 * nnz + 4 * 2048 * 2048, stream, args))
        results.append(_decompress_case(torch, H, L, "c1 12-bit 2048x2048", d, 1,
                                        2048 * 2048 * 3 // 4 + CB_BYTES + 12 * nnz + 2 * 2048 * 2048, stream, args))
    elif args.workload == "c2":
        d = synth.scalar(4096, 4096, synth.SEED_C2)
        nnz = len(d["rows"])
        n = 4096 * 4096
        results.append(_decompress_case(torch, H, L, "c2 scalar 4096x4096", d, 0, n + 1024 + 12 * nnz + 4 * n,
                                        stream, args))
        results.append(_decompress_case(torch, H, L, "c2 scalar 4096x4096", d, 1, n + 1024 + 12 * nnz + 2 * n,
                                        stream, args))
    else:
        for N in (1, 8, 64, 512, 4096):
            results.append(_affine_case(torch, H, L, N, stream, args))
    print(json.dumps({"workload": args.workload, "data": "synthetic", "results": results}), flush=True)


def _randf_stream(seed: int, n: int) -> np.ndarray:
    """The reference Lloyd tests' generator (LCG, float(state >> 16) / 32768 - 1)."""
    hi = np.empty(n, np.uint32)
    s = seed
    for i in range(n):
        s = (s * 1103515245 + 12345) & 0xFFFFFFFF
        hi[i] = s >> 16
    return (hi.astype(np.float32) / np.float32(32768.0) - np.float32(1.0)).astype(np.float32)


def _graph_ms(torch, stream, launch, n_launch: int, warmup: int) -> float:
    """Device time of one of n_launch captured calls (CUDA graph, CUDA events)."""
    with torch.cuda.stream(stream):
        launch()
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for _ in range(n_launch):
            launch()
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            g.replay()
    stream.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        g.replay()
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / n_launch
    del g
    return ms


def run_compression_workloads(args):
    """The compression-side rows, one JSON line.
      lloyd: one Lloyd iteration (assign, centroid update, dead-centroid
             reinit) on the reference's benchmark inputs (test/test_lloyd.c:
             590,000 vectors x k 256 x d 2 and 295,000 x 256 x 4, its LCG
             generator), device arrays; vectors per second.
      pq:    PolarQuant rotation of 1,048,576 KV-cache head vectors of 128
             fp32 (512 MB) in place, Q from pq_generate_rotation(128, 42);
             vectors per second and bytes (read + write) per second.
    Each beside the reference compiled from its own sources (oracle/_ref) on
    one host thread (its OpenMP is not available in this image): Lloyd on
    the same input, the rotation on a 16,384-vector sample."""
    import torch

    import hxq_b200 as H
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    L = H.lib()
    stream = torch.cuda.Stream()
    hbm, peak_kind = measured_peaks()
    results = []
    if args.workload == "lloyd":
        for n, k, d, seed in ((590000, 256, 2, 999), (295000, 256, 4, 777)):
            r = _randf_stream(seed, n * d + k * d)
            w, cb = r[:n * d].copy(), r[n * d:].copy()
            dw = torch.from_numpy(w).cuda()
            dcb = torch.from_numpy(cb.copy()).cuda()
            didx = torch.zeros(n, dtype=torch.uint8, device="cuda")
            dnd = torch.zeros(1, dtype=torch.int32, device="cuda")

            def launch():
                if L.hxq_cuda_lloyd_reassign(dw.data_ptr(), dcb.data_ptr(), didx.data_ptr(), n, k, d, dnd.data_ptr(),
                                             C.c_void_p(stream.cuda_stream)) != 0:
                    raise RuntimeError("lloyd failed")
            ms = _graph_ms(torch, stream, launch, max(4, args.steps), args.warmup)
            res = {"case": f"lloyd n={n} k={k} d={d}", "ms_per_iteration": ms, "vectors_per_s": n / (ms * 1e-3)}
            if not args.no_cpu_baseline:
                from oracle.oracle import ReferenceLloyd
                rl = ReferenceLloyd()
                t0 = time.perf_counter()
                rc, _, _, _ = rl.reassign(w, cb, k, d)
                dt = time.perf_counter() - t0
                res["cpu_baseline"] = {"value": n / dt, "unit": "vectors/s", "cores": 1, "kind": "reference",
                                       "sample": "one iteration on the same input, oracle/_ref, one thread",
                                       "ms_per_iteration": dt * 1e3}
            results.append(res)
    else:
        nvec, hd = 1 << 20, 128
        Q = np.zeros(hd * hd, np.float32)
        if L.pq_generate_rotation(hd, 42, Q.ctypes.data) != 0:
            raise RuntimeError("pq_generate_rotation failed")
        rng = np.random.Generator(np.random.PCG64(0x5051))
        x = torch.from_numpy(rng.standard_normal(nvec * hd, dtype=np.float32)).cuda()
        dQ = torch.from_numpy(Q).cuda()
        flip = [0]

        def launch():
            fn = L.hxq_cuda_pq_rotate if flip[0] % 2 == 0 else L.hxq_cuda_pq_unrotate
            flip[0] += 1
            H.check(fn(x.data_ptr(), dQ.data_ptr(), nvec, hd, C.c_void_p(stream.cuda_stream)), "pq")
        ms = _graph_ms(torch, stream, launch, max(4, args.steps) // 2 * 2, args.warmup)
        gbs = 2 * nvec * hd * 4 / (ms * 1e-3) / 1e9
        res = {"case": f"pq rotate n={nvec} head_dim={hd}", "ms_per_call": ms, "vectors_per_s": nvec / (ms * 1e-3),
               "gbs": gbs, "hbm_frac": gbs / hbm, "peak_source": peak_kind,
               "fp32_ops_per_s": 2.0 * nvec * hd * hd / (ms * 1e-3),
               "bound": "fp32 pipe (each output a sequential fp32 sum: one multiply and one add per term)"}
        if not args.no_cpu_baseline:
            from oracle.oracle import ReferencePolarQuant
            rp = ReferencePolarQuant()
            sample = 16384
            xs = x[:sample * hd].cpu().numpy()
            t0 = time.perf_counter()
            rp.apply(xs, Q.reshape(hd, hd), hd, True)
            dt = time.perf_counter() - t0
            res["cpu_baseline"] = {"value": sample / dt, "unit": "vectors/s", "cores": 1, "kind": "reference",
                                   "sample": f"{sample} vectors, oracle/_ref pq_rotate, one thread"}
        results.append(res)
    print(json.dumps({"workload": args.workload, "data": "synthetic", "results": results}), flush=True)


def run_fused_matmul_workload(args):
    """The fused dequant-matmul sweep on one 7B layer (q, k, v, o, gate, up,
    down): the same matrices as 12-bit 2D-VQ images (codebook gather +
    sidecar, no dense weights) and as affine 4-bit codes in groups of 128,
    bf16 activations at 1, 16 and 2048 tokens.  Output features are split
    across the ranks (hxq_b200.sharded.ColumnSplitLayer: each rank holds the
    rows of its shard).  With more than one rank two ways of assembling the
    full outputs are timed:
      nccl: each matrix's output shard is all-gathered over NCCL into
            [ranks * tokens, rows];
      p2p:  every rank's [tokens, out_features] output buffer is mapped into
            every other rank (CUDA IPC) and the matmul stores each output
            element into all of them over NVLink; after the layer's seven
            matmuls one flag kernel tells the peers, one wait kernel waits
            for them.  Two buffers alternate by step parity.
    One step = the 7 matrices (+ assembly), captured in a CUDA graph; device
    time, max over ranks, and every rank's own time."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import hxq_b200 as H
    from hxq_b200 import synth
    from hxq_b200.sharded import ColumnSplitLayer
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    L = H.lib()
    stream = torch.cuda.Stream()
    hbm, peak_kind = measured_peaks()
    steps = args.steps + (args.steps % 2)          # even: the p2p buffers alternate by parity

    def over_ranks(x: float) -> list:
        if world == 1:
            return [x]
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t)
        return [float(q.item()) for q in parts]

    Ns = (1, 16, 2048)
    mats = []
    for p, (name, O, I) in enumerate(synth.LLAMA7B_PROJ):
        mats.append(dict(name=name, O=O, I=I, vq=synth.vq12(O, I, synth.llama7b_seed(0, p)),
                         affine=synth.affine(O, I, 128, synth.llama7b_seed(0, p) + 1000)))
    layers = {fmt: ColumnSplitLayer(mats, fmt, p2p=world > 1, max_tokens=max(Ns), rank=rank, world=world,
                                    torch=torch, lib=L) for fmt in ("vq12", "affine")}
    del mats
    flops_per_token = 2.0 * sum(O * I for _, O, I in synth.LLAMA7B_PROJ)

    def time_graph(step):
        with torch.cuda.stream(stream):
            for k in range(2):
                step(k)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for k in range(steps):
                step(k)
        with torch.cuda.stream(stream):
            for _ in range(max(1, args.warmup // 3)):
                graph.replay()
        stream.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        with torch.cuda.stream(stream):
            graph.replay()
        e1.record(stream)
        e1.synchronize()
        per_rank = over_ranks(e0.elapsed_time(e1) / steps)
        del graph
        return max(per_rank), per_rank

    results = []
    for fmt in ("vq12", "affine"):
        layer = layers[fmt]
        for N in Ns:
            xh4, _ = synth.activations(N, 4096, synth.SEED_C5 + N)
            xh11, _ = synth.activations(N, 11008, synth.SEED_C5 + N + 1)
            xs = {4096: torch.from_numpy(xh4.view(np.int16)).cuda(), 11008: torch.from_numpy(xh11.view(np.int16)).cuda()}
            modes = ["nccl" if world > 1 else "local"] + (["p2p"] if world > 1 else [])
            for mode in modes:
                ms, per_rank = time_graph(lambda k: layer.forward(xs, N, stream, step=k, assembly=mode))
                if L.hxq_cuda_affine_device_status() != 0:
                    raise RuntimeError("a tensor-core kernel reported a timeout")
                per_rank_gbs = layer.weight_bytes / (ms * 1e-3) / 1e9
                res = {"case": f"{fmt} 7B layer N={N} {mode}", "format": fmt, "tokens": N, "assembly": mode,
                       "us_per_layer": ms * 1e3, "tflops": flops_per_token * N / (ms * 1e-3) / 1e12,
                       "weight_bytes_per_rank": layer.weight_bytes, "weight_gbs_per_rank": per_rank_gbs,
                       "hbm_frac_per_rank": per_rank_gbs / hbm,
                       "output_bytes_per_layer": sum(N * O * 4 for _, O, _ in synth.LLAMA7B_PROJ),
                       "path": ("tensor-core GEMV" if N <= 8 else
                                "tensor-core GEMV for the 4096-wide matrices, tcgen05 GEMM for down"
                                if N <= 16 else "tcgen05 GEMM")}
                if world > 1:
                    res["per_rank_us"] = [t * 1e3 for t in per_rank]
                if mode == "p2p":
                    # one step outside the graph: the assembled outputs must equal
                    # the NCCL-gathered shards, bit for bit
                    torch.cuda.synchronize()
                    dist.barrier()
                    with torch.cuda.stream(stream):
                        layer.forward(xs, N, stream, step=0, assembly="nccl")
                        layer.forward(xs, N, stream, step=0, assembly="p2p")
                    stream.synchronize()
                    # differing outputs, in this rank's own columns and in the
                    # columns its peers stored over NVLink
                    bad = torch.zeros(2, dtype=torch.float64, device="cuda")
                    for e, a, b in zip(layer.mats, layer.outputs(N, 0, "p2p"), layer.outputs(N, 0, "nccl")):
                        diff = a.view(torch.int32) != b.contiguous().view(torch.int32)
                        cols = torch.arange(e["O"], device="cuda")
                        mine = (cols >= e["r0"]) & (cols < e["r0"] + e["rows"])
                        bad[0] += diff[:, mine].sum()
                        bad[1] += diff[:, ~mine].sum()
                    dist.all_reduce(bad, op=dist.ReduceOp.SUM)
                    res["p2p_equals_nccl"] = bool(bad.sum().item() == 0)
                    res["p2p_mismatch"] = {"own_columns": int(bad[0].item()), "peer_columns": int(bad[1].item())}
                    res["peer_wait_status"] = layer.peer_wait_status()
                results.append(res)
            del xs
    for layer in layers.values():
        layer.close()
    if rank == 0:
        print(json.dumps({"workload": "c5", "data": "synthetic", "n_gpus": world,
                          "parallelism": f"output features split x{world}",
                          "driver": "hxq_b200.sharded.ColumnSplitLayer",
                          "peak": {"hbm_gbs": hbm, "kind": peak_kind}, "results": results}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_kernel_cases(args):
    """One call each of the matmul kernels on a 4096 x 4096 matrix, for
    profiling: affine GEMV (1 token), VQ GEMV (1 token), VQ tcgen05 GEMM
    (2048 tokens), affine tcgen05 GEMM (4096 tokens), VQ tcgen05 GEMM with
    the small tile (64 tokens, split along K); bf16 activations.  Prints
    each call's device time (CUDA events, cold start)."""
    import torch

    import hxq_b200 as H
    from hxq_b200 import synth
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    L = H.lib()
    da = synth.affine(4096, 4096, 128, synth.SEED_C3)
    codes = torch.from_numpy(da["codes"]).cuda()
    sc = torch.from_numpy(da["scales"]).cuda()
    of = torch.from_numpy(da["offsets"]).cuda()
    at = H.AffineTensor(codes.data_ptr(), sc.data_ptr(), of.data_ptr(), None, 4096, 4096, 128)
    dv = synth.vq12(4096, 4096, synth.SEED_C5)
    t = H.Tensor().load(dv)
    img = C.c_void_p()
    H.check(L.hxq_cuda_image_create_ex(t.ref, 0, 4096, H.HXQ_IMAGE_MATMUL, C.byref(img)), "image")
    xs = {n: torch.from_numpy(synth.activations(n, 4096, 11 + n)[0].view(np.int16)).cuda() for n in (1, 64, 2048, 4096)}
    y = torch.empty(4096 * 4096, dtype=torch.float32, device="cuda")
    cases = [("affine GEMV N=1", lambda: L.hxq_affine_group_matmul_bf16(xs[1].data_ptr(), C.byref(at), y.data_ptr(), 1, None)),
             ("vq12 GEMV N=1", lambda: L.hxq_cuda_vq_matmul(img, xs[1].data_ptr(), 1, y.data_ptr(), 4096, None)),
             ("vq12 GEMM N=2048", lambda: L.hxq_cuda_vq_matmul(img, xs[2048].data_ptr(), 2048, y.data_ptr(), 4096, None)),
             ("affine GEMM N=4096", lambda: L.hxq_affine_group_matmul_bf16(xs[4096].data_ptr(), C.byref(at), y.data_ptr(), 4096, None)),
             ("vq12 GEMM N=64", lambda: L.hxq_cuda_vq_matmul(img, xs[64].data_ptr(), 64, y.data_ptr(), 4096, None))]
    out = []
    for name, fn in cases:
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        if fn() != 0:
            raise RuntimeError(name)
        e1.record()
        e1.synchronize()
        out.append({"case": name, "ms": e0.elapsed_time(e1)})
    if L.hxq_cuda_affine_device_status() != 0:
        raise RuntimeError("tcgen05 GEMM reported a timeout")
    L.hxq_cuda_image_destroy(img)
    print(json.dumps({"workload": "kernels", "data": "synthetic", "results": out}), flush=True)


# ---------------------------------------------------------------------------

def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--no-aux", action="store_true",
                    help="skip the short measurements of the other configurations (c1, c2, c3, c5)")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="layers to run (profiling aid; the workload is 32 layers)")
    ap.add_argument("--workload", choices=["llama7b", "c1", "c2", "c3", "c5", "kernels", "lloyd", "pq"],
                    default="llama7b",
                    help="llama7b: the headline (default); c1/c2/c3: single-tensor decompress "
                         "and the affine batch sweep; c5: the fused dequant-matmul sweep on a 7B "
                         "layer (column-split over the ranks); kernels: one call of each matmul "
                         "kernel (for profiling); lloyd / pq: the compression-side rows (Lloyd "
                         "iteration, PolarQuant rotation); one JSON line each")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    if args.impl == "reference":
        run_reference_arm(args)
        return
    if args.workload == "c5":
        run_fused_matmul_workload(args)
        return
    if args.workload == "kernels":
        run_kernel_cases(args)
        return
    if args.workload in ("lloyd", "pq"):
        run_compression_workloads(args)
        return
    if args.workload != "llama7b":
        run_aux_workload(args)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import hxq_b200 as H

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    L = H.lib()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    def gather_over_ranks(x: float) -> list:
        if world == 1:
            return [x]
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t)
        return [float(p.item()) for p in parts]

    from hxq_b200.sharded import ShardedDecompress

    t_setup = time.time()
    nl = args.layers
    layers = [layer_matrices(torch, layer, lazy=True) for layer in range(nl)]
    model = ShardedDecompress(layers, rank=rank, world=world, torch=torch, lib=L, log=log)
    log(f"[rank {rank}] images built in {time.time() - t_setup:.1f}s")
    n_mat = model.n_matrices

    stream = torch.cuda.Stream()
    launches0 = L.hxq_cuda_launch_count()
    with torch.cuda.stream(stream):
        model.step(stream.cuda_stream)  # creates the stream's scratch before any capture
    stream.synchronize()
    H.check(L.hxq_cuda_stream_synchronize(C.c_void_p(stream.cuda_stream)), "first step")
    launches_per_step = L.hxq_cuda_launch_count() - launches0

    graph = None
    if not args.no_graph:
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                model.step(stream.cuda_stream)
            graph = g
        except Exception as e:  # keep direct launches if capture is refused
            log(f"[rank {rank}] graph capture failed, direct launches: {e}")
            graph = None
            torch.cuda.synchronize()

    def run_steps(n):
        with torch.cuda.stream(stream):
            for _ in range(n):
                if graph is not None:
                    graph.replay()
                else:
                    model.step(stream.cuda_stream)

    run_steps(args.warmup)
    stream.synchronize()
    barrier()
    torch.cuda.synchronize()
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(local).uuid)
    except Exception:
        pass
    clocks = ClockSampler(uuid)
    clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")
    ev0.record(stream)
    run_steps(args.steps)
    ev1.record(stream)
    torch.cuda.nvtx.range_pop()
    ev1.synchronize()
    barrier()
    torch.cuda.synchronize()
    clk = clocks.stop()
    my_ms = ev0.elapsed_time(ev1)
    H.check(L.hxq_cuda_stream_synchronize(C.c_void_p(stream.cuda_stream)), "timed steps")
    ms = max_over_ranks(my_ms)
    per_rank_ms = gather_over_ranks(my_ms)
    total_weights = int(sum_over_ranks(float(model.numel())))
    value = total_weights * args.steps / (ms / 1e3)

    # the confidences every matrix reports after a step: the reference's
    # (fp32 running sum, bit-identical to hxq.c) and the exact fp64 one
    ref_conf = model.reference_confidences()
    exact_conf = model.exact_confidences()
    conf_rel = max((abs(a - b) / b if b else abs(a)) for a, b in zip(exact_conf, ref_conf)) if ref_conf else 0.0

    # roofline of the fused decompress kernel: one launch per layer group,
    # each followed by the small kernel that adds the group's exact sums of
    # squares in order; the whole step time is charged to the decompress
    # launches (conservative by the reductions' few microseconds)
    my_bytes = model.algorithmic_bytes()
    decomp_per_step = len(model.groups)
    my_launch_ms = my_ms / (args.steps * decomp_per_step)
    achieved = my_bytes / decomp_per_step / (my_launch_ms / 1e3) / 1e9
    peak, peak_kind = measured_peaks()
    traffic = profiled_traffic(my_bytes / decomp_per_step, world)

    # end to end through the public API: host images streamed every step
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(torch, H, L, model, args, world, max_over_ranks, sum_over_ranks)
        model.restore_pool()
    dropin = None
    if not args.no_e2e and world == 1:
        dropin = run_dropin(torch, H, L, args)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        layer0 = layer_matrices(torch, 0)
        run_once, cores, kind, weights = cpu_reference_runner(layer0)
        run_once()
        times, t_end = [], time.time() + 10.0
        while time.time() < t_end or len(times) < 3:
            times.append(run_once())
        cpu = {"value": weights / statistics.median(times), "unit": UNIT, "cores": cores, "kind": kind,
               "sample": f"layer 0 (7 matrices, {weights} weights) per rep, {len(times)} reps, "
                         f"median, {cores} host threads"}
        # the reference is single-threaded: its own speed, one core
        run1, _, _, _ = cpu_reference_runner(layer0, threads=1)
        t1 = [run1() for _ in range(3)]
        cpu["value_1core"] = weights / statistics.median(t1)
        del layer0

    aux = None
    if rank == 0 and world == 1 and not args.no_aux:
        aux = run_aux_block(torch, H, L, args)

    if rank == 0:
        lpl = len(model.groups[0]) if model.groups else 1
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "llama7b-vq12-decompress", "layers": nl, "matrices": n_mat,
                       "weights": total_weights, "sidecar_frac": SIDECAR_FRAC, "shard": "rows by out_features",
                       "launch": f"one per {lpl} layer(s) ({7 * lpl} matrices)", "graph": graph is not None,
                       "l2": "no flush: 5.3 GB read + 25.9 GB written per step >> 126 MB L2",
                       "parallelism": f"row-shard x{world}", "driver": "hxq_b200.sharded.ShardedDecompress"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_source": peak_kind,
                         "kernel": "vq_fast_kernel (12-bit, fp32 out)",
                         "bytes_per_launch": my_bytes / decomp_per_step,
                         "launch_ms": my_launch_ms, "launches_per_step": decomp_per_step,
                         "other_kernels": "sumsq_reduce_kernel after each launch (exact sums, ordered)"},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "e2e_dropin": dropin,
            "confidence": {"reported": "reference (hxq.c fp32 running sum), every matrix",
                           "max_rel_exact_vs_reference": conf_rel},
            "clocks": clk,
            "gpu_launches": int(launches_per_step * args.steps),
        }
        if world > 1:
            line["per_rank_ms_per_step"] = [t / args.steps for t in per_rank_ms]
            line["rank_spread"] = max(per_rank_ms) / min(per_rank_ms)
        if aux is not None:
            line["aux"] = aux
        print(json.dumps(line), flush=True)

    del graph
    model.close()
    barrier()
    if world > 1:
        dist.destroy_process_group()


def run_e2e(torch, H, L, model, args, world, max_over_ranks, sum_over_ranks):
    """Weights live in pinned host memory; every step uploads every layer's
    images (copy stream) while the previous layer decompresses (compute
    stream), then reads the confidences back."""
    copy_s, comp_s = torch.cuda.Stream(), torch.cuda.Stream()
    host_conf = torch.empty(model.n_matrices, dtype=torch.float32, pin_memory=True)
    steps = args.e2e_steps or max(3, min(args.steps, 10))
    for _ in range(2):
        model.stream_step(copy_s, comp_s, host_conf)
    comp_s.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp_s)
    copy_s.wait_event(e0)
    for _ in range(steps):
        model.stream_step(copy_s, comp_s, host_conf)
    e1.record(comp_s)
    e1.synchronize()
    H.check(L.hxq_cuda_stream_synchronize(C.c_void_p(comp_s.cuda_stream)), "e2e")
    ms = max_over_ranks(e0.elapsed_time(e1))
    h2d = sum_over_ranks(float(model.host_block_bytes()))
    weights = sum_over_ranks(float(model.numel()))
    return {"value": weights * steps / (ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(model.n_matrices * 4 * world), "steps": steps,
            "ms_per_step": ms / steps,
            "path": "hxq_cuda_image_upload (pinned host -> HBM) + hxq_cuda_decompress_images, "
                    "copy/compute overlapped by layer, confidences read back"}


def run_dropin(torch, H, L, args):
    """The reference's own entry point, unchanged: hxq_dequant(t, arena,
    HXQ_BACKEND_CUDA, &result) once per matrix, all 224 of them in turn, into
    one device arena (the shared buffer), each call synchronous with its
    confidence written back.  The first pass builds each tensor's device image
    (host preprocessing + upload) and is reported separately; timed passes
    reuse the cached images, as a model that stays loaded does."""
    nl = args.layers
    tensors = []
    for layer in range(nl):
        for d in layer_matrices(torch, layer):
            tensors.append((H.Tensor().load(d), d["out_f"] * d["in_f"]))
            del d
    arena = H.SharedBuffer()
    H.check(L.hxq_cuda_arena_init(C.byref(arena), 0), "arena")
    r = H.Result()

    def one_pass():
        for t, _ in tensors:
            H.check(L.hxq_dequant(t.ref, C.byref(arena), H.HXQ_BACKEND_CUDA, C.byref(r)), "hxq_dequant")

    torch.cuda.synchronize()
    t0 = time.perf_counter()
    one_pass()
    first = time.perf_counter() - t0
    one_pass()
    steps = max(3, min(args.steps, 10))
    t0 = time.perf_counter()
    for _ in range(steps):
        one_pass()
    dt = (time.perf_counter() - t0) / steps
    weights = sum(n for _, n in tensors)
    L.hxq_shared_buffer_free(C.byref(arena))
    for t, _ in tensors:
        t.free()
    return {"value": weights / dt, "unit": UNIT, "ms_per_step": dt * 1e3, "steps": steps,
            "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 20 * len(tensors),
            "first_pass_s": first,
            "path": "hxq_dequant(HXQ_BACKEND_CUDA) per matrix into a device arena (the reference API), "
                    "synchronous, host wall clock; device images cached after the first pass, whose "
                    "time (image build + upload) is first_pass_s"}


def run_aux_block(torch, H, L, args) -> list:
    """The other configurations, one short measurement each, beside the
    headline: c1 12-bit 2048x2048 fp32, c2 scalar 4096x4096 fp32 and bf16
    (fused decompress, HBM roofline), the c3 affine GEMV 4096x4096 at one
    token, and one 7B layer of the fused dequant-matmul at one token (VQ and
    affine, HBM roofline of the weight bytes)."""
    from hxq_b200 import synth
    from hxq_b200.sharded import ColumnSplitLayer
    stream = torch.cuda.Stream()
    a = argparse.Namespace(steps=max(2, min(args.steps, 10)), warmup=3)
    out = []
    d = synth.vq12(2048, 2048, synth.SEED_C1)
    nnz = len(d["rows"])
    r = _decompress_case(torch, H, L, "c1 12-bit 2048x2048", d, 0,
                         2048 * 2048 * 3 // 4 + CB_BYTES + 12 * nnz + 4 * 2048 * 2048, stream, a)
    out.append({"case": "c1 vq12 2048x2048 fp32", "us": r["us_per_launch"], "frac": r["roofline"]["frac"],
                "gbs": r["roofline"]["achieved"], "weights_per_s": r["weights_per_s"]})
    d = synth.scalar(4096, 4096, synth.SEED_C2)
    nnz, n = len(d["rows"]), 4096 * 4096
    for dt, ob in ((0, 4), (1, 2)):
        r = _decompress_case(torch, H, L, "c2 scalar 4096x4096", d, dt, n + 1024 + 12 * nnz + ob * n, stream, a)
        out.append({"case": f"c2 scalar 4096x4096 {'fp32' if dt == 0 else 'bf16'}", "us": r["us_per_launch"],
                    "frac": r["roofline"]["frac"], "gbs": r["roofline"]["achieved"],
                    "weights_per_s": r["weights_per_s"],
                    "dequant_api_sync_us_median": r["dequant_api_sync_us_median"]})
    r = _affine_case(torch, H, L, 1, stream, a)
    out.append({"case": "c3 affine 4096x4096 g128 N=1", "us": r["us_per_call"], "frac": r["hbm_frac"],
                "gbs": r["gbs"]})
    hbm, _ = measured_peaks()
    mats = []
    for p, (name, O, I) in enumerate(synth.LLAMA7B_PROJ):
        mats.append(dict(name=name, O=O, I=I, vq=gen_matrix(torch, synth.llama7b_seed(0, p), O, I),
                         affine=dict(synth.affine(O, I, 128, synth.llama7b_seed(0, p) + 1000), gs=128)))
    xh4, _ = synth.activations(1, 4096, synth.SEED_C5 + 1)
    xh11, _ = synth.activations(1, 11008, synth.SEED_C5 + 2)
    xs = {4096: torch.from_numpy(xh4.view(np.int16)).cuda(), 11008: torch.from_numpy(xh11.view(np.int16)).cuda()}
    for fmt in ("vq12", "affine"):
        layer = ColumnSplitLayer(mats, fmt, max_tokens=1, rank=0, world=1, torch=torch, lib=L)
        n_launch = 10 * a.steps
        ms = _graph_ms(torch, stream, lambda: layer.forward(xs, 1, stream), n_launch, a.warmup)
        gbs = layer.weight_bytes / (ms * 1e-3) / 1e9
        out.append({"case": f"c5 7B layer {fmt} N=1", "us": ms * 1e3, "frac": gbs / hbm, "gbs": gbs,
                    "weight_bytes": layer.weight_bytes})
        layer.close()
    if L.hxq_cuda_affine_device_status() != 0:
        raise RuntimeError("a tensor-core kernel reported a timeout")
    return out


if __name__ == "__main__":
    main()
