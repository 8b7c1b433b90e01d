#!/usr/bin/env python
"""HCT weight-decode benchmark on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Headline workload: the whole Llama-2-70B -- 80 layers
(q/o 8192x8192, k/v 1024x8192, gate/up 28672x8192, down 8192x28672, two
RMSNorm weights), the 32000x8192 embedding and lm_head and the final norm,
723 tensors, 69.0 G parameters -- as HCT-Q4 files (DCT-II, retention 0.30,
INT4 coefficients with FP16 block scales, 16 KiB LZ4 blocks) resident in
HBM, decoded to bf16.  Under torchrun the model is layer-sharded: every rank
decodes its contiguous layer range (partition.rs create_for_layers) plus its
share of the other tensors; there is no collective on the decode path.  A
step decodes the whole model once (strong scaling: the work is fixed as N
grows); the timed region is bracketed by a barrier and CUDA events and the
reported time is the max over ranks.

Reported beside it: the same decode end to end with each step's compressed
files copied from pinned host memory (`e2e`), the roofline of the kernel with
the largest share of the step, the whole Llama-3-8B (config 4), one 70B layer
per GPU (config 3, with the replicated-weights mode at N > 1), LZ4 on config
2, INT4 on config 1, the V3 / HoloTensor / Zstandard formats, and the
reference's CPU decode restated by the oracle (`cpu_baseline`, N = 1), which
also checks a sample of the GPU's outputs.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

LAYER_70B = [  # (name, rows, cols)
    ("q_proj", 8192, 8192), ("k_proj", 1024, 8192), ("v_proj", 1024, 8192),
    ("o_proj", 8192, 8192), ("gate_proj", 28672, 8192), ("up_proj", 28672, 8192),
    ("down_proj", 8192, 28672),
]
SEED = 2
RETENTION = 0.30
HOLO_FRAGMENTS = 8  # HoloTensorEncoder's default fragment count


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return dict(hbm=float(d["hbm_gbs"]), tflops=float(d["bf16_tflops"]),
                    tflops_sustained=float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                    source="measured")
    return dict(hbm=6650.0, tflops=1590.0, tflops_sustained=1400.0, source="fallback")


# ------------------------------------------------------------------ inputs

def layer_files(rank_local: int, world: int, barrier, dev) -> dict:
    """HCT-Q4 (and V3 / HoloTensor) files of the layer, encoded once per node by the
    torch writer on the GPU (float64 DCT-II) from the seeded numpy weights, and
    cached under the temporary directory."""
    import torch

    from haagenti_b200 import encode as E
    from haagenti_b200 import encode_gpu as G

    cache = os.path.join(tempfile.gettempdir(),
                         f"hct_b200_bench_l70b_s{SEED}_r{int(RETENTION*100)}_q4v3holo_tw")
    done = os.path.join(cache, "DONE")
    if rank_local == 0 and not os.path.exists(done):
        os.makedirs(cache, exist_ok=True)
        t0 = time.time()
        for i, (name, m, n) in enumerate(LAYER_70B):
            w = E.synthetic_weight((m, n), SEED * 100 + i)
            c = G.dct_2d_gpu(torch.from_numpy(w).to(dev))  # one DCT for the three formats
            bitmap, vals = G.spectral_select_gpu(c, RETENTION)
            payload = torch.cat([bitmap, G.quantize_int4_gpu(vals)]).cpu().numpy()
            del bitmap, vals
            with open(os.path.join(cache, name + ".hct"), "wb") as f:
                f.write(E.write_hct(payload, [m, n], E.DTYPE_I4, E.FLAG_SPECTRAL_Q4, 1))
            c = c.cpu().numpy()
            with open(os.path.join(cache, name + ".v3"), "wb") as f:
                f.write(E.encode_hct_v3(w, RETENTION, 1, coeffs=c))
            with open(os.path.join(cache, name + ".holo"), "wb") as f:
                f.write(E.encode_holotensor(w, HOLO_FRAGMENTS, coeffs=c))
            del w, c
        torch.cuda.empty_cache()
        with open(done, "w") as f:
            f.write(f"{time.time() - t0:.1f}\n")
    barrier()
    out = {}
    for name, m, n in LAYER_70B:
        for ext in ("hct", "v3", "holo"):
            with open(os.path.join(cache, f"{name}.{ext}"), "rb") as f:
                out[name if ext == "hct" else name + "." + ext] = f.read()
    return out


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.dev}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ helpers

def kernel_stats(H, ctx):
    import ctypes as C
    from haagenti_b200 import _lib as L

    arr = (L.KernelStats * 16)()
    n = C.c_int(0)
    rc = L.load().hct_b200_ctx_profile_read(ctx.handle, arr, 16, C.byref(n))
    if rc:
        raise RuntimeError(f"profile_read failed: {rc}")
    return {arr[i].name.decode(): dict(launches=int(arr[i].launches), ms=arr[i].total_ms,
                                       work=arr[i].work) for i in range(n.value)}


def set_profiling(ctx, on: bool):
    from haagenti_b200 import _lib as L

    L.load().hct_b200_ctx_profile(ctx.handle, 1 if on else 0)


KERNEL_NAMES = {  # profile record -> kernel
    "lz4_decode_blocks": "hct::lz4_decode_blocks_kernel",
    "spectral_rank": "hct::chunk_rank_kernel + hct::chunk_scan_kernel",
    "spectral_pack": "hct::spectral_pack_kernel (bitmap/INT4 decode + Makhoul pack, row axis)",
    "makhoul_pack": "hct::makhoul_pack_kernel (Makhoul pack, column axis)",
    "dft_stage1": "hct::dft_stage_t_kernel modes 4/6 (tcgen05 DFT over k1, twiddle and, "
                  "on column passes with 2P <= 128, the Makhoul pack folded into per-k2 matrices)",
    "dft_stage2": "hct::dft_stage_t_kernel mode 5 (tcgen05 DFT over k2 from the MN-major "
                  "intermediate, quartet store)",
    "umma_gemm": "hct::umma_gemm_kernel (dense-basis tcgen05 IDCT contraction)",
    "spectral_scatter": "hct::chunk_scan_kernel + hct::spectral_scatter_kernel",
    "dequant_int4": "hct::dequant_int4_tiles_kernel (bulk-staged INT4 dequant)",
}
TRAFFIC_PROFILE = os.path.join(REPO, "profiles", "hct_decode_layer70b.md")


MODEL_TRAFFIC_PROFILE = os.path.join(REPO, "profiles", "hct_decode_llama2_70b.md")


def read_traffic(kind, path=TRAFFIC_PROFILE):
    """DRAM bytes per launch of one kernel (ncu dram__bytes_read + write), from a
    committed profile summary: a line `traffic_bytes_per_launch[<record>]: <bytes>`."""
    if not os.path.exists(path):
        return None
    key = f"traffic_bytes_per_launch[{kind}]:"
    for line in open(path):
        if line.startswith(key):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


# ------------------------------------------------------------------ CPU baseline

CPU_SAMPLE = ["k_proj", "v_proj", "q_proj", "o_proj"]


def cpu_decode_sample(files: dict, threads: int, keep: bool = False):
    """The reference's CPU decode (oracle restatement: LZ4 + INT4 + scatter + Makhoul
    IDCT) of the CPU_SAMPLE tensors; with keep, their f32 outputs are returned too."""
    from oracle import hct as OH

    t0 = time.perf_counter()
    elems, outs = 0, {}
    for name in CPU_SAMPLE:
        x = OH.decode_spectral_q4_cpu(files[name], threads)
        elems += x.size
        if keep:
            outs[name] = x
    dt = time.perf_counter() - t0
    return elems * 2 / dt / 1e9, dt, elems, outs


def cpu_scipy_idct(files: dict, threads: int) -> dict:
    """scipy.fft.idctn (the orthonormal DCT-III, pocketfft) over the host cores on the
    dense f32 coefficients of q_proj: a second CPU timing of the IDCT alone."""
    import scipy.fft

    from oracle import hct as OH

    c = OH.decode_spectral_q4_cpu(files["q_proj"], threads, stage="coeffs")
    scipy.fft.idctn(c, type=2, norm="ortho", workers=threads)
    t0 = time.perf_counter()
    reps = 2
    for _ in range(reps):
        scipy.fft.idctn(c, type=2, norm="ortho", workers=threads)
    dt = (time.perf_counter() - t0) / reps
    return {"value": round(c.size * 2 / dt / 1e9, 4), "unit": "GB/s", "cores": threads,
            "kind": "library",
            "sample": f"scipy {scipy.__version__} fft.idctn(type=2, norm='ortho', f32, "
                      f"workers={threads}) of q_proj's dense coefficients (8192x8192): the IDCT "
                      f"alone, no LZ4/INT4, {dt:.2f} s per call"}


def cpu_zstd_sample(frames, total_bytes: int) -> dict:
    """libzstd (the library the reference's `zstd` crate binds) decoding the
    same 64 KiB frames on the host cores, one frame per task."""
    from concurrent.futures import ThreadPoolExecutor

    from oracle import zstd_ref as Z

    import ctypes

    threads = os.cpu_count() or 1
    n = len(frames)

    def work(lo_hi):
        buf = ctypes.create_string_buffer(65536)
        for i in range(*lo_hi):
            if Z.decompress_into(frames[i], buf) != 65536:
                raise RuntimeError("libzstd failed on a bench frame")

    spans = [(i * n // threads, (i + 1) * n // threads) for i in range(threads)]
    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(work, spans))  # warm-up
        t0 = time.perf_counter()
        list(ex.map(work, spans))
        dt = time.perf_counter() - t0
    return {"value": round(total_bytes / dt / 1e9, 2), "unit": "GB/s decompressed",
            "cores": threads, "kind": "reference",
            "sample": f"all {n} frames once, libzstd {Z.version()} via ctypes, {threads} threads"}


# ------------------------------------------------------------------ arms

REF_BUDGET_S = 150.0  # CPU seconds the reference arm's warm-up + timed steps may take


def run_reference(args):
    """The reference's CPU decode path (the oracle's line-by-line restatement of
    block.rs, quantization.rs and dct.rs; the Rust crates cannot be built here)
    on the host cores, on the product arm's workload: the Llama-2-70B model
    (config 5).  Its inputs are layer 0 of that model, encoded by the oracle's
    own writer from numpy weights of the same shapes, seeds and distribution.
    A step decodes the whole layer while the run fits REF_BUDGET_S; otherwise
    each step decodes the next tensors of the layer in turn, about the share
    of the layer that keeps the run inside the budget."""
    import shutil

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from oracle import hct as OH

    threads = os.cpu_count() or 1
    files, layer_elems = ref_model_sample_files("llama2-70b", 4)
    names = list(files)
    shapes = {n: OH.parse_hct(files[n]).header.shape for n in names}
    elems = {n: int(np.prod(shapes[n])) for n in names}

    def decode(ns):
        t0 = time.perf_counter()
        for n in ns:
            OH.decode_spectral_q4_cpu(files[n], threads)
        return time.perf_counter() - t0

    t_layer = decode(names)  # first warm-up step: the whole layer
    rest = max(args.warmup - 1, 0) + args.steps
    frac = min(1.0, REF_BUDGET_S / (rest * t_layer))
    cursor = [0]

    def next_sample():
        if frac >= 1.0:
            return names
        ns, acc = [], 0
        while not ns or acc < frac * layer_elems:
            n = names[cursor[0] % len(names)]
            cursor[0] += 1
            ns.append(n)
            acc += elems[n]
        return ns

    for _ in range(max(args.warmup - 1, 0)):
        decode(next_sample())
    t_sum, e_sum, first = 0.0, 0, None
    for _ in range(args.steps):
        ns = next_sample()
        first = first or ns
        t_sum += decode(ns)
        e_sum += sum(elems[n] for n in ns)
    value = e_sum * 2 / t_sum / 1e9
    ms = 1e3 * t_sum / args.steps
    sample = ("per step all of layer 0 (%d tensors, %d elements)" % (len(names), layer_elems)
              if frac >= 1.0 else
              "per step the next tensors of layer 0 in turn (first step: %s), about %.0f%% of "
              "the layer" % ("+".join(n.split(".", 3)[-1] for n in first), 100 * frac))
    line = {
        "impl": "reference", "metric": "decoded_weight_GBps", "value": round(value, 4),
        "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "llama2-70b whole model, HCT-Q4 (BASELINE config 5)",
                   "retention": RETENTION, "seed": 4, "block_size": 16384,
                   "inputs": "layer 0 of the model encoded by the oracle's writer "
                             "(oracle/hct.py encode_spectral_q4) from numpy PCG64 weights "
                             "N(0,0.02) with 1% outlier columns, seed 4 * 100000 + tensor "
                             "index"},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads,
                         "kind": "port",
                         "sample": sample + ": LZ4 + INT4 + bitmap scatter + f32 Makhoul IDCT "
                                            "(oracle/hct_oracle.c, OpenMP), bf16-equivalent "
                                            "bytes out"},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "host": {"cpu_count": threads, "cargo": shutil.which("cargo"),
                 "rustc": shutil.which("rustc")},
    }
    print(json.dumps(line), flush=True)
    return 0


def model_files(H, torch, dev, arch: str, seed: int, units) -> tuple[dict, float]:
    """HCT-Q4 files of this rank's tensors of a whole model, made by the torch
    writer on the GPU (weights from torch's Philox generator, seed = model seed
    * 100000 + the tensor's index in the model); the LZ4 + container step of
    one tensor runs on a host thread while the next is encoded on the GPU."""
    from concurrent.futures import ThreadPoolExecutor

    from haagenti_b200 import encode as E
    from haagenti_b200 import encode_gpu as G
    from haagenti_b200 import shard

    index = {n: i for i, (n, _, _) in enumerate(shard.model_units(arch))}
    t0 = time.time()
    files, futs = {}, {}
    with ThreadPoolExecutor(max_workers=1) as ex:
        for name, shape, _ in units:
            w = G.synthetic_weight_gpu(shape, seed * 100000 + index[name], dev)
            rows, cols = E.tensor_dims(shape)
            payload = G.spectral_payload_gpu(w.reshape(rows, cols), RETENTION).cpu().numpy()
            del w
            futs[name] = ex.submit(E.write_hct, payload, list(shape), E.DTYPE_I4,
                                   E.FLAG_SPECTRAL_Q4, 1)
        for name, f in futs.items():
            files[name] = f.result()
    torch.cuda.empty_cache()
    return files, time.time() - t0


MODEL_WINDOW = 32  # decodes in flight before the loader reads a status back
RESIDENT_OUT_LIMIT = 100e9  # bf16 bytes a rank keeps resident; beyond, outputs rotate


def model_leg(H, torch, dev, args, arch: str, seed: int, world: int, rank: int, local: int,
              barrier, clocks: bool = False, profile: bool = True) -> dict:
    """Whole-model decode (BASELINE configs 4 and 5): every rank decodes its own
    layer range plus its share of the other tensors (shard.rank_units), all
    HCT-Q4 files resident in HBM; a step decodes all of them once."""
    from collections import deque

    from haagenti_b200 import encode as E
    from haagenti_b200 import shard

    units = shard.rank_units(arch, world, rank)
    files, enc_s = model_files(H, torch, dev, arch, seed, units)
    barrier()
    ctxs = (H.Context(local), H.Context(local))
    stream = torch.cuda.current_stream(dev)
    if args.priority:
        # the two decode streams above the library's side streams (default,
        # lowest priority): stage-kernel CTAs are scheduled before front-end ones
        streams = (torch.cuda.Stream(dev, priority=-args.priority),
                   torch.cuda.Stream(dev, priority=-args.priority))
    else:
        streams = (stream, torch.cuda.Stream(dev))
    copy_stream = torch.cuda.Stream(dev)
    lane = {n: i % 2 for i, (n, _, _) in enumerate(units)}
    readers = {n: H.HctReader(files[n], ctxs[lane[n]]) for n, _, _ in units}
    out_bytes = sum(2 * shard._numel(s) for _, s, _ in units)
    comp_bytes = sum(len(files[n]) for n, _, _ in units)
    # outputs: one buffer per tensor when they fit beside the inputs, else the
    # layers' outputs rotate over two layer-sized pools (layer l and l + 2 keep
    # their tensors on the same stream, so a buffer is never written twice at once)
    resident = out_bytes <= RESIDENT_OUT_LIMIT
    outs = {}
    pools = {}
    for n, s, l in units:
        if resident or l < 0:
            outs[n] = torch.empty(s, dtype=torch.bfloat16, device=dev)
        else:
            key = (l % 2, n.split(".", 3)[-1])
            if key not in pools:
                pools[key] = torch.empty(s, dtype=torch.bfloat16, device=dev)
            outs[n] = pools[key]
    names = [n for n, _, _ in units]
    window = max(1, min(getattr(args, "window", MODEL_WINDOW), len(names) - 1))
    pinned = None

    def run(steps, upload=False, serial=False):
        pend = deque()
        for _ in range(steps):
            if upload and args.upload_first:
                # the step's files go to the copy stream first (each waits only
                # for the previous decode of its own reader), so that the copy
                # engine never waits for the host's decode loop
                for n in names:
                    readers[n].upload(pinned[n], stream=copy_stream)
            for n in names:
                r = readers[n]
                if upload and not args.upload_first:
                    r.upload(pinned[n], stream=copy_stream)
                r.decode_async(outs[n], H.BF16, stream=streams[lane[n]])
                pend.append(r)
                if serial or len(pend) > window:
                    pend.popleft().wait()
        while pend:
            pend.popleft().wait()

    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)

    def timed(steps, upload=False):
        barrier()
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for s_ in streams + (copy_stream,):
            if s_ != stream:
                s_.wait_event(e0)
        run(steps, upload)
        for s_ in streams:
            if s_ != stream:
                done = torch.cuda.Event()
                done.record(s_)
                stream.wait_event(done)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        return e0.elapsed_time(e1)

    run(1)
    torch.cuda.synchronize(dev)
    for n in names[:4]:
        v = outs[n].float()
        assert torch.isfinite(v).all() and 0.001 < v.std().item() < 1.0, n
    run(max(args.warmup - 1, 2))
    clk = ClockSampler(local) if clocks else None
    if clk:
        clk.__enter__()
    try:
        ms_total = timed(args.steps)
    finally:
        if clk:
            clk.__exit__()
    ms_total = shard.max_over_ranks(ms_total, dev)
    ms_step = ms_total / args.steps
    all_bytes = sum(2 * shard._numel(s) for _, s, _ in shard.model_units(arch))
    value = all_bytes / (ms_step / 1e3) / 1e9

    ks, ms_prof = {}, None
    if profile:
        for c in ctxs:
            set_profiling(c, True)
        barrier()
        torch.cuda.synchronize(dev)
        t_prof = time.perf_counter()
        run(1, serial=True)
        torch.cuda.synchronize(dev)
        ms_prof = 1e3 * (time.perf_counter() - t_prof)
        barrier()
        for c in ctxs:
            for k, v in kernel_stats(H, c).items():
                a = ks.setdefault(k, dict(launches=0, ms=0.0, work=0.0))
                a["launches"] += v["launches"]
                a["ms"] += v["ms"]
                a["work"] += v["work"]
            set_profiling(c, False)

    # end to end: each step's compressed files copied from pinned host memory
    # (copy stream, overlapping earlier tensors' decode) and every status read back
    pinned = {}
    for n in names:
        a = torch.empty(len(files[n]), dtype=torch.uint8, pin_memory=True)
        a.numpy()[:] = np.frombuffer(files[n], np.uint8)
        pinned[n] = a.numpy()
    run(1, upload=True)
    e2e_ms = shard.max_over_ranks(timed(args.steps, upload=True), dev) / args.steps
    # the copies alone, every rank at once: this box's concurrent pinned -> HBM ceiling
    barrier()
    torch.cuda.synchronize(dev)
    c0 = torch.cuda.Event(enable_timing=True)
    c1 = torch.cuda.Event(enable_timing=True)
    c0.record(copy_stream)
    for n in names:
        readers[n].upload(pinned[n], stream=copy_stream)
    c1.record(copy_stream)
    torch.cuda.synchronize(dev)
    copy_ms = shard.max_over_ranks(c0.elapsed_time(c1), dev)
    barrier()
    h2d = sum(_data_len(files[n]) for n in names)
    d2h = sum(32 * readers[n].num_blocks() + 4 for n in names)
    e2e_value = all_bytes / (e2e_ms / 1e3) / 1e9
    # per-rank copy bandwidth of the end-to-end steps
    h2d_gbs = h2d / (e2e_ms / 1e3) / 1e9

    res = {
        "arch": arch, "value": round(value, 3), "unit": "GB/s", "ms_per_step": round(ms_step, 3),
        "per_gpu_GBps": round(value / world, 3),
        "decoded_bytes_per_step": all_bytes,
        "this_rank": {"tensors": len(names), "decoded_bytes": out_bytes,
                      "compressed_bytes": comp_bytes, "encode_s": round(enc_s, 1),
                      "outputs": "resident" if resident else
                                 "layer outputs rotate over two layer-sized pools"},
        "e2e": {"value": round(e2e_value, 3), "unit": "GB/s", "ms_per_step": round(e2e_ms, 3),
                "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
                "h2d_GBps_per_rank": round(h2d_gbs, 2),
                "h2d_ceiling_GBps_per_rank": round(h2d / (copy_ms / 1e3) / 1e9, 2),
                "h2d_ceiling_note": "the same uploads alone on every rank at once (copy "
                                    "stream, no decode), the slowest rank",
                "path": "HctReader.upload (pinned host -> HBM, copy stream"
                        + (", a step's uploads enqueued before its decodes"
                           if getattr(args, "upload_first", True) else "")
                        + ") + HctReader.decode_async per tensor, statuses read back "
                        f"{window} tensors behind",
                "host_binding": getattr(args, "host_binding", None)},
        "kernels": ks, "ms_prof": ms_prof, "clocks": clk.summary() if clk else None,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sample = [n for n, _, l in units if l == 0]
        res["oracle_check"] = check_units_against_oracle(H, torch, readers, files, sample)
    for r in readers.values():
        r.close()
    for c in ctxs:
        c.close()
    del outs, pools, pinned
    torch.cuda.empty_cache()
    return res


def check_units_against_oracle(H, torch, readers, files, names) -> dict:
    """The checker for a sample of model tensors: the oracle's CPU decode of the
    product's file against the GPU's f32 decode (max-abs 1e-3, cosine 0.99999)
    and its bf16 decode (the same bound plus the bf16 half-ulp)."""
    from oracle import hct as OH

    res = {"tensors": names, "max_abs_f32": 0.0, "min_cos_f32": 1.0, "max_excess_bf16": -1.0}
    for n in names:
        r = OH.decode_spectral_q4_cpu(files[n], os.cpu_count() or 1)
        g = readers[n].decode(H.F32).cpu().numpy().reshape(r.shape)
        a, b = g.astype(np.float64).ravel(), r.astype(np.float64).ravel()
        res["max_abs_f32"] = max(res["max_abs_f32"], float(np.abs(a - b).max()))
        res["min_cos_f32"] = min(res["min_cos_f32"],
                                 float((a @ b) / np.sqrt((a @ a) * (b @ b))))
        gb = readers[n].decode(H.BF16).float().cpu().numpy().reshape(r.shape)
        ex = np.abs(gb - r) - (1e-3 + np.abs(r) * 2.0 ** -8)
        res["max_excess_bf16"] = max(res["max_excess_bf16"], float(ex.max()))
    res["ok"] = (res["max_abs_f32"] <= 1e-3 and res["min_cos_f32"] >= 0.99999
                 and res["max_excess_bf16"] <= 0.0)
    if not res["ok"]:
        raise AssertionError(f"GPU decode differs from the oracle: {res}")
    for k in ("max_abs_f32", "min_cos_f32", "max_excess_bf16"):
        res[k] = float(f"{res[k]:.6g}")
    return res


def roofline_of(ks: dict, ms_prof, ms_per_step: float, steps: int,
                traffic_file: str = TRAFFIC_PROFILE) -> tuple:
    """(roofline of the kernel with the largest share, per-kernel table) from the
    library's per-launch CUDA-event records of `steps` profiled steps; ms_per_step
    is the uninstrumented step time."""
    pk = peaks()
    if not ks:
        return None, {}
    top = max(ks, key=lambda k: ks[k]["ms"])
    t = ks[top]
    tensor = top == "umma_gemm"
    scale = 1e12 if tensor else 1e9
    achieved = t["work"] / (t["ms"] / 1e3) / scale
    peak = pk["tflops_sustained"] if tensor else pk["hbm"]
    roof = {
        "bound": "tensor" if tensor else "hbm", "kernel": KERNEL_NAMES.get(top, top),
        "achieved": round(achieved, 2), "peak": peak,
        "unit": "TFLOP/s" if tensor else "GB/s", "frac": round(achieved / peak, 4),
        "peak_kind": (f"bf16 cuBLAS sustained, of {pk['source']}" if tensor
                      else f"STREAM copy, of {pk['source']}"),
        "traffic": read_traffic(top, traffic_file),
        "traffic_source": os.path.relpath(traffic_file, REPO),
        "algorithmic_per_launch": round(t["work"] / t["launches"]),
        "launches_per_step": t["launches"] / steps,
        "share_of_step": round(t["ms"] / ms_prof, 4) if ms_prof else None,
        "step_hbm_frac": round(sum(v["work"] for k, v in ks.items() if k != "umma_gemm")
                               / steps / (ms_per_step / 1e3) / 1e9 / pk["hbm"], 4),
    }
    kern = {k: {"launches": v["launches"], "ms_total": round(v["ms"], 3),
                "share": round(v["ms"] / ms_prof, 4) if ms_prof else None,
                "rate": round(v["work"] / (v["ms"] / 1e3) / (1e12 if k == "umma_gemm" else 1e9), 2),
                "rate_unit": "TFLOP/s" if k == "umma_gemm" else "GB/s"} for k, v in ks.items()}
    return roof, kern


def bind_host_cpus(torch, local: int, enabled: bool = True) -> dict:
    """Pin this rank's process to the CPUs NVML reports as local to its GPU, so
    that the pinned host buffers it first-touches (the end-to-end uploads) sit
    on the GPU's own NUMA node.  Reads the topology only; changes no GPU
    setting.  Returns what was done (for the JSON line)."""
    if not enabled:
        return {"bound": False, "why": "--no-bind"}
    try:
        import pynvml

        p = torch.cuda.get_device_properties(local)
        bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            ncpu = os.cpu_count() or 1
            masks = pynvml.nvmlDeviceGetCpuAffinity(h, (ncpu + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
        cpus = {64 * i + b for i, m in enumerate(masks) for b in range(64) if (int(m) >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return {"bound": False, "why": "no local CPUs reported"}
        os.sched_setaffinity(0, cpus)
        return {"bound": True, "pci": bus, "cpus": len(cpus)}
    except Exception as e:  # no NVML, or no topology: run unbound
        return {"bound": False, "why": f"{type(e).__name__}: {e}"[:120]}


def run_b200(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    args.host_binding = bind_host_cpus(torch, local, not args.no_bind)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=900), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    import haagenti_b200 as H

    # ---- headline: the whole Llama-2-70B (config 5), layer-sharded --------
    m70 = model_leg(H, torch, dev, args, "llama2-70b", 4, world, rank, local, barrier,
                    clocks=True)
    # ---- config 4: the whole Llama-3-8B, layer-sharded ----------------------
    m8 = (model_leg(H, torch, dev, args, "llama3-8b", 3, world, rank, local, barrier,
                    profile=False) if not args.no_secondary else None)
    # ---- config 3: one 70B layer per GPU (roofline table, replicate mode) ---
    layer = layer_leg(H, torch, dev, args, world, rank, local, barrier)

    stream = torch.cuda.current_stream(dev)
    sec = rank == 0 and not args.no_secondary
    lz4 = bench_lz4(H, torch, dev, stream, args) if sec else None
    int4 = bench_int4(H, torch, dev, stream, args) if sec else None
    v3 = holo = zstd = None
    if sec:
        files = layer.pop("_files")
        ctx = H.Context(local)
        tens = layer.pop("_tens")
        v3 = bench_v3(H, torch, dev, stream, files, tens, ctx)
        holo = bench_holo(H, torch, dev, stream, files, tens, ctx)
        ctx.close()
        zstd = bench_zstd(H, torch, dev, stream, args)
    layer.pop("_files", None)
    layer.pop("_tens", None)

    cpu = None
    if cpu_ok(args):
        # the reference's CPU decode (oracle port) of layer 0 of the same model
        cpu = cpu_model_sample("llama2-70b", 4)

    roof, kern = roofline_of(m70.pop("kernels"), m70.pop("ms_prof"), m70["ms_per_step"], 1,
                             MODEL_TRAFFIC_PROFILE)
    launches = sum(v["launches"] for v in kern.values()) * args.steps
    if rank == 0:
        line = {
            "metric": "decoded_weight_GBps", "value": m70["value"], "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": m70["ms_per_step"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {
                "workload": "llama2-70b whole model, HCT-Q4 (BASELINE config 5)",
                "layers": 80, "hidden": 8192, "intermediate": 28672, "heads": 64,
                "kv_heads": 8, "head_dim": 128, "vocab": 32000, "tensors": 723,
                "decoded_bytes_per_step": m70["decoded_bytes_per_step"],
                "retention": RETENTION, "seed": 4, "block_size": 16384, "out_dtype": "bf16",
                "weights": "N(0,0.02) f32 from torch's Philox generator on the GPU (seed "
                           "4 * 100000 + tensor index), 1% of columns x10 on 2-D tensors; "
                           "encoded by the torch writer (float64 DCT-II, top 30%, INT4, LZ4)",
                "parallelism": f"layer-sharded over {world} GPU(s): contiguous layer ranges "
                               "(partition.rs create_for_layers), embed/lm_head/norm by size; "
                               "no collective on the decode path",
                "pipelining": "every tensor's decode enqueued on one of two decode contexts "
                              f"(own stream each); statuses read back {args.window} tensors "
                              "behind; steps follow each other without a drain",
                "instrumentation": "value and e2e timed without the per-kernel profiling "
                                   "hook; kernel times from one more step with it, one tensor "
                                   "at a time",
                "l2": "each step reads 20 GB of compressed files and writes 138 GB; no flush",
            },
            "e2e": m70["e2e"],
            "per_gpu_GBps": m70["per_gpu_GBps"],
            "this_rank": m70["this_rank"],
            "roofline": roof,
            "kernels": kern,
            "gpu_launches": launches,
            "oracle_check": m70.get("oracle_check"),
            "cpu_baseline": cpu,
            "clocks": m70["clocks"],
            "llama3_8b": m8,
            "layer70b": layer,
            "lz4": lz4, "int4": int4, "hct_v3": v3, "holotensor": holo, "zstd": zstd,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def cpu_model_sample(arch: str, seed: int) -> dict:
    """The reference's CPU decode (oracle: LZ4 + INT4 + scatter + f32 Makhoul IDCT,
    OpenMP) of layer 0 of the model, encoded by the oracle's writer from numpy
    weights of the same shapes, seeds and distribution."""
    files, elems = ref_model_sample_files(arch, seed)
    threads = os.cpu_count() or 1
    from oracle import hct as OH

    t0 = time.perf_counter()
    for f in files.values():
        OH.decode_spectral_q4_cpu(f, threads)
    dt = time.perf_counter() - t0
    return {"value": round(elems * 2 / dt / 1e9, 4), "unit": "GB/s", "cores": threads,
            "kind": "port",
            "sample": f"layer 0 of {arch} ({len(files)} tensors, {elems} elements, {dt:.1f} s): "
                      "oracle LZ4 + INT4 + bitmap scatter + f32 Makhoul IDCT, OpenMP, "
                      "bf16-equivalent bytes out"}


def ref_model_sample_files(arch: str, seed: int) -> tuple[dict, int]:
    """Layer 0 of the model encoded by the oracle's writer (cached per node)."""
    from haagenti_b200 import shard
    from oracle import hct as OH

    units = shard.model_units(arch)
    index = {n: i for i, (n, _, _) in enumerate(units)}
    sample = [(n, s) for n, s, l in units if l == 0]
    cache = os.path.join(tempfile.gettempdir(), f"hct_b200_ref_{arch}_s{seed}_layer0_oracle")
    done = os.path.join(cache, "DONE")
    if not os.path.exists(done):
        os.makedirs(cache, exist_ok=True)
        for n, s in sample:
            w = OH.gen_weight(s, seed * 100000 + index[n])
            with open(os.path.join(cache, n), "wb") as f:
                f.write(OH.encode_spectral_q4(w, RETENTION, version=1))
        with open(done, "w") as f:
            f.write("ok\n")
    files = {}
    for n, _ in sample:
        with open(os.path.join(cache, n), "rb") as f:
            files[n] = f.read()
    return files, sum(shard._numel(s) for _, s in sample)


def layer_leg(H, torch, dev, args, world: int, rank: int, local: int, barrier) -> dict:
    """every rank decodes its own copy of one 70B layer per step
    (the round-1 workload, kept for its per-kernel table and the replicate mode)."""
    from haagenti_b200 import shard

    TENS = [t for t in LAYER_70B if not args.tensors or t[0] in args.tensors.split(",")]
    files = layer_files(local, world, barrier, dev)
    idct_mode = {"auto": H.IDCT_AUTO, "scatter": H.IDCT_SCATTER, "dense": H.IDCT_DENSE}[args.idct]
    ctx = H.Context(local)
    ctx2 = H.Context(local)
    for c in (ctx, ctx2):
        c.set_idct(idct_mode)
    stream = torch.cuda.current_stream(dev)
    stream2 = torch.cuda.Stream(dev)
    TENS = sorted(TENS, key=lambda t: -t[1] * t[2])
    lane = {n: i % 2 for i, (n, _, _) in enumerate(TENS)}
    ctxs, streams = (ctx, ctx2), (stream, stream2)
    readers = {n: H.HctReader(files[n], ctxs[lane[n]]) for n, _, _ in TENS}
    outs = {n: torch.empty((m, c), dtype=torch.bfloat16, device=dev) for n, m, c in TENS}
    out_bytes = sum(2 * m * c for _, m, c in TENS)
    comp_bytes = sum(len(files[n]) for n, _, _ in TENS)
    readers_b = {n: H.HctReader(files[n], ctxs[lane[n]]) for n, _, _ in TENS}
    outs_b = {n: torch.empty((m, c), dtype=torch.bfloat16, device=dev) for n, m, c in TENS}
    sets = [(readers, outs), (readers_b, outs_b)]
    pinned = None
    copy_stream = torch.cuda.Stream(dev)

    def issue(k, upload):
        rs, os_ = sets[k % 2]
        for n, _, _ in TENS:
            if upload:
                rs[n].upload(pinned[n], stream=copy_stream)
            rs[n].decode_async(os_[n], H.BF16, stream=streams[lane[n]])

    def wait(k):
        rs, _ = sets[k % 2]
        for n, _, _ in TENS:
            rs[n].wait()

    def run(steps, upload=False):
        for k in range(steps):
            issue(k, upload)
            if k:
                wait(k - 1)
        wait(steps - 1)

    run(2)
    torch.cuda.synchronize(dev)
    for n in outs:
        v = outs[n].float()
        assert torch.isfinite(v).all() and 0.005 < v.std().item() < 1.0, n
        assert torch.equal(outs[n], outs_b[n]), n
    run(max(args.warmup, 3))
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)

    def timed(steps, upload=False):
        barrier()
        torch.cuda.synchronize(dev)
        e0.record(stream)
        stream2.wait_event(e0)
        copy_stream.wait_event(e0)
        run(steps, upload)
        done2 = torch.cuda.Event()
        done2.record(stream2)
        stream.wait_event(done2)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        return e0.elapsed_time(e1)

    # enough steps for a timed region of about a second
    steps = max(args.steps, 200)
    ms_total = shard.max_over_ranks(timed(steps), dev)
    ms_step = ms_total / steps
    value = world * out_bytes / (ms_step / 1e3) / 1e9

    def run_serial(nsteps):
        for k in range(nsteps):
            rs, os_ = sets[k % 2]
            for n, _, _ in TENS:
                rs[n].decode_async(os_[n], H.BF16, stream=streams[lane[n]])
                rs[n].wait()

    for c in ctxs:
        set_profiling(c, True)
    barrier()
    torch.cuda.synchronize(dev)
    t_prof = time.perf_counter()
    run_serial(args.steps)
    torch.cuda.synchronize(dev)
    ms_prof = 1e3 * (time.perf_counter() - t_prof)
    barrier()
    ks = {}
    for c in ctxs:
        for k, v in kernel_stats(H, c).items():
            a = ks.setdefault(k, dict(launches=0, ms=0.0, work=0.0))
            a["launches"] += v["launches"]
            a["ms"] += v["ms"]
            a["work"] += v["work"]
        set_profiling(c, False)
    roof, kern = roofline_of(ks, ms_prof, ms_step, args.steps)

    pinned = {}
    for n, _, _ in TENS:
        a = torch.empty(len(files[n]), dtype=torch.uint8, pin_memory=True)
        a.numpy()[:] = np.frombuffer(files[n], np.uint8)
        pinned[n] = a.numpy()
    run(2, upload=True)
    e2e_ms = shard.max_over_ranks(timed(args.steps, upload=True), dev) / args.steps
    for n in outs_b:
        assert torch.equal(outs_b[n], outs[n]), n
    for r in readers_b.values():
        r.close()
    h2d = sum(_data_len(files[n]) for n, _, _ in TENS)
    d2h = sum(32 * readers[n].num_blocks() + 4 for n in readers)
    e2e_value = world * out_bytes / (e2e_ms / 1e3) / 1e9

    replicate = None
    if world > 1:
        names = [f"{n}@{r}" for r in range(world) for n, _, _ in TENS]
        owner = {f"{n}@{r}": r for r in range(world) for n, _, _ in TENS}
        specs = {f"{n}@{r}": ((m, c), torch.bfloat16, dev) for r in range(world) for n, m, c in TENS}
        mine = {f"{n}@{rank}": outs[n] for n, _, _ in TENS}
        shard.replicate_units(mine, owner, specs)
        barrier()
        torch.cuda.synchronize(dev)
        e0.record(stream)
        got = shard.replicate_units(mine, owner, specs)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        rep_ms = shard.max_over_ranks(e0.elapsed_time(e1), dev)
        same = all(torch.equal(got[k], outs[k.split("@")[0]]) for k in names)
        recv = (world - 1) * out_bytes
        replicate = {"ms": round(rep_ms, 3), "bytes_received_per_rank": recv,
                     "GBps_received_per_rank": round(recv / (rep_ms / 1e3) / 1e9, 2),
                     "units": len(names), "copies_equal": same,
                     "path": "shard.replicate_units: one NCCL all-gather per tensor of the layer"}
        del got

    res = {"config": "llama2-70b layer (BASELINE config 3), one copy per GPU"
                     + (f", subset {args.tensors}" if args.tensors else ""),
           "value": round(value, 3), "unit": "GB/s", "ms_per_step": round(ms_step, 3),
           "steps_timed": steps, "scaling": "weak",
           "decoded_bytes_per_gpu_step": out_bytes, "compressed_bytes_per_gpu_step": comp_bytes,
           "e2e": {"value": round(e2e_value, 3), "unit": "GB/s", "ms_per_step": round(e2e_ms, 3),
                   "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world},
           "roofline": roof, "kernels": kern, "replicate": replicate}
    if cpu_ok(args):
        threads = os.cpu_count() or 1
        gbs, dt, elems, ref = cpu_decode_sample(files, threads, keep=True)
        res["cpu_baseline"] = {
            "value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{'+'.join(CPU_SAMPLE)} of the layer ({elems} elements, {dt:.1f} s): "
                      "oracle LZ4 + INT4 + scatter + f32 Makhoul IDCT, OpenMP"}
        res["cpu_baseline_scipy_idct"] = cpu_scipy_idct(files, threads)
        res["oracle_check"] = check_against_oracle(H, torch, dev, readers, outs, ref)
        del ref
    for r in readers.values():
        r.close()
    ctx.close()
    ctx2.close()
    res["_files"] = files
    res["_tens"] = TENS
    return res


def check_against_oracle(H, torch, dev, readers, outs, ref) -> dict:
    """The checker: the oracle's CPU decode of the sample tensors against the GPU's
    f32 decode of the same files (max-abs 1e-3, cosine 0.99999) and against the
    bf16 outputs of the timed steps (the same bound plus the bf16 half-ulp)."""
    res = {"tensors": sorted(ref), "max_abs_f32": 0.0, "min_cos_f32": 1.0,
           "max_excess_bf16": -1.0}
    for n, r in ref.items():
        g = readers[n].decode(H.F32).cpu().numpy()
        a, b = g.astype(np.float64).ravel(), r.astype(np.float64).ravel()
        res["max_abs_f32"] = max(res["max_abs_f32"], float(np.abs(a - b).max()))
        res["min_cos_f32"] = min(res["min_cos_f32"],
                                 float((a @ b) / np.sqrt((a @ a) * (b @ b))))
        gb = outs[n].float().cpu().numpy()
        ex = np.abs(gb - r) - (1e-3 + np.abs(r) * 2.0 ** -8)
        res["max_excess_bf16"] = max(res["max_excess_bf16"], float(ex.max()))
    res["ok"] = (res["max_abs_f32"] <= 1e-3 and res["min_cos_f32"] >= 0.99999
                 and res["max_excess_bf16"] <= 0.0)
    if not res["ok"]:
        raise AssertionError(f"GPU decode differs from the oracle: {res}")
    for k in ("max_abs_f32", "min_cos_f32", "max_excess_bf16"):
        res[k] = float(f"{res[k]:.6g}")
    return res


def _data_len(f: bytes) -> int:
    import struct

    nb = struct.unpack_from("<I", f, 32)[0]
    ver = struct.unpack_from("<I", f, 4)[0]
    flags = struct.unpack_from("<H", f, 10)[0]
    ent = 16 if (ver >= 2 and flags & 2) else 8
    q = 8 if (ver >= 2 and flags & 4) else 0
    return len(f) - 64 - q - nb * ent


def bench_v3(H, torch, dev, stream, files, tens, ctx):
    """The same layer as HCT V3 fragment containers (bitmap + fp16 coefficients, one
    fragment per tensor) decoded to bf16, inputs resident in HBM."""
    decs = {n: H.HctV3Decoder(files[n + ".v3"], m, c, ctx) for n, m, c in tens}
    outs = {n: torch.empty((m, c), dtype=torch.bfloat16, device=dev) for n, m, c in tens}

    def step():
        for n, _, _ in tens:
            decs[n].decode(H.BF16, out=outs[n], stream=stream)

    for _ in range(2):
        step()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for _ in range(reps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / reps
    out_bytes = sum(2 * m * c for _, m, c in tens)
    in_bytes = sum(len(files[n + ".v3"]) for n, _, _ in tens)
    for d in decs.values():
        d.close()
    return {"config": "BASELINE config 3 layer as HCT V3 fragments (bitmap + fp16, 1 per tensor)",
            "value": round(out_bytes / (ms / 1e3) / 1e9, 2), "unit": "GB/s bf16 out",
            "ms": round(ms, 3), "compressed_bytes": in_bytes,
            "path": "HctV3Decoder.decode per tensor (scatter -> factored IDCT), synchronous"}


def bench_holo(H, torch, dev, stream, files, tens, ctx):
    """The same layer as spectral HoloTensor files (HOLO_FRAGMENTS "SV03" raster slices of
    the f32 DCT coefficients per tensor), all fragments decoded to bf16, inputs resident
    in HBM."""
    readers = {n: H.HoloTensorReader(files[n + ".holo"], ctx) for n, _, _ in tens}
    outs = {n: torch.empty((m, c), dtype=torch.bfloat16, device=dev) for n, m, c in tens}

    def step():
        for n, _, _ in tens:
            readers[n].decode(out_dtype=H.BF16, out=outs[n], stream=stream)

    for _ in range(2):
        step()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for _ in range(reps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / reps
    out_bytes = sum(2 * m * c for _, m, c in tens)
    in_bytes = sum(len(files[n + ".holo"]) for n, _, _ in tens)
    for r in readers.values():
        r.close()
    return {"config": f"BASELINE config 3 layer as spectral HoloTensor files "
                      f"({HOLO_FRAGMENTS} SV03 fragments of f32 coefficients per tensor)",
            "value": round(out_bytes / (ms / 1e3) / 1e9, 2), "unit": "GB/s bf16 out",
            "ms": round(ms, 3), "file_bytes": in_bytes,
            "path": "HoloTensorReader.decode per tensor (SV03 interleave -> factored IDCT), "
                    "synchronous"}


def bench_zstd(H, torch, dev, stream, args):
    """The LZ4 config-2 data (256 MiB of N(0,0.02) fp16, seed 1) as 4096 independent
    64 KiB zstd frames (level 3), decoded in one batched launch (a warp per frame)."""
    from haagenti_b200 import encode as E

    rng = np.random.default_rng(1)
    raw = (rng.standard_normal(128 * 1024 * 1024, dtype=np.float32) * np.float32(0.02)).astype(
        np.float16).view(np.uint8)
    chunk = 65536
    nb = raw.size // chunk
    frames = [E.zstd_compress(raw[i * chunk:(i + 1) * chunk], 3) for i in range(nb)]
    jobs = np.zeros(nb, dtype=H.ZSTD_JOB)
    offs = np.zeros(nb + 1, np.uint64)
    offs[1:] = np.cumsum([(len(f) + 15) // 16 * 16 for f in frames])
    jobs["src_off"] = offs[:-1]
    jobs["src_len"] = [len(f) for f in frames]
    jobs["dst_off"] = np.arange(nb, dtype=np.uint64) * chunk
    jobs["dst_cap"] = chunk
    packed = np.zeros(int(offs[-1]), np.uint8)
    for i, f in enumerate(frames):
        packed[int(offs[i]): int(offs[i]) + len(f)] = np.frombuffer(f, np.uint8)
    d_src = torch.from_numpy(packed).to(dev)
    d_dst = torch.empty(raw.size, dtype=torch.uint8, device=dev)
    z = H.ZstdDecompressor()
    st = z.decompress_jobs(d_src, jobs, d_dst, stream)
    ok = bool((st["code"] == 0).all()) and bool(
        torch.equal(d_dst, torch.from_numpy(raw).to(dev)))
    from haagenti_b200 import _lib as L
    lib = L.load()
    d_jobs = torch.from_numpy(jobs.view(np.uint8).copy()).to(dev)
    d_status = torch.zeros(nb * 32, dtype=torch.uint8, device=dev)

    def launch():
        lib.hct_b200_zstd_decompress_jobs(z.ctx.handle, d_src.data_ptr(), d_jobs.data_ptr(), nb,
                                          d_dst.data_ptr(), d_status.data_ptr(), stream.cuda_stream)

    for _ in range(3):
        launch()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for _ in range(reps):
        launch()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / reps

    # one large frame (the form of a zstd-compressed weight fragment): its
    # 128 KiB blocks decode in parallel; as zstd::encode_all writes it (no
    # content checksum) and with a checksum (XXH64 of the frame is serial)
    big = raw[: 64 << 20]
    bjob = np.zeros(1, dtype=H.ZSTD_JOB)
    b_dst = torch.empty(big.size, dtype=torch.uint8, device=dev)
    ref_big = torch.from_numpy(big).to(dev)

    def time_big(checksum):
        bf = E.zstd_compress(big, 3, checksum=checksum)
        b_src = torch.from_numpy(np.frombuffer(bf, np.uint8).copy()).to(dev)
        bjob[0] = (0, len(bf), 0, big.size)
        b_jobs = torch.from_numpy(bjob.view(np.uint8).copy()).to(dev)

        def launch_big():
            lib.hct_b200_zstd_decompress_jobs(z.ctx.handle, b_src.data_ptr(), b_jobs.data_ptr(), 1,
                                              b_dst.data_ptr(), d_status.data_ptr(),
                                              stream.cuda_stream)

        for _ in range(3):
            launch_big()
        torch.cuda.synchronize(dev)
        n = 10 if not checksum else 3
        e0.record(stream)
        for _ in range(n):
            launch_big()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ms_b = e0.elapsed_time(e1) / n
        ok_b = (int(d_status[:4].view(torch.int32)[0]) == 0 and bool(torch.equal(b_dst, ref_big)))
        return ms_b, ok_b

    ms_big, ok_big = time_big(False)
    ms_ck, ok_ck = time_big(True)
    out = {"config": "BASELINE config 2 data (256 MiB fp16 N(0,0.02) seed 1) as 4096 x 64 KiB "
                     "zstd frames (libzstd level 3)",
           "value": round(raw.size / (ms / 1e3) / 1e9, 2), "unit": "GB/s decompressed",
           "ms": round(ms, 3), "ratio": round(raw.size / sum(len(f) for f in frames), 4),
           "bytes_checked_ok": ok,
           "single_frame": {"config": "first 64 MiB of the same data as one frame (level 3, "
                                      "no content checksum, as zstd::encode_all; 512 blocks "
                                      "decoded block-parallel)",
                            "value": round(big.size / (ms_big / 1e3) / 1e9, 2),
                            "unit": "GB/s decompressed", "ms": round(ms_big, 3),
                            "bytes_checked_ok": ok_big,
                            "with_checksum": {"value": round(big.size / (ms_ck / 1e3) / 1e9, 2),
                                              "ms": round(ms_ck, 3), "bytes_checked_ok": ok_ck,
                                              "note": "XXH64 of one frame is a serial chain"}}}
    if not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_zstd_sample(frames, raw.size)
    return out


def bench_lz4(H, torch, dev, stream, args):
    """256 MiB of N(0,0.02) fp16 (seed 1), 4096 independent 64 KiB blocks."""
    from haagenti_b200 import _lib as L
    from haagenti_b200 import encode as E

    rng = np.random.default_rng(1)
    raw = (rng.standard_normal(128 * 1024 * 1024, dtype=np.float32) * np.float32(0.02)).astype(
        np.float16).view(np.uint8)
    packed, lens = E.lz4_compress_chunks(raw, 65536)
    nb = len(lens)
    blk = np.zeros(nb, dtype=[("src_off", "<u8"), ("dst_off", "<u8"), ("src_len", "<u4"),
                              ("dst_cap", "<u4"), ("out_size", "<u4"), ("pad", "<u4")])
    blk["src_off"][1:] = np.cumsum(lens[:-1], dtype=np.uint64)
    blk["dst_off"] = np.arange(nb, dtype=np.uint64) * 65536
    blk["src_len"] = lens
    blk["dst_cap"] = 65536
    blk["out_size"] = 65536
    d_src = torch.from_numpy(packed).to(dev)
    d_blk = torch.from_numpy(blk.view(np.uint8).copy()).to(dev)
    d_dst = torch.empty(raw.size, dtype=torch.uint8, device=dev)
    d_st = torch.zeros(nb * 32, dtype=torch.uint8, device=dev)
    lib = L.load()
    sp = stream.cuda_stream

    def launch():
        rc = lib.hct_b200_lz4_decompress_blocks(d_src.data_ptr(), d_blk.data_ptr(), nb,
                                                d_dst.data_ptr(), d_st.data_ptr(),
                                                int(lens.max()), sp)
        assert rc == 0

    for _ in range(3):
        launch()
    torch.cuda.synchronize(dev)
    ok = bool(torch.equal(d_dst[: 1 << 20].cpu(), torch.from_numpy(raw[: 1 << 20].copy())))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(args.steps, 5)
    e0.record(stream)
    for _ in range(reps):
        launch()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / reps
    pk = peaks()
    alg = raw.size + packed.size
    out = {"config": "BASELINE config 2 (256 MiB fp16 N(0,0.02) seed 1, 4096 x 64 KiB blocks)",
           "value": round(raw.size / (ms / 1e3) / 1e9, 2), "unit": "GB/s decompressed",
           "ms": round(ms, 4), "ratio": round(raw.size / packed.size, 4),
           "hbm_frac": round(alg / (ms / 1e3) / 1e9 / pk["hbm"], 4), "bytes_checked_ok": ok}
    if cpu_ok(args):
        import oracle

        threads = os.cpu_count() or 1
        d = np.zeros(nb, dtype=oracle.BLOCK_DESC)
        for f in ("src_off", "dst_off", "src_len", "dst_cap", "out_size"):
            d[f] = blk[f]
        oracle.lz4_decompress_batch(packed, d, raw.size, threads)
        t0 = time.perf_counter()
        reps_c = 3
        for _ in range(reps_c):
            got, st = oracle.lz4_decompress_batch(packed, d, raw.size, threads)
        dt = (time.perf_counter() - t0) / reps_c
        assert (st["code"] == 0).all() and np.array_equal(got, raw)
        out["cpu_baseline"] = {
            "value": round(raw.size / dt / 1e9, 3), "unit": "GB/s decompressed", "cores": threads,
            "kind": "port",
            "sample": f"all 4096 blocks, decompress_block restated (oracle/hct_oracle.c), one "
                      f"block per task over {threads} OpenMP threads, {dt:.3f} s per pass"}
    return out


def cpu_ok(args) -> bool:
    """CPU baselines run on rank 0 of a one-GPU run only."""
    return (not args.no_cpu_baseline and int(os.environ.get("WORLD_SIZE", "1")) == 1
            and int(os.environ.get("RANK", "0")) == 0)


def bench_int4(H, torch, dev, stream, args):
    """dequantize_int4 of 4096x4096 (seed 0) to f32."""
    import ctypes as C
    from haagenti_b200 import _lib as L
    from haagenti_b200 import encode as E

    w = E.synthetic_weight((4096, 4096), 0)
    q = E.quantize_int4(w)
    # 4 input/output pairs (306 MB) rotated so no launch finds its data in the 126 MB L2
    copies = 4
    d_q = [torch.from_numpy(q).to(dev) for _ in range(copies)]
    outs = [torch.empty(w.size, dtype=torch.float32, device=dev) for _ in range(copies)]
    lib = L.load()
    written = C.c_size_t(0)
    sp = stream.cuda_stream

    def launch(i):
        rc = lib.hct_b200_dequantize_int4(d_q[i % copies].data_ptr(), q.size, w.size,
                                          outs[i % copies].data_ptr(), L.F32, C.byref(written), sp)
        assert rc == 0

    for i in range(3):
        launch(i)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 48
    e0.record(stream)
    for i in range(reps):
        launch(i)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / reps
    alg = q.size + 4 * w.size
    pk = peaks()
    # the four copies in one batched launch (hct_b200_dequantize_int4_batch), as a
    # loader decoding a model of plain INT4 tensors would call it
    jobs = (L.Int4Job * copies)()
    for i in range(copies):
        jobs[i] = L.Int4Job(d_q[i].data_ptr(), q.size, w.size, outs[i].data_ptr())
    wr = (C.c_size_t * copies)()

    def launch_batch():
        rc = lib.hct_b200_dequantize_int4_batch(jobs, copies, L.F32, wr, sp)
        assert rc == 0

    for _ in range(3):
        launch_batch()
    reps_b = 12
    e0.record(stream)
    for _ in range(reps_b):
        launch_batch()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms_b = e0.elapsed_time(e1) / reps_b / copies  # per tensor
    out = {"config": "BASELINE config 1 (4096x4096 seed 0, f32 out)",
           "value": round(4 * w.size / (ms / 1e3) / 1e9, 2), "unit": "GB/s f32 out",
           "ms": round(ms, 4), "hbm_frac": round(alg / (ms / 1e3) / 1e9 / pk["hbm"], 4),
           "l2": "4 rotating input/output pairs (306 MB) > 126 MB L2",
           "batched": {"value": round(4 * w.size / (ms_b / 1e3) / 1e9, 2),
                       "unit": "GB/s f32 out", "ms_per_tensor": round(ms_b, 4),
                       "hbm_frac": round(alg / (ms_b / 1e3) / 1e9 / pk["hbm"], 4),
                       "path": f"{copies} tensors per hct_b200_dequantize_int4_batch launch"}}
    if cpu_ok(args):
        import oracle

        threads = os.cpu_count() or 1
        ref = oracle.dequantize_int4_threads(q, w.size, threads)
        t0 = time.perf_counter()
        reps_c = 10
        for _ in range(reps_c):
            oracle.dequantize_int4_threads(q, w.size, threads)
        dt = (time.perf_counter() - t0) / reps_c
        got = outs[(reps - 1) % copies].cpu().numpy()
        out["bit_exact"] = bool(np.array_equal(got.view(np.uint32), ref.view(np.uint32)))
        out["cpu_baseline"] = {
            "value": round(4 * w.size / dt / 1e9, 3), "unit": "GB/s f32 out", "cores": threads,
            "kind": "port",
            "sample": f"the whole config-1 tensor, dequantize_int4 restated (oracle/hct_oracle.c) "
                      f"over {threads} OpenMP threads by 32-element block, {1e3 * dt:.2f} ms"}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-bind", action="store_true",
                    help="leave the process unbound (default: the GPU's local CPUs)")
    ap.add_argument("--interleave-uploads", dest="upload_first", action="store_false",
                    help="end to end: upload each file just before its decode "
                         "(default: a step's uploads are enqueued before its decodes)")
    ap.add_argument("--priority", type=int, default=0,
                    help="whole-model legs: decode streams at this priority above the default")
    ap.add_argument("--window", type=int, default=MODEL_WINDOW,
                    help="whole-model legs: decodes in flight before a status is read back")
    ap.add_argument("--no-secondary", action="store_true", help="skip the LZ4 / INT4 lines")
    ap.add_argument("--tensors", default="", help="comma list of layer tensors (default: all)")
    ap.add_argument("--idct", choices=["auto", "scatter", "dense"], default="auto",
                    help="IDCT mode of the decode context (hct_b200_ctx_set_idct)")
    ap.add_argument("--leg", choices=["zstd", "lz4", "int4", "layer", "model", "model8b"],
                    default="",
                    help="run only this secondary measurement on cuda:0 and print its object")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.leg:
        return run_leg(args)
    return run_b200(args)


def run_leg(args):
    """One secondary measurement alone (profiling runs of its kernels)."""
    import torch

    import haagenti_b200 as H

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    args.host_binding = bind_host_cpus(torch, 0, not args.no_bind)
    stream = torch.cuda.current_stream(dev)
    if args.leg in ("model", "model8b", "layer"):
        # the decode legs alone on one GPU (profiling runs of their kernels)
        if args.leg == "layer":
            res = layer_leg(H, torch, dev, args, 1, 0, 0, lambda: None)
            res.pop("_files")
            res.pop("_tens")
        else:
            arch, seed = ("llama2-70b", 4) if args.leg == "model" else ("llama3-8b", 3)
            res = model_leg(H, torch, dev, args, arch, seed, 1, 0, 0, lambda: None)
        print(json.dumps({"leg": args.leg, **res}), flush=True)
        return 0
    fn = {"zstd": bench_zstd, "lz4": bench_lz4, "int4": bench_int4}[args.leg]
    print(json.dumps({"leg": args.leg, **fn(H, torch, dev, stream, args)}), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
