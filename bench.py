"""Benchmark of the quantized decode GEMV path (BASELINE.json metric: weight-stream
GB/s per quant matvec).

Workload (the configuration the metric is quoted on): one step =
one batch-1 GEMV over each of 16 resident packs, {Q4_K, Q5_K, IQ2_S, IQ3_S} x
{4096x4096, 14336x4096, 4096x14336, 128256x8192} (out x in), through the C-ABI
entry point qg_gemv.  Packs are seeded synthetic data with the BASELINE
distributions; 2.37 GB of packs per step, far larger than L2, so no flush is needed.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

value       = algorithmic bytes (packed weights + x + y) of all GEMVs / device time,
              summed over ranks (each rank runs the whole sweep: weak scaling).
e2e         = the same metric with every step's x copied from pinned host memory and
              every y copied back inside the timed region.
roofline    = the dominant GEMV's algorithmic bytes / its CUDA-event time vs the
              measured HBM copy bandwidth (MEASURED_PEAKS.json).
cpu_baseline= the reference's own CPU matvec (oracle/_ref; the C restatement if the
              reference was not built) on a bounded row sample, all host threads.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "local-ai-gpu-acceleration_b200"))

import numpy as np  # noqa: E402

from qgemv_b200 import packs  # noqa: E402

SWEEP_FORMATS = [packs.Q4K_RAW, packs.Q5K, packs.IQ2S, packs.IQ3S]
SWEEP_SHAPES = [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 8192)]
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum, one ncu capture
# each, `ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum --clock-control none
# -k regex:gemv_tiled -s 2 -c 1 python bench.py --only F:128256x8192 --steps 3 --warmup 3`) of the sweep's
# largest GEMVs, one of which is the dominant kernel of the step.
TRAFFIC_BYTES = {
    (packs.Q4K_RAW, 128256, 8192): 591090688 + 2896640,
    (packs.Q5K, 128256, 8192): 722437376 + 3758592,
    (packs.IQ2S, 128256, 8192): 336776960 + 3912448,
    (packs.IQ3S, 128256, 8192): 451657728 + 3459072,
}
METRIC = "weight-stream GB/s, quant matvec sweep (Q4_K/Q5_K/IQ2_S/IQ3_S x 4 shapes, batch 1)"
CONFIG = {
    "workload": "BASELINE config 2: batch-1 GEMV sweep {Q4_K,Q5_K,IQ2_S,IQ3_S} x "
                "{4096x4096,14336x4096,4096x14336,128256x8192} (out x in), 16 GEMVs per step",
    "batch": 1,
    "l2": "no flush: 2.37 GB of packs streamed per step (> 126 MB L2)",
    "entry_point": "qg_act_prepare once per distinct x + qg_gemv_act per GEMV (C-ABI), one CUDA graph per step",
    "activation_precision": "fp32 x quantized per 32 columns into two int8 planes "
                            "(x ~= s*(hi + lo/256), |error| <= 3.2e-5*||x||_inf per element) for "
                            "the batch-1 GEMVs; int16 per (vector, column slice) on the CUDA-core "
                            "multi-vector path (batch 2-4, |error| <= 1.6e-5*||x||_inf); fp16 "
                            "(power-of-two scaled per row) on the tcgen05 batched path (batch >= 5); "
                            "fp32 accumulation and fp32 outputs",
}


def algorithmic_bytes(fmt: int, rows: int, cols: int, batch: int = 1) -> int:
    return packs.pack_bytes(fmt, rows, cols) + 4 * batch * (cols + rows)


def measured_peak() -> tuple[float, str]:
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return float(json.loads(path.read_text())["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback 6.65 TB/s"


def prewarm(fn, sync, seconds: float = 0.6, minimum: int = 3) -> int:
    """Untimed calls of `fn` for at least `seconds` of wall time (and `minimum` calls),
    so that SM clocks have ramped up from idle before a timed region; `sync` drains the
    queue every few calls.  Only for work without collectives (ranks may differ in the
    number of calls)."""
    t0 = time.perf_counter()
    n = 0
    while n < minimum or time.perf_counter() - t0 < seconds:
        fn()
        n += 1
        if n % 4 == 0:
            sync()
    sync()
    return n


class ClockSampler:
    """nvidia-smi sampling of SM clocks / throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self) -> dict:
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (self.out or "").splitlines():
            f = [p.strip() for p in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax),
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_reference_sample(row_fraction: int, threads: int, seed: int = 0) -> dict:
    """Time the reference's CPU matvec on the first rows/row_fraction rows of every
    sweep matrix (same formats, cols and value distributions)."""
    sys.path.insert(0, str(REPO / "oracle"))
    import qoracle

    ref = qoracle.Ref.load(build=False)
    kind = "reference"
    if ref is None:
        ref, kind = None, "port"
        port = qoracle.Port()
    total_bytes, total_t = 0, 0.0
    for fmt in SWEEP_FORMATS:
        for rows, cols in SWEEP_SHAPES:
            r = max(16, rows // row_fraction)
            pk = packs.synthetic_pack(fmt, r, cols, seed=seed + fmt * 7 + rows + cols)
            x = packs.synthetic_activation(cols, fmt)
            if ref is not None:
                t, _ = ref.time_matvec(fmt, pk.payload, pk.meta, x, r, cols, threads)
            else:
                t0 = time.perf_counter()
                port.matvec(fmt, pk.payload, pk.meta, x, r, cols)
                t = time.perf_counter() - t0
            total_t += t
            total_bytes += algorithmic_bytes(fmt, r, cols)
    used = threads if kind == "reference" else 1
    return {"value": total_bytes / total_t / 1e9, "unit": "GB/s", "cores": used, "kind": kind,
            "sample": f"first rows/{row_fraction} rows (min 16) of each of the 16 sweep matrices, "
                      f"{total_bytes / 1e6:.1f} MB of packs, {total_t:.2f} s wall on {used} threads"}


def run_reference(args) -> int:
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    threads = os.cpu_count() or 1
    fraction = 32
    cpu_reference_sample(256, threads)  # warm-up of the code path (not timed)
    vals = []
    for _ in range(args.warmup):
        cpu_reference_sample(fraction, threads, seed=1)
    t0 = time.perf_counter()
    for k in range(args.steps):
        vals.append(cpu_reference_sample(fraction, threads, seed=2 + k))
    elapsed = time.perf_counter() - t0
    value = statistics.median(v["value"] for v in vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": elapsed / max(1, args.steps) * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded packs, BASELINE distributions)",
        "config": dict(CONFIG, sample=vals[0]["sample"]),
        "cpu_baseline": {k: vals[0][k] for k in ("kind", "cores", "sample")} | {"value": value, "unit": "GB/s"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


def measure_slice(device, args) -> dict:
    """one mixed-format layer slice (hidden 4096, Q/K/V/O IQ3_S,
    gate/up IQ2_S, down Q5_K) captured as one graph with the C-ABI graph API and
    replayed; reported beside the headline metric."""
    import torch

    from qgemv_b200.slice import LayerSlice, StepGraph

    sl = LayerSlice(seed=3, device=device)
    x = torch.randn(sl.dims["hidden"], device=device)
    out = torch.empty_like(x)
    stream = torch.cuda.Stream(device)
    sl.forward(x, out, stream)  # eager warm-up (kernel attributes)
    stream.synchronize()
    g = StepGraph(stream, lambda: sl.forward(x, out, stream))
    for _ in range(max(3, args.warmup)):
        g.launch()
    prewarm(g.launch, stream.synchronize, seconds=0.4)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    n = max(20, args.steps * 5)
    e0.record(stream)
    for _ in range(n):
        g.launch()
    e1.record(stream)
    stream.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / n
    g.close()
    res = {"workload": "BASELINE config 3 layer slice, 8 kernels in one graph",
           "us_per_step": us, "steps_per_s": 1e6 / us,
           "weight_bytes": sl.weight_bytes, "GBps": sl.weight_bytes / (us * 1e-6) / 1e9}
    res["batch_buckets"] = measure_slice_buckets(sl, device, stream, args)
    return res


SLICE_BUCKETS = [1, 2, 4, 8, 16]


def measure_slice_buckets(sl, device, stream, args) -> dict:
    """The same slice for a batch of hidden vectors through one captured graph per batch
    bucket (qg_slice_buckets_*): each run copies the batch into its bucket's rows,
    replays that bucket's graph and copies the rows out (all inside the timed region)."""
    import torch

    from qgemv_b200.slice import SliceBuckets

    sb = SliceBuckets(sl, SLICE_BUCKETS, stream)
    cases = []
    for batch in [1, 2, 3, 4, 8, 16]:
        x = torch.randn(batch, sl.dims["hidden"], device=device)
        out = torch.empty_like(x)
        with torch.cuda.stream(stream):
            for _ in range(max(3, args.warmup)):
                sb.run(x, out)
            prewarm(lambda: sb.run(x, out), stream.synchronize, seconds=0.2)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            n = max(20, args.steps * 5)
            e0.record(stream)
            for _ in range(n):
                sb.run(x, out)
            e1.record(stream)
        stream.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / n
        cases.append({"batch": batch, "bucket": sb.bucket(batch), "us_per_step": round(us, 2),
                      "rows_per_s": round(batch * 1e6 / us, 1),
                      "weight_GBps": round(sl.weight_bytes / (us * 1e-6) / 1e9, 1)})
    sb.close()
    return {"buckets": SLICE_BUCKETS, "cases": cases,
            "path": "GEMVs: batch 1 GEMV, 2-4 CUDA-core multi-vector, >= 5 tensor-core tiles"}


REF_LAUNCHERS = {
    # the reference's launcher per sweep format (decode_kernels.h:345-394,502-513); the
    # Q4_K one is its fastest raw-block variant, the others take rows_limit = rows
    packs.Q4K_RAW: ("rtxllm_launch_q4k_matvec_decode_warp_broadcast_vec4x4", False),
    packs.Q5K: ("rtxllm_launch_q5k_matvec_decode_probe", True),
    packs.IQ2S: ("rtxllm_launch_iq2s_matvec_decode_probe", True),
    packs.IQ3S: ("rtxllm_launch_iq3s_matvec_decode_probe", True),
}


def measure_reference_gpu(device, mats, xs, args) -> dict | None:
    """The reference's own GPU launchers -- runtime/kernels/decode/decode_kernels.cu compiled
    unmodified for sm_100a into oracle/_ref -- on the sweep's packs, beside this library's
    launchers of the same names and arguments (logits + token update, no KV pages).  One
    step = the 16 matrices in sweep order (no L2 reuse between uses of a matrix); per-launch
    times from event nodes inside one graph per arm, after an untimed warm-up."""
    import ctypes

    import torch

    from qgemv_b200 import _lib

    path = REPO / "oracle" / "_ref" / "libref_oracle.so"
    if not path.exists():
        return None
    arms = {"reference": ctypes.CDLL(str(path)), "ours": _lib.lib()}
    P, U = ctypes.c_void_p, ctypes.c_uint32
    token = torch.zeros(1, dtype=torch.int32, device=device)
    kv = torch.zeros(64, dtype=torch.float32, device=device)
    stream = torch.cuda.Stream(device)
    out = {}
    for arm, lib in arms.items():
        fns = {}
        for fmt, (name, has_limit) in REF_LAUNCHERS.items():
            fn = getattr(lib, name)
            fn.restype = ctypes.c_int
            fn.argtypes = [P, P, P, P, P, U, U] + ([U] if has_limit else []) + [U, U, U, P]
            fns[fmt] = (fn, has_limit)

        def step(events=None, fns=fns):
            for i, m in enumerate(mats):
                fn, has_limit = fns[m["fmt"]]
                lim = (m["rows"],) if has_limit else ()
                rc = fn(m["payload"].data_ptr(), xs[m["cols"]].data_ptr(), m["y"].data_ptr(), kv.data_ptr(),
                        token.data_ptr(), m["rows"], m["cols"], *lim, 0, 0, 0, stream.cuda_stream)
                if rc != 0:
                    raise RuntimeError(f"{arm} launcher for format {m['fmt']} returned {rc}")
                if events is not None:
                    events[i + 1].record(stream)

        with torch.cuda.stream(stream):
            step()
        stream.synchronize()
        evs = [[torch.cuda.Event(enable_timing=True, external=True) for _ in range(len(mats) + 1)]
               for _ in range(args.steps)]
        graphs = []
        for ev in evs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                ev[0].record(stream)
                step(ev)
            graphs.append(g)
        with torch.cuda.stream(stream):
            prewarm(lambda: [g.replay() for g in graphs], stream.synchronize, seconds=0.5, minimum=1)
            for g in graphs:
                g.replay()
        stream.synchronize()
        out[arm] = [statistics.median(ev[i].elapsed_time(ev[i + 1]) for ev in evs) for i in range(len(mats))]
        del graphs
    per = []
    for i, m in enumerate(mats):
        r_ms, o_ms = out["reference"][i], out["ours"][i]
        per.append({"format": packs.FORMAT_NAMES[m["fmt"]], "rows": m["rows"], "cols": m["cols"],
                    "reference_us": round(r_ms * 1e3, 2), "ours_us": round(o_ms * 1e3, 2),
                    "speedup": round(r_ms / o_ms, 2)})
    total_bytes = sum(m["bytes"] for m in mats)
    ref_ms, our_ms = sum(out["reference"]), sum(out["ours"])
    return {"kind": "reference GPU kernels (decode_kernels.cu, unmodified, compiled for sm_100a)",
            "launchers": {packs.FORMAT_NAMES[f]: n for f, (n, _) in REF_LAUNCHERS.items()},
            "sweep_us_reference": round(ref_ms * 1e3, 1), "sweep_us_ours": round(our_ms * 1e3, 1),
            "GBps_reference": round(total_bytes / (ref_ms * 1e-3) / 1e9, 1),
            "GBps_ours": round(total_bytes / (our_ms * 1e-3) / 1e9, 1),
            "speedup": round(ref_ms / our_ms, 2), "per_matvec": per}


BATCHED_FORMATS = [packs.Q4K_RAW, packs.IQ2S]
BATCHED_SHAPES = [(28672, 8192), (8192, 28672)]
BATCHED_SIZES = [1, 8, 16, 32]
# first batch qg_gemm_batched runs on the tensor cores (the library reads the same variable)
TC_MIN_BATCH = int(os.environ.get("QG_TC_MIN_BATCH", "5"))


def batch_slices(fmt: int, batch: int, rows: int, cols: int) -> int:
    """Column slices (= launches per 8-vector group) of the multi-vector GEMV: 8 warps of
    32 sub-blocks per slice with 5..8 vectors, 16 warps with 2..4."""
    kb = cols // 256
    per = 4 * (8 if min(batch, 8) > 4 else 16)
    return -(-kb // per)


def measure_batched(device, args, peak: float, only: tuple | None = None) -> dict:
    """{Q4_K, IQ2_S} x {28672x8192, 8192x28672} at batch 1, 8, 16, 32.
    Batch 1 is the GEMV (qg_act_prepare + qg_gemv_act); batch 2..15 is qg_gemm_batched's
    CUDA-core multi-vector GEMV (one weight pass per 8 vectors, one launch per column
    slice), batch >= 16 its tensor-core path.  Each graph replay walks a rotation of pack copies totalling >= 400 MB,
    so no call finds its weights in L2; time per call = replay time / copies."""
    import torch

    from qgemv_b200 import ops

    stream = torch.cuda.Stream(device)
    cases = []
    formats, shapes, sizes = BATCHED_FORMATS, BATCHED_SHAPES, BATCHED_SIZES
    if only is not None:  # profiling case: one (format, rows, cols, batch)
        formats, shapes, sizes = [only[0]], [(only[1], only[2])], [only[3]]
    for fmt in formats:
        for rows, cols in shapes:
            pk = packs.synthetic_pack(fmt, rows, cols, seed=rows ^ cols ^ fmt)
            nbytes = packs.pack_bytes(fmt, rows, cols)
            copies = max(2, -(-400_000_000 // nbytes))
            base = torch.from_numpy(pk.payload).to(device)
            payloads = [base] + [base.clone() for _ in range(copies - 1)]
            del pk
            for batch in sizes:
                x = torch.randn(batch, cols, device=device)
                y = torch.empty(batch, rows, device=device)
                if batch == 1:
                    act = torch.empty(ops.act_bytes(cols), dtype=torch.uint8, device=device)

                    def call(p, x=x, y=y, act=act):
                        ops.act_prepare(x[0], act, stream=stream)
                        ops.gemv_act(fmt, p, None, x[0], act, rows, cols, y=y[0], stream=stream)
                    launches = 2
                else:
                    ws = torch.empty(ops.gemm_batched_workspace_bytes(fmt, batch, rows, cols),
                                     dtype=torch.uint8, device=device)

                    def call(p, x=x, y=y, ws=ws, batch=batch):
                        ops.gemm_batched(fmt, p, None, x, rows, cols, y=y, workspace=ws, stream=stream)
                    launches = 3 if batch >= TC_MIN_BATCH else -(-batch // 8) * batch_slices(fmt, batch, rows, cols)
                with torch.cuda.stream(stream):
                    for p in payloads:  # eager warm-up: kernel attributes
                        call(p)
                stream.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    for p in payloads:
                        call(p)
                with torch.cuda.stream(stream):
                    for _ in range(max(3, args.warmup)):
                        g.replay()
                    prewarm(g.replay, stream.synchronize, seconds=0.3)
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                reps = max(5, args.steps)
                with torch.cuda.stream(stream):
                    e0.record(stream)
                    for _ in range(reps):
                        g.replay()
                    e1.record(stream)
                stream.synchronize()
                us = e0.elapsed_time(e1) * 1e3 / (reps * copies)
                gbps = nbytes / (us * 1e-6) / 1e9
                cases.append({
                    "fmt": packs.FORMAT_NAMES[fmt], "rows": rows, "cols": cols, "batch": batch,
                    "path": "gemv" if batch == 1 else "tcgen05" if batch >= TC_MIN_BATCH else "cuda-core multi-vector",
                    "us": round(us, 2),
                    "weight_GBps": round(gbps, 1), "frac_hbm": round(gbps / peak, 3),
                    "TFLOPs": round(2.0 * rows * cols * batch / (us * 1e-6) / 1e12, 2),
                    "launches": launches,
                })
                del g
            del payloads, base
            torch.cuda.empty_cache()
    return {"workload": "BASELINE config 4: {Q4_K, IQ2_S} x {28672x8192, 8192x28672} x batch {1,8,16,32}",
            "l2": ">= 400 MB of pack copies rotated per replay", "cases": cases}


def measure_decode(device, args, world: int, rank: int, layers: int | None = None) -> dict:
    """the 80-layer 70B-class mixed-quant decode step (IQ3_S
    attention, IQ2_S gate/up, Q5_K down, Q4_K vocab head, fp16 KV cache at context
    4096), tensor-parallel over the job's N GPUs, one graph per token.  Every rank cuts
    its shards from the same seeded global weights.  With N > 1 the step is timed twice:
    exchanges fused into the GEMVs over NVLink peer memory (the reported numbers) and the
    same exchange words moved by ncclAllGather between the kernels (`nccl`, the baseline);
    then rank 0 runs the same step unsharded (TP 1, the whole model on one GPU) and
    reports whether the token and the final hidden state are bit-identical."""
    import torch
    import torch.distributed as dist

    from qgemv_b200 import decoder, ops
    from qgemv_b200.slice import StepGraph

    spec = decoder.ModelSpec() if layers is None else decoder.ModelSpec(layers=layers)
    w = decoder.synthetic_rank_weights(spec, rank, world, device, seed=1,
                                       keep_full=(world > 1 and rank == 0))
    gen = torch.Generator(device=device)
    gen.manual_seed(4242)
    x = torch.randn(spec.hidden, device=device, generator=gen)  # same on every rank
    pos = spec.ctx_max - 1

    def timed(weights, tp: int, tp_rank: int, collective: int, group: bool) -> dict:
        nid = None
        if tp > 1:
            obj = [decoder.nccl_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(obj, src=0)
            nid = obj[0]
        dec = decoder.Decoder(spec, weights, rank=tp_rank, tp=tp, nccl_id=nid, device=device,
                              collective=collective)
        stream = torch.cuda.Stream(device)
        stream.wait_stream(torch.cuda.current_stream(device))
        for _ in range(2):
            dec.step(x, pos, stream)
        stream.synchronize()
        g = StepGraph(stream, lambda: dec.step(x, pos, stream))
        # warm-up: a fixed number of replays on every rank (the graph holds collectives)
        for i in range(max(3, args.warmup) + 20):
            g.launch()
            if i % 4 == 3:
                stream.synchronize()
        stream.synchronize()
        if group:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            g.launch()
        e1.record(stream)
        stream.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        # a bounded exchange wait that ran out fails the measurement (the error word is
        # sticky over the replays)
        err = ops.get_error()
        if err:
            raise RuntimeError(f"decode step (tp {tp}) set error word {err:#x}")
        if group:
            t = torch.tensor([ms], dtype=torch.float64, device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        out = {"ms_per_token": ms, "tok_per_s": 1000.0 / ms, "token": int(dec.token.item()),
               "hidden": dec.hidden().clone()}
        g.close()
        dec.close()
        return out

    fused = timed(w, world, rank, decoder.COLLECTIVE_NVLINK, world > 1)
    res = {"workload": f"BASELINE config 5: {spec.layers}-layer 70B-class decode step, ctx 4096, batch 1",
           "tp": world}
    moved = spec.weight_bytes() + spec.kv_bytes_read(spec.ctx_max)
    res.update({"ms_per_token": fused["ms_per_token"], "tok_per_s": fused["tok_per_s"],
                "token": fused["token"], "GBps_aggregate": moved / (fused["ms_per_token"] * 1e-3) / 1e9,
                "weight_bytes": spec.weight_bytes(), "kv_bytes": spec.kv_bytes_read(spec.ctx_max),
                "launches_per_token": spec.layers * 9 + 4})
    if world > 1:
        nccl = timed(w, world, rank, decoder.COLLECTIVE_NCCL, True)
        dist.barrier()
        if rank == 0:
            # TP 1 on rank 0: the whole model, the same x and position
            tp1 = timed(w["full"], 1, 0, decoder.COLLECTIVE_NVLINK, False)
            same = lambda a, b: bool(torch.equal(a.view(torch.int32), b.view(torch.int32)))  # noqa: E731
            res["collective"] = "fused NVLink exchange in the Wo/Wd GEMVs (pairwise rank tree)"
            res["nccl"] = {"ms_per_token": nccl["ms_per_token"], "tok_per_s": nccl["tok_per_s"],
                           "token": nccl["token"], "matches_tp1": nccl["token"] == tp1["token"] and
                           same(nccl["hidden"], tp1["hidden"])}
            res["tp1_on_rank0"] = {"ms_per_token": tp1["ms_per_token"], "tok_per_s": tp1["tok_per_s"],
                                   "token": tp1["token"]}
            res["token_tp1"] = tp1["token"]
            res["hidden_bits_equal_tp1"] = same(fused["hidden"], tp1["hidden"])
            res["matches_tp1"] = fused["token"] == tp1["token"] and res["hidden_bits_equal_tp1"]
            res["speedup_vs_tp1"] = tp1["ms_per_token"] / fused["ms_per_token"]
        dist.barrier()
    del w
    torch.cuda.empty_cache()
    return res


def run_ours(args) -> int:
    import torch
    import torch.distributed as dist

    from qgemv_b200 import check, ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    if args.only and args.only.startswith("batched:"):
        # profiling case: one batched GEMM, batched:FMT:ROWSxCOLS:BATCH
        _, f, shape, b = args.only.split(":")
        r, c = shape.lower().split("x")
        peak, _ = measured_peak()
        stats = measure_batched(device, args, peak, only=(int(f), int(r), int(c), int(b)))
        if rank == 0:
            print(json.dumps({"profiling_case": args.only, "batched": stats}))
        return 0
    if args.only == "slice":
        # the layer slice (config 3) alone: one graph, then the batch-bucket graphs
        stats = measure_slice(device, args)
        if rank == 0:
            print(json.dumps({"profiling_case": args.only, "slice": stats}))
        return 0
    if args.only and args.only.startswith("decode:"):
        # profiling case: the decode step alone with the given number of layers
        stats = measure_decode(device, args, world, rank, layers=int(args.only.split(":")[1]))
        if rank == 0:
            print(json.dumps({"profiling_case": args.only, "decode": stats}))
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return 0

    # Resident packs + activations (setup, untimed).
    mats = []
    xs = {}
    cases = [(f, r, c) for f in SWEEP_FORMATS for r, c in SWEEP_SHAPES]
    if args.only:
        f, shape = args.only.split(":")
        r, c = shape.lower().split("x")
        cases = [(int(f), int(r), int(c))]
    for fmt, rows, cols in cases:
        pk = packs.synthetic_pack(fmt, rows, cols, seed=1000 * fmt + rows + cols)
        payload, meta = ops.to_device(pk, device)
        if cols not in xs:
            xs[cols] = torch.from_numpy(packs.synthetic_activation(cols, cols)).to(device)
        y = torch.empty(rows, dtype=torch.float32, device=device)
        mats.append({"fmt": fmt, "rows": rows, "cols": cols, "payload": payload, "meta": meta,
                     "y": y, "bytes": algorithmic_bytes(fmt, rows, cols)})
        del pk
    stream = torch.cuda.current_stream(device)

    acts = {c: torch.empty(ops.act_bytes(c), dtype=torch.uint8, device=device) for c in xs}

    def launch(m, x, act):
        check("qg_gemv_act", m["fmt"], m["payload"].data_ptr(),
              None if m["meta"] is None else m["meta"].data_ptr(), x.data_ptr(), act.data_ptr(),
              m["y"].data_ptr(), m["rows"], m["cols"], torch.cuda.current_stream().cuda_stream)

    def step(events=None):
        # Each distinct x is prepared once (int8 planes), then read by every GEMV on it.
        for c in xs:
            check("qg_act_prepare", xs[c].data_ptr(), c, acts[c].data_ptr(),
                  torch.cuda.current_stream().cuda_stream)
        if events is not None:
            events[0].record()
        for i, m in enumerate(mats):
            launch(m, xs[m["cols"]], acts[m["cols"]])
            if events is not None:
                events[i + 1].record()

    for _ in range(max(3, args.warmup)):  # eager warm-up: sets kernel attributes, fills caches
        step()
    torch.cuda.synchronize()

    # The step as one CUDA graph (the way the reference replays its decode step); the
    # timed region is K replays of it.  Kernels carry programmatic-dependency edges, so
    # the graph has no event nodes between them.
    step_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(step_graph):
        step()
    for _ in range(max(3, args.warmup)):
        step_graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    with ClockSampler(local) as clocks:
        # keep the GPU busy (untimed) while the sampler starts and the clocks settle
        prewarm(step_graph.replay, torch.cuda.synchronize, seconds=0.6)
        if world > 1:
            dist.barrier()
        t_begin = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_begin.record(stream)
        for _ in range(args.steps):
            step_graph.replay()
        t_end.record(stream)
        torch.cuda.synchronize()
    elapsed_ms = t_begin.elapsed_time(t_end)
    if world > 1:
        t = torch.tensor([elapsed_ms], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
        dist.barrier()
    bytes_per_step = sum(m["bytes"] for m in mats)
    value = world * bytes_per_step * args.steps / (elapsed_ms * 1e-3) / 1e9

    # Per-GEMV durations: the same step with an event-record node after every GEMV
    # (one graph per replay so each keeps its own timestamps), replayed K times.
    graphs, evs = [], []
    for _ in range(args.steps):
        ev = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(len(mats) + 1)]
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step(ev)
        graphs.append(g)
        evs.append(ev)
    for g in graphs:
        g.replay()
    torch.cuda.synchronize()
    warm = 0

    per = []
    timed = evs[warm:]
    for i, m in enumerate(mats):
        ms = statistics.mean(timed[k][i].elapsed_time(timed[k][i + 1]) for k in range(args.steps))
        per.append({"format": packs.FORMAT_NAMES[m["fmt"]], "rows": m["rows"], "cols": m["cols"],
                    "ms": ms, "GBps": m["bytes"] / (ms * 1e-3) / 1e9})
    peak, peak_src = measured_peak()
    dom = max(range(len(mats)), key=lambda i: per[i]["ms"])
    dm = mats[dom]
    traffic = TRAFFIC_BYTES.get((dm["fmt"], dm["rows"], dm["cols"]))
    # The dominant GEMV alone: R launches back to back in one graph (its weights exceed
    # L2, so every launch streams them from HBM), CUDA events on the launching stream.
    R = 8
    chain = torch.cuda.CUDAGraph()
    with torch.cuda.graph(chain):
        for _ in range(R):
            launch(dm, xs[dm["cols"]], acts[dm["cols"]])
    prewarm(chain.replay, torch.cuda.synchronize, seconds=0.2)
    c0 = torch.cuda.Event(enable_timing=True)
    c1 = torch.cuda.Event(enable_timing=True)
    c0.record()
    for _ in range(args.steps):
        chain.replay()
    c1.record()
    torch.cuda.synchronize()
    dom_ms = c0.elapsed_time(c1) / (args.steps * R)
    del chain
    dom_gbps = dm["bytes"] / (dom_ms * 1e-3) / 1e9
    roofline = {
        "bound": "hbm", "kernel": f"gemv_tiled_kernel<{packs.FORMAT_NAMES[dm['fmt']]}> {dm['rows']}x{dm['cols']}",
        "achieved": dom_gbps, "peak": peak, "unit": "GB/s",
        "frac": dom_gbps / peak, "peak_source": peak_src,
        "launch_us": dom_ms * 1e3,
        "timing": f"{R} back-to-back launches of this GEMV in one graph, CUDA events, {args.steps} replays",
        "algorithmic_bytes_per_launch": dm["bytes"],
        "traffic": traffic,
        "traffic_source": None if traffic is None else
        "ncu dram__bytes_read.sum + dram__bytes_write.sum of the same kernel and shape (bench.py --only)",
    }
    for row in per:
        row["frac_of_peak"] = row["GBps"] / peak

    # End to end through the C-ABI: every step copies each distinct x from pinned host
    # memory, prepares it, runs the 16 GEMVs and copies every y back to pinned host
    # memory, as one graph.  The GEMVs run largest output first, and each y is copied
    # back on a side branch as soon as its GEMV has finished, overlapping the GEMVs
    # after it.
    host_x = {c: xs[c].cpu().pin_memory() for c in xs}
    host_y = [torch.empty(m["rows"], dtype=torch.float32).pin_memory() for m in mats]
    h2d = sum(4 * c for c in xs)
    d2h = sum(4 * m["rows"] for m in mats)
    side = torch.cuda.Stream(device)

    def e2e_body():
        main = torch.cuda.current_stream()
        for c in xs:  # the step's inputs: one host copy per distinct x
            xs[c].copy_(host_x[c], non_blocking=True)
        for c in xs:
            check("qg_act_prepare", xs[c].data_ptr(), c, acts[c].data_ptr(), main.cuda_stream)
        for i in sorted(range(len(mats)), key=lambda j: -mats[j]["rows"]):
            m = mats[i]
            launch(m, xs[m["cols"]], acts[m["cols"]])
            side.wait_stream(main)
            with torch.cuda.stream(side):
                host_y[i].copy_(m["y"], non_blocking=True)
        main.wait_stream(side)

    e2e_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(e2e_graph):
        e2e_body()

    def e2e_step():
        e2e_graph.replay()

    for _ in range(max(3, args.warmup)):
        e2e_step()
    prewarm(e2e_step, torch.cuda.synchronize, seconds=0.4)
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * bytes_per_step * args.steps / (e2e_ms * 1e-3) / 1e9

    del e2e_graph
    ref_gpu = measure_reference_gpu(device, mats, xs, args) if world == 1 and not args.only else None
    slice_stats = measure_slice(device, args) if not args.only else None
    launches_per_step = len(mats) + len(xs)
    del mats, step_graph, graphs
    torch.cuda.empty_cache()
    decode_stats = measure_decode(device, args, world, rank) if not args.only else None
    batched_stats = measure_batched(device, args, peak) if not args.only else None
    err = ops.get_error()
    if rank == 0:
        cpu = cpu_reference_sample(8, os.cpu_count() or 1) if world == 1 and not args.only else None
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded packs, BASELINE distributions)",
            "config": CONFIG,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "copies": "x from and every y to pinned host memory inside the step graph; "
                              "largest outputs first, each y copied back as soon as its GEMV ends"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks.summary(),
            "error_word": err,
            "per_matvec": per,
            "reference_gpu": ref_gpu,
            "slice": slice_stats,
            "batched": batched_stats,
            "decode": decode_stats,  # last: the driver keeps the end of the line
        }
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--only", default=None,
                    help="profiling case: run a single GEMV FMT:ROWSxCOLS (e.g. 0:32768x8192) "
                         "instead of the sweep, decode:LAYERS (the decode step alone with "
                         "that many layers), slice (config 3 and its batch-bucket graphs) "
                         "or batched:FMT:ROWSxCOLS:BATCH (one config-4 case); "
                         "skips the CPU baseline")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    raise SystemExit(main())
