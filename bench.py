"""Deep f32 MLP inference throughput on 1..8 B200 (samples/s).

Workload (the headline configuration): a global batch of 65536 rows x 4096
f32 features, 8 x [Linear(4096, 4096) + GELU], then Linear(4096, 1000) and a
row softmax.  Weights are Kaiming-normal (std sqrt(2/4096)), biases zero, the
input N(0, 1), all seeded synthetic data.  Each layer is the reference's op
sequence MATMUL -> ADD(bias) -> GELU (magnetron/magnetron_cpu.c:2151, :1616,
:942-1000), built as a deferred graph of magnetron tensors and executed by
this backend as one CUDA graph in which each layer is one tensor-core GEMM
(bias, GELU and the next layer's operand split in its epilogue); the softmax
is the backend's row-softmax extension.  The batch is sharded by rows over one process per GPU; logits are
collected with an NCCL all-gather.

One step = one forward over the whole batch.  `value` is whole-job samples/s
with inputs resident in HBM; `e2e` adds, every step, the host->device copy of
each rank's input shard from pinned host memory and the device->host copy of
each rank's rows of the softmax output (the ranks' copies run in parallel; the
all-gather still gives every GPU the whole output), both through the backend's
asynchronous copy API.  The activations (1 GiB per layer at one GPU) exceed the
126 MB L2, so no flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "magnetron-pre-oss-release-old_b200")
sys.path.insert(0, PKG)

GLOBAL_BATCH = 65536
D_IN, D_HID, N_HID, D_OUT = 4096, 4096, 8, 1000
METRIC = "MLP fwd samples/s"
FLOP_PER_SAMPLE = 2 * (N_HID * D_IN * D_HID + D_HID * D_OUT)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# The tensor-core matmul's operand split (MAG_CUDA_TC_SPLIT; the backend's default is f16).
SPLIT_NAME = "3xTF32" if os.environ.get("MAG_CUDA_TC_SPLIT") == "tf32" else "3xFP16 (scaled)"


def split_roofline(pk, pk_src):
    """Effective f32-product peak of the split: three tensor-core products per f32 product at
    the kind::f16 rate (the measured bf16 GEMM rate) or the kind::tf32 rate (half of it)."""
    bf16 = pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
    if SPLIT_NAME == "3xTF32":
        return bf16 / 2.0 / 3.0, f"3xTF32 effective = {pk_src} bf16 sustained / 2 (TF32 rate) / 3 (products)"
    return bf16 / 3.0, f"3xFP16 effective = {pk_src} bf16 sustained (f16 rate) / 3 (products)"


class ClockSampler:
    """SM clock and clock-event (throttle) reasons of one GPU, read through NVML
    every 5 ms while the timed region runs (read-only queries)."""

    def __init__(self, index: int, interval: float = 0.005):
        self.index = index
        self.interval = interval
        self.samples = []
        self.stamps = []
        self.reasons = set()
        self.max_mhz = None
        self.stop_flag = threading.Event()
        self.t = None
        self.err = None

    def start(self):
        try:
            import pynvml as N
            N.nvmlInit()
            self.N = N
            self.h = N.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = float(N.nvmlDeviceGetMaxClockInfo(self.h, N.NVML_CLOCK_SM))
            self.names = {N.nvmlClocksEventReasonHwSlowdown: "hw_slowdown",
                          N.nvmlClocksEventReasonHwThermalSlowdown: "hw_thermal_slowdown",
                          N.nvmlClocksEventReasonSwThermalSlowdown: "sw_thermal_slowdown",
                          N.nvmlClocksEventReasonSwPowerCap: "sw_power_cap"}
        except Exception as e:  # no NVML: report it instead of guessing
            self.err = str(e)
            return
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()

    def _run(self):
        N = self.N
        while not self.stop_flag.is_set():
            try:
                self.samples.append(float(N.nvmlDeviceGetClockInfo(self.h, N.NVML_CLOCK_SM)))
                self.stamps.append(time.perf_counter())
                bits = N.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for b, nm in self.names.items():
                    if bits & b:
                        self.reasons.add(nm)
            except Exception as e:
                self.err = str(e)
                return
            time.sleep(self.interval)

    def around(self, t0: float, t1: float):
        """Median SM clock sampled in [t0, t1], else the sample nearest to that window."""
        inside = [c for c, t in zip(self.samples, self.stamps) if t0 <= t <= t1]
        if inside:
            return statistics.median(inside)
        if not self.samples:
            return None
        mid = 0.5 * (t0 + t1)
        return min(zip(self.stamps, self.samples), key=lambda p: abs(p[0] - mid))[1]

    def stop(self):
        self.stop_flag.set()
        if self.t is not None:
            self.t.join(timeout=2)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [f"no samples: {self.err}"]}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ----------------------------------------------------------- CPU baselines
def _ref_mlp_rows(rows: int, seed: int, use_ref: bool):
    """Forward of `rows` samples through the reference library (or the oracle
    port when the reference library is absent); returns seconds."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle import Oracle, RefLib, REF_SO, pad6
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, D_IN), dtype=np.float32)
    ws = [(rng.standard_normal((D_IN, D_HID), dtype=np.float32) * np.float32((2.0 / D_IN) ** 0.5))
          for _ in range(N_HID)]
    wo = rng.standard_normal((D_HID, D_OUT), dtype=np.float32) * np.float32((2.0 / D_HID) ** 0.5)
    if use_ref and os.path.exists(REF_SO):
        R = RefLib()
        tx = R.tensor_nd((rows, D_IN))
        R.write(tx, x)
        tws = []
        for w in ws:
            t = R.tensor_nd((D_IN, D_HID))
            R.write(t, w)
            tws.append(t)
        to = R.tensor_nd((D_HID, D_OUT))
        R.write(to, wo)
        tb = R.tensor_nd((rows, D_HID))
        tbo = R.tensor_nd((rows, D_OUT))
        t0 = time.perf_counter()
        h = tx
        for t in tws:
            m = R.op("MATMUL", h, t)
            a = R.op("ADD", m, tb)
            g = R.op("GELU", a)
            if h is not tx:
                R.free(h)
            R.free(m, a)
            h = g
        z = R.op("MATMUL", h, to)
        z2 = R.op("ADD", z, tbo)
        logits = R.read(z2).reshape(rows, D_OUT)
        o = Oracle()
        o.softmax_rows(logits, rows, D_OUT)
        dt = time.perf_counter() - t0
        R.close()
        return dt, "reference"
    o = Oracle()
    t0 = time.perf_counter()
    h = x.reshape(-1)
    for w in ws:
        h = o.matmul(h, w, rows, D_IN, D_HID)
        h = o.unary("GELU", h, pad6((rows, D_HID)))
    z = o.matmul(h, wo, rows, D_HID, D_OUT)
    o.softmax_rows(z, rows, D_OUT)
    return time.perf_counter() - t0, "port"


_REF_STATE = {}


def _ref_init(seed):
    """Per-process set-up for the reference arm: one reference CPU context holding the weights."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle import RefLib, REF_SO
    rng = np.random.default_rng(seed)
    st = {}
    if os.path.exists(REF_SO):
        R = RefLib()
        ws = []
        for _ in range(N_HID):
            t = R.tensor_nd((D_IN, D_HID))
            R.write(t, rng.standard_normal(D_IN * D_HID, dtype=np.float32) * np.float32((2.0 / D_IN) ** 0.5))
            ws.append(t)
        wo = R.tensor_nd((D_HID, D_OUT))
        R.write(wo, rng.standard_normal(D_HID * D_OUT, dtype=np.float32) * np.float32((2.0 / D_HID) ** 0.5))
        st.update(R=R, ws=ws, wo=wo, kind="reference")
    else:
        st.update(ws=[rng.standard_normal(D_IN * D_HID, dtype=np.float32) * np.float32((2.0 / D_IN) ** 0.5)
                      for _ in range(N_HID)],
                  wo=rng.standard_normal(D_HID * D_OUT, dtype=np.float32) * np.float32((2.0 / D_HID) ** 0.5),
                  kind="port")
    _REF_STATE.update(st)


def _ref_step(rows):
    """One forward of `rows` samples on this process's context; returns (seconds, kind)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle import Oracle, pad6
    st = _REF_STATE
    x = np.random.default_rng(rows).standard_normal(rows * D_IN, dtype=np.float32)
    o = Oracle()
    t0 = time.perf_counter()
    if st["kind"] == "reference":
        R = st["R"]
        tx = R.tensor_nd((rows, D_IN))
        R.write(tx, x)
        tb, tbo = R.tensor_nd((rows, D_HID)), R.tensor_nd((rows, D_OUT))
        h = tx
        for w in st["ws"]:
            m = R.op("MATMUL", h, w)
            a = R.op("ADD", m, tb)
            g = R.op("GELU", a)
            R.free(h, m, a)
            h = g
        z = R.op("MATMUL", h, st["wo"])
        z2 = R.op("ADD", z, tbo)
        o.softmax_rows(R.read(z2), rows, D_OUT)
        R.free(h, z, z2, tb, tbo)
    else:
        h = x
        for w in st["ws"]:
            h = o.matmul(h, w, rows, D_IN, D_HID)
            h = o.unary("GELU", h, pad6((rows, D_HID)))
        o.softmax_rows(o.matmul(h, st["wo"], rows, D_HID, D_OUT), rows, D_OUT)
    return time.perf_counter() - t0, st["kind"]


def cpu_baseline():
    rows = 256
    dt, kind = _ref_mlp_rows(rows, 1234, True)
    return {"value": rows / dt, "unit": "samples/s", "cores": 1, "kind": kind,
            "sample": f"{rows} rows of the same MLP forward (8x4096^2 + 4096x1000 matmuls, GELU, softmax), "
                      f"single thread as the reference CPU backend runs ({dt:.1f} s)"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import multiprocessing as mp
    ncpu = os.cpu_count() or 1
    try:
        avail = int(open("/proc/meminfo").read().split("MemAvailable:")[1].split()[0]) * 1024
    except Exception:
        avail = 16 << 30
    procs = max(1, min(ncpu, int(avail // (2 << 30))))
    rows_per = 8
    ctx = mp.get_context("spawn")
    times = []
    kind = "reference"
    with ctx.Pool(procs, initializer=_ref_init, initargs=(1234,)) as pool:
        for step in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            res = pool.map(_ref_step, [rows_per] * procs, chunksize=1)
            dt = time.perf_counter() - t0
            kind = res[0][1]
            if step >= args.warmup:
                times.append(dt)
    per_step = statistics.median(times)
    value = procs * rows_per / per_step
    cfg = bench_config(args.gpus)
    line = {"metric": METRIC, "value": value, "unit": "samples/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg,
            "cpu_baseline": {"value": value, "unit": "samples/s", "cores": procs, "kind": kind,
                             "sample": f"{procs} processes x {rows_per} rows of the MLP forward per step "
                                       "(the reference CPU backend is single-threaded; rows are split across processes)"},
            "e2e": {"value": value, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def bench_config(n):
    return {"workload": "deep f32 MLP inference: batch 65536 x 4096, 8 x (Linear 4096x4096 + GELU), "
                        "Linear 4096x1000 + row softmax", "global_batch": GLOBAL_BATCH, "d_in": D_IN,
            "hidden_layers": N_HID, "d_out": D_OUT, "parallelism": f"dp{n} (rows sharded, logits all-gathered)",
            "l2_flush": "not needed: every activation (>= 128 MiB per rank at 8 GPUs) exceeds the 126 MB L2"}


# ----------------------------------------------------------------- ours
class _CudaArray:
    def __init__(self, ptr, n, stream):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3,
                                         "stream": None}


def sharded_check(dev, MB, torch, world, rank, local, stream):
    """Element ranges and the full SUM sharded over the ranks, checked against one GPU's result
    (run by every rank after the timed region, same collectives in the same order): every rank
    generates the same seeded 2^24 + 6-element vectors, adds its contiguous range, the ranges are
    all-gathered over NCCL and compared bit for bit with the whole ADD on this GPU; each rank
    reduces its range to a 24-byte record, the records are combined in rank order into the full
    SUM, compared with the one-GPU full SUM of the same vector."""
    import torch.distributed as dist
    import dp

    total = (1 << 24) + 6  # not a multiple of 2, 4 or 8 ranks: shards of unequal length
    start, n = dp.shard_rows(total, world, rank)
    dvc = torch.device("cuda", local)
    x, y, rf = dev.tensor((total,)), dev.tensor((total,)), dev.tensor((total,))
    xs, ys, rs = dev.tensor((n,)), dev.tensor((n,)), dev.tensor((n,))
    dev.fill_random_normal(x, 0.0, 1.0, MB.Pcg(0x5EED0E00))
    dev.fill_random_normal(y, 0.0, 1.0, MB.Pcg(0x5EED0E01))
    view = lambda t, k: torch.as_tensor(_CudaArray(t.data_ptr, k, dev.stream), device=dvc)
    # this rank's range, copied by the backend (x * 1.0 is x), so it knows the shard is written
    for src, dst in ((x, xs), (y, ys)):
        MB.check(dev.L.mag_cuda_unary_f32(dev.p, MB.OP["MULS"], dst.data_ptr, src.data_ptr + 4 * start, 1, n, n, n,
                                          1.0), "range copy")
    d6 = lambda k: (MB.i64x6([k, 1, 1, 1, 1, 1]), MB.i64x6(MB.strides6([k, 1, 1, 1, 1, 1])))
    dn, sn = d6(n)
    dt, stt = d6(total)
    MB.check(dev.L.mag_cuda_binary_f32(dev.p, MB.OP["ADD"], rs.data_ptr, xs.data_ptr, ys.data_ptr, dn, sn, sn, dn,
                                       sn), "sharded add")
    MB.check(dev.L.mag_cuda_binary_f32(dev.p, MB.OP["ADD"], rf.data_ptr, x.data_ptr, y.data_ptr, dt, stt, stt, dt,
                                       stt), "whole add")
    res = dev.tensor((2,))
    dp.reduce_full(dev, "SUM", xs, res.data_ptr, world)
    MB.check(dev.L.mag_cuda_reduce_f32(dev.p, MB.OP["SUM"], res.data_ptr + 4, x.data_ptr, dt, stt), "whole sum")
    with torch.cuda.stream(stream):
        gathered = dp.gather_rows(view(rs, n), total, 1, world, rank)
        same = torch.equal(gathered.view(torch.int32), view(rf, total).view(torch.int32))
        flag = torch.tensor([1 if same else 0], dtype=torch.int32, device=dvc)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dev.sync()
    torch.cuda.synchronize()
    s_sharded, s_one = (float(v) for v in res.read())
    for t in (x, y, rf, xs, ys, rs, res):
        t.free()
    return {"elements": total, "ranks": world, "add_gathered_bitwise_equal_one_gpu": bool(flag.item()),
            "sum_sharded": s_sharded, "sum_one_gpu": s_one,
            "sum_rel_diff": abs(s_sharded - s_one) / max(abs(s_one), 1e-30),
            "note": "every rank's range added and all-gathered over NCCL; range records combined in rank order"}


def run_ours(args):
    import torch
    import torch.distributed as dist
    import mag_b200 as MB

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    os.environ["MAG_CUDA_DEVICE"] = str(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    import dp
    _, rows = dp.shard_rows(GLOBAL_BATCH, world, rank)
    dev = MB.Device()
    stream = torch.cuda.ExternalStream(dev.stream, device=torch.device("cuda", local))

    # ---- model: magnetron tensors, deferred graph (MATMUL -> ADD -> GELU per layer)
    g = torch.Generator().manual_seed(1234)
    std = (2.0 / D_IN) ** 0.5
    X = dev.tensor((rows, D_IN))
    Ws, Bs = [], []
    for _ in range(N_HID):
        W = dev.tensor((D_IN, D_HID))
        W.write((torch.randn(D_IN * D_HID, generator=g) * std).numpy())
        Ws.append(W)
        Bs.append(dev.tensor((rows, D_HID)))  # zero bias, full shape: the core tiles y by modulo (F5)
    Wo = dev.tensor((D_HID, D_OUT))
    Wo.write((torch.randn(D_HID * D_OUT, generator=g) * std).numpy())
    Bo = dev.tensor((rows, D_OUT))
    def forward(x_in):
        dev.eager = False
        h = x_in
        for W, B in zip(Ws, Bs):
            h = dev.op("MATMUL", h, W)
            h = dev.op("ADD", h, B)
            h = dev.op("GELU", h, inplace=True)
        out = dev.op("MATMUL", h, Wo)
        out = dev.op("ADD", out, Bo)
        dev.eager = True
        return out
    z = forward(X)
    P = dev.tensor((rows * D_OUT,))
    gathered = {}

    # ---- inputs in pinned host memory
    xh = torch.randn(rows * D_IN, generator=torch.Generator().manual_seed(99 + rank)).pin_memory()
    X.write(xh.numpy())
    dev.sync()

    # ---- two input buffers and two forward graphs (z, P) / (z2, P2), used alternately: step i's
    # logits all-gather (N > 1) runs on its own stream and overlaps step i+1's kernels, and in the
    # end-to-end run step i+1's input upload and step i's output download overlap step i
    X2 = dev.tensor((rows, D_IN))
    X2.write(xh.numpy())
    z2 = forward(X2)
    P2 = dev.tensor((rows * D_OUT,))
    bufs = [(X, z, P), (X2, z2, P2)]
    gstream = torch.cuda.Stream(device=f"cuda:{local}")
    gdone = [None, None]  # per buffer: the event after its last all-gather

    def step(i):
        _, zc, pc = bufs[i % 2]
        if gdone[i % 2] is not None:
            stream.wait_event(gdone[i % 2])  # that buffer's previous gather has read it
        dev.graph_exec(zc, fused=True)
        MB.check(dev.L.mag_cuda_softmax_rows_f32(dev.p, pc.data_ptr, zc.data_ptr, rows, D_OUT), "softmax")
        if world > 1:
            ready = torch.cuda.Event()
            ready.record(stream)
            gstream.wait_event(ready)
            with torch.cuda.stream(gstream):
                src = torch.as_tensor(_CudaArray(pc.data_ptr, rows * D_OUT, dev.stream), device=f"cuda:{local}")
                gathered[i % 2] = dp.gather_rows(src, GLOBAL_BATCH, D_OUT, world, rank)
                ev = torch.cuda.Event()
                ev.record(gstream)
                gdone[i % 2] = ev

    def join():  # the backend's stream waits for every gather issued so far
        stream.wait_stream(gstream)

    # every rank copies its own rows of the probabilities to the host (in parallel over the
    # ranks' PCIe links); the all-gather still gives every GPU the whole result
    out_h = [torch.empty(rows * D_OUT, dtype=torch.float32).pin_memory() for _ in range(2)]

    def e2e_run(steps):
        dev.upload_async(bufs[0][0], xh.data_ptr(), xh.numel() * 4)
        for i in range(steps):
            if i + 1 < steps:
                dev.upload_async(bufs[(i + 1) % 2][0], xh.data_ptr(), xh.numel() * 4)
            step(i)
            dev.download_async(bufs[i % 2][2], out_h[i % 2].data_ptr(), rows * D_OUT * 4)
        join()
        dev.copies_sync()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()
        dev.sync()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    launches0 = dev.launches()
    dev.profile_start()  # graph captured on the first step carries per-op event nodes
    for i in range(args.warmup):
        step(i)
    join()
    barrier()
    dev.profile_collect()
    dev.profile_start()  # reset the per-op totals; timing below only
    clocks = ClockSampler(local)
    barrier()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    launches_before = dev.launches()
    clocks.start()
    ev0.record(stream)
    for i in range(args.steps):
        step(i)  # a replay's op events are read when its graph is next replayed (no stream sync)
    join()
    ev1.record(stream)
    barrier()
    clk = clocks.stop()
    dev.profile_collect()  # the last replays' op events
    launches_timed = dev.launches() - launches_before
    ms = ev0.elapsed_time(ev1)
    ms = max_over_ranks(ms)
    n_mm, us_mm = dev.profile_stats("MATMUL")

    # ---- end to end (pinned host buffers through the backend's asynchronous copies)
    e2e_run(2)
    barrier()
    t0 = time.perf_counter()
    ev0.record(stream)
    e2e_run(args.steps)
    ev1.record(stream)
    barrier()
    e2e_ms = max_over_ranks(max(ev0.elapsed_time(ev1), (time.perf_counter() - t0) * 1e3))
    dev.profile_stop(os.devnull)

    value = GLOBAL_BATCH * args.steps / (ms / 1e3)
    e2e_value = GLOBAL_BATCH * args.steps / (e2e_ms / 1e3)
    pk, pk_src = peaks()
    split_peak, split_note = split_roofline(pk, pk_src)
    mm_flop_per_step = 2.0 * rows * (N_HID * D_IN * D_HID + D_HID * D_OUT)
    mm_ms_per_step = (us_mm / 1e3) / args.steps if args.steps else 0.0
    achieved = (mm_flop_per_step / (mm_ms_per_step / 1e3)) / 1e12 if mm_ms_per_step else 0.0
    line = {
        "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) input, Kaiming-normal weights, zero biases)",
        "config": bench_config(world),
        "e2e": {"value": e2e_value, "unit": "samples/s",
                "h2d_bytes_per_step": rows * D_IN * 4 * world,
                "d2h_bytes_per_step": world * rows * D_OUT * 4},
        "gpu_launches": launches_timed,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": split_peak, "unit": "TFLOP/s",
                     "frac": achieved / split_peak if split_peak else None,
                     "traffic": (0.686e9 + 0.119e9) * rows / 8192,
                     "traffic_note": "DRAM bytes per hidden-layer GEMM launch: ncu capture of the fused "
                                     "layer at 8192 rows, scaled by rows",
                     "kernel": "MATMUL op (per-op CUDA events inside the replayed graph)",
                     "peak_note": split_note,
                     "matmul_ms_per_step": mm_ms_per_step, "matmul_launches": n_mm},
        "clocks": clk,
        "device": dev.name,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline()
    if rank == 0 and world == 1 and not args.no_sweep:
        line["sweep"] = sweep(dev, MB, torch, local)
    if world > 1:
        line["sharded_check"] = sharded_check(dev, MB, torch, world, rank, local, stream)
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def sweep(dev, MB, torch, local):
    """Short device-timed throughput of the other benchmarked op families (HBM GB/s, TFLOP/s)."""
    out = {}
    stream = torch.cuda.ExternalStream(dev.stream, device=torch.device("cuda", local))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timeit(fn, reps=5):
        fn()
        dev.sync()
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        dev.sync()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    n = 1 << 28
    x, y, r = dev.tensor((n,)), dev.tensor((n,)), dev.tensor((n,))
    xv = torch.randn(n // 4, generator=torch.Generator().manual_seed(5)).numpy()
    for t in (x, y):
        for k in range(4):
            t.write(xv, offset_elems=k * (n // 4))
    dims, st = MB.i64x6([n, 1, 1, 1, 1, 1]), MB.i64x6(MB.strides6([n, 1, 1, 1, 1, 1]))
    ms = timeit(lambda: dev.L.mag_cuda_binary_f32(dev.p, MB.OP["ADD"], r.data_ptr, x.data_ptr, y.data_ptr, dims, st, st, dims, st))
    out["add_2^28_GBps"] = 12.0 * n / (ms / 1e3) / 1e9
    ms = timeit(lambda: dev.L.mag_cuda_unary_f32(dev.p, MB.OP["SIGMOID"], r.data_ptr, x.data_ptr, n // 1024, 1024, 1024, 1024, 0.0))
    out["sigmoid_2^28_GBps"] = 8.0 * n / (ms / 1e3) / 1e9
    ms = timeit(lambda: dev.L.mag_cuda_reduce_f32(dev.p, MB.OP["SUM"], r.data_ptr, x.data_ptr, dims, st))
    out["sum_2^28_GBps"] = 4.0 * n / (ms / 1e3) / 1e9
    ms = timeit(lambda: dev.L.mag_cuda_softmax_rows_f32(dev.p, r.data_ptr, x.data_ptr, 4096, 32768))
    out["softmax_rows_4096x32768_GBps"] = 8.0 * 4096 * 32768 / (ms / 1e3) / 1e9
    m = 4096
    ms = timeit(lambda: dev.L.mag_cuda_matmul_f32(dev.p, r.data_ptr, x.data_ptr, y.data_ptr, m, m, m), reps=2)
    out["matmul_4096^3_TFLOPs"] = 2.0 * m ** 3 / (ms / 1e3) / 1e12
    for t in (x, y, r):
        t.free()
    return out


def run_storage(args):
    """.magnetron save/load of one f32 tensor of --size elements between HBM and a file
    (page-cache resident: the load follows the save), beside pinned-memory DMA peaks and
    the reference's own CPU save/load of the same tensor on this host."""
    import tempfile
    import torch
    import mag_b200 as MB
    dev = MB.Device()
    n = args.size or (1 << 28)
    nbytes = 4 * n
    tmp = tempfile.mkdtemp(prefix="magsto")
    path = os.path.join(tmp, "t.magnetron")
    x = dev.tensor((n,))
    g = MB.Pcg(7)
    dev.fill_random_uniform(x, -1.0, 1.0, g)
    dev.sync()
    reps = max(1, args.steps)

    def rate(fn):
        fn()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return nbytes / statistics.median(ts) / 1e9

    out = {"case": "storage", "size": n, "bytes": nbytes, "unit": "GB/s", "file_dir": tmp}
    out["save"] = rate(lambda: dev.save(path, [x]))
    y = dev.tensor((n,))
    arr = (ctypes.c_void_p * 1)(y.ptr)
    out["load"] = rate(lambda: MB.check(dev.L.mag_cuda_tensor_load(dev.p, path.encode(), arr, 1), "load"))
    assert np.array_equal(y.read(1 << 20), x.read(1 << 20))
    host = torch.empty(n, dtype=torch.float32).pin_memory()
    gpu = torch.empty(n, dtype=torch.float32, device="cuda")
    out["pinned_h2d"] = rate(lambda: (gpu.copy_(host, non_blocking=True), torch.cuda.synchronize()))
    out["pinned_d2h"] = rate(lambda: (host.copy_(gpu, non_blocking=True), torch.cuda.synchronize()))
    del host, gpu
    if not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        from oracle import RefLib, REF_SO
        if os.path.exists(REF_SO):
            R = RefLib()
            R.L.mag_tensor_save.argtypes = [ctypes.c_void_p, ctypes.c_char_p]
            R.L.mag_tensor_load.argtypes = [ctypes.c_void_p, ctypes.c_char_p]
            R.L.mag_tensor_load.restype = ctypes.c_void_p
            t = R.tensor_nd((n,))
            rpath = os.path.join(tmp, "ref.magnetron").encode()
            out["reference_cpu_save"] = rate(lambda: R.L.mag_tensor_save(t, rpath))

            def ref_load():
                R.free(R.L.mag_tensor_load(R.ctx, rpath))
            out["reference_cpu_load"] = rate(ref_load)
            R.free(t)
            R.close()
    for k in list(out):
        if isinstance(out[k], float):
            out[k] = round(out[k], 2)
    for f in os.listdir(tmp):
        os.remove(os.path.join(tmp, f))
    os.rmdir(tmp)
    print(json.dumps(out), flush=True)


def run_image(args):
    """Image pixel work on a 3840 x 2160 RGB frame: decoded u8 pixels (host memory) to a planar
    f32 tensor, with and without a resize to 1920 x 1080, and back to u8 (host memory), beside
    the reference's own CPU code on the same pixels (through its image callbacks)."""
    import mag_b200 as MB
    dev = MB.Device()
    w, h, c = 3840, 2160, 3
    src = np.random.default_rng(5).integers(0, 256, w * h * c, dtype=np.uint8)
    reps = max(1, args.steps)
    out = {"case": "image", "frame": [w, h, c], "unit": "Mpixel/s"}

    def rate(fn, pixels):
        fn()
        dev.sync()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            dev.sync()
            ts.append(time.perf_counter() - t0)
        return round(pixels / statistics.median(ts) / 1e6, 1)

    full, half = dev.tensor((c, h, w)), dev.tensor((c, h // 2, w // 2))
    u8 = np.empty(w * h * c, np.uint8)
    out["load"] = rate(lambda: dev.L.mag_cuda_img_from_u8(dev.p, full.ptr, src.ctypes.data, w, h, c, 0, 0), w * h)
    out["load_resize_1080p"] = rate(lambda: dev.L.mag_cuda_img_from_u8(dev.p, half.ptr, src.ctypes.data, w, h, c,
                                                                       w // 2, h // 2), w * h)
    out["save"] = rate(lambda: dev.L.mag_cuda_img_to_u8(dev.p, full.ptr, u8.ctypes.data), w * h)
    if not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        from oracle import REF_SO
        if os.path.exists(REF_SO):
            import gen_images as GI
            L = ctypes.CDLL(REF_SO)
            vp = ctypes.c_void_p
            L.mag_ctx_create.argtypes = [ctypes.POINTER(GI.CtxInfo)]
            L.mag_ctx_create.restype = vp
            L.mag_tensor_load_image.argtypes = [vp, ctypes.c_char_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_uint32]
            L.mag_tensor_load_image.restype = vp
            L.mag_tensor_save_image.argtypes = [vp, ctypes.c_char_p]
            L.mag_tensor_decref.argtypes = [vp]
            L.mag_ctx_destroy.argtypes = [vp]

            @GI.LOAD_FN
            def load(path, whc, channels):
                whc.contents[0], whc.contents[1], whc.contents[2] = w, h, c
                return src.ctypes.data

            @GI.FREE_FN
            def free(p):
                pass

            @GI.SAVE_FN
            def save(path, data, whc):
                return True

            info = GI.CtxInfo()
            info.image_load_fn, info.image_load_free_fn, info.image_save_fn = load, free, save
            ctx = L.mag_ctx_create(ctypes.byref(info))

            def ref(rw, rh):
                t = L.mag_tensor_load_image(ctx, b"frame", 0, rw, rh)
                L.mag_tensor_decref(t)
            out["reference_cpu_load"] = rate(lambda: ref(0, 0), w * h)
            out["reference_cpu_load_resize_1080p"] = rate(lambda: ref(w // 2, h // 2), w * h)
            t = L.mag_tensor_load_image(ctx, b"frame", 0, 0, 0)
            out["reference_cpu_save"] = rate(lambda: L.mag_tensor_save_image(t, b"frame.png"), w * h)
            L.mag_tensor_decref(t)
            L.mag_ctx_destroy(ctx)
    print(json.dumps(out), flush=True)


def build_mlp2(dev, torch, batch=256, d_in=784, d_hid=256, d_out=10, seed=12):
    """The two-layer MLP forward of the reference's MNIST-shaped example: X (batch x 784) U(0,1),
    Glorot-uniform W1 (784 x 256) and W2 (256 x 10), a zero 1-D bias of 256 (tiling broadcast)
    and a zero full-shape (batch x 10) bias, MATMUL -> ADD -> SIGMOID -> MATMUL -> ADD as one
    recorded graph run by the fused executor (each bias and the SIGMOID in its product's
    epilogue), then the normalised row softmax over the 10 logits.  Returns the forward (graph
    replay + softmax, on the device's stream), the probability tensor and every tensor to free."""
    import mag_b200 as MB
    g = torch.Generator().manual_seed(seed)
    lim1, lim2 = (6.0 / (d_in + d_hid)) ** 0.5, (6.0 / (d_hid + d_out)) ** 0.5
    X, W1, W2 = dev.tensor((batch, d_in)), dev.tensor((d_in, d_hid)), dev.tensor((d_hid, d_out))
    B1, B2, P = dev.tensor((d_hid,)), dev.tensor((batch, d_out)), dev.tensor((batch * d_out,))
    X.write(torch.rand(batch * d_in, generator=g).numpy())
    W1.write(((torch.rand(d_in * d_hid, generator=g) * 2 - 1) * lim1).numpy())
    W2.write(((torch.rand(d_hid * d_out, generator=g) * 2 - 1) * lim2).numpy())
    dev.eager = False
    try:
        h = dev.op("SIGMOID", dev.op("ADD", dev.op("MATMUL", X, W1), B1), inplace=True)
        z = dev.op("ADD", dev.op("MATMUL", h, W2), B2)
    finally:
        dev.eager = True

    def fwd():
        rc = dev.L.mag_cuda_graph_exec_fused(dev.p, z.ptr)
        return rc or dev.L.mag_cuda_softmax_rows_f32(dev.p, P.data_ptr, z.data_ptr, batch, d_out)
    return fwd, P, [X, W1, W2, B1, B2, P]


def run_case(args):
    """One kernel family, a few launches, for profilers: `--case gemm|add|sigmoid|sum|softmax`."""
    import torch
    import mag_b200 as MB
    dev = MB.Device()
    n = args.size
    if args.case == "mlp2":
        # the two-layer MLP forward, batch --size (default 256): graph replay + row softmax
        rows = n
        fn, _, _ = build_mlp2(dev, torch, batch=rows)
        work, unit = float(rows), "samples/s"
    elif args.case == "layer":
        # two dense layers of the MLP (rows = --size, 4096 features), fused graph:
        # layer 1 = GEMM + bias + GELU + operand split, layer 2 reads the split
        rows = n
        g = torch.Generator().manual_seed(3)
        X = dev.tensor((rows, D_IN))
        W1, W2 = dev.tensor((D_IN, D_HID)), dev.tensor((D_HID, D_HID))
        B1, B2 = dev.tensor((rows, D_HID)), dev.tensor((rows, D_HID))
        X.write(torch.randn(rows * D_IN, generator=g).numpy())
        for W in (W1, W2):
            W.write((torch.randn(D_IN * D_HID, generator=g) * (2.0 / D_IN) ** 0.5).numpy())
        dev.eager = False
        h = dev.op("GELU", dev.op("ADD", dev.op("MATMUL", X, W1), B1), inplace=True)
        z = dev.op("ADD", dev.op("MATMUL", h, W2), B2)
        dev.eager = True
        fn = lambda: dev.L.mag_cuda_graph_exec_fused(dev.p, z.ptr)
        work, unit = 2 * 2.0 * rows * D_IN * D_HID / 1e12, "TFLOP/s"
    elif args.case == "gemm":
        MB.check(dev.L.mag_cuda_set_matmul_mode(dev.p, 2), "tc")
        x, y, r = dev.tensor((n * n,)), dev.tensor((n * n,)), dev.tensor((n * n,))
        v = torch.randn(n * n, generator=torch.Generator().manual_seed(3)).numpy()
        x.write(v)
        y.write(v)
        fn = lambda: dev.L.mag_cuda_matmul_f32(dev.p, r.data_ptr, x.data_ptr, y.data_ptr, n, n, n)
        work, unit = 2.0 * n ** 3 / 1e12, "TFLOP/s"
    else:
        x, y, r = dev.tensor((n,)), dev.tensor((n,)), dev.tensor((n,))
        v = torch.randn(n, generator=torch.Generator().manual_seed(3)).numpy()
        x.write(v)
        y.write(v)
        dims, st = MB.i64x6([n, 1, 1, 1, 1, 1]), MB.i64x6(MB.strides6([n, 1, 1, 1, 1, 1]))
        if args.case in ("tile", "bcast2", "bcast2s"):
            if args.case == "tile":   # x rm [8,16,32,64,8,256] (+) y rm [1,16,1,64,1,256]
                xs, ys = (256, 8, 64, 32, 16, 8), (256, 1, 64, 1, 16, 1)
                rs = xs
            elif args.case == "bcast2":  # [8,16,1,64,1,256] (+) [1,16,32,1,128,256] -> 2^33 outputs
                xs, ys, rs = (256, 1, 64, 1, 16, 8), (256, 128, 1, 32, 16, 1), (256, 128, 64, 32, 16, 8)
            else:                     # profiling size: [1,16,1,4,1,256] (+) [1,16,32,1,128,256] -> 2^28
                xs, ys, rs = (256, 1, 4, 1, 16, 1), (256, 128, 1, 32, 16, 1), (256, 128, 4, 32, 16, 1)
            for t in (x, y, r):
                t.free()
            nx, ny, nr = int(np.prod(xs)), int(np.prod(ys)), int(np.prod(rs))
            x, y, r = dev.tensor((nx,)), dev.tensor((ny,)), dev.tensor((nr,))
            x.write(np.resize(v, nx))
            y.write(np.resize(v, ny))
            if args.case == "tile":
                dx, sx = MB.i64x6(xs), MB.i64x6(MB.strides6(xs))
                dy, sy = MB.i64x6(ys), MB.i64x6(MB.strides6(ys))
                fn = lambda: dev.L.mag_cuda_binary_f32(dev.p, MB.OP["ADD"], r.data_ptr, x.data_ptr, y.data_ptr, dx, sx, sx, dy, sy)
            else:
                fn = lambda: dev.L.mag_cuda_broadcast2_f32(dev.p, MB.OP["ADD"], r.data_ptr, x.data_ptr, y.data_ptr,
                                                           MB.i64x6(rs), MB.i64x6(xs), MB.i64x6(ys))
            work = 4.0 * (nx + ny + nr) / 1e9
        elif args.case == "add":
            fn = lambda: dev.L.mag_cuda_binary_f32(dev.p, MB.OP["ADD"], r.data_ptr, x.data_ptr, y.data_ptr, dims, st, st, dims, st)
            work = 12.0 * n / 1e9
        elif args.case == "sigmoid":
            fn = lambda: dev.L.mag_cuda_unary_f32(dev.p, MB.OP["SIGMOID"], r.data_ptr, x.data_ptr, n // 1024, 1024, 1024, 1024, 0.0)
            work = 8.0 * n / 1e9
        elif args.case == "sum":
            fn = lambda: dev.L.mag_cuda_reduce_f32(dev.p, MB.OP["SUM"], r.data_ptr, x.data_ptr, dims, st)
            work = 4.0 * n / 1e9
        elif args.case == "softmax256k":
            fn = lambda: dev.L.mag_cuda_softmax_rows_f32(dev.p, r.data_ptr, x.data_ptr, n // 262144, 262144)
            work = 8.0 * n / 1e9
        elif args.case == "softmax1k":
            fn = lambda: dev.L.mag_cuda_softmax_rows_f32(dev.p, r.data_ptr, x.data_ptr, n // 1024, 1024)
            work = 8.0 * n / 1e9
        elif args.case == "fill_const":
            fn = lambda: dev.L.mag_cuda_fill_f32(dev.p, r.data_ptr, n, 1.5)
            work = 4.0 * n / 1e9
        elif args.case in ("fill_uniform", "fill_normal"):
            g = MB.Pcg(0x5EED0002)
            fill = getattr(dev.L, f"mag_cuda_{args.case}_pcg_f32")
            fn = lambda: fill(dev.p, r.data_ptr, n, 0.0, 1.0, ctypes.byref(g.state), g.inc)
            work = 4.0 * n / 1e9
        elif args.case in ("fill_mt_uniform", "fill_mt_normal"):
            g = MB.Mt19937(0x5EED0002)
            fill = getattr(dev.L, f"mag_cuda_fill_{args.case[8:]}_mt19937_f32")
            fn = lambda: fill(dev.p, r.data_ptr, n, 0.0, 1.0, ctypes.byref(g.st))
            work = 4.0 * n / 1e9
        elif args.case == "batched":  # 64 products of 512 x 512 x 512
            fn = lambda: dev.L.mag_cuda_matmul_batched_f32(dev.p, r.data_ptr, x.data_ptr, y.data_ptr, 64, 512, 512, 512)
            work = 2.0 * 64 * 512 ** 3 / 1e12
        elif args.case in ("skinny", "skinny8"):  # M = 1 or 8, K = N = 4096
            mr = 1 if args.case == "skinny" else 8
            fn = lambda: dev.L.mag_cuda_matmul_f32(dev.p, r.data_ptr, x.data_ptr, y.data_ptr, mr, 4096, 4096)
            work = 4.0 * (mr * 4096 + 4096 * 4096 + mr * 4096) / 1e9
        elif args.case == "rowsum":  # SUM along rows of 32768
            fn = lambda: dev.L.mag_cuda_reduce_rows_f32(dev.p, MB.OP["SUM"], r.data_ptr, x.data_ptr, n // 32768, 32768)
            work = 4.0 * n / 1e9
        else:
            fn = lambda: dev.L.mag_cuda_softmax_rows_f32(dev.p, r.data_ptr, x.data_ptr, n // 32768, 32768)
            work = 8.0 * n / 1e9
        unit = "TFLOP/s" if args.case == "batched" else "GB/s"
    stream = torch.cuda.ExternalStream(dev.stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    MB.check(fn(), args.case)
    dev.sync()
    e0.record(stream)
    for _ in range(args.steps):
        MB.check(fn(), args.case)
    e1.record(stream)
    dev.sync()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    print(json.dumps({"case": args.case, "size": n, "ms": ms, "rate": work / (ms / 1e3), "unit": unit}))


def run_sharded(args):
    """Element ranges sharded over the ranks (`--case sharded`, launched like the main bench):
    ADD on each rank's contiguous range of the 2^28-element sweep vectors (kernel-aggregate
    GB/s, and with the all-gather that collects r on every rank), and the full SUM with
    one 24-byte record per rank all-gathered and combined in rank order.  Device time with
    CUDA events on the backend's stream, max over ranks."""
    import datetime
    import torch
    import torch.distributed as dist
    import mag_b200 as MB
    import dp

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    os.environ["MAG_CUDA_DEVICE"] = str(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    total = args.size or (1 << 28)
    start, n = dp.shard_rows(total, world, rank)
    dev = MB.Device()
    stream = torch.cuda.ExternalStream(dev.stream, device=torch.device("cuda", local))
    x, y, r = dev.tensor((n,)), dev.tensor((n,)), dev.tensor((n,))
    dev.fill_random_normal(x, 0.0, 1.0, MB.Pcg(0x5EED0002 + 2 * rank))
    dev.fill_random_normal(y, 0.0, 1.0, MB.Pcg(0x5EED0003 + 2 * rank))
    res = dev.tensor((1,))
    dims, st = MB.i64x6([n, 1, 1, 1, 1, 1]), MB.i64x6(MB.strides6([n, 1, 1, 1, 1, 1]))
    local_r = torch.as_tensor(_CudaArray(r.data_ptr, n, dev.stream), device=f"cuda:{local}")

    def add():
        MB.check(dev.L.mag_cuda_binary_f32(dev.p, MB.OP["ADD"], r.data_ptr, x.data_ptr, y.data_ptr, dims, st, st,
                                           dims, st), "add")

    def add_gather():
        add()
        if world > 1:
            with torch.cuda.stream(stream):
                dp.gather_rows(local_r, total, 1, world, rank)

    def full_sum():
        if world > 1:
            dp.reduce_full(dev, "SUM", x, res.data_ptr, world)
        else:
            MB.check(dev.L.mag_cuda_reduce_f32(dev.p, MB.OP["SUM"], res.data_ptr, x.data_ptr, dims, st), "sum")

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()
        dev.sync()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            fn()
        e1.record(stream)
        dev.sync()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64, device=f"cuda:{local}")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    ms_add, ms_gather, ms_sum = timed(add), timed(add_gather), timed(full_sum)
    sum_value = float(res.read()[0])
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps({
            "case": "sharded", "n_gpus": world, "elements": total, "steps": args.steps, "warmup": args.warmup,
            "add_ms": ms_add, "add_GBps": 12.0 * total / (ms_add / 1e3) / 1e9,
            "add_with_gather_ms": ms_gather, "add_with_gather_GBps": 12.0 * total / (ms_gather / 1e3) / 1e9,
            "sum_ms": ms_sum, "sum_GBps": 4.0 * total / (ms_sum / 1e3) / 1e9, "sum": sum_value,
            "note": "ADD 12 B/element, SUM 4 B/element over all ranks; the gather moves (N-1)/N of r to every rank"}),
            flush=True)


def run_sweep_full(args):
    """Every other benchmarked configuration on one GPU: elementwise/broadcast/unary (config 2),
    row reductions and softmax (config 3), the matmul sweep (config 4), each with its roofline
    fraction, and single-thread reference CPU rates for the sizes the CPU finishes quickly."""
    import torch
    import mag_b200 as MB
    dev = MB.Device()
    pk, pk_src = peaks()
    hbm = pk["hbm_gbs"]
    tf, _ = split_roofline(pk, pk_src)
    stream = torch.cuda.ExternalStream(dev.stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    rows_out = []
    gen = torch.Generator().manual_seed(11)
    chunk = torch.randn(1 << 24, generator=gen).pin_memory()

    def filled(n, fn=None):
        t = dev.tensor((n,))
        src = chunk if fn is None else fn(chunk)
        src = src.contiguous().pin_memory() if fn is not None else src
        step = src.numel()
        for off in range(0, n, step):
            m = min(step, n - off)
            t.write(src[:m].numpy(), offset_elems=off)
        return t

    # 5 ms between samples: a faster in-process sampler competes with the launching thread and
    # stretches the short rows
    clocks = ClockSampler(torch.cuda.current_device(), interval=0.005)
    clocks.start()
    window = [0.0, 0.0]

    def timeit(fn, reps):
        MB.check(fn(), "warm")
        dev.sync()
        window[0] = time.perf_counter()
        e0.record(stream)
        for _ in range(reps):
            MB.check(fn(), "op")
        e1.record(stream)
        dev.sync()
        torch.cuda.synchronize()
        window[1] = time.perf_counter()
        return e0.elapsed_time(e1) / reps

    def rec(group, name, ms, work, unit, peak):
        rate = work / (ms / 1e3)
        mhz = clocks.around(window[0], window[1])
        rows_out.append({"group": group, "case": name, "ms": round(ms, 4), "rate": round(rate, 1), "unit": unit,
                         "frac": round(rate / peak, 3) if peak else None, "sm_mhz": mhz})
        print(json.dumps(rows_out[-1]), flush=True)

    def dims_strides(shape):
        d = MB.pad6(shape)
        return MB.i64x6(d), MB.i64x6(MB.strides6(d))

    # ---- config 2: binary, same shape
    for lg in (20, 24, 28):
        n = 1 << lg
        x, y, r = filled(n), filled(n, lambda c: c.abs() + 0.5), dev.tensor((n,))
        d, s_ = dims_strides((n,))
        for op in ("ADD", "SUB", "MUL", "DIV"):
            ms = timeit(lambda: dev.L.mag_cuda_binary_f32(dev.p, MB.OP[op], r.data_ptr, x.data_ptr, y.data_ptr,
                                                          d, s_, s_, d, s_), 20 if lg < 28 else 5)
            rec("elementwise", f"{op} 2^{lg}", ms, 12.0 * n / 1e9, "GB/s", hbm)
        for t in (x, y, r):
            t.free()
    # ---- config 2: tiling broadcast (reference-legal) and two-sided broadcast (extension)
    xs, ys = (256, 8, 64, 32, 16, 8), (256, 1, 64, 1, 16, 1)
    nx, ny = int(np.prod(xs)), int(np.prod(ys))
    x, y, r = filled(nx), filled(ny), dev.tensor((nx,))
    dx, sx = dims_strides(xs)
    dy, sy = dims_strides(ys)
    ms = timeit(lambda: dev.L.mag_cuda_binary_f32(dev.p, MB.OP["ADD"], r.data_ptr, x.data_ptr, y.data_ptr,
                                                  dx, sx, sx, dy, sy), 5)
    rec("elementwise", "ADD tiling [8,16,32,64,8,256]+[1,16,1,64,1,256]", ms, 4.0 * (2 * nx + ny) / 1e9, "GB/s", hbm)
    for t in (x, y, r):
        t.free()
    xs, ys, rs = (256, 1, 64, 1, 16, 8), (256, 128, 1, 32, 16, 1), (256, 128, 64, 32, 16, 8)
    nx, ny, nr = int(np.prod(xs)), int(np.prod(ys)), int(np.prod(rs))
    x, y, r = filled(nx), filled(ny), dev.tensor((nr,))
    ms = timeit(lambda: dev.L.mag_cuda_broadcast2_f32(dev.p, MB.OP["ADD"], r.data_ptr, x.data_ptr, y.data_ptr,
                                                      MB.i64x6(rs), MB.i64x6(xs), MB.i64x6(ys)), 3)
    rec("elementwise", "ADD two-sided [8,16,1,64,1,256]+[1,16,32,1,128,256] (2^33 out)", ms,
        4.0 * (nx + ny + nr) / 1e9, "GB/s", hbm)
    for t in (x, y, r):
        t.free()
    # ---- config 2: unary at 2^28
    n = 1 << 28
    x, xa, xl, r = filled(n), filled(n, lambda c: c.abs()), filled(n, lambda c: c.abs() + 1.0), dev.tensor((n,))
    for op in ("ABS", "NEG", "LOG", "SQR", "SQRT", "SOFTMAX", "SIGMOID", "TANH", "RELU", "GELU"):
        src = xl if op == "LOG" else (xa if op == "SQRT" else x)
        ms = timeit(lambda: dev.L.mag_cuda_unary_f32(dev.p, MB.OP[op], r.data_ptr, src.data_ptr, n // 4096, 4096,
                                                     4096, 4096, 0.0), 5)
        rec("unary", f"{op} 2^28", ms, 8.0 * n / 1e9, "GB/s", hbm)
    for t in (xa, xl):
        t.free()
    # ---- config 3: row reductions, softmax, full reductions
    for rows, cols in ((65536, 1024), (4096, 32768), (1024, 262144)):
        out = dev.tensor((rows * cols,))
        for op in ("SUM", "MEAN", "MIN", "MAX"):
            ms = timeit(lambda: dev.L.mag_cuda_reduce_rows_f32(dev.p, MB.OP[op], out.data_ptr, x.data_ptr, rows, cols), 5)
            rec("reduce", f"row {op} ({rows},{cols})", ms, (4.0 * rows * cols + 4.0 * rows) / 1e9, "GB/s", hbm)
        ms = timeit(lambda: dev.L.mag_cuda_softmax_rows_f32(dev.p, out.data_ptr, x.data_ptr, rows, cols), 5)
        rec("reduce", f"row softmax ({rows},{cols})", ms, 8.0 * rows * cols / 1e9, "GB/s", hbm)
        out.free()
    d, s_ = dims_strides((n,))
    for op in ("SUM", "MIN", "MAX"):
        ms = timeit(lambda: dev.L.mag_cuda_reduce_f32(dev.p, MB.OP[op], r.data_ptr, x.data_ptr, d, s_), 5)
        rec("reduce", f"full {op} 2^28", ms, 4.0 * n / 1e9, "GB/s", hbm)
    for t in (x, r):
        t.free()
    # ---- seeded fills on the device (the PCG stream of a reference context, jumped per thread);
    # before the matmul rows, whose power draw lowers the clocks of the integer-bound fills
    n = 1 << 28
    r = dev.tensor((n,))
    g = MB.Pcg(0x5EED0002)
    ms = timeit(lambda: dev.L.mag_cuda_fill_uniform_pcg_f32(dev.p, r.data_ptr, n, -1.0, 1.0, ctypes.byref(g.state),
                                                           g.inc), 5)
    rec("fill", "uniform PCG 2^28", ms, 4.0 * n / 1e9, "GB/s", hbm)
    ms = timeit(lambda: dev.L.mag_cuda_fill_normal_pcg_f32(dev.p, r.data_ptr, n, 0.0, 1.0, ctypes.byref(g.state),
                                                          g.inc), 5)
    rec("fill", "normal PCG + Box-Muller 2^28", ms, 4.0 * n / 1e9, "GB/s", hbm)
    # the reference's default stream (Mersenne twister, jumped per substream); each fill reads
    # the last block back, so it waits for its kernels
    mt = MB.Mt19937(0x5EED0002)
    ms = timeit(lambda: dev.L.mag_cuda_fill_uniform_mt19937_f32(dev.p, r.data_ptr, n, -1.0, 1.0, ctypes.byref(mt.st)),
                5)
    rec("fill", "uniform MT19937 2^28", ms, 4.0 * n / 1e9, "GB/s", hbm)
    ms = timeit(lambda: dev.L.mag_cuda_fill_normal_mt19937_f32(dev.p, r.data_ptr, n, 0.0, 1.0, ctypes.byref(mt.st)),
                5)
    rec("fill", "normal MT19937 + Box-Muller 2^28", ms, 4.0 * n / 1e9, "GB/s", hbm)
    r.free()
    # ---- config 4: matmul (skinny and batched first, and config 1 before the square products:
    # the large products' power draw lowers the clock for a while after them)
    k = nn = 4096
    b = filled(k * nn, lambda c: c * (k ** -0.25))
    for m in (1, 8, 64):
        a = filled(m * k, lambda c: c * (k ** -0.25))
        c_ = dev.tensor((m * nn,))
        ms = timeit(lambda: dev.L.mag_cuda_matmul_f32(dev.p, c_.data_ptr, a.data_ptr, b.data_ptr, m, k, nn), 10)
        rec("matmul", f"skinny M={m} K=N=4096 (HBM: Y once)", ms, 4.0 * (m * k + k * nn + m * nn) / 1e9, "GB/s", hbm)
        a.free()
        c_.free()
    b.free()
    bt, mm = 64, 512
    a, c_ = filled(bt * mm * mm, lambda c: c * (mm ** -0.25)), dev.tensor((bt * mm * mm,))
    ms = timeit(lambda: dev.L.mag_cuda_matmul_batched_f32(dev.p, c_.data_ptr, a.data_ptr, a.data_ptr, bt, mm, mm, mm), 5)
    rec("matmul", f"batched 64 x [512x512 . 512x512] ({SPLIT_NAME} tcgen05, batch-indexed tiles)", ms,
        2.0 * bt * mm ** 3 / 1e12, "TFLOP/s", tf)
    a.free()
    c_.free()
    # ---- config 1: two-layer MLP forward, batch 256 (launch-bound: graph replay of the five
    # recorded ops, then the row softmax)
    fwd, _, keep = build_mlp2(dev, torch)
    ms = timeit(fwd, 200)
    rec("mlp", "two-layer MLP fwd, batch 256 (784-256-10, sigmoid, row softmax; graph replay)", ms, 256.0,
        "samples/s", None)
    for t in keep:
        t.free()
    for m in (1024, 4096, 8192, 16384):
        a = filled(m * m, lambda c: c * (m ** -0.25))
        c_ = dev.tensor((m * m,))
        ms = timeit(lambda: dev.L.mag_cuda_matmul_f32(dev.p, c_.data_ptr, a.data_ptr, a.data_ptr, m, m, m),
                    5 if m < 16384 else 2)
        rec("matmul", f"square {m}^3 ({SPLIT_NAME} tcgen05)", ms, 2.0 * m ** 3 / 1e12, "TFLOP/s", tf)
        a.free()
        c_.free()
    # ---- reference CPU, single thread, on this host
    cpu = []
    if not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        from oracle import RefLib, REF_SO
        if os.path.exists(REF_SO):
            R = RefLib()
            n = 1 << 24
            v = np.random.default_rng(1).standard_normal(n).astype(np.float32)
            tx, ty = R.tensor_nd((n,)), R.tensor_nd((n,))
            R.write(tx, v)
            R.write(ty, np.abs(v) + 0.5)

            def cpu_time(fn, reps=3):
                ts = []
                for _ in range(reps):
                    t0 = time.perf_counter()
                    out = fn()
                    ts.append(time.perf_counter() - t0)
                    R.free(out)
                return statistics.median(ts)
            for op in ("ADD", "DIV"):
                dt = cpu_time(lambda: R.op(op, tx, ty))
                cpu.append({"case": f"{op} 2^24", "rate": 12.0 * n / dt / 1e9, "unit": "GB/s"})
            for op in ("SIGMOID", "GELU"):
                dt = cpu_time(lambda: R.op(op, tx))
                cpu.append({"case": f"{op} 2^24", "rate": 8.0 * n / dt / 1e9, "unit": "GB/s"})
            dt = cpu_time(lambda: R.op("SUM", tx))
            cpu.append({"case": "full SUM 2^24", "rate": 4.0 * n / dt / 1e9, "unit": "GB/s"})
            for alg, seed_fn in (("PCG", R.seed), ("MT19937", R.seed_mt)):
                seed_fn(0x5EED0002)
                for kind in ("uniform", "normal"):
                    fill = getattr(R.L, f"mag_tensor_fill_random_{kind}")
                    t0 = time.perf_counter()
                    fill(tx, 0.0, 1.0)
                    cpu.append({"case": f"fill {kind} {alg} 2^24",
                                "rate": 4.0 * n / (time.perf_counter() - t0) / 1e9, "unit": "GB/s"})
            m = 1024
            ta, tb = R.tensor_nd((m, m)), R.tensor_nd((m, m))
            R.write(ta, v[:m * m])
            R.write(tb, v[:m * m])
            dt = cpu_time(lambda: R.op("MATMUL", ta, tb), reps=1)
            cpu.append({"case": "MATMUL 1024^3", "rate": 2.0 * m ** 3 / dt / 1e12, "unit": "TFLOP/s"})
            # the two-layer MLP forward through the reference's ops (SOFTMAX is its elementwise
            # exp; the 256 x 10 row normalisation is left out of this CPU figure)
            tx1, tw1, tw2 = R.tensor_nd((256, 784)), R.tensor_nd((784, 256)), R.tensor_nd((256, 10))
            tb1, tb2 = R.tensor_nd((256,)), R.tensor_nd((256, 10))
            R.write(tx1, np.abs(v[:256 * 784]))
            R.write(tw1, v[:784 * 256] * 0.07)
            R.write(tw2, v[:2560] * 0.15)
            R.write(tb1, np.zeros(256, np.float32))
            R.write(tb2, np.zeros(2560, np.float32))

            def mlp2_ref():
                a1 = R.op("MATMUL", tx1, tw1)
                a2 = R.op("ADD", a1, tb1)
                a3 = R.op("SIGMOID", a2)
                a4 = R.op("MATMUL", a3, tw2)
                a5 = R.op("ADD", a4, tb2)
                out = R.op("SOFTMAX", a5)
                for t in (a1, a2, a3, a4, a5):
                    R.free(t)
                return out
            dt = cpu_time(mlp2_ref, reps=5)
            cpu.append({"case": "two-layer MLP fwd, batch 256", "rate": 256.0 / dt, "unit": "samples/s"})
            R.close()
            for c in cpu:
                c["rate"] = round(c["rate"], 4)
                print(json.dumps({"cpu_reference_1thread": c}), flush=True)
    clk = clocks.stop()
    if args.out:
        with open(args.out, "w") as f:
            json.dump({"clocks": clk, "gpu": rows_out, "cpu_reference_1thread": cpu, "peaks": {"hbm_gbs": hbm, "split_tflops": tf, "split": SPLIT_NAME,
                                                                                 "source": pk_src},
                       "device": dev.name}, f, indent=1)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--case", default=None, choices=["gemm", "layer", "add", "sigmoid", "sum", "softmax", "softmax1k", "softmax256k", "skinny", "skinny8", "rowsum", "tile", "bcast2", "bcast2s", "batched",
                                                      "fill_uniform", "fill_normal", "fill_const", "fill_mt_uniform", "fill_mt_normal", "storage", "image", "sharded", "mlp2"],
                    help="run one kernel family for a profiler instead of the benchmark")
    ap.add_argument("--size", type=int, default=None)
    ap.add_argument("--sweep-full", action="store_true", help="measure every other benchmarked configuration")
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    if args.sweep_full:
        run_sweep_full(args)
        return
    if args.case:
        args.size = args.size or (8192 if args.case in ("gemm", "layer") else 256 if args.case == "mlp2" else 1 << 28)
        {"storage": run_storage, "image": run_image, "sharded": run_sharded}.get(args.case, run_case)(args)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
