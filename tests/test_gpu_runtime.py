"""CLONE, the per-op profiler and the bounded waits of the tensor-core GEMM, on the device.

CLONE is the reference's memcpy of the result's data size (magnetron/magnetron_cpu.c:1022-1032);
the profiler's table and CSV follow the core's layout (magnetron/magnetron.c:1085-1111); a
GEMM whose wait expires records MAG_CUDA_E_DEVICE_WAIT in the device's status word, which
mag_cuda_synchronize reports once, and the device stays usable.
"""
import os

import numpy as np
import pytest

import mag_b200 as MB
from harness import oracle, bits_equal
from gpu_util import device, run_op

pytestmark = pytest.mark.gpu


# ---------------------------------------------------------------- CLONE
def test_clone_copies_every_bit():
    """A clone equals its input bit for bit, NaN payloads, signed zeros and subnormals included,
    and a later write to the input leaves the clone unchanged."""
    dev = device()
    x = oracle().stream(9500).uniform(3 * 5 * 7, -4, 4)
    x[:6] = np.array([0.0, -0.0, np.inf, -np.inf, 1e-40, -3e-39], np.float32)
    x[6:8] = np.array([0x7FC00123, 0xFFC00042], np.uint32).view(np.float32)
    got, r, (tx,) = run_op(dev, "CLONE", [x], [(7, 5, 3)])
    assert np.array_equal(got.view(np.uint32), x.view(np.uint32))
    tx.write(np.zeros_like(x))
    assert np.array_equal(r.read().view(np.uint32), x.view(np.uint32))


def test_clone_into_part_of_a_larger_buffer_keeps_the_rest_zero():
    """A CLONE whose result covers the first 100 floats of a fresh 1000-float buffer (a view):
    those hold the input, and the other 900 keep the zeros that new storage holds by contract
    (magnetron/magnetron_cpu.c:2336-2349), although the buffer's clear was still pending."""
    dev = device()
    x = oracle().stream(9501).uniform(100, -1, 1)
    tx = dev.tensor((100,))
    tx.write(x)
    big = dev.tensor((1000,))
    r = MB.Tensor(dev, (100,), view_of=big)
    r.t.op = MB.OP["CLONE"]
    r.t.op_inputs[0] = tx.ptr
    r.inputs = [tx]
    dev.exec(r)
    out = big.read()
    assert bits_equal(out[:100], x).all()
    assert np.all(out[100:].view(np.uint32) == 0)


def test_clone_in_a_deferred_graph_replays_new_input():
    dev = device()
    s = oracle().stream(9502)
    x1, x2 = s.uniform(4096, -1, 1), s.uniform(4096, -1, 1)
    tx = dev.tensor((64, 64))
    dev.eager = False
    try:
        r = dev.op("SQR", dev.op("CLONE", tx))
    finally:
        dev.eager = True
    try:
        tx.write(x1)
        dev.graph_exec(r)
        a = r.read()
        tx.write(x2)
        dev.graph_exec(r)
        b = r.read()
    finally:
        dev.graph_release(r)
    assert bits_equal(a, x1 * x1).all() and bits_equal(b, x2 * x2).all()


# ---------------------------------------------------------------- profiler
def _csv_rows(path):
    with open(path) as f:
        lines = [ln.rstrip("\n") for ln in f]
    assert lines[0] == "Operation,Executions,Usage,AVG Time,Total Time"
    rows = []
    for ln in lines[1:]:
        name, n, usage, avg, tot = ln.split(",")
        rows.append((name, int(n), usage, float(avg), float(tot)))
    return rows


def test_profiler_counts_a_known_sequence_and_writes_the_core_csv(tmp_path):
    """Three ADDs, two SIGMOIDs and one MATMUL, eager: the per-op counts are exactly those, every
    op has device time, and the CSV has the core's header and columns (Usage = share of
    executions with one decimal, AVG = Total / Executions), rows by total time, longest first."""
    dev = device()
    s = oracle().stream(9600)
    a, b = dev.tensor((512, 512)), dev.tensor((512, 512))
    a.write(s.uniform(512 * 512, -1, 1))
    b.write(s.uniform(512 * 512, -1, 1))
    dev.profile_start()
    keep = []
    for _ in range(3):
        keep.append(dev.op("ADD", a, b))
    for _ in range(2):
        keep.append(dev.op("SIGMOID", a))
    keep.append(dev.op("MATMUL", a, b))
    dev.profile_collect()
    counts = {op: dev.profile_stats(op) for op in ("ADD", "SIGMOID", "MATMUL", "SUB")}
    assert [counts[op][0] for op in ("ADD", "SIGMOID", "MATMUL", "SUB")] == [3, 2, 1, 0]
    assert all(counts[op][1] > 0 for op in ("ADD", "SIGMOID", "MATMUL"))
    path = str(tmp_path / "prof.csv")
    dev.profile_stop(path)
    rows = _csv_rows(path)
    assert sorted(r[0] for r in rows) == ["ADD", "MATMUL", "SIGMOID"]
    totals = [r[4] for r in rows]
    assert totals == sorted(totals, reverse=True)
    for name, n, usage, avg, tot in rows:
        assert n == counts[name][0]
        assert usage == f"{100.0 * n / 6:.1f}"
        assert abs(avg - tot / n) <= 1e-5 * max(1.0, tot)
        assert abs(tot - counts[name][1]) <= 1e-5 * max(1.0, tot)


def test_profiler_times_the_ops_of_replayed_graphs():
    """A graph captured while profiling carries per-op event nodes: two replays of
    MATMUL -> ADD -> GELU, each collected, count two of each."""
    dev = device()
    s = oracle().stream(9601)
    x, w, bias = dev.tensor((256, 384)), dev.tensor((384, 128)), dev.tensor((256, 128))
    x.write(s.uniform(256 * 384, -1, 1))
    w.write(s.uniform(384 * 128, -1, 1))
    dev.eager = False
    try:
        r = dev.op("GELU", dev.op("ADD", dev.op("MATMUL", x, w), bias))
    finally:
        dev.eager = True
    dev.profile_start()
    try:
        for _ in range(2):  # a replay's events are read before the next replay reuses them
            dev.graph_exec(r)
            dev.profile_collect()
        assert [dev.profile_stats(op)[0] for op in ("MATMUL", "ADD", "GELU")] == [2, 2, 2]
    finally:
        dev.profile_stop(os.devnull)
        dev.graph_release(r)


# ---------------------------------------------------------------- bounded waits
@pytest.mark.parametrize("split,m", [(MB.TC_SPLIT_F16, 512), (MB.TC_SPLIT_F16, 128), (MB.TC_SPLIT_TF32, 512)])
def test_gemm_wait_that_expires_reports_device_wait(split, m):
    """MAG_CUDA_TC_TEST_STALL=1 gives the GEMM a first wait on a barrier phase that nothing
    completes, before any copy or MMA is issued: the wait runs out, every role leaves, TMEM is
    released, and mag_cuda_synchronize returns MAG_CUDA_E_DEVICE_WAIT once.  The next product on
    the same device is correct (CTA pairs at m = 512 with the f16 split, single CTAs otherwise)."""
    dev = device()
    MB.check(dev.L.mag_cuda_set_tc_split(dev.p, split), "split")
    MB.check(dev.L.mag_cuda_set_matmul_mode(dev.p, 2), "tc mode")
    s = oracle().stream(9700 + m)
    k, n = 256, 512
    x, y = s.uniform(m * k, -1, 1), s.uniform(k * n, -1, 1)
    tx, ty, tr = dev.tensor((m * k,)), dev.tensor((k * n,)), dev.tensor((m * n,))
    tx.write(x)
    ty.write(y)
    try:
        os.environ["MAG_CUDA_TC_TEST_STALL"] = "1"
        try:
            MB.check(dev.L.mag_cuda_matmul_f32(dev.p, tr.data_ptr, tx.data_ptr, ty.data_ptr, m, k, n), "mm")
            rc = dev.L.mag_cuda_synchronize(dev.p)
        finally:
            del os.environ["MAG_CUDA_TC_TEST_STALL"]
        assert rc == MB.E_DEVICE_WAIT
        assert dev.L.mag_cuda_synchronize(dev.p) == 0  # reported once
        MB.check(dev.L.mag_cuda_matmul_f32(dev.p, tr.data_ptr, tx.data_ptr, ty.data_ptr, m, k, n), "mm")
        assert dev.L.mag_cuda_synchronize(dev.p) == 0
        got = tr.read()
    finally:
        dev.L.mag_cuda_set_matmul_mode(dev.p, 0)
        dev.L.mag_cuda_set_tc_split(dev.p, MB.TC_SPLIT_F16)
    x64, y64 = x.reshape(m, k).astype(np.float64), y.reshape(k, n).astype(np.float64)
    err = np.abs(got.reshape(m, n) - x64 @ y64) / np.maximum(np.abs(x64) @ np.abs(y64), 1e-30)
    assert float(err.max()) <= 1e-5
