"""Host logic of the multi-GPU path on CPU: two gloo ranks shard an MLP batch
by rows, run the oracle forward on their rows and all-gather the outputs; the
result must equal the single-process forward bit for bit (shards of a
multiple of 4 rows, as the benchmark's 65536/N are).  A rank that fails
before the collective makes the other end with an error, not hang."""
import os
import socket
import subprocess
import sys
import textwrap

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

WORKER = textwrap.dedent("""
    import datetime, os, sys
    import numpy as np, torch, torch.distributed as dist
    sys.path[:0] = [{pkg!r}, {orc!r}]
    import dp
    from oracle import Oracle, pad6
    rank, world = int(sys.argv[1]), int(sys.argv[2])
    mode = sys.argv[3]
    dist.init_process_group("gloo", init_method="tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    o = Oracle()
    # shards of 20 rows: a MATMUL result's dim 0 is its row count, and the reference
    # splits unary ops into vector lanes / scalar tail by dim 0 mod 4, so shards
    # keep multiples of 4 rows to stay bit-identical to the unsharded forward
    rows, d_in, d_hid, d_out = 40, 24, 16, 10
    s = o.stream(0x5EED0D00)
    x = s.uniform(rows * d_in, -1, 1)
    w1 = s.uniform(d_in * d_hid, -0.5, 0.5)
    w2 = s.uniform(d_hid * d_out, -0.5, 0.5)
    start, n = dp.shard_rows(rows, world, rank)
    xs = x[start * d_in:(start + n) * d_in]
    h = o.unary("GELU", o.matmul(xs, w1, n, d_in, d_hid), pad6((n, d_hid)))
    z = o.softmax_rows(o.matmul(h, w2, n, d_hid, d_out), n, d_out)
    if mode == "fail" and rank == 1:
        raise SystemExit(3)
    if mode == "records":
        # a sharded full SUM/MIN/MAX: one (double sum, min, max, count) record per
        # rank, all-gathered in rank order, combined in that order
        n = 1001
        v = o.stream(0x5EED0D01).uniform(n, -1, 1)
        start, cnt = dp.shard_rows(n, world, rank)
        part = v[start:start + cnt]
        rec = np.zeros(3, np.float64)
        rec[0] = sum(float(e) for e in part)
        rec[1:2].view(np.float32)[:] = [part.min(), part.max()]
        rec[2:3].view(np.uint64)[0] = cnt
        recs = dp.gather_records(torch.from_numpy(rec), world).numpy().reshape(world, 3)
        total = 0.0
        for r in range(world):
            s_, c_ = dp.shard_rows(n, world, r)
            assert recs[r, 2].view(np.uint64) == c_, "records out of rank order"
            total += recs[r, 0]
        mn = recs[:, 1].copy().view(np.float32).reshape(world, 2)[:, 0].min()
        mx = recs[:, 1].copy().view(np.float32).reshape(world, 2)[:, 1].max()
        s6 = pad6((n,))
        assert abs(np.float32(total) - o.reduce("SUM", v, s6)) <= 1e-6
        assert mn == o.reduce("MIN", v, s6) and mx == o.reduce("MAX", v, s6)
        print("OK", flush=True)
        dist.destroy_process_group()
        raise SystemExit(0)
    try:
        full = dp.gather_rows(torch.from_numpy(z), rows, d_out, world, rank).numpy()
    except Exception as e:
        print("COLLECTIVE_ERROR", type(e).__name__, flush=True)
        raise SystemExit(4)
    if rank == 0:
        h = o.unary("GELU", o.matmul(x, w1, rows, d_in, d_hid), pad6((rows, d_hid)))
        ref = o.softmax_rows(o.matmul(h, w2, rows, d_hid, d_out), rows, d_out)
        assert np.array_equal(full.view(np.uint32), ref.view(np.uint32)), "gathered forward differs"
        print("OK", flush=True)
    dist.destroy_process_group()
""")


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(mode):
    code = WORKER.format(pkg=os.path.join(ROOT, "magnetron-pre-oss-release-old_b200"),
                         orc=os.path.join(ROOT, "oracle"), port=_port())
    procs = [subprocess.Popen([sys.executable, "-c", code, str(r), "2", mode], stdout=subprocess.PIPE,
                              stderr=subprocess.PIPE, text=True) for r in range(2)]
    outs = []
    for p in procs:
        try:
            out, err = p.communicate(timeout=120)
        except subprocess.TimeoutExpired:
            p.kill()
            out, err = p.communicate()
        outs.append((p.returncode, out, err))
    return outs


def test_shard_rows_cover_the_batch():
    import dp
    for total in (1, 7, 37, 65536):
        for world in (1, 2, 3, 8):
            spans = [dp.shard_rows(total, world, r) for r in range(world)]
            assert sum(n for _, n in spans) == total
            assert all(spans[i][0] + spans[i][1] == spans[i + 1][0] for i in range(world - 1))


def test_two_gloo_ranks_gather_the_exact_forward():
    outs = _run("ok")
    assert outs[0][0] == 0 and "OK" in outs[0][1], outs[0][2][-2000:]
    assert outs[1][0] == 0, outs[1][2][-2000:]


def test_failed_rank_ends_the_collective_with_an_error():
    outs = _run("fail")
    assert outs[1][0] == 3
    assert outs[0][0] != 0  # rank 0 sees the peer gone (error or timeout), it does not hang


def test_two_gloo_ranks_exchange_reduction_records_in_rank_order():
    outs = _run("records")
    for rc, out, err in outs:
        assert rc == 0 and "OK" in out, err[-2000:]
