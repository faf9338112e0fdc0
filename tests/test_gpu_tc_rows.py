"""The tensor-core product with 128-byte ring rows (64 f16 of K per row, the default for pair
products of the f16 split) against 64-byte rows (MAG_CUDA_TC_ROW128=0, MAG_CUDA_TC_ROW128_FUSED=0;
read when the library first launches a product, so each form runs in a process of its own).
Both issue the MMAs over K in the same order, so every result is bit-identical: a single product,
a last-wave split product, a batched product and a fused layer (bias + GELU), all within 1e-5 of
|X||Y|."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

pytestmark = pytest.mark.gpu

SCRIPT = r'''
import sys, json, numpy as np
sys.path[:0] = [{root!r}, {pkg!r}, {orc!r}, {tests!r}, {golden!r}]
import mag_b200 as MB
from harness import oracle
dev = MB.Device()
o = oracle()
out = {{}}
def product(name, m, k, n, seed):
    s = o.stream(seed)
    x, y = s.uniform(m * k, -1, 1), s.normal(k * n, 0.0, k ** -0.5)
    tx, ty, tr = dev.tensor((m * k,)), dev.tensor((k * n,)), dev.tensor((m * n,))
    tx.write(x); ty.write(y)
    MB.check(dev.L.mag_cuda_matmul_f32(dev.p, tr.data_ptr, tx.data_ptr, ty.data_ptr, m, k, n), name)
    out[name] = tr.read()
product("single", 2048, 1024, 1536, 11)     # pair tiles, K a multiple of 64
product("tail", 4096, 512, 4096, 12)        # 256 tiles on 74 pairs: the last wave split along K
s = o.stream(13)
b, m = 8, 512
x, y = s.uniform(b * m * m, -1, 1), s.normal(b * m * m, 0.0, m ** -0.5)
tx, ty, tr = dev.tensor((b * m * m,)), dev.tensor((b * m * m,)), dev.tensor((b * m * m,))
tx.write(x); ty.write(y)
MB.check(dev.L.mag_cuda_matmul_batched_f32(dev.p, tr.data_ptr, tx.data_ptr, ty.data_ptr, b, m, m, m), "batched")
out["batched"] = tr.read()
s = o.stream(14)
rows, d_in, d_out = 4096, 1024, 1024
x, w = s.uniform(rows * d_in, -1, 1), s.normal(d_in * d_out, 0.0, d_in ** -0.5)
bias = s.uniform(rows * d_out, -0.1, 0.1)
tx, tw, tb = dev.tensor((rows, d_in)), dev.tensor((d_in, d_out)), dev.tensor((rows, d_out))
tx.write(x); tw.write(w); tb.write(bias)
dev.eager = False
r = dev.op("GELU", dev.op("ADD", dev.op("MATMUL", tx, tw), tb), inplace=True)
dev.eager = True
dev.graph_exec(r, fused=True)
out["fused"] = r.read()
dev.graph_release(r)
np.savez({path!r}, **out)
print(json.dumps({{"ok": True}}))
'''


def _run(tmp_path, tag, env_extra):
    path = str(tmp_path / f"{tag}.npz")
    code = SCRIPT.format(root=ROOT, pkg=os.path.join(ROOT, "magnetron-pre-oss-release-old_b200"),
                         orc=os.path.join(ROOT, "oracle"), tests=HERE, golden=os.path.join(HERE, "golden"), path=path)
    env = dict(os.environ, **env_extra)
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-3000:]
    return np.load(path)


def test_wide_and_narrow_ring_rows_are_bit_identical(tmp_path):
    wide = _run(tmp_path, "wide", {"MAG_CUDA_TC_ROW128": "1", "MAG_CUDA_TC_ROW128_FUSED": "1"})
    narrow = _run(tmp_path, "narrow", {"MAG_CUDA_TC_ROW128": "0", "MAG_CUDA_TC_ROW128_FUSED": "0"})
    for name in ("single", "tail", "batched", "fused"):
        a, b = wide[name], narrow[name]
        assert a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32)), name
        assert np.all(np.isfinite(a)), name
