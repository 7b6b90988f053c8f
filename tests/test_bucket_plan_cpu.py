"""The gradient exchange plan of the step runner, on the CPU (host-only ABI).

The runner keeps every gradient in one arena in Module.parameters() order and
all-reduces it in per-layer buckets, last layer first.  Checked against the
order the reference's own Sequential yields (tests/golden/param_order.json,
recorded from python/orca/nn/module.py:32-44 by make_param_order.py):

* the arena layout: parameter i starts where parameters 0..i-1 end, with the
  reference's shapes (W [in, out], then b [1, out], per Linear);
* the buckets tile the arena exactly once, each inside one layer's (W, b)
  range and no larger than the bucket size, layers in reverse order and the
  pieces of a layer in ascending order.
"""
import ctypes
import json
import os

import numpy as np
import pytest

from orcaml_b200 import _lib as L

HERE = os.path.dirname(os.path.abspath(__file__))


def plan(dims, bucket_bytes):
    lib = L.load()
    d = (ctypes.c_int64 * len(dims))(*dims)
    n = ctypes.c_int()
    L.check(lib.orca_mlp_bucket_plan(len(dims) - 1, d, bucket_bytes, 0, None, None, None,
                                     ctypes.byref(n)))
    off = (ctypes.c_int64 * n.value)()
    cnt = (ctypes.c_int64 * n.value)()
    lay = (ctypes.c_int * n.value)()
    L.check(lib.orca_mlp_bucket_plan(len(dims) - 1, d, bucket_bytes, n.value, off, cnt, lay,
                                     ctypes.byref(n)))
    return list(off), list(cnt), list(lay)


def arena_ranges(shapes):
    """(start, end) of each parameter when stored back to back in order."""
    out, pos = [], 0
    for s in shapes:
        n = int(np.prod(s))
        out.append((pos, pos + n))
        pos += n
    return out


with open(os.path.join(HERE, "golden", "param_order.json")) as f:
    MODELS = json.load(f)
WIDE = [[784, 8192, 8192, 10], [4096] + [16384] * 6 + [1000]]


@pytest.mark.parametrize("case", MODELS, ids=lambda c: "-".join(map(str, c["dims"])))
def test_arena_is_module_parameters_order(case):
    dims, shapes = case["dims"], [tuple(s) for s in case["parameter_shapes"]]
    assert shapes == [s for l in range(len(dims) - 1)
                      for s in ((dims[l], dims[l + 1]), (1, dims[l + 1]))]
    ranges = arena_ranges(shapes)
    off, cnt, lay = plan(dims, 0)
    # One bucket per layer (bucket size 0), covering exactly its W and b.
    assert lay == list(range(len(dims) - 2, -1, -1))
    for o, c, l in zip(off, cnt, lay):
        assert (o, o + c) == (ranges[2 * l][0], ranges[2 * l + 1][1])


@pytest.mark.parametrize("dims", [m["dims"] for m in MODELS] + WIDE, ids=str)
@pytest.mark.parametrize("bucket_bytes", [0, 4, 1000, 64 << 20, 25 << 20])
def test_buckets_tile_the_arena_layer_by_layer(dims, bucket_bytes):
    shapes = [s for l in range(len(dims) - 1) for s in ((dims[l], dims[l + 1]), (1, dims[l + 1]))]
    ranges = arena_ranges(shapes)
    total = ranges[-1][1]
    chunk = bucket_bytes // 4 if bucket_bytes else total
    if total // max(chunk, 1) > 200_000:
        pytest.skip("too many buckets to list")
    off, cnt, lay = plan(dims, bucket_bytes)
    covered = sorted(zip(off, cnt))
    pos = 0
    for o, c in covered:
        assert o == pos and 0 < c <= max(chunk, 1)
        pos += c
    assert pos == total
    for o, c, l in zip(off, cnt, lay):
        lo, hi = ranges[2 * l][0], ranges[2 * l + 1][1]
        assert lo <= o and o + c <= hi
    assert lay == sorted(lay, reverse=True)
    for l in set(lay):
        mine = [o for o, x in zip(off, lay) if x == l]
        assert mine == sorted(mine)


def test_plan_rejects_bad_arguments():
    lib = L.load()
    n = ctypes.c_int()
    d = (ctypes.c_int64 * 3)(4, 0, 2)
    assert lib.orca_mlp_bucket_plan(2, d, 0, 0, None, None, None, ctypes.byref(n)) != 0
    d = (ctypes.c_int64 * 3)(4, 3, 2)
    off = (ctypes.c_int64 * 1)()
    assert lib.orca_mlp_bucket_plan(2, d, 4, 1, off, None, None, ctypes.byref(n)) != 0
