"""Generate tests/golden/loader.json from the reference's own DataLoader.

Run in the development container, where the reference source tree is mounted:

    python tests/golden/make_loader_golden.py /path/to/reference/python

The reference's `orca.data` (python/orca/data/dataloader.py) is pure Python;
oracle/orca_shim.py stands in for the compiled `orca.orca_python` module it
imports.  For each case the script records what the reference's DataLoader /
ArrayDataset / random_split / from_arrays produce -- batch values (which
encode the sample indices), shapes, lengths -- and the exception type and
message of each invalid argument, so that orcaml_b200/dataloader.py can be
checked against them without the reference present.
"""
from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)


def dataset_arrays(n):
    # Feature row i = [i, i + 0.25, -i]; label i % 3.
    return [[float(i), i + 0.25, -float(i)] for i in range(n)], [i % 3 for i in range(n)]


LOADER_CASES = [
    dict(n=10, batch_size=3),
    dict(n=10, batch_size=3, drop_last=True),
    dict(n=10, batch_size=3, shuffle=True, seed=7),
    dict(n=10, batch_size=3, shuffle=True, seed=7, drop_last=True),
    dict(n=37, batch_size=8, shuffle=True, seed=123),
    dict(n=37, batch_size=8, shuffle=True, seed=123, num_workers=3, prefetch_factor=1),
    dict(n=64, batch_size=16, shuffle=True, seed=0, drop_last=True),
    dict(n=5, batch_size=7),
    dict(n=5, batch_size=7, drop_last=True),
    dict(n=1, batch_size=1, shuffle=True, seed=3),
]

ERROR_CASES = [
    ("batch_size", dict(batch_size=0)),
    ("batch_size", dict(batch_size=True)),
    ("batch_size", dict(batch_size=2.0)),
    ("shuffle", dict(shuffle=1)),
    ("drop_last", dict(drop_last=None)),
    ("seed", dict(seed=True)),
    ("seed", dict(seed=1.5)),
    ("num_workers", dict(num_workers=True)),
    ("num_workers", dict(num_workers=-1)),
    ("prefetch_factor", dict(num_workers=1, prefetch_factor=0)),
]


def _err(fn):
    try:
        fn()
    except Exception as e:   # noqa: BLE001 -- the fixture records the type
        return [type(e).__name__, str(e)]
    return None


def main(ref_dir):
    from oracle import orca_shim
    orca = orca_shim.install(ref_dir)
    data = orca.data
    out = {"loader": [], "errors": [], "dataset_errors": [], "split": [], "collate_errors": []}
    for case in LOADER_CASES:
        kw = dict(case)
        n = kw.pop("n")
        X, y = dataset_arrays(n)
        ds = data.ArrayDataset(X, y, one_hot_classes=3)
        loader = data.DataLoader(ds, **kw)
        batches = [[t.to_list() for t in b] for b in loader]
        shapes = [[list(t.shape) for t in b] for b in loader]
        out["loader"].append({"case": case, "len": len(loader), "batches": batches,
                              "shapes": shapes})
    X, y = dataset_arrays(4)
    ds = data.ArrayDataset(X, y)
    for name, kw in ERROR_CASES:
        out["errors"].append({"arg": name, "kwargs": kw,
                              "error": _err(lambda: data.DataLoader(ds, **kw))})
    out["dataset_errors"] = [
        {"what": "no arrays", "error": _err(lambda: data.ArrayDataset())},
        {"what": "length mismatch", "error": _err(lambda: data.ArrayDataset([[1.0], [2.0]], [0]))},
        {"what": "label out of range",
         "error": _err(lambda: data.ArrayDataset([[1.0]], [3], one_hot_classes=3))},
        {"what": "fractional label",
         "error": _err(lambda: data.ArrayDataset([[1.0]], [0.5], one_hot_classes=3))},
        {"what": "vector label",
         "error": _err(lambda: data.ArrayDataset([[1.0]], [[0, 1]], one_hot_classes=3))},
        {"what": "index out of range", "error": _err(lambda: data.ArrayDataset([[1.0]])[1])},
    ]
    ragged = data.ArrayDataset([[1.0], [2.0, 3.0]], [[1.0], [2.0]])
    out["collate_errors"].append({"what": "ragged batch",
                                  "error": _err(lambda: list(data.DataLoader(ragged,
                                                                             batch_size=2)))})
    one = data.ArrayDataset([0, 1, 2])
    out["single_array"] = {"batches": [[t.to_list() for t in b]
                                       for b in data.DataLoader(one, batch_size=2)],
                           "item": list(one[1])}
    for lengths, seed in (([8, 2], 5), ([3, 3, 4], 11), ([10, 0], None)):
        X, y = dataset_arrays(10)
        ds = data.ArrayDataset(X, y)
        parts = data.random_split(ds, lengths, seed=seed)
        out["split"].append({"lengths": lengths, "seed": seed,
                             "indices": [list(p.indices) for p in parts] if seed is not None
                             else None,
                             "lens": [len(p) for p in parts]})
    fa = data.from_arrays([[1.0, 2.0], [3.0, 4.0], [5.0, 6.0]], [0, 1, 2], batch_size=2,
                          one_hot_classes=3)
    out["from_arrays"] = [[t.to_list() for t in b] for b in fa]
    path = os.path.join(HERE, "loader.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", path)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    main(sys.argv[1])
