"""The input pipeline's host side (orcaml_b200/dataloader.py), without a GPU.

* Batches, lengths, shapes, split indices and error messages equal what the
  reference's own DataLoader / ArrayDataset / random_split / from_arrays
  (python/orca/data/dataloader.py) produced for the same arguments
  (tests/golden/loader.json, written by tests/golden/make_loader_golden.py).
* The row-gather fast path and the per-sample collation path agree, the
  thread prefetch keeps the batch order and reports the failing index
  (python/tests/test_high_level_api.py:60-120 are the reference's own tests of
  these).
* StagedFeeder against a stand-in trainer whose "copy" reads the staged host
  arrays only when the step runs -- the latest moment an asynchronous copy can
  complete -- so a ring buffer reused too early would show up as a wrong batch.
"""
import json
import os
import time

import numpy as np
import pytest

from orcaml_b200 import dataloader as D

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def fx():
    with open(os.path.join(HERE, "golden", "loader.json")) as f:
        return json.load(f)


def _arrays(n):
    return [[float(i), i + 0.25, -float(i)] for i in range(n)], [i % 3 for i in range(n)]


def _flat(batch):
    return [np.asarray(a, np.float32).reshape(-1).tolist() for a in batch]


def test_batches_match_reference(fx):
    for rec in fx["loader"]:
        kw = dict(rec["case"])
        X, y = _arrays(kw.pop("n"))
        for as_numpy in (False, True):
            Xa = np.asarray(X, np.float32) if as_numpy else X
            loader = D.DataLoader(D.ArrayDataset(Xa, y, one_hot_classes=3), **kw)
            assert len(loader) == rec["len"], rec["case"]
            got = [_flat(b) for b in loader.numpy_batches()]
            assert got == rec["batches"], rec["case"]
            assert [[list(a.shape) for a in b] for b in loader.numpy_batches()] == rec["shapes"]


def test_generic_collation_matches_gather(fx):
    class ListDataset(D.Dataset):          # per-sample __getitem__, no fast path
        def __init__(self, X, y):
            self.X, self.y = X, y

        def __len__(self):
            return len(self.X)

        def __getitem__(self, i):
            hot = [0.0, 0.0, 0.0]
            hot[self.y[i]] = 1.0
            return (self.X[i], hot)

    for rec in fx["loader"]:
        kw = dict(rec["case"])
        X, y = _arrays(kw.pop("n"))
        loader = D.DataLoader(ListDataset(X, y), **kw)
        assert [_flat(b) for b in loader.numpy_batches()] == rec["batches"], rec["case"]


def test_argument_errors_match_reference(fx):
    X, y = _arrays(4)
    ds = D.ArrayDataset(X, y)
    for rec in fx["errors"]:
        exc = {"TypeError": TypeError, "ValueError": ValueError}[rec["error"][0]]
        with pytest.raises(exc) as info:
            D.DataLoader(ds, **rec["kwargs"])
        assert str(info.value) == rec["error"][1]


def test_dataset_errors_match_reference(fx):
    cases = {
        "no arrays": lambda: D.ArrayDataset(),
        "length mismatch": lambda: D.ArrayDataset([[1.0], [2.0]], [0]),
        "label out of range": lambda: D.ArrayDataset([[1.0]], [3], one_hot_classes=3),
        "fractional label": lambda: D.ArrayDataset([[1.0]], [0.5], one_hot_classes=3),
        "vector label": lambda: D.ArrayDataset([[1.0]], [[0, 1]], one_hot_classes=3),
        "index out of range": lambda: D.ArrayDataset([[1.0]])[1],
    }
    for rec in fx["dataset_errors"]:
        exc = {"ValueError": ValueError, "IndexError": IndexError}[rec["error"][0]]
        with pytest.raises(exc) as info:
            cases[rec["what"]]()
        assert str(info.value) == rec["error"][1], rec["what"]


def test_ragged_single_array_split_from_arrays(fx):
    ragged = D.ArrayDataset([[1.0], [2.0, 3.0]], [[1.0], [2.0]])
    with pytest.raises(ValueError) as info:
        list(D.DataLoader(ragged, batch_size=2).numpy_batches())
    assert str(info.value) == fx["collate_errors"][0]["error"][1]
    one = D.ArrayDataset([0, 1, 2])
    assert [_flat(b) for b in D.DataLoader(one, batch_size=2).numpy_batches()] == \
        fx["single_array"]["batches"]
    assert list(one[1]) == fx["single_array"]["item"]
    for rec in fx["split"]:
        X, y = _arrays(10)
        parts = D.random_split(D.ArrayDataset(X, y), rec["lengths"], seed=rec["seed"])
        assert [len(p) for p in parts] == rec["lens"]
        if rec["indices"] is not None:
            assert [p.indices for p in parts] == rec["indices"]
    fa = D.from_arrays([[1.0, 2.0], [3.0, 4.0], [5.0, 6.0]], [0, 1, 2], batch_size=2,
                       one_hot_classes=3)
    assert [_flat(b) for b in fa.numpy_batches()] == fx["from_arrays"]


def test_subset_of_array_dataset_uses_rows():
    X = np.arange(40, dtype=np.float32).reshape(10, 4)
    ds = D.ArrayDataset(X, np.arange(10) % 2, one_hot_classes=2)
    part = D.random_split(ds, [6, 4], seed=9)[0]
    fast = list(D.DataLoader(part, batch_size=3, shuffle=True, seed=1).numpy_batches())
    slow = [D.DataLoader._collate_numpy([part[i] for i in b])[0]
            for b in D.DataLoader(part, batch_size=3, shuffle=True, seed=1).batch_indices()]
    for a, b in zip(fast, slow):
        assert all(np.array_equal(u, v) for u, v in zip(a, b))


def test_prefetch_order_and_error_note():
    class Delayed(D.Dataset):
        def __len__(self):
            return 4

        def __getitem__(self, idx):
            time.sleep((4 - idx) * 0.005)
            return [float(idx)]

    loader = D.DataLoader(Delayed(), batch_size=1, num_workers=4, prefetch_factor=1)
    assert [b.reshape(-1)[0] for b in loader.numpy_batches()] == [0.0, 1.0, 2.0, 3.0]

    class Failing(D.Dataset):
        def __len__(self):
            return 3

        def __getitem__(self, idx):
            if idx == 1:
                raise ValueError("bad sample")
            return [float(idx)]

    with pytest.raises(ValueError, match="bad sample") as info:
        list(D.DataLoader(Failing(), batch_size=1, num_workers=2).numpy_batches())
    assert "DataLoader failed while loading dataset index 1" in getattr(info.value,
                                                                        "__notes__", [])


class _LateCopyTrainer:
    """Stands in for MlpTrainer: stage_batch keeps references to the host
    arrays and the step reads them, i.e. the copy lands as late as it may."""

    def __init__(self, dims, batch):
        self.dims, self.batch = list(dims), batch
        self.slots = [None, None]
        self.seen = []

    def stage_batch(self, slot, x, t):
        assert self.slots[slot] is None, "slot restaged before its step"
        self.slots[slot] = (x, t)

    def step_staged(self, slot):
        x, t = self.slots[slot]
        self.slots[slot] = None
        self.seen.append((x.copy(), t.copy()))
        time.sleep(0.001)
        return float(x.sum())


@pytest.mark.parametrize("depth", [1, 2, 4])
def test_staged_feeder_ring_and_order(depth):
    rng = np.random.default_rng(0)
    X = rng.random((96, 5), dtype=np.float32)
    y = rng.integers(0, 3, 96)
    loader = D.DataLoader(D.ArrayDataset(X, y, one_hot_classes=3), batch_size=8, shuffle=True,
                          seed=4)
    tr = _LateCopyTrainer([5, 7, 3], 8)
    feeder = D.StagedFeeder(tr, loader, depth=depth,
                            host_alloc=lambda s: np.empty(s, np.float32))
    losses = feeder.run()
    want = list(loader.numpy_batches())
    assert len(tr.seen) == len(want) == 12
    for (x, t), (wx, wt) in zip(tr.seen, want):
        assert np.array_equal(x, wx) and np.array_equal(t, wt)
    assert losses == [float(wx.sum()) for wx, _ in want]
    assert feeder.run(max_steps=5) == losses[:5]


def test_staged_feeder_rejects_mismatch_and_reports_worker_errors():
    X = np.zeros((10, 5), np.float32)
    loader = D.DataLoader(D.ArrayDataset(X, np.zeros(10), one_hot_classes=3), batch_size=4)
    alloc = lambda s: np.empty(s, np.float32)  # noqa: E731
    with pytest.raises(ValueError, match="drop_last"):
        D.StagedFeeder(_LateCopyTrainer([5, 3], 4), loader, host_alloc=alloc)
    with pytest.raises(ValueError, match="batch"):
        D.StagedFeeder(_LateCopyTrainer([5, 3], 8), loader, host_alloc=alloc)

    class Failing(D.Dataset):
        def __len__(self):
            return 8

        def __getitem__(self, idx):
            if idx == 5:
                raise ValueError("bad sample")
            return ([0.0] * 5, [1.0, 0.0, 0.0])

    feeder = D.StagedFeeder(_LateCopyTrainer([5, 3], 2), D.DataLoader(Failing(), batch_size=2),
                            host_alloc=alloc)
    with pytest.raises(ValueError, match="bad sample"):
        feeder.run()
    three = D.ArrayDataset(np.zeros((4, 5)), np.zeros((4, 3)), np.zeros((4, 1)))
    feeder = D.StagedFeeder(_LateCopyTrainer([5, 3], 2), D.DataLoader(three, batch_size=2),
                            host_alloc=alloc)
    with pytest.raises(ValueError, match="fields"):
        feeder.run()
