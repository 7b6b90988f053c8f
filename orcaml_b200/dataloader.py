"""The input pipeline: the reference's DataLoader with numpy collation into
page-locked memory, and a feeder that overlaps each batch's host->device copy
with the previous training step.

Reference: python/orca/data/dataloader.py
  * DataLoader (:152-350): arguments and their validation, __len__, the batch
    order (random.Random(seed).shuffle of range(n), consecutive slices,
    drop_last), num_workers / prefetch_factor thread prefetch of samples with
    batches yielded in order, and collation of each sample field into one
    [batch, ...] tensor (:309-350).
  * ArrayDataset (:353-408), SubsetDataset / random_split (:536-595),
    from_arrays (:598-626).
The reference collates every batch through nested Python lists into
Tensor.from_list, about a second per configs[2] batch (4096 x 784).  Here a
field is stacked by numpy, an ArrayDataset batch is a single row gather, and
the training feeder writes it straight into a page-locked buffer that the
step runner copies to the device on its own stream while the previous step
computes (orca_mlp_stage_batch / orca_mlp_step_staged).
"""
from __future__ import annotations

import ctypes
import queue
import random
import threading
import weakref
from collections.abc import Sequence
from concurrent.futures import FIRST_COMPLETED, ThreadPoolExecutor, wait
from typing import Any, Iterator, List, Optional

import numpy as np

from . import _lib as L


# ----------------------------------------------------------- page-locked memory
def pinned_empty(shape, dtype=np.float32) -> np.ndarray:
    """A numpy array in page-locked host memory (orca_host_alloc); the memory
    is returned with orca_host_free when the last view of it is gone."""
    shape = tuple(int(s) for s in shape)
    nbytes = max(1, int(np.prod(shape, dtype=np.int64)) * np.dtype(dtype).itemsize)
    ptr = ctypes.c_void_p()
    lib = L.load()
    L.check(lib.orca_host_alloc(nbytes, ctypes.byref(ptr)))
    raw = (ctypes.c_uint8 * nbytes).from_address(ptr.value)
    weakref.finalize(raw, lib.orca_host_free, ptr.value)
    return np.frombuffer(raw, dtype=dtype, count=int(np.prod(shape, dtype=np.int64))).reshape(shape)


# ----------------------------------------------------------------- validation
def _is_sequence(value: Any) -> bool:
    return isinstance(value, Sequence) and not isinstance(value, (str, bytes, bytearray))


def _validate_positive_int(name: str, value) -> int:
    if isinstance(value, bool) or not isinstance(value, int):
        raise TypeError(f"{name} must be a positive integer")
    if value <= 0:
        raise ValueError(f"{name} must be positive")
    return value


def _validate_non_negative_int(name: str, value) -> int:
    if isinstance(value, bool) or not isinstance(value, int):
        raise TypeError(f"{name} must be a non-negative integer")
    if value < 0:
        raise ValueError(f"{name} must be non-negative")
    return value


def _check_seed(seed):
    if seed is not None and (isinstance(seed, bool) or not isinstance(seed, int)):
        raise TypeError("seed must be an integer or None")


def _shape_of(value) -> List[int]:
    """Shape of a sample field; ragged nesting raises as the reference's
    _shape_of (dataloader.py:27-41)."""
    if isinstance(value, np.ndarray):
        return list(value.shape)
    if hasattr(value, "tolist") and not _is_sequence(value):
        value = value.tolist()
    if not _is_sequence(value):
        return []
    if len(value) == 0:
        return [0]
    first = _shape_of(value[0])
    for i, item in enumerate(value[1:], start=1):
        s = _shape_of(item)
        if s != first:
            raise ValueError("Samples must be rectangular; "
                             f"item at index {i} has shape {s}, expected {first}")
    return [len(value)] + first


def _as_float_array(array) -> np.ndarray:
    """An ArrayDataset input as a float array, or None when it is ragged."""
    if hasattr(array, "numpy") and hasattr(array, "shape") and not isinstance(array, np.ndarray):
        array = array.numpy()
    elif hasattr(array, "to_list") and hasattr(array, "shape"):
        array = np.asarray(array.to_list(), np.float64).reshape(list(array.shape))
    if isinstance(array, np.ndarray):
        a = array
    else:
        if not _is_sequence(array):
            raise ValueError("ArrayDataset arrays must be sequences")
        try:
            _shape_of(array)
        except ValueError:
            return None
        a = np.asarray(array, dtype=np.float64)
    if a.ndim == 0:
        raise ValueError("ArrayDataset arrays must be sequences")
    if a.dtype != np.float32:
        a = a.astype(np.float64)
    return a


# ------------------------------------------------------------------- datasets
class Dataset:
    """Map-style dataset (dataloader.py:141-148)."""

    def __len__(self) -> int:
        raise NotImplementedError

    def __getitem__(self, idx: int):
        raise NotImplementedError


class ArrayDataset(Dataset):
    """Equal-length in-memory arrays, one sample per row (dataloader.py:353-408).

    Rectangular inputs are held as numpy arrays (float32 kept as float32,
    anything else as float64), 1-D inputs as one column, and the last array
    one-hot encoded when one_hot_classes is given.  Samples read through
    __getitem__ come back as Python lists, as the reference returns them.
    """

    def __init__(self, *arrays, one_hot_classes: Optional[int] = None):
        if not arrays:
            raise ValueError("At least one array must be provided to ArrayDataset")
        cols = []
        for a in arrays:
            arr = _as_float_array(a)
            if arr is None:                        # ragged: kept as samples
                cols.append([list(v) if _is_sequence(v) else [float(v)] for v in a])
                continue
            if len(arr) == 0:
                raise ValueError("ArrayDataset arrays cannot be empty")
            cols.append(arr.reshape(len(arr), 1) if arr.ndim == 1 else arr)
        self.length = len(cols[0])
        for i, c in enumerate(cols):
            if len(c) != self.length:
                raise ValueError(f"Array at index {i} has length {len(c)}, expected {self.length}")
        if one_hot_classes is not None:
            k = _validate_positive_int("one_hot_classes", one_hot_classes)
            labels = cols[-1]
            if isinstance(labels, list) or labels.ndim != 2 or labels.shape[1] != 1:
                raise ValueError("one_hot_classes requires scalar class labels")
            lab = labels[:, 0]
            finite = np.isfinite(lab)
            idx = np.where(finite, lab, 0).astype(np.int64)
            frac = ~finite | (lab != idx)
            oob = (idx < 0) | (idx >= k)
            first = np.nonzero(frac | oob)[0]
            if first.size:                       # the first bad label decides, in order
                i = int(first[0])
                if frac[i]:
                    raise ValueError("one_hot_classes requires integer class labels")
                raise ValueError(f"Class label {int(idx[i])} is out of bounds for "
                                 f"one_hot_classes={k}")
            hot = np.zeros((self.length, k), np.float32)
            hot[np.arange(self.length), idx] = 1.0
            cols[-1] = hot
        self.arrays = cols

    @property
    def rectangular(self) -> bool:
        return all(isinstance(c, np.ndarray) for c in self.arrays)

    def __len__(self) -> int:
        return self.length

    def __getitem__(self, idx: int):
        if idx < 0:
            idx += self.length
        if idx < 0 or idx >= self.length:
            raise IndexError(f"ArrayDataset index {idx} out of range")
        return tuple(c[idx].tolist() if isinstance(c, np.ndarray) else c[idx]
                     for c in self.arrays)


class SubsetDataset(Dataset):
    """A subset of another dataset by index (dataloader.py:536-565)."""

    def __init__(self, dataset, indices: List[int]):
        if not hasattr(dataset, "__len__") or not hasattr(dataset, "__getitem__"):
            raise TypeError("dataset must implement __len__ and __getitem__")
        n = len(dataset)
        self.dataset = dataset
        self.indices = []
        for index in indices:
            if isinstance(index, bool) or not isinstance(index, int):
                raise TypeError("SubsetDataset indices must be integers")
            if index < 0:
                index += n
            if index < 0 or index >= n:
                raise IndexError(f"SubsetDataset index {index} out of range")
            self.indices.append(index)

    def __len__(self) -> int:
        return len(self.indices)

    def __getitem__(self, idx: int):
        if idx < 0:
            idx += len(self.indices)
        if idx < 0 or idx >= len(self.indices):
            raise IndexError(f"SubsetDataset index {idx} out of range")
        return self.dataset[self.indices[idx]]


def random_split(dataset, lengths: List[int], seed: Optional[int] = None) -> List[SubsetDataset]:
    """Non-overlapping random subsets (dataloader.py:568-595): the same
    random.Random(seed) permutation, cut in order."""
    _check_seed(seed)
    n = len(dataset)
    if any(isinstance(x, bool) or not isinstance(x, int) for x in lengths):
        raise TypeError("lengths must contain integers")
    if any(x < 0 for x in lengths):
        raise ValueError("lengths must be non-negative")
    if sum(lengths) != n:
        raise ValueError("Sum of input lengths does not equal the length of the input dataset")
    indices = list(range(n))
    random.Random(seed).shuffle(indices)
    out, start = [], 0
    for x in lengths:
        out.append(SubsetDataset(dataset, indices[start:start + x]))
        start += x
    return out


def _rows_of(dataset):
    """(base ArrayDataset, index map) when every sample is a row gather of a
    rectangular ArrayDataset, else None."""
    index_map = None
    while isinstance(dataset, SubsetDataset):
        idx = np.asarray(dataset.indices, np.int64)
        index_map = idx if index_map is None else idx[index_map]
        dataset = dataset.dataset
    if isinstance(dataset, ArrayDataset) and dataset.rectangular:
        return dataset, index_map
    return None


# ----------------------------------------------------------------- the loader
class DataLoader:
    """Batches of a map-style dataset (dataloader.py:152-350): same arguments,
    validation, order and yielded structure (a tuple of tensors when samples
    are tuples).  Tensors are the CUDA drop-in's (orcaml_b200.orca_python);
    `numpy_batches()` yields the same batches as float32 arrays, and
    `StagedFeeder` trains an MlpTrainer from them."""

    def __init__(self, dataset, batch_size: int = 1, shuffle: bool = False,
                 drop_last: bool = False, seed: Optional[int] = None, dtype=None, device=None,
                 num_workers: int = 0, prefetch_factor: int = 2):
        if not hasattr(dataset, "__len__") or not hasattr(dataset, "__getitem__"):
            raise TypeError("dataset must implement __len__ and __getitem__")
        if not isinstance(shuffle, bool):
            raise TypeError("shuffle must be a bool")
        if not isinstance(drop_last, bool):
            raise TypeError("drop_last must be a bool")
        _check_seed(seed)
        self.dataset = dataset
        self.batch_size = _validate_positive_int("batch_size", batch_size)
        self.shuffle = shuffle
        self.drop_last = drop_last
        self.seed = seed
        self.dtype = dtype
        if isinstance(device, str):
            from .orca_python import Device
            device = Device(device)
        self.device = device
        self.num_workers = _validate_non_negative_int("num_workers", num_workers)
        self.prefetch_factor = _validate_positive_int("prefetch_factor", prefetch_factor)
        self._n = len(dataset)
        if self._n < 0:
            raise ValueError("dataset length cannot be negative")

    def __len__(self) -> int:
        if self.drop_last:
            return self._n // self.batch_size
        return (self._n + self.batch_size - 1) // self.batch_size

    def batch_indices(self) -> List[List[int]]:
        """The sample indices of each batch of one pass, in yield order
        (dataloader.py:229-241)."""
        indices = list(range(self._n))
        if self.shuffle:
            random.Random(self.seed).shuffle(indices)
        out = []
        for start in range(0, len(indices), self.batch_size):
            b = indices[start:start + self.batch_size]
            if self.drop_last and len(b) < self.batch_size:
                continue
            out.append(b)
        return out

    # -- samples (dataloader.py:243-306)
    def _load_samples(self, batch: List[int]) -> List[Any]:
        samples = []
        for i in batch:
            try:
                samples.append(self.dataset[i])
            except Exception as exc:
                if hasattr(exc, "add_note"):
                    exc.add_note(f"DataLoader failed while loading dataset index {i}")
                raise
        return samples

    def _sample_batches(self, batches: List[List[int]]) -> Iterator[List[Any]]:
        if self.num_workers == 0:
            for b in batches:
                yield self._load_samples(b)
            return
        if not batches:
            return
        limit = max(1, self.num_workers * self.prefetch_factor)
        pending, done = {}, {}
        nxt_submit = nxt_yield = 0
        with ThreadPoolExecutor(max_workers=self.num_workers,
                                thread_name_prefix="orca-dataloader") as ex:
            def top_up():
                nonlocal nxt_submit
                while nxt_submit < len(batches) and len(pending) < limit:
                    pending[ex.submit(self._load_samples, batches[nxt_submit])] = nxt_submit
                    nxt_submit += 1
            try:
                top_up()
                while nxt_yield < len(batches):
                    if nxt_yield not in done:
                        finished, _ = wait(pending, return_when=FIRST_COMPLETED)
                        for f in finished:
                            done[pending.pop(f)] = f.result()
                        top_up()
                    while nxt_yield in done:
                        yield done.pop(nxt_yield)
                        nxt_yield += 1
                        top_up()
            finally:
                for f in pending:
                    f.cancel()

    # -- collation (dataloader.py:309-350), into float32 arrays
    @staticmethod
    def _collate_numpy(samples: List[Any], out: Optional[List[np.ndarray]] = None):
        """(fields, was_tuple): one float32 array per sample field."""
        norm = [s if isinstance(s, tuple) else (s,) for s in samples]
        arity = len(norm[0])
        for i, s in enumerate(norm[1:], start=1):
            if len(s) != arity:
                raise ValueError(f"Sample at index {i} has {len(s)} fields, expected {arity}")
        if out is not None and len(out) != arity:
            raise ValueError(f"samples have {arity} fields, the staging buffers {len(out)}")
        fields = []
        for f in range(arity):
            values = [s[f] for s in norm]
            shape = _shape_of(values[0])
            for i, v in enumerate(values[1:], start=1):
                vs = _shape_of(v)
                if vs != shape:
                    raise ValueError("All samples in a batch must have the same shape; "
                                     f"field {f} sample {i} has shape {vs}, expected {shape}")
            dst = out[f] if out is not None else np.empty([len(values)] + shape, np.float32)
            if list(dst.shape) != [len(values)] + shape:
                raise ValueError(f"field {f}: batch shape {[len(values)] + shape} does not match "
                                 f"the staging buffer {list(dst.shape)}")
            for i, v in enumerate(values):
                dst[i] = np.asarray(v, dtype=np.float64)   # one f64 -> f32 rounding, as from_list
            fields.append(dst)
        return fields, isinstance(samples[0], tuple)

    def _gather(self, rows, batch: List[int], out: Optional[List[np.ndarray]] = None):
        """An ArrayDataset batch as one row gather per field."""
        base, index_map = rows
        if out is not None and len(out) != len(base.arrays):
            raise ValueError(f"samples have {len(base.arrays)} fields, the staging buffers "
                             f"{len(out)}")
        idx = np.asarray(batch, np.int64)
        if index_map is not None:
            idx = index_map[idx]
        fields = []
        for f, col in enumerate(base.arrays):
            shape = [len(idx)] + list(col.shape[1:])
            dst = out[f] if out is not None else np.empty(shape, np.float32)
            if list(dst.shape) != shape:
                raise ValueError(f"field {f}: batch shape {shape} does not match the staging "
                                 f"buffer {list(dst.shape)}")
            if col.dtype == np.float32:
                np.take(col, idx, axis=0, out=dst)
            else:
                dst[...] = np.take(col, idx, axis=0)
            fields.append(dst)
        return fields, True

    def _numpy_iter(self, out_for=None) -> Iterator[tuple]:
        """Yields (fields, was_tuple) per batch; out_for(batch) may supply the
        destination arrays."""
        batches = self.batch_indices()
        rows = _rows_of(self.dataset)
        if rows is not None:
            for b in batches:
                yield self._gather(rows, b, out_for(b) if out_for else None)
            return
        for b, samples in zip(batches, self._sample_batches(batches)):
            yield self._collate_numpy(samples, out_for(b) if out_for else None)

    def numpy_batches(self) -> Iterator[Any]:
        """The batches of one pass as float32 numpy arrays (same structure as
        iterating the loader)."""
        for fields, was_tuple in self._numpy_iter():
            yield tuple(fields) if was_tuple else fields[0]

    def __iter__(self) -> Iterator[Any]:
        from . import orca_python as op
        for fields, was_tuple in self._numpy_iter():
            tensors = []
            for a in fields:
                t = op.Tensor._from_numpy(a.reshape(-1), list(a.shape), self.device)
                if self.dtype is not None:
                    t = t.to_dtype(self.dtype)
                tensors.append(t)
            yield tuple(tensors) if was_tuple else tensors[0]


def from_arrays(*arrays, batch_size: int = 32, shuffle: bool = False,
                one_hot_classes: Optional[int] = None, drop_last: bool = False,
                seed: Optional[int] = None, dtype=None, device=None, num_workers: int = 0,
                prefetch_factor: int = 2) -> DataLoader:
    """dataloader.py:598-626."""
    return DataLoader(ArrayDataset(*arrays, one_hot_classes=one_hot_classes),
                      batch_size=batch_size, shuffle=shuffle, drop_last=drop_last, seed=seed,
                      dtype=dtype, device=device, num_workers=num_workers,
                      prefetch_factor=prefetch_factor)


# ------------------------------------------------------------------ the feeder
class StagedFeeder:
    """Trains an MlpTrainer over a DataLoader with the input copies hidden.

    A collation thread gathers each batch (inputs, one-hot targets) into one
    of a ring of page-locked buffers; the calling thread stages batch k+1
    into a device slot (orca_mlp_stage_batch: an asynchronous copy on the
    step runner's copy stream) and then runs step k on the other slot
    (orca_mlp_step_staged), so the copy overlaps step k's kernels.  A buffer
    returns to the ring only after the step that consumed it has returned.
    Every step is the same as MlpTrainer.step on the same batch.

    The step runner has a fixed batch size: the loader's batch_size must
    equal it, and a pass whose last batch would be short needs drop_last.
    """

    def __init__(self, trainer, loader: DataLoader, depth: int = 2, host_alloc=None):
        if loader.batch_size != trainer.batch:
            raise ValueError(f"loader batch_size {loader.batch_size} != trainer batch "
                             f"{trainer.batch}")
        if not loader.drop_last and len(loader.dataset) % loader.batch_size:
            raise ValueError("the last batch would be short of the trainer's fixed batch; "
                             "use drop_last=True")
        self.trainer = trainer
        self.loader = loader
        self.depth = _validate_positive_int("depth", depth)
        alloc = host_alloc or pinned_empty      # the ring's allocator (shape -> float32 array)
        B, D0, C = trainer.batch, trainer.dims[0], trainer.dims[-1]
        self._ring = [(alloc((B, D0)), alloc((B, C))) for _ in range(self.depth + 2)]

    def run(self, max_steps: Optional[int] = None) -> List[float]:
        """One pass over the loader (or its first max_steps batches); returns
        the loss of every step."""
        total = len(self.loader)
        if max_steps is not None:
            total = min(total, _validate_non_negative_int("max_steps", max_steps))
        if total == 0:
            return []
        free: "queue.Queue[int]" = queue.Queue()
        for i in range(len(self._ring)):
            free.put(i)
        ready: "queue.Queue" = queue.Queue()
        stop = threading.Event()
        done = object()
        slot_of = [0]          # the ring buffer the worker is filling

        def worker():
            try:
                it = self.loader._numpy_iter(out_for=lambda b: list(self._ring[slot_of[0]]))
                for _ in range(total):
                    while True:
                        if stop.is_set():
                            return
                        try:
                            slot_of[0] = free.get(timeout=0.05)
                            break
                        except queue.Empty:
                            continue
                    next(it)
                    ready.put(slot_of[0])
                ready.put(done)
            except BaseException as exc:   # handed to the training thread
                ready.put(exc)

        th = threading.Thread(target=worker, name="orca-feeder", daemon=True)
        th.start()

        def take():
            item = ready.get()
            if isinstance(item, BaseException):
                raise item
            return item

        losses = []
        try:
            cur = take()
            x, t = self._ring[cur]
            self.trainer.stage_batch(0, x, t)
            for k in range(total):
                nxt = take() if k + 1 < total else done
                if nxt is not done:
                    x, t = self._ring[nxt]
                    self.trainer.stage_batch((k + 1) % 2, x, t)
                losses.append(self.trainer.step_staged(k % 2))
                free.put(cur)          # its copy finished before step k ran; step k is done
                cur = nxt
        finally:
            stop.set()
            th.join(timeout=10.0)
        return losses
