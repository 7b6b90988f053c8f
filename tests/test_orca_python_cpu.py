"""The CUDA drop-in for `orca.orca_python`, checked without a GPU: it imports,
exports the reference module's names (orca-python/src/lib.rs:909-919), parses
devices like the reference, and install() registers it under the name the
reference's Python package imports its compiled core from."""
import sys

import pytest

from orcaml_b200 import orca_python as op


def test_exports_match_reference_module():
    mod = op.install()
    try:
        assert sys.modules["orca.orca_python"] is mod
        for name in ["Tensor", "DType", "Device", "save_tensors", "load_tensors",
                     "set_grad_enabled", "is_grad_enabled"]:
            assert getattr(mod, name) is getattr(op, name)
    finally:
        sys.modules.pop("orca.orca_python", None)


def test_device_parsing_and_dtypes():
    assert op.Device("cuda:3").index == 3 and op.Device("gpu").index == 0
    assert op.Device("cpu").kind == "cpu"
    with pytest.raises(ValueError):
        op.Device("tpu:0")
    assert op.DType.FLOAT32 == op.DType.FLOAT32 and op.DType.FLOAT32 != op.DType.INT64
    with pytest.raises(TypeError):
        op.DType.FLOAT32 == 1
    with pytest.raises(TypeError):
        op.Tensor()


def test_grad_mode_is_thread_local():
    import threading
    seen = []
    op.set_grad_enabled(False)
    try:
        t = threading.Thread(target=lambda: seen.append(op.is_grad_enabled()))
        t.start()
        t.join()
        assert seen == [True] and not op.is_grad_enabled()
    finally:
        op.set_grad_enabled(True)


def test_broadcast_rule():
    assert op._broadcast([4, 1, 3], [2, 1]) == [4, 2, 3]
    assert op._broadcast([2, 3], [4, 3]) is None


def test_safetensors_container_roundtrip(tmp_path):
    """The container layout orca-serialize reads: 8-byte size, JSON header
    padded to 8, data offsets relative to the data section."""
    import json
    import struct
    import numpy as np
    from orcaml_b200 import safetensors_io as st
    a = np.arange(12, dtype=np.float32).reshape(3, 4)
    b = np.array([1, -2], dtype=np.int64)
    path = str(tmp_path / "x.safetensors")
    st.write(path, {"b": ("I64", [2], b.tobytes()), "a": ("F32", [3, 4], a.tobytes())},
             {"step": "7"})
    raw = open(path, "rb").read()
    (n,) = struct.unpack("<Q", raw[:8])
    assert n % 8 == 0
    hdr = json.loads(raw[8:8 + n])
    assert hdr["__metadata__"] == {"step": "7"}
    assert hdr["a"] == {"dtype": "F32", "shape": [3, 4], "data_offsets": [0, 48]}
    entries, meta = st.read(path)
    assert meta == {"step": "7"}
    assert np.array_equal(np.frombuffer(entries["a"][2], np.float32).reshape(3, 4), a)
    assert np.array_equal(np.frombuffer(entries["b"][2], np.int64), b)
    with pytest.raises(ValueError):
        st.write(path, {"a": ("F32", [5], a.tobytes())})
    open(path, "wb").write(raw[:20])
    with pytest.raises(ValueError):
        st.read(path)
