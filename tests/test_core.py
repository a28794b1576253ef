"""Foundation types and Config: the reference's TensorTest / ConfigTest /
TensorUtilsTest cases (turbol_vllm/tests/test_tensor.cpp, test_config.cpp,
test_tensor_utils.cpp) as behaviour contracts, plus the zero-copy bridge."""
import os

import numpy as np
import pytest
import torch

import turbol_b200 as turbol


def test_tensor_construction_and_shape():
    t = turbol.Tensor([2, 3], "float32", "cpu")
    assert t.numel() == 6
    assert t.shape().to_list() == [2, 3]
    assert len(t.shape()) == 2 and t.shape()[1] == 3 and t.shape()[-1] == 3
    assert t.dtype() == "float32"
    assert t.device() == "CPU"
    assert not t.is_cuda()
    assert np.all(t.to_numpy() == 0)  # zero-initialised (reference leaves memory uninitialised)


def test_tensor_copy_is_deep_and_numpy_view_writes_through():
    t = turbol.Tensor([4], "float32", "cpu")
    t.to_numpy()[:] = [1, 2, 3, 4]
    c = t.clone()
    t.to_numpy()[0] = 42
    assert c.to_numpy().tolist() == [1, 2, 3, 4]
    assert t.to_numpy()[0] == 42


@pytest.mark.parametrize("dt,size", [("float32", 4), ("float16", 2), ("int32", 4), ("int64", 8), ("int8", 1),
                                     ("uint8", 1), ("bool", 1), ("bfloat16", 2)])
def test_dtype_sizes(dt, size):
    t = turbol.Tensor([3], dt, "cpu")
    assert t.size_bytes() == 3 * size  # int32 is 4 bytes (the reference's CPU tree says 8)


def test_zero_copy_torch_bridge():
    x = torch.arange(6, dtype=torch.float32)
    t = turbol.from_torch(x)
    y = turbol.to_torch(t)
    assert y.data_ptr() == x.data_ptr()
    y[0] = 7
    assert x[0] == 7
    assert torch.utils.dlpack.from_dlpack(t).data_ptr() == x.data_ptr()


def test_status_and_shape():
    s = turbol.Status()
    assert s.ok() and bool(s) and s.code() == 0
    sh = turbol.Shape([2, 5])
    assert sh.numel() == 10 and repr(sh) == "Shape(2, 5)"
    with pytest.raises(IndexError):
        sh[5]


def test_status_codes_match_reference_values():
    # turbol_vllm/include/turbol/common.hpp:97-108: the integer codes and names
    sc = turbol.StatusCode
    expect = {"kOk": 0, "kInvalidArgument": 1, "kNotFound": 2, "kAlreadyExists": 3, "kResourceExhausted": 4,
              "kUnimplemented": 5, "kInternalError": 6, "kUnavailable": 7, "kTimeout": 8, "kCudaError": 100}
    for name, val in expect.items():
        assert int(getattr(sc, name)) == val, name
    assert int(sc.kOutOfMemory) == 4 and int(sc.kNotImplemented) == 5  # aliases


def test_config_roundtrip(tmp_path):
    c = turbol.Config()
    c.set("lr", 3e-4)
    c.set("steps", 200)
    c.set("use_gae", True)
    c.set("name", "ppo")
    assert c.has("lr") and not c.has("nope")
    assert abs(c.get_float("lr", 0.0) - 3e-4) < 1e-12
    assert c.get_int("steps", 0) == 200
    assert c.get_bool("use_gae", False) is True
    assert c.get_str("name", "") == "ppo"
    assert c.get_int("name", -1) == -1  # unparsable -> default
    p = str(tmp_path / "cfg.txt")
    assert c.save(p).ok()
    lines = open(p).read().splitlines()
    assert lines == sorted(lines)  # sorted by key
    d = turbol.Config()
    assert d.load(p).ok()
    assert d.get_int("steps", 0) == 200 and d.get_str("name", "") == "ppo"


def test_config_parsing_rules(tmp_path):
    p = tmp_path / "c.cfg"
    p.write_text("# comment\n\n  a = 1 \nflag=yes\nf=off\n")
    c = turbol.Config()
    assert c.load(str(p)).ok()
    assert c.get_int("a", 0) == 1 and c.get_bool("flag", False) and not c.get_bool("f", True)
    st = turbol.Config().load(str(tmp_path / "missing"))
    assert not st.ok() and st.code() == int(turbol.StatusCode.kNotFound)
    bad = tmp_path / "bad.cfg"
    bad.write_text("novalue\n")
    st = turbol.Config().load(str(bad))
    assert not st.ok() and st.code() == int(turbol.StatusCode.kInvalidArgument)


def test_tensor_utils_cpu():
    a = turbol.Tensor([5], "float32", "cpu")
    assert turbol.TensorUtils.fill(a, 2.0).ok()
    assert turbol.TensorUtils.add_scalar(a, 1.0).ok()
    assert turbol.TensorUtils.scale(a, 2.0).ok()
    assert a.to_numpy().tolist() == [6.0] * 5
    b = turbol.Tensor([5], "float32", "cpu")
    turbol.TensorUtils.fill(b, 1.0)
    out = turbol.Tensor()
    assert turbol.TensorUtils.add(a, b, out).ok()
    assert out.to_numpy().tolist() == [7.0] * 5
    assert turbol.TensorUtils.sub(a, b, out).ok()
    assert out.to_numpy().tolist() == [5.0] * 5
    assert not turbol.TensorUtils.add(a, turbol.Tensor([4], "float32", "cpu"), out).ok()


def test_helpers():
    assert turbol.get_version() == "1.0.0"
    info = turbol.get_build_info()
    assert info["arch"] == "sm_100a"
    mi = turbol.get_memory_info(0)
    assert set(mi) == {"total", "free", "used", "utilization"}


@pytest.mark.gpu
def test_tensor_cuda_and_utils(dev):
    t = turbol.Tensor([1000], "float32", dev)
    assert t.is_cuda() and t.device() == "CUDA:0"
    assert turbol.TensorUtils.fill(t, 3.0).ok()
    assert turbol.TensorUtils.scale(t, 2.0).ok()
    assert np.allclose(t.to_numpy(), 6.0)
    u = turbol.Tensor([1000], "float32", dev)
    turbol.TensorUtils.fill(u, 1.0)
    out = turbol.Tensor()
    assert turbol.TensorUtils.sub(t, u, out).ok()
    assert np.allclose(out.to_numpy(), 5.0)
    c = turbol.Tensor([3], "float32", "cpu")
    assert c.to_device(dev).ok() and c.is_cuda()
    x = torch.ones(8, device=dev)
    assert turbol.to_torch(turbol.from_torch(x)).data_ptr() == x.data_ptr()
