"""Quantized .qraf files end to end on the GPU: written with the device quantizer,
loaded by qraf_cuda_model_open, and multiplied through the loaded weights.

The file's quantized bytes must equal the oracle quantizer's (the device
quantizer is byte-exact to quantize_q8_0 / quantize_q4_0,
src/tensor/quantize.cpp:105-183); the device copy must hold the file's bytes
unchanged; a matvec through a loaded weight must equal the oracle's
dispatch_matvec_q bit for bit in EXACT mode.  The host-cache preload
(qraf_cuda_host_cache_add, the call a host integration makes at
Transformer::init) must leave the later qraf_cuda_matvec_q_host calls nothing
to upload."""
from __future__ import annotations

import struct

import numpy as np
import pytest

import qraf_b200 as qb
from qraf_b200 import qraf_file as qf

pytestmark = pytest.mark.gpu

H, INTER = 256, 512
SHAPES = [("attn.q_proj.weight", qb.Q8_0, H, H, 32), ("attn.k_proj.weight", qb.Q8_0, 64, H, 32),
          ("mlp.gate_proj.weight", qb.Q4_0, INTER, H, 32), ("mlp.down_proj.weight", qb.Q4_0, H, INTER, 32),
          ("lm_head.weight", qb.Q8_0, 1000, H, 64), ("ragged.weight", qb.Q8_0, 7, 300, 32),
          ("big.weight", qb.Q4_0, 4096, 4096, 32)]


def _device_bytes(w: qb.Weight, torch) -> bytes:
    class _View:
        __cuda_array_interface__ = {"shape": (w.nbytes,), "typestr": "|u1", "data": (w.desc.data, False),
                                    "version": 3, "strides": None}

    return torch.as_tensor(_View(), device="cuda").cpu().numpy().tobytes()


@pytest.fixture(scope="module")
def model_file(tmp_path_factory, cuda):
    import torch

    path = str(tmp_path_factory.mktemp("qraf") / "model.qraf")
    w = qf.QrafFileWriter()
    w.set_config_string("architecture", "llama")
    w.set_config("hidden_size", H)
    w.set_config("intermediate_size", INTER)
    w.set_config("rope_theta", 10000.0)
    w.add_tensor("norm.weight", (H,), qf.DTYPE_F32, np.ones(H, np.float32))
    floats = {}
    for i, (name, dt, n, k, bs) in enumerate(SHAPES):
        wf = qb.fill_normal(100 + i, 0.0, 0.02, n * k).reshape(n, k)
        floats[name] = wf
        w.add_quantized(name, torch.from_numpy(wf).to(cuda), dt, bs)
    w.write(path)
    return path, floats


def test_file_bytes_are_the_reference_quantizer_bytes(model_file, oracle_lib):
    path, floats = model_file
    d = qf.read_directory(path)
    raw = open(path, "rb").read()
    for name, dt, n, k, bs in SHAPES:
        e = d["tensors"][name]
        assert (e.dtype, e.shape, e.block_size) == (dt, (n, k), bs)
        want = oracle_lib.quantize_rows(dt, floats[name], bs).tobytes()
        assert raw[e.data_offset:e.data_offset + e.data_size] == want, name
    # one scheme per (dtype, block size), group 1, flags 1 (writer.cpp:35-47)
    assert sorted((q[1], q[2], q[3], q[6]) for q in d["quant"]) == [(10, 32, 1, 1), (10, 64, 1, 1), (20, 32, 1, 1)]


def test_model_store_holds_the_file_and_multiplies_exactly(model_file, cuda, oracle_lib):
    import torch

    path, _ = model_file
    raw = open(path, "rb").read()
    d = qf.read_directory(path)
    m = qb.DeviceModel(path)
    assert m.names == [s[0] for s in SHAPES]       # F32 tensors are not uploaded
    info = m.info()
    assert info["num_weights"] == len(SHAPES) and info["device"] == 0
    assert info["device_bytes"] >= sum(d["tensors"][s[0]].data_size for s in SHAPES)
    assert m.config_u32("hidden_size") == H
    assert struct.unpack("<f", struct.pack("<I", m.config_u32("rope_theta")))[0] == 10000.0
    with pytest.raises(qb.QrafError):
        m.weight("norm.weight")
    with pytest.raises(qb.QrafError):
        m.config_u32("architecture")        # a string entry
    for name, dt, n, k, bs in SHAPES:
        w = m.weight(name)
        assert (w.rows, w.cols, w.dtype, w.desc.block_size, w.desc.owned) == (n, k, dt, bs, 0)
        assert w.desc.data % 256 == 0
        e = d["tensors"][name]
        assert _device_bytes(w, torch) == raw[e.data_offset:e.data_offset + e.data_size], name
        x = qb.fill_normal(7, 0.0, 1.0, k)
        y = qb.matvec_q(w, torch.from_numpy(x).to(cuda), mode=qb.MODE_EXACT).cpu().numpy()
        q = np.frombuffer(raw, np.uint8, e.data_size, e.data_offset)
        want = oracle_lib.matvec(dt, q, n, k, x, bs)
        assert y.tobytes() == want.tobytes(), name
    assert qb.device_status() == qb.OK
    torch.cuda.synchronize(cuda)
    free_open = torch.cuda.mem_get_info(cuda)[0]
    m.close()
    assert torch.cuda.mem_get_info(cuda)[0] - free_open >= info["device_bytes"] - (2 << 20)


def test_three_dimensional_tensor_is_rows_by_last_dim(tmp_path, cuda, oracle_lib):
    import torch

    w = qf.QrafFileWriter()
    vals = qb.fill_normal(5, 0.0, 0.05, 2 * 3 * 64).reshape(6, 64)
    q = oracle_lib.quantize_rows(qb.Q4_0, vals)
    sid = w.add_quant_scheme(qb.Q4_0, 32)
    w.add_tensor("stacked", (2, 3, 64), qb.Q4_0, q, sid)
    path = str(tmp_path / "s.qraf")
    w.write(path)
    m = qb.DeviceModel(path)
    wt = m.weight("stacked")
    assert (wt.rows, wt.cols) == (6, 64)
    x = qb.fill_normal(6, 0.0, 1.0, 64)
    y = qb.matvec_q(wt, torch.from_numpy(x).to(cuda), mode=qb.MODE_EXACT).cpu().numpy()
    assert y.tobytes() == oracle_lib.matvec(qb.Q4_0, q, 6, 64, x).tobytes()
    m.close()


def test_host_cache_preload(model_file, cuda, oracle_lib):
    path, _ = model_file
    d = qf.read_directory(path)
    host = np.fromfile(path, dtype=np.uint8)          # the bytes a host integration has mapped
    qb.host_cache_clear()
    assert qb.host_cache_info() == (0, 0)
    views = {}
    for name, dt, n, k, bs in SHAPES:
        e = d["tensors"][name]
        views[name] = host[e.data_offset:e.data_offset + e.data_size]
        qb.host_cache_add(views[name], dt, n, k, bs)
    entries, nbytes = qb.host_cache_info()
    assert entries == len(SHAPES)
    assert nbytes == sum(d["tensors"][s[0]].data_size for s in SHAPES)
    qb.host_cache_add(views["lm_head.weight"], qb.Q8_0, 1000, H, 64)      # again: no new entry
    assert qb.host_cache_info() == (entries, nbytes)
    for name, dt, n, k, bs in SHAPES:
        x = qb.fill_normal(9, 0.0, 1.0, k)
        y = np.empty(n, np.float32)
        qb.dispatch_matvec_q(views[name], views[name].size, dt, bs, n, k, x, y, 1, qb.MODE_EXACT)
        assert y.tobytes() == oracle_lib.matvec(dt, views[name], n, k, x, bs).tobytes(), name
    assert qb.host_cache_info() == (entries, nbytes)     # every call found its preloaded weight
    qb.host_cache_clear()
    assert qb.host_cache_info() == (0, 0)


def test_host_cache_add_rejects_a_short_buffer(cuda):
    buf = np.zeros(100, np.uint8)
    with pytest.raises(qb.QrafError) as e:
        qb.host_cache_add(buf, qb.Q8_0, 4, 64)
    assert e.value.code == qb.ERR_INVALID


def test_f32_tensors_join_the_allocation(model_file, cuda):
    """qraf_cuda_model_open_ex(QRAF_MODEL_F32): F32 tensors are on the device with
    the file's values; without the flag they are absent; string config entries
    and the quantized tensors are the same either way."""
    import torch

    path, _ = model_file
    m = qb.DeviceModel(path, f32=True)
    ptr, n = m.tensor_f32("norm.weight")
    assert n == H
    got = qb._wrap_device_floats(ptr, n, cuda).cpu().numpy()
    assert np.array_equal(got, np.ones(H, np.float32))
    assert sorted(m.names) == sorted(s[0] for s in SHAPES)
    plain = qb.DeviceModel(path)
    with pytest.raises(qb.QrafError) as e:
        plain.tensor_f32("norm.weight")
    assert e.value.code == qb.ERR_INVALID and "QRAF_MODEL_F32" in str(e.value)
    assert m.info()["device_bytes"] > plain.info()["device_bytes"]
    plain.close()
    m.close()
    torch.cuda.synchronize()
