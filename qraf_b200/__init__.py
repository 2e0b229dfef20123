"""qraf_b200 — B200-native block-quantized (Q8_0 / Q4_0) matvec for QRAF.

Host-side Python mirror of the reference's operator API for this one path
(simonpierreboucher02/qraf: ``qraf::dispatch_matvec_q`` in src/nn/backend.cpp:131-199,
``dot_q8_0_f32`` / ``dot_q4_0_f32`` and ``quantize_q8_0`` / ``quantize_q4_0`` in
src/tensor/quantize.cpp), calling the sm_100a kernels of ``libqraf_cuda.so``
through its C ABI (include/qraf_cuda.h).  PyTorch is used only to hold device
memory and streams.

There is no CPU fallback: every compute entry point runs on the GPU, and
the first call into it raises ImportError if the CUDA library has not been
built.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import build as _build

Q8_0 = 10
Q4_0 = 20

MODE_EXACT = 0
MODE_FAST = 1
MODE_TC = 2
MODE_AUTO = 3
MODE_FLAG_OVERLAP = 0x100
MODEL_F32 = 1               # qraf_cuda_model_open_ex: upload the F32 tensors too
DECODER_KV_INT8 = 1         # qraf_cuda_decoder_open_ex: int8 KV cache (the reference's QuantizedKVCache)

OK = 0
ERR_INVALID = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3
ERR_TIMEOUT = 4
ERR_COMM = 5
ERR_NOMEM = 6

LIB_PATH = _build.LIB


class QrafError(RuntimeError):
    """A non-zero status from the C ABI (the reference raises QrafError too, include/core/error.h)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"qraf_cuda error {code}: {msg}")
        self.code = code


class qraf_weight_t(C.Structure):
    _fields_ = [
        ("data", C.c_void_p),
        ("bytes", C.c_uint64),
        ("row_bytes", C.c_uint64),
        ("dtype", C.c_uint32),
        ("block_size", C.c_uint32),
        ("rows", C.c_uint32),
        ("cols", C.c_uint32),
        ("device", C.c_int32),
        ("owned", C.c_uint32),
    ]


def _load() -> C.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: run `python -m qraf_b200.build` (nvcc, sm_100a) first")
    lib = C.CDLL(LIB_PATH)
    W = C.POINTER(qraf_weight_t)
    vp, u32, u64, i32, f32p = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int, C.POINTER(C.c_float)
    sig = {
        "qraf_cuda_version": (C.c_char_p, []),
        "qraf_cuda_init": (i32, [i32]),
        "qraf_cuda_shutdown": (i32, []),
        "qraf_cuda_last_error": (i32, [C.c_char_p, C.c_size_t]),
        "qraf_cuda_device_status": (i32, [i32]),
        "qraf_row_bytes": (u64, [u32, u32, u32]),
        "qraf_cuda_weight_wrap": (i32, [vp, u64, u32, u32, u32, u32, W]),
        "qraf_cuda_weight_upload": (i32, [vp, u64, u32, u32, u32, u32, W]),
        "qraf_cuda_weight_free": (i32, [W]),
        "qraf_cuda_weight_shard": (i32, [W, u32, u32, W]),
        "qraf_cuda_matvec_q": (i32, [W, vp, vp, u32, i32, vp]),
        "qraf_cuda_matvec_q_multi": (i32, [W, u32, vp, C.POINTER(vp), u32, i32, vp]),
        "qraf_cuda_matvec_q_swiglu": (i32, [W, W, vp, vp, u32, i32, vp]),
        "qraf_cuda_matvec_q_multi_ex": (i32, [W, u32, vp, vp, C.c_float, C.POINTER(vp), C.POINTER(vp), u32, i32, vp]),
        "qraf_cuda_matvec_q_swiglu_ex": (i32, [W, W, vp, vp, C.c_float, vp, u32, i32, vp]),
        "qraf_cuda_matmul_tc_noalloc": (i32, [W, vp, vp, u32, i32, vp]),
        "qraf_cuda_dot_q": (i32, [u32, vp, vp, u64, u32, vp, i32, vp]),
        "qraf_cuda_block_partials": (i32, [W, vp, vp, vp]),
        "qraf_cuda_limb_partials": (i32, [W, vp, vp, vp, vp]),
        "qraf_cuda_quantize": (i32, [u32, vp, u64, u32, vp, vp]),
        "qraf_cuda_quantize_rows": (i32, [u32, vp, u32, u32, u32, vp, vp]),
        "qraf_cuda_dequantize": (i32, [u32, vp, u64, u32, vp, vp]),
        "qraf_cuda_matvec_q_host": (i32, [vp, u64, u32, u32, u32, u32, vp, vp, u32, i32]),
        "qraf_cuda_host_cache_clear": (i32, []),
        "qraf_cuda_host_cache_add": (i32, [vp, u64, u32, u32, u32, u32]),
        "qraf_cuda_host_cache_info": (i32, [C.POINTER(u32), C.POINTER(u64)]),
        "qraf_cuda_model_open": (i32, [C.c_char_p, C.POINTER(vp)]),
        "qraf_cuda_model_weight": (i32, [vp, C.c_char_p, W]),
        "qraf_cuda_model_info": (i32, [vp, C.POINTER(u32), C.POINTER(u64), C.POINTER(i32)]),
        "qraf_cuda_model_weight_name": (C.c_char_p, [vp, u32]),
        "qraf_cuda_model_config_u32": (i32, [vp, C.c_char_p, C.POINTER(u32)]),
        "qraf_cuda_model_close": (i32, [vp]),
        "qraf_cuda_launch_count": (u64, []),
        "qraf_cuda_decoder_open": (i32, [C.c_char_p, u32, u32, C.POINTER(vp)]),
        "qraf_cuda_decoder_step": (i32, [vp, u32, vp, vp, vp, vp, i32, vp]),
        "qraf_cuda_decoder_info": (i32, [vp, C.POINTER(u32), C.POINTER(u32), C.POINTER(u32), C.POINTER(u32),
                                         C.POINTER(u32)]),
        "qraf_cuda_decoder_close": (i32, [vp]),
        "qraf_cuda_decoder_open_ex": (i32, [C.c_char_p, u32, u32, u32, C.POINTER(vp)]),
        "qraf_cuda_decoder_kv_read": (i32, [vp, u32, u32, u32, vp, vp, f32p, f32p]),
        "qraf_cuda_model_open_ex": (i32, [C.c_char_p, u32, C.POINTER(vp)]),
        "qraf_cuda_model_tensor_f32": (i32, [vp, C.c_char_p, C.POINTER(vp), C.POINTER(u64)]),
        "qraf_fill_normal": (None, [u32, C.c_float, C.c_float, f32p, u64]),
        "qraf_cuda_comm_create": (i32, [i32, i32, u64, C.POINTER(vp)]),
        "qraf_cuda_comm_handle": (i32, [vp, vp]),
        "qraf_cuda_comm_open": (i32, [vp, vp]),
        "qraf_cuda_comm_open_local": (i32, [C.POINTER(vp), i32]),
        "qraf_cuda_comm_destroy": (i32, [vp]),
        "qraf_cuda_matvec_q_sharded": (i32, [vp, W, u32, u32, vp, u32, i32, vp, C.POINTER(vp)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_LIB = None


def _get_lib() -> C.CDLL:
    """The loaded libqraf_cuda.so; raises ImportError when it has not been built."""
    global _LIB
    if _LIB is None:
        _LIB = _load()
    return _LIB


def __getattr__(name):
    if name == "lib":
        return _get_lib()
    raise AttributeError(name)


def last_error() -> str:
    buf = C.create_string_buffer(512)
    _get_lib().qraf_cuda_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != OK:
        raise QrafError(rc, last_error())


def row_bytes(dtype: int, cols: int, block_size: int = 32) -> int:
    return int(_get_lib().qraf_row_bytes(dtype, block_size, cols))


def fill_normal(seed: int, mean: float, std: float, n: int) -> np.ndarray:
    """std::mt19937(seed) + std::normal_distribution<float>(mean, std), the reference's seeding idiom."""
    out = np.empty(n, dtype=np.float32)
    _get_lib().qraf_fill_normal(seed, mean, std, out.ctypes.data_as(C.POINTER(C.c_float)), n)
    return out


# ── device side (torch tensors as device memory) ─────────────────────────
def _torch():
    import torch

    return torch


def _stream(stream) -> C.c_void_p:
    torch = _torch()
    if stream is None:
        stream = torch.cuda.current_stream()
    return C.c_void_p(stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream))


def init(device: int = 0) -> None:
    check(_get_lib().qraf_cuda_init(device))


def device_status(clear: bool = True) -> int:
    return int(_get_lib().qraf_cuda_device_status(1 if clear else 0))


class Weight:
    """A quantized [rows][cols] weight in the reference's native block layout on one device."""

    def __init__(self, desc: qraf_weight_t, keepalive=None):
        self.desc = desc
        self._keep = keepalive

    @classmethod
    def from_device(cls, data, dtype: int, rows: int, cols: int, block_size: int = 32) -> "Weight":
        """Wrap a CUDA uint8 tensor holding rows * row_bytes native bytes (no copy)."""
        d = qraf_weight_t()
        check(_get_lib().qraf_cuda_weight_wrap(C.c_void_p(data.data_ptr()), data.numel() * data.element_size(), dtype,
                                        block_size, rows, cols, C.byref(d)))
        return cls(d, keepalive=data)

    @classmethod
    def upload(cls, host: np.ndarray, dtype: int, rows: int, cols: int, block_size: int = 32) -> "Weight":
        host = np.ascontiguousarray(host, dtype=np.uint8)
        d = qraf_weight_t()
        check(_get_lib().qraf_cuda_weight_upload(host.ctypes.data_as(C.c_void_p), host.nbytes, dtype, block_size, rows,
                                          cols, C.byref(d)))
        return cls(d)

    def shard(self, world: int, rank: int) -> "Weight":
        d = qraf_weight_t()
        check(_get_lib().qraf_cuda_weight_shard(C.byref(self.desc), world, rank, C.byref(d)))
        return Weight(d, keepalive=self)

    @property
    def rows(self) -> int:
        return self.desc.rows

    @property
    def cols(self) -> int:
        return self.desc.cols

    @property
    def dtype(self) -> int:
        return self.desc.dtype

    @property
    def nbytes(self) -> int:
        return self.desc.bytes

    def free(self) -> None:
        if self.desc.owned:
            check(_get_lib().qraf_cuda_weight_free(C.byref(self.desc)))

    def __del__(self):
        try:
            if self.desc.owned and self.desc.data:
                _get_lib().qraf_cuda_weight_free(C.byref(self.desc))
        except Exception:
            pass


class DeviceModel:
    """A .qraf file with its Q8_0 / Q4_0 tensors resident on the current device
    (qraf_cuda_model_open: one allocation, the file's bytes unchanged)."""

    def __init__(self, path: str, f32: bool = False):
        h = C.c_void_p()
        check(_get_lib().qraf_cuda_model_open_ex(os.fsencode(path), MODEL_F32 if f32 else 0, C.byref(h)))
        self._h = h

    def tensor_f32(self, name: str):
        """(device address, element count) of an F32 tensor (a model opened with f32=True)."""
        p, n = C.c_void_p(), C.c_uint64()
        check(_get_lib().qraf_cuda_model_tensor_f32(self._h, name.encode(), C.byref(p), C.byref(n)))
        return p.value, n.value

    @property
    def names(self) -> list:
        """Quantized tensors in directory order."""
        lib, out = _get_lib(), []
        while True:
            n = lib.qraf_cuda_model_weight_name(self._h, len(out))
            if n is None:
                return out
            out.append(n.decode())

    def info(self) -> dict:
        n, b, d = C.c_uint32(), C.c_uint64(), C.c_int()
        check(_get_lib().qraf_cuda_model_info(self._h, C.byref(n), C.byref(b), C.byref(d)))
        return {"num_weights": n.value, "device_bytes": b.value, "device": d.value}

    def weight(self, name: str) -> Weight:
        d = qraf_weight_t()
        check(_get_lib().qraf_cuda_model_weight(self._h, name.encode(), C.byref(d)))
        return Weight(d, keepalive=self)

    def config_u32(self, key: str) -> int:
        """Raw bits of a u32 / f32 config entry."""
        v = C.c_uint32()
        check(_get_lib().qraf_cuda_model_config_u32(self._h, key.encode(), C.byref(v)))
        return v.value

    def close(self) -> None:
        if self._h:
            h, self._h = self._h, C.c_void_p()
            check(_get_lib().qraf_cuda_model_close(h))

    def __del__(self):
        try:
            if self._h:
                _get_lib().qraf_cuda_model_close(self._h)
        except Exception:
            pass


def launch_count() -> int:
    """Kernels the library has launched in this process (a captured launch counts once)."""
    return int(_get_lib().qraf_cuda_launch_count())


class Decoder:
    """A Llama / Qwen2 decode engine over a .qraf file (qraf_cuda_decoder_*):
    step() runs one decode step for M slots at once, each with its own KV cache."""

    def __init__(self, path: str, max_slots: int = 1, max_seq: int = 2048, kv_int8: bool = False):
        h = C.c_void_p()
        check(_get_lib().qraf_cuda_decoder_open_ex(os.fsencode(path), max_slots, max_seq,
                                                   DECODER_KV_INT8 if kv_int8 else 0, C.byref(h)))
        self.kv_int8 = kv_int8
        self._h = h
        v, hd, l, ms, mq = (C.c_uint32() for _ in range(5))
        check(_get_lib().qraf_cuda_decoder_info(h, C.byref(v), C.byref(hd), C.byref(l), C.byref(ms), C.byref(mq)))
        self.vocab, self.hidden, self.layers = v.value, hd.value, l.value
        self.max_slots, self.max_seq = ms.value, mq.value

    def step(self, tokens, positions, slots, mode: int = MODE_AUTO, logits=None, stream=None):
        """tokens, positions, slots: contiguous CUDA int32 tensors of M; returns logits [M, vocab]."""
        torch = _torch()
        m = tokens.numel()
        for t in (tokens, positions, slots):
            if t.dtype != torch.int32 or not t.is_cuda or not t.is_contiguous() or t.numel() != m:
                raise ValueError("tokens, positions and slots must be contiguous CUDA int32 tensors of one length")
        if logits is None:
            logits = torch.empty((m, self.vocab), dtype=torch.float32, device=tokens.device)
        check(_get_lib().qraf_cuda_decoder_step(self._h, m, C.c_void_p(tokens.data_ptr()),
                                                C.c_void_p(positions.data_ptr()), C.c_void_p(slots.data_ptr()),
                                                C.c_void_p(logits.data_ptr()), mode, _stream(stream)))
        return logits

    def kv_read(self, slot: int, layer: int, pos: int, kv_heads: int, head_dim: int):
        """One cache row: (k, v) float32 [kv_heads * head_dim], or with the int8 cache
        (k codes, v codes, k scales, v scales)."""
        n = kv_heads * head_dim
        if self.kv_int8:
            k, v = np.empty(n, np.int8), np.empty(n, np.int8)
            ks, vs = np.empty(kv_heads, np.float32), np.empty(kv_heads, np.float32)
            check(_get_lib().qraf_cuda_decoder_kv_read(self._h, slot, layer, pos, k.ctypes.data, v.ctypes.data,
                                                       ks.ctypes.data_as(C.POINTER(C.c_float)),
                                                       vs.ctypes.data_as(C.POINTER(C.c_float))))
            return k, v, ks, vs
        k, v = np.empty(n, np.float32), np.empty(n, np.float32)
        check(_get_lib().qraf_cuda_decoder_kv_read(self._h, slot, layer, pos, k.ctypes.data, v.ctypes.data, None, None))
        return k, v

    def close(self) -> None:
        if self._h:
            h, self._h = self._h, C.c_void_p()
            check(_get_lib().qraf_cuda_decoder_close(h))

    def __del__(self):
        try:
            if self._h:
                _get_lib().qraf_cuda_decoder_close(self._h)
        except Exception:
            pass


def host_cache_add(w_host: np.ndarray, dtype: int, rows: int, cols: int, block_size: int = 32) -> None:
    """Preload a host weight into the cache qraf_cuda_matvec_q_host (dispatch_matvec_q) looks up."""
    check(_get_lib().qraf_cuda_host_cache_add(w_host.ctypes.data, w_host.nbytes, dtype, block_size, rows, cols))


def host_cache_info() -> tuple:
    """(entries, device bytes) of that cache."""
    n, b = C.c_uint32(), C.c_uint64()
    check(_get_lib().qraf_cuda_host_cache_info(C.byref(n), C.byref(b)))
    return n.value, b.value


def matvec_q(w: Weight, x, y=None, mode: int = MODE_AUTO, stream=None):
    """Y[m] = dispatch_matvec_q(W, X[m]) on the GPU.  x: CUDA fp32 [M, cols] or [cols]."""
    torch = _torch()
    squeeze = x.dim() == 1
    x2 = x.reshape(1, -1) if squeeze else x
    if x2.dtype != torch.float32 or not x2.is_cuda or not x2.is_contiguous():
        raise ValueError("x must be a contiguous CUDA float32 tensor")
    m = x2.shape[0]
    if x2.shape[1] != w.cols:
        raise ValueError(f"x has {x2.shape[1]} columns, the weight has {w.cols}")
    if y is None:
        y = torch.empty((m, w.rows), dtype=torch.float32, device=x.device)
    check(_get_lib().qraf_cuda_matvec_q(C.byref(w.desc), C.c_void_p(x2.data_ptr()), C.c_void_p(y.data_ptr()), m, mode,
                                 _stream(stream)))
    return y.reshape(w.rows) if squeeze else y


MULTI_MAX_WEIGHTS = 4


def matvec_q_multi(weights, x, ys=None, mode: int = MODE_AUTO, stream=None, norm_w=None, norm_eps: float = 1e-6,
                   biases=None):
    """[W_i X for each weight] in one launch (qraf_cuda_matvec_q_multi): projections of
    the same activations, e.g. a layer's Q, K and V, or gate and up.  Returns the list
    of outputs ([M, rows_i] each, or [rows_i] for a 1-D x).  norm_w: RMSNorm of x
    first; biases: per-weight bias tensors (or None entries) added to the outputs
    (qraf_cuda_matvec_q_multi_ex)."""
    torch = _torch()
    if not 1 <= len(weights) <= MULTI_MAX_WEIGHTS:
        raise ValueError(f"1 to {MULTI_MAX_WEIGHTS} weights")
    squeeze = x.dim() == 1
    x2 = x.reshape(1, -1) if squeeze else x
    if x2.dtype != torch.float32 or not x2.is_cuda or not x2.is_contiguous():
        raise ValueError("x must be a contiguous CUDA float32 tensor")
    m = x2.shape[0]
    if ys is None:
        ys = [torch.empty((m, w.rows), dtype=torch.float32, device=x.device) for w in weights]
    descs = (qraf_weight_t * len(weights))(*[w.desc for w in weights])
    outs = (C.c_void_p * len(weights))(*[y.data_ptr() for y in ys])
    if norm_w is None and biases is None:
        check(_get_lib().qraf_cuda_matvec_q_multi(descs, len(weights), C.c_void_p(x2.data_ptr()), outs, m, mode,
                                                  _stream(stream)))
    else:
        bs = None
        if biases is not None:
            bs = (C.c_void_p * len(weights))(*[b.data_ptr() if b is not None else None for b in biases])
        check(_get_lib().qraf_cuda_matvec_q_multi_ex(
            descs, len(weights), C.c_void_p(x2.data_ptr()), C.c_void_p(norm_w.data_ptr() if norm_w is not None else 0),
            norm_eps, bs, outs, m, mode, _stream(stream)))
    return [y.reshape(w.rows) for y, w in zip(ys, weights)] if squeeze else ys


def matvec_q_swiglu(gate: Weight, up: Weight, x, h=None, mode: int = MODE_AUTO, stream=None, norm_w=None,
                    norm_eps: float = 1e-6):
    """silu(W_gate X) * (W_up X) (qraf_cuda_matvec_q_swiglu): one launch in FAST / AUTO
    for one or two vectors.  Returns [M, rows] (or [rows] for a 1-D x)."""
    torch = _torch()
    squeeze = x.dim() == 1
    x2 = x.reshape(1, -1) if squeeze else x
    if x2.dtype != torch.float32 or not x2.is_cuda or not x2.is_contiguous():
        raise ValueError("x must be a contiguous CUDA float32 tensor")
    m = x2.shape[0]
    if h is None:
        h = torch.empty((m, gate.rows), dtype=torch.float32, device=x.device)
    if norm_w is None:
        check(_get_lib().qraf_cuda_matvec_q_swiglu(C.byref(gate.desc), C.byref(up.desc), C.c_void_p(x2.data_ptr()),
                                                   C.c_void_p(h.data_ptr()), m, mode, _stream(stream)))
    else:
        check(_get_lib().qraf_cuda_matvec_q_swiglu_ex(C.byref(gate.desc), C.byref(up.desc),
                                                      C.c_void_p(x2.data_ptr()), C.c_void_p(norm_w.data_ptr()),
                                                      norm_eps, C.c_void_p(h.data_ptr()), m, mode, _stream(stream)))
    return h.reshape(gate.rows) if squeeze else h


def dot_q(dtype: int, q, x, count: int, block_size: int = 32, mode: int = MODE_EXACT, stream=None):
    """dot_q8_0_f32 / dot_q4_0_f32 on device buffers; returns a 1-element CUDA tensor."""
    torch = _torch()
    out = torch.empty(1, dtype=torch.float32, device=x.device)
    check(_get_lib().qraf_cuda_dot_q(dtype, C.c_void_p(q.data_ptr()), C.c_void_p(x.data_ptr()), count, block_size,
                              C.c_void_p(out.data_ptr()), mode, _stream(stream)))
    return out


def dot_q8_0_f32(q, x, count: int, block_size: int = 32, mode: int = MODE_EXACT):
    return dot_q(Q8_0, q, x, count, block_size, mode)


def dot_q4_0_f32(q, x, count: int, block_size: int = 32, mode: int = MODE_EXACT):
    return dot_q(Q4_0, q, x, count, block_size, mode)


def block_partials(w: Weight, x, stream=None):
    torch = _torch()
    nb = (w.cols + w.desc.block_size - 1) // w.desc.block_size
    out = torch.empty((w.rows, nb), dtype=torch.float32, device=x.device)
    check(_get_lib().qraf_cuda_block_partials(C.byref(w.desc), C.c_void_p(x.data_ptr()), C.c_void_p(out.data_ptr()),
                                       _stream(stream)))
    return out


def limb_partials(w: Weight, x, stream=None):
    """(D [rows][cols/32][4] int32, c [cols/32] fp32): the FAST kernels' per-block integer partial sums for x."""
    torch = _torch()
    nb = w.cols // 32
    d = torch.empty((w.rows, nb, 4), dtype=torch.int32, device=x.device)
    c = torch.empty(nb, dtype=torch.float32, device=x.device)
    check(_get_lib().qraf_cuda_limb_partials(C.byref(w.desc), C.c_void_p(x.data_ptr()), C.c_void_p(d.data_ptr()),
                                              C.c_void_p(c.data_ptr()), _stream(stream)))
    return d, c


def quantize(dtype: int, x, block_size: int = 32, stream=None):
    """quantize_q8_0 / quantize_q4_0 of a contiguous CUDA fp32 tensor (all elements as one sequence)."""
    torch = _torch()
    n = x.numel()
    out = torch.empty(row_bytes(dtype, n, block_size), dtype=torch.uint8, device=x.device)
    check(_get_lib().qraf_cuda_quantize(dtype, C.c_void_p(x.data_ptr()), n, block_size, C.c_void_p(out.data_ptr()),
                                 _stream(stream)))
    return out


def quantize_q8_0(x, block_size: int = 32):
    return quantize(Q8_0, x, block_size)


def quantize_q4_0(x, block_size: int = 32):
    return quantize(Q4_0, x, block_size)


def quantize_rows(dtype: int, x2d, block_size: int = 32, stream=None):
    """Quantize each row of a [rows, cols] CUDA fp32 tensor; returns uint8 [rows, row_bytes]."""
    torch = _torch()
    rows, cols = x2d.shape
    out = torch.empty((rows, row_bytes(dtype, cols, block_size)), dtype=torch.uint8, device=x2d.device)
    check(_get_lib().qraf_cuda_quantize_rows(dtype, C.c_void_p(x2d.data_ptr()), rows, cols, block_size,
                                      C.c_void_p(out.data_ptr()), _stream(stream)))
    return out


def dequantize(dtype: int, q, count: int, block_size: int = 32, stream=None):
    torch = _torch()
    out = torch.empty(count, dtype=torch.float32, device=q.device)
    check(_get_lib().qraf_cuda_dequantize(dtype, C.c_void_p(q.data_ptr()), count, block_size, C.c_void_p(out.data_ptr()),
                                   _stream(stream)))
    return out


# ── host side: the reference-facing entry ────────────────────────────────
def dispatch_matvec_q(w_data: np.ndarray, w_size: int, w_dtype: int, block_size: int, out_dim: int, in_dim: int,
                      x: np.ndarray, y: np.ndarray, m: int = 1, mode: int = MODE_EXACT) -> None:
    """qraf::dispatch_matvec_q with host buffers (backend.cpp:131-199); y is overwritten."""
    if not (w_data.flags.c_contiguous and x.flags.c_contiguous and y.flags.c_contiguous):
        raise ValueError("host buffers must be C-contiguous")
    # plain integer addresses: a third of the cost of ctypes.data_as per argument
    check(_get_lib().qraf_cuda_matvec_q_host(w_data.ctypes.data, w_size, w_dtype, block_size, out_dim, in_dim,
                                             x.ctypes.data, y.ctypes.data, m, mode))


def host_cache_clear() -> None:
    check(_get_lib().qraf_cuda_host_cache_clear())


# ── row-sharded matvec over several GPUs ─────────────────────────────────
COMM_HANDLE_BYTES = 512
COMM_BUFFERS = 4


class Comm:
    """One rank's buffers for the fused row-sharded matvec (qraf_cuda_comm_*)."""

    def __init__(self, world: int, rank: int, capacity_floats: int):
        h = C.c_void_p()
        check(_get_lib().qraf_cuda_comm_create(world, rank, capacity_floats, C.byref(h)))
        self.h, self.world, self.rank = h, world, rank

    def handle(self) -> bytes:
        buf = C.create_string_buffer(COMM_HANDLE_BYTES)
        check(_get_lib().qraf_cuda_comm_handle(self.h, buf))
        return buf.raw

    def open(self, all_handles: list[bytes]) -> None:
        blob = b"".join(all_handles)
        check(_get_lib().qraf_cuda_comm_open(self.h, C.create_string_buffer(blob, len(blob))))

    @staticmethod
    def open_local(comms: list["Comm"]) -> None:
        arr = (C.c_void_p * len(comms))(*[c.h for c in comms])
        check(_get_lib().qraf_cuda_comm_open_local(arr, len(comms)))

    def matvec_q(self, shard: Weight, total_rows: int, row_offset: int, x, mode: int = MODE_FAST, stream=None):
        """Rows of `shard` into every rank's y; returns this rank's full y ([M, total_rows], a view)."""
        torch = _torch()
        x2 = x.reshape(1, -1) if x.dim() == 1 else x
        m = x2.shape[0]
        yp = C.c_void_p()
        check(_get_lib().qraf_cuda_matvec_q_sharded(self.h, C.byref(shard.desc), total_rows, row_offset,
                                                    C.c_void_p(x2.data_ptr()), m, mode, _stream(stream), C.byref(yp)))
        return _wrap_device_floats(yp.value, m * total_rows, x.device).view(m, total_rows)

    def destroy(self) -> None:
        if self.h:
            _get_lib().qraf_cuda_comm_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


def _wrap_device_floats(ptr: int, n: int, device):
    """A torch view of n fp32 values at a device address owned by the library."""
    torch = _torch()

    class _Holder:
        __cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3,
                                    "strides": None}

    return torch.as_tensor(_Holder(), device=device)


def make_comm(world: int, rank: int, capacity_floats: int, all_gather_bytes) -> Comm:
    """Create this rank's Comm and open it, exchanging handles with `all_gather_bytes`
    (a callable taking this rank's bytes and returning every rank's, in rank order)."""
    c = Comm(world, rank, capacity_floats)
    handles = all_gather_bytes(c.handle())
    if len(handles) != world or any(len(h) != COMM_HANDLE_BYTES for h in handles):
        raise QrafError(ERR_COMM, "handle exchange returned the wrong number or size of handles")
    c.open(handles)
    return c


def torch_all_gather_bytes(group=None):
    """all_gather_bytes for make_comm over an initialised torch.distributed group."""
    import torch.distributed as dist

    def gather(b: bytes) -> list[bytes]:
        out = [None] * dist.get_world_size(group)
        dist.all_gather_object(out, b, group=group)
        return out

    return gather
