"""ctypes bindings for the parity checkers (TEST INFRASTRUCTURE ONLY).

Two libraries live here, both CPU-only:

* ``libqraf_oracle.so`` — the C restatement of the reference's quantized
  matvec path (``qraf_oracle.c``), built by ``make -C oracle``.
* ``_ref/libqraf_ref.so`` — the reference's own sources compiled in place by
  ``make -C oracle ref`` (only where the reference tree exists; the built file
  travels with the repository snapshot).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import this package.  The product (``qraf_b200``) never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "libqraf_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libqraf_ref.so")
# The reference checkout: QRAF_REFERENCE_TREE, else the directory `reference`
# beside this repository (oracle/Makefile uses the same default).
REF_TREE = os.environ.get("QRAF_REFERENCE_TREE",
                          os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))

Q8_0 = 10
Q4_0 = 20

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")


def build(with_ref: bool | None = None) -> None:
    """Compile the restatement, and the reference library when its tree exists."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    if with_ref is None:
        with_ref = os.path.isdir(os.path.join(REF_TREE, "src"))
    if with_ref:
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={REF_TREE}"], check=True)


def block_bytes(dtype: int, bs: int) -> int:
    return 4 + bs if dtype == Q8_0 else 2 + bs // 2


def row_bytes(dtype: int, bs: int, k: int) -> int:
    return (k + bs - 1) // bs * block_bytes(dtype, bs)


class Oracle:
    """The C restatement (qraf_oracle.c)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build(with_ref=False)
        lib = C.CDLL(path)
        lib.qo_fp16_to_fp32.restype = C.c_float
        lib.qo_fp16_to_fp32.argtypes = [C.c_uint16]
        lib.qo_fp32_to_fp16.restype = C.c_uint16
        lib.qo_fp32_to_fp16.argtypes = [C.c_float]
        for q in ("qo_quantize_q8_0", "qo_quantize_q4_0"):
            getattr(lib, q).restype = C.c_size_t
            getattr(lib, q).argtypes = [_f32p, C.c_size_t, C.c_int, _u8p]
        for d in ("qo_dot_q8_0_f32", "qo_dot_q4_0_f32"):
            getattr(lib, d).restype = C.c_float
            getattr(lib, d).argtypes = [_u8p, _f32p, C.c_size_t, C.c_int]
        for d in ("qo_dequantize_block_q8_0", "qo_dequantize_block_q4_0"):
            getattr(lib, d).restype = None
            getattr(lib, d).argtypes = [_u8p, _f32p, C.c_int]
        lib.qo_matvec_q.restype = None
        lib.qo_matvec_q.argtypes = [_u8p, C.c_uint32, C.c_int, C.c_uint32, C.c_uint32, _f32p, _f32p]
        lib.qo_matmul_q.restype = None
        lib.qo_matmul_q.argtypes = [_u8p, C.c_uint32, C.c_int, C.c_uint32, C.c_uint32, C.c_uint32,
                                    _f32p, _f32p]
        lib.qo_block_partials.restype = None
        lib.qo_block_partials.argtypes = [_u8p, C.c_uint32, C.c_int, C.c_uint32, C.c_uint32, _f32p, _f32p]
        lib.qo_matvec_q_f64.restype = None
        lib.qo_matvec_q_f64.argtypes = [_u8p, C.c_uint32, C.c_int, C.c_uint32, C.c_uint32, _f32p, _f64p]
        lib.qo_limb_partials.restype = None
        lib.qo_rms_norm.restype = None
        lib.qo_rms_norm.argtypes = [_f32p, _f32p, C.c_int, C.c_float]
        lib.qo_limb_partials.argtypes = [_u8p, C.c_uint32, C.c_uint32, C.c_uint32, _f32p,
                                         np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS"), _f32p]
        self.lib = lib

    def fp32_to_fp16(self, f: float) -> int:
        return int(self.lib.qo_fp32_to_fp16(f))

    def fp16_to_fp32(self, h: int) -> float:
        return float(self.lib.qo_fp16_to_fp32(h))

    def quantize(self, dtype: int, data: np.ndarray, bs: int = 32) -> np.ndarray:
        data = np.ascontiguousarray(data, dtype=np.float32).ravel()
        out = np.zeros(row_bytes(dtype, bs, data.size), dtype=np.uint8)
        fn = self.lib.qo_quantize_q8_0 if dtype == Q8_0 else self.lib.qo_quantize_q4_0
        n = fn(data, data.size, bs, out)
        assert n == out.size
        return out

    def quantize_rows(self, dtype: int, w: np.ndarray, bs: int = 32) -> np.ndarray:
        """Per-row quantization of a [N][K] weight (the layout the matvec reads)."""
        w = np.ascontiguousarray(w, dtype=np.float32)
        n, k = w.shape
        rb = row_bytes(dtype, bs, k)
        out = np.zeros((n, rb), dtype=np.uint8)
        for r in range(n):
            out[r] = self.quantize(dtype, w[r], bs)
        return out

    def dot(self, dtype: int, q: np.ndarray, x: np.ndarray, count: int, bs: int = 32) -> float:
        fn = self.lib.qo_dot_q8_0_f32 if dtype == Q8_0 else self.lib.qo_dot_q4_0_f32
        return float(fn(np.ascontiguousarray(q, dtype=np.uint8).ravel(),
                        np.ascontiguousarray(x, dtype=np.float32).ravel(), count, bs))

    def dequantize_block(self, dtype: int, q: np.ndarray, bs: int) -> np.ndarray:
        out = np.zeros(bs, dtype=np.float32)
        fn = self.lib.qo_dequantize_block_q8_0 if dtype == Q8_0 else self.lib.qo_dequantize_block_q4_0
        fn(np.ascontiguousarray(q, dtype=np.uint8).ravel(), out, bs)
        return out

    def matvec(self, dtype: int, w: np.ndarray, n: int, k: int, x: np.ndarray, bs: int = 32) -> np.ndarray:
        y = np.zeros(n, dtype=np.float32)
        self.lib.qo_matvec_q(np.ascontiguousarray(w, dtype=np.uint8).ravel(), dtype, bs, n, k,
                             np.ascontiguousarray(x, dtype=np.float32).ravel(), y)
        return y

    def matmul(self, dtype: int, w: np.ndarray, n: int, k: int, x: np.ndarray, bs: int = 32) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        m = x.size // k
        y = np.zeros((m, n), dtype=np.float32)
        self.lib.qo_matmul_q(np.ascontiguousarray(w, dtype=np.uint8).ravel(), dtype, bs, n, k, m,
                             x.ravel(), y.ravel())
        return y

    def block_partials(self, dtype: int, w: np.ndarray, n: int, k: int, x: np.ndarray, bs: int = 32):
        nb = (k + bs - 1) // bs
        p = np.zeros((n, nb), dtype=np.float32)
        self.lib.qo_block_partials(np.ascontiguousarray(w, dtype=np.uint8).ravel(), dtype, bs, n, k,
                                   np.ascontiguousarray(x, dtype=np.float32).ravel(), p.ravel())
        return p

    def limb_partials(self, dtype: int, w: np.ndarray, n: int, k: int, x: np.ndarray):
        """(D [n][k/32][4] int32, c [k/32] float32): the FAST kernels' per-block integer partial sums."""
        nb = k // 32
        d = np.zeros((n, nb, 4), dtype=np.int32)
        c = np.zeros(nb, dtype=np.float32)
        self.lib.qo_limb_partials(np.ascontiguousarray(w, dtype=np.uint8).ravel(), dtype, n, k,
                                  np.ascontiguousarray(x, dtype=np.float32).ravel(), d.reshape(-1), c)
        return d, c

    def rms_norm(self, x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
        out = np.array(x, dtype=np.float32, copy=True).ravel()
        self.lib.qo_rms_norm(out, np.ascontiguousarray(w, dtype=np.float32).ravel(), out.size, eps)
        return out

    def matvec_f64(self, dtype: int, w: np.ndarray, n: int, k: int, x: np.ndarray, bs: int = 32):
        y = np.zeros(n, dtype=np.float64)
        self.lib.qo_matvec_q_f64(np.ascontiguousarray(w, dtype=np.uint8).ravel(), dtype, bs, n, k,
                                 np.ascontiguousarray(x, dtype=np.float32).ravel(), y)
        return y


class Reference:
    """The reference's own compiled code (oracle/_ref/libqraf_ref.so)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle ref` where the reference tree exists")
        lib = C.CDLL(path)
        lib.qref_quantize.restype = C.c_size_t
        lib.qref_quantize.argtypes = [C.c_uint32, _f32p, C.c_size_t, C.c_int, _u8p]
        lib.qref_dot.restype = C.c_float
        lib.qref_dot.argtypes = [C.c_uint32, _u8p, _f32p, C.c_size_t, C.c_int]
        lib.qref_dequantize_block.restype = None
        lib.qref_dequantize_block.argtypes = [C.c_uint32, _u8p, _f32p, C.c_int]
        lib.qref_dispatch_matvec_q.restype = None
        lib.qref_dispatch_matvec_q.argtypes = [_u8p, C.c_uint64, C.c_uint32, C.c_int, C.c_uint32,
                                               C.c_uint32, _f32p, _f32p]
        lib.qref_ops_matvec_quantized.restype = None
        lib.qref_ops_matvec_quantized.argtypes = lib.qref_dispatch_matvec_q.argtypes
        lib.qref_matvec_q_threaded.restype = None
        lib.qref_matvec_q_threaded.argtypes = [_u8p, C.c_uint32, C.c_int, C.c_uint32, C.c_uint32,
                                               _f32p, _f32p, C.c_int]
        lib.qref_fp32_to_fp16.restype = C.c_uint16
        lib.qref_fp32_to_fp16.argtypes = [C.c_float]
        lib.qref_fp16_to_fp32.restype = C.c_float
        lib.qref_fp16_to_fp32.argtypes = [C.c_uint16]
        lib.qref_fill_normal.restype = None
        lib.qref_fill_normal.argtypes = [C.c_uint32, C.c_float, C.c_float, _f32p, C.c_size_t]
        lib.qref_rms_norm.restype = None
        lib.qref_rms_norm.argtypes = [_f32p, _f32p, C.c_int, C.c_float]
        vp, cp = C.c_void_p, C.c_char_p
        for name, res, args in (
                ("qref_writer_new", vp, []), ("qref_writer_free", None, [vp]),
                ("qref_writer_config_u32", None, [vp, cp, C.c_uint32]),
                ("qref_writer_config_f32", None, [vp, cp, C.c_float]),
                ("qref_writer_config_string", None, [vp, cp, cp]),
                ("qref_writer_quant_scheme", C.c_uint32, [vp, C.c_uint32, C.c_uint32, C.c_uint32]),
                ("qref_writer_tensor", None, [vp, cp, C.c_uint32, C.POINTER(C.c_uint32), C.c_uint32, vp,
                                              C.c_uint64, C.c_uint32]),
                ("qref_writer_vocab", None, [vp, C.POINTER(cp), _f32p, C.c_uint32]),
                ("qref_writer_merges", None, [vp, C.POINTER(C.c_uint32), _f32p, C.c_uint32]),
                ("qref_writer_special", None, [vp, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]),
                ("qref_writer_write", C.c_int, [vp, cp]),
                ("qref_model_open", vp, [cp]), ("qref_model_close", None, [vp]),
                ("qref_model_tensor", C.c_int, [vp, cp, C.POINTER(vp), C.POINTER(C.c_uint64),
                                                C.POINTER(C.c_uint32), C.POINTER(C.c_uint32),
                                                C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]),
                ("qref_model_hidden_size", C.c_uint32, [vp]),
                ("qref_transformer_open", vp, [cp]), ("qref_transformer_close", None, [vp]),
                ("qref_transformer_reset", None, [vp]),
                ("qref_transformer_forward", C.c_int, [vp, C.c_uint32, C.c_int, _f32p, C.c_uint32]),
                ("qref_kvq_store", None, [_f32p, _f32p, C.c_int, C.c_int, vp, vp, _f32p, _f32p])):
            fn = getattr(lib, name)
            fn.restype, fn.argtypes = res, args
        self.lib = lib

    def kv_quantize(self, k: np.ndarray, v: np.ndarray, kv_heads: int, head_dim: int):
        """QuantizedKVCache::store of one K/V row: (k codes, v codes, k scales, v scales)."""
        n = kv_heads * head_dim
        kq, vq = np.empty(n, np.int8), np.empty(n, np.int8)
        ks, vs = np.empty(kv_heads, np.float32), np.empty(kv_heads, np.float32)
        self.lib.qref_kvq_store(np.ascontiguousarray(k, np.float32), np.ascontiguousarray(v, np.float32), kv_heads,
                                head_dim, kq.ctypes.data, vq.ctypes.data, ks, vs)
        return kq, vq, ks, vs

    def fill_normal(self, seed: int, mean: float, std: float, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        self.lib.qref_fill_normal(seed, mean, std, out, n)
        return out

    def quantize(self, dtype: int, data: np.ndarray, bs: int = 32) -> np.ndarray:
        data = np.ascontiguousarray(data, dtype=np.float32).ravel()
        out = np.zeros(row_bytes(dtype, bs, data.size), dtype=np.uint8)
        n = self.lib.qref_quantize(dtype, data, data.size, bs, out)
        assert n == out.size
        return out

    def quantize_rows(self, dtype: int, w: np.ndarray, bs: int = 32) -> np.ndarray:
        w = np.ascontiguousarray(w, dtype=np.float32)
        n, k = w.shape
        out = np.zeros((n, row_bytes(dtype, bs, k)), dtype=np.uint8)
        for r in range(n):
            out[r] = self.quantize(dtype, w[r], bs)
        return out

    def dot(self, dtype: int, q: np.ndarray, x: np.ndarray, count: int, bs: int = 32) -> float:
        return float(self.lib.qref_dot(dtype, np.ascontiguousarray(q, dtype=np.uint8).ravel(),
                                       np.ascontiguousarray(x, dtype=np.float32).ravel(), count, bs))

    def dequantize_block(self, dtype: int, q: np.ndarray, bs: int) -> np.ndarray:
        out = np.zeros(bs, dtype=np.float32)
        self.lib.qref_dequantize_block(dtype, np.ascontiguousarray(q, dtype=np.uint8).ravel(), out, bs)
        return out

    def matvec(self, dtype: int, w: np.ndarray, n: int, k: int, x: np.ndarray, bs: int = 32,
               threads: int = 1) -> np.ndarray:
        y = np.zeros(n, dtype=np.float32)
        wb = np.ascontiguousarray(w, dtype=np.uint8).ravel()
        xb = np.ascontiguousarray(x, dtype=np.float32).ravel()
        if threads > 1:
            self.lib.qref_matvec_q_threaded(wb, dtype, bs, n, k, xb, y, threads)
        else:
            self.lib.qref_dispatch_matvec_q(wb, wb.size, dtype, bs, n, k, xb, y)
        return y

    def ops_matvec(self, dtype: int, w: np.ndarray, n: int, k: int, x: np.ndarray, bs: int = 32):
        y = np.zeros(n, dtype=np.float32)
        wb = np.ascontiguousarray(w, dtype=np.uint8).ravel()
        self.lib.qref_ops_matvec_quantized(wb, wb.size, dtype, bs, n, k,
                                           np.ascontiguousarray(x, dtype=np.float32).ravel(), y)
        return y


    def rms_norm(self, x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
        out = np.array(x, dtype=np.float32, copy=True).ravel()
        self.lib.qref_rms_norm(out, np.ascontiguousarray(w, dtype=np.float32).ravel(), out.size, eps)
        return out

    def write_qraf(self, path: str, config=(), tensors=(), schemes=(), vocab=None, merges=(), special=None) -> None:
        """The reference's QrafWriter (src/qraf/writer.cpp): config = [(key, value)]
        with int -> u32, float -> f32, str -> string; schemes = [(dtype, block_size,
        group_size)] added in order; tensors = [(name, shape, dtype, bytes, quant_id)];
        vocab = (tokens, scores); merges = [(a, b, result, priority)];
        special = (bos, eos, pad, unk)."""
        lib = self.lib
        h = lib.qref_writer_new()
        try:
            for key, v in config:
                if isinstance(v, str):
                    lib.qref_writer_config_string(h, key.encode(), v.encode())
                elif isinstance(v, (int, np.integer)):
                    lib.qref_writer_config_u32(h, key.encode(), int(v))
                else:
                    lib.qref_writer_config_f32(h, key.encode(), float(v))
            for dt, bs, gs in schemes:
                lib.qref_writer_quant_scheme(h, dt, bs, gs)
            for name, shape, dt, data, qid in tensors:
                raw = np.ascontiguousarray(np.frombuffer(bytes(data), dtype=np.uint8))
                sh = (C.c_uint32 * len(shape))(*shape)
                lib.qref_writer_tensor(h, name.encode(), len(shape), sh, dt, raw.ctypes.data, raw.size, qid)
            if vocab is not None:
                toks, scores = vocab
                arr = (C.c_char_p * len(toks))(*[t.encode() for t in toks])
                sc = np.ascontiguousarray(scores, dtype=np.float32)
                lib.qref_writer_vocab(h, arr, sc, len(toks))
            if merges:
                abr = np.ascontiguousarray([m[:3] for m in merges], dtype=np.uint32).ravel()
                pr = np.ascontiguousarray([m[3] for m in merges], dtype=np.float32)
                lib.qref_writer_merges(h, abr.ctypes.data_as(C.POINTER(C.c_uint32)), pr, len(merges))
            if special is not None:
                lib.qref_writer_special(h, *special)
            if lib.qref_writer_write(h, path.encode()) != 0:
                raise OSError(f"reference writer failed on {path}")
        finally:
            lib.qref_writer_free(h)

    def read_qraf(self, path: str, names) -> dict:
        """Tensors read back by the reference's QrafModel (src/qraf/loader.cpp):
        name -> (dtype, shape, block_size, bytes); plus hidden_size from its config."""
        lib = self.lib
        h = lib.qref_model_open(path.encode())
        if not h:
            raise ValueError(f"reference loader rejected {path}")
        try:
            out = {"hidden_size": lib.qref_model_hidden_size(h)}
            for name in names:
                data, size, dt, nd, bs = C.c_void_p(), C.c_uint64(), C.c_uint32(), C.c_uint32(), C.c_uint32()
                shape = (C.c_uint32 * 8)()
                if lib.qref_model_tensor(h, name.encode(), C.byref(data), C.byref(size), C.byref(dt), C.byref(nd),
                                         shape, C.byref(bs)) != 0:
                    raise KeyError(name)
                out[name] = (dt.value, tuple(shape[:nd.value]), bs.value, C.string_at(data.value, size.value))
            return out
        finally:
            lib.qref_model_close(h)


class RefTransformer:
    """The reference's Transformer over a .qraf file (oracle/_ref,
    src/nn/transformer.cpp): forward(token, pos) -> logits, one request at a time
    with its own KV cache; reset() clears that cache."""

    def __init__(self, ref: "Reference", path: str, vocab: int):
        self.lib, self.vocab = ref.lib, vocab
        self.h = ref.lib.qref_transformer_open(path.encode())
        if not self.h:
            raise ValueError(f"reference Transformer rejected {path}")

    def forward(self, token: int, pos: int) -> np.ndarray:
        out = np.empty(self.vocab, dtype=np.float32)
        if self.lib.qref_transformer_forward(self.h, token, pos, out, self.vocab) != 0:
            raise ValueError("vocab size mismatch")
        return out

    def reset(self) -> None:
        self.lib.qref_transformer_reset(self.h)

    def close(self) -> None:
        if self.h:
            self.lib.qref_transformer_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def reference_available() -> bool:
    return os.path.exists(REF_SO)
