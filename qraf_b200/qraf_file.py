"""Quantized .qraf model files: a writer for Q8_0 / Q4_0 weights and a directory reader.

The reference writes .qraf files with QrafWriter (src/qraf/writer.cpp) and reads
them with QrafModel (src/qraf/loader.cpp) in the layout of include/qraf/format.h;
its converters only write F32 tensors (tools/qraf_convert.py:113-117), so no tool
produces the quantized files its Q8_0 / Q4_0 matvec path consumes.  This writer
produces them: 2-D weights are quantized on the GPU by the byte-exact quantizer
(qraf_cuda_quantize_rows, the same bytes as quantize_q8_0 / quantize_q4_0,
src/tensor/quantize.cpp:105-183), with one QuantScheme per (dtype, block size)
as QrafWriter::add_quant_scheme makes it (src/qraf/writer.cpp:35-47).  The file
layout follows format.h exactly (it is a file format: the reference's loader must
read it), and the string table is filled in the order QrafWriter fills it
(writer.cpp:83-98: config string values when set, then config keys, tensor
names and vocabulary at write time, each string once), so the same inputs give
the same file bytes:

  [QrafHeader 128 B][config block][tokenizer block][tensor directory 80 B each]
  [quant directory 32 B each][string table][tensor data, each 64-B aligned]

sections 8-byte aligned, the data start and every tensor 64-byte aligned, gaps
and the tail zero-filled.  read_directory() parses a file's header and tensor
directory on the host (no GPU)."""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

QRAF_MAGIC = 0x46415251      # "QRAF", little-endian (include/core/types.h:24)
QRAF_VERSION = 1
DATA_ALIGNMENT = 64
NO_QUANT = 0xFFFFFFFF
DTYPE_F32 = 0
DTYPE_Q8_0 = 10
DTYPE_Q4_0 = 20

_HEADER = struct.Struct("<II12QIIII8s")                 # QrafHeader, 128 bytes
_CONFIG_ENTRY = struct.Struct("<III")                   # key_offset, value_type, value
_TENSOR_META = struct.Struct("<QII8IIIQQII")            # TensorMeta, 80 bytes
_QUANT = struct.Struct("<IIIIffII")                     # QuantScheme, 32 bytes
_TOKEN = struct.Struct("<IIfI")
_MERGE = struct.Struct("<IIIf")
_SPECIAL = struct.Struct("<IIII")
assert _HEADER.size == 128 and _TENSOR_META.size == 80 and _QUANT.size == 32


def fnv1a64(data: bytes) -> int:
    """FNV-1a, 64-bit, as format.h's fnv1a_hash (include/qraf/format.h:136-143),
    which widens each signed char to 64 bits: bytes >= 0x80 are sign-extended."""
    h = 14695981039346656037
    for b in data:
        h ^= b if b < 0x80 else (b | 0xFFFFFFFFFFFFFF00)
        h = (h * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def _align(off: int, a: int) -> int:
    return (off + a - 1) // a * a


@dataclass
class _Tensor:
    name: str
    shape: tuple
    dtype: int
    data: bytes
    quant_id: int


@dataclass
class QrafFileWriter:
    """Builds a .qraf file.  Tensors are written in the order they are added."""
    _config: list = field(default_factory=list)          # (key, type, raw u32)
    _quant: list = field(default_factory=list)           # (dtype, block_size, group_size)
    _tensors: list = field(default_factory=list)
    _strings: bytearray = field(default_factory=bytearray)
    _string_off: dict = field(default_factory=dict)
    _vocab: list | None = None
    _scores: list = field(default_factory=list)
    _merges: list = field(default_factory=list)
    _special: tuple = (1, 2, 0, 0)                       # bos, eos, pad, unk (QrafWriter's defaults)

    def _add_string(self, s: str) -> int:
        if s in self._string_off:
            return self._string_off[s]
        off = len(self._strings)
        self._strings += s.encode() + b"\0"
        self._string_off[s] = off
        return off

    # ── config ──
    def set_config(self, key: str, value) -> None:
        """u32 for ints, f32 for floats (QrafWriter::set_config overloads)."""
        if isinstance(value, (bool, int, np.integer)):
            self._config.append((key, 0, int(value) & 0xFFFFFFFF))
        else:
            self._config.append((key, 1, struct.unpack("<I", struct.pack("<f", float(value)))[0]))

    def set_config_string(self, key: str, value: str) -> None:
        self._config.append((key, 2, self._add_string(value)))

    # ── quantization schemes and tensors ──
    def add_quant_scheme(self, dtype: int, block_size: int, group_size: int = 1) -> int:
        self._quant.append((dtype, block_size, group_size))
        return len(self._quant) - 1

    def _scheme(self, dtype: int, block_size: int) -> int:
        for i, (d, b, g) in enumerate(self._quant):
            if d == dtype and b == block_size and g == 1:
                return i
        return self.add_quant_scheme(dtype, block_size)

    def add_tensor(self, name: str, shape, dtype: int, data, quant_id: int = NO_QUANT) -> None:
        """Raw tensor bytes as they go into the file (F32 values, or quantized blocks)."""
        raw = data.tobytes() if hasattr(data, "tobytes") else bytes(data)
        self._tensors.append(_Tensor(name, tuple(int(s) for s in shape), dtype, raw, quant_id))

    def add_quantized(self, name: str, weight, dtype: int, block_size: int = 32, device=None) -> None:
        """A 2-D fp32 weight [rows][cols], quantized on the GPU row by row (the
        reference's Q8_0 / Q4_0 bytes), with the (dtype, block size) scheme."""
        import torch

        from . import quantize_rows

        w = weight if isinstance(weight, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(weight, np.float32))
        if w.dim() != 2:
            raise ValueError("add_quantized takes a 2-D weight")
        dev = device or (w.device if w.is_cuda else torch.device("cuda", torch.cuda.current_device()))
        q = quantize_rows(dtype, w.to(dev, torch.float32).contiguous(), block_size)
        self.add_tensor(name, tuple(w.shape), dtype, q.cpu().numpy(), self._scheme(dtype, block_size))

    # ── tokenizer ──
    def set_vocab(self, tokens, scores=None) -> None:
        self._vocab = list(tokens)
        scores = list(scores or [])
        self._scores = scores + [0.0] * (len(self._vocab) - len(scores))

    def set_merges(self, merges) -> None:
        self._merges = list(merges)

    def set_special_tokens(self, bos: int, eos: int, pad: int = 0, unk: int = 0) -> None:
        self._special = (bos, eos, pad, unk)

    # ── file ──
    def _layout(self):
        """Every section but the tensor data, placed: (file_size, [(offset, bytes)], tensor offsets)."""
        for key, _, _ in self._config:
            self._add_string(key)
        for t in self._tensors:
            self._add_string(t.name)
        if self._vocab is not None:
            for tok in self._vocab:
                self._add_string(tok)

        config = struct.pack("<I", len(self._config)) + b"".join(
            _CONFIG_ENTRY.pack(self._add_string(k), ty, v) for k, ty, v in self._config)
        tok = b""
        if self._vocab is not None:
            tok = struct.pack("<IIII", len(self._vocab), len(self._merges), 4, 0)
            tok += b"".join(_TOKEN.pack(self._add_string(t), len(t.encode()), float(sc), 0)
                            for t, sc in zip(self._vocab, self._scores))
            tok += b"".join(_MERGE.pack(a, b, r, float(p)) for a, b, r, p in self._merges)
            tok += b"".join(_SPECIAL.pack(0, 0, tid, ty) for ty, tid in enumerate(self._special))

        off = _HEADER.size
        config_off, off = off, _align(off + len(config), 8)
        tok_off, off = off, _align(off + len(tok), 8)
        tdir_off = off
        tdir_size = len(self._tensors) * _TENSOR_META.size
        off = _align(off + tdir_size, 8)
        qdir_off = off
        qdir_size = len(self._quant) * _QUANT.size
        off = _align(off + qdir_size, 8)
        str_off = off
        strings = bytes(self._strings)
        off = _align(off + len(strings), DATA_ALIGNMENT)
        data_start = off
        metas, offsets = [], []
        for t in self._tensors:
            shape8 = list(t.shape[:8]) + [0] * (8 - min(8, len(t.shape)))
            metas.append(_TENSOR_META.pack(fnv1a64(t.name.encode()), self._add_string(t.name), len(t.shape), *shape8,
                                           t.dtype, t.quant_id, off, len(t.data), 0, 0))
            offsets.append(off)
            off = _align(off + len(t.data), DATA_ALIGNMENT)
        file_size = off
        header = _HEADER.pack(QRAF_MAGIC, QRAF_VERSION, file_size, config_off, len(config), tok_off, len(tok), tdir_off,
                              tdir_size, qdir_off, qdir_size, str_off, len(strings), data_start, len(self._tensors),
                              len(self._quant), 0, 0, b"\0" * 8)
        quant = b"".join(_QUANT.pack(i, d, b, g, 0.0, 0.0, 1, 0) for i, (d, b, g) in enumerate(self._quant))
        sections = [(0, header), (config_off, config), (tok_off, tok), (tdir_off, b"".join(metas)), (qdir_off, quant),
                    (str_off, strings)]
        return file_size, sections, offsets

    def to_bytes(self) -> bytes:
        file_size, sections, offsets = self._layout()
        out = bytearray(file_size)
        for o, b in sections:
            out[o:o + len(b)] = b
        for t, o in zip(self._tensors, offsets):
            out[o:o + len(t.data)] = t.data
        return bytes(out)

    def write(self, path: str) -> int:
        """The file written section by section (the zero padding between them
        included), without building it in memory first."""
        file_size, sections, offsets = self._layout()
        pieces = sorted(sections + [(o, t.data) for t, o in zip(self._tensors, offsets)], key=lambda p: p[0])
        at = 0
        with open(path, "wb") as f:
            for o, b in pieces:
                if o > at:
                    f.write(b"\0" * (o - at))
                f.write(b)
                at = o + len(b)
            if file_size > at:
                f.write(b"\0" * (file_size - at))
        return file_size


@dataclass
class TensorEntry:
    name: str
    shape: tuple
    dtype: int
    quant_id: int
    block_size: int          # of the tensor's QuantScheme (0 when not quantized)
    data_offset: int
    data_size: int


def read_directory(path: str) -> dict:
    """File size, data offset, quant schemes and the tensor directory (name ->
    TensorEntry, directory order) of a .qraf file."""
    with open(path, "rb") as f:
        return read_directory_bytes(f.read())


def read_directory_bytes(raw: bytes) -> dict:
    h = _HEADER.unpack_from(raw, 0)
    if h[0] != QRAF_MAGIC or h[1] != QRAF_VERSION:
        raise ValueError("not a version-1 .qraf file")
    (_, _, file_size, _, _, _, _, tdir_off, _, qdir_off, _, str_off, str_size, data_off, ntensors, nquant, _, _,
     _) = h
    strings = raw[str_off:str_off + str_size]
    quant = [_QUANT.unpack_from(raw, qdir_off + i * _QUANT.size) for i in range(nquant)]
    tensors = {}
    for i in range(ntensors):
        m = _TENSOR_META.unpack_from(raw, tdir_off + i * _TENSOR_META.size)
        name_off, ndim = m[1], m[2]
        name = strings[name_off:strings.index(b"\0", name_off)].decode()
        qid = m[12]
        bs = quant[qid][2] if qid != NO_QUANT and qid < len(quant) else 0
        tensors[name] = TensorEntry(name, tuple(m[3:3 + ndim]), m[11], qid, bs, m[13], m[14])
    return {"file_size": file_size, "data_offset": data_off, "tensors": tensors, "quant": quant}
