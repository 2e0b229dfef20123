"""The .qraf writer and the model store's file checks, on the CPU.

QrafFileWriter must produce the reference's bytes: against the committed file
the reference's own QrafWriter wrote (tests/golden/make_qraf_golden.py) and,
where oracle/_ref is built, against the live reference writer on seeded random
models, with the reference's loader (QrafModel, src/qraf/loader.cpp) reading
our files back.  qraf_cuda_model_open must reject malformed files before any
device work (header.cpp:8-55, loader.cpp:178-211), which runs without a GPU."""
from __future__ import annotations

import ctypes as C
import os
import struct

import numpy as np
import pytest

import oracle
import qraf_spec
from qraf_b200 import qraf_file as qf

GOLDEN_QRAF = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "llama_like_ref.qraf")
needs_ref = pytest.mark.skipif(not oracle.reference_available(), reason="oracle/_ref not built (no reference tree)")


def _ours(spec, quantize) -> bytes:
    w = qf.QrafFileWriter()
    qraf_spec.write_with(w, spec, quantize)
    return w.to_bytes()


def _meta_offset(raw, name):
    names = list(qf.read_directory_bytes(bytes(raw))["tensors"])
    tdir = struct.unpack_from("<Q", raw, 48)[0]     # QrafHeader::tensor_dir_offset
    return tdir + 80 * names.index(name)


def test_writer_matches_the_reference_golden_file(oracle_lib):
    with open(GOLDEN_QRAF, "rb") as f:
        want = f.read()
    got = _ours(qraf_spec.llama_like(), oracle_lib.quantize_rows)
    assert len(got) == len(want)
    assert got == want, f"first difference at byte {next(i for i in range(len(got)) if got[i] != want[i])}"


def test_read_directory_of_the_golden_file():
    d = qf.read_directory(GOLDEN_QRAF)
    spec = qraf_spec.llama_like()
    assert list(d["tensors"]) == [t[0] for t in spec["tensors"]]
    for name, shape, dt, _, sid in spec["tensors"]:
        e = d["tensors"][name]
        assert e.shape == shape and e.dtype == dt
        assert e.quant_id == (qf.NO_QUANT if sid is None else sid)
        assert e.block_size == (0 if sid is None else spec["schemes"][sid][1])
        assert e.data_offset % qf.DATA_ALIGNMENT == 0
    assert d["file_size"] == os.path.getsize(GOLDEN_QRAF)


def test_fnv1a_sign_extends_like_the_reference():
    # format.h:136-143 widens a signed char, so bytes >= 0x80 enter sign-extended
    assert qf.fnv1a64(b"") == 14695981039346656037
    assert qf.fnv1a64(b"a") == 0xAF63DC4C8601EC8C
    plain = 14695981039346656037
    for b in "é".encode():
        plain = ((plain ^ b) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    assert qf.fnv1a64("é".encode()) != plain
    # the hash the reference's writer stored for the non-ASCII name
    raw = open(GOLDEN_QRAF, "rb").read()
    stored = struct.unpack_from("<Q", raw, _meta_offset(raw, "blk.é.ragged"))[0]
    assert stored == qf.fnv1a64("blk.é.ragged".encode())


@needs_ref
@pytest.mark.parametrize("seed", range(12))
def test_writer_matches_the_live_reference_writer(tmp_path, oracle_lib, seed):
    ref = oracle.Reference()
    spec = qraf_spec.random_spec(seed)
    path = str(tmp_path / "ref.qraf")
    ref.write_qraf(path, **qraf_spec.reference_args(spec, ref.quantize_rows))
    with open(path, "rb") as f:
        want = f.read()
    assert _ours(spec, oracle_lib.quantize_rows) == want


@needs_ref
def test_reference_loader_reads_our_file(tmp_path, oracle_lib):
    spec = qraf_spec.llama_like(seed=11)
    w = qf.QrafFileWriter()
    qraf_spec.write_with(w, spec, oracle_lib.quantize_rows)
    path = str(tmp_path / "ours.qraf")
    w.write(path)
    got = oracle.Reference().read_qraf(path, [t[0] for t in spec["tensors"]])
    assert got["hidden_size"] == 64
    for t in spec["tensors"]:
        name, shape, dt, _, sid = t
        gdt, gshape, gbs, gbytes = got[name]
        assert (gdt, gshape) == (dt, shape)
        assert gbs == (0 if sid is None else spec["schemes"][sid][1])
        assert gbytes == qraf_spec.tensor_bytes(spec, t, oracle_lib.quantize_rows)


def test_to_bytes_is_repeatable():
    w = qf.QrafFileWriter()
    w.set_config("n", 7)
    w.set_config("f", 0.5)
    w.set_config_string("s", "n")          # a value equal to a key shares its string
    w.add_tensor("x", (2,), qf.DTYPE_F32, np.array([1.0, 2.0], np.float32))
    raw = w.to_bytes()
    assert raw == w.to_bytes()
    assert qf.read_directory_bytes(raw)["tensors"]["x"].data_size == 8


# ── qraf_cuda_model_open: malformed files are refused before any device work ──
def _open_rc(path):
    import qraf_b200 as qb

    h = C.c_void_p()
    rc = qb._get_lib().qraf_cuda_model_open(os.fsencode(path), C.byref(h))
    return rc, qb.last_error(), h


def _patched(tmp_path, edit) -> str:
    raw = bytearray(open(GOLDEN_QRAF, "rb").read())
    raw = edit(raw) or raw
    p = tmp_path / "bad.qraf"
    p.write_bytes(bytes(raw))
    return str(p)


@pytest.mark.parametrize("case,edit,words", [
    ("truncated", lambda r: r[:-64], "header says"),
    ("bad magic", lambda r: r.__setitem__(slice(0, 4), b"GGUF"), "magic"),
    ("version 2", lambda r: r.__setitem__(slice(4, 8), struct.pack("<I", 2)), "version"),
    ("tensor past the end", lambda r: struct.pack_into("<Q", r, _meta_offset(r, "lm_head.weight") + 56, len(r)),
     "past the end"),
    ("quantized bytes short of the shape", lambda r: struct.pack_into(
        "<Q", r, _meta_offset(r, "model.layers.0.self_attn.q_proj.weight") + 64, 100), "q_proj"),
    ("name outside the string table", lambda r: struct.pack_into(
        "<I", r, _meta_offset(r, "model.norm.weight") + 8, 1 << 30), "no name"),
    ("directory size", lambda r: struct.pack_into("<Q", r, 56, 81), "tensor directory"),
    ("section past the end", lambda r: struct.pack_into("<Q", r, 88, 1 << 40), "section"),
])
def test_model_open_rejects_malformed_files(tmp_path, case, edit, words):
    import qraf_b200 as qb

    rc, msg, h = _open_rc(_patched(tmp_path, edit))
    assert rc == qb.ERR_INVALID, (case, rc, msg)
    assert words in msg, (case, msg)
    assert not h.value


def test_model_open_missing_file(tmp_path):
    import qraf_b200 as qb

    rc, msg, _ = _open_rc(str(tmp_path / "absent.qraf"))
    assert rc == qb.ERR_INVALID and "cannot open" in msg


@pytest.mark.skipif(not oracle.reference_available(), reason="oracle/_ref not built")
@pytest.mark.parametrize("arch,dt", [("qwen2", qraf_spec.Q8), ("llama", qraf_spec.Q4)])
def test_reference_transformer_runs_our_quantized_file(tmp_path, oracle_lib, arch, dt):
    """A decoder written by QrafFileWriter loads in the reference's own
    Transformer (the decode engine's oracle) and decodes: finite logits that
    follow the token and position, and reset() restarts the sequence."""
    spec = qraf_spec.tiny_decoder(arch, dt)
    w = qf.QrafFileWriter()
    qraf_spec.write_with(w, spec, oracle_lib.quantize_rows)
    path = str(tmp_path / "dec.qraf")
    w.write(path)
    vocab = dict(spec["config"])["vocab_size"]
    ref = oracle.RefTransformer(oracle.Reference(), path, vocab)
    a0 = ref.forward(5, 0)
    a1 = ref.forward(17, 1)
    ref.reset()
    b0 = ref.forward(5, 0)
    ref.close()
    assert np.isfinite(a0).all() and np.isfinite(a1).all()
    assert np.array_equal(a0, b0)
    assert not np.array_equal(a0, a1)


def test_write_streams_the_same_bytes(tmp_path, oracle_lib):
    """write() puts the sections and the padding down one after another; the
    file is to_bytes() exactly, for the spec the reference's writer is pinned on."""
    spec = qraf_spec.llama_like()
    w = qf.QrafFileWriter()
    qraf_spec.write_with(w, spec, oracle_lib.quantize_rows)
    path = str(tmp_path / "s.qraf")
    assert w.write(path) == len(w.to_bytes())
    with open(path, "rb") as f:
        assert f.read() == w.to_bytes()
