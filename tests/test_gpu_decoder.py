"""The device decode engine (qraf_cuda_decoder_*) against the reference's own
Transformer::forward_llama (src/nn/transformer.cpp:573-620), both reading the
same quantized .qraf file: logits token by token for one slot in EXACT and FAST,
sequences long enough that attention splits over several chunks and merges them,
and several slots stepping together (continuous batching, each slot with its own
sequence, position and KV cache) against one reference run per sequence.

RoPE, softmax and SiLU call CUDA's powf / sinf / cosf / expf where the reference
calls the C library's, and the attention sums run in another order, so the bar
is closeness (1e-4 relative plus 1e-4 of the largest logit) and the same argmax,
not identical bits."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import qraf_b200 as qb
import qraf_spec
from qraf_b200 import qraf_file as qf

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not oracle.reference_available(), reason="oracle/_ref not built")]


def _close(got, want, label):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    tol = 1e-4 * np.abs(want) + 1e-4 * np.abs(want).max()
    bad = np.abs(got - want) > tol
    assert not bad.any(), f"{label}: {int(bad.sum())} logits off, worst {np.abs(got - want).max():.3g}"
    assert int(np.argmax(got)) == int(np.argmax(want)), f"{label}: argmax differs"


def _model(tmp_path, oracle_lib, arch, dt, tied=False, **kw):
    spec = qraf_spec.tiny_decoder(arch, dt, **kw)
    if tied:
        spec["tensors"] = [t for t in spec["tensors"] if t[0] != "lm_head.weight"]
    w = qf.QrafFileWriter()
    qraf_spec.write_with(w, spec, oracle_lib.quantize_rows)
    path = str(tmp_path / f"{arch}_{dt}_{int(tied)}.qraf")
    w.write(path)
    return path, dict(spec["config"])["vocab_size"]


def _i32(vals, cuda):
    import torch

    return torch.tensor(vals, dtype=torch.int32, device=cuda)


def _reference_runs(path, vocab, seqs):
    ref = oracle.RefTransformer(oracle.Reference(), path, vocab)
    out = []
    for s in seqs:
        ref.reset()
        out.append([ref.forward(t, p) for p, t in enumerate(s)])
    ref.close()
    return out


@pytest.mark.parametrize("arch,dt,tied", [("qwen2", qb.Q8_0, False), ("llama", qb.Q4_0, False),
                                          ("llama", qb.Q8_0, True)])
def test_one_slot_matches_the_reference_forward(tmp_path, cuda, oracle_lib, arch, dt, tied):
    path, vocab = _model(tmp_path, oracle_lib, arch, dt, tied)
    tokens = [5, 17, 300, 5, 511, 0, 42, 42]
    want = _reference_runs(path, vocab, [tokens])[0]
    for mode in (qb.MODE_EXACT, qb.MODE_FAST):
        dec = qb.Decoder(path, max_slots=2, max_seq=64)
        for p, t in enumerate(tokens):
            got = dec.step(_i32([t], cuda), _i32([p], cuda), _i32([1], cuda), mode=mode).cpu().numpy()[0]
            _close(got, want[p], f"{arch} dtype {dt} tied={tied} mode {mode} position {p}")
        dec.close()
    assert qb.device_status() == qb.OK


@pytest.mark.parametrize("max_seq,n", [(160, 150), (1024, 600), (2200, 1100)])
def test_long_sequence_splits_attention(tmp_path, cuda, oracle_lib, max_seq, n):
    """From position 32 on, a slot's attention runs over several chunks (one CTA
    per 32 positions of max_seq, at most 64) whose partials the last CTA merges;
    with few CTAs per chunk count a chunk spans several 32-position tiles, and past
    1024 positions more than 32 chunks meet in the merge (lanes take several
    chunks each).  GQA with 4 query heads per KV head."""
    path, vocab = _model(tmp_path, oracle_lib, "qwen2", qb.Q8_0, heads=8, kv_heads=2, max_seq=max_seq)
    rng = np.random.default_rng(3)
    tokens = [int(t) for t in rng.integers(0, vocab, n)]
    want = _reference_runs(path, vocab, [tokens])[0]
    dec = qb.Decoder(path, max_slots=1, max_seq=max_seq)
    for p, t in enumerate(tokens):
        got = dec.step(_i32([t], cuda), _i32([p], cuda), _i32([0], cuda), mode=qb.MODE_FAST).cpu().numpy()[0]
        _close(got, want[p], f"max_seq {max_seq} position {p}")
    dec.close()
    assert qb.device_status() == qb.OK


@pytest.mark.parametrize("mode", [qb.MODE_AUTO, qb.MODE_FAST, qb.MODE_TC])
def test_slots_step_together(tmp_path, cuda, oracle_lib, mode):
    """Three sequences in slots 3, 0 and 2 (slot 1 stays empty); the third joins
    forty steps late, so every step mixes positions; each slot's logits follow
    its own reference run."""
    path, vocab = _model(tmp_path, oracle_lib, "qwen2", qb.Q8_0, max_seq=128)
    rng = np.random.default_rng(5)
    seqs = [[int(t) for t in rng.integers(0, vocab, n)] for n in (90, 70, 50)]
    slot_of, start = [3, 0, 2], [0, 0, 40]
    want = _reference_runs(path, vocab, seqs)
    dec = qb.Decoder(path, max_slots=4, max_seq=128)
    for step in range(90):
        active = [(i, step - start[i]) for i in range(3) if 0 <= step - start[i] < len(seqs[i])]
        got = dec.step(_i32([seqs[i][p] for i, p in active], cuda), _i32([p for _, p in active], cuda),
                       _i32([slot_of[i] for i, _ in active], cuda), mode=mode).cpu().numpy()
        for row, (i, p) in enumerate(active):
            _close(got[row], want[i][p], f"mode {mode} step {step} sequence {i} position {p}")
    dec.close()
    assert qb.device_status() == qb.OK


def test_graph_replay_of_a_step(tmp_path, cuda, oracle_lib):
    """A step captured once in a CUDA graph and replayed with new device-side
    tokens and positions gives the reference's logits at each position."""
    import torch

    path, vocab = _model(tmp_path, oracle_lib, "llama", qb.Q4_0, max_seq=64)
    tokens = [9, 8, 7, 6, 5, 4, 3, 2, 1, 0] * 4
    want = _reference_runs(path, vocab, [tokens])[0]
    dec = qb.Decoder(path, max_slots=1, max_seq=64)
    tok, pos, slot = _i32([tokens[0]], cuda), _i32([0], cuda), _i32([0], cuda)
    logits = torch.empty((1, vocab), device=cuda)
    s = torch.cuda.Stream(cuda)
    with torch.cuda.stream(s):
        dec.step(tok, pos, slot, mode=qb.MODE_FAST, logits=logits, stream=s)
    torch.cuda.synchronize()
    _close(logits.cpu().numpy()[0], want[0], "eager position 0")
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        dec.step(tok, pos, slot, mode=qb.MODE_FAST, logits=logits, stream=s)
    for p in range(1, len(tokens)):
        tok.fill_(tokens[p])
        pos.fill_(p)
        g.replay()
        torch.cuda.synchronize()
        _close(logits.cpu().numpy()[0], want[p], f"replay position {p}")
    del g
    dec.close()
    assert qb.device_status() == qb.OK


def test_launch_count_of_a_step(tmp_path, cuda, oracle_lib):
    """qraf_cuda_launch_count sees every kernel of a step: the embedding, per layer
    at least QKV, attention, O, SwiGLU and down, and the LM head; two steps of one
    shape launch the same number."""
    path, _ = _model(tmp_path, oracle_lib, "qwen2", qb.Q8_0)
    dec = qb.Decoder(path, max_slots=2, max_seq=16)
    counts = []
    for p in range(2):
        c0 = qb.launch_count()
        dec.step(_i32([3, 4], cuda), _i32([p, p], cuda), _i32([0, 1], cuda), mode=qb.MODE_FAST)
        counts.append(qb.launch_count() - c0)
    dec.close()
    assert counts[0] == counts[1] >= 2 + 5 * dec.layers


def test_bad_position_raises_the_device_status(tmp_path, cuda, oracle_lib):
    """A position at max_seq is refused on the device (kErrBadLaunch), not written."""
    path, _ = _model(tmp_path, oracle_lib, "qwen2", qb.Q8_0)
    dec = qb.Decoder(path, max_slots=1, max_seq=16)
    dec.step(_i32([1], cuda), _i32([16], cuda), _i32([0], cuda), mode=qb.MODE_FAST)
    assert qb.device_status() == qb.ERR_INVALID
    assert qb.device_status() == qb.OK
    dec.close()


def test_decoder_rejects_a_file_without_the_tensors(tmp_path, cuda):
    w = qf.QrafFileWriter()
    w.set_config_string("architecture", "llama")
    w.set_config("hidden_size", 64)
    w.set_config("num_layers", 1)
    w.set_config("num_heads", 2)
    w.set_config("intermediate_size", 128)
    w.set_config("vocab_size", 8)
    w.add_tensor("model.embed_tokens.weight", (8, 64), qf.DTYPE_F32, np.zeros((8, 64), np.float32))
    path = str(tmp_path / "bad.qraf")
    w.write(path)
    with pytest.raises(qb.QrafError) as e:
        qb.Decoder(path, 1, 16)
    assert e.value.code == qb.ERR_INVALID and "missing" in str(e.value)


@pytest.mark.parametrize("arch,dt,tied", [("llama", qb.Q4_0, True), ("qwen2", qb.Q8_0, False)])
def test_tensor_core_route(tmp_path, cuda, oracle_lib, arch, dt, tied):
    """Three or more slots under AUTO take the tensor-core route: per layer one
    prep + tile pair for Q/K/V (RMSNorm in the prep, three outputs and biases in
    the store), one for O (residual in the store), one for gate/up, one for down
    (silu(gate) * up formed in the prep, residual in the store), and the attention
    launch; four slots at different positions against the reference."""
    path, vocab = _model(tmp_path, oracle_lib, arch, dt, tied, max_seq=64)
    rng = np.random.default_rng(9)
    seqs = [[int(t) for t in rng.integers(0, vocab, 40)] for _ in range(4)]
    start = [0, 3, 7, 12]
    want = _reference_runs(path, vocab, seqs)
    dec = qb.Decoder(path, max_slots=4, max_seq=64)
    per_layer = None
    for step in range(52):
        active = [(i, step - start[i]) for i in range(4) if 0 <= step - start[i] < len(seqs[i])]
        c0 = qb.launch_count()
        got = dec.step(_i32([seqs[i][p] for i, p in active], cuda), _i32([p for _, p in active], cuda),
                       _i32([i for i, _ in active], cuda),
                       mode=qb.MODE_AUTO).cpu().numpy()
        if len(active) >= 3:
            per_layer = (qb.launch_count() - c0 - 1 - 2) / dec.layers   # embedding; head: two launches
        for row, (i, p) in enumerate(active):
            _close(got[row], want[i][p], f"{arch} tied={tied} step {step} sequence {i} position {p}")
    dec.close()
    assert per_layer == 9
    assert qb.device_status() == qb.OK


def test_int8_cache_holds_the_reference_quantizer_bytes(tmp_path, cuda, oracle_lib):
    """QRAF_DECODER_KV_INT8: the codes and scales the step stores are the reference's
    QuantizedKVCache::store of the row the f32 cache holds (layer 0, where both
    decoders see the same inputs), at every position."""
    path, vocab = _model(tmp_path, oracle_lib, "qwen2", qb.Q8_0, max_seq=64)
    spec = dict(qraf_spec.tiny_decoder("qwen2", qb.Q8_0)["config"])
    kvh, hd = spec["num_kv_heads"], spec["hidden_size"] // spec["num_heads"]
    ref = oracle.Reference()
    f32 = qb.Decoder(path, max_slots=1, max_seq=64)
    i8 = qb.Decoder(path, max_slots=1, max_seq=64, kv_int8=True)
    for p, t in enumerate([3, 9, 27, 81, 243, 217, 139, 1]):
        for dec in (f32, i8):
            dec.step(_i32([t], cuda), _i32([p], cuda), _i32([0], cuda), mode=qb.MODE_FAST)
        k, v = f32.kv_read(0, 0, p, kvh, hd)
        got = i8.kv_read(0, 0, p, kvh, hd)
        want = ref.kv_quantize(k, v, kvh, hd)
        for g, w, name in zip(got, want, ("k codes", "v codes", "k scales", "v scales")):
            assert g.tobytes() == w.tobytes(), f"position {p}: {name} differ"
    f32.close()
    i8.close()
    assert qb.device_status() == qb.OK


@pytest.mark.parametrize("route", ["one slot", "tensor cores"])
def test_int8_cache_decodes_close_to_the_reference(tmp_path, cuda, oracle_lib, route):
    """With the int8 cache the logits stay close to the reference's f32-cache
    forward (the codes carry 1/254 of each row's range): every position's logits
    within 2e-2 of the largest and a cosine above 0.9999 (measured on B200: 6.8e-3, 0.99998); one slot over 150
    positions (split attention), and three slots on the tensor-core route."""
    path, vocab = _model(tmp_path, oracle_lib, "qwen2", qb.Q8_0, heads=8, kv_heads=2, max_seq=160)
    rng = np.random.default_rng(31)
    n_seq, n = (1, 150) if route == "one slot" else (3, 40)
    seqs = [[int(t) for t in rng.integers(0, vocab, n)] for _ in range(n_seq)]
    want = _reference_runs(path, vocab, seqs)
    dec = qb.Decoder(path, max_slots=n_seq, max_seq=160, kv_int8=True)
    worst, low_cos = 0.0, 1.0
    for p in range(n):
        got = dec.step(_i32([s[p] for s in seqs], cuda), _i32([p] * n_seq, cuda), _i32(list(range(n_seq)), cuda),
                       mode=qb.MODE_AUTO).cpu().numpy()
        for i in range(n_seq):
            w = np.asarray(want[i][p], np.float64)
            g = got[i].astype(np.float64)
            worst = max(worst, float(np.abs(g - w).max() / np.abs(w).max()))
            low_cos = min(low_cos, float(g @ w / np.linalg.norm(g) / np.linalg.norm(w)))
    dec.close()
    print(f"int8 cache ({route}): worst |d| / max |logit| {worst:.2e}, lowest cosine {low_cos:.6f}")
    assert worst < 2e-2 and low_cos > 0.9999
    assert qb.device_status() == qb.OK
