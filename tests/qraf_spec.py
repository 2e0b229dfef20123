"""Small synthetic .qraf models, described writer-independently so the same model
can be written by the reference's QrafWriter (through oracle/_ref) and by
qraf_b200.qraf_file.QrafFileWriter and the two files compared byte for byte.

A spec is a dict: config [(key, value)] in insertion order (int -> u32, float ->
f32, str -> string), schemes [(dtype, block_size, group_size)], tensors
[(name, shape, dtype, fp32 values, scheme id or None for F32)], vocab (tokens,
scores) or None, merges [(a, b, result, priority)], special (bos, eos, pad, unk)
or None.  quantize(dtype, w2d, bs) -> native bytes is supplied by the caller
(the oracle in the tests, the reference in the fixture script)."""
from __future__ import annotations

import numpy as np

F32, Q8, Q4 = 0, 10, 20
NO_QUANT = 0xFFFFFFFF


def llama_like(seed: int = 7) -> dict:
    """One Llama-style layer with Q8_0 attention, Q4_0 MLP, a block-64 Q8_0 LM
    head, a ragged-K tensor with a non-ASCII name and a 3-D quantized tensor."""
    rng = np.random.default_rng(seed)
    h, inter, vocab = 64, 96, 12

    def w(*shape):
        return rng.normal(0.0, 0.02, size=shape).astype(np.float32)

    lay = "model.layers.0."
    tensors = [
        ("model.embed_tokens.weight", (vocab, h), F32, w(vocab, h), None),
        (lay + "input_layernorm.weight", (h,), F32, np.ones(h, np.float32), None),
        (lay + "self_attn.q_proj.weight", (h, h), Q8, w(h, h), 0),
        (lay + "self_attn.k_proj.weight", (32, h), Q8, w(32, h), 0),
        (lay + "self_attn.v_proj.weight", (32, h), Q8, w(32, h), 0),
        (lay + "self_attn.o_proj.weight", (h, h), Q8, w(h, h), 0),
        (lay + "post_attention_layernorm.weight", (h,), F32, np.ones(h, np.float32), None),
        (lay + "mlp.gate_proj.weight", (inter, h), Q4, w(inter, h), 1),
        (lay + "mlp.up_proj.weight", (inter, h), Q4, w(inter, h), 1),
        (lay + "mlp.down_proj.weight", (h, inter), Q4, w(h, inter), 1),
        ("model.norm.weight", (h,), F32, np.ones(h, np.float32), None),
        ("lm_head.weight", (vocab, h), Q8, w(vocab, h), 2),
        ("blk.é.ragged", (5, 70), Q8, w(5, 70), 0),
        ("extra.stacked.weight", (2, 3, h), Q4, w(2, 3, h), 1),
    ]
    return {
        "config": [("architecture", "llama"), ("vocab_size", vocab), ("hidden_size", h), ("num_layers", 1),
                   ("num_heads", 4), ("num_kv_heads", 2), ("intermediate_size", inter), ("max_seq_len", 128),
                   ("rope_theta", 10000.0), ("rms_norm_eps", 1e-5), ("source", "synthetic")],
        "schemes": [(Q8, 32, 1), (Q4, 32, 1), (Q8, 64, 1)],
        "tensors": tensors,
        "vocab": (["<unk>", "<s>", "</s>", "a", "b", "ab", "é", "hello", " world", "x", "y", "z"],
                  [0.0, 0.0, 0.0, -1.0, -2.0, -3.0, -4.0, -5.0, -6.0, -7.0, -8.0, -9.0]),
        "merges": [(3, 4, 5, -1.0)],
        "special": (1, 2, 0, 0),
    }


def random_spec(seed: int) -> dict:
    """A random mix of quantized and F32 tensors (shapes, block sizes, names,
    config entries, with or without a tokenizer) for the byte-for-byte writer test."""
    rng = np.random.default_rng(seed)
    schemes = []
    for _ in range(int(rng.integers(1, 4))):
        schemes.append((int(rng.choice([Q8, Q4])), int(rng.choice([16, 32, 64])), int(rng.integers(1, 3))))
    tensors = []
    for t in range(int(rng.integers(1, 9))):
        name = f"t{t}." + "".join(rng.choice(list("abcxyz._0123456789"), size=int(rng.integers(1, 12))))
        if rng.random() < 0.3:
            shape = tuple(int(s) for s in rng.integers(1, 9, size=int(rng.integers(1, 4))))
            tensors.append((name, shape, F32, rng.normal(size=shape).astype(np.float32), None))
        else:
            sid = int(rng.integers(0, len(schemes)))
            dt, bs, _ = schemes[sid]
            rows, cols = int(rng.integers(1, 9)), int(rng.integers(1, 4 * bs))
            if dt == Q4 and cols % 2:
                cols += 1
            tensors.append((name, (rows, cols), dt, rng.normal(0, 0.05, size=(rows, cols)).astype(np.float32), sid))
    config = []
    for c in range(int(rng.integers(0, 6))):
        kind = int(rng.integers(0, 3))
        value = [int(rng.integers(0, 1 << 31)), float(rng.normal()), f"value{c}"][kind]
        config.append((f"key{c}", value))
    spec = {"config": config, "schemes": schemes, "tensors": tensors, "vocab": None, "merges": [], "special": None}
    if rng.random() < 0.5:
        n = int(rng.integers(1, 6))
        spec["vocab"] = ([f"tok{i}" for i in range(n)], [float(-i) for i in range(n)])
        spec["merges"] = [(0, 0, 0, 0.5)]
        spec["special"] = (0, 0, 0, 0)
    return spec


def tiny_decoder(arch: str = "qwen2", dt: int = Q8, seed: int = 11, layers: int = 2, hidden: int = 256, heads: int = 4,
                 kv_heads: int = 2, inter: int = 512, vocab: int = 512, max_seq: int = 64) -> dict:
    """A small random-init Llama / Qwen2 decoder under the tensor names the
    reference's Transformer reads (src/nn/transformer.cpp:96-126, :320-400): F32
    embedding and norms, quantized projections, an explicit quantized LM head,
    and for qwen2 the Q/K/V biases."""
    rng = np.random.default_rng(seed)
    hd = hidden // heads
    q_dim, kv_dim = heads * hd, kv_heads * hd

    def w(*shape, std=0.05):
        return rng.normal(0.0, std, size=shape).astype(np.float32)

    tensors = [("model.embed_tokens.weight", (vocab, hidden), F32, w(vocab, hidden, std=1.0), None)]
    for l in range(layers):
        p = f"model.layers.{l}."
        tensors += [
            (p + "input_layernorm.weight", (hidden,), F32, (1.0 + w(hidden, std=0.1)), None),
            (p + "self_attn.q_proj.weight", (q_dim, hidden), dt, w(q_dim, hidden), 0),
            (p + "self_attn.k_proj.weight", (kv_dim, hidden), dt, w(kv_dim, hidden), 0),
            (p + "self_attn.v_proj.weight", (kv_dim, hidden), dt, w(kv_dim, hidden), 0),
            (p + "self_attn.o_proj.weight", (hidden, q_dim), dt, w(hidden, q_dim), 0),
            (p + "post_attention_layernorm.weight", (hidden,), F32, (1.0 + w(hidden, std=0.1)), None),
            (p + "mlp.gate_proj.weight", (inter, hidden), dt, w(inter, hidden), 0),
            (p + "mlp.up_proj.weight", (inter, hidden), dt, w(inter, hidden), 0),
            (p + "mlp.down_proj.weight", (hidden, inter), dt, w(hidden, inter), 0),
        ]
        if arch == "qwen2":
            tensors += [(p + f"self_attn.{x}_proj.bias", (n,), F32, w(n, std=0.1), None)
                        for x, n in (("q", q_dim), ("k", kv_dim), ("v", kv_dim))]
    tensors += [("model.norm.weight", (hidden,), F32, (1.0 + w(hidden, std=0.1)), None),
                ("lm_head.weight", (vocab, hidden), dt, w(vocab, hidden), 0)]
    return {
        "config": [("architecture", arch), ("vocab_size", vocab), ("hidden_size", hidden), ("num_layers", layers),
                   ("num_heads", heads), ("num_kv_heads", kv_heads), ("intermediate_size", inter),
                   ("max_seq_len", max_seq), ("rope_theta", 10000.0), ("rms_norm_eps", 1e-6)],
        "schemes": [(dt, 32, 1)],
        "tensors": tensors,
        "vocab": None, "merges": [], "special": None,
    }


def tensor_bytes(spec, spec_tensor, quantize) -> bytes:
    """The bytes a tensor of the spec has in the file: fp32 values, or the
    quantizer's native blocks row by row with its scheme's block size."""
    name, shape, dt, values, sid = spec_tensor
    if dt == F32:
        return np.ascontiguousarray(values, np.float32).tobytes()
    bs = spec["schemes"][sid][1]
    return np.ascontiguousarray(quantize(dt, values.reshape(-1, shape[-1]), bs), np.uint8).tobytes()


def write_with(writer, spec, quantize) -> None:
    """Feed a spec to a QrafFileWriter."""
    for key, v in spec["config"]:
        if isinstance(v, str):
            writer.set_config_string(key, v)
        else:
            writer.set_config(key, v)
    for dt, bs, gs in spec["schemes"]:
        writer.add_quant_scheme(dt, bs, gs)
    for t in spec["tensors"]:
        name, shape, dt, _, sid = t
        writer.add_tensor(name, shape, dt, tensor_bytes(spec, t, quantize), NO_QUANT if sid is None else sid)
    if spec["vocab"] is not None:
        writer.set_vocab(*spec["vocab"])
    if spec["merges"]:
        writer.set_merges(spec["merges"])
    if spec["special"] is not None:
        writer.set_special_tokens(*spec["special"])


def reference_args(spec, quantize) -> dict:
    """The same spec as keyword arguments of oracle.Reference.write_qraf."""
    return {
        "config": spec["config"],
        "schemes": spec["schemes"],
        "tensors": [(t[0], t[1], t[2], tensor_bytes(spec, t, quantize), NO_QUANT if t[4] is None else t[4])
                    for t in spec["tensors"]],
        "vocab": spec["vocab"],
        "merges": spec["merges"],
        "special": spec["special"],
    }
