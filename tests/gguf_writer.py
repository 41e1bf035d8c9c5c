"""Writes a decoder model descriptor as a GGUF v3 file, in the layout of the
reference's writer (internal/gguf/writer.go:23-95): header, metadata,
tensor table, padding to 32 bytes, tensor data each starting on a 32-byte
boundary. Test fixture code: the GGUF loader tests write synthetic models
with it, under whisper.cpp or Hugging Face tensor names."""
import ctypes
import struct

import numpy as np

import wgdec

T_U32, T_STR, T_ARR = 4, 8, 9
ROW_BYTES = {0: lambda c: 4 * c, 1: lambda c: 2 * c, 2: lambda c: c // 32 * 18, 3: lambda c: c // 32 * 20,
             6: lambda c: c // 32 * 22, 7: lambda c: c // 32 * 24, 8: lambda c: c // 32 * 34}

HF = {
    "decoder.token_embedding.weight": "model.decoder.embed_tokens.weight",
    "decoder.positional_embedding": "model.decoder.embed_positions.weight",
    "decoder.ln.weight": "model.decoder.layer_norm.weight",
    "decoder.ln.bias": "model.decoder.layer_norm.bias",
}
HF_BLOCK = {
    "self_attn_ln": "self_attn_layer_norm", "self_attn.query": "self_attn.q_proj", "self_attn.key": "self_attn.k_proj",
    "self_attn.value": "self_attn.v_proj", "self_attn.out": "self_attn.out_proj",
    "cross_attn_ln": "encoder_attn_layer_norm", "cross_attn.query": "encoder_attn.q_proj",
    "cross_attn.key": "encoder_attn.k_proj", "cross_attn.value": "encoder_attn.v_proj",
    "cross_attn.out": "encoder_attn.out_proj", "mlp_ln": "final_layer_norm", "mlp.0": "fc1", "mlp.2": "fc2",
}
FIELDS = [  # (whisper.cpp suffix, wg_layer_desc field, kind)
    ("self_attn_ln.weight", "self_ln_w", "v"), ("self_attn_ln.bias", "self_ln_b", "v"),
    ("self_attn.query.weight", "self_q", "m"), ("self_attn.query.bias", "self_q_b", "v"),
    ("self_attn.key.weight", "self_k", "m"), ("self_attn.value.weight", "self_v", "m"),
    ("self_attn.value.bias", "self_v_b", "v"), ("self_attn.out.weight", "self_o", "m"),
    ("self_attn.out.bias", "self_o_b", "v"), ("cross_attn_ln.weight", "cross_ln_w", "v"),
    ("cross_attn_ln.bias", "cross_ln_b", "v"), ("cross_attn.query.weight", "cross_q", "m"),
    ("cross_attn.query.bias", "cross_q_b", "v"), ("cross_attn.key.weight", "cross_k", "m"),
    ("cross_attn.value.weight", "cross_v", "m"), ("cross_attn.value.bias", "cross_v_b", "v"),
    ("cross_attn.out.weight", "cross_o", "m"), ("cross_attn.out.bias", "cross_o_b", "v"),
    ("mlp_ln.weight", "mlp_ln_w", "v"), ("mlp_ln.bias", "mlp_ln_b", "v"), ("mlp.0.weight", "mlp0", "m"),
    ("mlp.0.bias", "mlp0_b", "v"), ("mlp.2.weight", "mlp2", "m"), ("mlp.2.bias", "mlp2_b", "v"),
]


def hf_name(name):
    if name in HF:
        return HF[name]
    _, _, i, rest = name.split(".", 3)
    stem, leaf = rest.rsplit(".", 1)
    return "model.decoder.layers.%s.%s.%s" % (i, HF_BLOCK[stem], leaf)


def _s(b):
    return struct.pack("<Q", len(b)) + b


def write(path, model, names="whisper.cpp", f16_vectors=False, meta=True, vocab_tokens=0):
    """Writes model (a SyntheticModel / ArrayModel) to path. f16_vectors stores
    the fp32 vectors as F16; vocab_tokens > 0 adds a string-array metadata
    entry of that many tokens (real files carry the vocabulary)."""
    d = wgdec._desc_ptr(model).contents
    V, D, H, L, C = d.n_vocab, d.n_state, d.n_head, d.n_layer, d.n_text_ctx
    tensors = []  # (name, shape, dtype, bytes)

    def vec(name, ptr, n, shape=None):
        a = np.ctypeslib.as_array(ptr, shape=(n,)).astype(np.float32)
        if f16_vectors:
            tensors.append((name, shape or [n], 1, a.astype(np.float16).tobytes()))
        else:
            tensors.append((name, shape or [n], 0, a.tobytes()))

    def mat(name, m):
        nb = m.rows * ROW_BYTES[m.qtype](m.cols)
        tensors.append((name, [m.rows, m.cols], m.qtype, ctypes.string_at(m.data, nb)))

    mat("decoder.token_embedding.weight", d.token_embedding)
    vec("decoder.positional_embedding", d.positional_embedding, C * D, [C, D])
    vec("decoder.ln.weight", d.ln_w, D)
    vec("decoder.ln.bias", d.ln_b, D)
    for i in range(L):
        ly = d.layers[i]
        for suffix, field, kind in FIELDS:
            name = "decoder.blocks.%d.%s" % (i, suffix)
            if kind == "m":
                mat(name, getattr(ly, field))
            else:
                n = 4 * D if field == "mlp0_b" else D
                vec(name, getattr(ly, field), n)
    if names == "hf":
        tensors = [(hf_name(n), s, t, b) for n, s, t, b in tensors]
    kv = []
    if meta:
        for k, v in [("whisper.decoder.attention.head_count", H), ("whisper.decoder.layer_count", L),
                     ("whisper.decoder.context_length", C), ("whisper.decoder.embedding_length", D),
                     ("whisper.vocab.size", V)]:
            kv.append(_s(k.encode()) + struct.pack("<II", T_U32, v))
    if vocab_tokens:
        toks = b"".join(_s(("tok%d" % i).encode()) for i in range(vocab_tokens))
        kv.append(_s(b"tokenizer.ggml.tokens") + struct.pack("<IIQ", T_ARR, T_STR, vocab_tokens) + toks)
    kv.append(_s(b"general.name") + struct.pack("<I", T_STR) + _s(b"synthetic whisper decoder"))
    offs, off = [], 0
    for _, _, _, b in tensors:
        offs.append(off)
        off += len(b)
        off += (32 - off % 32) % 32
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kv)) + b"".join(kv)
    for (n, shape, t, _), o in zip(tensors, offs):
        head += _s(n.encode()) + struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", x) for x in shape)
        head += struct.pack("<IQ", t, o)
    head += b"\0" * ((32 - len(head) % 32) % 32)
    with open(path, "wb") as f:
        f.write(head)
        for i, (_, _, _, b) in enumerate(tensors):
            f.write(b)
            if i < len(tensors) - 1:
                f.write(b"\0" * ((32 - len(b) % 32) % 32))
