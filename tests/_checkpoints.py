"""Checkpoint files for the model-file tests: writers of safetensors and
audio.cpp-layout GGUF files (from the published formats), config.json from a
ModelConfig, and the generator's tensors of a seeded checkpoint (the same
values vx_generator_create uploads), so a generator read from files can be
compared with the seeded one bit for bit.
"""

from __future__ import annotations

import json
import struct

import numpy as np

import oracle
from oracle.model import Q8_SCALE_STD, MATRIX_STD, tensor_id

# ggml tensor types.
GGML_F32, GGML_F16, GGML_Q8_0, GGML_I32, GGML_BF16 = 0, 1, 8, 26, 30
SAFETENSORS_DTYPES = {"F32": 4, "BF16": 2, "F16": 2, "I64": 8, "I32": 4, "U8": 1}


class T:
    """One tensor to write: dtype name, shape (outermost first), raw bytes."""

    def __init__(self, dtype: str, shape, data: np.ndarray):
        self.dtype, self.shape, self.data = dtype, tuple(int(s) for s in shape), np.ascontiguousarray(data)

    @property
    def raw(self) -> bytes:
        return self.data.tobytes()


# ------------------------------------------------------------ safetensors

def write_safetensors(path, tensors: dict, metadata: dict | None = None, header_pad: bool = True) -> None:
    header = {}
    if metadata is not None:
        header["__metadata__"] = metadata
    at = 0
    payload = []
    for name, t in tensors.items():
        raw = t.raw
        header[name] = {"dtype": t.dtype, "shape": list(t.shape), "data_offsets": [at, at + len(raw)]}
        payload.append(raw)
        at += len(raw)
    text = json.dumps(header).encode()
    if header_pad:
        text += b" " * (-len(text) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(text)))
        f.write(text)
        for raw in payload:
            f.write(raw)


def write_directory(root, tensors: dict, config_text: str, tokenizer_text: str | None = None) -> None:
    root.mkdir(parents=True, exist_ok=True)
    (root / "config.json").write_text(config_text)
    if tokenizer_text is not None:
        (root / "tokenizer.json").write_text(tokenizer_text)
    write_safetensors(root / "model.safetensors", tensors)


# ------------------------------------------------------------ GGUF

def _gguf_string(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _gguf_value(kind: str, value) -> bytes:
    """(type, payload) of a metadata value: kind is 'str', 'u32', 'u64',
    'strs' (string array) or an integer array ('u8s', 'i8s', 'u64s', 'i64s')."""
    if kind == "str":
        return struct.pack("<I", 8) + _gguf_string(value)
    if kind == "u32":
        return struct.pack("<II", 4, value)
    if kind == "u64":
        return struct.pack("<IQ", 10, value)
    if kind == "strs":
        return struct.pack("<IIQ", 9, 8, len(value)) + b"".join(_gguf_string(v) for v in value)
    element, fmt = {"u8s": (0, "B"), "i8s": (1, "b"), "u64s": (10, "Q"), "i64s": (11, "q")}[kind]
    return struct.pack("<IIQ", 9, element, len(value)) + struct.pack("<" + fmt * len(value), *value)


def write_gguf(path, model: dict, vae: dict | None = None, config_text: str = "{}",
               tokenizer_text: str = "{}", family: str = "voxcpm2", abbreviate=(), alignment: int = 32,
               version: int = 3, extra_meta: list | None = None, embedded: bool = True,
               data_kind: str = "u8s") -> None:
    """An audio.cpp GGUF: `model` tensors under weights/, `vae` under
    audiovae_weights/, names in `abbreviate` stored as _audiocpp.<i> with the
    full name in audiocpp.tensor_names. model/vae values are (ggml type,
    dims innermost first, raw bytes)."""
    entries = [("weights/" + n, v) for n, v in model.items()]
    entries += [("audiovae_weights/" + n, v) for n, v in (vae or {}).items()]
    names = []
    stored = []
    for full, v in entries:
        if full.split("/", 1)[1] in abbreviate:
            stored.append((f"_audiocpp.{len(names)}", v))
            names.append(full)
        else:
            stored.append((full, v))
    meta = [("general.architecture", "str", "audiocpp"), ("audiocpp.model_spec.family", "str", family),
            ("general.alignment", "u32", alignment)]
    if names:
        meta.append(("audiocpp.tensor_names", "strs", names))
    if embedded:
        files = [("config.json", config_text.encode()), ("tokenizer.json", tokenizer_text.encode())]
        offsets = [0]
        data = b""
        for _, b in files:
            data += b
            offsets.append(len(data))
        values = list(data) if data_kind == "u8s" else [x - 256 if x > 127 else x for x in data]
        meta += [("audiocpp.embedded_files.names", "strs", [n for n, _ in files]),
                 ("audiocpp.embedded_files.offsets", "u64s", offsets),
                 ("audiocpp.embedded_files.data", data_kind, values)]
    meta += extra_meta or []
    out = bytearray(b"GGUF" + struct.pack("<IQQ", version, len(stored), len(meta)))
    for key, kind, value in meta:
        out += _gguf_string(key) + _gguf_value(kind, value)
    at = 0
    blobs = []
    for name, (ggml_type, dims, raw) in stored:
        out += _gguf_string(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims)
        out += struct.pack("<IQ", ggml_type, at)
        blobs.append((at, raw))
        at += len(raw)
        at += -at % alignment
    out += b"\0" * (-len(out) % alignment)
    base = len(out)
    out += b"\0" * at
    for offset, raw in blobs:
        out[base + offset: base + offset + len(raw)] = raw
    with open(path, "wb") as f:
        f.write(out)


# ------------------------------------------------------------ config.json

def config_json(c, max_positions: int = 32768, original: int = 32768, short=None, long=None, **overrides) -> str:
    """config.json of an openbmb VoxCPM2 directory with the shapes of `c`."""
    half = c.lm.head_dim // 2
    short = [float(c.rope_factors[i]) for i in range(half)] if short is None else short
    long = short if long is None else long

    def derived(s):
        return {"hidden_dim": s.hidden, "ffn_dim": s.intermediate, "num_heads": s.heads,
                "num_layers": s.layers, "kv_channels": s.head_dim}

    doc = {
        "architecture": "voxcpm2",
        "lm_config": {
            "hidden_size": c.lm.hidden, "intermediate_size": c.lm.intermediate,
            "num_hidden_layers": c.lm.layers, "num_attention_heads": c.lm.heads,
            "num_key_value_heads": c.lm.kv_heads, "kv_channels": c.lm.head_dim,
            "vocab_size": c.vocab, "rms_norm_eps": float(np.float32(c.lm.rms_eps)),
            "no_rope": not c.lm.rope, "use_mup": False, "scale_emb": 12, "scale_depth": 1.4,
            "rope_theta": c.rope_theta, "max_position_embeddings": max_positions,
            "rope_scaling": {"type": "longrope", "original_max_position_embeddings": original,
                             "short_factor": short, "long_factor": long},
        },
        "residual_lm_num_layers": c.residual_lm.layers,
        "residual_lm_no_rope": not c.residual_lm.rope,
        "encoder_config": derived(c.encoder),
        "dit_config": dict(derived(c.dit), cfm_config={"sigma_min": 1e-6}),
        "patch_size": c.patch_size, "feat_dim": c.feat_dim,
        "scalar_quantization_latent_dim": c.fsq_latent_dim,
        "scalar_quantization_scale": float(c.fsq_scale),
        "max_length": c.max_length, "dtype": "bfloat16",
        "audio_vae_config": {"latent_dim": c.feat_dim},
    }
    for key, value in overrides.items():
        node = doc
        parts = key.split(".")
        for p in parts[:-1]:
            node = node[p]
        if value is None:
            node.pop(parts[-1], None)
        else:
            node[parts[-1]] = value
    return json.dumps(doc)


# ------------------------------------------------------------ seeded tensors

def tensor_list(c):
    """(name, shape, kind, mean, std) of every generator tensor in the
    reference's order (weights.cpp:268-304); kind 'matrix' or 'vector'."""
    hidden, local, dit, feat = c.lm.hidden, c.encoder.hidden, c.dit.hidden, c.feat_dim
    out = []

    def vector(name, shape, mean, std):
        out.append((name, tuple(shape), "vector", mean, std))

    def matrix(name, rows, cols):
        out.append((name, (rows, cols), "matrix", 0.0, MATRIX_STD))

    def linear(prefix, n_in, n_out, bias):
        matrix(prefix + ".weight", n_out, n_in)
        if bias:
            vector(prefix + ".bias", (n_out,), 0.0, MATRIX_STD)

    def stack(prefix, s):
        h, q, kv = s.hidden, s.heads * s.head_dim, s.kv_heads * s.head_dim
        for i in range(s.layers):
            l = f"{prefix}.layers.{i}"
            a = l + ".self_attn."
            vector(l + ".input_layernorm.weight", (h,), 1.0, 0.05)
            matrix(a + "q_proj.weight", q, h)
            matrix(a + "k_proj.weight", kv, h)
            matrix(a + "v_proj.weight", kv, h)
            matrix(a + "o_proj.weight", h, q)
            vector(l + ".post_attention_layernorm.weight", (h,), 1.0, 0.05)
            matrix(l + ".mlp.gate_proj.weight", s.intermediate, h)
            matrix(l + ".mlp.up_proj.weight", s.intermediate, h)
            matrix(l + ".mlp.down_proj.weight", h, s.intermediate)
        vector(prefix + ".norm.weight", (h,), 1.0, 0.05)

    if c.vocab:
        vector("base_lm.embed_tokens.weight", (c.vocab, hidden), 0.0, 0.5)
    stack("base_lm", c.lm)
    stack("residual_lm", c.residual_lm)
    stack("feat_encoder.encoder", c.encoder)
    vector("feat_encoder.special_token", (1, 1, 1, local), 0.0, 1.0)
    linear("feat_encoder.in_proj", feat, local, True)
    stack("feat_decoder.estimator.decoder", c.dit)
    e = "feat_decoder.estimator."
    linear(e + "in_proj", feat, dit, True)
    linear(e + "cond_proj", feat, dit, True)
    linear(e + "out_proj", dit, feat, True)
    for n in ("time_mlp.linear_1", "time_mlp.linear_2", "delta_time_mlp.linear_1", "delta_time_mlp.linear_2"):
        linear(e + n, dit, dit, True)
    linear("enc_to_lm_proj", local, hidden, True)
    linear("lm_to_dit_proj", hidden, dit, True)
    linear("res_to_dit_proj", hidden, dit, True)
    linear("fusion_concat_proj", 2 * hidden, hidden, True)
    linear("fsq_layer.in_proj", hidden, c.fsq_latent_dim, True)
    linear("fsq_layer.out_proj", c.fsq_latent_dim, hidden, True)
    linear("stop_proj", hidden, hidden, True)
    linear("stop_head", hidden, 2, False)
    return out


def seeded_values(name, shape, kind, mean, std, seed, q8):
    """The seeded checkpoint's value of one tensor: ('Q8_0', blocks) or
    ('BF16', bits)."""
    if kind == "matrix" and q8:
        return "Q8_0", oracle.random_q8_0(seed, tensor_id(name), shape[0], shape[1], Q8_SCALE_STD)
    count = int(np.prod(shape))
    return "BF16", oracle.random_bf16(seed, tensor_id(name), count, mean, std)


def as_dtype(kind: str, values: np.ndarray, dtype: str) -> np.ndarray:
    """Re-encodes bf16 bits (kind 'BF16') as F32 (exact) or keeps them."""
    if kind == "Q8_0" or dtype == "BF16":
        return values
    if dtype == "F32":
        return oracle.bf16_value(values).astype(np.float32)
    raise ValueError(dtype)


def ggml_entry(kind: str, shape, values: np.ndarray):
    dims = list(reversed(shape))
    ggml = {"Q8_0": GGML_Q8_0, "BF16": GGML_BF16, "F32": GGML_F32, "F16": GGML_F16}[kind]
    return ggml, dims, np.ascontiguousarray(values).tobytes()
