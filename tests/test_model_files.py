"""The checkpoint readers on the host (no GPU): safetensors directories and
audio.cpp GGUF files written here from the published formats, the
audio.cpp layout (abbreviated names, components, embedded config and
tokenizer), malformed files, and config.json parsing (config.cpp:149-301).
Mirrors tests/weights_test.cpp's sample checks (dtypes, shapes, values,
rejected files).
"""

import json
import os
import struct
from pathlib import Path

import numpy as np
import pytest

from voxcpm_b200._lib import VxError
from voxcpm_b200.generator import released_config, small_config
from voxcpm_b200.model_files import ModelFiles, ParseConfig

from _checkpoints import (GGML_BF16, GGML_F16, GGML_F32, GGML_I32, GGML_Q8_0, T, config_json, write_directory,
                          write_gguf, write_safetensors)

# A safetensors file written by the reference's own tooling: its golden
# fixture (tests/fixtures/generator_golden.safetensors of the reference tree),
# found through VOXCPM_REFERENCE_FIXTURE when that names it. Hosts without
# the reference tree skip the test.
REFERENCE_FIXTURE = Path(os.environ.get("VOXCPM_REFERENCE_FIXTURE", "generator_golden.safetensors"))


def sample_tensors():
    rng = np.random.default_rng(0)
    return {
        "layer.weight": T("F32", (2, 3), np.array([1.5, -2.0, 3.25, 0.0, 4.0, -0.5], np.float32)),
        "layer.bias": T("I32", (4,), np.array([7, -8, 9, 2147483647], np.int32)),
        "half": T("BF16", (2,), np.array([0x3F80, 0xC040], np.uint16)),
        "f16": T("F16", (3,), np.array([1.0, -0.5, 65504.0], np.float16)),
        "ids": T("I64", (2,), np.array([1 << 40, -3], np.int64)),
        "bytes": T("U8", (5,), rng.integers(0, 256, 5).astype(np.uint8)),
        "scalar": T("F32", (), np.array([0.25], np.float32)),
        "empty": T("F32", (0, 4), np.zeros(0, np.float32)),
    }


def test_safetensors_directory(tmp_path):
    tensors = sample_tensors()
    write_directory(tmp_path, tensors, '{"a": 1}', tokenizer_text='{"tok": true}')
    with ModelFiles(tmp_path) as files:
        assert not files.gguf()
        assert files.config() == '{"a": 1}'
        assert files.tokenizer() == '{"tok": true}'
        got = files.model_tensors()
        assert [t.name for t in got] == sorted(tensors)
        assert files.vae_tensors() == []
        for name, t in tensors.items():
            f = files.Model(name)
            assert f is not None and f.dtype == t.dtype and f.shape == t.shape, name
            assert f.bytes == len(t.raw) and f.raw().tobytes() == t.raw, name
        assert files.Model("absent") is None
        # Offsets are byte positions in the file: the payload follows the header.
        raw = (tmp_path / "model.safetensors").read_bytes()
        n = struct.unpack("<Q", raw[:8])[0]
        layer = files.Model("layer.weight")
        assert raw[layer.offset: layer.offset + layer.bytes] == tensors["layer.weight"].raw
        assert layer.offset >= 8 + n


def test_directory_without_tokenizer(tmp_path):
    write_directory(tmp_path, {"x": T("F32", (1,), np.ones(1, np.float32))}, "{}")
    with ModelFiles(tmp_path) as files:
        assert files.tokenizer() == ""


def corrupt(tmp_path, mutate):
    write_directory(tmp_path, {"a": T("F32", (2,), np.ones(2, np.float32)),
                               "b": T("F32", (2,), np.ones(2, np.float32))}, "{}")
    path = tmp_path / "model.safetensors"
    raw = bytearray(path.read_bytes())
    path.write_bytes(bytes(mutate(raw)))


def header_of(raw):
    n = struct.unpack("<Q", raw[:8])[0]
    return json.loads(bytes(raw[8:8 + n])), raw[8 + n:]


def with_header(header, payload):
    text = json.dumps(header).encode()
    return struct.pack("<Q", len(text)) + text + payload


def edit(fn):
    def mutate(raw):
        header, payload = header_of(raw)
        fn(header)
        return with_header(header, payload)
    return mutate


@pytest.mark.parametrize("mutate, message", [
    (lambda raw: raw[:5], "shorter than its 8-byte header length"),
    (lambda raw: struct.pack("<Q", 0) + raw[8:], "header length 0 is implausible"),
    (lambda raw: struct.pack("<Q", 1 << 40) + raw[8:], "header length .* is implausible"),
    (lambda raw: raw[:8] + b"x" + raw[9:], "header is not valid JSON"),
    (lambda raw: raw[:8] + b"[" + raw[9:-1] + b"]", "JSON"),
    (edit(lambda h: h["a"].update(data_offsets=[0, 100])), "outside the payload"),
    (edit(lambda h: h["a"].update(data_offsets=[8, 4])), "outside the payload"),
    (edit(lambda h: h["a"].update(data_offsets=[0])), "two byte positions"),
    (edit(lambda h: h["a"].update(dtype="F64")), "type F64, which this library does not read"),
    (edit(lambda h: h["a"].update(shape=[3])), "but its shape and dtype need"),
    (edit(lambda h: h["a"].update(shape=[-2])), "not a list of sizes"),
    (edit(lambda h: h["b"].update(data_offsets=[4, 12])), "share bytes"),
    (edit(lambda h: h["a"].pop("dtype")), "needs all of dtype, shape and data_offsets"),
    (edit(lambda h: h.update(a=[1])), "must be an object"),
    (edit(lambda h: [h.pop("a"), h.pop("b")]), "declares no tensors"),
])
def test_safetensors_rejected(tmp_path, mutate, message):
    corrupt(tmp_path, mutate)
    with pytest.raises(VxError, match=message):
        ModelFiles(tmp_path)


def test_missing_files(tmp_path):
    with pytest.raises(VxError, match="config.json"):
        ModelFiles(tmp_path)
    (tmp_path / "config.json").write_text("{}")
    with pytest.raises(VxError, match="model.safetensors"):
        ModelFiles(tmp_path)
    with pytest.raises(VxError, match="cannot open"):
        ModelFiles(tmp_path / "absent.gguf")


def q8_blocks(rows, cols, seed=0):
    rng = np.random.default_rng(seed)
    blocks = np.zeros((rows, cols // 32, 34), np.uint8)
    scales = rng.uniform(0.001, 0.01, (rows, cols // 32)).astype(np.float16)
    blocks[:, :, :2] = scales.view(np.uint8).reshape(rows, cols // 32, 2)
    blocks[:, :, 2:] = rng.integers(-127, 128, (rows, cols // 32, 32)).astype(np.int8).view(np.uint8)
    return blocks


def gguf_model():
    return {
        "stop_head.weight": (GGML_Q8_0, [64, 2], q8_blocks(2, 64).tobytes()),
        "stop_proj.bias": (GGML_F32, [3], np.array([1, 2, 3], np.float32).tobytes()),
        "norm.weight": (GGML_BF16, [4], np.array([1, 2, 3, 4], np.uint16).tobytes()),
        "half": (GGML_F16, [2, 2], np.array([1, 2, 3, 4], np.float16).tobytes()),
        "ids": (GGML_I32, [2], np.array([5, -6], np.int32).tobytes()),
    }


@pytest.mark.parametrize("version", [2, 3])
@pytest.mark.parametrize("alignment", [32, 64])
def test_gguf_layout(tmp_path, version, alignment):
    path = tmp_path / "voxcpm2-q8_0.gguf"
    model = gguf_model()
    vae = {"decoder.conv.weight": (GGML_F32, [3, 2, 1], np.arange(6, dtype=np.float32).tobytes())}
    tokenizer = '{"model": "bpe", "vocab": {"é": 1}}'
    write_gguf(path, model, vae, config_text='{"architecture": "voxcpm2"}', tokenizer_text=tokenizer,
               abbreviate=("stop_head.weight", "decoder.conv.weight"), version=version, alignment=alignment)
    assert ModelFiles.IsVoxCpm2Gguf(path)
    with ModelFiles(path) as files:
        assert files.gguf()
        assert files.config() == '{"architecture": "voxcpm2"}'
        assert files.tokenizer() == tokenizer
        assert sorted(t.name for t in files.model_tensors()) == sorted(model)
        assert [t.name for t in files.vae_tensors()] == ["decoder.conv.weight"]
        dtypes = {GGML_Q8_0: "Q8_0", GGML_F32: "F32", GGML_BF16: "BF16", GGML_F16: "F16", GGML_I32: "I32"}
        for name, (ggml, dims, raw) in model.items():
            t = files.Model(name)
            assert t.dtype == dtypes[ggml] and t.shape == tuple(reversed(dims)), name
            assert t.bytes == len(raw) and t.raw().tobytes() == raw, name
            assert t.offset % alignment == 0
        v = files.Vae("decoder.conv.weight")
        assert v.shape == (1, 2, 3) and np.array_equal(v.raw().view(np.float32), np.arange(6))
        data = path.read_bytes()
        t = files.Model("half")
        assert data[t.offset: t.offset + t.bytes] == model["half"][2]


def test_gguf_signed_embedded_bytes(tmp_path):
    """Embedded file bytes stored as an int8 array (values above 127 wrap)."""
    path = tmp_path / "m.gguf"
    tokenizer = '{"ü": "中"}'
    write_gguf(path, gguf_model(), tokenizer_text=tokenizer, data_kind="i8s")
    with ModelFiles(path) as files:
        assert files.tokenizer() == tokenizer


def test_is_voxcpm2_gguf(tmp_path):
    good = tmp_path / "a.gguf"
    write_gguf(good, gguf_model())
    assert ModelFiles.IsVoxCpm2Gguf(good)
    other = tmp_path / "b.gguf"
    write_gguf(other, gguf_model(), family="qwen3-tts")
    assert not ModelFiles.IsVoxCpm2Gguf(other)
    renamed = tmp_path / "a.bin"
    renamed.write_bytes(good.read_bytes())
    assert not ModelFiles.IsVoxCpm2Gguf(renamed)
    assert not ModelFiles.IsVoxCpm2Gguf(tmp_path / "absent.gguf")
    assert not ModelFiles.IsVoxCpm2Gguf(tmp_path)
    with pytest.raises(VxError, match="not an audio.cpp VoxCPM2 GGUF"):
        ModelFiles(other)


def gguf_case(tmp_path, message, mutate=None, **kwargs):
    path = tmp_path / "m.gguf"
    write_gguf(path, kwargs.pop("model", gguf_model()), **kwargs)
    if mutate is not None:
        path.write_bytes(bytes(mutate(bytearray(path.read_bytes()))))
    with pytest.raises(VxError, match=message):
        ModelFiles(path)


def test_gguf_rejected(tmp_path):
    gguf_case(tmp_path, "not a GGUF file", mutate=lambda b: b"GGUG" + b[4:])
    gguf_case(tmp_path, "unsupported GGUF version 1", version=1)
    gguf_case(tmp_path, "counts exceed the file", mutate=lambda b: b[:60])
    gguf_case(tmp_path, "runs past the end", mutate=lambda b: b[:200])
    gguf_case(tmp_path, "unsupported type", model={"x": (2, [32], bytes(18))})
    gguf_case(tmp_path, "whole blocks", model={"x": (GGML_Q8_0, [48, 1], bytes(51))})
    gguf_case(tmp_path, "no listed name",
              extra_meta=[("audiocpp.tensor_names", "strs", [])], abbreviate=("stop_head.weight",),
              model={"stop_head.weight": (GGML_F32, [1], bytes(4))},
              mutate=None)
    gguf_case(tmp_path, "lacks the string array audiocpp.embedded_files.names", embedded=False)
    gguf_case(tmp_path, "dimensions", model={"x": (GGML_F32, [1, 1, 1, 1, 1], bytes(4))})


def test_gguf_out_of_data_section(tmp_path):
    path = tmp_path / "m.gguf"
    write_gguf(path, {"x": (GGML_F32, [8], bytes(32))})
    raw = path.read_bytes()
    path.write_bytes(raw[:-16])
    with pytest.raises(VxError, match="outside the data section"):
        ModelFiles(path)


def test_gguf_misaligned_offset(tmp_path):
    path = tmp_path / "m.gguf"
    write_gguf(path, {"a": (GGML_F32, [8], bytes(32)), "b": (GGML_F32, [8], bytes(32))})
    raw = bytearray(path.read_bytes())
    # The second tensor info's offset (32) is the last 8 bytes before the
    # header padding: find it after the name "weights/b".
    at = raw.index(b"weights/b") + len(b"weights/b") + 4 + 8 + 4
    assert struct.unpack("<Q", raw[at: at + 8])[0] == 32
    raw[at: at + 8] = struct.pack("<Q", 36)
    path.write_bytes(bytes(raw))
    with pytest.raises(VxError, match="outside the data section"):
        ModelFiles(path)


def test_gguf_no_component(tmp_path):
    path = tmp_path / "m.gguf"
    write_gguf(path, {"x": (GGML_F32, [1], bytes(4))})
    raw = path.read_bytes().replace(b"weights/x", b"weightsxx")
    path.write_bytes(raw)
    with pytest.raises(VxError, match="belongs to no component"):
        ModelFiles(path)


def test_gguf_malformed_embedded_table(tmp_path):
    path = tmp_path / "m.gguf"
    write_gguf(path, gguf_model(), extra_meta=[])
    raw = bytearray(path.read_bytes())
    # The offsets array (u64s) of two files: [0, len(config), len(config)+len(tokenizer)];
    # make the last offset run past the data.
    key = b"audiocpp.embedded_files.offsets"
    at = raw.index(key) + len(key) + 4 + 4 + 8 + 16
    raw[at: at + 8] = struct.pack("<Q", 1 << 20)
    path.write_bytes(bytes(raw))
    with pytest.raises(VxError, match="embedded file table is malformed"):
        ModelFiles(path)


@pytest.mark.skipif(not REFERENCE_FIXTURE.exists(), reason="the reference tree is not on this host")
def test_reference_fixture_reads(tmp_path):
    """A safetensors file written by the reference's own tooling (the golden
    fixture's header and payload, read in place through a directory link)."""
    (tmp_path / "config.json").write_text("{}")
    (tmp_path / "model.safetensors").symlink_to(REFERENCE_FIXTURE)
    raw = REFERENCE_FIXTURE.read_bytes()
    n = struct.unpack("<Q", raw[:8])[0]
    header = json.loads(raw[8:8 + n])
    header.pop("__metadata__", None)
    with ModelFiles(tmp_path) as files:
        assert len(files.model_tensors()) == len(header)
        for name, entry in header.items():
            t = files.Model(name)
            begin, end = entry["data_offsets"]
            assert t.dtype == entry["dtype"] and list(t.shape) == entry["shape"]
            assert t.raw().tobytes() == raw[8 + n + begin: 8 + n + end]


# ------------------------------------------------------------ config.json

def fields(c):
    out = {}
    for s in ("lm", "residual_lm", "encoder", "dit"):
        st = getattr(c, s)
        out[s] = tuple(getattr(st, f) for f in ("hidden", "intermediate", "layers", "heads", "kv_heads",
                                                 "head_dim", "rope"))
        out[s + ".eps"] = np.float32(st.rms_eps)
    for f in ("patch_size", "feat_dim", "fsq_latent_dim", "max_length", "vocab", "rope_theta", "rope_scaling"):
        out[f] = getattr(c, f)
    out["fsq_scale"] = np.float32(c.fsq_scale)
    out["factors"] = tuple(c.rope_factors[: c.lm.head_dim // 2])
    return out


def test_parse_config_released_shapes():
    c = released_config()
    c.vocab = 73448
    c.max_length = 8192
    parsed = ParseConfig(config_json(c))
    assert fields(parsed) == fields(c)


def test_parse_config_small_and_factors():
    c = small_config()
    short = [1.0 + i / 100 for i in range(64)]
    long = [2.0 + i / 100 for i in range(64)]
    p = ParseConfig(config_json(c, max_positions=32768, original=32768, short=short, long=long))
    assert list(p.rope_factors[:64]) == short and p.rope_scaling == 1.0
    assert p.lm.layers == c.lm.layers and p.dit.layers == c.dit.layers and p.vocab == c.vocab
    # Long factors once max_position_embeddings exceeds the original length,
    # and the LongRoPE magnitude sqrt(1 + ln(scale) / ln(original)).
    p = ParseConfig(config_json(c, max_positions=65536, original=32768, short=short, long=long))
    assert list(p.rope_factors[:64]) == long
    assert p.rope_scaling == pytest.approx(np.sqrt(1 + np.log(2.0) / np.log(32768.0)), rel=1e-15)


def test_parse_config_defaults():
    """Absent optional keys take the reference's defaults (patch 4, feat 64,
    FSQ 512 at scale 9, max_length 8192, 8 residual layers, derived stacks
    of 1024/4096/16 heads/4 layers; kv_channels falls back to hidden /
    heads, which the attention kernels reject)."""
    c = small_config()
    text = config_json(c, **{"patch_size": None, "feat_dim": None, "scalar_quantization_latent_dim": None,
                             "scalar_quantization_scale": None, "max_length": None,
                             "residual_lm_num_layers": None, "encoder_config": {"kv_channels": 128},
                             "audio_vae_config": None,
                             "lm_config.kv_channels": None, "dtype": None})
    p = ParseConfig(text)
    assert (p.patch_size, p.feat_dim, p.fsq_latent_dim, p.fsq_scale, p.max_length) == (4, 64, 512, 9.0, 8192)
    assert p.residual_lm.layers == 8
    e = p.encoder
    assert (e.hidden, e.intermediate, e.heads, e.layers, e.head_dim, e.kv_heads) == (1024, 4096, 16, 4, 128, 2)
    assert p.lm.head_dim == 2048 // 16
    with pytest.raises(VxError, match="head size of 128"):
        ParseConfig(config_json(c, encoder_config={}))


@pytest.mark.parametrize("overrides, message", [
    ({"architecture": "minicpm"}, "this library loads \"voxcpm2\""),
    ({"lm_config.use_mup": None}, "muP"),
    ({"lm_config.use_mup": True}, "muP"),
    ({"lm_config.kv_channels": 64}, "head size of 128"),
    ({"lm_config.num_key_value_heads": 3}, "multiple of the KV heads"),
    ({"dtype": "float32"}, "only bfloat16"),
    ({"dit_config.dit_mean_mode": True}, "dit_mean_mode"),
    ({"audio_vae_config": {"latent_dim": 32}}, "latent_dim"),
    ({"audio_vae_config": 5}, "audio_vae_config must be an object"),
    ({"lm_config.rope_scaling.short_factor": [1.0] * 32}, "LongRoPE factor per rotary pair"),
    ({"lm_config.hidden_size": 0}, "hidden_size must be a whole number"),
    ({"lm_config.hidden_size": 2048.5}, "hidden_size must be a whole number"),
    ({"lm_config.rms_norm_eps": "1e-5"}, "rms_norm_eps must be a finite number"),
    ({"lm_config.no_rope": 1}, "no_rope must be true or false"),
    ({"lm_config.vocab_size": None}, "lm_config.vocab_size is missing"),
    ({"dit_config": None}, "dit_config is missing"),
    ({"encoder_config": [1]}, "encoder_config must be an object"),
    ({"lm_config.rope_scaling.long_factor": []}, "long_factor must be a list"),
    ({"lm_config.rope_scaling.long_factor": [1.0, "x"]}, "long_factor must be a list"),
])
def test_parse_config_rejected(overrides, message):
    with pytest.raises(VxError, match=message):
        ParseConfig(config_json(small_config(), **overrides))


@pytest.mark.parametrize("text", ["", "{", "[1,]", '{"a" 1}', '{"a": tru}', '"\\x"', "01", '{"a": 1} x',
                                  '"\\ud800"', "[" * 300 + "]" * 300])
def test_parse_config_bad_json(text):
    with pytest.raises(VxError, match="JSON"):
        ParseConfig(text)


def test_parse_config_unicode_and_escapes():
    c = small_config()
    doc = json.loads(config_json(c))
    doc["description"] = "café \U0001f600 \t\"q\""
    p = ParseConfig(json.dumps(doc, ensure_ascii=True))
    assert p.lm.hidden == c.lm.hidden
