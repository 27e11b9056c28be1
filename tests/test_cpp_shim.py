"""The C++ mirror header (include/voxcpm_b200.hpp) compiles with g++, links
the library and gives the same host results as the oracle (no GPU); and, on
a B200, the products and the generator called from C++ through it match the
oracle (tests/cpp/shim_device.cpp)."""

import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle
from voxcpm_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent


def test_cpp_shim_compiles_links_and_runs(tmp_path):
    _lib.load()
    exe = tmp_path / "shim_host"
    lib_dir = str(_lib.LIBRARY.parent)
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", str(ROOT / "include"), "-I", "/usr/local/cuda/include",
                    str(ROOT / "tests" / "cpp" / "shim_host.cpp"), "-o", str(exe), "-L", lib_dir,
                    "-l:libvoxcpm_b200.so", f"-Wl,-rpath,{lib_dir}"], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines()
    steps = [line.split() for line in out if line.startswith("step")]
    t, dt, ev = oracle.euler_schedule(10)
    assert len(steps) == 10
    for (_, ts, dts, evs), a, b, c in zip(steps, t, dt, ev):
        assert np.float32(float(ts)) == a and np.float32(float(dts)) == b and bool(int(evs)) == c
    plan = next(line for line in out if line.startswith("plan")).split()
    assert int(plan[1]) >= 1 and int(plan[3]) == 0 and int(plan[4]) == 0
    tiles = next(line for line in out if line.startswith("tiles")).split()
    assert tiles[1:] == [str(6144 // 16 * 64 * 544), str(5 * 32 * 1024)]
    table = oracle.rope_table(10000.0, 128, np.ones(64), 1.0, 4)
    rope = next(line for line in out if line.startswith("rope")).split()
    assert np.float32(float(rope[1])) == table[1, 1] and np.float32(float(rope[2])) == table[3, 64 + 5]
    assert "error ok" in out
    assert "bucket 256 128" in out and "matmul rejects ok" in out


def test_cpp_shim_model_files(tmp_path):
    """ModelFiles / ParseConfig through the C++ mirror on a GGUF written here."""
    from _checkpoints import GGML_Q8_0, config_json, write_gguf
    from voxcpm_b200.generator import small_config

    _lib.load()
    exe = tmp_path / "shim_host"
    lib_dir = str(_lib.LIBRARY.parent)
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", str(ROOT / "include"), "-I", "/usr/local/cuda/include",
                    str(ROOT / "tests" / "cpp" / "shim_host.cpp"), "-o", str(exe), "-L", lib_dir,
                    "-l:libvoxcpm_b200.so", f"-Wl,-rpath,{lib_dir}"], check=True)
    c = small_config(layers=3, max_length=128, vocab=77)
    path = tmp_path / "m.gguf"
    write_gguf(path, {"stop_head.weight": (GGML_Q8_0, [2048, 2], bytes(2 * 64 * 34))},
               config_text=config_json(c), abbreviate=("stop_head.weight",))
    out = subprocess.run([str(exe), str(path)], check=True, capture_output=True, text=True).stdout.split("\n")
    assert out[0] == "files 1 1"
    assert out[1] == f"tensor {_lib.DTYPE_Q8_0} 2 2048 {2 * 64 * 34}"
    assert out[2] == "config 2048 3 77 128"
    bad = subprocess.run([str(exe), str(tmp_path / "absent.gguf")], check=True, capture_output=True,
                         text=True).stdout
    assert bad.startswith("files error") and "absent.gguf" in bad


def _build_device_shim(tmp_path):
    """Compiles tests/cpp/shim_device.cpp against include/voxcpm_b200.hpp
    and links the library and the CUDA runtime."""
    _lib.load()
    exe = tmp_path / "shim_device"
    lib_dir = str(_lib.LIBRARY.parent)
    cuda = "/usr/local/cuda"
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", str(ROOT / "include"),
                    "-I", f"{cuda}/include", str(ROOT / "tests" / "cpp" / "shim_device.cpp"), "-o", str(exe),
                    "-L", lib_dir, "-l:libvoxcpm_b200.so", f"-Wl,-rpath,{lib_dir}", "-L", f"{cuda}/lib64",
                    "-lcudart", f"-Wl,-rpath,{cuda}/lib64"], check=True)
    return exe


def test_cpp_device_shim_compiles(tmp_path):
    """The device program of the C++ mirror compiles and links on any host."""
    assert _build_device_shim(tmp_path).exists()


@pytest.mark.gpu
def test_cpp_mirror_on_device(tmp_path, cuda):
    """Bf16Gemm::Linear (Q8_0 tiles and bf16 rows), a seeded Generator's
    Prefill and two Steps and the AudioVae decoding the last latent, called
    from C++ through include/voxcpm_b200.hpp,
    against the oracle: products within 1e-5 of sum |x w|
    (tests/products_test.cpp:115-145), latents relative L2 2e-2 and stop
    logits within 5e-3 (the generator tests' limits)."""
    from _checkpoints import config_json
    from oracle.model import OracleGenerator
    from voxcpm_b200.generator import small_config

    exe = _build_device_shim(tmp_path)
    rng = np.random.default_rng(5)
    rows, columns, out = 22, 1024, 2560
    x = oracle.bf16_bits(rng.normal(0, 1, (rows, columns)).astype(np.float32))
    blocks = oracle.random_q8_0(3, 1, out, columns)
    w = oracle.bf16_bits(rng.normal(0, 0.02, (out, columns)).astype(np.float32))
    c = small_config()
    p_rows, steps = 9, 2
    tokens = rng.integers(0, c.vocab, p_rows).astype(np.int32)
    audio = np.zeros(p_rows, np.int32)
    audio[-1] = 1
    feats = np.zeros((p_rows, c.patch_size * c.feat_dim), np.float32)
    feats[-1] = rng.normal(0, 1, c.patch_size * c.feat_dim)
    noise = rng.normal(0, 1, (steps, c.patch_size * c.feat_dim)).astype(np.float32)
    (tmp_path / "dims.txt").write_text(f"{rows} {columns} {out} {steps} {p_rows}\n")
    for name, array in (("x.u16", x), ("blocks.u8", blocks), ("w.u16", w), ("tokens.i32", tokens),
                        ("text.i32", (1 - audio).astype(np.int32)), ("audio.i32", audio),
                        ("feats.f32", feats), ("noise.f32", noise)):
        array.tofile(tmp_path / name)
    (tmp_path / "config.json").write_text(config_json(c))
    run = subprocess.run([str(exe), str(tmp_path)], capture_output=True, text=True)
    assert run.returncode == 0, run.stderr
    assert f"positions {p_rows + steps}" in run.stdout

    for file, fmt, weights in (("y_q8.f32", oracle.Q8_0, blocks), ("y_bf16.f32", oracle.BF16_ROWS, w)):
        y = np.fromfile(tmp_path / file, np.float32).reshape(rows, out)
        exact, mag = oracle.product_exact(x, fmt, weights, rows, columns, out)
        err = oracle.relative_error(y, exact, mag)
        print(f"{file}: {err:.3e}")
        assert err <= 1e-5, file
    ref = OracleGenerator(c, seed=7)
    ref.prefill(tokens, 1 - audio, audio, feats.reshape(p_rows, c.patch_size, c.feat_dim))
    latents = np.fromfile(tmp_path / "latents.f32", np.float32).reshape(steps, -1)
    stops = np.fromfile(tmp_path / "stops.f32", np.float32).reshape(steps, 2)
    for s in range(steps):
        latent_r, stop_r = ref.step(noise[s].reshape(c.patch_size, c.feat_dim), 10, 2.0)
        e = float(np.linalg.norm(latents[s] - latent_r.reshape(-1)) / np.linalg.norm(latent_r))
        print(f"step {s}: latent {e:.3e} stop {np.abs(stops[s] - stop_r).max():.3e}")
        assert e < 2e-2 and float(np.abs(stops[s] - stop_r).max()) < 5e-3

    # AudioVae: Enqueue(latent, latent_event) + Collect equals Decode of the
    # same latent from the host, and both match the oracle decoder
    # (tests/vae_test.cpp:127's 1e-4 relative L2).
    from oracle.vae import OracleVae, VaeConfig

    enqueued = np.fromfile(tmp_path / "vae_enqueued.f32", np.float32)
    decoded = np.fromfile(tmp_path / "vae_decoded.f32", np.float32)
    np.testing.assert_array_equal(enqueued, decoded)
    vae = OracleVae(VaeConfig(latent_dim=c.feat_dim, decoder_dim=64, decoder_rates=(2, 3)), seed=11)
    expected = vae.decode(latents[-1].reshape(c.patch_size, c.feat_dim))
    assert decoded.shape == expected.shape
    assert float(np.linalg.norm(decoded - expected) / np.linalg.norm(expected)) <= 1e-4
