"""The C++ mirror header (include/voxcpm_b200.hpp) compiles with g++, links
the library and gives the same host results as the oracle (no GPU)."""

import subprocess
from pathlib import Path

import numpy as np

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
