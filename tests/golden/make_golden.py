"""Generates tests/golden/torch_numerics.json: golden vectors that pin the CPU
oracle's weight-free arithmetic to torch's float32 semantics, which the
reference restates from OpenBMB's PyTorch model:

- torch.linspace(1, 0, n) in float32 (generator.cpp:21-37);
- the sway-sampled Euler time span of UnifiedCFM.solve_euler
  (generator.cpp:63-80): t + sway * (cos(pi/2 t) - 1 + t);
- float32 -> bfloat16 conversion (round to nearest even) and float16 decode
  (kernels/device_math.hpp:12-24);
- FSQ: bf16(round(tanh(x) * 9) / 9) with round half to even
  (kernels/generator_kernels.hip:291-297);
- SinusoidalPosEmb(1024)(t) with scale 1000 (generator.cpp:39-53);
- the LongRoPE cos/sin table in float32 (transformer.cpp:20-45) for seeded
  factors (the released short factors are config data, not needed here).

Run from the repository root: ``python tests/golden/make_golden.py``.
"""

import json
import math
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "torch_numerics.json"


def f32_hex(values) -> list[str]:
    a = np.asarray(values, dtype=np.float32).reshape(-1)
    return [f"{int(v):08x}" for v in a.view(np.uint32)]


def main() -> None:
    torch.manual_seed(0)
    golden: dict = {"source": "torch " + torch.__version__ + " (CPU, float32)"}

    golden["linspace"] = {str(n): f32_hex(torch.linspace(1.0, 0.0, n, dtype=torch.float32).numpy())
                          for n in (2, 3, 5, 10, 11, 17, 33)}

    spans = {}
    for n in (4, 10, 16, 32):
        t = torch.linspace(1.0, 0.0, n + 1, dtype=torch.float32)
        sway = torch.tensor(1.0, dtype=torch.float32)
        t = t + sway * (torch.cos(torch.tensor(math.pi / 2, dtype=torch.float32) * t) - 1 + t)
        spans[str(n)] = f32_hex(t.numpy())
    golden["sway_span"] = spans

    specials = np.array([0.0, -0.0, 1.0, -1.0, 1.00390625, 1.01171875, 3.0e38, -3.0e38, 1e-40, 65504.0,
                         float("inf"), float("-inf"), 0.1, 0.2, 0.3, 1.0 / 3.0], dtype=np.float32)
    randoms = (torch.randn(4096, dtype=torch.float32) * torch.exp(torch.randn(4096) * 4)).numpy()
    x = np.concatenate([specials, randoms]).astype(np.float32)
    golden["bf16"] = {
        "x": f32_hex(x),
        "bits": [f"{int(v):04x}" for v in torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)],
    }

    half_bits = np.arange(0, 65536, 97, dtype=np.uint32).astype(np.uint16)
    half_bits = half_bits[(half_bits & 0x7C00) != 0x7C00]
    golden["half"] = {"bits": [f"{int(b):04x}" for b in half_bits],
                      "value": f32_hex(half_bits.view(np.float16).astype(np.float32))}

    xq = torch.cat([torch.randn(2048) * 2, torch.tensor([0.0, 0.5, -0.5, 3.0, -3.0])]).to(torch.float32)
    q = torch.round(torch.tanh(xq) * 9.0) / 9.0
    golden["fsq"] = {"x": f32_hex(xq.numpy()),
                     "bits": [f"{int(v):04x}" for v in q.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)]}

    sinus = {}
    for t in (0.0, 0.63, 0.9564, 1.0):
        half = 512
        emb = math.log(10000) / (half - 1)
        freq = torch.exp(torch.arange(half, dtype=torch.float32) * -emb)
        arg = 1000.0 * torch.tensor([t], dtype=torch.float32)[:, None] * freq[None]
        e = torch.cat([arg.sin(), arg.cos()], dim=-1)[0]
        sinus[repr(t)] = f32_hex(e.numpy())
    golden["sinusoid"] = sinus

    rng = np.random.default_rng(3)
    factors = (1.0 + rng.random(64) * 3.0).astype(np.float64)
    dim, positions, theta = 128, 64, 10000.0
    inv_freq = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    t = torch.arange(positions, dtype=torch.float32)
    freqs = torch.outer(t, 1.0 / torch.tensor(factors, dtype=torch.float32)) * inv_freq
    table = torch.cat([freqs.cos(), freqs.sin()], dim=-1)
    golden["rope"] = {"theta": theta, "dim": dim, "positions": positions,
                      "factors": [float(f) for f in factors], "table": f32_hex(table.numpy())}

    OUT.write_text(json.dumps(golden, indent=0))
    print(OUT, OUT.stat().st_size)


if __name__ == "__main__":
    main()
