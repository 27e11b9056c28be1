"""The oracle's generator: the reference's ForwardStack, DiT evaluation,
Euler/CFG patch, local encoder, FSQ, prefill and step composed from the C
primitives of vxoracle.c — TEST INFRASTRUCTURE ONLY (the checker of the
generator parity tests and the timed CPU baseline).

Weights are the library's seeded checkpoint, regenerated here from the same
rule (tensor id = FNV-1a of the tensor name; Q8_0 blocks or bf16 values from
the seeded hash, see vxoracle.c) and kept in canonical form: GGML Q8_0 blocks
or bf16 rows. Control flow follows, per method, the reference file:line cited.
"""

from __future__ import annotations

import numpy as np

from . import (BF16_ROWS, Q8_0, _f32, add_bias, assemble_dit, attention, bf16_bits, bf16_value,
               concat_rows, euler_schedule, gather_rows, guided_euler, linear, prepend_special, q8_0_dequant,
               quantize, qkv_rope, random_bf16, random_q8_0, rms_norm, rope_table, sinusoid, swiglu, to_bf16)

Q8_SCALE_STD = 0.02 / 127
MATRIX_STD = 0.02


def tensor_id(name: str) -> int:
    """FNV-1a 64 of the tensor name (the library's TensorId)."""
    h = 0xCBF29CE484222325
    for c in name.encode():
        h ^= c
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


class Projection:
    """y = x W^T (+ b) with W as GGML Q8_0 blocks or bf16 rows."""

    def __init__(self, fmt, weight, bias, n_in, n_out):
        self.format, self.weight, self.bias, self.n_in, self.n_out = fmt, weight, bias, n_in, n_out


class Stack:
    def __init__(self, config, layers, norm):
        self.config, self.layers, self.norm = config, layers, norm


def _stack_config(s) -> dict:
    return dict(hidden=s.hidden, intermediate=s.intermediate, layers=s.layers, heads=s.heads,
                kv_heads=s.kv_heads, head_dim=s.head_dim, rms_eps=float(np.float32(s.rms_eps)),
                rope=bool(s.rope))


class Weights:
    """weights.cpp:268-304: every tensor in the reference's order and names."""

    def __init__(self, config, seed: int, q8: bool, source: dict | None = None):
        """`source` (name -> ("Q8_0", GGML blocks) or ("BF16", bits)) stands
        for checkpoint files: matrices follow the file rule of
        weights.cpp:44-144 (Q8_0 blocks when every part is Q8_0 and, for
        fused parts, fills whole 16-row tiles; bf16 rows otherwise, Q8_0
        parts dequantized to bf16(scale * q))."""
        self.seed, self.q8, self.source = seed, q8, source
        c = config
        hidden, local, dit, feat = c.lm.hidden, c.encoder.hidden, c.dit.hidden, c.feat_dim
        self.embed = self.vector("base_lm.embed_tokens.weight", c.vocab * hidden, 0.0, 0.5) if c.vocab else None
        self.base_lm = self.stack("base_lm", c.lm)
        self.residual_lm = self.stack("residual_lm", c.residual_lm)
        self.encoder = self.stack("feat_encoder.encoder", c.encoder)
        self.special = self.vector("feat_encoder.special_token", local, 0.0, 1.0)
        self.encoder_in = self.linear("feat_encoder.in_proj", feat, local, True)
        self.dit = self.stack("feat_decoder.estimator.decoder", c.dit)
        e = "feat_decoder.estimator."
        self.dit_in = self.linear(e + "in_proj", feat, dit, True)
        self.dit_cond = self.linear(e + "cond_proj", feat, dit, True)
        self.dit_out = self.linear(e + "out_proj", dit, feat, True)
        self.time_1 = self.linear(e + "time_mlp.linear_1", dit, dit, True)
        self.time_2 = self.linear(e + "time_mlp.linear_2", dit, dit, True)
        self.delta_time_1 = self.linear(e + "delta_time_mlp.linear_1", dit, dit, True)
        self.delta_time_2 = self.linear(e + "delta_time_mlp.linear_2", dit, dit, True)
        self.enc_to_lm = self.linear("enc_to_lm_proj", local, hidden, True)
        self.lm_to_dit = self.linear("lm_to_dit_proj", hidden, dit, True)
        self.res_to_dit = self.linear("res_to_dit_proj", hidden, dit, True)
        self.fusion = self.linear("fusion_concat_proj", 2 * hidden, hidden, True)
        self.fsq_in = self.linear("fsq_layer.in_proj", hidden, c.fsq_latent_dim, True)
        self.fsq_out = self.linear("fsq_layer.out_proj", c.fsq_latent_dim, hidden, True)
        self.stop_proj = self.linear("stop_proj", hidden, hidden, True)
        self.stop_head = self.linear("stop_head", hidden, 2, False)

    def vector(self, name, count, mean, std):
        if self.source is not None:
            kind, values = self.source[name]
            assert kind == "BF16" and values.size == count, name
            return values
        return random_bf16(self.seed, tensor_id(name), count, mean, std)

    def matrix(self, names, outs, n_in, fused=True):
        if self.source is not None:
            parts = [self.source[n] for n in names]
            whole = all(o % 16 == 0 for o in outs) or not fused
            if all(kind == "Q8_0" for kind, _ in parts) and whole and n_in % 32 == 0:
                return Q8_0, np.concatenate([v for _, v in parts])
            rows = [v if kind == "BF16" else bf16_bits(q8_0_dequant(v, o, n_in))
                    for (kind, v), o in zip(parts, outs)]
            return BF16_ROWS, np.concatenate([r.reshape(-1) for r in rows])
        if self.q8:
            parts = [random_q8_0(self.seed, tensor_id(n), o, n_in, Q8_SCALE_STD) for n, o in zip(names, outs)]
            return Q8_0, np.concatenate(parts)
        parts = [random_bf16(self.seed, tensor_id(n), o * n_in, 0.0, MATRIX_STD) for n, o in zip(names, outs)]
        return BF16_ROWS, np.concatenate(parts)

    def linear(self, prefix, n_in, n_out, bias):
        fmt, w = self.matrix([prefix + ".weight"], [n_out], n_in, fused=False)
        b = self.vector(prefix + ".bias", n_out, 0.0, MATRIX_STD) if bias else None
        return Projection(fmt, w, b, n_in, n_out)

    def stack(self, prefix, s):
        cfg = _stack_config(s)
        h, q, kv = s.hidden, s.heads * s.head_dim, s.kv_heads * s.head_dim
        layers = []
        for i in range(s.layers):
            l = f"{prefix}.layers.{i}"
            a = l + ".self_attn."
            fmt, qkv = self.matrix([a + "q_proj.weight", a + "k_proj.weight", a + "v_proj.weight"],
                                   [q, kv, kv], h)
            gfmt, gate_up = self.matrix([l + ".mlp.gate_proj.weight", l + ".mlp.up_proj.weight"],
                                        [s.intermediate, s.intermediate], h)
            layers.append(dict(
                input_norm=self.vector(l + ".input_layernorm.weight", h, 1.0, 0.05),
                qkv=Projection(fmt, qkv, None, h, q + 2 * kv),
                o=self.linear(a + "o_proj", q, h, False),
                post_norm=self.vector(l + ".post_attention_layernorm.weight", h, 1.0, 0.05),
                gate_up=Projection(gfmt, gate_up, None, h, 2 * s.intermediate),
                down=self.linear(l + ".mlp.down_proj", s.intermediate, h, False),
            ))
        return Stack(cfg, layers, self.vector(prefix + ".norm.weight", h, 1.0, 0.05))


class Cache:
    """[layer][kv_head][capacity][head_dim] keys and values (float32; bf16
    caches keep bf16-rounded values)."""

    def __init__(self, cfg: dict, capacity: int, bf16: bool):
        shape = (cfg["layers"], cfg["kv_heads"], capacity, cfg["head_dim"])
        self.k = np.zeros(shape, np.float32)
        self.v = np.zeros(shape, np.float32)
        self.bf16 = bf16
        self.capacity = capacity


class OracleGenerator:
    """generator.cpp:82-538 on the CPU."""

    def __init__(self, config, seed: int = 0, q8: bool = True, bf16_cache: bool = False, threads: int = 0,
                 source: dict | None = None):
        self.c = config
        self.threads = threads
        self.bf16_cache = bf16_cache
        self.w = Weights(config, seed, q8, source)
        positions = max(config.max_length, 64)
        factors = np.array(list(config.rope_factors)[: config.lm.head_dim // 2], np.float64)
        self.rope = rope_table(config.rope_theta, config.lm.head_dim, factors, config.rope_scaling, positions)
        self.patch = config.patch_size
        self.feat = config.feat_dim
        self.base_cache = Cache(self.w.base_lm.config, config.max_length, bf16_cache)
        self.residual_cache = Cache(self.w.residual_lm.config, config.max_length, bf16_cache)
        dit_rows = 2 * (3 + 2 * self.patch)
        self.dit_cache = Cache(self.w.dit.config, dit_rows, bf16_cache)
        self.position = 0
        hidden = config.lm.hidden
        self.lm_hidden = np.zeros(hidden, np.float32)
        self.residual_hidden = np.zeros(hidden, np.float32)
        self.prefix_cond = np.zeros((self.patch, self.feat), np.float32)
        self.mu = np.zeros(2 * config.dit.hidden, np.float32)
        self.stop = np.zeros(2, np.float32)
        self.time_vectors: dict[float, np.ndarray] = {}
        # delta_time_mlp(sinusoid(0)) (generator.cpp:150-166)
        zero = sinusoid(0.0, config.dit.hidden)
        middle = self.project(self.w.delta_time_1, to_bf16(zero[None]), 1)
        self.delta_time = self.project(self.w.delta_time_2, to_bf16(middle, True), 1)[0]

    # ---------------------------------------------------------------- pieces

    def linear(self, p: Projection, x_bits, rows, y=None, accumulate=False):
        """Bf16Gemm::Linear (gemm.cpp:259-313) in the oracle's fp32 form."""
        return linear(np.asarray(x_bits).reshape(rows, p.n_in), p.format, p.weight, rows, p.n_in, p.n_out,
                      y=y, accumulate=accumulate, threads=self.threads)

    def project(self, p: Projection, x_bits, rows):
        """transformer.cpp:47-53"""
        y = self.linear(p, x_bits, rows)
        return add_bias(y, p.bias) if p.bias is not None else y

    def forward_stack(self, stack: Stack, rope: bool, layout: dict, cache: Cache, hidden: np.ndarray):
        """transformer.cpp:55-100; `hidden` [rows][width] updated in place;
        returns the final norm's fp32 output."""
        cfg = stack.config
        rows = hidden.shape[0]
        heads, kv, d = cfg["heads"], cfg["kv_heads"], cfg["head_dim"]
        for index, layer in enumerate(stack.layers):
            normed, _ = rms_norm(hidden, layer["input_norm"], cfg["rms_eps"])
            qkv = self.linear(layer["qkv"], normed, rows)
            kc, vc = cache.k[index], cache.v[index]
            q = qkv_rope(qkv, self.rope if (rope and cfg["rope"]) else None, layout["positions"],
                         layout["cache_rows"], kc, vc, heads, kv, d)
            if cache.bf16:
                for r in layout["cache_rows"]:
                    kc[:, r] = bf16_value(bf16_bits(kc[:, r])).reshape(kc[:, r].shape)
                    vc[:, r] = bf16_value(bf16_bits(vc[:, r])).reshape(vc[:, r].shape)
            att = attention(q, kc, vc, layout["rows_per_sequence"], layout["keys_per_sequence"],
                            layout["past"], layout["causal"], heads, kv, d)
            self.linear(layer["o"], att, rows, y=hidden, accumulate=True)
            normed, _ = rms_norm(hidden, layer["post_norm"], cfg["rms_eps"])
            gate_up = self.linear(layer["gate_up"], normed, rows)
            act = swiglu(gate_up)
            self.linear(layer["down"], act, rows, y=hidden, accumulate=True)
        _, out = rms_norm(hidden, stack.norm, cfg["rms_eps"], want_f32=True)
        return out

    def time_vector(self, t: float) -> np.ndarray:
        """generator.cpp:212-237"""
        key = float(np.float32(t))
        if key not in self.time_vectors:
            width = self.c.dit.hidden
            s = sinusoid(key, width)
            middle = self.project(self.w.time_1, to_bf16(s[None]), 1)
            vector = self.delta_time[None].copy()
            self.linear(self.w.time_2, to_bf16(middle, True), 1, y=vector, accumulate=True)
            self.time_vectors[key] = add_bias(vector, self.w.time_2.bias)[0]
        return self.time_vectors[key]

    def dit_cond(self):
        return self.project(self.w.dit_cond, to_bf16(self.prefix_cond), self.patch)

    def evaluate_dit(self, x: np.ndarray, t: float, cond_rows: np.ndarray) -> np.ndarray:
        """generator.cpp:297-324 -> velocity [2][patch][feat]."""
        p = self.patch
        rows = 2 * (3 + 2 * p)
        x_rows = self.project(self.w.dit_in, to_bf16(x), p)
        hidden = assemble_dit(self.mu.reshape(2, -1), self.time_vector(t), cond_rows, x_rows, p)
        length = rows // 2
        layout = dict(positions=np.arange(rows) % length, cache_rows=np.arange(rows), rows_per_sequence=length,
                      keys_per_sequence=length, past=0, causal=False)
        out = self.forward_stack(self.w.dit, True, layout, self.dit_cache, hidden)
        idx = [s * length + 3 + p + i for s in range(2) for i in range(p)]
        gathered = gather_rows(out, idx)
        return self.project(self.w.dit_out, to_bf16(gathered), 2 * p).reshape(2, p, self.feat)

    def velocity(self, mu, cond, x, t):
        """generator.cpp:515-538"""
        self.mu = _f32(mu).reshape(-1).copy()
        self.prefix_cond = _f32(cond).reshape(self.patch, self.feat).copy()
        return self.evaluate_dit(_f32(x).reshape(self.patch, self.feat), t, self.dit_cond())

    def euler(self, x: np.ndarray, timesteps: int, cfg: float, cond_rows: np.ndarray) -> np.ndarray:
        """generator.cpp:457-463 (CFG-Zero*: the skipped step leaves x)."""
        x = _f32(x).reshape(-1).copy()
        ts, dts, evaluate = euler_schedule(timesteps)
        for t, dt, ev in zip(ts, dts, evaluate):
            if not ev:
                continue
            v = self.evaluate_dit(x.reshape(self.patch, self.feat), float(t), cond_rows)
            x = guided_euler(v.reshape(2, -1), x, cfg, float(dt))
        return x.reshape(self.patch, self.feat)

    def dit_patch(self, mu, cond, noise, timesteps=10, cfg=2.0):
        self.mu = _f32(mu).reshape(-1).copy()
        self.prefix_cond = _f32(cond).reshape(self.patch, self.feat).copy()
        return self.euler(noise, timesteps, cfg, self.dit_cond())

    def encode(self, latents: np.ndarray, patches: int) -> np.ndarray:
        """generator.cpp:252-295 -> embeddings [patches][lm hidden]."""
        p = self.patch
        width = self.c.encoder.hidden
        rows = patches * (p + 1)
        a = self.project(self.w.encoder_in, to_bf16(_f32(latents).reshape(patches * p, self.feat)), patches * p)
        b = prepend_special(a, self.w.special, patches, p)
        cache = Cache(self.w.encoder.config, max(rows, 64), self.bf16_cache)
        layout = dict(positions=np.arange(rows) % (p + 1), cache_rows=np.arange(rows), rows_per_sequence=p + 1,
                      keys_per_sequence=p + 1, past=0, causal=False)
        out = self.forward_stack(self.w.encoder, True, layout, cache, b)
        firsts = gather_rows(out, [i * (p + 1) for i in range(patches)])
        assert firsts.shape == (patches, width)
        return self.project(self.w.enc_to_lm, to_bf16(firsts), patches)

    def fsq(self, x: np.ndarray, rows: int) -> np.ndarray:
        """generator.cpp:239-250"""
        latent = self.project(self.w.fsq_in, to_bf16(x), rows)
        return self.project(self.w.fsq_out, quantize(latent, self.c.fsq_scale), rows)

    # ---------------------------------------------------------------- sequence

    def prefill(self, tokens, text_mask, audio_mask, feats):
        """generator.cpp:326-422"""
        tokens, text_mask, audio_mask = (np.asarray(a, np.int32) for a in (tokens, text_mask, audio_mask))
        rows = tokens.size
        hidden = self.c.lm.hidden
        feats = _f32(feats).reshape(rows, self.patch * self.feat)
        if self.w.embed is not None:
            table = bf16_value(self.w.embed).reshape(self.c.vocab, hidden)
            combined = np.where(text_mask[:, None] != 0, table[np.clip(tokens, 0, self.c.vocab - 1)], 0.0)
            combined = combined.astype(np.float32)
        else:
            combined = np.zeros((rows, hidden), np.float32)
        audio_embeds = np.zeros((rows, hidden), np.float32)
        audio_rows = np.nonzero(audio_mask)[0]
        if audio_rows.size:
            emb = self.encode(feats[audio_rows], audio_rows.size)
            combined[audio_rows] = emb
            audio_embeds[audio_rows] = emb
        layout = dict(positions=np.arange(rows), cache_rows=np.arange(rows), rows_per_sequence=rows,
                      keys_per_sequence=0, past=0, causal=True)
        lm_out = self.forward_stack(self.w.base_lm, True, layout, self.base_cache, combined)
        self.lm_output = lm_out[-1].copy()
        quantized = self.fsq(lm_out, rows)
        selected = np.where(audio_mask[:, None] != 0, quantized, lm_out).astype(np.float32)
        self.lm_hidden = selected[-1].copy()
        residual_in = self.project(self.w.fusion, concat_rows(selected, audio_embeds), rows)
        res_out = self.forward_stack(self.w.residual_lm, False, layout, self.residual_cache, residual_in)
        self.residual_hidden = res_out[-1].copy()
        self.prefix_cond = feats[-1].reshape(self.patch, self.feat).copy()
        self.position = rows

    def step(self, noise, timesteps=10, cfg=2.0):
        """generator.cpp:424-513 -> (latent [patch][feat], stop logits [2])."""
        hidden = self.c.lm.hidden
        dit = self.c.dit.hidden
        lm_bits = to_bf16(self.lm_hidden[None])
        mu_lm = self.project(self.w.lm_to_dit, lm_bits, 1)[0]
        stop_a = self.project(self.w.stop_proj, lm_bits, 1)
        self.stop = self.project(self.w.stop_head, to_bf16(stop_a, True), 1)[0]
        mu_res = self.project(self.w.res_to_dit, to_bf16(self.residual_hidden[None]), 1)[0]
        self.mu = np.concatenate([mu_lm, mu_res]).astype(np.float32)
        assert self.mu.size == 2 * dit
        x = self.euler(noise, timesteps, cfg, self.dit_cond())
        stop = self.stop.copy()
        self.prefix_cond = x.copy()
        embed = self.encode(x[None], 1)[0]
        pos = self.position
        layout = dict(positions=[pos], cache_rows=[pos], rows_per_sequence=1, keys_per_sequence=0, past=pos,
                      causal=True)
        lm_out = self.forward_stack(self.w.base_lm, True, layout, self.base_cache, embed[None].copy())
        self.lm_output = lm_out[0].copy()
        self.lm_hidden = self.fsq(lm_out, 1)[0]
        fused = self.project(self.w.fusion, concat_rows(self.lm_hidden[None], embed[None]), 1)
        self.residual_hidden = self.forward_stack(self.w.residual_lm, False, layout, self.residual_cache,
                                                  fused)[0]
        self.position += 1
        assert self.residual_hidden.size == hidden
        return x, stop
