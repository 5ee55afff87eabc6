"""Seeded synthetic GPT-OSS-shaped model containers in picchio's on-disk format.

The container is the one picchio's loader reads (picchio.c:2852-2912 file
discovery, picchio.c:2385-2650 dense tensors, picchio.c:698-888 experts):
``config.json`` plus ``model-00000.safetensors`` holding

* ``model.embed_tokens.weight`` / ``lm_head.weight``: I8 [V, D] + ``.qs`` F32 [V]
* ``model.norm.weight``: F32 [D]
* per layer ``model.layers.L.``:
  ``input_layernorm.weight`` / ``post_attention_layernorm.weight`` F32 [D];
  ``self_attn.{q,k,v,o}_proj.weight`` as I8 + ``.qs`` (default), F32, or
  U8 INT4 + ``.qs``; ``self_attn.{q,k,v,o}_proj.bias`` F32;
  ``self_attn.sinks`` F32 [H]; ``mlp.router.weight`` F32 [E, D];
  ``mlp.router.bias`` F32 [E]; ``mlp.experts.gate_up_proj_bias`` F32 [E, I2];
  ``mlp.experts.down_proj_bias`` F32 [E, D];
  per expert ``mlp.experts.gate_up_proj.E`` / ``mlp.experts.down_proj.E``
  U8 packed INT4 + ``.qs`` F32 group scales; or, with ``expert_format =
  "mxfp4"``, the checkpoint's own MXFP4 form instead:
  ``mlp.experts.gate_up_proj_blocks`` U8 [E, I2, D/32, 16] with
  ``..._scales`` U8 [E, I2, D/32] (E8M0), and the same for ``down_proj``.

Quantizers follow the reference converter (convert.py:45-93 INT4: amax/7
with a 1e-8 floor, round half to even, clip [-8, 7], low nibble = even
column; convert.py:106-126 INT8: amax/127, rint, clip [-127, 127]).
Weights are N(0, 0.02), router N(0, 0.1) (make_test_model.py:111), biases
N(0, 0.01), norm weights 1 + N(0, 0.05), sinks N(0, 0.5).  All draws come from
``numpy.random.default_rng(seed)`` in a fixed order, so a (config, seed)
pair always gives the same bytes.
"""
from __future__ import annotations

import json
import os
import struct
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, asdict, field

import numpy as np


@dataclass
class SynthConfig:
    """Model shape.  ``intermediate_size`` is half of the fused gate_up rows."""
    hidden_size: int = 256
    num_hidden_layers: int = 2
    num_attention_heads: int = 8
    num_key_value_heads: int = 2
    head_dim: int = 32
    intermediate_size: int = 256
    num_local_experts: int = 8
    num_experts_per_tok: int = 2
    vocab_size: int = 1024
    max_position_embeddings: int = 4096
    sliding_window: int = 128
    rms_norm_eps: float = 1e-5
    rope_theta: float = 150000.0
    swiglu_limit: float = 7.0
    layer_types: list = field(default_factory=lambda: ["sliding_attention", "full_attention"])
    # container options (not written to config.json)
    group_size: int = 32          # expert INT4 group size; 0 = per-row scale
    expert_format: str = "int4"   # "int4" | "mxfp4" (the checkpoint's own _blocks/_scales form)
    attn_format: str = "i8"       # "i8" | "f32" | "i4"
    attn_group_size: int = 0      # for attn_format == "i4"
    rope_scaling: dict | None = None  # e.g. {"rope_type": "yarn", "factor": 32.0, ...}

    def config_json(self) -> dict:
        d = {k: v for k, v in asdict(self).items()
             if k not in ("group_size", "attn_format", "attn_group_size", "rope_scaling", "expert_format")}
        d["model_type"] = "gpt_oss"
        d["attention_bias"] = True
        if self.rope_scaling:
            d["rope_scaling"] = dict(self.rope_scaling)
        return d


TINY = SynthConfig()


def quantize_int4(w: np.ndarray, group_size: int):
    """INT4 packing as convert.py:45-93 produces it -> (packed [O, ceil(I/2)], scales)."""
    O, I = w.shape
    if group_size <= 0 or group_size >= I:
        amax = np.max(np.abs(w), axis=1)
        sc = np.where(amax > 1e-8, amax / 7.0, 1e-8).astype(np.float32)
        q = np.clip(np.round(w / sc[:, None]), -8, 7).astype(np.int8)
        scales = sc
    elif I % group_size == 0:
        # whole groups: the loop below, one reshape at a time (same operations, same bits)
        ng = I // group_size
        blk = w.reshape(O, ng, group_size)
        amax = np.max(np.abs(blk), axis=2)
        scales = np.where(amax > 1e-8, amax / 7.0, 1e-8).astype(np.float32)
        q = np.clip(np.round(blk / scales[:, :, None]), -8, 7).astype(np.int8).reshape(O, I)
    else:
        ng = (I + group_size - 1) // group_size
        scales = np.empty((O, ng), dtype=np.float32)
        q = np.empty((O, I), dtype=np.int8)
        for g in range(ng):
            a, b = g * group_size, min((g + 1) * group_size, I)
            blk = w[:, a:b]
            amax = np.max(np.abs(blk), axis=1)
            sc = np.where(amax > 1e-8, amax / 7.0, 1e-8).astype(np.float32)
            scales[:, g] = sc
            q[:, a:b] = np.clip(np.round(blk / sc[:, None]), -8, 7).astype(np.int8)
    u = (q.astype(np.int16) + 8).astype(np.uint8)
    if I % 2:
        u = np.concatenate([u, np.full((O, 1), 8, np.uint8)], axis=1)
    packed = (u[:, 0::2] & 0xF) | ((u[:, 1::2] & 0xF) << 4)
    if I % 2:
        packed[:, -1] &= 0xF
    return packed.astype(np.uint8), scales


E2M1_MIDS = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)


def quantize_mxfp4(w: np.ndarray):
    """MXFP4 by the OCP microscaling rule, per 32-column block: shared
    exponent floor(log2 max|w|) - 2 (2 = the largest E2M1 exponent), clamped
    to [-127, 127] and stored as the E8M0 byte exp + 127; each w / 2^exp
    rounds to the nearest E2M1 value (0, 0.5, 1, 1.5, 2, 3, 4, 6; ties to the
    even code; saturating at 6), sign in bit 3.  Returns (blocks uint8 [O,
    I/32, 16], two codes per byte with the low nibble the even column, and
    scales uint8 [O, I/32]): the checkpoint layout convert.py:400-431 reads."""
    O, I = w.shape
    assert I % 32 == 0
    b = w.astype(np.float32).reshape(O, I // 32, 32)
    amax = np.abs(b).max(-1)
    bits = amax.view(np.uint32)
    ex = np.where(amax > 0, ((bits >> 23) & 0xFF).astype(np.int32) - 127 - 2, -127)
    ex = np.clip(ex, -127, 127)
    v = (b * np.ldexp(np.float32(1), -ex)[..., None].astype(np.float32)).astype(np.float32)
    a = np.abs(v)
    idx = np.searchsorted(E2M1_MIDS, a, side="left")  # mids strictly below a
    tie = (idx < 7) & (a == E2M1_MIDS[np.minimum(idx, 6)]) & ((idx & 1) == 1)
    idx = idx + tie
    code = (idx | np.where(v < 0, 8, 0)).astype(np.uint8).reshape(O, I)
    packed = (code[:, 0::2] | (code[:, 1::2] << 4)).astype(np.uint8).reshape(O, I // 32, 16)
    return packed, (ex + 127).astype(np.uint8)


def quantize_int8(w: np.ndarray):
    """Per-row INT8 as convert.py:106-126 produces it -> (q [O, I] int8, scales [O])."""
    amax = np.abs(w).max(axis=1)
    s = np.where(amax > 0, amax / 127.0, 1.0).astype(np.float32)
    q = np.clip(np.rint(w / s[:, None]), -127, 127).astype(np.int8)
    return q, s


_ST_DTYPES = {np.dtype(np.float32): "F32", np.dtype(np.int8): "I8",
              np.dtype(np.uint8): "U8", np.dtype(np.float16): "F16",
              np.dtype(np.int32): "I32"}


def write_safetensors(path: str, tensors: dict) -> None:
    """Minimal safetensors writer: u64 header length, JSON header, raw data."""
    header, offset, blobs = {}, 0, []
    for name, arr in tensors.items():
        arr = np.ascontiguousarray(arr)
        if arr.dtype.name == "bfloat16" or getattr(arr, "_st_dtype", None) == "BF16":
            dt = "BF16"
        else:
            dt = _ST_DTYPES[arr.dtype]
        nb = arr.nbytes
        header[name] = {"dtype": dt, "shape": list(arr.shape),
                        "data_offsets": [offset, offset + nb]}
        blobs.append(arr)
        offset += nb
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for a in blobs:
            f.write(a.tobytes())


def make_model(out_dir: str, cfg: SynthConfig = TINY, seed: int = 1234) -> dict:
    """Write ``config.json`` + ``model-00000.safetensors`` under ``out_dir``.

    Returns the float/quantized tensors as numpy arrays (same dict that was
    written), so tests can build oracle inputs without re-reading the file.
    """
    os.makedirs(out_dir, exist_ok=True)
    rng = np.random.default_rng(seed)
    D, L = cfg.hidden_size, cfg.num_hidden_layers
    H, KVH, hd = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    E, I2, V = cfg.num_local_experts, 2 * cfg.intermediate_size, cfg.vocab_size
    Iin = cfg.intermediate_size
    f32 = np.float32
    t: dict[str, np.ndarray] = {}

    def normal(shape, std):
        return (rng.standard_normal(shape, dtype=f32) * f32(std)).astype(f32)

    q, s = quantize_int8(normal((V, D), 0.02))
    t["model.embed_tokens.weight"], t["model.embed_tokens.weight.qs"] = q, s
    q, s = quantize_int8(normal((V, D), 0.02))
    t["lm_head.weight"], t["lm_head.weight.qs"] = q, s
    t["model.norm.weight"] = (1.0 + normal((D,), 0.05)).astype(f32)

    def put_dense(name, O, I):
        w = normal((O, I), 0.02)
        if cfg.attn_format == "f32":
            t[name] = w
        elif cfg.attn_format == "i8":
            t[name], t[name + ".qs"] = quantize_int8(w)
        elif cfg.attn_format == "i4":
            p, sc = quantize_int4(w, cfg.attn_group_size)
            t[name], t[name + ".qs"] = p, sc
        else:
            raise ValueError(cfg.attn_format)

    pool = ThreadPoolExecutor(max_workers=max(1, min(4, (os.cpu_count() or 1) - 1)))
    for l in range(L):
        p = f"model.layers.{l}."
        t[p + "input_layernorm.weight"] = (1.0 + normal((D,), 0.05)).astype(f32)
        t[p + "post_attention_layernorm.weight"] = (1.0 + normal((D,), 0.05)).astype(f32)
        put_dense(p + "self_attn.q_proj.weight", H * hd, D)
        put_dense(p + "self_attn.k_proj.weight", KVH * hd, D)
        put_dense(p + "self_attn.v_proj.weight", KVH * hd, D)
        put_dense(p + "self_attn.o_proj.weight", D, H * hd)
        t[p + "self_attn.q_proj.bias"] = normal((H * hd,), 0.01)
        t[p + "self_attn.k_proj.bias"] = normal((KVH * hd,), 0.01)
        t[p + "self_attn.v_proj.bias"] = normal((KVH * hd,), 0.01)
        t[p + "self_attn.o_proj.bias"] = normal((D,), 0.01)
        t[p + "self_attn.sinks"] = normal((H,), 0.5)
        t[p + "mlp.router.weight"] = normal((E, D), 0.1)
        t[p + "mlp.router.bias"] = normal((E,), 0.01)
        t[p + "mlp.experts.gate_up_proj_bias"] = normal((E, I2), 0.01)
        t[p + "mlp.experts.down_proj_bias"] = normal((E, D), 0.01)
        if cfg.expert_format == "mxfp4":
            # one aggregated tensor per projection, [E][rows][I/32][16] codes
            # and [E][rows][I/32] E8M0 scales
            gub, gus, dnb, dns = [], [], [], []
            for e in range(E):
                b_, s_ = quantize_mxfp4(normal((I2, D), 0.02))
                gub.append(b_)
                gus.append(s_)
                b_, s_ = quantize_mxfp4(normal((D, Iin), 0.02))
                dnb.append(b_)
                dns.append(s_)
            t[p + "mlp.experts.gate_up_proj_blocks"] = np.stack(gub)
            t[p + "mlp.experts.gate_up_proj_scales"] = np.stack(gus)
            t[p + "mlp.experts.down_proj_blocks"] = np.stack(dnb)
            t[p + "mlp.experts.down_proj_scales"] = np.stack(dns)
            continue
        # draws stay in order on this thread; the quantization of each
        # matrix runs on a worker while the next one is drawn
        # (at most LAG experts in flight, which bounds the float copies held)
        LAG = 4
        futs = {}

        def collect(e):
            pk, sc = futs[e][0].result()
            t[p + f"mlp.experts.gate_up_proj.{e}"] = pk
            t[p + f"mlp.experts.gate_up_proj.{e}.qs"] = sc
            pk, sc = futs.pop(e)[1].result()
            t[p + f"mlp.experts.down_proj.{e}"] = pk
            t[p + f"mlp.experts.down_proj.{e}.qs"] = sc

        for e in range(E):
            futs[e] = (pool.submit(quantize_int4, normal((I2, D), 0.02), cfg.group_size),
                       pool.submit(quantize_int4, normal((D, Iin), 0.02), cfg.group_size))
            if e >= LAG:
                collect(e - LAG)
        for e in range(max(0, E - LAG), E):
            collect(e)

    pool.shutdown()
    write_safetensors(os.path.join(out_dir, "model-00000.safetensors"), t)
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(cfg.config_json(), f, indent=1)
    return t


def random_prompt(n: int, vocab: int, seed: int = 7) -> list[int]:
    """Uniform random token ids in [0, vocab)."""
    return [int(v) for v in np.random.default_rng(seed).integers(0, vocab, size=n)]


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("out_dir")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--group-size", type=int, default=32)
    ap.add_argument("--attn-format", default="i8", choices=["i8", "f32", "i4"])
    a = ap.parse_args()
    make_model(a.out_dir, SynthConfig(group_size=a.group_size, attn_format=a.attn_format), a.seed)
    print("wrote", a.out_dir)
