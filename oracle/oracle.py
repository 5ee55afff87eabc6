"""CPU oracle for picchio's per-token MoE hot path (TEST INFRASTRUCTURE ONLY).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import
this module, and only as the checker.  It drives ``oracle.c`` (built into
``oracle/_build/liboracle.so``), the plain-C restatement of the reference's
arithmetic, through ctypes, and restates the reference's forward driver
(picchio.c:1655-1756 ``forward_token``; picchio.c:349-425 ``cfg_load``;
picchio.c:2385-2650 weight loading; picchio.c:698-888 expert loading) in
Python on top of it.  When the reference itself has been built here
(``oracle/_ref/``) :func:`ref_lib` exposes its own functions for pinning.
"""
from __future__ import annotations

import ctypes as C
import json
import math
import os
import re
import struct
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libpicchio_ref.so")
REF_BIN_PATH = os.path.join(HERE, "_ref", "picchio")

_fp = C.POINTER(C.c_float)
_i8p = C.POINTER(C.c_int8)
_u8p = C.POINTER(C.c_uint8)
_ip = C.POINTER(C.c_int)


def reference_dir():
    """The reference's source directory: the REF environment variable, else
    the ``reference_path`` of the repository's BASELINE.json; None when
    neither names an existing directory (e.g. on a GPU box, which only gets
    the prebuilt oracle/_ref)."""
    cand = os.environ.get("REF")
    if not cand:
        try:
            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
                cand = json.load(f).get("reference_path")
        except (OSError, ValueError):
            cand = None
    return cand if cand and os.path.isfile(os.path.join(cand, "picchio.c")) else None


def build(ref: bool = False) -> None:
    """Compile the oracle (and, with ref=True, the reference from
    reference_dir()) via oracle/Makefile."""
    args = ["make", "-s", "-C", HERE, "oracle"]
    if ref:
        src = reference_dir()
        if src is None:
            raise RuntimeError("reference sources not found: set REF to the reference checkout")
        args += ["ref", f"REF={src}"]
    subprocess.run(args, check=True)


def _ptr(a: np.ndarray, t):
    return a.ctypes.data_as(t)


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        L.or_matmul_f32.argtypes = [_fp, _fp, _fp, C.c_int, C.c_int, C.c_int]
        L.or_matmul_q8.argtypes = [_fp, _fp, _i8p, _fp, C.c_int, C.c_int, C.c_int]
        L.or_matmul_i4.argtypes = [_fp, _fp, _u8p, _fp, C.c_int, C.c_int, C.c_int]
        L.or_matmul_i4_gs.argtypes = [_fp, _fp, _u8p, _fp, C.c_int, C.c_int, C.c_int, C.c_int]
        L.or_dequant_i4.argtypes = [_fp, _u8p, _fp, C.c_int, C.c_int, C.c_int]
        L.or_dequant_i8.argtypes = [_fp, _i8p, _fp, C.c_int, C.c_int]
        L.or_quantize_rows_i4.argtypes = [_fp, _u8p, _fp, C.c_int, C.c_int]
        L.or_rmsnorm.argtypes = [_fp, _fp, _fp, C.c_int, C.c_float]
        L.or_softmax.argtypes = [_fp, C.c_int]
        L.or_router_topk.argtypes = [_fp, _fp, _fp, C.c_int, C.c_int, C.c_int, C.c_int,
                                     _fp, _ip, _fp]
        L.or_swiglu.argtypes = [_fp, _fp, C.c_int, C.c_float, C.c_float]
        L.or_yarn_inv_freq.argtypes = [C.c_int, C.c_float, C.c_float, C.c_float, C.c_float,
                                       C.c_int, C.c_int, C.c_int]
        L.or_yarn_inv_freq.restype = C.c_float
        L.or_rope_cs.argtypes = [_fp, C.c_int, C.c_int, C.c_float, _fp, _fp]
        L.or_rope_rotate.argtypes = [_fp, C.c_int, _fp, _fp]
        L.or_attention.argtypes = [_fp, _fp, _fp, _fp, _fp, C.c_int, C.c_int, C.c_int,
                                   C.c_int, C.c_int]
        L.or_axpy.argtypes = [_fp, _fp, C.c_float, C.c_int]
        L.or_argmax.argtypes = [_fp, C.c_int]
        L.or_argmax.restype = C.c_int
        L.or_sample.argtypes = [_fp, C.c_int, C.c_float, C.c_float, C.c_int, C.c_float, _ip, _ip,
                                C.POINTER(C.c_uint64)]
        L.or_sample.restype = C.c_int
        _lib = L
    return _lib


def ref_lib():
    """The reference's own functions (oracle/_ref/libpicchio_ref.so) or None."""
    global _ref
    if _ref is None and os.path.exists(REF_LIB_PATH):
        R = C.CDLL(REF_LIB_PATH)
        R.ref_matmul_f32.argtypes = [_fp, _fp, _fp, C.c_int, C.c_int, C.c_int]
        R.ref_matmul_q8.argtypes = [_fp, _fp, _i8p, _fp, C.c_int, C.c_int, C.c_int]
        R.ref_matmul_i4.argtypes = [_fp, _fp, _u8p, _fp, C.c_int, C.c_int, C.c_int]
        R.ref_matmul_i4_gs.argtypes = [_fp, _fp, _u8p, _fp, C.c_int, C.c_int, C.c_int, C.c_int]
        R.ref_quantize_rows_i4.argtypes = [_fp, _u8p, _fp, C.c_int, C.c_int]
        R.ref_rmsnorm.argtypes = [_fp, _fp, _fp, C.c_int, C.c_float]
        R.ref_softmax.argtypes = [_fp, C.c_int]
        R.ref_sigmoidf.argtypes = [C.c_float]
        R.ref_sigmoidf.restype = C.c_float
        R.ref_rope_apply.argtypes = [_fp, _fp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                                     C.c_float, C.c_float, C.c_float, C.c_int, C.c_int]
        R.ref_yarn_inv_freq.argtypes = [C.c_int, C.c_float, C.c_float, C.c_float, C.c_float,
                                        C.c_int, C.c_int, C.c_int]
        R.ref_yarn_inv_freq.restype = C.c_float
        if hasattr(R, "ref_sample_logits"):
            R.ref_sample_logits.argtypes = [_fp, C.c_int, C.c_float, C.c_float, C.c_int, C.c_float, _ip, _ip,
                                            C.POINTER(C.c_uint64)]
            R.ref_sample_logits.restype = C.c_int
        _ref = R
    return _ref


# ----------------------------------------------------------------------------
# numpy-facing wrappers (inputs are converted to contiguous arrays)
# ----------------------------------------------------------------------------

def _f(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def matmul_i4_gs(x, q4, scales, O, I, gs):
    """y[S, O] for group-scaled INT4 (quant.h:259-319)."""
    x = _f(x).reshape(-1, I)
    y = np.empty((x.shape[0], O), np.float32)
    lib().or_matmul_i4_gs(_ptr(y, _fp), _ptr(x, _fp), _ptr(np.ascontiguousarray(q4, np.uint8), _u8p),
                          _ptr(_f(scales), _fp), x.shape[0], I, O, gs)
    return y


def matmul_i4(x, q4, scales, O, I):
    """y[S, O] for per-row INT4 (quant.h:191-253)."""
    x = _f(x).reshape(-1, I)
    y = np.empty((x.shape[0], O), np.float32)
    lib().or_matmul_i4(_ptr(y, _fp), _ptr(x, _fp), _ptr(np.ascontiguousarray(q4, np.uint8), _u8p),
                       _ptr(_f(scales), _fp), x.shape[0], I, O)
    return y


def matmul_q8(x, q, scales, O, I):
    """y[S, O] for per-row INT8 (quant.h:152-186)."""
    x = _f(x).reshape(-1, I)
    y = np.empty((x.shape[0], O), np.float32)
    lib().or_matmul_q8(_ptr(y, _fp), _ptr(x, _fp), _ptr(np.ascontiguousarray(q, np.int8), _i8p),
                       _ptr(_f(scales), _fp), x.shape[0], I, O)
    return y


def matmul_f32(x, W, O, I):
    """y[S, O] for fp32 weights (quant.h:117-148)."""
    x = _f(x).reshape(-1, I)
    y = np.empty((x.shape[0], O), np.float32)
    lib().or_matmul_f32(_ptr(y, _fp), _ptr(x, _fp), _ptr(_f(W), _fp), x.shape[0], I, O)
    return y


def dequant_i4(q4, scales, O, I, gs):
    out = np.empty((O, I), np.float32)
    lib().or_dequant_i4(_ptr(out, _fp), _ptr(np.ascontiguousarray(q4, np.uint8), _u8p),
                        _ptr(_f(scales), _fp), O, I, gs)
    return out


def dequant_i8(q, scales, O, I):
    out = np.empty((O, I), np.float32)
    lib().or_dequant_i8(_ptr(out, _fp), _ptr(np.ascontiguousarray(q, np.int8), _i8p),
                        _ptr(_f(scales), _fp), O, I)
    return out


def rmsnorm(x, w, eps):
    x = _f(x)
    out = np.empty_like(x)
    lib().or_rmsnorm(_ptr(out, _fp), _ptr(x, _fp), _ptr(_f(w), _fp), x.size, eps)
    return out


def router_topk(x, R, bias, K, bias_first=False):
    """(logits[E], sel[K], weights[K]) as moe_forward computes them."""
    E, D = R.shape
    logits = np.empty(E, np.float32)
    sel = np.empty(K, np.int32)
    w = np.empty(K, np.float32)
    b = _f(bias) if bias is not None else None
    lib().or_router_topk(_ptr(_f(x), _fp), _ptr(_f(R), _fp), _ptr(b, _fp) if b is not None else None,
                         E, D, K, int(bias_first), _ptr(logits, _fp), _ptr(sel, _ip), _ptr(w, _fp))
    return logits, sel, w


def swiglu(gu, limit, alpha=1.702):
    gu = _f(gu)
    act = np.empty(gu.size // 2, np.float32)
    lib().or_swiglu(_ptr(act, _fp), _ptr(gu, _fp), gu.size, limit, alpha)
    return act


def argmax(logits):
    return int(lib().or_argmax(_ptr(_f(logits), _fp), logits.size))


class SamplerState:
    """The sampler's mutable globals (picchio.c:1516-1520): the repetition
    history (at most 4096 ids) and the xorshift64 state."""

    def __init__(self, rng: int, history=()):
        self.rng = int(rng)
        self.history = [int(t) for t in history][:4096]

    def copy(self):
        return SamplerState(self.rng, self.history)


def _sample_with(fn, logits, temperature, top_p, top_k, rep, state: SamplerState):
    lg = _f(logits).copy()
    hist = np.zeros(4096, np.int32)
    hist[:len(state.history)] = state.history
    hl = C.c_int(len(state.history))
    rng = C.c_uint64(state.rng)
    tid = int(fn(_ptr(lg, _fp), lg.size, float(temperature), float(top_p), int(top_k), float(rep),
                 _ptr(hist, _ip), C.byref(hl), C.byref(rng)))
    state.rng = int(rng.value)
    state.history = hist[:hl.value].tolist()
    return tid, lg


def sample(logits, temperature, top_p, top_k, rep, state: SamplerState):
    """sample_logits (picchio.c:1540-1649) restated (oracle.c or_sample):
    returns (id, the logits array as the reference leaves it); updates state."""
    return _sample_with(lib().or_sample, logits, temperature, top_p, top_k, rep, state)


def ref_sample(logits, temperature, top_p, top_k, rep, state: SamplerState):
    """The reference's own sample_logits (oracle/_ref), same contract as sample()."""
    R = ref_lib()
    if R is None or not hasattr(R, "ref_sample_logits"):
        raise RuntimeError("the reference library is not built (oracle/_ref)")
    return _sample_with(R.ref_sample_logits, logits, temperature, top_p, top_k, rep, state)


# ----------------------------------------------------------------------------
# container reading + config (restating picchio.c:349-425 and json.h)
# ----------------------------------------------------------------------------

_DT = {"F32": np.float32, "F16": np.float16, "I8": np.int8, "U8": np.uint8,
       "I32": np.int32, "I16": np.int16, "F64": np.float64, "BF16": np.uint16}


def read_safetensors(path: str) -> dict:
    """name -> (dtype string, numpy array) for every tensor in one file."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        hdr = json.loads(f.read(n))
        data = f.read()
    out = {}
    for name, m in hdr.items():
        if name == "__metadata__":
            continue
        a, b = m["data_offsets"]
        arr = np.frombuffer(data[a:b], dtype=_DT[m["dtype"]]).reshape(m["shape"])
        out[name] = (m["dtype"], arr)
    return out


def _json_find(js: str, key: str):
    """json_find_key (json.h:42-62): first '"key"' followed by ':' anywhere."""
    p = 0
    while True:
        p = js.find(key, p)
        if p < 0:
            return None
        if p > 0 and js[p - 1] == '"' and js[p + len(key):p + len(key) + 1] == '"':
            q = p + len(key) + 1
            while q < len(js) and js[q].isspace():
                q += 1
            if q < len(js) and js[q] == ":":
                return js[q + 1:].lstrip()
        p += 1


def _atoi(s: str) -> int:
    m = re.match(r"\s*[+-]?\d+", s)
    return int(m.group(0)) if m else 0


def _atof(s: str) -> float:
    m = re.match(r"\s*[+-]?(\d+\.?\d*([eE][+-]?\d+)?|\.\d+([eE][+-]?\d+)?)", s)
    return float(m.group(0)) if m else 0.0


@dataclass
class Cfg:
    hidden: int; n_layers: int; n_heads: int; n_kv_heads: int; head_dim: int
    n_experts: int; topk: int; moe_inter: int; vocab: int; ctx_len: int
    sliding_window: int; eps: float; theta: float; rope_factor: float
    rope_beta_fast: float; rope_beta_slow: float; rope_original_ctx: int
    rope_truncate: int; rope_attn_factor: float; swiglu_limit: float
    swiglu_alpha: float; routed_scale: float; has_attn_bias: int; layer_type: list


def cfg_load(model_dir: str) -> Cfg:
    """cfg_load (picchio.c:349-425) over json.h's key search semantics."""
    js = open(os.path.join(model_dir, "config.json")).read()

    def gi(k, d):
        v = _json_find(js, k)
        return d if v is None or v.startswith("n") else _atoi(v)

    def gf(k, d):
        v = _json_find(js, k)
        return np.float32(d) if v is None or v.startswith("n") else np.float32(_atof(v))

    def gb(k, d):
        v = _json_find(js, k)
        if v is None:
            return d
        return 1 if v.startswith("t") else 0 if v.startswith("f") else d

    L = gi("num_hidden_layers", 36)
    ctx = gi("max_position_embeddings", 131072)
    factor = gf("factor", 1.0)
    lt = [i % 2 for i in range(L)]
    v = _json_find(js, "layer_types")
    if v is not None and v.startswith("["):
        names = re.findall(r'"([^"]*)"', v[:v.find("]")])
        if names:
            lt = [1 if "full" in names[i % len(names)] else 0 for i in range(L)]
    attn_factor = np.float32(np.float32(0.1) * np.float32(math.log(factor)) + np.float32(1.0)) \
        if factor > 1.0 else np.float32(1.0)
    return Cfg(hidden=gi("hidden_size", 2880), n_layers=L, n_heads=gi("num_attention_heads", 64),
               n_kv_heads=gi("num_key_value_heads", 8), head_dim=gi("head_dim", 64),
               n_experts=gi("num_local_experts", 128), topk=gi("num_experts_per_tok", 4),
               moe_inter=gi("intermediate_size", 2880) * 2, vocab=gi("vocab_size", 201088),
               ctx_len=ctx, sliding_window=gi("sliding_window", 128), eps=gf("rms_norm_eps", 1e-5),
               theta=gf("rope_theta", 150000.0), rope_factor=factor,
               rope_beta_fast=gf("beta_fast", 32.0), rope_beta_slow=gf("beta_slow", 1.0),
               rope_original_ctx=gi("original_max_position_embeddings", ctx),
               rope_truncate=gb("truncate", 1), rope_attn_factor=attn_factor,
               swiglu_limit=gf("swiglu_limit", 7.0), swiglu_alpha=np.float32(1.702),
               routed_scale=gf("routed_scaling_factor", 1.0),
               has_attn_bias=gb("attention_bias", 1), layer_type=lt)


class QT:
    """A weight as the reference holds it (quant.h:32-41): fmt 0/1/2."""

    def __init__(self, fmt, O, I, data, s=None, block_size=0):
        self.fmt, self.O, self.I, self.data, self.s, self.block_size = fmt, O, I, data, s, block_size

    def matmul(self, x):
        if self.fmt == 0:
            return matmul_f32(x, self.data, self.O, self.I)
        if self.fmt == 1:
            return matmul_q8(x, self.data, self.s, self.O, self.I)
        if self.block_size > 0:
            return matmul_i4_gs(x, self.data, self.s, self.O, self.I, self.block_size)
        return matmul_i4(x, self.data, self.s, self.O, self.I)


def _load_qt(t: dict, name: str, O: int, I: int) -> QT:
    """load_qt_i4 (picchio.c:2441-2527) for the U8 / I8 / F32 cases."""
    dt, arr = t[name]
    if dt == "U8":
        qs = t.get(name + ".qs")
        if qs is None:
            return QT(2, O, I, arr.reshape(-1), np.ones(O, np.float32), 0)
        n = qs[1].size
        bs = (O * I) // n if n > O else 0
        if n > O and bs <= 0:
            bs = 64
        return QT(2, O, I, arr.reshape(-1), qs[1].reshape(-1).astype(np.float32), bs)
    if dt == "I8":
        return QT(1, O, I, arr.reshape(O, I), t[name + ".qs"][1].reshape(-1).astype(np.float32))
    if dt == "F32":
        return QT(0, O, I, arr.reshape(O, I).astype(np.float32))
    raise ValueError(f"{name}: dtype {dt} not handled by the oracle")


# E2M1 values of the 16 codes (convert.py:98-103), code 8 is -0.0
FP4_LUT = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                    -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], np.float32)


def dequant_mxfp4(packed, e8m0, O, I):
    """MXFP4 -> fp32 exactly as convert.py dequantizes it before its INT4
    requantization (convert.py:413-431, decode_e8m0 convert.py:129-134):
    two codes per byte (low nibble = even column), value = FP4_LUT[code] *
    2^(e - 127) as one float32 multiply."""
    b = np.asarray(packed, np.uint8).reshape(O, I // 2)
    codes = np.empty((O, I), np.uint8)
    codes[:, 0::2] = b & 0x0F
    codes[:, 1::2] = b >> 4
    vals = FP4_LUT[codes]
    sc = np.ldexp(np.ones((O, I // 32), np.float32), np.asarray(e8m0).reshape(O, I // 32).astype(np.int32) - 127)
    return (vals * np.repeat(sc.astype(np.float32), 32, axis=1)).astype(np.float32)


def bf16_round(a):
    """fp32 -> bf16 -> fp32 with round-to-nearest-even (what the device's
    __float2bfloat16_rn stores), for finite values."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


class OracleModel:
    """forward_token (picchio.c:1655-1756) restated over oracle.c.

    The KV cache is fp32, as the reference keeps it (picchio.c:142-151).
    With kv_bf16 every stored K and V row is rounded to bf16 first: the
    device's bf16 cache, the one departure from the reference's arithmetic,
    restated so that the device's bf16 path has an oracle of its own.
    ``forward_token`` returns the greedy next id; ``self.dumps`` holds the
    stage tensors of the last call under the reference's ORACLE_DIR names
    (picchio.c:204-249).
    """

    def __init__(self, model_dir: str, ctx: int = 512, kv_bf16: bool = False):
        self.kv_bf16 = kv_bf16
        self.c = c = cfg_load(model_dir)
        t = {}
        for fn in sorted(os.listdir(model_dir)):
            if fn.endswith(".safetensors"):
                for k, v in read_safetensors(os.path.join(model_dir, fn)).items():
                    t.setdefault(k, v)
        self.t = t
        D, H, KVH, hd = c.hidden, c.n_heads, c.n_kv_heads, c.head_dim
        self.max_pos = min(ctx, c.ctx_len)
        self.embed = _load_qt(t, "model.embed_tokens.weight", c.vocab, D)
        self.lm_head = _load_qt(t, "lm_head.weight", c.vocab, D)
        self.final_norm = t["model.norm.weight"][1].astype(np.float32)
        self.layers = []
        for l in range(c.n_layers):
            p = f"model.layers.{l}."
            g = lambda n: t[p + n][1].astype(np.float32) if (p + n) in t else None
            ly = dict(in_ln=g("input_layernorm.weight"), post_ln=g("post_attention_layernorm.weight"),
                      wq=_load_qt(t, p + "self_attn.q_proj.weight", H * hd, D),
                      wk=_load_qt(t, p + "self_attn.k_proj.weight", KVH * hd, D),
                      wv=_load_qt(t, p + "self_attn.v_proj.weight", KVH * hd, D),
                      wo=_load_qt(t, p + "self_attn.o_proj.weight", D, H * hd),
                      bq=g("self_attn.q_proj.bias"), bk=g("self_attn.k_proj.bias"),
                      bv=g("self_attn.v_proj.bias"), bo=g("self_attn.o_proj.bias"),
                      sinks=g("self_attn.sinks"), router=g("mlp.router.weight").reshape(c.n_experts, D),
                      router_bias=g("mlp.router.bias"), layer_type=c.layer_type[l],
                      gu_bias=g("mlp.experts.gate_up_proj_bias"), d_bias=g("mlp.experts.down_proj_bias"))
            ly["experts"] = {}
            self.layers.append(ly)
        inv = np.array([lib().or_yarn_inv_freq(hd, c.theta, c.rope_factor, c.rope_beta_fast,
                                               c.rope_beta_slow, c.rope_original_ctx,
                                               c.rope_truncate, j) for j in range(hd // 2)],
                       np.float32)
        self.inv_freq = inv
        kvd = KVH * hd
        self.K = [np.zeros((self.max_pos, kvd), np.float32) for _ in range(c.n_layers)]
        self.V = [np.zeros((self.max_pos, kvd), np.float32) for _ in range(c.n_layers)]
        self.dumps: dict = {}

    def expert(self, l: int, e: int):
        """(gate_up QT, down QT, gu_bias, d_bias) as expert_load gives them
        (picchio.c:698-888).  Experts in the checkpoint's MXFP4 form
        (``<proj>_blocks`` / ``<proj>_scales``, which the reference only
        reaches after convert.py turns them into INT4) are dequantized as
        convert.py does and applied with the reference's fp32 matmul
        (matmul_f32, quant.h:117-148): the reference's fmt 3 semantics."""
        ly = self.layers[l]
        if e not in ly["experts"]:
            c, t = self.c, self.t
            p = f"model.layers.{l}.mlp.experts."
            if (p + "gate_up_proj_blocks") in t:
                def mx(which, O, I):
                    blk, sc = t[p + which + "_blocks"][1], t[p + which + "_scales"][1]
                    return QT(0, O, I, dequant_mxfp4(blk[e], sc[e], O, I))
                gu = mx("gate_up_proj", c.moe_inter, c.hidden)
                dn = mx("down_proj", c.hidden, c.moe_inter // 2)
                ly["experts"][e] = (gu, dn, ly["gu_bias"][e], ly["d_bias"][e])
                return ly["experts"][e]
            gu = _load_qt(t, p + f"gate_up_proj.{e}", c.moe_inter, c.hidden)
            dn = _load_qt(t, p + f"down_proj.{e}", c.hidden, c.moe_inter // 2)
            ly["experts"][e] = (gu, dn, ly["gu_bias"][e], ly["d_bias"][e])
        return ly["experts"][e]

    def rope_cs(self, pos):
        half = self.c.head_dim // 2
        cs = np.empty(half, np.float32)
        sn = np.empty(half, np.float32)
        lib().or_rope_cs(_ptr(self.inv_freq, _fp), half, pos, self.c.rope_attn_factor,
                         _ptr(cs, _fp), _ptr(sn, _fp))
        return cs, sn

    def attention(self, x, l, pos):
        """gqa_attention (picchio.c:504-623)."""
        c, ly, d = self.c, self.layers[l], self.dumps
        H, KVH, hd = c.n_heads, c.n_kv_heads, c.head_dim
        q = ly["wq"].matmul(x)[0]
        k = ly["wk"].matmul(x)[0]
        v = ly["wv"].matmul(x)[0]
        if ly["bq"] is not None:
            q = (q + ly["bq"]).astype(np.float32)
            k = (k + ly["bk"]).astype(np.float32)
            v = (v + ly["bv"]).astype(np.float32)
        d[f"layer{l}.q_bias"], d[f"layer{l}.k_bias"], d[f"layer{l}.v_bias"] = q.copy(), k.copy(), v.copy()
        cs, sn = self.rope_cs(pos)
        q = np.ascontiguousarray(q)
        k = np.ascontiguousarray(k)
        for h in range(H):
            seg = q[h * hd:(h + 1) * hd].copy()
            lib().or_rope_rotate(_ptr(seg, _fp), hd, _ptr(cs, _fp), _ptr(sn, _fp))
            q[h * hd:(h + 1) * hd] = seg
        for h in range(KVH):
            seg = k[h * hd:(h + 1) * hd].copy()
            lib().or_rope_rotate(_ptr(seg, _fp), hd, _ptr(cs, _fp), _ptr(sn, _fp))
            k[h * hd:(h + 1) * hd] = seg
        d[f"layer{l}.q_rope"], d[f"layer{l}.k_rope"] = q.copy(), k.copy()
        if pos < self.max_pos:
            self.K[l][pos] = bf16_round(k) if self.kv_bf16 else k
            self.V[l][pos] = bf16_round(v) if self.kv_bf16 else v
        end = min(pos, self.max_pos - 1)
        start = 0
        if ly["layer_type"] == 0:
            start = max(end - c.sliding_window + 1, 0)
        out = np.empty(H * hd, np.float32)
        sinks = ly["sinks"]
        lib().or_attention(_ptr(out, _fp), _ptr(q, _fp), _ptr(self.K[l], _fp), _ptr(self.V[l], _fp),
                           _ptr(sinks, _fp) if sinks is not None else None, H, KVH, hd, start, end)
        d[f"layer{l}.attn_concat"] = out.copy()
        o = ly["wo"].matmul(out)[0]
        if ly["bo"] is not None:
            o = (o + ly["bo"]).astype(np.float32)
        d[f"layer{l}.attn_out"] = o.copy()
        return o

    def moe(self, x, l, sel=None, wts=None):
        """moe_forward (picchio.c:1309-1466); explicit sel/wts bypass the router."""
        c, ly, d = self.c, self.layers[l], self.dumps
        if sel is None:
            logits, sel, wts = router_topk(x, ly["router"], ly["router_bias"], c.topk, bias_first=False)
            d[f"layer{l}.router_logits"] = logits
        d[f"layer{l}.top_indices"] = np.asarray(sel, np.int32).copy()
        d[f"layer{l}.top_weights"] = np.asarray(wts, np.float32).copy()
        out = np.zeros(c.hidden, np.float32)
        for k, e in enumerate(sel):
            gu, dn, gub, db = self.expert(l, int(e))
            g = (gu.matmul(x)[0] + gub).astype(np.float32)
            d[f"layer{l}.expert{k}.gate_up"] = g
            act = swiglu(g, c.swiglu_limit, c.swiglu_alpha)
            d[f"layer{l}.expert{k}.activated"] = act
            eo = (dn.matmul(act)[0] + db).astype(np.float32)
            d[f"layer{l}.expert{k}.output"] = eo
            w = np.float32(np.float32(wts[k]) * c.routed_scale)
            lib().or_axpy(_ptr(out, _fp), _ptr(eo, _fp), w, c.hidden)
        d[f"layer{l}.moe_out"] = out.copy()
        return out

    def embed_token(self, tok):
        """embed_token (picchio.c:1472-1503), INT8 or F32 table."""
        e, D = self.embed, self.c.hidden
        if tok < 0 or tok >= e.O:
            return np.zeros(D, np.float32)
        if e.fmt == 1:
            return (e.data[tok].astype(np.float32) * e.s[tok]).astype(np.float32)
        if e.fmt == 0:
            return e.data[tok].copy()
        raise ValueError("INT4 embedding not handled by the oracle")

    def forward_token(self, tok: int, pos: int, return_logits: bool = False):
        c, d = self.c, self.dumps
        d.clear()
        h = self.embed_token(tok)
        d["embedding"] = h.copy()
        for l in range(c.n_layers):
            ly = self.layers[l]
            d[f"layer{l}.input"] = h.copy()
            hn = rmsnorm(h, ly["in_ln"], c.eps)
            d[f"layer{l}.pre_attn_norm"] = hn
            a = self.attention(hn, l, pos)
            h = (h + a).astype(np.float32)
            d[f"layer{l}.post_attn_residual"] = h.copy()
            hn = rmsnorm(h, ly["post_ln"], c.eps)
            d[f"layer{l}.pre_moe_norm"] = hn
            m = self.moe(hn, l)
            h = (h + m).astype(np.float32)
            d[f"layer{l}.output"] = h.copy()
        hn = rmsnorm(h, self.final_norm, c.eps)
        d["final_norm"] = hn
        logits = self.lm_head.matmul(hn)[0]
        d["logits"] = logits
        nxt = argmax(logits)
        return (nxt, logits) if return_logits else nxt

    def generate(self, prompt, n_steps):
        """Sequential prefill then greedy decode; returns the emitted ids in the
        order the reference prints them with OUTPUT=ids (picchio.c:3196-3287)."""
        last = prompt[0]
        for i, t in enumerate(prompt):
            last = self.forward_token(t, i)
        out, pos, tok = [], len(prompt), last
        for _ in range(n_steps):
            out.append(tok)
            tok = self.forward_token(tok, pos)
            pos += 1
        return out
