"""ctypes mirror of include/picchio_b200.h.

Names follow the reference engine (picchio.c): ``Model.forward_token``
replaces ``forward_token`` (picchio.c:1655), ``Model.prefill_tokens``
replaces ``prefill_tokens`` (picchio.c:1936), ``Model.moe_forward`` replaces
``moe_forward`` (picchio.c:1309) and ``QT.matmul`` replaces ``matmul_qt``
(quant.h:323).  Errors come back as :class:`PicchioError` carrying the
library's status code; nothing here falls back to a CPU implementation.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, field

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpicchio_b200.so")

FMT_F32, FMT_INT8, FMT_INT4, FMT_MXFP4 = 0, 1, 2, 3

STATUS = ["PC_OK", "PC_ERR_INVALID_ARG", "PC_ERR_IO", "PC_ERR_FORMAT", "PC_ERR_MISSING_TENSOR",
          "PC_ERR_CUDA", "PC_ERR_OOM", "PC_ERR_RANGE", "PC_ERR_TIMEOUT", "PC_ERR_NCCL", "PC_ERR_STATE"]


class PicchioError(RuntimeError):
    def __init__(self, status: int, msg: str):
        self.status = status
        self.status_name = STATUS[status] if 0 <= status < len(STATUS) else str(status)
        super().__init__(f"{self.status_name}: {msg}")


class _Opts(C.Structure):
    _fields_ = [("device", C.c_int), ("ctx_len", C.c_int), ("kv_bf16", C.c_int), ("max_batch", C.c_int),
                ("ep_rank", C.c_int), ("ep_size", C.c_int), ("nccl_id", C.c_void_p), ("use_graphs", C.c_int),
                ("expert_residency", C.c_int), ("expert_cache_slots", C.c_int), ("prefill_chunk", C.c_int)]


class _Cfg(C.Structure):
    _fields_ = [("hidden", C.c_int), ("n_layers", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("n_experts", C.c_int), ("topk", C.c_int), ("intermediate", C.c_int),
                ("vocab", C.c_int), ("ctx_len", C.c_int), ("sliding_window", C.c_int), ("eps", C.c_float),
                ("theta", C.c_float), ("swiglu_limit", C.c_float), ("swiglu_alpha", C.c_float),
                ("routed_scale", C.c_float), ("rope_factor", C.c_float), ("rope_beta_fast", C.c_float),
                ("rope_beta_slow", C.c_float), ("rope_original_ctx", C.c_int), ("rope_truncate", C.c_int),
                ("group_size", C.c_int), ("attn_format", C.c_int), ("attn_group_size", C.c_int),
                ("layer_type", C.c_int * 256), ("expert_format", C.c_int)]


@dataclass
class ModelConfig:
    """Model shape for :meth:`Model.synthetic` (config.json field meanings)."""
    hidden: int = 256
    n_layers: int = 2
    n_heads: int = 8
    n_kv_heads: int = 2
    head_dim: int = 32
    n_experts: int = 8
    topk: int = 2
    intermediate: int = 256
    vocab: int = 1024
    ctx_len: int = 131072
    sliding_window: int = 128
    eps: float = 1e-5
    theta: float = 150000.0
    swiglu_limit: float = 7.0
    swiglu_alpha: float = 1.702
    routed_scale: float = 1.0
    rope_factor: float = 1.0
    rope_beta_fast: float = 32.0
    rope_beta_slow: float = 1.0
    rope_original_ctx: int = 4096
    rope_truncate: int = 1
    group_size: int = 32
    attn_format: int = FMT_INT8
    attn_group_size: int = 0
    layer_types: list = field(default_factory=list)  # default: alternate sliding/full
    expert_format: int = FMT_INT4  # FMT_MXFP4: experts as MXFP4 (group size 32)

    @staticmethod
    def gpt_oss_20b(**kw) -> "ModelConfig":
        return ModelConfig(hidden=2880, n_layers=24, n_heads=64, n_kv_heads=8, head_dim=64, n_experts=32,
                           topk=4, intermediate=2880, vocab=201088, **kw)

    @staticmethod
    def gpt_oss_120b(**kw) -> "ModelConfig":
        return ModelConfig(hidden=2880, n_layers=36, n_heads=64, n_kv_heads=8, head_dim=64, n_experts=128,
                           topk=4, intermediate=2880, vocab=201088, **kw)

    def _c(self) -> _Cfg:
        c = _Cfg()
        for f, _ in _Cfg._fields_:
            if f == "layer_type":
                continue
            setattr(c, f, getattr(self, f))
        lt = self.layer_types or [i % 2 for i in range(self.n_layers)]
        for i in range(self.n_layers):
            c.layer_type[i] = int(lt[i % len(lt)])
        return c


_lib = None


class _Sampling(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_int), ("rep_penalty", C.c_float)]


def lib():
    """The loaded C library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise PicchioError(5, f"{LIB_PATH} is missing: run `python -m picchio_b200.build`")
        L = C.CDLL(LIB_PATH)
        st = C.c_int
        vp = C.c_void_p
        ip = C.POINTER(C.c_int)
        fp = C.POINTER(C.c_float)
        L.pc_default_opts.argtypes = [C.POINTER(_Opts)]
        L.pc_status_string.restype = C.c_char_p
        L.pc_status_string.argtypes = [st]
        L.pc_last_error.restype = C.c_char_p
        L.pc_init.argtypes = [C.c_char_p, C.POINTER(_Opts), C.POINTER(vp)]
        L.pc_init_synthetic.argtypes = [C.POINTER(_Cfg), C.c_uint64, C.POINTER(_Opts), C.POINTER(vp)]
        L.pc_free.argtypes = [vp]
        L.pc_free.restype = None
        L.pc_get_config.argtypes = [vp, C.POINTER(_Cfg)]
        L.pc_forward_token.argtypes = [vp, C.c_int, C.c_int, ip]
        L.pc_prefill.argtypes = [vp, ip, C.c_int, C.c_int, ip]
        L.pc_prefill_seq.argtypes = [vp, C.c_int, ip, C.c_int, C.c_int, ip]
        L.pc_decode_batch.argtypes = [vp, ip, ip, C.c_int, ip]
        L.pc_get_logits.argtypes = [vp, C.c_int, fp, C.c_int]
        L.pc_moe_layer.argtypes = [vp, C.c_int, vp, vp, C.c_int]
        L.pc_moe_experts.argtypes = [vp, C.c_int, vp, vp, vp, C.c_int, vp]
        L.pc_set_trace.argtypes = [vp, C.c_int]
        L.pc_get_routing.argtypes = [vp, ip, C.c_int, ip]
        L.pc_get_stage.argtypes = [vp, C.c_char_p, fp, C.c_int]
        L.pc_dump.argtypes = [vp, C.c_char_p]
        L.pc_expert_prefetch.argtypes = [vp, C.c_int, ip, C.c_int]
        L.pc_qt_create.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, vp, fp, C.POINTER(vp)]
        L.pc_qt_matmul.argtypes = [vp, vp, vp, C.c_int, vp]
        L.pc_qt_matmul_noalloc.argtypes = [vp, vp, vp, C.c_int, vp]
        L.pc_qt_dequant.argtypes = [vp, vp, vp]
        L.pc_qt_check.argtypes = [vp, vp]
        L.pc_qt_free.argtypes = [vp]
        L.pc_qt_free.restype = None
        L.pc_nccl_unique_id.argtypes = [vp]
        L.pc_check_device.argtypes = [vp]
        L.pc_kernel_launches.argtypes = [vp]
        L.pc_kernel_launches.restype = C.c_uint64
        L.pc_tensor_core_min_rows.argtypes = [vp]
        L.pc_tensor_core_min_rows.restype = C.c_int
        L.pc_generate.argtypes = [vp, C.c_int, C.c_int, C.c_int, ip, fp]
        L.pc_kv_fill_synthetic.argtypes = [vp, C.c_int, C.c_int, C.c_uint64]
        L.pc_kv_fill_synthetic.restype = st
        L.pc_profile_begin.argtypes = [vp]
        L.pc_profile_end.argtypes = [vp]
        L.pc_profile_get.argtypes = [vp, C.c_char_p, C.POINTER(C.c_double), ip]
        L.pc_set_sampling.argtypes = [vp, C.POINTER(_Sampling)]
        L.pc_set_rng.argtypes = [vp, C.c_uint64]
        L.pc_get_rng.argtypes = [vp, C.POINTER(C.c_uint64)]
        L.pc_history_reset.argtypes = [vp]
        L.pc_history_push.argtypes = [vp, ip, C.c_int]
        L.pc_history_get.argtypes = [vp, ip, C.c_int, ip]
        L.pc_sample.argtypes = [vp, vp, ip]
        L.pc_expert_stats.argtypes = [vp, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]
        L.pc_expert_stats.restype = st
        for name in ("pc_generate", "pc_profile_begin", "pc_profile_end", "pc_profile_get", "pc_set_sampling",
                     "pc_set_rng", "pc_get_rng", "pc_history_reset", "pc_history_push", "pc_history_get",
                     "pc_sample"):
            getattr(L, name).restype = st
        for name in ("pc_init", "pc_init_synthetic", "pc_get_config", "pc_forward_token", "pc_prefill", "pc_prefill_seq",
                     "pc_decode_batch", "pc_get_logits", "pc_moe_layer", "pc_moe_experts", "pc_set_trace",
                     "pc_get_routing",
                     "pc_get_stage", "pc_dump", "pc_expert_prefetch", "pc_qt_create", "pc_qt_matmul", "pc_qt_matmul_noalloc",
                     "pc_qt_dequant", "pc_qt_check", "pc_nccl_unique_id", "pc_check_device"):
            getattr(L, name).restype = st
        _lib = L
    return _lib


def _check(status: int):
    if status != 0:
        raise PicchioError(status, lib().pc_last_error().decode(errors="replace"))


def nccl_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    _check(lib().pc_nccl_unique_id(buf))
    return buf.raw


def _dev_ptr(t):
    """Device pointer of a CUDA tensor (torch is plumbing here)."""
    if not t.is_cuda or not t.is_contiguous():
        raise ValueError("expected a contiguous CUDA tensor")
    return C.c_void_p(t.data_ptr())


def _torch_done(*ts):
    """Waits for torch's pending work on the tensors' devices: a context runs
    on its own non-blocking stream, which is not ordered after torch's, so a
    tensor torch is still writing (a host copy in flight) must be complete
    before the library reads it."""
    import torch
    for dev in {t.device for t in ts}:
        torch.cuda.current_stream(dev).synchronize()


class Model:
    """A device-resident model: the replacement for picchio's Model + engine."""

    def __init__(self, model_dir: str | None = None, *, cfg: ModelConfig | None = None, seed: int = 0,
                 ctx: int = 512, kv_bf16: bool = False, max_batch: int = 1, device: int = 0,
                 use_graphs: bool = True, ep_rank: int = 0, ep_size: int = 1, nccl_id: bytes | None = None,
                 expert_residency: int = 0, expert_cache_slots: int = 0, prefill_chunk: int = 64):
        L = lib()
        o = _Opts()
        L.pc_default_opts(C.byref(o))
        o.device, o.ctx_len, o.kv_bf16, o.max_batch = device, ctx, int(kv_bf16), max_batch
        o.use_graphs, o.ep_rank, o.ep_size = int(use_graphs), ep_rank, ep_size
        o.expert_residency, o.expert_cache_slots = int(expert_residency), int(expert_cache_slots)
        o.prefill_chunk = int(prefill_chunk)
        self._nid = C.create_string_buffer(nccl_id, 128) if nccl_id is not None else None
        o.nccl_id = C.cast(self._nid, C.c_void_p) if self._nid is not None else None
        h = C.c_void_p()
        if model_dir is not None:
            _check(L.pc_init(model_dir.encode(), C.byref(o), C.byref(h)))
        else:
            c = (cfg or ModelConfig())._c()
            _check(L.pc_init_synthetic(C.byref(c), C.c_uint64(seed), C.byref(o), C.byref(h)))
        self._h = h
        self.ctx_len, self.device = ctx, device
        cc = _Cfg()
        _check(L.pc_get_config(h, C.byref(cc)))
        self.config = {f: (list(cc.layer_type[:cc.n_layers]) if f == "layer_type" else getattr(cc, f))
                       for f, _ in _Cfg._fields_}

    @classmethod
    def synthetic(cls, cfg: ModelConfig, seed: int = 0, **kw) -> "Model":
        return cls(None, cfg=cfg, seed=seed, **kw)

    def close(self):
        if getattr(self, "_h", None):
            lib().pc_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # --- the reference's engine entry points ---
    def forward_token(self, tok: int, pos: int) -> int:
        out = C.c_int()
        _check(lib().pc_forward_token(self._h, int(tok), int(pos), C.byref(out)))
        return out.value

    def prefill_tokens(self, ids, pos_base: int = 0, seq: int = 0) -> int:
        a = (C.c_int * len(ids))(*[int(v) for v in ids])
        out = C.c_int()
        if seq == 0:
            _check(lib().pc_prefill(self._h, a, len(ids), int(pos_base), C.byref(out)))
        else:
            _check(lib().pc_prefill_seq(self._h, int(seq), a, len(ids), int(pos_base), C.byref(out)))
        return out.value

    def decode_batch(self, toks, pos) -> list:
        B = len(toks)
        t = (C.c_int * B)(*[int(v) for v in toks])
        p = (C.c_int * B)(*[int(v) for v in pos])
        o = (C.c_int * B)()
        _check(lib().pc_decode_batch(self._h, t, p, B, o))
        return list(o)

    def generate(self, prompt, n_steps: int) -> list:
        """Prefill then greedy decode; ids in the order picchio prints them
        with OUTPUT=ids (picchio.c:3196-3287)."""
        tok = self.prefill_tokens(prompt, 0)
        out, pos = [], len(prompt)
        for _ in range(n_steps):
            out.append(tok)
            tok = self.forward_token(tok, pos)
            pos += 1
        return out

    def generate_device(self, tok: int, pos: int, n: int):
        """n greedy steps on the device (pc_generate): returns (ids, device_ms)."""
        out = (C.c_int * n)()
        ms = C.c_float()
        _check(lib().pc_generate(self._h, int(tok), int(pos), int(n), out, C.byref(ms)))
        return list(out), float(ms.value)

    def kv_fill_synthetic(self, n_pos: int, seq: int = 0, seed: int = 99):
        _check(lib().pc_kv_fill_synthetic(self._h, seq, n_pos, seed))

    def profile_begin(self):
        _check(lib().pc_profile_begin(self._h))

    def profile_end(self) -> dict:
        """Ends profiling; returns {label: (total_ms, launches)}."""
        _check(lib().pc_profile_end(self._h))
        res = {}
        for lab in ("expert_gate_up", "expert_down", "qkv", "o_proj", "lm_head", "attention", "router",
                    "ep_exchange", "combine"):
            t, n = C.c_double(), C.c_int()
            _check(lib().pc_profile_get(self._h, lab.encode(), C.byref(t), C.byref(n)))
            if n.value:
                res[lab] = (t.value, n.value)
        return res

    def logits(self, row: int = 0) -> np.ndarray:
        v = np.empty(self.config["vocab"], np.float32)
        _check(lib().pc_get_logits(self._h, row, v.ctypes.data_as(C.POINTER(C.c_float)), v.size))
        return v

    def set_sampling(self, temperature: float | None = None, top_p: float = 1.0, top_k: int = 0,
                     rep_penalty: float = 1.0):
        """Device sample_logits for later single-sequence steps (None: argmax)."""
        if temperature is None:
            _check(lib().pc_set_sampling(self._h, None))
            return
        s = _Sampling(float(temperature), float(top_p), int(top_k), float(rep_penalty))
        _check(lib().pc_set_sampling(self._h, C.byref(s)))

    @property
    def rng(self) -> int:
        v = C.c_uint64(0)
        _check(lib().pc_get_rng(self._h, C.byref(v)))
        return int(v.value)

    @rng.setter
    def rng(self, state: int):
        _check(lib().pc_set_rng(self._h, int(state)))

    def history(self) -> list:
        buf = np.zeros(4096, np.int32)
        n = C.c_int(0)
        _check(lib().pc_history_get(self._h, buf.ctypes.data_as(C.POINTER(C.c_int)), buf.size, C.byref(n)))
        return buf[:n.value].tolist()

    def history_reset(self):
        _check(lib().pc_history_reset(self._h))

    def history_push(self, ids):
        a = np.ascontiguousarray(ids, np.int32)
        _check(lib().pc_history_push(self._h, a.ctypes.data_as(C.POINTER(C.c_int)), a.size))

    def sample(self, logits) -> int:
        """One device draw from a [vocab] float32 CUDA tensor."""
        out = C.c_int(0)
        _torch_done(logits)
        _check(lib().pc_sample(self._h, _dev_ptr(logits), C.byref(out)))
        return int(out.value)

    def expert_prefetch(self, layer: int, eids):
        a = np.ascontiguousarray(eids, np.int32)
        _check(lib().pc_expert_prefetch(self._h, int(layer), a.ctypes.data_as(C.POINTER(C.c_int)), a.size))

    def expert_stats(self) -> dict:
        """Streamed-residency counters: HBM-slot hits, host reads, bytes copied."""
        h, m, b = C.c_uint64(), C.c_uint64(), C.c_uint64()
        _check(lib().pc_expert_stats(self._h, C.byref(h), C.byref(m), C.byref(b)))
        return {"hits": h.value, "misses": m.value, "bytes_h2d": b.value}

    def moe_forward(self, x, layer: int):
        """moe_forward for the rows of x ([M, D] float32 CUDA tensor)."""
        import torch
        out = torch.empty_like(x)
        _torch_done(x, out)
        _check(lib().pc_moe_layer(self._h, layer, _dev_ptr(x), _dev_ptr(out), x.shape[0]))
        return out

    def moe_experts(self, x, sel, w, layer: int):
        """The expert half of moe_forward with routing given (sel int32 [M, K], w float32 [M, K])."""
        import torch
        out = torch.empty_like(x)
        _torch_done(x, sel, w, out)
        _check(lib().pc_moe_experts(self._h, layer, _dev_ptr(x), _dev_ptr(sel), _dev_ptr(w), x.shape[0],
                                    _dev_ptr(out)))
        return out

    def set_trace(self, on: bool = True):
        _check(lib().pc_set_trace(self._h, int(on)))

    def routing(self) -> np.ndarray:
        """Router top-k of the last step: int32 [n_layers, rows, topk] expert ids."""
        L, K = self.config["n_layers"], self.config["topk"]
        rows = C.c_int()
        lib().pc_get_routing(self._h, None, 0, C.byref(rows))  # row count only
        v = np.empty(max(L * rows.value * K, 1), np.int32)
        _check(lib().pc_get_routing(self._h, v.ctypes.data_as(C.POINTER(C.c_int)), v.size, C.byref(rows)))
        return v[:L * rows.value * K].reshape(L, rows.value, K)

    def stage(self, name: str, n: int) -> np.ndarray:
        v = np.empty(n, np.float32)
        _check(lib().pc_get_stage(self._h, name.encode(), v.ctypes.data_as(C.POINTER(C.c_float)), n))
        return v

    def dump(self, directory: str):
        _check(lib().pc_dump(self._h, directory.encode()))

    def check_device(self):
        _check(lib().pc_check_device(self._h))

    @property
    def launches(self) -> int:
        return int(lib().pc_kernel_launches(self._h))

    @property
    def tensor_core_min_rows(self) -> int:
        """Rows per step from which the dense projections use the tensor cores (0: off)."""
        return int(lib().pc_tensor_core_min_rows(self._h))


class QT:
    """One weight matrix on the device: the replacement for quant.h's QT +
    matmul_qt.  ``data``/``scales`` use the reference's host layout."""

    def __init__(self, fmt: int, O: int, I: int, data: np.ndarray, scales: np.ndarray | None = None,
                 block_size: int = 0, device: int = 0):
        data = np.ascontiguousarray(data)
        sp = None
        if scales is not None:
            scales = np.ascontiguousarray(scales, np.float32)
            sp = scales.ctypes.data_as(C.POINTER(C.c_float))
        h = C.c_void_p()
        _check(lib().pc_qt_create(device, fmt, O, I, block_size, data.ctypes.data_as(C.c_void_p), sp, C.byref(h)))
        self._h, self.O, self.I, self.fmt, self.device = h, O, I, fmt, device

    def matmul(self, x, stream=None):
        import torch
        y = torch.empty((x.shape[0], self.O), dtype=torch.float32, device=x.device)
        st = stream if stream is not None else torch.cuda.current_stream(x.device).cuda_stream
        _check(lib().pc_qt_matmul(self._h, _dev_ptr(x), _dev_ptr(y), x.shape[0], C.c_void_p(st)))
        return y

    def matmul_noalloc(self, x, out=None, stream=None):
        """pc_qt_matmul_noalloc: the same product with no device allocation in
        the library call (at most 64 rows); ``out`` may be given."""
        import torch
        y = out if out is not None else torch.empty((x.shape[0], self.O), dtype=torch.float32, device=x.device)
        st = stream if stream is not None else torch.cuda.current_stream(x.device).cuda_stream
        _check(lib().pc_qt_matmul_noalloc(self._h, _dev_ptr(x), _dev_ptr(y), x.shape[0], C.c_void_p(st)))
        return y

    def check(self, stream=None):
        """pc_qt_check: waits for the stream and raises if an earlier product
        on this weight (or a no-alloc product on its device) reported a
        device-side failure."""
        import torch
        st = stream if stream is not None else torch.cuda.current_stream(self.device).cuda_stream
        _check(lib().pc_qt_check(self._h, C.c_void_p(st)))

    def dequant(self):
        import torch
        out = torch.empty((self.O, self.I), dtype=torch.float32, device=f"cuda:{self.device}")
        st = torch.cuda.current_stream(out.device).cuda_stream
        _check(lib().pc_qt_dequant(self._h, _dev_ptr(out), C.c_void_p(st)))
        return out

    def close(self):
        if getattr(self, "_h", None):
            lib().pc_qt_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
