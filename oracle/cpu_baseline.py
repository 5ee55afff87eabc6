"""The reference's CPU decode, timed on this host's cores (bench.py's
cpu_baseline leg and its --impl reference arm; TEST INFRASTRUCTURE ONLY).

It runs the reference's own functions, compiled from its sources into
oracle/_ref/libpicchio_ref.so, on one decode layer of a GPT-OSS shape with
random weights: gqa_attention (picchio.c:504-623, INT8 projections, fp32 KV
cache, window or full span), the router dot + top-k of moe_forward
(picchio.c:1316-1340, restated in oracle.c; ~1% of the layer) and
expert_apply (picchio.c:1769-1791) on the K routed experts, then the INT8
lm_head (matmul_q8, quant.h:152-186).  Per-token time = n_full x full layer
+ n_sliding x sliding layer + lm_head; the expert store is taken as resident
in RAM (no disk), which is the reference's best case.
"""
from __future__ import annotations

import ctypes as C
import os
import time

import numpy as np

from oracle import oracle as O

fp = C.POINTER(C.c_float)
u8 = C.POINTER(C.c_uint8)
i8 = C.POINTER(C.c_int8)


def _p(a, t):
    return a.ctypes.data_as(t)


def _setup_ref():
    R = O.ref_lib()
    if R is None:
        return None
    R.ref_expert_apply.argtypes = [u8, fp, C.c_int, fp, u8, fp, C.c_int, fp, C.c_int, C.c_int, fp, fp,
                                   C.c_float, C.c_float]
    R.ref_gqa_attention.argtypes = [i8, fp, i8, fp, i8, fp, i8, fp, fp, fp, fp, fp, fp, fp, fp, C.c_int,
                                    C.c_int, C.c_int, C.c_int, fp, fp, C.c_int, C.c_int, C.c_int, C.c_int,
                                    C.c_float]
    return R


def measure(D=2880, H=64, KVH=8, hd=64, E=128, K=4, inter=2880, V=201088, gs=32, n_layers=36,
            ctx=4096, window=128, budget_s=20.0, threads=None) -> dict:
    """Returns {"tok_s", "layer_full_ms", "layer_sliding_ms", "head_ms", "cores", "kind", "sample"}."""
    threads = threads or len(os.sched_getaffinity(0)) or 1
    os.environ["OMP_NUM_THREADS"] = str(threads)
    R = _setup_ref()
    if R is not None and hasattr(R, "ref_set_threads"):
        # the OpenMP runtime may already be up (torch loads it; torchrun sets
        # OMP_NUM_THREADS=1): set the team size directly and read it back
        R.ref_set_threads(threads)
        R.ref_max_threads.restype = C.c_int
        threads = int(R.ref_max_threads())
    rng = np.random.default_rng(0)
    I2 = 2 * inter
    f32 = np.float32

    def q8(o, i):
        return rng.integers(-127, 128, size=(o, i), dtype=np.int8), rng.uniform(1e-4, 2e-4, o).astype(f32)

    wq, sq = q8(H * hd, D)
    wk, sk = q8(KVH * hd, D)
    wv, sv = q8(KVH * hd, D)
    wo, so = q8(D, H * hd)
    bq, bk, bv, bo = (rng.standard_normal(n).astype(f32) * 0.01 for n in (H * hd, KVH * hd, KVH * hd, D))
    sinks = rng.standard_normal(H).astype(f32)
    Kc = rng.standard_normal((ctx, KVH * hd)).astype(f32)
    Vc = rng.standard_normal((ctx, KVH * hd)).astype(f32)
    router = rng.standard_normal((E, D)).astype(f32) * 0.1
    experts = []
    for _ in range(K):
        experts.append((rng.integers(0, 256, size=I2 * D // 2, dtype=np.uint8),
                        rng.uniform(1e-3, 2e-3, I2 * (D // gs)).astype(f32), rng.standard_normal(I2).astype(f32) * 0.01,
                        rng.integers(0, 256, size=D * inter // 2, dtype=np.uint8),
                        rng.uniform(1e-3, 2e-3, D * (inter // gs)).astype(f32), rng.standard_normal(D).astype(f32) * 0.01))
    x = rng.standard_normal(D).astype(f32)
    out = np.zeros(D, f32)

    def layer(layer_type):
        pos = ctx - 1
        if R is not None:
            R.ref_gqa_attention(_p(wq, i8), _p(sq, fp), _p(wk, i8), _p(sk, fp), _p(wv, i8), _p(sv, fp),
                                _p(wo, i8), _p(so, fp), _p(bq, fp), _p(bk, fp), _p(bv, fp), _p(bo, fp),
                                _p(sinks, fp), _p(Kc, fp), _p(Vc, fp), ctx, layer_type, window, pos,
                                _p(x, fp), _p(out, fp), D, H, KVH, hd, 150000.0)
        else:
            q = O.matmul_q8(x, wq, sq, H * hd, D)[0]
            O.lib().or_attention(_p(out, fp), _p(np.ascontiguousarray(q[: H * hd]), fp), _p(Kc, fp), _p(Vc, fp),
                                 _p(sinks, fp), H, KVH, hd, 0 if layer_type else pos - window + 1, pos)
        O.router_topk(x, router, None, K)
        acc = np.zeros(D, f32)
        for (gq, gsc, gb, dq, dsc, db) in experts:
            if R is not None:
                R.ref_expert_apply(_p(gq, u8), _p(gsc, fp), gs, _p(gb, fp), _p(dq, u8), _p(dsc, fp), gs,
                                   _p(db, fp), D, I2, _p(x, fp), _p(acc, fp), 0.25, 7.0)
            else:
                g = O.matmul_i4_gs(x, gq, gsc, I2, D, gs)[0] + gb
                a = O.swiglu(g, 7.0)
                acc += 0.25 * (O.matmul_i4_gs(a, dq, dsc, D, inter, gs)[0] + db)

    def timed(fn, reps):
        fn()  # warm caches / OpenMP pool
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        return (time.perf_counter() - t0) / reps

    t_full = timed(lambda: layer(1), 2)
    t_slide = timed(lambda: layer(0), 2)
    # lm_head: a slice of the vocabulary, scaled to the full one (matmul_q8
    # time is linear in the rows)
    vs = min(V, 32768)
    wh, sh = q8(vs, D)
    y = np.empty(vs, f32)
    if R is not None:
        t_head = timed(lambda: R.ref_matmul_q8(_p(y, fp), _p(x, fp), _p(wh, i8), _p(sh, fp), 1, D, vs), 3) * V / vs
    else:
        t_head = timed(lambda: O.matmul_q8(x, wh, sh, vs, D), 1) * V / vs
    n_full = sum(1 for i in range(n_layers) if i % 2 == 1)
    n_slide = n_layers - n_full
    t_tok = n_full * t_full + n_slide * t_slide + t_head
    return {
        "tok_s": 1.0 / t_tok,
        "layer_full_ms": t_full * 1e3,
        "layer_sliding_ms": t_slide * 1e3,
        "head_ms": t_head * 1e3,
        "cores": threads if R is not None else 1,
        "kind": "reference" if R is not None else "port",
        "sample": (f"one full-attention and one sliding-window decode layer at position {ctx - 1} "
                   f"(D={D}, {H}q/{KVH}kv x {hd}, {K} of {E} experts INT4 gs{gs}, INT8 attention), "
                   f"timed and scaled to {n_full}+{n_slide} layers, plus INT8 lm_head on {vs} of {V} rows "
                   f"scaled to {V}; {'reference functions from oracle/_ref, OpenMP ' + str(threads) + ' threads' if R is not None else 'oracle port, 1 thread'}"),
    }


def measure_e2e(threads=None, prompt_len=64, steps=32, seed=1234) -> dict | None:
    """The unmodified reference binary (oracle/_ref/picchio) end to end on
    BASELINE configs[0], the tiny seeded model: a prompt_len-id random prompt,
    then `steps` greedy tokens (MODEL, INPUT_FILE, OUTPUT=ids, TEMPERATURE=0,
    REP=1; ECAP = every expert, so the expert cache holds the whole model).
    Returns the decode and prefill rates the binary itself reports, or None
    when the binary has not been built."""
    import re
    import subprocess
    import tempfile

    from picchio_b200.synth import SynthConfig, make_model, random_prompt
    if not os.path.exists(O.REF_BIN_PATH):
        return None
    threads = threads or len(os.sched_getaffinity(0)) or 1
    cfg = SynthConfig()
    with tempfile.TemporaryDirectory() as d:
        make_model(d, cfg, seed)
        pf = os.path.join(d, "prompt.txt")
        with open(pf, "w") as f:
            f.write(" ".join(map(str, random_prompt(prompt_len, cfg.vocab_size, 7))))
        env = dict(os.environ, MODEL=d, INPUT_FILE=pf, OUTPUT="ids", TEMPERATURE="0", REP="1", MAX=str(steps),
                   CTX="512", ECAP=str(cfg.num_local_experts), OMP_NUM_THREADS=str(threads))
        r = subprocess.run([O.REF_BIN_PATH], env=env, capture_output=True, text=True, cwd=d, timeout=300)
    if r.returncode != 0:
        return None
    # "generated N tokens in T s (R tok/s)": R from the binary's own clock
    # (T is printed with two decimals only)
    gen = re.search(r"generated (\d+) tokens in ([0-9.]+) s \(([0-9.]+) tok/s\)", r.stderr)
    pre = re.search(r"prefill in ([0-9.]+) s", r.stderr)
    if not gen:
        return None
    n, rate = int(gen.group(1)), float(gen.group(3))
    return {"value": rate if rate > 0 else None, "unit": "tok/s", "cores": threads, "kind": "reference",
            "prefill_s": float(pre.group(1)) if pre else None,
            "sample": (f"unmodified reference binary end to end on the tiny seeded model (configs[0]): "
                       f"{prompt_len}-id prompt, {n} greedy tokens, OMP_NUM_THREADS={threads}, "
                       f"decode rate as the binary reports it")}


if __name__ == "__main__":
    import json
    print(json.dumps(measure()))
