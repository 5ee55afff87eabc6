"""Regenerate the golden fixtures in this folder from the reference itself.

Runs the unmodified reference engine, built from its own sources by
``oracle/Makefile`` into ``oracle/_ref/picchio``, on seeded synthetic
containers written by ``picchio_b200.synth`` and records:

* ``<name>.json``: container options and seeds, prompt, the greedy ids the
  reference prints with ``OUTPUT=ids TEMPERATURE=0 REP=1`` both with its
  batched prefill (default) and with ``PREFILL_BATCH=1``;
* ``<name>_dumps.npz``: the reference's ``ORACLE_DIR`` stage dumps of its last
  forward (picchio.c:204-249), used as per-layer parity probes;
* ``kernels.npz``: reference ``matmul_qt`` outputs (quant.h:117-319) on seeded
  small inputs, via ``oracle/_ref/libpicchio_ref.so``.

Needs ``/root/reference`` (or REF=...) only to build ``oracle/_ref``; the
fixtures it writes are small and committed, and the tests read only them.
Usage: ``python tests/golden/make_golden.py``.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from picchio_b200.synth import SynthConfig, make_model, random_prompt, quantize_int4, quantize_int8  # noqa: E402
from oracle import oracle as O  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
STEPS = 128
PROMPT_LEN = 64

VARIANTS = {
    # INT4 gs32 experts, INT8 attention
    "tiny_gs32_i8": dict(group_size=32, attn_format="i8"),
    # the reference converter's own format: gs64 experts, F32 attention
    "tiny_gs64_f32": dict(group_size=64, attn_format="f32"),
    # per-row INT4 experts, INT4 gs32 attention (matmul_i4 + matmul_i4_gs paths)
    "tiny_rowi4_i4": dict(group_size=0, attn_format="i4", attn_group_size=32),
}


def run_ref(model_dir, prompt_file, steps, extra_env=None):
    env = dict(os.environ, MODEL=model_dir, INPUT_FILE=prompt_file, OUTPUT="ids",
               TEMPERATURE="0", REP="1", MAX=str(steps), CTX="512", OMP_NUM_THREADS="4")
    env.update(extra_env or {})
    out = subprocess.run([O.REF_BIN_PATH], env=env, capture_output=True, text=True,
                         cwd=model_dir, check=True).stdout
    return [int(v) for v in out.split()]


def make_variant(name, opts, seed=1234, prompt_seed=7):
    cfg = SynthConfig(**opts)
    with tempfile.TemporaryDirectory() as d:
        make_model(d, cfg, seed)
        prompt = random_prompt(PROMPT_LEN, cfg.vocab_size, prompt_seed)
        pf = os.path.join(d, "prompt.txt")
        with open(pf, "w") as f:
            f.write(" ".join(map(str, prompt)))
        ids_batched = run_ref(d, pf, STEPS)
        ids_seq = run_ref(d, pf, STEPS, {"PREFILL_BATCH": "1"})
        dd = os.path.join(d, "dumps")
        os.makedirs(dd)
        run_ref(d, pf, 8, {"ORACLE_DIR": dd})
        dumps = {fn[:-4]: np.load(os.path.join(dd, fn)) for fn in sorted(os.listdir(dd))}
    np.savez_compressed(os.path.join(HERE, f"{name}_dumps.npz"), **dumps)
    meta = dict(name=name, options=opts, seed=seed, prompt_seed=prompt_seed, prompt=prompt,
                steps=STEPS, ctx=512, ids_batched=ids_batched, ids_sequential=ids_seq,
                dump_steps=8, dump_last_pos=PROMPT_LEN + 8 - 1)
    with open(os.path.join(HERE, f"{name}.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print(name, "ids", ids_batched[:12], "...", "batched==sequential:", ids_batched == ids_seq)


# Reference runs with its sampler on (sample_logits, picchio.c:1540-1649):
# the default settings (top-k 50, the in-block candidate sort on the device)
# and a top-k-free nucleus (the large candidate sort).
SAMPLED = [
    {"TEMPERATURE": "1.0", "TOPP": "0.95", "TOPK": "50", "REP": "1.1", "SEED": "4242"},
    {"TEMPERATURE": "0.8", "TOPP": "0.9", "TOPK": "0", "REP": "1.0", "SEED": "77"},
]
SAMPLED_STEPS = 48


def add_sampled(name):
    """Adds the reference's sampled ids (key "sampled") to <name>.json."""
    path = os.path.join(HERE, f"{name}.json")
    with open(path) as f:
        meta = json.load(f)
    with tempfile.TemporaryDirectory() as d:
        make_model(d, SynthConfig(**meta["options"]), meta["seed"])
        pf = os.path.join(d, "prompt.txt")
        with open(pf, "w") as f:
            f.write(" ".join(map(str, meta["prompt"])))
        meta["sampled"] = [{"env": env, "ids": run_ref(d, pf, SAMPLED_STEPS, env)} for env in SAMPLED]
    with open(path, "w") as f:
        json.dump(meta, f, indent=1)
    print(name, "sampled", [r["ids"][:8] for r in meta["sampled"]])


def make_kernels():
    import ctypes as C
    R = O.ref_lib()
    fp, u8, i8 = C.POINTER(C.c_float), C.POINTER(C.c_uint8), C.POINTER(C.c_int8)
    rng = np.random.default_rng(42)
    out = {}
    for tag, (Oo, I, gs, S) in {"a": (64, 256, 32, 1), "b": (48, 2880, 32, 4),
                                "c": (32, 512, 64, 2), "d": (16, 256, 0, 3)}.items():
        w = (rng.standard_normal((Oo, I)) * 0.02).astype(np.float32)
        x = rng.standard_normal((S, I)).astype(np.float32)
        pk, sc = quantize_int4(w, gs)
        y = np.empty((S, Oo), np.float32)
        if gs:
            R.ref_matmul_i4_gs(y.ctypes.data_as(fp), x.ctypes.data_as(fp), pk.ctypes.data_as(u8),
                               sc.ctypes.data_as(fp), S, I, Oo, gs)
        else:
            R.ref_matmul_i4(y.ctypes.data_as(fp), x.ctypes.data_as(fp), pk.ctypes.data_as(u8),
                            sc.ctypes.data_as(fp), S, I, Oo)
        out.update({f"i4_{tag}_x": x, f"i4_{tag}_q": pk, f"i4_{tag}_s": sc, f"i4_{tag}_y": y,
                    f"i4_{tag}_shape": np.array([Oo, I, gs, S])})
        q, s = quantize_int8(w)
        y8 = np.empty((S, Oo), np.float32)
        R.ref_matmul_q8(y8.ctypes.data_as(fp), x.ctypes.data_as(fp), q.ctypes.data_as(i8),
                        s.ctypes.data_as(fp), S, I, Oo)
        out.update({f"i8_{tag}_q": q, f"i8_{tag}_s": s, f"i8_{tag}_y": y8})
    np.savez_compressed(os.path.join(HERE, "kernels.npz"), **out)
    print("kernels.npz", len(out), "arrays")


if __name__ == "__main__":
    O.build(ref=True)
    for n, o in VARIANTS.items():
        make_variant(n, o)
    add_sampled("tiny_gs32_i8")
    make_kernels()
