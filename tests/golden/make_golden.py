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
  small inputs, via ``oracle/_ref/libpicchio_ref.so``;
* ``mxfp4.npz``: MXFP4 blocks / E8M0 scales (every code and a spread of
  exponents) and their fp32 values from the reference converter's own
  ``dequant_mxfp4_fast`` / ``dequant_mxfp4`` and ``decode_e8m0``
  (convert.py:129-213), imported from the reference sources.

Needs the reference sources (``REF=...``, else BASELINE.json's
``reference_path``) only to build ``oracle/_ref``; the
fixtures it writes are small and committed, and the tests read only them.
Usage: ``python tests/golden/make_golden.py [tiny] [gptoss] [gptoss_bf16kv] [service] [mxfp4]`` (all by
default).
"""
from __future__ import annotations

import json
import os
import re
import shutil
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


# GPT-OSS-shaped two-layer container: d_model 2880, 64 q / 8 kv heads x 64,
# sinks, a 128-window layer and a full layer, 32 experts top-4 INT4 gs32,
# INT8 dense weights; a 4096-id vocabulary keeps the file near 1 GB.  These
# are the head and expert shapes of the GPT-OSS-20B/120B configurations.
GPTOSS = dict(hidden_size=2880, num_hidden_layers=2, num_attention_heads=64, num_key_value_heads=8,
              head_dim=64, intermediate_size=2880, num_local_experts=32, num_experts_per_tok=4,
              vocab_size=4096, group_size=32, attn_format="i8")
GPTOSS_SEED = 4321
GPTOSS_PROMPT = 120      # decode then crosses positions 127/128/129 and 255/256/257
GPTOSS_STEPS = 144       # forward_token calls after the prefill (positions 120..263)
# calls whose stage tensors are kept (call s runs at position 120 + s - 1):
# positions 126-130 (window edge of the sliding layer), 255-257, and the last
GPTOSS_PROBES = [7, 8, 9, 10, 11, 136, 137, 138, 144]
GPTOSS_PROBE_KEYS = ["layer0.output", "layer1.output", "layer0.attn_concat", "layer1.attn_concat",
                     "final_norm"]
GPTOSS_LONG_PROMPT = 300  # 1200 routed pairs: the expert GEMMs of a long prefill chunk
GPTOSS_LONG_STEPS = 8


# the stage tensors pc_get_stage exposes (the rest of the reference's dumps
# are intermediate forms it has no separate buffer for)
STAGE_RE = re.compile(r"^(embedding|final_norm|logits|layer\d+\.(input|pre_attn_norm|q_rope|attn_concat|attn_out|"
                      r"post_attn_residual|pre_moe_norm|router_logits|top_indices|top_weights|"
                      r"expert\d+\.(activated|output)|moe_out|output))$")


def _dumps(d, pf, steps, threads):
    dd = os.path.join(d, f"dumps{steps}")
    os.makedirs(dd, exist_ok=True)
    ids = run_ref(d, pf, steps, {"ORACLE_DIR": dd, "OMP_NUM_THREADS": str(threads)})
    out = {fn[:-4]: np.load(os.path.join(dd, fn)) for fn in sorted(os.listdir(dd))}
    return ids, out


def make_gptoss(threads=8):
    """gptoss_2l.json / gptoss_2l_dumps.npz: the reference's greedy ids for
    GPTOSS_STEPS steps, the router top-k and logits of every one of those
    forward_token calls (one reference run per call, each dumping its last
    forward), the GPTOSS_PROBE_KEYS stage tensors at the probe calls, every
    stage tensor of the last call, and the same for a GPTOSS_LONG_PROMPT-id
    prompt over GPTOSS_LONG_STEPS calls."""
    cfg = SynthConfig(**GPTOSS)
    with tempfile.TemporaryDirectory() as d:
        make_model(d, cfg, GPTOSS_SEED)
        prompt = random_prompt(GPTOSS_PROMPT, cfg.vocab_size, 11)
        pf = os.path.join(d, "prompt.txt")
        with open(pf, "w") as f:
            f.write(" ".join(map(str, prompt)))
        thr = {"OMP_NUM_THREADS": str(threads)}
        ids = run_ref(d, pf, GPTOSS_STEPS, thr)
        arrays, topk, rlog = {}, [], []
        for s in range(1, GPTOSS_STEPS + 1):
            ids_s, dm = _dumps(d, pf, s, threads)
            assert ids_s == ids[:s], s
            topk.append([dm[f"layer{l}.top_indices"].reshape(-1).astype(int).tolist() for l in range(2)])
            rlog.append(np.stack([dm[f"layer{l}.router_logits"].reshape(-1) for l in range(2)]))
            if s in GPTOSS_PROBES:
                for k in GPTOSS_PROBE_KEYS:
                    arrays[f"probe{s}.{k}"] = dm[k].reshape(-1)
            if s == GPTOSS_STEPS:
                for k, v in dm.items():
                    if STAGE_RE.match(k):
                        arrays[f"last.{k}"] = v.reshape(-1)
            shutil.rmtree(os.path.join(d, f"dumps{s}"))
        arrays["router_logits"] = np.stack(rlog).astype(np.float32)
        long_prompt = random_prompt(GPTOSS_LONG_PROMPT, cfg.vocab_size, 12)
        pf2 = os.path.join(d, "prompt_long.txt")
        with open(pf2, "w") as f:
            f.write(" ".join(map(str, long_prompt)))
        dd = os.path.join(d, "dumps_long")
        os.makedirs(dd)
        long_ids = run_ref(d, pf2, GPTOSS_LONG_STEPS, {"ORACLE_DIR": dd, **thr})
        for fn in sorted(os.listdir(dd)):
            if STAGE_RE.match(fn[:-4]):
                arrays[f"long.{fn[:-4]}"] = np.load(os.path.join(dd, fn)).reshape(-1)
    np.savez_compressed(os.path.join(HERE, "gptoss_2l_dumps.npz"), **arrays)
    meta = dict(name="gptoss_2l", options=GPTOSS, seed=GPTOSS_SEED, prompt=prompt, steps=GPTOSS_STEPS, ctx=512,
                ids=ids, top_indices=topk, probes=GPTOSS_PROBES, probe_keys=GPTOSS_PROBE_KEYS,
                long_prompt=long_prompt, long_steps=GPTOSS_LONG_STEPS, long_ids=long_ids)
    with open(os.path.join(HERE, "gptoss_2l.json"), "w") as f:
        json.dump(meta, f)
    print("gptoss_2l ids", ids[:12], "... long", long_ids)


def make_gptoss_bf16kv():
    """gptoss_2l_bf16kv.npz: the same calls as make_gptoss on the oracle with
    a bf16 KV cache (OracleModel(kv_bf16=True): every stored K/V row rounded
    to bf16, the device's cache format; the rest is the oracle restatement
    pinned bit-exact to the reference).  Teacher-forced on the reference's
    ids, as the device test runs; the greedy next id and router top-k of
    every call, the GPTOSS_PROBE_KEYS stage tensors at the probe calls, every
    stage tensor of the last call, and of the last call after the long
    prompt."""
    with open(os.path.join(HERE, "gptoss_2l.json")) as f:
        meta = json.load(f)
    cfg = SynthConfig(**GPTOSS)
    arrays = {}
    with tempfile.TemporaryDirectory() as d:
        make_model(d, cfg, GPTOSS_SEED)
        m = O.OracleModel(d, ctx=meta["ctx"], kv_bf16=True)
        prompt, ids = meta["prompt"], meta["ids"]
        nxt, topk = [], []
        for i, t in enumerate(prompt):
            first = m.forward_token(t, i)
        nxt.append(first)
        for s in range(1, GPTOSS_STEPS + 1):
            nxt.append(m.forward_token(ids[s - 1], len(prompt) + s - 1))
            topk.append(np.stack([m.dumps[f"layer{l}.top_indices"].reshape(-1) for l in range(2)]))
            if s in GPTOSS_PROBES:
                for k in GPTOSS_PROBE_KEYS:
                    arrays[f"probe{s}.{k}"] = m.dumps[k].reshape(-1).astype(np.float32)
            if s == GPTOSS_STEPS:
                for k, v in m.dumps.items():
                    if STAGE_RE.match(k):
                        arrays[f"last.{k}"] = np.asarray(v).reshape(-1).astype(np.float32)
        arrays["next_ids"] = np.array(nxt, np.int32)          # after the prompt, then after each call
        arrays["top_indices"] = np.stack(topk).astype(np.int32)  # [call][layer][k]
        m = O.OracleModel(d, ctx=meta["ctx"], kv_bf16=True)
        lp, lids = meta["long_prompt"], meta["long_ids"]
        for i, t in enumerate(lp):
            m.forward_token(t, i)
        for s in range(1, GPTOSS_LONG_STEPS + 1):
            m.forward_token(lids[s - 1], len(lp) + s - 1)
        for k, v in m.dumps.items():
            if STAGE_RE.match(k):
                arrays[f"long.{k}"] = np.asarray(v).reshape(-1).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "gptoss_2l_bf16kv.npz"), **arrays)
    print("gptoss_2l_bf16kv", len(arrays), "arrays")


# The reference's command-line contract on the tiny model: a SERVICE=1
# session (service_loop, picchio.c:2700-2795) with prefix reuse (TURN keep),
# greedy and sampled turns, the range and vocabulary errors, RESET and
# SHUTDOWN; and a one-shot OUTPUT=ids run from INPUT_FILE.  stdout is kept
# byte for byte.
SERVICE_ENV = {"CTX": "128", "SEED": "42", "REP": "1.1", "ECAP": "8"}


def service_script(prompt):
    p = prompt
    turns = [
        f"TURN 8 0 0 1 0 12 {' '.join(map(str, p[:12]))}",
        f"TURN 6 20 0 1 0 5 {' '.join(map(str, p[12:17]))}",     # keep the whole first turn
        f"TURN 5 7 0.8 0.9 40 4 {' '.join(map(str, p[17:21]))}",  # keep a prefix; sampled
        f"TURN 4 999 0 1 0 3 {' '.join(map(str, p[21:24]))}",      # keep > pos: BAD_RANGE
        "TURN 4 0 0 1 0 2 5 5000",                                  # id outside the vocabulary
        "TURN 5 0 0 1 0 125 " + " ".join(map(str, (p * 3)[:125])),  # runs into the context end
        "RESET",
        f"TURN 6 0 1.0 0.95 50 10 {' '.join(map(str, p[24:34]))}",
        "SHUTDOWN",
    ]
    return "\n".join(turns) + "\n"


def make_service():
    cfg = SynthConfig()
    with tempfile.TemporaryDirectory() as d:
        make_model(d, cfg, 1234)
        prompt = random_prompt(PROMPT_LEN, cfg.vocab_size, 7)
        script = service_script(prompt)
        env = dict(os.environ, MODEL=d, SERVICE="1", OMP_NUM_THREADS="4", **SERVICE_ENV)
        svc = subprocess.run([O.REF_BIN_PATH], env=env, input=script, capture_output=True, text=True, cwd=d,
                             check=True).stdout
        pf = os.path.join(d, "prompt.txt")
        with open(pf, "w") as f:
            f.write(" ".join(map(str, prompt)))
        ids_env = {"OUTPUT": "ids", "TEMPERATURE": "0", "REP": "1", "MAX": "24", "CTX": "512"}
        env = dict(os.environ, MODEL=d, INPUT_FILE=pf, OMP_NUM_THREADS="4", **ids_env)
        ids_out = subprocess.run([O.REF_BIN_PATH], env=env, capture_output=True, text=True, cwd=d,
                                 check=True).stdout
    meta = dict(seed=1234, prompt=prompt, service_env=SERVICE_ENV, script=script, service_stdout=svc,
                ids_env=ids_env, ids_stdout=ids_out)
    with open(os.path.join(HERE, "service_tiny.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print("service transcript:", svc.count("\n"), "lines;", "ids run:", ids_out.split()[:8])


def make_mxfp4():
    """mxfp4.npz: the reference converter's MXFP4 dequantization on seeded
    inputs.  Shapes (rows, columns): a GPT-OSS gate_up row block and two
    small ones; codes uniform over all 16 (so -0 and +-6 occur), E8M0 bytes
    over [100, 140] plus the extremes 0 and 254 in the small case."""
    src = O.reference_dir()
    if not src:
        raise SystemExit("set REF=<reference checkout> (convert.py is imported from it)")
    sys.path.insert(0, src)
    import convert  # the reference converter (needs numpy only for these functions)
    rng = np.random.default_rng(4)
    out = {}
    for tag, (rows, cols) in {"a": (64, 2880), "b": (16, 64), "c": (8, 96)}.items():
        nb = cols // 32
        blocks = rng.integers(0, 256, size=(rows, nb, 16), dtype=np.uint8)
        e8 = rng.integers(100, 141, size=(rows, nb), dtype=np.uint8)
        if tag == "b":
            e8[0, 0], e8[1, 1] = 0, 254
        sc = convert.decode_e8m0(e8.reshape(-1))
        fast = convert.dequant_mxfp4_fast(blocks.reshape(-1), sc, (rows, cols), 32)
        if tag != "a":
            slow = convert.dequant_mxfp4(blocks.reshape(-1), sc, (rows, cols), 32)
            assert np.array_equal(fast.view(np.uint32), slow.view(np.uint32)), tag
        out.update({f"{tag}_blocks": blocks, f"{tag}_e8m0": e8, f"{tag}_values": fast.astype(np.float32)})
    np.savez_compressed(os.path.join(HERE, "mxfp4.npz"), **out)
    print("mxfp4.npz", len(out), "arrays")


if __name__ == "__main__":
    O.build(ref=True)
    which = sys.argv[1:] or ["tiny", "gptoss", "service", "mxfp4"]
    if "tiny" in which:
        for n, o in VARIANTS.items():
            make_variant(n, o)
        add_sampled("tiny_gs32_i8")
        make_kernels()
    if "gptoss" in which:
        make_gptoss()
    if "gptoss" in which or "gptoss_bf16kv" in which:
        make_gptoss_bf16kv()
    if "service" in which:
        make_service()
    if "mxfp4" in which:
        make_mxfp4()
