"""Parity at the GPT-OSS head and expert shapes the bench runs.

The container (tests/golden/make_golden.py, GPTOSS) has d_model 2880, 64 q /
8 kv heads x 64 with sinks, a 128-window layer and a full layer, 32 experts
top-4 INT4 gs32 and INT8 dense weights.  The goldens come from the
reference binary itself: its greedy ids, the router top-k and logits of
every forward_token call (one reference run per call, each dumping its last
forward, picchio.c:204-249), the hidden states at calls that cross the
window edge (positions 126-130) and 255-257, and every stage tensor of the
last call.

Bars: greedy ids identical, router top-k identical,
per-layer hidden states within 1e-2 relative L2.  With the reference's fp32
KV cache the hidden states are also held to 1e-4 (the GEMVs round each
input row to 22 significant bits; measured errors stay near 1e-5).

The bf16 KV cache stores K and V rounded to bf16 (2^-9 relative).  On this
random-weight model that alone moves the hidden states by up to ~1.8 %
from the reference's fp32-cache values (the oracle with the same rounding,
OracleModel(kv_bf16=True), shows the same gap) and reorders near-tied
router logits, so the bf16 decode is teacher-forced on the reference's ids
and checked against the bf16 oracle (gptoss_2l_bf16kv.npz): each call's
next id and top-k equal to the bf16 oracle's, the hidden states within
1e-3 and every other stage tensor within 1e-2 of its.
"""
import json
import os

import numpy as np
import pytest

from picchio_b200.synth import SynthConfig, make_model

GOLD = os.path.join(os.path.dirname(__file__), "golden")
HIDDEN_REL_L2 = 1e-2
FP32_KV_REL_L2 = 1e-4
BF16_KV_REL_L2 = 1e-3

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def gold():
    with open(os.path.join(GOLD, "gptoss_2l.json")) as f:
        meta = json.load(f)
    return meta, np.load(os.path.join(GOLD, "gptoss_2l_dumps.npz"))


@pytest.fixture(scope="module")
def gold_bf16():
    """The bf16-KV oracle's stage tensors for the same (teacher-forced) calls."""
    return np.load(os.path.join(GOLD, "gptoss_2l_bf16kv.npz"))


@pytest.fixture(scope="module")
def model_dir(gold, tmp_path_factory):
    meta, _ = gold
    d = str(tmp_path_factory.mktemp("gptoss_2l"))
    make_model(d, SynthConfig(**meta["options"]), meta["seed"])
    return d


def _stage_checks(model, dumps, prefix, names, bar):
    """Compares traced stage tensors with the golden ones; returns the count.
    Every tensor within HIDDEN_REL_L2, the hidden states within bar, top-k
    indices identical."""
    n = 0
    for name in names:
        ref = dumps[prefix + name]
        got = model.stage(name, ref.size)
        if name.endswith("top_indices"):
            assert np.array_equal(got, ref), (prefix, name)
        else:
            err = rel_l2(got, ref)
            assert err < HIDDEN_REL_L2, (prefix, name, err)
            if name.endswith((".input", ".output", "final_norm", "pre_moe_norm", "pre_attn_norm")):
                assert err < bar, (prefix, name, err)
        n += 1
    return n


@pytest.mark.parametrize("kv_bf16", [False, True], ids=["fp32_kv", "bf16_kv"])
def test_decode_against_reference(gold, gold_bf16, model_dir, kv_bf16):
    """Prefill of 120 ids, then 143 decode calls (positions 120..262) on the
    fast path (CUDA graphs; with the bf16 cache the tensor-core attention):
    the next id and the router top-k of both layers at every call; traced
    stage tensors at the probe calls and all of them at the last call."""
    from picchio_b200 import Model
    meta, dumps = gold
    ids, topk, probes = meta["ids"], meta["top_indices"], set(meta["probes"])
    P = len(meta["prompt"])
    bar = BF16_KV_REL_L2 if kv_bf16 else FP32_KV_REL_L2
    stages = gold_bf16 if kv_bf16 else dumps
    last_names = [k[len("last."):] for k in dumps.files if k.startswith("last.")]
    with Model(model_dir, ctx=meta["ctx"], kv_bf16=kv_bf16) as m:
        tok = m.prefill_tokens(meta["prompt"], 0)
        assert tok == (int(gold_bf16["next_ids"][0]) if kv_bf16 else ids[0])
        n_stage = 0
        for s in range(1, meta["steps"] + 1):
            pos = P + s - 1
            tok_in = ids[s - 1] if kv_bf16 else tok  # bf16: teacher-forced on the reference's ids
            tok = m.forward_token(tok_in, pos)
            if kv_bf16:
                assert tok == int(gold_bf16["next_ids"][s]), (s, pos)
                assert m.routing()[:, 0, :].tolist() == gold_bf16["top_indices"][s - 1].tolist(), (s, pos)
            else:
                if s < len(ids):
                    assert tok == ids[s], (s, pos)
                assert m.routing()[:, 0, :].tolist() == topk[s - 1], (s, pos)
            if s in probes:
                # the same call again with stage tracing (idempotent: it
                # rewrites the KV rows of this position with the same values)
                m.set_trace(True)
                assert m.forward_token(tok_in, pos) == tok
                names = last_names if s == meta["steps"] else meta["probe_keys"]
                prefix = "last." if s == meta["steps"] else f"probe{s}."
                n_stage += _stage_checks(m, stages, prefix, names, bar)
                m.set_trace(False)
        assert n_stage >= 60


@pytest.mark.parametrize("chunk", [64, 1024])
@pytest.mark.parametrize("kv_bf16", [False, True], ids=["fp32_kv", "bf16_kv"])
def test_long_prefill_against_reference(gold, gold_bf16, model_dir, chunk, kv_bf16):
    """A 300-id prompt in 64-position steps (GEMV experts) and in one
    300-position step (1200 routed pairs: expert GEMMs on tcgen05, dense
    projections on tcgen05), then 8 greedy calls; the stage tensors of the
    last call against the reference's."""
    from picchio_b200 import Model
    meta, dumps = gold
    lp, want = meta["long_prompt"], meta["long_ids"]
    names = [k[len("long."):] for k in dumps.files if k.startswith("long.")]
    with Model(model_dir, ctx=meta["ctx"], kv_bf16=kv_bf16, max_batch=1, prefill_chunk=chunk) as m:
        tok = m.prefill_tokens(lp, 0)
        got = [tok]
        pos = len(lp)
        for s in range(1, meta["long_steps"] + 1):
            tok_in = want[s - 1] if kv_bf16 else tok
            if s == meta["long_steps"]:
                m.set_trace(True)
            tok = m.forward_token(tok_in, pos)
            got.append(tok)
            pos += 1
        assert got[:len(want)] == want
        if kv_bf16:  # against the bf16-KV oracle; f16 expert operands at chunk 1024
            tol = 3e-3 if chunk > 64 else BF16_KV_REL_L2
            assert _stage_checks(m, gold_bf16, "long.", names, tol) >= 40
        else:
            tol = 2e-3 if chunk > 64 else FP32_KV_REL_L2
            assert _stage_checks(m, dumps, "long.", names, tol) >= 40


@pytest.mark.parametrize("M", [1, 4, 64, 512])
def test_moe_experts_configs1_against_oracle(model_dir, M):
    """BASELINE configs[1] (d_model 2880, expert FFN 2880, 32 experts, top-4,
    INT4 gs32): pc_moe_experts with uniform random top-4 routing against the
    oracle's moe_forward restatement (oracle.c, pinned bit-exact to the
    reference).  M <= 64 runs the GEMV path (within 1e-5); M = 512 routes 64
    pairs per expert onto the tcgen05 expert GEMMs (f16 operands, within
    2e-3), checked on every 16th row."""
    import torch
    from oracle import oracle as O
    from picchio_b200 import Model
    orc = O.OracleModel(model_dir, ctx=64)
    D, E, K = orc.c.hidden, orc.c.n_experts, orc.c.topk
    rng = np.random.default_rng(100 + M)
    sel = np.stack([rng.choice(E, K, replace=False) for _ in range(M)]).astype(np.int32)
    w = rng.random((M, K)).astype(np.float32)
    w /= w.sum(1, keepdims=True)
    x = rng.standard_normal((M, D)).astype(np.float32)
    with Model(model_dir, ctx=64, max_batch=max(M, 1)) as m:
        out = m.moe_experts(torch.from_numpy(x).cuda(), torch.from_numpy(sel).cuda(), torch.from_numpy(w).cuda(),
                            0).cpu().numpy()
    tol = 2e-3 if M >= 256 else 1e-5
    rows = range(0, M, 16) if M >= 256 else range(M)
    for layer in (0,):
        for r in rows:
            ref = orc.moe(x[r], layer, sel=sel[r].tolist(), wts=w[r])
            bad = np.where(~np.isfinite(out[r]))[0]
            assert len(bad) == 0 and np.isfinite(ref).all(), (M, r, bad[:8].tolist(), len(bad),
                                                              bool(np.isfinite(ref).all()))
            assert rel_l2(out[r], ref) < tol, (M, r, rel_l2(out[r], ref))
