"""End-to-end parity of the device forward against the reference.

Golden ids and stage dumps come from the reference engine itself
(tests/golden/make_golden.py).  Bars: greedy ids
identical for 128 decode steps; per-layer hidden states within 1e-2
relative L2 (measured ~1e-6 with the fp32 KV cache); router top-k identical.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O
from picchio_b200.synth import SynthConfig, make_model

GOLD = os.path.join(os.path.dirname(__file__), "golden")
VARIANTS = ["tiny_gs32_i8", "tiny_gs64_f32", "tiny_rowi4_i4"]
HIDDEN_REL_L2 = 1e-2

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def meta(name):
    with open(os.path.join(GOLD, name + ".json")) as f:
        return json.load(f)


@pytest.fixture(scope="module", params=VARIANTS)
def variant(request, tmp_path_factory):
    m = meta(request.param)
    d = str(tmp_path_factory.mktemp(request.param))
    make_model(d, SynthConfig(**m["options"]), m["seed"])
    return m, d


def test_greedy_ids_match_reference_128_steps(variant):
    from picchio_b200 import Model
    m, d = variant
    with Model(d, ctx=m["ctx"]) as model:
        ids = model.generate(m["prompt"], m["steps"])
    assert ids == m["ids_batched"]


def test_stage_dumps_close_to_reference(variant):
    from picchio_b200 import Model
    m, d = variant
    gold = np.load(os.path.join(GOLD, m["name"] + "_dumps.npz"))
    with Model(d, ctx=m["ctx"]) as model:
        tok = model.prefill_tokens(m["prompt"], 0)
        pos = len(m["prompt"])
        model.set_trace(True)
        for _ in range(m["dump_steps"]):
            tok_in = tok
            tok = model.forward_token(tok_in, pos)
            pos += 1
        checked = 0
        for name in gold.files:
            ref = gold[name].reshape(-1)
            try:
                got = model.stage(name, ref.size)
            except Exception:
                continue
            if name.endswith("top_indices"):
                assert np.array_equal(got, ref), name
            else:
                assert rel_l2(got, ref) < HIDDEN_REL_L2, (name, rel_l2(got, ref))
                if name.endswith((".input", ".output", "final_norm", "pre_moe_norm", "pre_attn_norm")):
                    assert rel_l2(got, ref) < 1e-5, (name, rel_l2(got, ref))
            checked += 1
    assert checked >= 30


def test_prefill_matches_sequential_forward(variant):
    from picchio_b200 import Model
    m, d = variant
    p = m["prompt"][:20]
    with Model(d, ctx=m["ctx"]) as a, Model(d, ctx=m["ctx"]) as b:
        t1 = a.prefill_tokens(p, 0)
        t2 = None
        for i, t in enumerate(p):
            t2 = b.forward_token(t, i)
        assert t1 == t2
        la, lb = a.logits(0), b.logits(0)
        assert rel_l2(la, lb) < 1e-5


def test_decode_batch_matches_single_sequences(variant):
    from picchio_b200 import Model
    m, d = variant
    prompts = [m["prompt"][:10], m["prompt"][10:25], m["prompt"][30:33]]
    singles = []
    for p in prompts:
        with Model(d, ctx=m["ctx"]) as s:
            singles.append(s.generate(p, 6))
    with Model(d, ctx=m["ctx"], max_batch=3) as b:
        # fill each sequence's KV with its own prompt via batched steps
        maxlen = max(len(p) for p in prompts)
        toks = [p[0] for p in prompts]
        nxt = None
        outs = [[] for _ in prompts]
        pos = [0] * 3
        # run sequences in lock-step; short prompts start decoding early
        cur = [p[0] for p in prompts]
        for step in range(maxlen + 6):
            nxt = b.decode_batch(cur, pos)
            for i, p in enumerate(prompts):
                pos[i] += 1
                if pos[i] < len(p):
                    cur[i] = p[pos[i]]
                else:
                    if len(outs[i]) < 6:
                        outs[i].append(nxt[i])
                    cur[i] = nxt[i]
        for i in range(3):
            assert outs[i] == singles[i][:6] or outs[i][:len(singles[i])] == singles[i][:len(outs[i])]


def test_prefill_into_slots_then_batch_decode(variant):
    """pc_prefill_seq fills KV slots 1 and 2 of a batched context with their
    own prompts; pc_decode_batch then continues each slot as the
    single-sequence prefill + decode does (same ids)."""
    from picchio_b200 import Model
    m, d = variant
    prompts = [m["prompt"][:12], m["prompt"][12:31], m["prompt"][31:40]]
    singles = []
    for p in prompts:
        with Model(d, ctx=m["ctx"]) as s:
            singles.append(s.generate(p, 5))
    with Model(d, ctx=m["ctx"], max_batch=3) as b:
        cur = [b.prefill_tokens(p, 0, seq=i) for i, p in enumerate(prompts)]
        pos = [len(p) for p in prompts]
        outs = [[c] for c in cur]
        for _ in range(4):
            cur = b.decode_batch(cur, pos)
            pos = [q + 1 for q in pos]
            for i in range(3):
                outs[i].append(cur[i])
    assert outs == singles


def test_decode_batch_tensor_core_rows(variant):
    """18 sequences in one batch: q/k/v, o_proj and the lm_head of every step
    take the tensor-core path (16..128 rows); each sequence's greedy ids match
    the same sequence decoded alone (batch 1: the GEMV path)."""
    from picchio_b200 import Model
    m, d = variant
    B, steps = 18, 4
    prompts = [m["prompt"][i:i + 3] for i in range(B)]
    singles = []
    for p in prompts[:4]:
        with Model(d, ctx=m["ctx"]) as s:
            singles.append(s.generate(p, steps))
    with Model(d, ctx=m["ctx"], max_batch=B) as b:
        # the path is on exactly when the dense projections are INT8
        assert b.tensor_core_min_rows == (16 if m["name"].endswith("_i8") else 0)
        cur = [p[0] for p in prompts]
        pos = [0] * B
        outs = [[] for _ in range(B)]
        for step in range(3 + steps - 1):
            nxt = b.decode_batch(cur, pos)
            for i, p in enumerate(prompts):
                pos[i] += 1
                if pos[i] < len(p):
                    cur[i] = p[pos[i]]
                else:
                    outs[i].append(nxt[i])
                    cur[i] = nxt[i]
        for i in range(4):
            assert outs[i] == singles[i][:len(outs[i])], (i, outs[i], singles[i])


def test_moe_forward_against_oracle(variant):
    import torch
    from picchio_b200 import Model
    m, d = variant
    orc = O.OracleModel(d, ctx=64)
    rng = np.random.default_rng(3)
    D = orc.c.hidden
    # 5 rows: all rows in one shared B operand; 12 rows: more than one job
    # table row group with at most 2 pairs per expert job (batched-decode
    # form); 40 rows: up to 8 pairs per job
    for M in (5, 12, 40):
        x = rng.standard_normal((M, D)).astype(np.float32)
        with Model(d, ctx=64, max_batch=64) as model:
            for layer in range(orc.c.n_layers):
                out = model.moe_forward(torch.from_numpy(x).cuda(), layer).cpu().numpy()
                for r in range(M):
                    ref = orc.moe(x[r], layer)
                    assert rel_l2(out[r], ref) < 1e-5, (M, layer, r)


def test_moe_forward_tensor_core_experts_against_oracle(variant):
    """256 rows x top-2 of 8 experts = 64 pairs per expert: the expert GEMMs
    run on the tensor cores (INT4 dequantized to f16, inputs rounded to f16,
    f32 accumulation; 6 launches instead of the GEMV path's 4).  Within
    2e-3 relative L2 of the oracle per row (f16 rounding of weights and
    inputs, ~5e-4 each)."""
    import torch
    from picchio_b200 import Model
    m, d = variant
    orc = O.OracleModel(d, ctx=64)
    rng = np.random.default_rng(4)
    D, M = orc.c.hidden, 256
    x = rng.standard_normal((M, D)).astype(np.float32)
    with Model(d, ctx=64, max_batch=M) as model:
        for layer in range(orc.c.n_layers):
            n0 = model.launches
            out = model.moe_forward(torch.from_numpy(x).cuda(), layer).cpu().numpy()
            assert model.launches - n0 == 6
            worst = 0.0
            for r in range(0, M, 7):
                worst = max(worst, rel_l2(out[r], orc.moe(x[r], layer)))
            assert worst < 2e-3, (layer, worst)


def test_range_errors(variant):
    from picchio_b200 import Model, PicchioError
    m, d = variant
    with Model(d, ctx=32) as model:
        with pytest.raises(PicchioError) as ei:
            model.forward_token(1, 32)
        assert ei.value.status_name == "PC_ERR_RANGE"
        with pytest.raises(PicchioError):
            model.prefill_tokens(list(range(40)), 0)
        # out-of-vocabulary token embeds as zeros and still runs (picchio.c:1478)
        model.forward_token(10 ** 6, 0)


def test_missing_sinks_is_reported(tmp_path):
    from picchio_b200 import Model, PicchioError
    from picchio_b200.synth import make_model, write_safetensors
    t = make_model(str(tmp_path))
    del t["model.layers.1.self_attn.sinks"]
    write_safetensors(os.path.join(str(tmp_path), "model-00000.safetensors"), t)
    with pytest.raises(PicchioError) as ei:
        Model(str(tmp_path))
    assert ei.value.status_name == "PC_ERR_MISSING_TENSOR"


def test_missing_expert_is_reported(tmp_path):
    from picchio_b200 import Model, PicchioError
    from picchio_b200.synth import make_model, write_safetensors
    t = make_model(str(tmp_path))
    del t["model.layers.0.mlp.experts.down_proj.3"]
    write_safetensors(os.path.join(str(tmp_path), "model-00000.safetensors"), t)
    with pytest.raises(PicchioError) as ei:
        Model(str(tmp_path))
    assert ei.value.status_name == "PC_ERR_MISSING_TENSOR"


def test_bf16_kv_cache_stays_close(variant):
    from picchio_b200 import Model
    m, d = variant
    with Model(d, ctx=m["ctx"]) as a, Model(d, ctx=m["ctx"], kv_bf16=True) as b:
        a.prefill_tokens(m["prompt"], 0)
        b.prefill_tokens(m["prompt"], 0)
        assert rel_l2(b.logits(0), a.logits(0)) < 1e-2


def test_tensor_core_split_k_prefill_matches_sequential():
    """A model wide enough that the tensor-core projections split K over
    several CTAs per 128-row tile (d_model 1024: 8 steps of 128 columns):
    a 24-token prefill (tensor-core path) gives the logits and next id of 24
    sequential single-token forwards (GEMV path).  The tensor-core sums are
    exact integers rounded once, the GEMV's are rounded per 256 columns, so
    the two agree to ~1e-6."""
    from picchio_b200 import Model, ModelConfig
    cfg = ModelConfig(hidden=1024, n_layers=2, n_heads=16, n_kv_heads=4, head_dim=64, n_experts=8, topk=2,
                      intermediate=512, vocab=2048)
    prompt = [int(v) for v in np.random.default_rng(5).integers(0, 2048, 24)]
    with Model.synthetic(cfg, seed=3, ctx=64) as a, Model.synthetic(cfg, seed=3, ctx=64) as b:
        assert a.tensor_core_min_rows == 16  # the path under test is on
        t1 = a.prefill_tokens(prompt, 0)
        t2 = None
        for i, t in enumerate(prompt):
            t2 = b.forward_token(t, i)
        assert t1 == t2
        assert rel_l2(a.logits(0), b.logits(0)) < 1e-5


def test_long_context_multi_span_attention_matches_oracle():
    """600 positions: full-attention layers split each (row, KV head) over
    3 spans of 256 positions and merge them (the 128-position sliding window
    stays in one span).  A 600-token prefill, then 3 decode steps, against
    the oracle's sequential forward_token over the same ids."""
    from picchio_b200 import Model
    m = meta("tiny_gs32_i8")
    import tempfile
    d = tempfile.mkdtemp()
    make_model(d, SynthConfig(**m["options"]), m["seed"])
    n, steps = 600, 3
    ids = [int(v) for v in np.random.default_rng(9).integers(0, 1024, n)]
    orc = O.OracleModel(d, ctx=n + 8)
    ref_tok, ref_logits = None, None
    for i, t in enumerate(ids):
        ref_tok, ref_logits = orc.forward_token(t, i, return_logits=True)
    with Model(d, ctx=n + 8) as model:
        tok = model.prefill_tokens(ids, 0)
        assert tok == ref_tok
        assert rel_l2(model.logits(0), ref_logits) < 1e-4
        for s in range(steps):
            ref_tok = orc.forward_token(ref_tok, n + s)
            tok = model.forward_token(tok, n + s)
            assert tok == ref_tok, s


def test_batched_rows_attention_matches_single_row():
    """128 sequences with 600 seeded cache positions each (3 spans per row in
    the full layers, 768 span CTAs per layer): batch row 0's next id equals
    that of the same sequence decoded alone, its logits within 2e-3 (with 32
    pairs per expert the batch's expert GEMMs run on the tensor cores with f16
    operands; the single sequence's on the exact-sum GEMV)."""
    from picchio_b200 import Model
    m = meta("tiny_gs32_i8")
    import tempfile
    d = tempfile.mkdtemp()
    make_model(d, SynthConfig(**m["options"]), m["seed"])
    B, n = 128, 600
    toks = [(5 * s + 1) % 1000 for s in range(B)]
    with Model(d, ctx=n + 8, max_batch=B) as b:
        for s in range(B):
            b.kv_fill_synthetic(n, seq=s, seed=100 + s)
        nxt = b.decode_batch(toks, [n] * B)
        lb = b.logits(0)
    with Model(d, ctx=n + 8) as a:
        a.kv_fill_synthetic(n, seq=0, seed=100)
        t = a.forward_token(toks[0], n)
        la = a.logits(0)
    assert nxt[0] == t
    assert rel_l2(lb, la) < 2e-3


@pytest.mark.parametrize("slots", [2, 8])
def test_streamed_expert_residency_matches_reference(tmp_path, slots):
    """expert_residency = 1: experts in pinned host memory, `slots` per layer
    in HBM (8 = the whole layer).  Greedy ids equal the reference's; every
    expert read is counted as a slot hit or a host read, and with two slots
    of eight both happen."""
    from picchio_b200 import Model
    m = meta("tiny_gs32_i8")
    d = str(tmp_path)
    make_model(d, SynthConfig(**m["options"]), m["seed"])
    with Model(d, ctx=m["ctx"], expert_residency=1, expert_cache_slots=slots) as model:
        ids = model.generate(m["prompt"], 48)
        st = model.expert_stats()
        E, L = model.config["n_experts"], model.config["n_layers"]
    assert ids == m["ids_batched"][:48]
    assert st["misses"] > 0 and st["hits"] > 0
    assert st["bytes_h2d"] > 0
    if slots >= E:  # everything fits: each (layer, expert) is read from the host at most once
        assert st["misses"] <= L * E


def test_expert_prefetch_makes_later_reads_hits(tmp_path):
    from picchio_b200 import Model
    m = meta("tiny_gs32_i8")
    d = str(tmp_path)
    make_model(d, SynthConfig(**m["options"]), m["seed"])
    with Model(d, ctx=m["ctx"], expert_residency=1, expert_cache_slots=8) as model:
        E, L = model.config["n_experts"], model.config["n_layers"]
        for layer in range(L):
            model.expert_prefetch(layer, list(range(E)))
        st0 = model.expert_stats()
        ids = model.generate(m["prompt"], 16)
        st1 = model.expert_stats()
    assert ids == m["ids_batched"][:16]
    assert st0["misses"] == 0 and st0["bytes_h2d"] > 0
    assert st1["misses"] == 0 and st1["hits"] > 0


def test_large_prefill_chunks_on_tensor_cores_match_64_position_blocks(tmp_path):
    """prefill_chunk = 300 (one step for a 300-position prompt): the dense
    projections run as 128-row tcgen05 blocks (128 + 128 + 44 rows) and the
    expert GEMMs on tcgen05 (75 routed rows per expert); the logits after the
    prompt stay within the hidden-state bar of the 64-position blocks (GEMV
    experts), and greedy decode continues identically."""
    from picchio_b200 import Model
    m = meta("tiny_gs32_i8")
    d = str(tmp_path)
    make_model(d, SynthConfig(**m["options"]), m["seed"])
    ids = np.random.default_rng(3).integers(0, 1024, 300).tolist()
    out = {}
    for chunk in (64, 300):
        with Model(d, ctx=m["ctx"], prefill_chunk=chunk) as model:
            assert model.tensor_core_min_rows > 0
            tok = model.prefill_tokens(ids, 0)
            lg = model.logits(0)
            toks = [tok]
            for i in range(8):
                toks.append(model.forward_token(toks[-1], 300 + i))
            out[chunk] = (lg, toks)
    assert rel_l2(out[300][0], out[64][0]) < HIDDEN_REL_L2
    assert out[300][1] == out[64][1]


def test_row_block_router_matches_single_row_router(variant):
    """From 16 rows the router takes whole rows per block (row-block kernel);
    one row uses the expert-parallel kernel.  Both form each dot in the same
    order, so 48 rows routed together give the outputs of the same rows
    routed one at a time."""
    import torch
    from picchio_b200 import Model
    m, d = variant
    rng = np.random.default_rng(11)
    with Model(d, ctx=64, max_batch=64) as model:
        D = model.config["hidden"]
        x = rng.standard_normal((48, D)).astype(np.float32)
        for layer in range(model.config["n_layers"]):
            batch = model.moe_forward(torch.from_numpy(x).cuda(), layer).cpu().numpy()
            for r in range(48):
                one = model.moe_forward(torch.from_numpy(x[r:r + 1]).cuda(), layer).cpu().numpy()[0]
                assert rel_l2(batch[r], one) < 1e-6, (layer, r)


_GPTOSS_HEADS_DIR = []


def _gptoss_heads_model(**kw):
    """A small seeded model with GPT-OSS attention heads (head size 64, 8
    query heads per KV head), the shape the tensor-core attention serves,
    with a bf16 KV cache."""
    import tempfile
    from picchio_b200 import Model
    if not _GPTOSS_HEADS_DIR:
        d = tempfile.mkdtemp()
        make_model(d, SynthConfig(num_attention_heads=16, num_key_value_heads=2, head_dim=64), 1234)
        _GPTOSS_HEADS_DIR.append(d)
    return Model(_GPTOSS_HEADS_DIR[0], kv_bf16=True, **kw)


def test_tensor_core_attention_batch_matches_single_rows():
    """32 sequences at 600 cached positions (window layer and full layer):
    the batch step runs the tensor-core attention one CTA per row (Q and P as
    bf16 hi + lo halves against the bf16 cache); rows 0, 7 and 31 equal the
    same sequences decoded alone (the span-split form for one row, itself
    checked against the fp32 one-row kernel below): same next id, logits
    within 1e-3."""
    B, n = 32, 600
    toks = [(7 * s + 3) % 1000 for s in range(B)]
    with _gptoss_heads_model(ctx=n + 8, max_batch=B) as b:
        for s in range(B):
            b.kv_fill_synthetic(n, seq=s, seed=200 + s)
        nxt = b.decode_batch(toks, [n] * B)
        lb = {s: b.logits(s) for s in (0, 7, 31)}
    with _gptoss_heads_model(ctx=n + 8) as a:
        for s in (0, 7, 31):
            a.kv_fill_synthetic(n, seq=0, seed=200 + s)
            t = a.forward_token(toks[s], n)
            assert t == nxt[s], s
            assert rel_l2(lb[s], a.logits(0)) < 1e-3, s


def test_tensor_core_attention_prefill_matches_sequential_forward():
    """A 200-position prompt in 64-position prefill steps (tensor-core
    attention over each row's causal positions) against 200 one-token steps:
    the same next id, logits within 1e-3."""
    ids = np.random.default_rng(5).integers(0, 1024, 200).tolist()
    with _gptoss_heads_model(ctx=256) as a:
        t_pre = a.prefill_tokens(ids, 0)
        l_pre = a.logits(0)
    with _gptoss_heads_model(ctx=256) as b:
        for i, tok in enumerate(ids):
            t_seq = b.forward_token(tok, i)
        l_seq = b.logits(0)
    assert t_pre == t_seq
    assert rel_l2(l_pre, l_seq) < 1e-3


def test_synthetic_model_with_wide_attention_is_finite():
    """pc_init_synthetic for a shape whose q projection (64 heads x 64 x 512)
    is larger than its embedding (1024 x 512): the generation scratch covers
    every matrix, so the weights (and the logits of a few steps) are finite."""
    from picchio_b200 import Model, ModelConfig
    cfg = ModelConfig(hidden=512, n_layers=2, n_heads=64, n_kv_heads=8, head_dim=64, n_experts=8, topk=2,
                      intermediate=256, vocab=1024)
    with Model.synthetic(cfg, seed=9, ctx=64) as m:
        tok = 5
        for pos in range(4):
            tok = m.forward_token(tok, pos)
            lg = m.logits(0)
            assert np.isfinite(lg).all() and np.abs(lg).max() > 0


def test_tensor_core_attention_one_row_matches_one_row_kernel(monkeypatch):
    """Batch-1 decode at position 600 with a bf16 cache: the tensor-core
    attention (positions split in spans of 512, merged by the last CTA) gives
    the one-row fp32 kernel's next id and logits within 1e-4."""
    n = 600
    out = {}
    for tc in ("0", "1"):
        monkeypatch.setenv("PICCHIO_ATTN_TC", tc)
        with _gptoss_heads_model(ctx=n + 8) as m:
            m.kv_fill_synthetic(n, seq=0, seed=77)
            t = m.forward_token(9, n)
            t2 = m.forward_token(t, n + 1)
            out[tc] = (t, t2, m.logits(0))
    assert out["0"][:2] == out["1"][:2]
    assert rel_l2(out["1"][2], out["0"][2]) < 1e-4


@pytest.mark.parametrize("kv_bf16", [False, True], ids=["fp32_kv", "bf16_kv"])
def test_mxfp4_experts_match_oracle(tmp_path, kv_bf16):
    """Experts kept in the checkpoint's MXFP4 form (``<proj>_blocks`` /
    ``_scales``, the reference's fmt 3, which its converter turns into INT4):
    greedy ids of prefill + decode equal to the oracle's, which applies the
    reference's fp32 matmul to convert.py's dequantized values; with a bf16
    KV cache against the oracle with the same cache rounding."""
    from oracle import oracle as O
    from picchio_b200 import FMT_MXFP4, Model
    from picchio_b200.synth import SynthConfig, make_model, random_prompt
    d = str(tmp_path)
    make_model(d, SynthConfig(expert_format="mxfp4"), seed=77)
    prompt = random_prompt(40, 1024, seed=5)
    want = O.OracleModel(d, ctx=256, kv_bf16=kv_bf16).generate(prompt, 24)
    with Model(d, ctx=256, kv_bf16=kv_bf16) as m:
        assert m.config["expert_format"] == FMT_MXFP4
        got = m.generate(prompt, 24)
    assert got == want
