"""Device sampling (sample_logits, picchio.c:1540-1649) through the C ABI.

Chains of draws are compared with the oracle's restatement (oracle.c
or_sample, which the CPU tests pin bit for bit to the reference's own
sample_logits): the same ids, generator state and history after every chain.
End to end, the sampled ids of the reference binary on the golden tiny
container (tests/golden/make_golden.py ``add_sampled``) are reproduced by
prefill + decode with the device sampler.
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

from oracle import oracle as O
from picchio_b200.synth import SynthConfig, make_model

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")

SETTINGS = [
    # (temperature, top_p, top_k, rep)
    (1.0, 0.95, 50, 1.1),     # the reference's defaults: candidates sorted in the block
    (0.7, 0.9, 0, 1.0),       # no top-k: the large candidate sort
    (1.0, 0.5, 3000, 1.2),    # top-k above the in-block limit: the large sort
    (0.8, 0.99, 2048, 1.05),  # top-k at the in-block limit
    (1.3, 1.0, 0, 1.0),       # no truncation: every sum runs over the whole vocabulary
    (0.0, 1.0, 0, 1.3),       # penalized greedy
]


@pytest.fixture(scope="module")
def model_for_vocab():
    from picchio_b200 import Model, ModelConfig
    models = {}

    def get(V):
        if V not in models:
            cfg = ModelConfig(hidden=256, n_layers=1, n_heads=8, n_kv_heads=2, head_dim=32, n_experts=8, topk=2,
                              intermediate=256, vocab=V)
            models[V] = Model.synthetic(cfg, seed=3, ctx=64)
        return models[V]

    yield get
    for m in models.values():
        m.close()


@pytest.mark.parametrize("V", [1024, 201088])
@pytest.mark.parametrize("setting", SETTINGS)
def test_device_draws_match_oracle(model_for_vocab, V, setting):
    import torch
    T, tp, tk, rep = setting
    m = model_for_vocab(V)
    rng = np.random.default_rng(V * 7 + tk)
    hist0 = rng.integers(0, V, 300)
    m.set_sampling(T, tp, tk, rep)
    m.rng = 123456789
    m.history_reset()
    m.history_push(hist0)
    st = O.SamplerState(123456789, hist0)
    for i in range(12 if V > 4096 else 40):
        lg = (rng.standard_normal(V) * 2.5).astype(np.float32)
        if i % 3 == 2:  # ties at the top-k threshold and among the probabilities
            lg = np.round(lg * 2.0).astype(np.float32) / 2.0
        d = m.sample(torch.from_numpy(lg).cuda())
        o, _ = O.sample(lg, T, tp, tk, rep, st)
        assert d == o, (i, d, o)
    assert m.rng == st.rng
    assert m.history() == st.history
    m.set_sampling(None)


def test_candidate_overflow_is_an_error_and_the_context_stays_usable(model_for_vocab):
    """More than 4096 top-p candidates with top-k <= 2048 (every value tied at
    the threshold) is reported as PC_ERR_RANGE by the device; the next draw
    works."""
    import torch
    from picchio_b200 import PicchioError
    V = 201088
    m = model_for_vocab(V)
    m.set_sampling(1.0, 0.9, 50, 1.0)
    m.rng = 5
    m.history_reset()
    with pytest.raises(PicchioError) as e:
        m.sample(torch.zeros(V, device="cuda"))
    assert e.value.status_name == "PC_ERR_RANGE"
    lg = np.random.default_rng(1).standard_normal(V).astype(np.float32)
    st = O.SamplerState(m.rng, m.history())
    assert m.sample(torch.from_numpy(lg).cuda()) == O.sample(lg, 1.0, 0.9, 50, 1.0, st)[0]
    m.set_sampling(None)


@pytest.fixture(scope="module")
def tiny():
    with open(os.path.join(GOLD, "tiny_gs32_i8.json")) as f:
        meta = json.load(f)
    return meta


@pytest.mark.parametrize("run", [0, 1])
def test_sampled_ids_match_reference_binary(tiny, tmp_path, run):
    """The reference's OUTPUT=ids with its sampler on (TEMPERATURE / TOPP /
    TOPK / REP / SEED): prefill (history seeded with the prompt when REP > 1,
    picchio.c:1963-1967) then forward_token steps, each drawing on the device."""
    from picchio_b200 import Model
    r = tiny["sampled"][run]
    env = r["env"]
    d = str(tmp_path)
    make_model(d, SynthConfig(**tiny["options"]), tiny["seed"])
    with Model(d, ctx=tiny["ctx"]) as model:
        model.set_sampling(float(env["TEMPERATURE"]), float(env["TOPP"]), int(env["TOPK"]), float(env["REP"]))
        model.rng = int(env["SEED"])
        model.history_reset()
        if float(env["REP"]) > 1.0:
            model.history_push(tiny["prompt"])
        ids = model.generate(tiny["prompt"], len(r["ids"]))
    assert ids == r["ids"]


def test_device_loop_samples_like_single_steps(tiny, tmp_path):
    """pc_generate (one graph per step, ids fed back on the device) draws the
    same ids as pc_forward_token steps from the same generator state; turning
    sampling off restores the greedy ids."""
    from picchio_b200 import Model
    d = str(tmp_path)
    make_model(d, SynthConfig(**tiny["options"]), tiny["seed"])
    prompt = tiny["prompt"]
    with Model(d, ctx=tiny["ctx"]) as model:
        model.set_sampling(1.0, 0.95, 50, 1.1)
        model.rng = 99
        model.history_reset()
        tok = model.prefill_tokens(prompt, 0)
        rng_after_prefill, hist = model.rng, model.history()
        steps, pos = [], len(prompt)
        t = tok
        for _ in range(24):
            t = model.forward_token(t, pos)
            steps.append(t)
            pos += 1
        model.rng = rng_after_prefill
        model.history_reset()
        model.history_push(hist)
        dev, _ = model.generate_device(tok, len(prompt), 24)
        assert dev == steps
        model.set_sampling(None)
        assert model.generate(prompt, 16) == tiny["ids_batched"][:16]
