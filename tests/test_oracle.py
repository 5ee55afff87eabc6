"""The CPU oracle against the reference: golden fixtures and known answers.

The fixtures under tests/golden were produced by the reference itself
(tests/golden/make_golden.py); these tests pin oracle/oracle.c to them bit for
bit.  When the reference has been built here (oracle/_ref), random shapes are
also cross-checked against its own functions.
"""
import json
import math
import os

import numpy as np
import pytest

from oracle import oracle as O
from picchio_b200.synth import SynthConfig, make_model

GOLD = os.path.join(os.path.dirname(__file__), "golden")
VARIANTS = ["tiny_gs32_i8", "tiny_gs64_f32", "tiny_rowi4_i4"]


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def load_meta(name):
    with open(os.path.join(GOLD, name + ".json")) as f:
        return json.load(f)


@pytest.fixture(scope="module", params=VARIANTS)
def variant(request, tmp_path_factory):
    meta = load_meta(request.param)
    d = str(tmp_path_factory.mktemp(request.param))
    make_model(d, SynthConfig(**meta["options"]), meta["seed"])
    return meta, d


def test_oracle_greedy_ids_match_reference(variant):
    meta, d = variant
    m = O.OracleModel(d, ctx=meta["ctx"])
    ids = m.generate(meta["prompt"], meta["steps"])
    assert ids == meta["ids_sequential"]
    assert ids == meta["ids_batched"]


def test_oracle_stage_dumps_bit_exact(variant):
    meta, d = variant
    m = O.OracleModel(d, ctx=meta["ctx"])
    m.generate(meta["prompt"], meta["dump_steps"])
    gold = np.load(os.path.join(GOLD, meta["name"] + "_dumps.npz"))
    checked = 0
    for name in gold.files:
        if name not in m.dumps:
            continue  # *_nobias, v_heads, contribution: not restated separately
        assert np.array_equal(bits(gold[name].reshape(-1)), bits(np.asarray(m.dumps[name]).reshape(-1))), name
        checked += 1
    assert checked >= 40


def test_oracle_matmuls_bit_exact_vs_golden():
    g = np.load(os.path.join(GOLD, "kernels.npz"))
    for tag in "abcd":
        Oo, I, gs, S = [int(v) for v in g[f"i4_{tag}_shape"]]
        x = g[f"i4_{tag}_x"]
        if gs:
            y = O.matmul_i4_gs(x, g[f"i4_{tag}_q"], g[f"i4_{tag}_s"], Oo, I, gs)
        else:
            y = O.matmul_i4(x, g[f"i4_{tag}_q"], g[f"i4_{tag}_s"], Oo, I)
        assert np.array_equal(bits(y), bits(g[f"i4_{tag}_y"])), tag
        y8 = O.matmul_q8(x, g[f"i8_{tag}_q"], g[f"i8_{tag}_s"], Oo, I)
        assert np.array_equal(bits(y8), bits(g[f"i8_{tag}_y"])), tag


def test_known_answers_from_reference_self_test():
    # rmsnorm([1,2,3,4], w=1) -> x / sqrt(mean(x^2)) (picchio.c:2250-2264)
    o = O.rmsnorm(np.array([1, 2, 3, 4], np.float32), np.ones(4, np.float32), 1e-5)
    assert abs(o[0] - 1 / math.sqrt(7.5)) < 1e-4
    # softmax sums to 1 and keeps order (picchio.c:2266-2280)
    x = np.array([1.0, 2.0, 3.0], np.float32)
    lib = O.lib()
    lib.or_softmax(x.ctypes.data_as(O._fp), 3)
    assert abs(x.sum() - 1) < 1e-5 and x[2] > x[1] > x[0]
    # SwiGLU with gate=0 is 0; gate/up clamps at the limit (picchio.c:1416-1424)
    act = O.swiglu(np.array([0.0, 5.0, 100.0, 100.0, 100.0, -100.0], np.float32), 7.0)
    assert act[0] == 0.0
    s = 1 / (1 + math.exp(-1.702 * 7))
    assert abs(act[1] - (7 + 1) * 7 * s) < 1e-4
    assert abs(act[2] - (-7 + 1) * 7 * s) < 1e-4
    # RoPE at pos 0 is the identity (picchio.c:2310-2325)
    cs = np.empty(8, np.float32); sn = np.empty(8, np.float32)
    inv = np.ones(8, np.float32)
    lib.or_rope_cs(inv.ctypes.data_as(O._fp), 8, 0, 1.0, cs.ctypes.data_as(O._fp), sn.ctypes.data_as(O._fp))
    v = np.arange(16, dtype=np.float32)
    w = v.copy()
    lib.or_rope_rotate(w.ctypes.data_as(O._fp), 16, cs.ctypes.data_as(O._fp), sn.ctypes.data_as(O._fp))
    assert np.array_equal(v, w)


def test_router_topk_ties_go_to_lowest_index():
    # strict '>' in K argmax rounds (picchio.c:1330-1340)
    D, E = 4, 6
    R = np.zeros((E, D), np.float32)
    R[[1, 3, 4], 0] = 2.0
    R[5, 0] = 1.0
    logits, sel, w = O.router_topk(np.array([1, 0, 0, 0], np.float32), R, None, 3)
    assert list(sel) == [1, 3, 4]
    assert np.allclose(w, 1 / 3)


def test_dequant_definition():
    rng = np.random.default_rng(3)
    from picchio_b200.synth import quantize_int4
    w = (rng.standard_normal((16, 96)) * 0.02).astype(np.float32)
    pk, sc = quantize_int4(w, 32)
    dq = O.dequant_i4(pk, sc, 16, 96, 32)
    u = np.stack([pk & 0xF, pk >> 4], -1).reshape(16, 96).astype(np.int32) - 8
    ref = (u.astype(np.float32) * np.repeat(sc.reshape(16, 3), 32, axis=1)).astype(np.float32)
    assert np.array_equal(bits(dq), bits(ref))


@pytest.mark.skipif(O.ref_lib() is None, reason="reference not built here (oracle/_ref)")
@pytest.mark.parametrize("shape", [(64, 256, 32), (40, 2880, 32), (24, 320, 64), (16, 768, 0)])
def test_oracle_matches_compiled_reference_random(shape):
    import ctypes as C
    from picchio_b200.synth import quantize_int4, quantize_int8
    Oo, I, gs = shape
    R = O.ref_lib()
    fp = C.POINTER(C.c_float)
    rng = np.random.default_rng(Oo * 7 + I)
    w = (rng.standard_normal((Oo, I)) * 0.02).astype(np.float32)
    x = rng.standard_normal((3, I)).astype(np.float32)
    pk, sc = quantize_int4(w, gs)
    yr = np.empty((3, Oo), np.float32)
    if gs:
        R.ref_matmul_i4_gs(yr.ctypes.data_as(fp), x.ctypes.data_as(fp), pk.ctypes.data_as(C.POINTER(C.c_uint8)),
                           sc.ctypes.data_as(fp), 3, I, Oo, gs)
        yo = O.matmul_i4_gs(x, pk, sc, Oo, I, gs)
    else:
        R.ref_matmul_i4(yr.ctypes.data_as(fp), x.ctypes.data_as(fp), pk.ctypes.data_as(C.POINTER(C.c_uint8)),
                        sc.ctypes.data_as(fp), 3, I, Oo)
        yo = O.matmul_i4(x, pk, sc, Oo, I)
    assert np.array_equal(bits(yo), bits(yr))
    q, s = quantize_int8(w)
    R.ref_matmul_q8(yr.ctypes.data_as(fp), x.ctypes.data_as(fp), q.ctypes.data_as(C.POINTER(C.c_int8)),
                    s.ctypes.data_as(fp), 3, I, Oo)
    assert np.array_equal(bits(O.matmul_q8(x, q, s, Oo, I)), bits(yr))
    xx = rng.standard_normal(I).astype(np.float32)
    ww = (1 + 0.1 * rng.standard_normal(I)).astype(np.float32)
    yn = np.empty(I, np.float32)
    R.ref_rmsnorm(yn.ctypes.data_as(fp), xx.ctypes.data_as(fp), ww.ctypes.data_as(fp), I, 1e-5)
    assert np.array_equal(bits(O.rmsnorm(xx, ww, 1e-5)), bits(yn))


SAMPLER_SETTINGS = [
    # (temperature, top_p, top_k, rep): the reference defaults, a top-k-free
    # nucleus, no truncation at all, penalized greedy, a large top-k
    (1.0, 0.95, 50, 1.1),
    (0.7, 0.9, 0, 1.0),
    (1.3, 1.0, 0, 1.0),
    (0.0, 1.0, 0, 1.3),
    (1.0, 0.5, 3000, 1.2),
]


@pytest.mark.skipif(O.ref_lib() is None or not hasattr(O.ref_lib(), "ref_sample_logits"),
                    reason="reference not built here (oracle/_ref)")
@pytest.mark.parametrize("V", [1024, 201088])
@pytest.mark.parametrize("setting", SAMPLER_SETTINGS)
def test_sampler_restatement_matches_reference(V, setting):
    """or_sample against the reference's own sample_logits over a chain of
    draws: same ids, same logits bits afterwards, same history and generator."""
    T, tp, tk, rep = setting
    rng = np.random.default_rng(V + tk)
    so = O.SamplerState(987654321, rng.integers(0, V, 200))
    sr = so.copy()
    for _ in range(8 if V > 4096 else 24):
        lg = (rng.standard_normal(V) * 2.5).astype(np.float32)
        a, la = O.sample(lg, T, tp, tk, rep, so)
        b, lb = O.ref_sample(lg, T, tp, tk, rep, sr)
        assert a == b
        assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
        assert so.rng == sr.rng and so.history == sr.history


def test_mxfp4_dequant_matches_reference_converter():
    """oracle.dequant_mxfp4 (the MXFP4 semantics the device follows) is
    bit-identical to the reference converter's own dequant_mxfp4_fast /
    decode_e8m0 (convert.py:129-213) on the committed vectors: all 16 codes
    (-0 included) and E8M0 bytes from 0 to 254."""
    g = np.load(os.path.join(GOLD, "mxfp4.npz"))
    for tag in "abc":
        blocks, e8, want = g[f"{tag}_blocks"], g[f"{tag}_e8m0"], g[f"{tag}_values"]
        rows, cols = want.shape
        with np.errstate(over="ignore"):
            got = O.dequant_mxfp4(blocks.reshape(rows, -1), e8, rows, cols)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), tag
