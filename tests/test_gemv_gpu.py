"""Device matmul_qt (the streaming dequant GEMV) against the oracle.

Dequantized weights must be bit-exact: (nibble-8)*scale in fp32, or q*scale
for INT8 (picchio.c:680-682, 1488-1491).  GEMV outputs are fp32 sums in a
different order than the reference's AVX2 lanes; the tolerance is a relative
L2 error of 2e-6 per output vector (measured errors are ~1e-7), well inside
the 1e-2 hidden-state bar of the parity spec.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from picchio_b200.synth import quantize_int4, quantize_int8, quantize_mxfp4

GOLD = os.path.join(os.path.dirname(__file__), "golden")
REL_L2 = 2e-6

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


# (40, 6000, 32): from 3 input rows the B operand of a long row and the weight
# rings no longer fit one CTA's shared memory; the product runs as jobs of two rows.
SHAPES = [(64, 256, 32), (48, 2880, 32), (5760, 2880, 32), (2880, 2880, 64), (40, 320, 64),
          (33, 100, 32), (17, 96, 16), (16, 768, 0), (29, 131, 0), (40, 6000, 32)]


@pytest.mark.parametrize("shape", SHAPES)
def test_int4_dequant_bit_exact_and_matmul(shape):
    import torch
    from picchio_b200 import QT, FMT_INT4
    Oo, I, gs = shape
    rng = np.random.default_rng(Oo * 31 + I)
    w = (rng.standard_normal((Oo, I)) * 0.02).astype(np.float32)
    pk, sc = quantize_int4(w, gs)
    q = QT(FMT_INT4, Oo, I, pk, sc, block_size=gs)
    dq = q.dequant().cpu().numpy()
    ref = O.dequant_i4(pk, sc, Oo, I, gs)
    assert np.array_equal(bits(dq), bits(ref))
    for S in (1, 3, 4, 5, 8, 13):
        x = rng.standard_normal((S, I)).astype(np.float32)
        y = q.matmul(torch.from_numpy(x).cuda()).cpu().numpy()
        yr = O.matmul_i4_gs(x, pk, sc, Oo, I, gs) if gs else O.matmul_i4(x, pk, sc, Oo, I)
        for s in range(S):
            assert rel_l2(y[s], yr[s]) < REL_L2, (S, s, rel_l2(y[s], yr[s]))


@pytest.mark.parametrize("shape", [(64, 256), (512, 2880), (2880, 4096), (1024, 256), (21, 70)])
def test_int8_dequant_bit_exact_and_matmul(shape):
    import torch
    from picchio_b200 import QT, FMT_INT8
    Oo, I = shape
    rng = np.random.default_rng(Oo + 7 * I)
    w = (rng.standard_normal((Oo, I)) * 0.02).astype(np.float32)
    q8, s8 = quantize_int8(w)
    q = QT(FMT_INT8, Oo, I, q8, s8)
    assert np.array_equal(bits(q.dequant().cpu().numpy()), bits(O.dequant_i8(q8, s8, Oo, I)))
    for S in (1, 4, 7, 8, 9):
        x = rng.standard_normal((S, I)).astype(np.float32)
        y = q.matmul(torch.from_numpy(x).cuda()).cpu().numpy()
        yr = O.matmul_q8(x, q8, s8, Oo, I)
        for s in range(S):
            assert rel_l2(y[s], yr[s]) < REL_L2


@pytest.mark.parametrize("shape", [(64, 256), (5760, 2880), (2880, 2880), (33, 96), (17, 160)])
def test_mxfp4_dequant_bit_exact_and_matmul(shape):
    """The reference's fmt 3 (MXFP4) natively: dequantized values bit-equal
    to convert.py's FP4_LUT[code] * 2^(e - 127) (-0.0 included), products
    against the reference's fp32 matmul (matmul_f32) of those values."""
    import torch
    from picchio_b200 import QT, FMT_MXFP4
    Oo, I = shape
    rng = np.random.default_rng(Oo * 13 + I)
    w = (rng.standard_normal((Oo, I)) * 0.02).astype(np.float32)
    blk, e8 = quantize_mxfp4(w)
    pk = blk.reshape(Oo, I // 2)
    sc = np.ldexp(np.ones((Oo, I // 32), np.float32), e8.astype(np.int32) - 127).astype(np.float32)
    q = QT(FMT_MXFP4, Oo, I, pk, sc, block_size=32)
    ref = O.dequant_mxfp4(pk, e8, Oo, I)
    assert np.array_equal(bits(q.dequant().cpu().numpy()), bits(ref))
    for S in (1, 3, 4, 5, 8, 13):
        x = rng.standard_normal((S, I)).astype(np.float32)
        y = q.matmul(torch.from_numpy(x).cuda()).cpu().numpy()
        yr = O.matmul_f32(x, ref, Oo, I)
        for s in range(S):
            assert rel_l2(y[s], yr[s]) < REL_L2, (S, s, rel_l2(y[s], yr[s]))


def test_mxfp4_dequant_matches_reference_converter():
    """Device MXFP4 tiles dequantize to exactly the values the reference
    converter's own code computes (tests/golden/mxfp4.npz, from
    convert.py:129-213): every code, E8M0 bytes 0..254."""
    from picchio_b200 import QT, FMT_MXFP4
    g = np.load(os.path.join(GOLD, "mxfp4.npz"))
    for tag in "abc":
        blocks, e8, want = g[f"{tag}_blocks"], g[f"{tag}_e8m0"], g[f"{tag}_values"]
        rows, cols = want.shape
        sc = np.ldexp(np.ones(e8.shape, np.float32), e8.astype(np.int32) - 127).astype(np.float32)
        q = QT(FMT_MXFP4, rows, cols, blocks.reshape(rows, -1), sc, block_size=32)
        assert np.array_equal(bits(q.dequant().cpu().numpy()), bits(want)), tag


def test_f32_matmul():
    import torch
    from picchio_b200 import QT, FMT_F32
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((96, 200)) * 0.02).astype(np.float32)
    q = QT(FMT_F32, 96, 200, w)
    x = rng.standard_normal((3, 200)).astype(np.float32)
    y = q.matmul(torch.from_numpy(x).cuda()).cpu().numpy()
    yr = O.matmul_f32(x, w, 96, 200)
    assert rel_l2(y, yr) < REL_L2


def test_against_reference_golden_outputs():
    import torch
    from picchio_b200 import QT, FMT_INT4, FMT_INT8
    g = np.load(os.path.join(GOLD, "kernels.npz"))
    for tag in "abcd":
        Oo, I, gs, S = [int(v) for v in g[f"i4_{tag}_shape"]]
        x = torch.from_numpy(g[f"i4_{tag}_x"]).cuda()
        y = QT(FMT_INT4, Oo, I, g[f"i4_{tag}_q"], g[f"i4_{tag}_s"], block_size=gs).matmul(x).cpu().numpy()
        assert rel_l2(y, g[f"i4_{tag}_y"]) < REL_L2
        y8 = QT(FMT_INT8, Oo, I, g[f"i8_{tag}_q"], g[f"i8_{tag}_s"]).matmul(x).cpu().numpy()
        assert rel_l2(y8, g[f"i8_{tag}_y"]) < REL_L2


def test_extreme_activation_scales():
    # rows of very different magnitude: the per-row power-of-two prescale
    # keeps the f16 hi/lo split exact to ~2^-22 for each row
    import torch
    from picchio_b200 import QT, FMT_INT4
    rng = np.random.default_rng(11)
    w = (rng.standard_normal((128, 512)) * 0.02).astype(np.float32)
    pk, sc = quantize_int4(w, 32)
    q = QT(FMT_INT4, 128, 512, pk, sc, block_size=32)
    x = rng.standard_normal((4, 512)).astype(np.float32)
    x[0] *= 1e-6
    x[1] *= 1e5
    x[2, :256] = 0.0
    x[3] = 0.0
    y = q.matmul(torch.from_numpy(x).cuda()).cpu().numpy()
    yr = O.matmul_i4_gs(x, pk, sc, 128, 512, 32)
    for s in range(3):
        assert rel_l2(y[s], yr[s]) < REL_L2
    assert np.all(y[3] == 0.0)
