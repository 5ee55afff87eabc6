"""pc_qt_matmul_noalloc against pc_qt_matmul (collected last on purpose: it
must pass alone and after every other test, whose state it shares).

Both run the same GEMV on the same job table, so the outputs must be equal
bit for bit, on two calls in a row (the second reuses the scratch the first
one wrote).  Row counts above PC_QT_NOALLOC_MAX_ROWS are rejected.
"""
import numpy as np
import pytest

from picchio_b200.synth import quantize_int4, quantize_int8

pytestmark = pytest.mark.gpu

MAX_ROWS = 64


def _qts():
    from picchio_b200 import FMT_INT4, FMT_INT8, QT
    rng = np.random.default_rng(11)
    out = []
    for O, I, gs in ((96, 320, 32), (48, 2880, 64), (33, 100, 0)):
        w = (rng.standard_normal((O, I)) * 0.02).astype(np.float32)
        pk, sc = quantize_int4(w, gs)
        out.append(QT(FMT_INT4, O, I, pk, sc, block_size=gs))
    w = (rng.standard_normal((64, 288)) * 0.02).astype(np.float32)
    q8, s8 = quantize_int8(w)
    out.append(QT(FMT_INT8, 64, 288, q8, s8))
    return out


def test_noalloc_equals_matmul_twice():
    import torch
    rng = np.random.default_rng(3)
    for q in _qts():
        for S in (1, 5, 8, 13, MAX_ROWS):
            x = torch.from_numpy(rng.standard_normal((S, q.I)).astype(np.float32)).cuda()
            ref = q.matmul(x)
            a = q.matmul_noalloc(x)
            b = q.matmul_noalloc(x)
            q.check()  # no device-side failure recorded by either call
            torch.cuda.synchronize()
            assert torch.equal(a.view(torch.int32), ref.view(torch.int32)), (q.O, q.I, S)
            assert torch.equal(b.view(torch.int32), ref.view(torch.int32)), (q.O, q.I, S)


def test_noalloc_rejects_too_many_rows():
    import torch
    from picchio_b200.api import PicchioError
    q = _qts()[0]
    x = torch.zeros((MAX_ROWS + 1, q.I), dtype=torch.float32, device="cuda")
    with pytest.raises(PicchioError, match="PC_ERR_RANGE"):
        q.matmul_noalloc(x)
