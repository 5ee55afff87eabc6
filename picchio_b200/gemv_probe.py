"""Times ``matmul_qt`` (pc_qt_matmul) on one seeded random matrix and prints
the achieved HBM rate; also the workload of the large-matrix ncu capture
under ``profiles/``.

    python -m picchio_b200.gemv_probe --rows 368640 --cols 2880 --gs 32 --S 1 --iters 20
"""
from __future__ import annotations

import argparse

import numpy as np


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=368640)
    ap.add_argument("--cols", type=int, default=2880)
    ap.add_argument("--gs", type=int, default=32, help="INT4 group size; 0 = per-row scale")
    ap.add_argument("--int8", action="store_true")
    ap.add_argument("--S", type=int, default=1, help="input rows")
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    import torch
    from picchio_b200 import FMT_INT4, FMT_INT8, QT
    O, I = args.rows, args.cols
    rng = np.random.default_rng(7)
    if args.int8:
        data = rng.integers(-127, 128, size=(O, I), dtype=np.int8)
        scales = np.full(O, 1e-3, np.float32)
        q = QT(FMT_INT8, O, I, data, scales)
        nbytes = O * I + 4 * O
    else:
        data = rng.integers(0, 256, size=(O, (I + 1) // 2), dtype=np.uint8)
        ng = (I + args.gs - 1) // args.gs if args.gs else 1
        scales = np.full(O * ng, 1e-3, np.float32)
        q = QT(FMT_INT4, O, I, data, scales, block_size=args.gs)
        nbytes = O * ((I + 1) // 2) + 4 * O * ng
    x = torch.from_numpy(rng.standard_normal((args.S, I)).astype(np.float32)).cuda()
    for _ in range(3):
        q.matmul(x)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.iters):
        q.matmul(x)
    b.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1e3 / args.iters
    print(f"rows={O} cols={I} {'int8' if args.int8 else f'int4 gs{args.gs}'} S={args.S}: "
          f"{us:.2f} us/launch, {nbytes / us / 1e3:.0f} GB/s (weight + scale bytes)")


if __name__ == "__main__":
    main()
