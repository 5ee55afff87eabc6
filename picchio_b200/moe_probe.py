"""The single-layer expert microbench of BASELINE configs[1] (d_model 2880,
expert FFN 2880, 32 experts, top-4, INT4 gs32) for one row count: the
workload of the expert-GEMM ncu captures under ``profiles/``.

    python -m picchio_b200.moe_probe --rows 512 --iters 3
"""
from __future__ import annotations

import argparse


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=512)
    ap.add_argument("--iters", type=int, default=3)
    args = ap.parse_args()
    import numpy as np
    import torch
    from picchio_b200 import Model, ModelConfig
    cfg = ModelConfig(hidden=2880, n_layers=1, n_heads=64, n_kv_heads=8, head_dim=64, n_experts=32, topk=4,
                      intermediate=2880, vocab=1024)
    M = args.rows
    m = Model.synthetic(cfg, seed=5, ctx=64, max_batch=max(M, 1))
    rng = np.random.default_rng(11)
    sel = np.stack([rng.choice(32, 4, replace=False) for _ in range(M)]).astype(np.int32)
    w = rng.random((M, 4)).astype(np.float32)
    w /= w.sum(1, keepdims=True)
    x = torch.from_numpy(rng.standard_normal((M, cfg.hidden)).astype(np.float32)).cuda()
    s_d, w_d = torch.from_numpy(sel).cuda(), torch.from_numpy(w).cuda()
    for _ in range(args.iters):
        out = m.moe_experts(x, s_d, w_d, 0)
    torch.cuda.synchronize()
    print("ok", float(out.abs().sum()))
    m.close()


if __name__ == "__main__":
    main()
