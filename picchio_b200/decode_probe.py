"""A few bs1 decode steps of a GPT-OSS-120B-shaped model with fewer layers,
without CUDA graphs: the small, repeatable workload the ncu captures under
``profiles/`` run (each kernel launch is then visible on its own).

    python -m picchio_b200.decode_probe --layers 2 --steps 4
"""
from __future__ import annotations

import argparse


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--context", type=int, default=4096)
    args = ap.parse_args()
    from picchio_b200 import Model, ModelConfig
    cfg = ModelConfig.gpt_oss_120b()
    cfg.n_layers = args.layers
    m = Model.synthetic(cfg, seed=1, ctx=args.context + args.steps + 8, use_graphs=False)
    m.kv_fill_synthetic(args.context)
    tok = 1
    for i in range(args.steps):
        tok = m.forward_token(tok, args.context + i)
    print("ok", tok)


if __name__ == "__main__":
    main()
