"""A few decode steps of a GPT-OSS-120B-shaped model with fewer layers,
without CUDA graphs: the small, repeatable workload the ncu captures under
``profiles/`` run (each kernel launch is then visible on its own).  With
--batch B > 1 every step is one pc_decode_batch over B sequences; with
--prefill N the probe instead encodes N seeded random ids in steps of
--chunk positions (pc_prefill).

    python -m picchio_b200.decode_probe --layers 2 --steps 4
    python -m picchio_b200.decode_probe --layers 2 --steps 2 --batch 64
    python -m picchio_b200.decode_probe --layers 1 --prefill 1024 --chunk 1024
"""
from __future__ import annotations

import argparse


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--context", type=int, default=4096)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--prefill", type=int, default=0)
    ap.add_argument("--chunk", type=int, default=64)
    args = ap.parse_args()
    if args.prefill > 0:
        import numpy as np
        from picchio_b200 import Model, ModelConfig
        cfg = ModelConfig.gpt_oss_120b()
        cfg.n_layers = args.layers
        m = Model.synthetic(cfg, seed=1, ctx=args.prefill + 8, use_graphs=False, kv_bf16=True,
                            prefill_chunk=args.chunk)
        ids = np.random.default_rng(7).integers(0, cfg.vocab, args.prefill).tolist()
        print("ok", m.prefill_tokens(ids, 0))
        return
    from picchio_b200 import Model, ModelConfig
    cfg = ModelConfig.gpt_oss_120b()
    cfg.n_layers = args.layers
    B = args.batch
    m = Model.synthetic(cfg, seed=1, ctx=args.context + args.steps + 8, use_graphs=False, kv_bf16=True,
                        max_batch=B)
    for s in range(B):
        m.kv_fill_synthetic(args.context, seq=s, seed=7 + s)
    if B == 1:
        tok = 1
        for i in range(args.steps):
            tok = m.forward_token(tok, args.context + i)
        print("ok", tok)
    else:
        toks = [(3 * s + 1) % 1000 for s in range(B)]
        for i in range(args.steps):
            toks = m.decode_batch(toks, [args.context + i] * B)
        print("ok", toks[:4])


if __name__ == "__main__":
    main()
