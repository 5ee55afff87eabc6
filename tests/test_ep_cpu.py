"""Expert parallelism, host side, on CPU with gloo ranks.

The device path shards the experts of every layer over the ranks with the
rule used by ``pc_init`` (model.cu): rank r of n holds experts
[E*r/n, E*(r+1)/n).  Attention, router and lm_head are replicated, so every
rank holds every token's hidden row and routes identically: the dispatch
side of the MoE all-to-all needs no transfer.  After the down projection a
rank holds the output rows of its own (token, k) pairs; the combine exchange
sends exactly those rows to every other rank (ep_push writes them into the
other GPUs' receive buffers), each rank knowing from the shared routing
which rows arrive from whom.  The weighted combine then runs in k order, as
moe_forward does (picchio.c:1445-1454), so the result is bit-identical to
one process.

These tests run that exchange with the oracle's expert arithmetic on gloo
ranks (point-to-point sends of the owned rows only) and require the
single-process moe_forward's bits.  They also cover a rank that fails before
the exchange: the others must get an error from the process group's timeout
instead of waiting forever.
"""
import datetime
import os
import socket
import tempfile

import numpy as np
import pytest

from oracle import oracle as O
from picchio_b200.synth import SynthConfig, make_model


def expert_range(E, rank, size):
    return E * rank // size, E * (rank + 1) // size


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_expert_ranges_partition():
    for E in (8, 32, 128):
        for n in (1, 2, 3, 4, 8):
            owned = []
            for r in range(n):
                lo, hi = expert_range(E, r, n)
                assert 0 <= lo <= hi <= E
                owned.extend(range(lo, hi))
            assert owned == list(range(E))


def _moe_rank(rank, world, port, model_dir, xs, out_path, fail_rank):
    import torch
    import torch.distributed as dist
    # a short timeout only where a rank is meant to fail: a healthy world of
    # four ranks on a loaded CPU can drift apart by more than a few seconds
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5 if fail_rank >= 0 else 120))
    try:
        if rank == fail_rank:
            raise SystemExit(3)  # leaves before the exchange; the others must not hang
        m = O.OracleModel(model_dir)
        c = m.c
        lo, hi = expert_range(c.n_experts, rank, world)
        outs = []
        for x in xs:
            for l in range(c.n_layers):
                ly = m.layers[l]
                _, sel, wts = O.router_topk(x, ly["router"], ly["router_bias"], c.topk, bias_first=False)
                ranges = [expert_range(c.n_experts, q, world) for q in range(world)]
                owner = [next(q for q, (a, b) in enumerate(ranges) if a <= int(e) < b) for e in sel]
                eo = np.full((c.topk, c.hidden), np.nan, np.float32)
                for k, e in enumerate(sel):
                    if lo <= int(e) < hi:
                        gu, dn, gub, db = m.expert(l, int(e))
                        g = (gu.matmul(x)[0] + gub).astype(np.float32)
                        act = O.swiglu(g, c.swiglu_limit, c.swiglu_alpha)
                        eo[k] = (dn.matmul(act)[0] + db).astype(np.float32)
                # combine exchange: my rows to every other rank, theirs to me
                reqs, recv = [], {}
                for k in range(c.topk):
                    if owner[k] == rank:
                        for q in range(world):
                            if q != rank:
                                reqs.append(dist.isend(torch.from_numpy(eo[k].copy()), q, tag=k))
                    else:
                        recv[k] = torch.empty(c.hidden, dtype=torch.float32)
                        reqs.append(dist.irecv(recv[k], owner[k], tag=k))
                for rq in reqs:
                    rq.wait()
                for k, t in recv.items():
                    eo[k] = t.numpy()
                assert not np.isnan(eo).any()
                out = np.zeros(c.hidden, np.float32)
                for k in range(c.topk):
                    w = np.float32(np.float32(wts[k]) * c.routed_scale)
                    O.lib().or_axpy(O._ptr(out, O._fp), O._ptr(np.ascontiguousarray(eo[k]), O._fp), w, c.hidden)
                outs.append(out)
        if rank == 0:
            np.save(out_path, np.stack(outs))
    finally:
        dist.destroy_process_group()


def _run(world, fail_rank=-1):
    import torch.multiprocessing as mp
    tmp = tempfile.mkdtemp()
    cfg = SynthConfig()
    make_model(tmp, cfg, seed=77)
    rng = np.random.default_rng(5)
    xs = [rng.standard_normal(cfg.hidden_size).astype(np.float32) for _ in range(3)]
    out_path = os.path.join(tmp, "ep_out.npy")
    mp.start_processes(_moe_rank, args=(world, free_port(), tmp, xs, out_path, fail_rank), nprocs=world,
                       join=True, start_method="spawn")
    return tmp, xs, np.load(out_path)


@pytest.mark.parametrize("world", [2, 4])
def test_ep_combine_exchange_is_exact(world):
    tmp, xs, got = _run(world)
    m = O.OracleModel(tmp)
    ref = []
    for x in xs:
        for l in range(m.c.n_layers):
            ref.append(m.moe(x, l))
    ref = np.stack(ref)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_ep_rank_failure_is_reported():
    import torch.multiprocessing as mp
    with pytest.raises((mp.ProcessExitedException, mp.ProcessRaisedException)):
        _run(2, fail_rank=1)
