"""Expert parallelism on two GPUs (skipped with fewer): one process per GPU,
the experts of every layer split between the ranks, the combine exchange
written into the other GPU's memory over NVLink (ep_push, kernels.cu).

Every rank must produce the single-GPU ids: greedy decode of the tiny seeded
model (equal to the CPU oracle's), a batched decode step, and a 300-id prompt
in one step, whose 600 routed pairs run the tcgen05 expert GEMMs.  A rank
that stops calling must make the other's next step fail with a timeout from
the bounded wait, not hang it.
"""
import multiprocessing as mp
import tempfile

import pytest

pytestmark = pytest.mark.gpu

PROMPT_LEN, STEPS, LONG = 16, 12, 300


def _two_gpus():
    try:
        import torch
        return torch.cuda.device_count() >= 2
    except Exception:
        return False


def _inputs():
    from picchio_b200.synth import random_prompt
    prompt = random_prompt(PROMPT_LEN, 1024, seed=7)
    long_prompt = random_prompt(LONG, 1024, seed=8)
    toks = [(5 * b + 3) % 1024 for b in range(8)]
    return prompt, long_prompt, toks


def _run(m, prompt, long_prompt, toks):
    ids = m.generate(prompt, STEPS)
    long_next = m.prefill_tokens(long_prompt, 0)
    batch = m.decode_batch(toks, [LONG + b for b in range(8)])
    return ids, long_next, batch


def _rank_main(rank, world, nid, model_dir, q, stall, done):
    """One rank.  stall = None: the three workloads; stall = this rank: it
    never steps and stays alive (its memory mapped by the other rank) until
    the other rank is done; otherwise: one step, expected to time out."""
    try:
        import torch
        torch.cuda.set_device(rank)
        from picchio_b200 import Model, PicchioError
        prompt, long_prompt, toks = _inputs()
        with Model(model_dir, ctx=512, device=rank, ep_rank=rank, ep_size=world, nccl_id=nid, max_batch=8,
                   prefill_chunk=LONG) as m:
            if stall is None:
                q.put((rank, _run(m, prompt, long_prompt, toks)))
            elif rank == stall:
                q.put((rank, "idle"))
                done.wait(120)
            else:
                try:
                    m.forward_token(1, 0)
                    q.put((rank, "no error"))
                except PicchioError as e:
                    q.put((rank, f"error {e}"))
                done.set()
    except Exception as e:  # reported to the parent, never a hang
        q.put((rank, f"exception {type(e).__name__}: {e}"))
        done.set()


def _launch(model_dir, stall=None, timeout=240):
    from picchio_b200 import nccl_unique_id
    ctx = mp.get_context("spawn")
    q, done = ctx.Queue(), ctx.Event()
    nid = nccl_unique_id()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, nid, model_dir, q, stall, done)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(2):
            r, v = q.get(timeout=timeout)
            out[r] = v
    finally:
        done.set()
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return out


@pytest.fixture(scope="module")
def model_dir():
    from picchio_b200.synth import SynthConfig, make_model
    with tempfile.TemporaryDirectory() as d:
        make_model(d, SynthConfig(), seed=1234)
        yield d


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
def test_two_rank_decode_matches_one_gpu(model_dir):
    out = _launch(model_dir)
    for r in (0, 1):
        assert not isinstance(out[r], str), out[r]
    from oracle import oracle as O
    from picchio_b200 import Model
    prompt, long_prompt, toks = _inputs()
    with Model(model_dir, ctx=512, device=0, max_batch=8, prefill_chunk=LONG) as m:
        want = _run(m, prompt, long_prompt, toks)
    assert want[0] == O.OracleModel(model_dir, ctx=512).generate(prompt, STEPS)
    for r in (0, 1):
        assert tuple(out[r]) == tuple(want), (r, out[r], want)


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
def test_stalled_rank_times_out(model_dir):
    out = _launch(model_dir, stall=1)
    assert out[1] == "idle"
    assert out[0].startswith("error") and "TIMEOUT" in out[0], out[0]
