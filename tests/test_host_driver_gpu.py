"""The C host driver (picchio_b200/picchio-gpu) against the reference binary's
own stdout, byte for byte.

tests/golden/service_tiny.json holds a SERVICE=1 session script and the
transcript the unmodified reference printed for it on the tiny seeded model
(service_loop, picchio.c:2700-2795: READY, TURN with prefix reuse and
per-turn sampling, TOKEN, DONE MAX_TOKENS / CONTEXT_FULL, ERROR BAD_RANGE /
BAD_TOKEN, RESET, SHUTDOWN), and the stdout of a one-shot OUTPUT=ids run
from INPUT_FILE (picchio.c:3096-3287).  The same environment is given to the
driver here.
"""
import json
import os
import subprocess

import pytest

from picchio_b200.synth import SynthConfig, make_model

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = os.path.join(os.path.dirname(__file__), "golden")
DRIVER = os.path.join(ROOT, "picchio_b200", "picchio-gpu")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def golden(tmp_path_factory):
    with open(os.path.join(GOLD, "service_tiny.json")) as f:
        g = json.load(f)
    d = str(tmp_path_factory.mktemp("tiny_service"))
    make_model(d, SynthConfig(), g["seed"])
    if not os.path.exists(DRIVER):
        from picchio_b200 import build
        build.build()
    return g, d


def _run(env, d, stdin=None):
    e = dict(os.environ, MODEL=d, **env)
    r = subprocess.run([DRIVER], env=e, input=stdin, capture_output=True, text=True, cwd=d, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    return r.stdout


def test_service_transcript_matches_reference(golden):
    g, d = golden
    out = _run(dict(SERVICE="1", **g["service_env"]), d, g["script"])
    assert out == g["service_stdout"]


def test_output_ids_matches_reference(golden):
    g, d = golden
    pf = os.path.join(d, "prompt.txt")
    with open(pf, "w") as f:
        f.write(" ".join(map(str, g["prompt"])))
    out = _run(dict(INPUT_FILE=pf, **g["ids_env"]), d)
    assert out == g["ids_stdout"]
