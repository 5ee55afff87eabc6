"""The C-ABI library without a GPU: it loads, exports every entry point the
header declares, and fails with a status (never a crash) when no device is
present."""
import ctypes as C
import os
import re
import subprocess

import pytest

from tests.conftest import HAS_GPU

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "picchio_b200.h")


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(pc_[a-z0-9_]+)\s*\(", src)))


def test_library_builds_and_exports_every_declared_symbol():
    from picchio_b200 import build
    lib_path = build.build(verbose=False)
    out = subprocess.run(["nm", "-D", "--defined-only", lib_path], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (pc_[a-z0-9_]+)\b", out))
    names = declared()
    assert len(names) >= 20
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    L = C.CDLL(lib_path)
    for n in names:
        assert hasattr(L, n)


def test_struct_layouts_match_the_header(tmp_path):
    """The ctypes mirrors of pc_opts, pc_model_cfg and pc_sampling have the
    sizes a C compiler gives the header's structs (a field added on one side
    only would make the library write past the Python struct)."""
    from picchio_b200.api import _Cfg, _Opts, _Sampling
    src = tmp_path / "sz.c"
    src.write_text('#include <stdio.h>\n#include "picchio_b200.h"\nint main(void) { printf("%zu %zu %zu\\n", '
                   "sizeof(pc_opts), sizeof(pc_model_cfg), sizeof(pc_sampling)); return 0; }\n")
    exe = tmp_path / "sz"
    subprocess.run(["gcc", "-I" + os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    sizes = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    assert sizes == [C.sizeof(_Opts), C.sizeof(_Cfg), C.sizeof(_Sampling)]


def test_status_strings_and_defaults_without_gpu():
    from picchio_b200.api import lib, _Opts
    L = lib()
    assert L.pc_status_string(0) == b"PC_OK"
    assert L.pc_status_string(8) == b"PC_ERR_TIMEOUT"
    o = _Opts()
    L.pc_default_opts(C.byref(o))
    assert o.ctx_len == 512 and o.max_batch == 1 and o.use_graphs == 1 and o.kv_bf16 == 0


@pytest.mark.skipif(HAS_GPU, reason="checks the no-device error path")
def test_init_without_device_returns_status(tmp_path):
    from picchio_b200 import Model, PicchioError
    from picchio_b200.synth import make_model
    make_model(str(tmp_path))
    with pytest.raises(PicchioError) as ei:
        Model(str(tmp_path))
    assert ei.value.status_name in ("PC_ERR_CUDA", "PC_ERR_OOM")


def test_missing_model_dir_is_an_error_not_a_crash():
    from picchio_b200 import Model, PicchioError
    with pytest.raises(PicchioError):
        Model("/nonexistent/model/dir")
