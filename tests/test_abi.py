"""CPU checks of the C ABI: the library loads, exports every entry point that
include/aspida_attn.h declares, and the binding covers exactly those."""
import ctypes
import os
import re

import pytest

from aspida_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "aspida_attn.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(aspida_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "aspida_attn_decode" in syms and "aspida_gpu_fattn_new" in syms


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_binding_matches_header():
    assert sorted(_lib.SIGNATURES) == declared_symbols()


def test_workspace_size_is_host_only_and_monotone():
    lib = _lib.load()
    a = lib.aspida_attn_decode_workspace_size(32, 32, 8, 128, 8192, 512)
    b = lib.aspida_attn_decode_workspace_size(32, 32, 8, 128, 16384, 512)
    c = lib.aspida_attn_decode_workspace_size(64, 32, 8, 128, 8192, 512)
    assert 0 < a <= b and a < c
    assert lib.aspida_attn_decode_workspace_size(0, 32, 8, 128, 8192, 512) == 0


@pytest.mark.gpu
def test_c_program_drives_the_library_like_the_ada_binding(tmp_path):
    """tests/c/abi_decode.c: dlopen + dlsym of the entry points, a KV state
    from the lifecycle calls, one batched decode, checked in C against a
    double-precision CPU loop (no Python in the data path)."""
    import shutil
    import subprocess
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    exe = tmp_path / "abi_decode"
    subprocess.run([gcc, "-O2", "-o", str(exe), os.path.join(ROOT, "tests", "c", "abi_decode.c"),
                    f"-I{cuda}/include", f"-L{cuda}/lib64", "-lcudart", "-ldl", "-lm"],
                   check=True, timeout=120)
    env = dict(os.environ, LD_LIBRARY_PATH=f"{cuda}/lib64:" + os.environ.get("LD_LIBRARY_PATH", ""))
    r = subprocess.run([str(exe), _lib.LIB_PATH], capture_output=True, text=True, timeout=120,
                       env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.startswith("max_abs")
