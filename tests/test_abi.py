"""CPU: libmoe_cuda.so loads and exports every entry point that
include/moe_cuda.h declares (no compute call: there may be no GPU)."""
import ctypes
import os
import re
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    src = open(os.path.join(ROOT, "include", "moe_cuda.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(moe_[a-z0-9_A-Z]+)\s*\(", src)))


def test_header_has_no_torch_types():
    src = open(os.path.join(ROOT, "include", "moe_cuda.h")).read()
    for bad in ("torch", "at::", "Tensor", "c10", "std::"):
        assert bad not in src


def test_every_declared_symbol_is_exported(cuda_lib):
    from flash_deepseek_b200 import _lib
    lib = ctypes.CDLL(_lib.LIB_PATH)
    names = declared()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python mirror binds every one of them
    assert sorted(_lib.SIGNATURES) == names


def test_create_rejects_bad_config(cuda_lib):
    from flash_deepseek_b200 import _lib, MoeConfig
    lib = _lib.load()
    bad = MoeConfig(hidden=7000).c()   # not a multiple of 256
    assert not lib.moe_create(ctypes.byref(bad), 0, 0, 1, None)
    bad = MoeConfig(top_k=17).c()
    assert not lib.moe_create(ctypes.byref(bad), 0, 0, 1, None)


def test_nccl_then_torch_import_in_one_process():
    """The library dlopens NCCL on first use; a later `import torch` in the
    same process must still find the NCCL it was built against."""
    code = ("import flash_deepseek_b200 as F\n"
            "assert len(F.get_unique_id()) == 128\n"
            "import torch\n"
            "print('ok')\n")
    env = {k: v for k, v in os.environ.items() if k != "MOE_NCCL_LIB"}
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr[-2000:]
