"""The C-ABI library loads on a CPU-only host and exports every symbol the
public headers declare; without a GPU every entry point fails cleanly with a
config error instead of crashing."""
import ctypes
import json
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
LIB = ROOT / "im-not-llm_b200" / "libinl_cuda.so"


def _declared():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        names |= set(re.findall(r"\b(inl_cuda_[a-z0-9_]+)\s*\(", h.read_text()))
    return names


@pytest.fixture(scope="module")
def lib():
    if not LIB.exists():
        import importlib.util

        spec = importlib.util.spec_from_file_location("_b", ROOT / "im-not-llm_b200" / "build.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()
    from im_not_llm_b200 import _native

    return _native.lib()


def test_every_declared_symbol_is_exported(lib):
    declared = _declared()
    assert len(declared) >= 15
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing
    from im_not_llm_b200 import _native

    assert set(_native.EXPORTED) == declared


def test_version_and_device_count(lib):
    assert b"sm_100a" in lib.inl_cuda_version()
    assert lib.inl_cuda_device_count() >= 0


def test_create_without_gpu_is_a_config_error(lib):
    import torch

    if torch.cuda.is_available():
        pytest.skip("GPU present")
    from im_not_llm_b200 import ConfigError, CudaModel, synthetic

    with pytest.raises(ConfigError):
        CudaModel(synthetic.QWEN3_TINY, {}, dtype="bf16")


def test_bad_config_and_null_arguments(lib):
    from im_not_llm_b200 import _native

    h = ctypes.c_void_p()
    assert lib.inl_cuda_model_create(None, b"x", 0, 1, ctypes.byref(h)) == 1
    assert lib.inl_cuda_model_create(b"{}", b"x", 0, 7, ctypes.byref(h)) == 1
    assert lib.inl_cuda_model_info(None, None) == 1
    assert "NULL" in _native.last_error()
    lib.inl_cuda_model_destroy(None)  # no-op
    assert lib.inl_cuda_forward_dense(None, None, 0, None, 0, 0, None, 0) == 1


def test_errors_map_to_reference_codes():
    from im_not_llm_b200.errors import error_for_status

    assert [error_for_status(s, "m").code for s in (1, 2, 3, 4)] == ["config", "inference", "timeout",
                                                                        "invalid_input"]
    assert str(error_for_status(3, "x")) == "inference timeout: x"


def test_header_compiles_as_c(tmp_path):
    import shutil
    import subprocess

    if not shutil.which("gcc"):
        pytest.skip("no gcc")
    src = tmp_path / "t.c"
    src.write_text('#include "inl_cuda.h"\n#include "inl_cuda_kernels.h"\nint main(void){return 0;}\n')
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", f"-I{ROOT / 'include'}", "-c", str(src), "-o",
                        str(tmp_path / "t.o")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
