"""The C++ host layer (include/inl_engine.hpp, im-not-llm_b200/host/): built
with g++ and run on the CPU.

* tests/cpp/test_engine.cpp: planning, BatchDeadline (timeout, then wedged),
  the error variants and the three engines over a test-double Backend.
* tests/cpp/test_checkpoint.cpp: the shard list of a sharded checkpoint's index.
* tests/cpp/backend_link.cpp: the CUDA backend links against libinl_cuda.so
  and a model load that cannot succeed here raises an InlError (no crash)."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HOST = ROOT / "im-not-llm_b200" / "host"
GXX = shutil.which("g++")
FLAGS = ["-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror", "-pthread", f"-I{ROOT / 'include'}"]

pytestmark = pytest.mark.skipif(GXX is None, reason="g++ not found")


def _run(cmd, **kw):
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, **kw)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout


def test_host_layer_with_a_test_backend(tmp_path):
    exe = tmp_path / "test_engine"
    _run([GXX, *FLAGS, str(HOST / "engine.cpp"), str(ROOT / "tests" / "cpp" / "test_engine.cpp"), "-o", str(exe)])
    assert "all passed" in _run([str(exe)])


def test_sharded_checkpoint_resolution(tmp_path):
    """csrc/checkpoint.h: the files a model load reads for a .safetensors
    path or a model.safetensors.index.json (crates/inl-core/src/hub.rs:324-353)."""
    exe = tmp_path / "test_checkpoint"
    _run([GXX, *FLAGS, f"-I{ROOT / 'im-not-llm_b200' / 'csrc'}", str(ROOT / "tests" / "cpp" / "test_checkpoint.cpp"),
          "-o", str(exe)])
    assert "all passed" in _run([str(exe), str(tmp_path)])


def test_cuda_backend_links_and_a_failed_load_is_an_inl_error(tmp_path):
    import torch

    from im_not_llm_b200 import _native

    lib = _native.LIB_PATH
    if not lib.exists():
        pytest.skip("libinl_cuda.so not built")
    exe = tmp_path / "backend_link"
    _run([GXX, *FLAGS, str(HOST / "engine.cpp"), str(HOST / "cuda_backend.cpp"),
          str(ROOT / "tests" / "cpp" / "backend_link.cpp"), f"-L{lib.parent}", "-linl_cuda",
          f"-Wl,-rpath,{lib.parent}", "-o", str(exe)])
    out = _run([str(exe)]).strip()
    code, _, message = out.partition("|")
    if not torch.cuda.is_available():
        assert code == "config" and message.startswith("config error: model load:"), out
    else:  # the checkpoint path does not exist
        assert code in ("config", "inference"), out


def test_host_layer_under_address_and_undefined_behaviour_sanitizers(tmp_path):
    """The same host tests built with -fsanitize=address,undefined: no memory
    error or undefined behaviour in the planners, the deadline's detached
    workers, the engines or the shard list."""
    exe = tmp_path / "test_engine_asan"
    flags = [f for f in FLAGS if f != "-O1"] + ["-O1", "-g", "-fsanitize=address,undefined", "-fno-omit-frame-pointer",
                                                "-fno-sanitize-recover=all"]
    probe = subprocess.run([GXX, *flags, "-x", "c++", "-", "-o", str(tmp_path / "probe")], input="int main(){}",
                           capture_output=True, text=True, timeout=120)
    if probe.returncode != 0:
        pytest.skip("g++ has no sanitizer runtime here")
    _run([GXX, *flags, str(HOST / "engine.cpp"), str(ROOT / "tests" / "cpp" / "test_engine.cpp"), "-o", str(exe)])
    assert "all passed" in _run([str(exe)])
    chk = tmp_path / "test_checkpoint_asan"
    _run([GXX, *flags, f"-I{ROOT / 'im-not-llm_b200' / 'csrc'}", str(ROOT / "tests" / "cpp" / "test_checkpoint.cpp"),
          "-o", str(chk)])
    assert "all passed" in _run([str(chk), str(tmp_path)])


def test_host_layer_under_thread_sanitizer(tmp_path):
    """The engine tests under -fsanitize=thread: the gate, the load lock and
    the deadline's worker hand-off are free of data races."""
    flags = [f for f in FLAGS if f != "-O1"] + ["-O1", "-g", "-fsanitize=thread"]
    probe = subprocess.run([GXX, *flags, "-x", "c++", "-", "-o", str(tmp_path / "probe")], input="int main(){}",
                           capture_output=True, text=True, timeout=120)
    if probe.returncode != 0:
        pytest.skip("g++ has no thread sanitizer runtime here")
    exe = tmp_path / "test_engine_tsan"
    _run([GXX, *flags, str(HOST / "engine.cpp"), str(ROOT / "tests" / "cpp" / "test_engine.cpp"), "-o", str(exe)])
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "all passed" in r.stdout and "WARNING: ThreadSanitizer" not in r.stderr, r.stderr
