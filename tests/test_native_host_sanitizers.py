"""Host-side native code under ThreadSanitizer and AddressSanitizer/UBSan, on
CPU: the two-tier allocator (harp_b200/csrc/alloc.cpp) built against a host
stand-in for the CUDA runtime calls it makes (tests/native/fake_cuda) and
driven by tests/native/alloc_stress.cpp (eight allocating threads plus one that
changes caps, reads statistics and empties the host cache; event-gated reuse
of freed host blocks; cap failures)."""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SRC = [os.path.join(HERE, "native", "alloc_stress.cpp"), os.path.join(ROOT, "harp_b200", "csrc", "alloc.cpp")]


@pytest.mark.parametrize("san", ["thread", "address,undefined"])
def test_allocator_under_sanitizer(tmp_path, san):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("no g++")
    exe = str(tmp_path / "alloc_stress")
    flags = [f"-fsanitize={san}", "-g", "-O1", "-pthread", "-std=c++17",
             "-I" + os.path.join(HERE, "native", "fake_cuda")]
    if "undefined" in san:
        flags.append("-fno-sanitize-recover=undefined")
    build = subprocess.run([gxx, *flags, *SRC, "-o", exe], capture_output=True, text=True, timeout=300)
    if build.returncode != 0 and "sanitizer" in (build.stderr or "").lower():
        pytest.skip(f"this toolchain cannot build with -fsanitize={san}")
    assert build.returncode == 0, build.stderr[-3000:]
    env = dict(os.environ, TSAN_OPTIONS="halt_on_error=1", ASAN_OPTIONS="detect_leaks=0")
    run = subprocess.run([exe], capture_output=True, text=True, timeout=600, env=env)
    out = run.stdout + run.stderr
    assert run.returncode == 0, out[-4000:]
    assert "WARNING: ThreadSanitizer" not in out and "ERROR: AddressSanitizer" not in out, out[-4000:]
    assert "alloc_stress: 0 failures" in out
