"""The CPU decoders of the native library (``ops/csrc/cpu_codec.cpp``) under
AddressSanitizer and UndefinedBehaviorSanitizer: a harness feeds them
truncated and corrupted copies of valid rANS and LC streams, each in an
allocation of exactly its size.  Any out-of-bounds access aborts the run."""

import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "kvserve_hpdps_b200", "ops", "csrc")


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_cpu_decoders_survive_corrupt_streams_under_asan(tmp_path):
    exe = str(tmp_path / "fuzz_cpu_codecs")
    build = subprocess.run(
        ["g++", "-O1", "-g", "-std=c++17", "-pthread", "-fsanitize=address,undefined",
         "-fno-sanitize-recover=undefined", "-fno-omit-frame-pointer", "-I", CSRC,
         os.path.join(ROOT, "tests", "native", "fuzz_cpu_codecs.cpp"),
         os.path.join(CSRC, "cpu_codec.cpp"), "-o", exe],
        capture_output=True, text=True, timeout=300)
    if build.returncode != 0 and "asan" in build.stderr.lower():
        pytest.skip("sanitizer runtime not available: " + build.stderr[-200:])
    assert build.returncode == 0, build.stderr[-2000:]
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=0:abort_on_error=1",
               UBSAN_OPTIONS="print_stacktrace=1")
    run = subprocess.run([exe, "3000"], capture_output=True, text=True, timeout=600, env=env)
    assert run.returncode == 0, (run.stdout + run.stderr)[-3000:]
    assert "rans:" in run.stdout and "lc:" in run.stdout


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_threaded_cpu_codecs_are_race_free_under_tsan(tmp_path):
    """The CPU coders run chunks on host threads; ThreadSanitizer checks the
    encoders, the record placement and the decoders for data races."""
    exe = str(tmp_path / "tsan_cpu_codecs")
    build = subprocess.run(
        ["g++", "-O1", "-g", "-std=c++17", "-pthread", "-fsanitize=thread", "-I", CSRC,
         os.path.join(ROOT, "tests", "native", "fuzz_cpu_codecs.cpp"),
         os.path.join(CSRC, "cpu_codec.cpp"), "-o", exe],
        capture_output=True, text=True, timeout=300)
    if build.returncode != 0 and "tsan" in build.stderr.lower():
        pytest.skip("sanitizer runtime not available: " + build.stderr[-200:])
    assert build.returncode == 0, build.stderr[-2000:]
    env = dict(os.environ, TSAN_OPTIONS="halt_on_error=1", KVS_CPU_THREADS="8")
    run = subprocess.run([exe, "200"], capture_output=True, text=True, timeout=600, env=env)
    assert run.returncode == 0 and "WARNING: ThreadSanitizer" not in run.stderr, \
        (run.stdout + run.stderr)[-3000:]
