"""Host code under AddressSanitizer and UndefinedBehaviorSanitizer (no GPU):
the page allocator, the GGUF parser and the byte-level BPE tokenizer, built
from the library's own sources with tests/sanitize/host_fuzz.cpp and run on
seeded random operations and inputs.  Any sanitizer report aborts the driver;
the driver's own checks are the properties listed in its header (a shadow
model of the pager, every parse of a damaged file returning a status, and
decode(encode(text)) == text)."""
import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CSRC = ROOT / "qwenasr.cpp_b200" / "csrc"
SOURCES = [ROOT / "tests" / "sanitize" / "host_fuzz.cpp", CSRC / "pager.cpp", CSRC / "gguf.cpp", CSRC / "bpe.cpp"]

# A small model file (about 0.3 MB) with the full byte-level vocabulary, so a
# fuzz iteration rewrites little.
SMALL = dict(n_layers=1, hidden=64, n_heads=2, n_kv_heads=1, head_dim=128, intermediate=64, vocab=300,
             rope_theta=1.0e6, rms_norm_eps=1.0e-6)


@pytest.fixture(scope="module")
def driver(tmp_path_factory):
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("g++ is not installed")
    out = tmp_path_factory.mktemp("sanitize") / "host_fuzz"
    cmd = [cxx, "-std=c++17", "-O1", "-g", "-fno-omit-frame-pointer", "-fsanitize=address,undefined",
           "-fno-sanitize-recover=all", f"-I{CSRC}", f"-I{ROOT / 'include'}", *map(str, SOURCES), "-o", str(out)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-4000:]
    return out


def run(driver, *args, timeout=300):
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=0", UBSAN_OPTIONS="print_stacktrace=1")
    r = subprocess.run([str(driver), *map(str, args)], capture_output=True, text=True, timeout=timeout, env=env)
    assert r.returncode == 0, (r.stdout + r.stderr)[-6000:]
    return r.stdout


@pytest.fixture(scope="module")
def small_file(synth, tmp_path_factory):
    return synth.write_gguf(tmp_path_factory.mktemp("small") / "small_bytes.gguf", dict(SMALL), seed=0,
                            norm_init="one_plus", tokenizer="bytes")


@pytest.mark.parametrize("seed", [1, 2])
def test_pager_under_sanitizers(driver, seed):
    run(driver, "pager", seed, 4000)


@pytest.mark.parametrize("seed", [1, 2])
def test_gguf_parser_under_sanitizers(driver, small_file, tmp_path, seed):
    out = run(driver, "gguf", small_file, tmp_path / "mutated.gguf", seed, 400)
    assert "mutated files opened" in out


@pytest.mark.parametrize("seed", [1, 2])
def test_tokenizer_under_sanitizers(driver, small_file, seed):
    run(driver, "tokenizer", small_file, seed, 300)
