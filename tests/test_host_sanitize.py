"""Host code under AddressSanitizer and UndefinedBehaviorSanitizer (no GPU):
the page allocator, the GGUF parser and the byte-level BPE tokenizer, built
from the library's own sources with tests/sanitize/host_fuzz.cpp and run on
seeded random operations and inputs.  Any sanitizer report aborts the driver;
the driver's own checks are the properties listed in its header (a shadow
model of the pager, every parse of a damaged file returning a status, and
decode(encode(text)) == text), and the CPU oracle itself."""
import os
import shutil
import subprocess
import sys
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


ORACLE_PROBE = r"""
import sys
from pathlib import Path
import numpy as np
sys.path.insert(0, sys.argv[1])
from oracle import oracle as ck
ck.ORACLE_SO = Path(sys.argv[2])            # the instrumented build
import __graft_entry__ as ge
s = ge.load_synth()
cfg = dict(s.TINY)
t = s.read_gguf(s.write_gguf(Path(sys.argv[3]), cfg, seed=0, norm_init="one_plus"))
rng = np.random.default_rng(0)
r = ck.OracleModel(cfg, t).generate(rng.standard_normal((37, cfg["hidden"])).astype(np.float32), 12, want_logits=True)
assert len(r["ids"]) == 12
rc, rows = ck.decoder_input(np.array([5, 7, 9, 9, 3], np.int32), np.array(t["text.token_embd.weight"]),
                            rng.standard_normal((2, cfg["hidden"])).astype(np.float32), 9)
assert rc == 0 and rows.shape == (5, cfg["hidden"])
L, n = 2, 3
caps = [40, 17, 70]
kc = [rng.standard_normal((L, c, 1024)).astype(np.float32) for c in caps]
vc = [rng.standard_normal((L, c, 1024)).astype(np.float32) for c in caps]
lens = np.array([15, 16, 64], np.int32)
ck.kv_step_batch(rng.standard_normal((L, n, 4096)).astype(np.float32), np.ones((L, 128), np.float32),
                 np.ones((L, 128), np.float32), kc, vc, lens, threads=2)
assert lens.tolist() == [16, 17, 65]
assert ck._lib._name == sys.argv[2]
print("oracle ok")
"""


def test_oracle_under_sanitizers(tmp_path):
    """The checker itself (oracle/qkv_oracle.c) under ASan/UBSan: the cached
    greedy loop with logits, the decoder-input splice and the batched KV step
    (page-boundary lengths 15/16/64) on the tiny model."""
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc is not installed")
    so = tmp_path / "libqkv_oracle_san.so"
    r = subprocess.run([gcc, "-O1", "-g", "-fPIC", "-ffp-contract=off", "-fno-fast-math", "-std=c11",
                        "-fsanitize=address,undefined", "-fno-sanitize-recover=all", "-fopenmp", "-shared", "-o",
                        str(so), str(ROOT / "oracle" / "qkv_oracle.c"), "-lm"], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    runtimes = [subprocess.run([gcc, f"-print-file-name={lib}"], capture_output=True, text=True).stdout.strip()
                for lib in ("libasan.so", "libubsan.so")]
    env = dict(os.environ, LD_PRELOAD=" ".join(runtimes), ASAN_OPTIONS="detect_leaks=0",
               UBSAN_OPTIONS="print_stacktrace=1")
    p = subprocess.run([sys.executable, "-c", ORACLE_PROBE, str(ROOT), str(so), str(tmp_path / "tiny.gguf")],
                       capture_output=True, text=True, timeout=600, env=env)
    assert p.returncode == 0 and "oracle ok" in p.stdout, (p.stdout + p.stderr)[-6000:]
