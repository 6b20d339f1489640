"""The C-ABI library loads on a machine without a GPU, exports every symbol
include/qkv.h declares, and reports a clean error (no crash) where a device
is needed."""
import ctypes as C
import re
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / "include" / "qkv.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(qkv_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported(pkg):
    syms = declared_symbols()
    assert len(syms) >= 30
    raw = C.CDLL(str(pkg.LIB_PATH))
    missing = [s for s in syms if not hasattr(raw, s)]
    assert not missing, missing
    assert set(syms) <= set(pkg.SIGNATURES), sorted(set(syms) - set(pkg.SIGNATURES))


def test_status_codes_agree_with_header(pkg):
    """The Python status names are the header's enum, value for value."""
    text = (ROOT / "include" / "qkv.h").read_text()
    body = re.search(r"enum qkv_status \{(.*?)\};", text, flags=re.S).group(1)
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    header = {int(v): k for k, v in re.findall(r"(QKV_[A-Z_]+)\s*=\s*(\d+)", body)}
    assert header == pkg.STATUS
    assert header[pkg.QKV_ERR_CAPACITY] == "QKV_ERR_CAPACITY"


def test_create_without_device_fails_cleanly(pkg, tiny_files):
    import torch
    if torch.cuda.is_available():
        return
    cfg, files = tiny_files
    rt = pkg.runtime_config(device=0)
    try:
        pkg.Decoder.from_gguf(files[("f32", "normal")], rt)
        raise AssertionError("expected an error without a GPU")
    except pkg.QkvError as e:
        assert e.code in (4, 9)


def test_create_rejects_bad_geometry(pkg, tiny_files):
    cfg, files = tiny_files
    bad = dict(cfg, n_kv_heads=4)
    rt = pkg.runtime_config(device=0)
    try:
        pkg.Decoder.from_gguf(files[("f32", "normal")], rt, cfg=bad)
        raise AssertionError("expected QKV_ERR_INVALID_ARG")
    except pkg.QkvError as e:
        assert e.code == 1


def test_kv_only_rejects_bad_page_size(pkg, synth):
    rt = pkg.runtime_config(device=0)
    rt.page_tokens = 32
    qn = np.ones((2, 128), np.float32)
    try:
        pkg.Decoder.kv_only(dict(synth.TINY), rt, qn, qn)
        raise AssertionError("expected QKV_ERR_INVALID_ARG")
    except pkg.QkvError as e:
        assert e.code == 1
