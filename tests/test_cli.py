"""The decoder harness CLI (qwen-asr-text-decode) speaks the reference tool's
key=value protocol (tools/qwen-asr-text-layer.cpp:487-517) and is driven here
as a subprocess, the way the reference's benchmarks/check_text_*.py drive
its binary.  GPU cases compare against the reference-scalar fixtures."""
import subprocess
from pathlib import Path

import numpy as np
import pytest

from conftest import rel_err

ROOT = Path(__file__).resolve().parents[1]
CLI = ROOT / "qwenasr.cpp_b200" / "bin" / "qwen-asr-text-decode"
GOLDEN = ROOT / "tests" / "golden"


def run(args):
    p = subprocess.run([str(CLI), *map(str, args)], capture_output=True, text=True, timeout=600)
    kv = dict(line.split("=", 1) for line in p.stdout.splitlines() if "=" in line)
    return p.returncode, kv, p.stderr


@pytest.fixture(scope="module")
def case(tiny_files, tmp_path_factory):
    cfg, files = tiny_files
    g = np.load(GOLDEN / "tiny_one_plus.npz")
    d = tmp_path_factory.mktemp("cli")
    inp = d / "input.f32"
    g["x"].astype(np.float32).tofile(inp)
    return files[("f32", "one_plus")], inp, g, d


def test_cli_usage_and_cpu_device_rejected(case):
    path, inp, g, d = case
    rc, kv, err = run([path, inp, "--generate", "2", "--device", "cpu"])
    assert rc == 1 and "GPU only" in err
    rc, kv, err = run([path])
    assert rc == 2


def test_cli_accepts_reference_flags(case):
    """The reference tool's flags parse (the run then stops at the CPU-device
    check, after parsing); bad backend values exit 2 with its messages."""
    path, inp, g, d = case
    rc, kv, err = run([path, inp, "--generate", "2", "--threads", "8", "--backend", "sched", "--audio-backend", "ggml",
                       "--kv-cache", "--language", "English", "--system", "x", "--device", "cpu"])
    assert rc == 1 and "GPU only" in err, err
    assert "--language is ignored" in err and "--system is ignored" in err
    rc, kv, err = run([path, inp, "--backend", "gpu"])
    assert rc == 2 and "--backend requires scalar, ggml, or sched" in err
    rc, kv, err = run([path, inp, "--audio-backend", "x"])
    assert rc == 2 and "--audio-backend requires ggml or sched" in err


@pytest.mark.parametrize("flags,msg", [(["--kv-dtype", "int8"], "--kv-dtype"), (["--weights", "int4"], "--weights"),
                                       (["--page-size", "32"], "16-token pages"), (["--gpu", "x"], "--gpu")])
def test_cli_rejects_bad_b200_options(case, flags, msg):
    """The B200 options are checked before any file or device is touched."""
    path, inp, g, d = case
    rc, kv, err = run([path, inp, "--generate", "2", *flags])
    assert rc == 2 and msg in err, err


@pytest.mark.gpu
def test_cli_generate_matches_reference(case):
    path, inp, g, d = case
    rc, kv, err = run([path, inp, "--generate", "16", "--no-stop"])
    assert rc == 0, err
    assert kv["mode"] == "generate" and kv["prompt_tokens"] == str(g["x"].shape[0])
    assert kv["kv_dtype"] == "f32" and kv["weights"] == "f32" and kv["page_tokens"] == "16"
    assert float(kv["tokens_per_s"]) > 0 and float(kv["decoder_input_ms"]) >= 0   # keys the reference's benches read
    assert [int(t) for t in kv["generated_ids"].split(",")] == g["ref_ids"].tolist()
    rc, kv, err = run([path, inp, "--generate", "16", "--stop-ids", str(int(g["stop_id"]))])
    assert rc == 0 and kv["stopped"] == "true"
    assert [int(t) for t in kv["generated_ids"].split(",")] == g["ref_ids_stop"].tolist()


@pytest.mark.gpu
def test_cli_b200_options(case):
    """--kv-dtype / --weights / --page-size / --gpu reach the backend: an e4m3
    cache with bf16 weights generates the requested count of in-vocabulary
    ids.  (Agreement with the reference's ids at these types is measured by
    the model tests; this tiny model's top-1 margin is too small to pin.)"""
    path, inp, g, d = case
    rc, kv, err = run([path, inp, "--generate", "16", "--no-stop", "--kv-dtype", "fp8", "--weights", "bf16",
                       "--page-size", "16", "--gpu", "0"])
    assert rc == 0, err
    assert kv["kv_dtype"] == "fp8" and kv["weights"] == "bf16"
    ids = [int(t) for t in kv["generated_ids"].split(",")]
    assert len(ids) == 16 and all(0 <= t < int(kv["vocab"]) for t in ids)


@pytest.mark.gpu
def test_cli_prefill_and_layer_outputs(case):
    path, inp, g, d = case
    out = d / "logits.f32"
    rc, kv, err = run([path, inp, "--prefill", "--out", out])
    assert rc == 0, err
    logits = np.fromfile(out, np.float32)
    assert rel_err(logits, g["ref_prefill_logits"]) < 1e-3
    assert int(kv["top_id"]) == int(np.argmax(g["ref_prefill_logits"]))
    # the reference tool's prefill keys (tools/qwen-asr-text-layer.cpp:603-625)
    assert int(kv["tokens"]) == g["x"].shape[0] and int(kv["values"]) == logits.size
    assert float(kv["top_logit"]) == pytest.approx(float(logits.max()), rel=1e-5)
    assert float(kv["min"]) == pytest.approx(float(logits.min()), rel=1e-5)
    assert float(kv["max"]) == pytest.approx(float(logits.max()), rel=1e-5)
    assert float(kv["mean"]) == pytest.approx(float(logits.astype(np.float64).mean()), rel=1e-4, abs=1e-6)
    assert float(kv["decoder_input_ms"]) >= 0 and kv["threads"] == "1"
    out = d / "layer0.f32"
    rc, kv, err = run([path, inp, "--layer", "0", "--out", out, "--threads", "8"])
    assert rc == 0, err
    vals = np.fromfile(out, np.float32).reshape(g["ref_layer0"].shape)
    assert rel_err(vals, g["ref_layer0"]) < 1e-4
    # the reference tool's layer keys (:715-735)
    assert float(kv["text_layer_ms"]) > 0 and int(kv["values"]) == vals.size and kv["threads"] == "8"
    assert float(kv["max"]) == pytest.approx(float(vals.max()), rel=1e-5)


def json_escape(b: bytes) -> bytes:
    """The reference tool's text_json escaping (tools/qwen-asr-text-layer.cpp:66-91)."""
    out = bytearray(b'"')
    for c in b:
        if c == 0x5C:
            out += b"\\\\"
        elif c == 0x22:
            out += b'\\"'
        elif c == 0x0A:
            out += b"\\n"
        elif c == 0x0D:
            out += b"\\r"
        elif c == 0x09:
            out += b"\\t"
        elif c < 0x20:
            out += b"\\u00%02x" % c
        else:
            out.append(c)
    return bytes(out + b'"')


@pytest.mark.gpu
def test_cli_generate_prints_text(case, synth, pkg, tmp_path):
    """With a tokenizer in the model file, --generate also prints text_json
    (the detokenised ids, special tokens skipped) and writes the text to
    --out, as the reference tool does (:478-517).  Same tensors as the golden
    model, so the ids are the reference's."""
    _, inp, g, _ = case
    model = synth.write_gguf(tmp_path / "bytes.gguf", dict(synth.TINY), seed=0, weights="f32", norm_init="one_plus",
                             tokenizer="bytes")
    out = tmp_path / "text.bin"
    p = subprocess.run([str(CLI), str(model), str(inp), "--generate", "16", "--no-stop", "--out", str(out)],
                       capture_output=True, timeout=600)
    assert p.returncode == 0, p.stderr
    kv = dict(line.split(b"=", 1) for line in p.stdout.splitlines() if b"=" in line)
    ids = [int(t) for t in kv[b"generated_ids"].split(b",")]
    assert ids == g["ref_ids"].tolist()
    text = pkg.Tokenizer(model).decode(ids, True)
    assert out.read_bytes() == text
    assert kv[b"text_json"] == json_escape(text)
