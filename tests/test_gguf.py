"""GGUF: the synthetic writer produces files the third-party `gguf` reader and
the native reader agree on; the native reader passes the reference loader's
known-answer checks (tools/qwen-asr-weights.cpp:97-143 exact floats,
native-model.cpp:299-330 names/shapes) and rejects damaged files."""
import struct

import numpy as np
import pytest


def test_known_answer_tensor(pkg, tmp_path):
    gguf = pytest.importorskip("gguf")
    p = tmp_path / "kat.gguf"
    w = gguf.GGUFWriter(str(p), "qwen3-asr")
    w.add_tensor("kat.weight", np.array([1.25, -2.5, 3.75, 4.5], np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    dims, ty, data = pkg.gguf_tensor(p, "kat.weight")
    assert dims == [4] and ty == 0
    assert data.view(np.float32).tolist() == [1.25, -2.5, 3.75, 4.5]


def test_writer_matches_third_party_reader(pkg, synth, tiny_files):
    gguf = pytest.importorskip("gguf")
    cfg, files = tiny_files
    path = files[("f32", "normal")]
    r = gguf.GGUFReader(str(path))
    mine = synth.read_gguf(path)
    names = [t.name for t in r.tensors]
    assert names == [n for n, _, _ in synth.tensor_specs(synth.ModelConfig.of(cfg))]
    for t in r.tensors:
        a = np.asarray(t.data).reshape(mine[t.name].shape)
        assert np.array_equal(a, mine[t.name])
        dims, ty, data = pkg.gguf_tensor(path, t.name)
        assert dims == [int(d) for d in t.shape] and ty == 0
        assert np.array_equal(data.view(np.float32).reshape(mine[t.name].shape), mine[t.name])
    f = r.fields
    assert int(f["qwen3-asr.text.hidden_size"].parts[-1][0]) == cfg["hidden"]


def test_fp8_projection_file(pkg, synth, tmp_path):
    """FP8 projection files: each projection an I8 tensor of e4m3 codes plus an
    f32 "<name>.scale" per row; the native reader sees both, the codes
    dequantise (code x row scale) to within e4m3's precision of the
    bf16-rounded values the same seed writes, and everything else is as in
    the f32 file."""
    cfg = dict(synth.TINY)
    p8 = synth.write_gguf(tmp_path / "fp8.gguf", cfg, seed=0, storage="fp8", tokenizer=False)
    pb = synth.write_gguf(tmp_path / "bf.gguf", cfg, seed=0, weights="bf16", tokenizer=False)
    dims, ty, codes = pkg.gguf_tensor(p8, "text.blk.1.ffn_down.weight")
    assert ty == 24 and dims == [cfg["intermediate"], cfg["hidden"]] and codes.nbytes == cfg["hidden"] * cfg["intermediate"]
    dims, ty, sc = pkg.gguf_tensor(p8, "text.blk.1.ffn_down.weight.scale")
    assert ty == 0 and dims == [cfg["hidden"]]
    a, b = synth.read_gguf(p8), synth.read_gguf(pb)
    assert set(a) == set(b)
    for name in b:
        if name.endswith(synth.PROJECTION_SUFFIXES):
            rows_max = np.abs(b[name]).max(axis=1, keepdims=True)
            assert np.all(np.abs(a[name] - b[name]) <= rows_max * 2.0 ** -4 + 1e-12), name
        else:
            assert np.array_equal(a[name], b[name]), name


def test_read_config(pkg, tiny_files):
    cfg, files = tiny_files
    got = pkg.read_gguf_config(files[("bf16", "one_plus")])
    for k in ("n_layers", "hidden", "n_heads", "n_kv_heads", "head_dim", "intermediate", "vocab"):
        assert got[k] == cfg[k]
    assert got["rope_theta"] == pytest.approx(cfg["rope_theta"])


def test_expected_tensor_set(synth):
    """612 tensors for 0.6B with the audio tower (native-model.cpp:299-330); the text part is 3 + 11 per layer."""
    specs = synth.tensor_specs(synth.ModelConfig.of(synth.QWEN3_ASR_0_6B))
    assert len(specs) == 3 + 11 * 28
    shapes = dict((n, s) for n, s, _ in specs)
    assert shapes["text.blk.0.attn_q.weight"] == (2048, 1024)      # GGML ne {1024, 2048}
    assert shapes["text.blk.27.ffn_down.weight"] == (1024, 3072)
    assert shapes["text.output.weight"] == (151936, 1024)


def test_bf16_rounding_is_rne(synth):
    a = np.array([1.0, 1.00390625, 1.005859375, -3.14159, 65504.0], np.float32)
    r = synth.bf16_round(a)
    # ties-to-even: 1 + 2^-8 is halfway between 1 and 1 + 2^-7 -> 1.0
    assert r[0] == 1.0 and r[1] == 1.0 and r[2] == np.float32(1.0078125)
    assert (r.view(np.uint32) & 0xFFFF).max() == 0


@pytest.mark.parametrize("damage", ["magic", "truncated", "offset", "version"])
def test_reader_rejects_damaged_files(pkg, tiny_files, tmp_path, damage):
    cfg, files = tiny_files
    data = bytearray(files[("f32", "normal")].read_bytes())
    if damage == "magic":
        data[0:4] = b"GGUX"
    elif damage == "truncated":
        data = data[: len(data) // 2]
    elif damage == "version":
        data[4:8] = struct.pack("<I", 9)
    else:
        # point the first tensor's offset far beyond the end of the file
        r = __import__("gguf").GGUFReader(str(files[("f32", "normal")]))
        off = r.tensors[0].field.offset
        field = r.tensors[0].field
        # the offset is the last part of the tensor-info field
        pos = off + sum(p.nbytes for p in field.parts[:-1])
        data[pos:pos + 8] = struct.pack("<Q", 1 << 40)
    p = tmp_path / f"bad_{damage}.gguf"
    p.write_bytes(bytes(data))
    with pytest.raises(pkg.QkvError) as ei:
        pkg.gguf_tensor(p, "text.token_embd.weight")
    assert ei.value.code in (6, 7)


def test_bf16_typed_file(pkg, synth, tmp_path):
    """A file whose tensors are stored as GGML bf16 (type 30): the library's
    reader (range checks of gguf-model.cpp:110-162) returns, per tensor, the
    upper 16 bits of the f32 file of the same bf16-rounded values."""
    a = synth.write_gguf(tmp_path / "f32.gguf", dict(synth.TINY), seed=0, weights="bf16", norm_init="one_plus",
                         tokenizer=False)
    b = synth.write_gguf(tmp_path / "bf16.gguf", dict(synth.TINY), seed=0, norm_init="one_plus", tokenizer=False,
                         storage="bf16")
    ta = synth.read_gguf(a)
    for name in ("text.token_embd.weight", "text.blk.1.ffn_down.weight", "text.blk.0.attn_q_norm.weight"):
        dims, ty, data = pkg.gguf_tensor(b, name)
        assert ty == 30 and dims == list(reversed(ta[name].shape))
        want = (np.ascontiguousarray(ta[name]).view(np.uint32) >> np.uint32(16)).astype(np.uint16)
        assert np.array_equal(data.view(np.uint16).reshape(want.shape), want)


def _string_array_file(path, count: int, payload: bytes):
    """A GGUF v3 file with no tensors and one key: tokenizer.ggml.tokens, a
    string array that claims `count` entries followed by `payload`."""
    key = b"tokenizer.ggml.tokens"
    head = b"GGUF" + struct.pack("<IQQ", 3, 0, 1)
    kv = struct.pack("<Q", len(key)) + key + struct.pack("<IIQ", 9, 8, count)
    path.write_bytes(head + kv + payload)
    return path


@pytest.mark.parametrize("case", ["huge_count", "count_past_end", "string_past_end"])
def test_reader_bounds_string_array_counts(pkg, tmp_path, case):
    """A string-array count larger than the rest of the file can hold (every
    entry takes at least its 8-byte length) is a format error found before
    any table is sized from it; a count that fits but whose strings run past
    the end is one too.  Neither may surface as an exception or an
    allocation of the claimed size."""
    entry = struct.pack("<Q", 2) + b"ab"
    if case == "string_past_end":
        count, payload = 2, entry + struct.pack("<Q", 100) + b"ab"    # the second string claims 100 bytes
    else:
        count, payload = (1 << 40) if case == "huge_count" else 3, entry * 2   # 2 entries present, 20 bytes
    p = _string_array_file(tmp_path / "strs.gguf", count, payload)
    with pytest.raises(pkg.QkvError) as ei:
        pkg.Tokenizer(p)
    assert ei.value.code == 7, ei.value
    assert "tokenizer.ggml.tokens" in str(ei.value)


def test_reader_accepts_exact_string_array(pkg, tmp_path):
    """The same file with the count it holds parses; the tokenizer then
    reports the missing merges key, which shows that the array was read."""
    entry = struct.pack("<Q", 2) + b"ab"
    p = _string_array_file(tmp_path / "strs.gguf", 2, entry * 2)
    with pytest.raises(pkg.QkvError) as ei:
        pkg.Tokenizer(p)
    assert ei.value.code == 7
    assert "incomplete" in str(ei.value)
