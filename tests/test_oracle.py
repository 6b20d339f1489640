"""The CPU oracle (oracle/qkv_oracle.c) is pinned to the reference's own code:
bit-exact against fixtures from the reference's scalar C++ path (oracle/_ref),
and within float32 tolerance of the reference's PyTorch restatement."""
from pathlib import Path

import numpy as np
import pytest

from conftest import rel_err

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module", params=["normal", "one_plus"])
def case(request, synth, checker, tmp_path_factory):
    import hashlib
    norm = request.param
    g = np.load(GOLDEN / f"tiny_{norm}.npz")
    cfg = dict(synth.TINY)
    path = synth.write_gguf(tmp_path_factory.mktemp("o") / "m.gguf", cfg, seed=0, norm_init=norm)
    tensors = synth.read_gguf(path)
    h = hashlib.sha256()
    for name in sorted(tensors):
        h.update(name.encode())
        h.update(np.ascontiguousarray(tensors[name]).tobytes())
    assert h.hexdigest() == str(g["weights_sha256"]), "synthetic weight generator drifted from the fixtures"
    return cfg, path, tensors, g, checker.OracleModel(cfg, tensors)


def test_prefill_logits_bit_exact(case):
    cfg, path, tensors, g, om = case
    assert np.array_equal(om.prefill_logits(g["x"]), g["ref_prefill_logits"])


def test_layer0_bit_exact(case):
    cfg, path, tensors, g, om = case
    out, k, v = om.layer_prefill(0, g["x"])
    assert np.array_equal(out, g["ref_layer0"])


def test_cached_greedy_ids(case):
    cfg, path, tensors, g, om = case
    r = om.generate(g["x"], 16)
    assert r["ids"].tolist() == g["ref_ids"].tolist()
    assert r["stopped"] == bool(g["ref_stopped"])


def test_stop_id_semantics(case):
    """Generation includes the stop id and stops right after it (text-decoder.cpp:2150-2161)."""
    cfg, path, tensors, g, om = case
    r = om.generate(g["x"], 16, stop_ids=[int(g["stop_id"])])
    assert r["ids"].tolist() == g["ref_ids_stop"].tolist()
    assert r["stopped"] and bool(g["ref_stopped_stop"])


def test_torch_restatement_agrees(case):
    cfg, path, tensors, g, om = case
    out, _, _ = om.layer_prefill(0, g["x"])
    assert rel_err(out, g["torch_layer0"]) < 1e-5
    assert rel_err(om.prefill_logits(g["x"]), g["torch_prefill_logits"]) < 1e-4
    assert om.generate(g["x"], 8)["ids"].tolist() == g["torch_ids"].tolist()


def test_teacher_forced_matches_free_run(case):
    cfg, path, tensors, g, om = case
    free = om.generate(g["x"], 10, want_logits=True)
    am, logits = om.generate_forced(g["x"], free["ids"][:-1], 10)
    assert am.tolist() == free["ids"].tolist()
    assert np.array_equal(logits, free["logits"])


def test_cache_contents_are_post_rope_k_and_raw_v(case, checker):
    """The cached K is post QK-norm + RoPE and V is raw (text-decoder.cpp:771-776, 1026-1027):
    re-deriving row t of layer 0 from its projections gives the cached rows."""
    cfg, path, tensors, g, om = case
    x = g["x"]
    r = om.generate(x, 3, want_cache=True)
    t = 7
    p = "text.blk.0."
    xn = x[t] / np.sqrt(np.mean(x[t].astype(np.float64) ** 2) + cfg["rms_norm_eps"]) * tensors[p + "attn_norm.weight"]
    raw = np.concatenate([tensors[p + "attn_q.weight"] @ xn, tensors[p + "attn_k.weight"] @ xn,
                          tensors[p + "attn_v.weight"] @ xn]).astype(np.float32)
    q, k, v = checker.append_qkv(raw, tensors[p + "attn_q_norm.weight"], tensors[p + "attn_k_norm.weight"], t)
    np.testing.assert_allclose(r["k"][0, t], k, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(r["v"][0, t], v, rtol=1e-4, atol=1e-5)


def test_reference_scalar_live(case, checker):
    """When the reference tree is present, the live reference agrees with the oracle too."""
    if not checker.ref_available():
        pytest.skip("oracle/_ref not built (reference sources absent)")
    cfg, path, tensors, g, om = case
    ref = checker.RefModel(path, cfg)
    rng = np.random.default_rng(3)
    x = rng.standard_normal((9, cfg["hidden"]), dtype=np.float32)
    assert np.array_equal(ref.prefill_logits(x), om.prefill_logits(x))
    ids, _ = ref.generate_cached(x, 5)
    assert ids.tolist() == om.generate(x, 5)["ids"].tolist()


def test_rope_table_formula(checker):
    """Host RoPE table formula: double angle, float cos/sin (text-decoder.cpp:610-616)."""
    import math
    for pos, i in [(0, 0), (1, 0), (17, 5), (4095, 63), (333, 31)]:
        c, s = checker.rope_cos_sin(pos, i)
        inv = math.exp(-math.log(1.0e6) * (2 * i) / 128.0)
        assert c == np.float32(math.cos(pos * inv)) and s == np.float32(math.sin(pos * inv))


# ---- decoder input (src/decoder-input.cpp:64-98) ----

def _digest(a):
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(a, np.float32).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def dec_input(synth, tmp_path_factory):
    """The decoder-input fixture (the reference's own assembly, see
    tests/golden/make_decoder_input_golden.py) with the tiny model's table."""
    g = np.load(GOLDEN / "decoder_input.npz")
    path = synth.write_gguf(tmp_path_factory.mktemp("di") / "m.gguf", dict(synth.TINY), seed=0, weights="f32",
                            norm_init="one_plus", tokenizer="bytes")
    embd = np.array(synth.read_gguf(path)["text.token_embd.weight"])
    assert _digest(embd) == str(g["embd_sha256"]), "synthetic weight generator drifted from the fixture"
    return g, embd, path


def test_decoder_input_bit_exact(dec_input, checker):
    g, embd, _ = dec_input
    aid = int(g["audio_token_id"])
    for k in range(3):
        rc, rows = checker.decoder_input(g[f"ids_{k}"], embd, g[f"audio_{k}"], aid)
        assert rc == 0
        assert _digest(rows) == str(g[f"rows_sha256_{k}"])
    rc, rows = checker.decoder_input(g["ids_0"], embd, g["audio_0"], aid)
    assert np.array_equal(rows, g["rows_0"])


def test_decoder_input_error_order(dec_input, checker):
    """The reference's checks in its order: 1 id outside the table, 2 more
    placeholders than audio rows (seen while scanning), 3 a count that differs
    at the end.  (The reference reports 2 as "prompt has more audio
    placeholders ..." and 3 as "audio placeholder count does not match ...",
    the two messages the fixture recorded from its own failures.)"""
    g, embd, _ = dec_input
    aid = int(g["audio_token_id"])
    ids, audio = g["ids_0"], g["audio_0"]
    assert checker.decoder_input(ids, embd, audio[:4], aid)[0] == 2
    assert checker.decoder_input(ids, embd, np.concatenate([audio, audio[:1]]), aid)[0] == 3
    bad = ids.copy()
    bad[1] = embd.shape[0]
    assert checker.decoder_input(bad, embd, audio, aid)[0] == 1
    bad[1] = -1
    assert checker.decoder_input(bad, embd, audio, aid)[0] == 1
    # an out-of-range id after a surplus placeholder: the placeholder is seen first
    extra = np.concatenate([ids[:1], [aid] * 6, [embd.shape[0]]]).astype(np.int32)
    assert checker.decoder_input(extra, embd, audio, aid)[0] == 2
    assert "more audio placeholders" in str(g["error_0"])
    assert "count does not match" in str(g["error_1"])


def test_decoder_input_reference_live(dec_input, checker):
    """With the reference tree built here (oracle/_ref), its assembly still
    gives the fixture."""
    if not checker.ref_available():
        pytest.skip("oracle/_ref not built")
    g, _, path = dec_input
    for k in range(3):
        rc, ids, rows, msg = checker.ref_decoder_input(str(path), g[f"audio_{k}"], int(g["audio_token_id"]),
                                                       str(g[f"system_{k}"]), str(g[f"language_{k}"]))
        assert rc == 0, msg
        assert np.array_equal(ids, g[f"ids_{k}"])
        assert _digest(rows) == str(g[f"rows_sha256_{k}"])


# ---- detokenisation (src/tokenizer.cpp:482-527) ----

def test_detokenize_matches_reference_known_answers(pkg, dec_input):
    """qkv_tokenizer_decode against the bytes the reference's own
    qwenasr_tokenizer_decode gave (fixture), with and without skipping the
    special tokens: prompt ids, out-of-range and negative ids, every id."""
    g, _, path = dec_input
    tok = pkg.Tokenizer(path)
    for k in range(3):
        ids = g[f"detok_ids_{k}"]
        for skip in (0, 1):
            assert tok.decode(ids, bool(skip)) == g[f"detok_bytes_{k}_{skip}"].tobytes()
    tok.close()


def test_detokenize_reference_live(pkg, dec_input, checker):
    if not checker.ref_available():
        pytest.skip("oracle/_ref not built")
    _, _, path = dec_input
    tok = pkg.Tokenizer(path)
    rng = np.random.default_rng(7)
    for _ in range(20):
        ids = rng.integers(-3, 1003, size=int(rng.integers(0, 300))).astype(np.int32)
        for skip in (False, True):
            assert tok.decode(ids, skip) == checker.ref_tokenizer_decode(str(path), ids, skip)


def test_detokenize_malformed_vocabulary_reference_live(pkg, dec_input, checker, tmp_path):
    """Vocabulary entries that are not byte-symbol strings (invalid UTF-8,
    a sequence cut off by the token's end), patched into a copy of the model
    file in place of filler tokens of the same length: decoding them matches
    the reference's own decoder, which reads a cut-off sequence on into the
    token's zero terminator.  Cut-offs are one byte short, the case where
    that read is defined."""
    if not checker.ref_available():
        pytest.skip("oracle/_ref not built")
    _, _, path = dec_input
    data = bytearray(Path(path).read_bytes())
    patches = {900: b"abcde\xc3", 901: b"abcd\xe4\xb8", 902: b"\xf0\x9f\x98xyz", 903: b"\xff\x80ab\xc2\xa0",
               904: b"\xc4\x80abc\xc3", 905: b"\xe4\xb8\xadxy\xce"}
    for tid, new in patches.items():
        old = f"<t{tid}>".encode()
        assert len(new) == len(old) and data.count(old) == 1
        data[data.index(old):data.index(old) + len(old)] = new
    bad = tmp_path / "malformed_vocab.gguf"
    bad.write_bytes(bytes(data))
    tok = pkg.Tokenizer(bad)
    ids = np.array([900, 901, 902, 903, 904, 905, 97, 900, 259, 905], np.int32)
    for skip in (False, True):
        want = checker.ref_tokenizer_decode(str(bad), ids, skip)
        assert tok.decode(ids, skip) == want
        assert tok.decode(ids[:1], skip) == b"abcde\xc3\x00"   # the terminator's zero byte, as the reference


def test_special_list_edge_cases_reference_live(pkg, synth, checker, tmp_path):
    """Special-token keys whose token strings repeat an earlier key's, or are
    empty: the reference lists a special only once and never an empty one,
    and decode skips only listed ids.  A tokenizer-only file (no tensors)
    written with the gguf package's writer; ids and bytes match the
    reference's own encoder and decoder."""
    if not checker.ref_available():
        pytest.skip("oracle/_ref not built")
    gguf = pytest.importorskip("gguf")
    tokens = synth.byte_symbols() + ["<|endoftext|>", "<|im_start|>", "<|im_end|>", "<|audio_start|>",
                                     "<|audio_end|>", "<|audio_pad|>", "<asr_text>", "<|im_end|>", "", "ab"]
    keys = {"endoftext": 256, "im_start": 257, "im_end": 258, "audio_start": 259,
            "audio_end": 263,        # the same string as im_end, under a later key
            "audio": 261, "asr_text": 264}   # an empty token
    p = tmp_path / "specials.gguf"
    w = gguf.GGUFWriter(str(p), "qwen3-asr")
    w.add_array("tokenizer.ggml.tokens", tokens)
    w.add_array("tokenizer.ggml.merges", ["a b"])
    w.add_uint32("tokenizer.ggml.eos_token_id", 258)
    for k, v in keys.items():
        w.add_uint32(f"qwen3-asr.token.{k}_token_id", v)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    tok = pkg.Tokenizer(p)
    ids = np.array([258, 263, 264, 97, 262, 265, 256, 260], np.int32)
    for skip in (False, True):
        assert tok.decode(ids, skip) == checker.ref_tokenizer_decode(str(p), ids, skip), skip
    assert tok.decode(np.array([263, 264], np.int32), True) == b"<|im_end|>"   # 263 is not listed, 264 is empty
    for text in (b"x<|im_end|>y", b"<asr_text>ab<|audio_pad|>", b"ab ab", b"<|audio_end|>"):
        for eos in (False, True):
            assert tok.encode(text, eos).tolist() == checker.ref_tokenizer_encode(str(p), text, eos).tolist(), text


def test_asr_prompt_ids_reference_live(pkg, dec_input, checker):
    """qkv_asr_prompt_ids against the ids the reference's own decoder-input
    assembly builds (qwenasr_build_asr_prompt + qwenasr_tokenizer_encode,
    reached through qwenasr_decoder_input_from_audio) for random system
    texts (special-token strings inside them included), languages and
    audio counts."""
    if not checker.ref_available():
        pytest.skip("oracle/_ref not built")
    g, embd, path = dec_input
    tok = pkg.Tokenizer(path)
    aid = int(g["audio_token_id"])
    rng = np.random.default_rng(31)
    pieces = ["You", " are", " a", " helpful", " assistant", ".", "\n", "  ", "'s", "42", "é", "中文", "<|im_end|>",
              "<|im_start|>", "<asr_text>", "language", " ", "\t", "!"]
    languages = ["", "English", "Chinese", "日本語", "x<asr_text>", " German", "fr-FR"]
    for _ in range(40):
        system = "".join(rng.choice(pieces, size=int(rng.integers(0, 12))))
        language = str(rng.choice(languages))
        n_audio = int(rng.integers(0, 40))
        rc, ref_ids, _, msg = checker.ref_decoder_input(str(path), np.zeros((n_audio, embd.shape[1]), np.float32), aid,
                                                       system, language)
        assert rc == 0, msg
        assert tok.asr_prompt_ids(n_audio, system, language).tolist() == ref_ids.tolist(), (system, language)


def test_tokenizer_open_errors(pkg, synth, tmp_path):
    p = synth.write_gguf(tmp_path / "none.gguf", dict(synth.TINY), seed=0, tokenizer=False)
    with pytest.raises(pkg.QkvError) as ei:
        pkg.Tokenizer(p)
    assert "incomplete" in str(ei.value)


# ---- tokenizer encode and the ASR prompt (src/tokenizer.cpp:438-480, 529-549) ----

def test_asr_prompt_ids_match_reference(pkg, dec_input):
    """qkv_asr_prompt_ids gives the ids the reference's own template +
    encoder gave for the fixture's prompts (system text, language, audio
    placeholders; the synthetic tokenizer has a learned merge table)."""
    g, _, path = dec_input
    tok = pkg.Tokenizer(path)
    a = [5, 37, 130]
    for k in range(3):
        ids = tok.asr_prompt_ids(a[k], str(g[f"system_{k}"]), str(g[f"language_{k}"]))
        assert ids.tolist() == g[f"ids_{k}"].tolist()


def test_encode_reference_live(pkg, dec_input, checker):
    if not checker.ref_available():
        pytest.skip("oracle/_ref not built")
    _, _, path = dec_input
    tok = pkg.Tokenizer(path)
    rng = np.random.default_rng(11)
    pieces = ["the", " quick", "isn't", "'LL", " 3.14", "\n\n", "  ", "\t", "Grüße", "日本", "<|im_end|>",
              "<|audio_pad|>", "<asr_text>", "!?", "speech", " We're", "\r\n", "x", "2024", " ", "é"]
    for _ in range(40):
        text = "".join(rng.choice(pieces, size=int(rng.integers(0, 30))))
        for eos in (False, True):
            assert tok.encode(text, eos).tolist() == checker.ref_tokenizer_encode(str(path), text, eos).tolist()


def test_tokenizer_capi_contract(pkg, dec_input):
    """QKV_ERR_CAPACITY with the needed count when the output is too small,
    then success with that count; bad arguments are refused; add_eos appends
    the file's end-of-sequence id."""
    import ctypes as C
    _, _, path = dec_input
    tok = pkg.Tokenizer(path)
    lib = pkg.lib
    text = b"You transcribe speech."
    ids = np.zeros(2, np.int32)
    n = C.c_size_t(0)
    i32 = C.POINTER(C.c_int32)
    rc = lib.qkv_tokenizer_encode(tok.h, text, len(text), 0, ids.ctypes.data_as(i32), 2, C.byref(n))
    assert rc == pkg.QKV_ERR_CAPACITY and n.value > 2
    big = np.zeros(n.value, np.int32)
    rc = lib.qkv_tokenizer_encode(tok.h, text, len(text), 0, big.ctypes.data_as(i32), n.value, C.byref(n))
    assert rc == 0 and big.tolist() == tok.encode(text).tolist()
    eos = tok.encode(text, add_eos=True)
    assert eos[:-1].tolist() == big.tolist() and eos[-1] == 258   # im_end, the synthetic file's eos id
    out = C.create_string_buffer(1)
    rc = lib.qkv_tokenizer_decode(tok.h, big.ctypes.data_as(i32), len(big), 1, out, 1, C.byref(n))
    assert rc == pkg.QKV_ERR_CAPACITY and n.value == len(tok.decode(big))
    assert lib.qkv_tokenizer_encode(None, text, len(text), 0, big.ctypes.data_as(i32), 8, C.byref(n)) == 1
    assert lib.qkv_asr_prompt_ids(tok.h, 2, b"", b"", None, 0, None) == 1
    tok.close()


def test_encode_reference_live_bytes(pkg, dec_input, checker):
    """Byte strings at the edges of the pre-tokeniser's classes, against the
    reference's own encoder: other whitespace (VT, FF, NBSP, ideographic
    space), non-ASCII digits and letters, invalid UTF-8 (lone continuation
    bytes, truncated sequences, 0xFF), contractions in other cases and
    fragments of the special tokens.

    A sequence cut off at the end of a segment (the text's end, or just
    before a special token) makes the reference read past the segment: one
    missing byte reads its string terminator, a zero byte, which ends up in
    the ids; two or three missing bytes read memory after the terminator,
    whose contents are not defined.  So every truncated piece here is short
    by one byte at most, whatever follows it."""
    if not checker.ref_available():
        pytest.skip("oracle/_ref not built")
    _, _, path = dec_input
    tok = pkg.Tokenizer(path)
    rng = np.random.default_rng(23)
    pieces = [b"a", b"Z", b" ", b"   ", b"\t", b"\x0b", b"\x0c", b"\n", b"\r", b"\r\n\n", b"\xc2\xa0", b"\xe3\x80\x80",
              b"0", b"42", b"\xd9\xa3", b"\xef\xbc\x91", b"\xc3\xa9", b"\xce\xb1\xce\xb2", b"\xe4\xb8\xad\xe6\x96\x87",
              b"\xf0\x9f\x98\x80", b"\xff", b"\xc3", b"\x80", b"\xe4\xb8", b"\xf0\x9f\x98", b"'s", b"'S", b"'LL", b"'", b"''",
              b"'ve", b" 'm", b"<|im_", b"end|>", b"<|im_end|>", b"<|audio_pad|><|audio_pad|>", b"<asr_text>",
              b"<", b"|>", b"!!", b"...", b"-", b"_", b"#", b"\x01", b"\x7f"]
    known = [b"\xc3", b"a\xc3", b"\xe4\xb8", b"x\xf0\x9f\x98", b"\xc3<|im_end|>", b"ab\xe4\xb8<asr_text>x",
             b" \xce", b"\t\xc3"]
    for text in known:
        assert tok.encode(text, False).tolist() == checker.ref_tokenizer_encode(str(path), text, False).tolist(), text
    assert 0 in tok.encode(b"a\xc3", False).tolist()     # the terminator's zero byte, as the reference
    for _ in range(120):
        text = b"".join(pieces[int(i)] for i in rng.integers(0, len(pieces), size=int(rng.integers(0, 40))))
        want = checker.ref_tokenizer_encode(str(path), text, False)
        got = tok.encode(text, False)
        assert got.tolist() == want.tolist(), text
