"""Generate tests/golden/decoder_input.npz from the reference's own decoder-input
assembly (run in a container that has the reference tree; the fixture is
committed and read without it).

Source of truth: qwenasr_decoder_input_from_audio (src/decoder-input.cpp:26-101)
with the reference's prompt template (src/tokenizer.cpp:529-549) and byte-level
BPE tokenizer (src/tokenizer.cpp), compiled unmodified into oracle/_ref
(`make -C oracle ref`).  The model is the seeded tiny model of
qwenasr.cpp_b200/synth.py with f32 weights and "one_plus" norms (the same
tensors as the other tiny fixtures) plus a byte-level tokenizer whose special
tokens sit at ids 256..262, inside the 1000-row embedding table.

Recorded per case: the prompt ids, the audio rows, a SHA-256 of the
reference's output rows (f32 bytes) and, for the smallest case, the rows
themselves; for the reference's own failure cases, its error message.  Also
detokenisation known answers: the bytes qwenasr_tokenizer_decode
(src/tokenizer.cpp:482-527) gives for a few id sequences, with and without
skipping the special tokens.

    python tests/golden/make_decoder_input_golden.py
"""
from __future__ import annotations

import hashlib
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

import __graft_entry__ as ge  # noqa: E402
from oracle import oracle as checker  # noqa: E402

OK_CASES = [  # (audio rows, system text, language)
    (5, "", ""),
    (37, "You transcribe speech.", "English"),
    (130, "Transcribe.\nBe exact.", "German"),
]
ERR_CASES = [  # (audio rows, system text, language, audio token id)
    (3, "ignore <|audio_pad|> this", "", None),   # one placeholder more than audio rows
    (4, "", "", "audio_start"),                   # the wrong id: one match, four audio rows
]


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a, np.float32).tobytes()).hexdigest()


def main() -> None:
    synth = ge.load_synth()
    checker.build(ref=True)
    cfg = dict(synth.TINY)
    ids_map = synth.BYTE_TOKEN_IDS
    out: dict[str, np.ndarray] = {}
    with tempfile.TemporaryDirectory() as d:
        path = synth.write_gguf(Path(d) / "tiny_bytes.gguf", cfg, seed=0, weights="f32", norm_init="one_plus",
                                tokenizer="bytes")
        embd = np.array(synth.read_gguf(path)["text.token_embd.weight"])
        out["embd_sha256"] = np.array(digest(embd))
        out["audio_token_id"] = np.array(ids_map["audio"], np.int32)
        for k, (a, system, lang) in enumerate(OK_CASES):
            audio = np.random.default_rng(2000 + k).standard_normal((a, cfg["hidden"])).astype(np.float32)
            rc, ids, rows, msg = checker.ref_decoder_input(str(path), audio, ids_map["audio"], system, lang)
            assert rc == 0, msg
            out[f"ids_{k}"] = ids
            out[f"audio_{k}"] = audio
            out[f"rows_sha256_{k}"] = np.array(digest(rows))
            out[f"system_{k}"] = np.array(system)
            out[f"language_{k}"] = np.array(lang)
            if k == 0:
                out["rows_0"] = rows
            print(f"case {k}: {ids.shape[0]} ids, {a} audio rows")
        for k, (a, system, lang, which) in enumerate(ERR_CASES):
            audio = np.random.default_rng(3000 + k).standard_normal((a, cfg["hidden"])).astype(np.float32)
            tid = ids_map["audio"] if which is None else ids_map[which]
            rc, _, _, msg = checker.ref_decoder_input(str(path), audio, tid, system, lang)
            assert rc != 0
            out[f"error_{k}"] = np.array(msg)
            print(f"error case {k}: {msg}")
        detok = [out["ids_1"],
                 np.array([300, 10, 32, 1000, -5, 257, 65, 0xC3, 0xA9, 999, 262], np.int32),
                 np.arange(0, 1000, dtype=np.int32)]
        for k, ids in enumerate(detok):
            out[f"detok_ids_{k}"] = ids
            for skip in (0, 1):
                out[f"detok_bytes_{k}_{skip}"] = np.frombuffer(
                    checker.ref_tokenizer_decode(str(path), ids, bool(skip)), np.uint8).copy()
    np.savez_compressed(HERE / "decoder_input.npz", **out)
    print("wrote", HERE / "decoder_input.npz")


if __name__ == "__main__":
    main()
