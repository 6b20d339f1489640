"""GPU parity of the device decoder input (qkv_decoder_input, qkv_prefill_ids)
against the reference's own assembly (tests/golden/decoder_input.npz, from
qwenasr_decoder_input_from_audio, src/decoder-input.cpp:26-101) and the
oracle's restatement of its splice.

Bars: f32 weights, bit-exact rows; bf16 weights, bit-exact against the splice
over the handle's bf16-rounded table; prefill from ids identical to prefill
from the same rows uploaded from the host; the reference's errors, with its
messages, in its order."""
import hashlib
from pathlib import Path

import numpy as np
import pytest

from conftest import rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def digest(a):
    return hashlib.sha256(np.ascontiguousarray(a, np.float32).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN / "decoder_input.npz")


@pytest.fixture(scope="module")
def files(synth, tmp_path_factory):
    d = tmp_path_factory.mktemp("dig")
    return {w: synth.write_gguf(d / f"tiny_bytes_{w}.gguf", dict(synth.TINY), seed=0, weights=w,
                                norm_init="one_plus", tokenizer="bytes") for w in ("f32", "bf16")}


def decoder(pkg, path, w, streams=4, batch_tokens=512):
    rt = pkg.runtime_config(device=0, weight_dtype=w, kv_dtype=1, max_streams=streams, max_context=512,
                            max_batch_tokens=batch_tokens)
    return pkg.Decoder.from_gguf(path, rt)


def cases(g):
    return [(g[f"ids_{k}"], g[f"audio_{k}"]) for k in range(3)]


@pytest.mark.parametrize("where", ["host", "device"])
def test_decoder_input_f32_matches_reference(pkg, golden, files, where):
    """Three prompts in one call (5, 37 and 130 audio rows), twice in a row."""
    cs = cases(golden)
    aid = int(golden["audio_token_id"])
    with decoder(pkg, files["f32"], pkg.F32) as dec:
        audio = [a if where == "host" else torch.tensor(a, device="cuda") for _, a in cs]
        T = sum(len(i) for i, _ in cs)
        for _ in range(2):
            x = torch.full((T, 256), float("nan"), device="cuda")
            dec.decoder_input([len(i) for i, _ in cs], [i for i, _ in cs], audio, aid, x.data_ptr())
            torch.cuda.synchronize()
            dec.sync()
            rows = x.cpu().numpy()
            t = 0
            for k, (ids, _) in enumerate(cs):
                assert digest(rows[t:t + len(ids)]) == str(golden[f"rows_sha256_{k}"])
                t += len(ids)
            assert np.array_equal(rows[:len(cs[0][0])], golden["rows_0"])


def test_decoder_input_bf16_matches_oracle(pkg, synth, checker, golden, files):
    cs = cases(golden)
    aid = int(golden["audio_token_id"])
    embd = np.array(synth.read_gguf(files["bf16"])["text.token_embd.weight"])   # bf16-representable values
    with decoder(pkg, files["bf16"], pkg.BF16) as dec:
        T = sum(len(i) for i, _ in cs)
        x = torch.zeros((T, 256), device="cuda")
        dec.decoder_input([len(i) for i, _ in cs], [i for i, _ in cs], [a for _, a in cs], aid, x.data_ptr())
        torch.cuda.synchronize()
        dec.sync()
        rows = x.cpu().numpy()
    t = 0
    for ids, audio in cs:
        rc, want = checker.decoder_input(ids, embd, audio, aid)
        assert rc == 0
        assert np.array_equal(rows[t:t + len(ids)], want)
        t += len(ids)


@pytest.mark.parametrize("w", ["f32", "bf16"])
def test_prefill_ids_matches_prefill_rows(pkg, synth, checker, golden, files, w):
    """Prefill from ids (rows built on the device) and from the same rows
    uploaded from the host: identical greedy ids, logits within the spread
    of two prefills of the same rows on one path.  The rows are bit-identical
    (the tests above); split-K projections add their partial sums atomically,
    so prefills of identical rows differ run to run (measured on this model:
    up to 6.5e-5 relative with f32 weights, 2.4e-3 with bf16 weights and
    activations, where a flipped bf16 rounding moves a value by 2^-8)."""
    cs = cases(golden)
    aid = int(golden["audio_token_id"])
    embd = np.array(synth.read_gguf(files[w])["text.token_embd.weight"])
    rows = [checker.decoder_input(i, embd, a, aid)[1] for i, a in cs]
    wd = pkg.F32 if w == "f32" else pkg.BF16
    with decoder(pkg, files[w], wd, streams=8) as dec:
        s1 = [dec.open() for _ in cs]
        ids1, lg1 = dec.prefill_ids(s1, [i for i, _ in cs], [torch.tensor(a, device="cuda") for _, a in cs], aid,
                                    want_logits=True)
        s2 = [dec.open() for _ in cs]
        ids2, lg2 = dec.prefill(s2, rows, want_logits=True)
    assert np.array_equal(ids1, ids2)
    assert rel_err(lg1, lg2) < (1e-4 if w == "f32" else 1e-2)


def test_decoder_input_errors(pkg, golden, files):
    """The reference's checks and messages, in its order; nothing is launched
    or appended when a check fails."""
    ids, audio = cases(golden)[0]
    aid = int(golden["audio_token_id"])
    with decoder(pkg, files["f32"], pkg.F32) as dec:
        x = torch.zeros((len(ids) + 8, 256), device="cuda")
        with pytest.raises(pkg.QkvError) as ei:
            dec.decoder_input([len(ids)], [ids], [audio[:4]], aid, x.data_ptr())
        assert str(golden["error_0"]) in str(ei.value)
        with pytest.raises(pkg.QkvError) as ei:
            dec.decoder_input([len(ids)], [ids], [np.concatenate([audio, audio[:1]])], aid, x.data_ptr())
        assert str(golden["error_1"]) in str(ei.value)
        bad = ids.copy()
        bad[2] = 1000
        with pytest.raises(pkg.QkvError) as ei:
            dec.decoder_input([len(ids)], [bad], [audio], aid, x.data_ptr())
        assert "out of embedding range" in str(ei.value)
        s = dec.open()
        with pytest.raises(pkg.QkvError):
            dec.prefill_ids([s], [bad], [audio], aid)
        assert dec.length(s) == 0
        ids_out = dec.prefill_ids([s], [ids], [audio], aid)   # the handle is still usable
        assert ids_out.shape == (1,)
