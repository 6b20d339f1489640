"""GPU parity of the model-level path (prefill with spliced audio rows, then
batched greedy decode over the paged cache) against the reference's scalar
arithmetic: the committed fixtures (reference scalar C++) and the live oracle.

Bars (from the task's north star):
  f32 weights + f32 cache: logits within 1e-3 relative, identical greedy ids;
  bf16 weights + bf16 cache: >= 99% teacher-forced greedy agreement, max logit
  deviation reported (asserted at full size; this file's tiny model holds 98%);
  8-bit caches: agreement and deviation reported, the e4m3-K / int8-V cache
  held to the bf16 cache's bar, the all-e4m3 cache to a stated lower one."""
from pathlib import Path

import numpy as np
import pytest

from conftest import rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def decoder(pkg, path, w=0, kv=0, streams=4, ctx=256, seed=0, pages=0, batch_tokens=0):
    rt = pkg.runtime_config(device=0, weight_dtype=w, kv_dtype=kv, max_streams=streams, max_context=ctx,
                            max_pages=pages, max_batch_tokens=batch_tokens, page_order_seed=seed)
    return pkg.Decoder.from_gguf(path, rt)


@pytest.mark.parametrize("norm", ["normal", "one_plus"])
def test_prefill_logits_f32(pkg, tiny_files, norm):
    cfg, files = tiny_files
    g = np.load(GOLDEN / f"tiny_{norm}.npz")
    with decoder(pkg, files[("f32", norm)]) as dec:
        s = dec.open()
        ids, logits = dec.prefill([s], [g["x"]], want_logits=True)
    assert rel_err(logits[0], g["ref_prefill_logits"]) < 1e-3
    assert ids[0] == int(np.argmax(g["ref_prefill_logits"]))


@pytest.mark.parametrize("norm", ["normal", "one_plus"])
def test_generate_f32_matches_reference_ids(pkg, tiny_files, norm):
    cfg, files = tiny_files
    g = np.load(GOLDEN / f"tiny_{norm}.npz")
    with decoder(pkg, files[("f32", norm)], seed=17) as dec:
        ids, stopped = dec.generate(g["x"], 16)
        assert ids.tolist() == g["ref_ids"].tolist() and not stopped
        ids, stopped = dec.generate(g["x"], 16, stop_ids=[int(g["stop_id"])])
        assert ids.tolist() == g["ref_ids_stop"].tolist() and stopped
        assert dec.pool_stats()[0] == dec.pool_stats()[1]   # temporary streams returned their pages


def test_generate_edge_counts(pkg, tiny_files):
    cfg, files = tiny_files
    g = np.load(GOLDEN / "tiny_normal.npz")
    with decoder(pkg, files[("f32", "normal")]) as dec:
        ids, _ = dec.generate(g["x"], 1)          # prefill only, no decode forward
        assert ids.tolist() == g["ref_ids"][:1].tolist()
        ids, _ = dec.generate(g["x"], 0)
        assert ids.size == 0
        with pytest.raises(pkg.QkvError) as ei:
            dec.generate(g["x"], 240)             # 24 + 240 > max_context 256
        assert ei.value.code == 3


def prompts(synth, tensors, n, seed, lo=5, hi=70):
    out = []
    for i in range(n):
        rng = np.random.default_rng(seed + i)
        P = int(rng.integers(lo, hi))
        x, _ = synth.prompt_rows(tensors["text.token_embd.weight"], P, rng, audio_rows=int(0.9 * P), audio_start=1)
        out.append(x)
    return out


def batched_ids(dec, xs, n_steps):
    streams = [dec.open() for _ in xs]
    ids = [dec.prefill(streams, xs)]
    for _ in range(n_steps - 1):
        ids.append(dec.decode_step(streams))
    return streams, np.stack(ids, axis=1)


def test_batched_decode_matches_per_stream_oracle(pkg, synth, checker, tiny_files):
    """4 streams of different prompt lengths, prefilled in one call and decoded
    together over a permuted page table, each equal to the single-stream reference loop."""
    cfg, files = tiny_files
    path = files[("f32", "one_plus")]
    tensors = synth.read_gguf(path)
    om = checker.OracleModel(cfg, tensors)
    xs = prompts(synth, tensors, 4, 40)
    with decoder(pkg, path, seed=1234) as dec:
        _, got = batched_ids(dec, xs, 12)
    for i, x in enumerate(xs):
        assert got[i].tolist() == om.generate(x, 12)["ids"].tolist(), f"stream {i}"


def teacher_forced(pkg, synth, checker, path, w, kv, n_streams=4, n_steps=24, seed=60):
    cfg = pkg.read_gguf_config(path)
    tensors = synth.read_gguf(path)
    om = checker.OracleModel(cfg, tensors)
    xs = prompts(synth, tensors, n_streams, seed)
    ref = [om.generate(x, n_steps, want_logits=True) for x in xs]
    agree = total = 0
    dev = 0.0
    with decoder(pkg, path, w=w, kv=kv, streams=n_streams, seed=9, batch_tokens=1024) as dec:
        streams = [dec.open() for _ in xs]
        ids, logits = dec.prefill(streams, xs, want_logits=True)
        for step in range(n_steps):
            for i in range(n_streams):
                want = ref[i]["logits"][step]
                dev = max(dev, rel_err(logits[i], want))
                agree += int(ids[i] == ref[i]["ids"][step])
                total += 1
            if step + 1 == n_steps:
                break
            feed = [int(r["ids"][step]) for r in ref]
            ids, logits = dec.decode_step(streams, in_ids=feed, want_logits=True)
    return agree / total, dev


def test_f32_teacher_forced_logits(pkg, synth, checker, tiny_files):
    cfg, files = tiny_files
    agree, dev = teacher_forced(pkg, synth, checker, files[("f32", "one_plus")], 0, 0)
    assert agree == 1.0 and dev < 1e-3, (agree, dev)


@pytest.mark.parametrize("norm", ["normal", "one_plus"])
def test_bf16_agreement(pkg, synth, checker, tiny_files, norm):
    cfg, files = tiny_files
    agree, dev = teacher_forced(pkg, synth, checker, files[("bf16", norm)], 1, 1, n_streams=8, n_steps=64)
    print(f"bf16 weights+cache ({norm}): teacher-forced agreement {agree:.4f}, max rel logit deviation {dev:.3e}")
    # The 99% bar is asserted at full size (tests/test_gpu_scale.py); this tiny
    # model's 1000-way logits have near-ties that bf16 rounding flips more often.
    assert agree >= 0.98 and dev < 0.02, (agree, dev)


@pytest.mark.parametrize("kv,bar", [(2, 0.90), (3, 0.93)])
def test_fp8_cache_deviation(pkg, synth, checker, tiny_files, kv, bar):
    """8-bit caches on the tiny model with trained-like norm weights (1 +
    N(0, 0.02)): its attention is peaked, so the 8-bit K error moves the
    softmax weights as much as the V error moves the output, and neither
    8-bit cache reaches the bf16 cache's 99% here (measured 94% for both;
    a float64 simulation gives 94.3% for e4m3 K and V, 96.2% for e4m3 K +
    int8 V and 98.4% even for int8 K + bf16 V).  Stated deviations, held to
    90% (e4m3 K and V) and 93% (e4m3 K + int8 V).  The 99% bar is asserted
    at full size on the configured N(0, 0.02) model (test_gpu_scale.py)."""
    cfg, files = tiny_files
    agree, dev = teacher_forced(pkg, synth, checker, files[("bf16", "one_plus")], 1, kv, n_streams=8, n_steps=64)
    print(f"8-bit cache kv={kv}: teacher-forced agreement {agree:.4f}, max rel logit deviation {dev:.3e}")
    assert agree >= bar, (agree, dev)


def test_out_of_pages_and_capacity_errors(pkg, synth, tiny_files):
    cfg, files = tiny_files
    path = files[("f32", "normal")]
    tensors = synth.read_gguf(path)
    x = prompts(synth, tensors, 1, 5, lo=40, hi=41)[0]
    with decoder(pkg, path, streams=2, ctx=64, pages=4) as dec:
        a, b = dec.open(), dec.open()
        dec.prefill([a], [x])                      # 40 tokens -> 3 pages
        with pytest.raises(pkg.QkvError) as ei:
            dec.prefill([b], [x])                  # needs 3, 1 free
        assert ei.value.code == 2
        assert dec.length(b) == 0
        with pytest.raises(pkg.QkvError) as ei:
            dec.decode_step([b])                   # no prompt yet
        assert ei.value.code == 8
        for _ in range(8):
            dec.decode_step([a])                   # 48 tokens, still 3 pages
        dec.decode_step([a])                       # token 49 opens the 4th page
        assert dec.pool_stats()[0] == 0
        with pytest.raises(pkg.QkvError) as ei:
            dec.prefill([b], [x[:1]])
        assert ei.value.code == 2


def test_compaction_preserves_decoding(pkg, synth, tiny_files):
    cfg, files = tiny_files
    path = files[("f32", "one_plus")]
    tensors = synth.read_gguf(path)
    xs = prompts(synth, tensors, 4, 70)
    with decoder(pkg, path, seed=5) as dec:
        streams, ids_a = batched_ids(dec, xs, 6)
        dec.close_stream(streams[0])
        dec.close_stream(streams[2])
        moved = dec.compact()
        more_a = np.stack([dec.decode_step([streams[1], streams[3]]) for _ in range(6)], axis=1)
    with decoder(pkg, path, seed=5) as dec:
        streams, ids_b = batched_ids(dec, xs, 6)
        dec.close_stream(streams[0])
        dec.close_stream(streams[2])
        more_b = np.stack([dec.decode_step([streams[1], streams[3]]) for _ in range(6)], axis=1)
    assert np.array_equal(ids_a, ids_b) and np.array_equal(more_a, more_b)
    assert moved >= 0


def test_fused_swiglu_epilogue_matches_swiglu_kernel(pkg, synth, monkeypatch, tmp_path):
    """Decode of 64 streams through a 2-layer model with the 1.7B layer
    shapes (hidden 2048, FFN 6144, bf16 weights), where the gate/up GEMM runs
    unsplit and takes the fused SwiGLU epilogue (gate and up rows interleaved
    one by one, partners exchanged by a lane shuffle): the ids equal those of
    the same GEMM followed by the SwiGLU kernel (QWENASR_B200_FUSED_SWIGLU=0)
    and the logits agree within 1e-2 relative (both round silu(g) * u to
    bf16 once, but the two kernels' exp and divide can differ in the last
    bit, which flips an occasional bf16 rounding: measured 2.0e-3), and the
    fused run launches one kernel fewer per layer."""
    cfg = dict(synth.TINY, hidden=2048, intermediate=6144)
    path = synth.write_gguf(tmp_path / "wide.gguf", cfg, seed=3, weights="bf16", norm_init="one_plus")
    tensors = synth.read_gguf(path)
    n = 64
    xs = []
    for i in range(n):
        rng = np.random.default_rng(500 + i)
        x, _ = synth.prompt_rows(tensors["text.token_embd.weight"], int(rng.integers(8, 40)), rng,
                                 audio_rows=4, audio_start=1)
        xs.append(x)
    runs = {}
    for fused in ("1", "0"):
        monkeypatch.setenv("QWENASR_B200_FUSED_SWIGLU", fused)
        with decoder(pkg, path, w=1, kv=1, streams=n, ctx=64, seed=2, batch_tokens=4096) as dec:
            streams = [dec.open() for _ in xs]
            dec.prefill(streams, xs)
            out = []
            for _ in range(3):
                l0 = dec.launches()
                ids, logits = dec.decode_step(streams, want_logits=True)
                out.append((ids, logits, dec.launches() - l0))
        runs[fused] = out
    for (ia, la, na), (ib, lb, nb) in zip(runs["1"], runs["0"]):
        d = float(np.max(np.abs(la - lb)) / np.max(np.abs(lb)))
        print(f"fused vs separate SwiGLU: ids equal {np.array_equal(ia, ib)}, max relative logit difference {d:.3e}")
        assert np.array_equal(ia, ib) and d < 1e-2, d
        assert na == nb - cfg["n_layers"], (na, nb)


@pytest.mark.parametrize("w", [1, 2])
def test_residual_slices_match_atomic_accumulation(pkg, synth, monkeypatch, tiny_files, w):
    """QWENASR_B200_RESIDUAL_SLICES=1 (the o and down projections of decode
    batches store split-K partial sums, which the next RMSNorm or the head's
    folds into the residual in slice order) against the default (the
    projections add into the residual with red.add): over prefill and 6
    decode steps of 4 streams, bf16 and FP8 projections, the ids are equal
    and the logits agree within 1e-2 relative: only the f32 summation order
    of the partial sums differs, but that flips an occasional bf16 (or e4m3)
    rounding of the normalised rows the next projection reads (measured
    1.2e-3 with bf16 projections)."""
    cfg, files = tiny_files
    path = files[("bf16", "one_plus")]
    xs = prompts(synth, synth.read_gguf(path), 4, 81, lo=10, hi=60)
    runs = {}
    for mode in ("1", "0"):
        monkeypatch.setenv("QWENASR_B200_RESIDUAL_SLICES", mode)
        with decoder(pkg, path, w=w, kv=1, seed=3, batch_tokens=512) as dec:
            streams = [dec.open() for _ in xs]
            out = [dec.prefill(streams, xs, want_logits=True)]
            out += [dec.decode_step(streams, want_logits=True) for _ in range(6)]
        runs[mode] = out
    for (ia, la), (ib, lb) in zip(runs["1"], runs["0"]):
        assert np.array_equal(ia, ib)
        assert rel_err(la, lb) < 1e-2, rel_err(la, lb)


@pytest.mark.parametrize("kv", [1, 2, 3])
def test_compaction_moves_cache_bytes_and_scales(pkg, synth, tiny_files, kv):
    """Compaction of a bf16 or 8-bit cache: after two streams close and the
    pool is compacted, the surviving streams' K/V bytes (and, for the 8-bit
    caches, their per-token scales) read back identical in every layer, and
    decoding continues."""
    cfg, files = tiny_files
    path = files[("bf16", "one_plus")]
    xs = prompts(synth, synth.read_gguf(path), 4, 71, lo=20, hi=70)
    with decoder(pkg, path, w=1, kv=kv, seed=5, batch_tokens=512) as dec:
        streams, _ = batched_ids(dec, xs, 4)
        dec.close_stream(streams[0])
        dec.close_stream(streams[2])
        keep = [streams[1], streams[3]]
        before = {(l, s): dec.gather(l, s, kv) for l in range(cfg["n_layers"]) for s in keep}
        pages_before = [dec.pages(s).tolist() for s in keep]
        moved = dec.compact()
        after = {(l, s): dec.gather(l, s, kv) for l in range(cfg["n_layers"]) for s in keep}
        assert moved > 0 and [dec.pages(s).tolist() for s in keep] != pages_before
        for key in before:
            for a, b in zip(before[key], after[key]):
                assert np.array_equal(a, b), key
        for _ in range(3):
            dec.decode_step(keep)


def test_stream_reuse_after_close(pkg, synth, checker, tiny_files):
    cfg, files = tiny_files
    path = files[("f32", "normal")]
    tensors = synth.read_gguf(path)
    om = checker.OracleModel(cfg, tensors)
    xs = prompts(synth, tensors, 2, 90)
    with decoder(pkg, path, streams=1) as dec:
        for x in xs:
            s = dec.open()
            got = [int(dec.prefill([s], [x])[0])] + [int(dec.decode_step([s])[0]) for _ in range(4)]
            assert got == om.generate(x, 5)["ids"].tolist()
            dec.close_stream(s)


@pytest.mark.parametrize("kv", [1, 2])
@pytest.mark.parametrize("tokens", [1, 17, 64, 65, 130, 300])
def test_prefill_attention_layer(pkg, synth, checker, tiny_files, tokens, kv):
    """The tensor-core prefill attention (bf16 cache, or e4m3 cache dequantised
    to f16 on the way into shared memory) through one block vs the reference's
    f32 block: prompt lengths around the 64-query item and the 128-key tile
    boundaries.  bf16: 3e-2 relative on the block's update; e4m3: 1e-1 (3
    mantissa bits in the cache)."""
    cfg, files = tiny_files
    path = files[("bf16", "one_plus")]
    tensors = synth.read_gguf(path)
    om = checker.OracleModel(cfg, tensors)
    rng = np.random.default_rng(tokens)
    x = rng.standard_normal((tokens, cfg["hidden"]), dtype=np.float32)
    want, _, _ = om.layer_prefill(1, x)
    with decoder(pkg, path, w=1, kv=kv, streams=2, ctx=512) as dec:
        got = dec.layer_forward(1, x)
    err = rel_err(got - x, want - x)     # compare the block's update, not the residual carried through
    assert err < (3e-2 if kv == 1 else 1e-1), err


@pytest.mark.parametrize("kv", [1, 2, 3])
def test_prefill_attention_tensor_cores_match_cuda_cores(pkg, synth, tiny_files, kv, monkeypatch):
    """Same cache, same prompts: K3 (tcgen05) and the CUDA-core prefill
    attention (f32 math over the exactly dequantised cache) agree.  K3 rounds
    Q and P to the 16-bit operand type (bf16 for a bf16 cache, f16 for e4m3,
    whose K/V are also scaled in f16), hence the tolerance."""
    cfg, files = tiny_files
    path = files[("bf16", "one_plus")]
    tensors = synth.read_gguf(path)
    xs = prompts(synth, tensors, 4, 77, lo=60, hi=300)
    outs = {}
    for mode in ("tensor", "cuda_core"):
        if mode == "cuda_core":
            monkeypatch.setenv("QWENASR_B200_PREFILL_ATTN", "cuda_core")
        else:
            monkeypatch.delenv("QWENASR_B200_PREFILL_ATTN", raising=False)
        with decoder(pkg, path, w=1, kv=kv, streams=4, ctx=512, batch_tokens=1024) as dec:
            streams = [dec.open() for _ in xs]
            outs[mode] = dec.prefill(streams, xs, want_logits=True)
    (ids_t, lg_t), (ids_c, lg_c) = outs["tensor"], outs["cuda_core"]
    worst = max(rel_err(lg_t[i], lg_c[i]) for i in range(len(xs)))
    print(f"kv={kv}: K3 vs CUDA-core prefill logits, max relative deviation {worst:.3e}")
    assert worst < 2e-2, worst
    assert (np.asarray(ids_t) == np.asarray(ids_c)).mean() >= 0.75


def test_bf16_prefill_logits_multi_stream(pkg, synth, checker, tiny_files):
    """Ragged multi-stream prefill through the tensor-core attention (bf16 cache) vs the f32 reference."""
    cfg, files = tiny_files
    path = files[("bf16", "one_plus")]
    tensors = synth.read_gguf(path)
    om = checker.OracleModel(cfg, tensors)
    xs = prompts(synth, tensors, 5, 300, lo=20, hi=200)
    with decoder(pkg, path, w=1, kv=1, streams=5, ctx=256, batch_tokens=1024) as dec:
        streams = [dec.open() for _ in xs]
        ids, logits = dec.prefill(streams, xs, want_logits=True)
    for i, x in enumerate(xs):
        ref = om.prefill_logits(x)
        assert rel_err(logits[i], ref) < 3e-2


def test_prefill_rows_entry_matches_contiguous(pkg, synth, tiny_files):
    """qkv_prefill_rows (one host block per stream, what Decoder.prefill
    passes) and qkv_prefill (one contiguous block) give identical ids and
    logits.  40 prompts of 700-1300 rows x 1 KB span several of the handle's
    16 MB pinned staging chunks, with streams split across chunk edges."""
    import ctypes as C
    cfg, files = tiny_files
    path = files[("bf16", "one_plus")]
    tensors = synth.read_gguf(path)
    xs = prompts(synth, tensors, 40, 900, lo=700, hi=1300)
    total = sum(x.shape[0] for x in xs)
    assert total * cfg["hidden"] * 4 > 2 * (16 << 20)
    with decoder(pkg, path, w=1, kv=1, streams=80, ctx=1400, batch_tokens=total) as dec:
        s_rows = [dec.open() for _ in xs]
        ids_rows, logits_rows = dec.prefill(s_rows, xs, want_logits=True)
        for s in s_rows:
            dec.close_stream(s)
        s_cat = np.array([dec.open() for _ in xs], np.int32)
        lens = np.array([x.shape[0] for x in xs], np.int32)
        emb = np.ascontiguousarray(np.concatenate(xs, axis=0), np.float32)
        ids_cat = np.zeros(len(xs), np.int32)
        logits_cat = np.zeros((len(xs), dec.cfg["vocab"]), np.float32)
        i32 = C.POINTER(C.c_int32)
        f32 = C.POINTER(C.c_float)
        rc = pkg.lib.qkv_prefill(dec.h, len(xs), s_cat.ctypes.data_as(i32), lens.ctypes.data_as(i32),
                                 emb.ctypes.data_as(f32), ids_cat.ctypes.data_as(i32), logits_cat.ctypes.data_as(f32))
        assert rc == 0
    assert np.array_equal(ids_rows, ids_cat)
    assert np.array_equal(logits_rows, logits_cat)


@pytest.mark.parametrize("w", [0, 1])
def test_bf16_typed_file_loads_like_f32_file(pkg, synth, tmp_path, w):
    """The same bf16-rounded weights stored as f32 (as the reference's
    converter writes) and as GGML bf16: identical greedy ids, logits within
    the parity bars (f32 1e-3, bf16 1e-2): two prefills of one file already
    differ by up to ~1.5e-4 (f32) / 2.4e-3 (bf16) because split-K sums are
    atomic, while a wrong conversion would be off by orders of magnitude."""
    a = synth.write_gguf(tmp_path / "f32.gguf", dict(synth.TINY), seed=0, weights="bf16", norm_init="one_plus",
                         tokenizer=False)
    b = synth.write_gguf(tmp_path / "bf16.gguf", dict(synth.TINY), seed=0, norm_init="one_plus", tokenizer=False,
                         storage="bf16")
    xs = prompts(synth, synth.read_gguf(a), 3, 500, lo=40, hi=120)
    out = []
    for path in (a, b):
        with decoder(pkg, path, w=w, kv=1, streams=3, ctx=256, batch_tokens=512) as dec:
            out.append(dec.prefill([dec.open() for _ in xs], xs, want_logits=True))
    assert np.array_equal(out[0][0], out[1][0])
    assert rel_err(out[0][1], out[1][1]) < (1e-3 if w == 0 else 1e-2)


@pytest.mark.parametrize("n", [4, 40])
def test_argmax_first_maximum_over_split_rows(pkg, synth, tmp_path, n, monkeypatch):
    """The device argmax (rows split over several CTAs for a 20000-word
    vocabulary) returns the first maximum of the logits it also returns, for
    the prefill and two decode steps (the f32 re-scoring of the bf16 head is
    off here: it may pick a token whose bf16-input logit is not the largest)."""
    monkeypatch.setenv("QWENASR_B200_EXACT_ARGMAX", "0")
    cfg = dict(synth.TINY, vocab=20000)
    path = synth.write_gguf(tmp_path / "v20k.gguf", cfg, seed=4, weights="bf16", norm_init="one_plus",
                            tokenizer=False)
    xs = prompts(synth, synth.read_gguf(path), n, 600, lo=10, hi=60)
    with decoder(pkg, path, w=1, kv=1, streams=n, ctx=128, batch_tokens=n * 64) as dec:
        s = [dec.open() for _ in xs]
        ids, logits = dec.prefill(s, xs, want_logits=True)
        assert np.array_equal(ids, np.argmax(logits, axis=1))
        for _ in range(2):
            ids, logits = dec.decode_step(s, want_logits=True)
            assert np.array_equal(ids, np.argmax(logits, axis=1))


def test_bf16_head_argmax_is_the_f32_argmax(pkg, synth, tmp_path, monkeypatch):
    """bf16 weights: the LM head's GEMM rounds the final hidden row to bf16,
    so its logits carry up to 2^-8 relative error; the device then re-scores
    in f32 every token within the proven error bound of the maximum.  The ids
    must equal the argmax of the f32 logits W . rmsnorm(x) computed here in
    float64 from the step's own residual rows (qkv_debug_residual), at every
    decode step; without the re-scoring some rows pick another token."""
    import ctypes as C
    cfg = dict(synth.TINY, vocab=20000)
    path = synth.write_gguf(tmp_path / "v20k.gguf", cfg, seed=4, weights="bf16", norm_init="normal",
                            tokenizer=False)
    t = synth.read_gguf(path)
    W = np.asarray(t["text.output.weight"], np.float64)
    g = np.asarray(t["text.output_norm.weight"], np.float64)
    n = 40
    xs = prompts(synth, t, n, 610, lo=10, hi=60)
    miss = {}
    for exact in ("1", "0"):
        monkeypatch.setenv("QWENASR_B200_EXACT_ARGMAX", exact)
        miss[exact] = 0
        with decoder(pkg, path, w=1, kv=1, streams=n, ctx=128, batch_tokens=n * 64) as dec:
            s = [dec.open() for _ in xs]
            dec.prefill(s, xs)
            for _ in range(6):
                ids = dec.decode_step(s)
                x = np.zeros((n, cfg["hidden"]), np.float32)
                assert pkg.lib.qkv_debug_residual(dec.h, n, x.ctypes.data) == 0
                xd = x.astype(np.float64)
                h = xd / np.sqrt((xd * xd).mean(axis=1, keepdims=True) + cfg["rms_norm_eps"]) * g
                want = np.argmax(h @ W.T, axis=1)
                miss[exact] += int(np.sum(np.asarray(ids) != want))
    print(f"rows whose id differs from the f32 argmax: re-scored {miss['1']}, bf16 logits only {miss['0']} (of {6 * n})")
    assert miss["1"] == 0


def test_fp8_weights_deviation(pkg, synth, checker, tiny_files):
    """FP8 projections (e4m3 weights with a scale per weight row, e4m3 token
    rows with a scale per row, tcgen05 kind::f8f6f4) with a bf16 cache,
    against the f32 oracle on the bf16-rounded file: e4m3 keeps 3 mantissa
    bits of every weight and every projection input, so this is a stated
    deviation, not a parity bar (printed; held to 80 % agreement)."""
    cfg, files = tiny_files
    agree, dev = teacher_forced(pkg, synth, checker, files[("bf16", "one_plus")], 2, 1, n_streams=8, n_steps=64)
    print(f"fp8 weights + bf16 cache: teacher-forced agreement {agree:.4f}, max rel logit deviation {dev:.3e}")
    assert agree >= 0.8 and dev < 0.5, (agree, dev)


def test_fp8_file_loads_like_device_quantisation(pkg, synth, checker, tmp_path):
    """An FP8 projection file (e4m3 codes + row scales, written on the host by
    the device quantiser's rule) and the bf16 file of the same seed quantised
    on the device at load give the same greedy ids and logits within the
    split-K atomics' spread; a bf16 handle refuses the FP8 file.  Against the
    f32 oracle run on the file's own dequantised weights, what remains is the
    e4m3 rounding of the projection inputs alone (printed)."""
    cfg = dict(synth.TINY)
    pb = synth.write_gguf(tmp_path / "bf16.gguf", cfg, seed=0, weights="bf16", norm_init="one_plus", tokenizer=False)
    p8 = synth.write_gguf(tmp_path / "fp8.gguf", cfg, seed=0, norm_init="one_plus", tokenizer=False, storage="fp8")
    t8 = synth.read_gguf(p8)
    xs = prompts(synth, t8, 3, 520, lo=40, hi=120)
    out = []
    for path in (pb, p8):
        with decoder(pkg, path, w=2, kv=1, streams=3, ctx=256, batch_tokens=512) as dec:
            s = [dec.open() for _ in xs]
            ids, lg = dec.prefill(s, xs, want_logits=True)
            steps = [ids]
            for _ in range(8):
                steps.append(dec.decode_step(s))
            out.append((np.asarray(steps), lg))
    assert np.array_equal(out[0][0], out[1][0])
    assert rel_err(out[1][1], out[0][1]) < 1e-2
    with pytest.raises(pkg.QkvError) as ei:
        decoder(pkg, p8, w=1, kv=1, streams=1, ctx=64)
    assert ei.value.code == 7
    om = checker.OracleModel(cfg, t8)
    dev = max(rel_err(out[1][1][i], om.prefill_logits(x)) for i, x in enumerate(xs))
    print(f"fp8 file vs the oracle on its own dequantised weights: prefill max rel logit deviation {dev:.3e}")
