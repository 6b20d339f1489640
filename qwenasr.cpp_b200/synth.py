"""Seeded synthetic model files and workloads for the Qwen3-ASR text decoder.

No checkpoint or audio is available offline, so the benches and tests run on
random-init weights written as a GGUF file with the tensor names, shapes and
metadata keys of the reference converter (convert.py: rename map :95-133,
metadata :310-354; f32 data like :386-388).  Weights are N(0, std) from
numpy's default_rng(seed), drawn tensor by tensor in a fixed order; the bf16
configurations store bf16-rounded (RNE) values in f32, so the reference's f32
loader reads exactly the values the bf16 device path uses.

Workloads (prompt rows = embedding rows of uniform random ids with a block of
N(0,1) "audio" rows spliced in, as decoder-input.cpp:75-92 splices projector
rows at <|audio_pad|> positions) are derived from seeds as well.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, asdict
from pathlib import Path

import numpy as np

GGUF_ALIGN = 32
GGML_F32 = 0
GGML_I8 = 24
GGML_BF16 = 30
# FP8 projection files (a B200-side format; the reference's converter writes f32
# only): each projection weight is a GGML I8 tensor holding e4m3 codes, followed
# by "<name>.scale", f32 [rows] (value = code x scale of its row); the metadata
# key below declares the convention so that no plain int8 tensor is misread.
FP8_PROJECTIONS_KEY = "qwen3-asr.b200.projections"
FP8_PROJECTIONS_VALUE = "e4m3-row-scale"
PROJECTION_SUFFIXES = ("attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_output.weight", "ffn_gate.weight",
                       "ffn_up.weight", "ffn_down.weight")


def quantize_rows_e4m3(a: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """float32 [rows][K] -> (e4m3 codes as uint8 [rows][K], f32 scales [rows]):
    scale = amax / 448 per row (1 for an all-zero row), code = RNE e4m3 of
    value x (1 / scale) saturated to +-448 (the device quantiser's rule)."""
    import torch
    a = np.ascontiguousarray(a, np.float32)
    amax = np.abs(a).max(axis=1, keepdims=True)
    with np.errstate(divide="ignore"):
        scale = np.where(amax > 0, amax / np.float32(448.0), np.float32(1.0)).astype(np.float32)
        inv = np.where(amax > 0, np.float32(1.0) / scale, np.float32(0.0)).astype(np.float32)
    v = np.clip(a * inv, np.float32(-448.0), np.float32(448.0)).astype(np.float32)
    codes = torch.from_numpy(v).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    return codes, scale[:, 0]

QWEN3_ASR_0_6B = dict(n_layers=28, hidden=1024, n_heads=16, n_kv_heads=8, head_dim=128,
                      intermediate=3072, vocab=151936, rope_theta=1.0e6, rms_norm_eps=1.0e-6)
QWEN3_ASR_1_7B = dict(QWEN3_ASR_0_6B, hidden=2048, intermediate=6144)
# Small model with the real attention geometry, for tests that must finish in seconds.
TINY = dict(n_layers=2, hidden=256, n_heads=16, n_kv_heads=8, head_dim=128,
            intermediate=512, vocab=1000, rope_theta=1.0e6, rms_norm_eps=1.0e-6)

TOKEN_IDS = dict(endoftext=151643, im_start=151644, im_end=151645, audio=151676,
                 audio_start=151669, audio_end=151670, asr_text=151704)

# Byte-level tokenizer for small synthetic vocabularies: ids 0..255 are the
# 256 byte symbols, the special tokens follow, so a prompt built from the ASR
# template tokenises inside a 1000-row embedding table.
BYTE_TOKEN_IDS = dict(endoftext=256, im_start=257, im_end=258, audio_start=259, audio_end=260, audio=261,
                      asr_text=262)
SPECIAL_STRINGS = dict(endoftext="<|endoftext|>", im_start="<|im_start|>", im_end="<|im_end|>",
                       audio_start="<|audio_start|>", audio_end="<|audio_end|>", audio="<|audio_pad|>",
                       asr_text="<asr_text>")


BPE_SAMPLE = ("You transcribe speech. Be exact. The quick brown fox jumps over the lazy dog; the dog "
              "sleeps. language English German French system user assistant transcription of the audio "
              "that follows, with punctuation and numbers like 2024 or 3.14, isn't it? We're there.\n")


def byte_merges(n_merges: int = 200) -> list[tuple[str, str]]:
    """A small byte-level BPE merge table learned from BPE_SAMPLE (most
    frequent adjacent pair first, ties broken by the pair's text), so the
    synthetic tokenizer exercises the merge path.  Words carry their leading
    space, as the byte-level pre-tokeniser keeps it."""
    sym = byte_symbols()
    words = []
    for i, w in enumerate(BPE_SAMPLE.split(" ")):
        text = (" " if i else "") + w
        words.append([sym[b] for b in text.encode()])
    merges = []
    for _ in range(n_merges):
        counts: dict[tuple[str, str], int] = {}
        for w in words:
            for a, b in zip(w, w[1:]):
                counts[(a, b)] = counts.get((a, b), 0) + 1
        if not counts:
            break
        best = min(counts, key=lambda k: (-counts[k], k))
        merges.append(best)
        for w in words:
            i = 0
            while i + 1 < len(w):
                if (w[i], w[i + 1]) == best:
                    w[i:i + 2] = [w[i] + w[i + 1]]
                else:
                    i += 1
    return merges


def byte_symbols() -> list[str]:
    """The byte-level BPE alphabet: byte b -> one printable character (the
    published GPT-2 mapping: printable Latin-1 bytes map to themselves, the
    other 68 bytes to code points 256, 257, ... in byte order)."""
    keep = list(range(0x21, 0x7F)) + list(range(0xA1, 0xAD)) + list(range(0xAE, 0x100))
    table, extra = {}, 0
    for b in range(256):
        if b in keep:
            table[b] = chr(b)
        else:
            table[b] = chr(256 + extra)
            extra += 1
    return [table[b] for b in range(256)]


@dataclass
class ModelConfig:
    n_layers: int
    hidden: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rope_theta: float
    rms_norm_eps: float

    @staticmethod
    def of(d: dict) -> "ModelConfig":
        return ModelConfig(**d)


def tensor_specs(cfg: ModelConfig, audio_hidden: int = 0) -> list[tuple[str, tuple[int, ...], str]]:
    """(name, numpy shape = reversed GGML ne, kind) in file order.  With
    audio_hidden > 0 the audio projector follows the text tensors (names and
    shapes of convert.py:145-150 and audio-encoder.cpp:776-790: LayerNorm
    weight and bias [Ha], proj.0 [Ha][Ha] + bias, proj.1 [H][Ha] + bias)."""
    H, F, V, D = cfg.hidden, cfg.intermediate, cfg.vocab, cfg.head_dim
    q, kv = cfg.n_heads * D, cfg.n_kv_heads * D
    out = [("text.token_embd.weight", (V, H), "w"),
           ("text.output_norm.weight", (H,), "norm"),
           ("text.output.weight", (V, H), "w")]
    for layer in range(cfg.n_layers):
        p = f"text.blk.{layer}."
        out += [(p + "attn_norm.weight", (H,), "norm"), (p + "ffn_norm.weight", (H,), "norm"),
                (p + "attn_q.weight", (q, H), "w"), (p + "attn_k.weight", (kv, H), "w"),
                (p + "attn_v.weight", (kv, H), "w"), (p + "attn_output.weight", (H, q), "w"),
                (p + "attn_q_norm.weight", (D,), "norm"), (p + "attn_k_norm.weight", (D,), "norm"),
                (p + "ffn_gate.weight", (F, H), "w"), (p + "ffn_up.weight", (F, H), "w"),
                (p + "ffn_down.weight", (H, F), "w")]
    if audio_hidden:
        A = audio_hidden
        out += [("audio.post_norm.weight", (A,), "norm"), ("audio.post_norm.bias", (A,), "w"),
                ("audio.proj.0.weight", (A, A), "w"), ("audio.proj.0.bias", (A,), "w"),
                ("audio.proj.1.weight", (H, A), "w"), ("audio.proj.1.bias", (H,), "w")]
    return out


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even), kept as float32."""
    u = a.astype(np.float32, copy=False).view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return r.view(np.float32)


# ---- GGUF v3 writer (own code, from the public format description) ----

def _kv_str(key: str, val: str) -> bytes:
    k, v = key.encode(), val.encode()
    return struct.pack("<Q", len(k)) + k + struct.pack("<I", 8) + struct.pack("<Q", len(v)) + v


def _kv_u32(key: str, val: int) -> bytes:
    k = key.encode()
    return struct.pack("<Q", len(k)) + k + struct.pack("<II", 4, val)


def _kv_f32(key: str, val: float) -> bytes:
    k = key.encode()
    return struct.pack("<Q", len(k)) + k + struct.pack("<If", 6, val)


def _kv_arr_str(key: str, items: list[str]) -> bytes:
    k = key.encode()
    body = b"".join(struct.pack("<Q", len(s.encode())) + s.encode() for s in items)
    return struct.pack("<Q", len(k)) + k + struct.pack("<IIQ", 9, 8, len(items)) + body


def _kv_arr_i32(key: str, items: np.ndarray) -> bytes:
    k = key.encode()
    return struct.pack("<Q", len(k)) + k + struct.pack("<IIQ", 9, 5, len(items)) + items.astype("<i4").tobytes()


def metadata(cfg: ModelConfig, name: str, tokenizer: bool | str) -> list[bytes]:
    """tokenizer: False (none), True (placeholder vocabulary with the real
    Qwen special-token ids) or "bytes" (byte-level vocabulary, BYTE_TOKEN_IDS)."""
    ids = BYTE_TOKEN_IDS if tokenizer == "bytes" else TOKEN_IDS
    kv = [_kv_str("general.architecture", "qwen3-asr"), _kv_str("general.name", name),
          _kv_str("qwen3-asr.arch", "qwen3-asr"), _kv_u32("general.alignment", GGUF_ALIGN),
          _kv_u32("qwen3-asr.audio.sample_rate", 16000), _kv_u32("qwen3-asr.audio.num_mel_bins", 128),
          _kv_u32("qwen3-asr.audio.d_model", 896), _kv_u32("qwen3-asr.audio.encoder_layers", 18),
          _kv_u32("qwen3-asr.audio.encoder_attention_heads", 14), _kv_u32("qwen3-asr.audio.encoder_ffn_dim", 3584),
          _kv_u32("qwen3-asr.audio.downsample_hidden_size", 480), _kv_u32("qwen3-asr.audio.output_dim", cfg.hidden),
          _kv_u32("qwen3-asr.text.vocab_size", cfg.vocab), _kv_u32("qwen3-asr.text.hidden_size", cfg.hidden),
          _kv_u32("qwen3-asr.text.intermediate_size", cfg.intermediate),
          _kv_u32("qwen3-asr.text.num_hidden_layers", cfg.n_layers),
          _kv_u32("qwen3-asr.text.num_attention_heads", cfg.n_heads),
          _kv_u32("qwen3-asr.text.num_key_value_heads", cfg.n_kv_heads),
          _kv_u32("qwen3-asr.text.head_dim", cfg.head_dim),
          _kv_f32("qwen3-asr.text.rope_theta", cfg.rope_theta),
          _kv_f32("qwen3-asr.text.rms_norm_eps", cfg.rms_norm_eps),
          _kv_u32("qwen3-asr.token.audio_token_id", ids["audio"]),
          _kv_u32("qwen3-asr.token.audio_start_token_id", ids["audio_start"]),
          _kv_u32("qwen3-asr.token.audio_end_token_id", ids["audio_end"])]
    merges: list[str] = []
    if tokenizer == "bytes":
        n = max(cfg.vocab, ids["asr_text"] + 1)
        tokens = byte_symbols() + [f"<t{i}>" for i in range(256, n)]
        for k, i in ids.items():
            tokens[i] = SPECIAL_STRINGS[k]
        # merged tokens right after the special ids (as many as fit)
        nxt = max(ids.values()) + 1
        for a, b in byte_merges():
            if nxt >= n:
                break
            tokens[nxt] = a + b
            merges.append(f"{a} {b}")
            nxt += 1
    else:
        n = max(cfg.vocab, ids["asr_text"] + 1)
        tokens = [f"<t{i}>" for i in range(n)]
    if tokenizer:
        kv += [_kv_str("tokenizer.ggml.model", "gpt2"),
               _kv_arr_str("tokenizer.ggml.tokens", tokens),
               _kv_arr_i32("tokenizer.ggml.token_type", np.ones(n, np.int32)),
               _kv_arr_str("tokenizer.ggml.merges", merges),
               _kv_u32("tokenizer.ggml.eos_token_id", ids["im_end"]),
               _kv_u32("qwen3-asr.token.endoftext_token_id", ids["endoftext"]),
               _kv_u32("qwen3-asr.token.im_start_token_id", ids["im_start"]),
               _kv_u32("qwen3-asr.token.im_end_token_id", ids["im_end"]),
               _kv_u32("qwen3-asr.token.asr_text_token_id", ids["asr_text"])]
    return kv


def _gen_tensor(rng: np.random.Generator, shape, kind: str, std: float, norm_init: str, round_bf16: bool):
    a = rng.standard_normal(size=shape, dtype=np.float32)
    a *= np.float32(std)
    if kind == "norm" and norm_init == "one_plus":
        a += np.float32(1.0)
    return bf16_round(a) if round_bf16 else a


def write_gguf(path: str | Path, cfg: ModelConfig | dict, seed: int = 0, std: float = 0.02,
               weights: str = "f32", norm_init: str = "normal", tokenizer: bool | str = True,
               audio_hidden: int = 0, storage: str = "f32") -> Path:
    """Write a random-init text-decoder GGUF; returns the path.

    weights: "f32" (plain N(0,std) floats) or "bf16" (bf16-rounded, stored f32).
    norm_init: "normal" -> norm weights ~ N(0,std) like every other tensor;
               "one_plus" -> 1 + N(0,std) (a trained-like scale).
    audio_hidden: > 0 adds the audio projector tensors (tensor_specs).
    storage: "f32" (GGML type 0, as the reference's converter writes),
             "bf16" (GGML type 30: the bf16-rounded values' upper 16 bits) or
             "fp8" (the projections as e4m3 codes + row scales, see
             FP8_PROJECTIONS_KEY, quantised from the bf16-rounded values;
             every other tensor f32).
    """
    if storage not in ("f32", "bf16", "fp8"):
        raise ValueError(storage)
    if storage in ("bf16", "fp8"):
        weights = "bf16"
    cfg = ModelConfig.of(cfg) if isinstance(cfg, dict) else cfg
    path = Path(path)
    specs = tensor_specs(cfg, audio_hidden)
    kv = metadata(cfg, f"qwen3-asr-synthetic-{cfg.hidden}", tokenizer)
    if storage == "fp8":
        kv.append(_kv_str(FP8_PROJECTIONS_KEY, FP8_PROJECTIONS_VALUE))
    base_es, base_type = (2, GGML_BF16) if storage == "bf16" else (4, GGML_F32)
    # (name, numpy shape, GGML type, bytes, generated-tensor index or -1 for a scale)
    layout = []
    for idx, (name, shape, _) in enumerate(specs):
        fp8 = storage == "fp8" and name.endswith(PROJECTION_SUFFIXES)
        if fp8:
            layout.append((name, shape, GGML_I8, int(np.prod(shape)), idx))
            layout.append((name + ".scale", (shape[0],), GGML_F32, shape[0] * 4, -1))
        else:
            layout.append((name, shape, base_type, int(np.prod(shape)) * base_es, idx))
    infos = []
    offset = 0
    for name, shape, gtype, nb, _ in layout:
        ne = tuple(reversed(shape))
        nm = name.encode()
        infos.append(struct.pack("<Q", len(nm)) + nm + struct.pack("<I", len(ne)) +
                     b"".join(struct.pack("<Q", d) for d in ne) + struct.pack("<IQ", gtype, offset))
        offset += (nb + GGUF_ALIGN - 1) // GGUF_ALIGN * GGUF_ALIGN
    head = b"GGUF" + struct.pack("<IQQ", 3, len(layout), len(kv)) + b"".join(kv) + b"".join(infos)
    pad = (-len(head)) % GGUF_ALIGN
    rng = np.random.default_rng(seed)
    with open(path, "wb") as f:
        f.write(head + b"\0" * pad)
        pending_scale = None
        for name, shape, gtype, nb, idx in layout:
            if idx < 0:
                a = pending_scale
            else:
                a = _gen_tensor(rng, shape, specs[idx][2], std, norm_init, weights == "bf16")
                if gtype == GGML_BF16:
                    a = (np.ascontiguousarray(a).view(np.uint32) >> np.uint32(16)).astype(np.uint16)
                elif gtype == GGML_I8:
                    a, pending_scale = quantize_rows_e4m3(a)
            f.write(memoryview(np.ascontiguousarray(a)).cast("B"))
            f.write(b"\0" * ((-a.nbytes) % GGUF_ALIGN))
    return path


# ---- minimal reader (for building prompts and for the oracle) ----

def read_gguf(path: str | Path) -> dict[str, np.ndarray]:
    """name -> float32 array (numpy shape = reversed ne): a read-only memmap
    for f32 tensors, a widened copy for bf16 ones."""
    path = Path(path)
    buf = np.memmap(path, dtype=np.uint8, mode="r")
    pos = 0

    def take(fmt):
        nonlocal pos
        vals = struct.unpack_from(fmt, buf, pos)
        pos += struct.calcsize(fmt)
        return vals

    def skip_str():
        nonlocal pos
        (n,) = take("<Q")
        pos += n

    def read_str():
        nonlocal pos
        (n,) = take("<Q")
        s = bytes(buf[pos:pos + n]).decode()
        pos += n
        return s

    sizes = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}
    magic = bytes(buf[:4])
    if magic != b"GGUF":
        raise ValueError("not a GGUF file")
    pos = 4
    version, n_t, n_kv = take("<IQQ")
    align = GGUF_ALIGN
    for _ in range(n_kv):
        key = read_str()
        (t,) = take("<I")
        if t == 8:
            skip_str()
        elif t == 9:
            at, n = take("<IQ")
            if at == 8:
                for _ in range(n):
                    skip_str()
            else:
                pos += sizes[at] * n
        else:
            if key == "general.alignment" and t == 4:
                (align,) = struct.unpack_from("<I", buf, pos)
            pos += sizes[t]
    infos = []
    for _ in range(n_t):
        name = read_str()
        (nd,) = take("<I")
        ne = take("<" + "Q" * nd)
        t, off = take("<IQ")
        infos.append((name, ne, t, off))
    data0 = (pos + align - 1) // align * align
    out = {}
    for name, ne, t, off in infos:
        shape = tuple(reversed(ne))
        if t == GGML_F32:
            out[name] = np.ndarray(shape, dtype=np.float32, buffer=buf, offset=data0 + off)
        elif t == GGML_BF16:   # widened to f32 (a copy)
            bits = np.ndarray(shape, dtype=np.uint16, buffer=buf, offset=data0 + off)
            out[name] = (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)
        elif t == GGML_I8:     # e4m3 codes of an FP8 projection file, dequantised below
            out[name] = np.ndarray(shape, dtype=np.uint8, buffer=buf, offset=data0 + off)
        else:
            raise ValueError(f"{name}: only f32, bf16 and FP8-projection tensors are read here")
    for name in [n for n, (_, _, t, _) in zip(list(out), infos) if t == GGML_I8]:
        import torch
        scale = out.pop(name + ".scale")
        codes = torch.from_numpy(np.array(out[name], copy=True)).view(torch.float8_e4m3fn)
        out[name] = (codes.float().numpy() * scale[:, None]).astype(np.float32)   # value = code x row scale
    return out


# ---- workloads ----

def prompt_rows(embd: np.ndarray, n_tokens: int, rng: np.random.Generator,
                audio_rows: int | None = None, audio_start: int = 9) -> tuple[np.ndarray, np.ndarray]:
    """[n_tokens, H] f32 decoder input: embedding rows of uniform random ids with
    audio_rows N(0,1) rows spliced in from audio_start (the layout the reference's
    decoder-input stage produces).  Returns (values, ids)."""
    V, H = embd.shape
    ids = rng.integers(0, V, size=n_tokens, dtype=np.int64)
    x = np.asarray(embd[ids], dtype=np.float32).copy()
    if audio_rows:
        start = min(audio_start, max(0, n_tokens - audio_rows))
        x[start:start + audio_rows] = rng.standard_normal((audio_rows, H), dtype=np.float32)
    return x, ids.astype(np.int32)


def config1_prompt(embd: np.ndarray, seed: int = 1001) -> np.ndarray:
    """160 tokens, ids ~ U[0, V), 143 N(0,1) audio rows at positions 9..151."""
    rng = np.random.default_rng(seed)
    x, _ = prompt_rows(embd, 160, rng, audio_rows=143, audio_start=9)
    return x


def config2_prompts(embd: np.ndarray, n_streams: int, seed: int = 1002, gpu: int = 0,
                    lo: int = 100, hi: int = 400, audio_frac: float = 0.9) -> list[np.ndarray]:
    """Per stream: P ~ U[lo, hi], audio rows filling audio_frac of the prompt as one
    block after a short text prefix."""
    out = []
    for s in range(n_streams):
        rng = np.random.default_rng(seed * 1_000_003 + gpu * 65_536 + s)
        P = int(rng.integers(lo, hi + 1))
        n_audio = int(round(audio_frac * P))
        prefix = min(9, (P - n_audio) // 2)
        x, _ = prompt_rows(embd, P, rng, audio_rows=n_audio, audio_start=prefix)
        out.append(x)
    return out


def log_uniform_lengths(n: int, lo: int, hi: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return np.exp(rng.uniform(np.log(lo), np.log(hi), size=n)).astype(np.int64).clip(lo, hi)


def config_dict(cfg: ModelConfig) -> dict:
    return asdict(cfg)
