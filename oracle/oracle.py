"""ctypes access to the CPU checkers (TEST INFRASTRUCTURE ONLY).

- OracleModel: the C restatement (oracle/qkv_oracle.c -> _build/libqkv_oracle.so)
- RefModel:    the reference's own scalar path (oracle/_ref/libqwenasr_ref.so,
               built by `make -C oracle ref` from the reference sources)

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs use this
module, and only to check or time the reference arithmetic on the CPU.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "libqkv_oracle.so"
REF_SO = HERE / "_ref" / "libqwenasr_ref.so"
# The reference checkout's src/ beside this repository unless QWENASR_REF_SRC names another.
REF_SRC = Path(os.environ.get("QWENASR_REF_SRC", str(HERE.parent.parent / "reference" / "src")))

_F = C.POINTER(C.c_float)
_I = C.POINTER(C.c_int32)


def build(ref: bool = True) -> None:
    """Build the checkers in-tree (the reference build only where its sources exist)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "all"], check=True)
    if ref and REF_SRC.is_dir():
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF_SRC={REF_SRC}"], check=True)


class _Layer(C.Structure):
    _fields_ = [(n, _F) for n in ("attn_norm", "ffn_norm", "q_w", "k_w", "v_w", "o_w", "q_norm", "k_norm",
                                  "gate_w", "up_w", "down_w")]


class _Model(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("hidden", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("intermediate", C.c_int), ("vocab", C.c_int),
                ("rope_theta", C.c_float), ("rms_norm_eps", C.c_float), ("layers", C.POINTER(_Layer)),
                ("embd", _F), ("output_norm", _F), ("output_w", _F)]


class _Cfg(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("hidden", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("intermediate", C.c_int), ("vocab", C.c_int),
                ("rope_theta", C.c_float), ("rms_norm_eps", C.c_float)]


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not ORACLE_SO.exists():
            build(ref=False)
        _lib = C.CDLL(str(ORACLE_SO))
        L = _lib
        L.oracle_layer_prefill.argtypes = [C.POINTER(_Model), C.c_int, _F, C.c_int, _F, _F, _F]
        L.oracle_prefill_logits.argtypes = [C.POINTER(_Model), _F, C.c_int, _F]
        L.oracle_generate_cached.argtypes = [C.POINTER(_Model), _F, C.c_int, C.c_int, _I, C.c_int, _I, _I, _I, _F,
                                             _F, _F]
        L.oracle_generate_forced.argtypes = [C.POINTER(_Model), _F, C.c_int, C.c_int, _I, _I, _F]
        L.oracle_append_qkv.argtypes = [_F, _F, _F, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, C.c_float, _F,
                                        _F, _F]
        L.oracle_attend.argtypes = [_F, _F, _F, C.c_int, C.c_int, C.c_int, C.c_int, _F]
        L.oracle_kv_step_batch.argtypes = [C.c_int, C.c_int, _F, _F, _F, C.POINTER(_F), C.POINTER(_F), _I, _I,
                                           C.c_int, C.c_int, C.c_int, C.c_float, C.c_float, _F, C.c_int]
        L.oracle_rope_cos_sin.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float, _F, _F]
        L.oracle_argmax.argtypes = [_F, C.c_int]
        L.oracle_argmax.restype = C.c_int32
        L.oracle_decoder_input.argtypes = [_I, C.c_int, _F, C.c_int, C.c_int, _F, C.c_int, C.c_int32, _F]
    return _lib


def ref_lib():
    global _ref
    if _ref is None:
        if not REF_SO.exists():
            raise FileNotFoundError(f"{REF_SO} not built (make -C oracle ref)")
        _ref = C.CDLL(str(REF_SO))
        P = C.POINTER(_Cfg)
        _ref.ref_prefill_logits.argtypes = [C.c_char_p, P, _F, C.c_int, _F]
        _ref.ref_generate_cached.argtypes = [C.c_char_p, P, _F, C.c_int, C.c_int, _I, C.c_int, _I, _I, _I]
        _ref.ref_generate_greedy.argtypes = [C.c_char_p, P, _F, C.c_int, C.c_int, _I, _I]
        _ref.ref_layer_forward.argtypes = [C.c_char_p, P, C.c_int, _F, C.c_int, _F]
        _ref.ref_decoder_input.argtypes = [C.c_char_p, C.c_int, C.c_int, _F, C.c_int, C.c_char_p, C.c_char_p, C.c_int,
                                           _I, _F, C.POINTER(C.c_int)]
        _ref.ref_tokenizer_decode.argtypes = [C.c_char_p, _I, C.c_int, C.c_int, C.c_char_p, C.c_int,
                                              C.POINTER(C.c_int)]
        _ref.ref_tokenizer_encode.argtypes = [C.c_char_p, C.c_char_p, C.c_int, C.c_int, _I, C.c_int,
                                              C.POINTER(C.c_int)]
        _ref.ref_last_error.restype = C.c_char_p
    return _ref


def ref_available() -> bool:
    return REF_SO.exists()


def _f(a: np.ndarray):
    return a.ctypes.data_as(_F)


def _i(a: np.ndarray):
    return a.ctypes.data_as(_I)


class OracleModel:
    """The C restatement over weights held in numpy arrays (name -> array)."""

    def __init__(self, cfg: dict, tensors: dict[str, np.ndarray]):
        self.cfg = cfg
        self._keep = []

        def t(name):
            a = np.ascontiguousarray(tensors[name], dtype=np.float32)
            self._keep.append(a)
            return _f(a)

        L = cfg["n_layers"]
        self._layers = (_Layer * L)()
        for l in range(L):
            p = f"text.blk.{l}."
            self._layers[l] = _Layer(t(p + "attn_norm.weight"), t(p + "ffn_norm.weight"), t(p + "attn_q.weight"),
                                     t(p + "attn_k.weight"), t(p + "attn_v.weight"), t(p + "attn_output.weight"),
                                     t(p + "attn_q_norm.weight"), t(p + "attn_k_norm.weight"),
                                     t(p + "ffn_gate.weight"), t(p + "ffn_up.weight"), t(p + "ffn_down.weight"))
        self.m = _Model(cfg["n_layers"], cfg["hidden"], cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"],
                        cfg["intermediate"], cfg["vocab"], cfg["rope_theta"], cfg["rms_norm_eps"], self._layers,
                        t("text.token_embd.weight"), t("text.output_norm.weight"), t("text.output.weight"))

    def layer_prefill(self, layer: int, x: np.ndarray):
        x = np.ascontiguousarray(x, np.float32)
        T = x.shape[0]
        kv = self.cfg["n_kv_heads"] * self.cfg["head_dim"]
        out = np.zeros_like(x)
        k = np.zeros((T, kv), np.float32)
        v = np.zeros((T, kv), np.float32)
        rc = lib().oracle_layer_prefill(C.byref(self.m), layer, _f(x), T, _f(out), _f(k), _f(v))
        assert rc == 0
        return out, k, v

    def prefill_logits(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        logits = np.zeros(self.cfg["vocab"], np.float32)
        assert lib().oracle_prefill_logits(C.byref(self.m), _f(x), x.shape[0], _f(logits)) == 0
        return logits

    def generate(self, x: np.ndarray, max_new: int, stop_ids=(), want_logits=False, want_cache=False):
        x = np.ascontiguousarray(x, np.float32)
        T = x.shape[0]
        ids = np.zeros(max(max_new, 1), np.int32)
        n, stopped = C.c_int(), C.c_int()
        stop = np.asarray(list(stop_ids) or [0], np.int32)
        V, L = self.cfg["vocab"], self.cfg["n_layers"]
        kv = self.cfg["n_kv_heads"] * self.cfg["head_dim"]
        logits = np.zeros((max(max_new, 1), V), np.float32) if want_logits else None
        kc = np.zeros((L, T + max_new, kv), np.float32) if want_cache else None
        vc = np.zeros((L, T + max_new, kv), np.float32) if want_cache else None
        rc = lib().oracle_generate_cached(C.byref(self.m), _f(x), T, max_new, _i(stop), len(stop_ids), _i(ids),
                                          C.byref(n), C.byref(stopped), _f(logits) if want_logits else None,
                                          _f(kc) if want_cache else None, _f(vc) if want_cache else None)
        assert rc == 0, rc
        out = {"ids": ids[:n.value].copy(), "stopped": bool(stopped.value)}
        if want_logits:
            out["logits"] = logits[:n.value]
        if want_cache:
            out["k"], out["v"] = kc, vc
        return out

    def generate_forced(self, x: np.ndarray, forced: np.ndarray, n_steps: int):
        x = np.ascontiguousarray(x, np.float32)
        forced = np.ascontiguousarray(forced, np.int32)
        am = np.zeros(n_steps, np.int32)
        logits = np.zeros((n_steps, self.cfg["vocab"]), np.float32)
        rc = lib().oracle_generate_forced(C.byref(self.m), _f(x), x.shape[0], n_steps, _i(forced), _i(am),
                                          _f(logits))
        assert rc == 0
        return am, logits


def append_qkv(qkv_raw, q_norm_w, k_norm_w, position, theta=1.0e6, eps=1.0e-6, n_heads=16, n_kv=8, D=128):
    qkv_raw = np.ascontiguousarray(qkv_raw, np.float32)
    qn = np.ascontiguousarray(q_norm_w, np.float32)
    kn = np.ascontiguousarray(k_norm_w, np.float32)
    q = np.zeros(n_heads * D, np.float32)
    k = np.zeros(n_kv * D, np.float32)
    v = np.zeros(n_kv * D, np.float32)
    lib().oracle_append_qkv(_f(qkv_raw), _f(qn), _f(kn), position, n_heads, n_kv, D, theta, eps, _f(q), _f(k), _f(v))
    return q, k, v


def attend(q, k_cache, v_cache, n_heads=16, n_kv=8, D=128):
    q = np.ascontiguousarray(q, np.float32)
    kc = np.ascontiguousarray(k_cache, np.float32)
    vc = np.ascontiguousarray(v_cache, np.float32)
    out = np.zeros(n_heads * D, np.float32)
    lib().oracle_attend(_f(q), _f(kc), _f(vc), kc.shape[0], n_heads, n_kv, D, _f(out))
    return out


def kv_step_batch(qkv, q_norm_w, k_norm_w, k_caches, v_caches, lens, theta=1.0e6, eps=1.0e-6, threads=0):
    """qkv [L][n][4096]; caches: list of per-stream arrays [L][cap_s][1024]; lens int32 [n] (updated)."""
    L, n, _ = qkv.shape
    caps = np.asarray([a.shape[1] for a in k_caches], np.int32)
    qkv = np.ascontiguousarray(qkv, np.float32)
    qn = np.ascontiguousarray(q_norm_w, np.float32)
    kn = np.ascontiguousarray(k_norm_w, np.float32)
    kp = (_F * n)(*[_f(a) for a in k_caches])
    vp = (_F * n)(*[_f(a) for a in v_caches])
    out = np.zeros((L, n, 2048), np.float32)
    rc = lib().oracle_kv_step_batch(n, L, _f(qkv), _f(qn), _f(kn), kp, vp, _i(caps), _i(lens), 16, 8, 128, theta, eps,
                                    _f(out), threads)
    assert rc == 0
    return out


def rope_cos_sin(position: int, i: int, head_dim=128, theta=1.0e6):
    c, s = C.c_float(), C.c_float()
    lib().oracle_rope_cos_sin(position, i, head_dim, theta, C.byref(c), C.byref(s))
    return c.value, s.value


class RefModel:
    """The reference's own scalar functions (text-decoder.h) on a GGUF file."""

    def __init__(self, gguf_path, cfg: dict):
        self.path = str(gguf_path).encode()
        self.cfg = cfg
        self.c = _Cfg(cfg["n_layers"], cfg["hidden"], cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"],
                      cfg["intermediate"], cfg["vocab"], cfg["rope_theta"], cfg["rms_norm_eps"])

    def _chk(self, rc):
        if rc != 0:
            raise RuntimeError(ref_lib().ref_last_error().decode())

    def prefill_logits(self, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(self.cfg["vocab"], np.float32)
        self._chk(ref_lib().ref_prefill_logits(self.path, C.byref(self.c), _f(x), x.shape[0], _f(out)))
        return out

    def generate_cached(self, x, max_new, stop_ids=()):
        x = np.ascontiguousarray(x, np.float32)
        ids = np.zeros(max(max_new, 1), np.int32)
        stop = np.asarray(list(stop_ids) or [0], np.int32)
        n, st = C.c_int32(), C.c_int32()
        self._chk(ref_lib().ref_generate_cached(self.path, C.byref(self.c), _f(x), x.shape[0], max_new, _i(stop),
                                                len(stop_ids), _i(ids), C.byref(n), C.byref(st)))
        return ids[:n.value].copy(), bool(st.value)

    def generate_greedy(self, x, max_new):
        x = np.ascontiguousarray(x, np.float32)
        ids = np.zeros(max(max_new, 1), np.int32)
        n = C.c_int32()
        self._chk(ref_lib().ref_generate_greedy(self.path, C.byref(self.c), _f(x), x.shape[0], max_new, _i(ids),
                                                C.byref(n)))
        return ids[:n.value].copy()

    def layer_forward(self, layer, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros_like(x)
        self._chk(ref_lib().ref_layer_forward(self.path, C.byref(self.c), layer, _f(x), x.shape[0], _f(out)))
        return out


def decoder_input(ids: np.ndarray, embd: np.ndarray, audio: np.ndarray, audio_token_id: int):
    """(status, rows): the reference's splice (src/decoder-input.cpp:64-98);
    status 0 ok, 1 id out of range, 2 more placeholders than audio rows,
    3 placeholder count differs from the audio rows."""
    ids = np.ascontiguousarray(ids, np.int32)
    embd = np.ascontiguousarray(embd, np.float32)
    audio = np.ascontiguousarray(audio, np.float32).reshape(-1, embd.shape[1])
    out = np.zeros((ids.shape[0], embd.shape[1]), np.float32)
    rc = lib().oracle_decoder_input(_i(ids), ids.shape[0], _f(embd), embd.shape[0], embd.shape[1], _f(audio),
                                    audio.shape[0], int(audio_token_id), _f(out))
    return rc, out


def ref_decoder_input(gguf: str, audio: np.ndarray, audio_token_id: int, system_text: str = "",
                      language: str = "", max_tokens: int = 8192):
    """The reference's own qwenasr_decoder_input_from_audio on `gguf` (its
    prompt template, tokenizer and splice): (status, ids, rows, message)."""
    audio = np.ascontiguousarray(audio, np.float32)
    ids = np.zeros(max_tokens, np.int32)
    rows = np.zeros((max_tokens, audio.shape[1]), np.float32)
    t = C.c_int(0)
    rc = ref_lib().ref_decoder_input(str(gguf).encode(), audio.shape[0], audio.shape[1], _f(audio), int(audio_token_id),
                                     system_text.encode(), language.encode(), max_tokens, _i(ids), _f(rows),
                                     C.byref(t))
    msg = ref_lib().ref_last_error().decode() if rc else ""
    n = t.value if rc == 0 else 0
    return rc, ids[:n].copy(), rows[:n].copy(), msg


def ref_tokenizer_decode(gguf: str, ids, skip_special: bool = True) -> bytes:
    """The reference's own qwenasr_tokenizer_decode on `gguf`'s tokenizer."""
    ids = np.ascontiguousarray(ids, np.int32)
    cap = 64 + 32 * ids.shape[0]
    buf = C.create_string_buffer(cap)
    n = C.c_int(0)
    rc = ref_lib().ref_tokenizer_decode(str(gguf).encode(), _i(ids), ids.shape[0], int(skip_special), buf, cap,
                                        C.byref(n))
    if rc != 0:
        raise RuntimeError(f"ref_tokenizer_decode failed ({rc}): {ref_lib().ref_last_error().decode()}")
    return buf.raw[:n.value]


def ref_tokenizer_encode(gguf: str, text, add_eos: bool = False) -> np.ndarray:
    """The reference's own qwenasr_tokenizer_encode on `gguf`'s tokenizer."""
    b = text.encode() if isinstance(text, str) else bytes(text)
    cap = 16 + 2 * len(b)
    ids = np.zeros(cap, np.int32)
    n = C.c_int(0)
    rc = ref_lib().ref_tokenizer_encode(str(gguf).encode(), b, len(b), int(add_eos), _i(ids), cap, C.byref(n))
    if rc != 0:
        raise RuntimeError(f"ref_tokenizer_encode failed ({rc}): {ref_lib().ref_last_error().decode()}")
    return ids[:n.value].copy()
