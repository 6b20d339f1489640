"""Python handle on the B200 Qwen3-ASR text-decoder KV-cache library.

The product is the native library libqwenasr_b200.so (C ABI declared in
include/qkv.h; CUDA sm_100a kernels + C++ runtime).  This module only binds
it with ctypes for the tests and the bench, the way the reference's Python
check scripts drive its native binary.  There is no Python or CPU fallback:
if the library is missing, importing this module raises.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libqwenasr_b200.so"

QKV_OK = 0
QKV_ERR_CAPACITY = 3
STATUS = {0: "QKV_OK", 1: "QKV_ERR_INVALID_ARG", 2: "QKV_ERR_OUT_OF_PAGES", 3: "QKV_ERR_CAPACITY",
          4: "QKV_ERR_CUDA", 5: "QKV_ERR_DEVICE", 6: "QKV_ERR_IO", 7: "QKV_ERR_FORMAT", 8: "QKV_ERR_STATE",
          9: "QKV_ERR_NO_DEVICE", 10: "QKV_ERR_HOST_MEMORY"}
F32, BF16, FP8 = 0, 1, 2
E4I8 = 3          # 8-bit cache: e4m3 K, int8 (excess-128) V


class ModelConfig(C.Structure):
    _fields_ = [("n_layers", C.c_int32), ("hidden", C.c_int32), ("n_heads", C.c_int32),
                ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("intermediate", C.c_int32),
                ("vocab", C.c_int32), ("rope_theta", C.c_float), ("rms_norm_eps", C.c_float)]


class RuntimeConfig(C.Structure):
    _fields_ = [("device", C.c_int32), ("weight_dtype", C.c_int32), ("kv_dtype", C.c_int32),
                ("page_tokens", C.c_int32), ("max_streams", C.c_int32), ("max_context", C.c_int32),
                ("max_pages", C.c_int64), ("max_batch_tokens", C.c_int32), ("page_order_seed", C.c_uint32)]


class QkvError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS.get(code, code)}: {msg}")
        self.code = code


_P = C.c_void_p
_I32P = C.POINTER(C.c_int32)
_F32P = C.POINTER(C.c_float)
_I64P = C.POINTER(C.c_int64)

# name -> (restype, argtypes); every symbol declared in include/qkv.h.
SIGNATURES = {
    "qkv_read_gguf_config": (C.c_int, [C.c_char_p, C.POINTER(ModelConfig), C.c_char_p, C.c_size_t]),
    "qkv_create": (C.c_int, [C.c_char_p, C.POINTER(ModelConfig), C.POINTER(RuntimeConfig), C.POINTER(_P),
                             C.c_char_p, C.c_size_t]),
    "qkv_create_kv_only": (C.c_int, [C.POINTER(ModelConfig), C.POINTER(RuntimeConfig), _F32P, _F32P,
                                     C.POINTER(_P), C.c_char_p, C.c_size_t]),
    "qkv_destroy": (None, [_P]),
    "qkv_last_error": (C.c_char_p, [_P]),
    "qkv_stream_open": (C.c_int, [_P, _I32P]),
    "qkv_stream_close": (C.c_int, [_P, C.c_int32]),
    "qkv_stream_length": (C.c_int, [_P, C.c_int32, _I32P]),
    "qkv_pool_stats": (C.c_int, [_P, _I64P, _I64P]),
    "qkv_compact": (C.c_int, [_P, _I64P]),
    "qkv_prefill": (C.c_int, [_P, C.c_int32, _I32P, _I32P, _F32P, _I32P, _F32P]),
    "qkv_prefill_rows": (C.c_int, [_P, C.c_int32, _I32P, _I32P, _P, _I32P, _F32P]),
    "qkv_decoder_input": (C.c_int, [_P, C.c_int32, _I32P, _I32P, _P, _I32P, C.c_int32, C.c_int32, _P, _P]),
    "qkv_audio_project": (C.c_int, [_P, C.c_int32, _P, _P, _P]),
    "qkv_audio_projector_width": (C.c_int, [_P, _I32P]),
    "qkv_prefill_ids": (C.c_int, [_P, C.c_int32, _I32P, _I32P, _I32P, _P, _I32P, C.c_int32, C.c_int32, _I32P,
                                  _F32P]),
    "qkv_decode_step": (C.c_int, [_P, C.c_int32, _I32P, _I32P, _I32P, _F32P]),
    "qkv_generate": (C.c_int, [_P, _F32P, C.c_int32, C.c_int32, _I32P, C.c_int32, _I32P, _I32P, _I32P]),
    "qkv_layer_forward": (C.c_int, [_P, C.c_int32, C.c_int32, _F32P, _F32P]),
    "qkv_kv_append": (C.c_int, [_P, C.c_int32, C.c_int32, _P, _P, _P, _P, _P]),
    "qkv_kv_attend": (C.c_int, [_P, C.c_int32, C.c_int32, _P, _P, _P, _P, _P]),
    "qkv_kv_step": (C.c_int, [_P, C.c_int32, _I32P, _P, _P, _P]),
    "qkv_kv_step_host": (C.c_int, [_P, C.c_int32, _I32P, _P, _P]),
    "qkv_stream_extend": (C.c_int, [_P, C.c_int32, C.c_int32]),
    "qkv_fill_random": (C.c_int, [_P, C.c_uint64]),
    "qkv_gather": (C.c_int, [_P, C.c_int32, C.c_int32, _P, _P, _F32P]),
    "qkv_stream_pages": (C.c_int, [_P, C.c_int32, _I32P, C.c_int32, _I32P]),
    "qkv_sync": (C.c_int, [_P]),
    "qkv_debug_wait_timeout": (C.c_int, [_P, C.c_int64]),
    "qkv_debug_residual": (C.c_int, [_P, C.c_int32, C.c_void_p]),
    "qkv_page_read_probe": (C.c_int, [_P, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p]),
    "qkv_last_launches": (C.c_int, [_P, _I64P]),
    "qkv_kv_attend_noalloc": (C.c_int, [_P, C.c_int32, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_int32, _P, _P,
                                        _P, _P, _P, C.c_char_p, C.c_size_t]),
    "qkv_gemm_bf16": (C.c_int, [_P, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_int32, _P]),
    "qkv_gemm_swiglu_bf16": (C.c_int, [_P, _P, _P, C.c_int32, C.c_int32, C.c_int32, _P, _P, C.c_int64, C.c_int32, _P]),
    "qkv_gemm_fp8": (C.c_int, [_P, _P, _P, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_int32, _P]),
    "qkv_quantize_rows_e4m3": (C.c_int, [_P, C.c_int32, C.c_int32, _P, _P, _P]),
    "qkv_prefill_attend": (C.c_int, [_P, C.c_int32, C.c_int32, _P, _P, _P, _P, _P]),
    "qkv_prefill_attend_q16": (C.c_int, [_P, C.c_int32, C.c_int32, _P, _P, _P, _P, _P]),
    "qkv_tokenizer_open": (C.c_int, [C.c_char_p, C.POINTER(C.c_void_p), C.c_char_p, C.c_size_t]),
    "qkv_tokenizer_decode": (C.c_int, [_P, _I32P, C.c_int32, C.c_int32, C.c_char_p, C.c_size_t,
                                       C.POINTER(C.c_size_t)]),
    "qkv_tokenizer_close": (None, [_P]),
    "qkv_tokenizer_encode": (C.c_int, [_P, C.c_char_p, C.c_size_t, C.c_int32, _I32P, C.c_size_t,
                                       C.POINTER(C.c_size_t)]),
    "qkv_asr_prompt_ids": (C.c_int, [_P, C.c_int32, C.c_char_p, C.c_char_p, _I32P, C.c_size_t,
                                     C.POINTER(C.c_size_t)]),
    "qkv_gguf_tensor": (C.c_int, [C.c_char_p, C.c_char_p, _I64P, _I32P, _I32P, _P, C.c_size_t, C.c_char_p,
                                  C.c_size_t]),
    "qkv_pager_create": (_P, [C.c_int64, C.c_int32, C.c_int32, C.c_int32, C.c_uint32]),
    "qkv_pager_destroy": (None, [_P]),
    "qkv_pager_open": (C.c_int, [_P, _I32P]),
    "qkv_pager_close": (C.c_int, [_P, C.c_int32]),
    "qkv_pager_append": (C.c_int, [_P, C.c_int32, C.c_int32, _I32P]),
    "qkv_pager_length": (C.c_int, [_P, C.c_int32, _I32P]),
    "qkv_pager_pages": (C.c_int, [_P, C.c_int32, _I32P, C.c_int32, _I32P]),
    "qkv_pager_free_pages": (C.c_int64, [_P]),
    "qkv_pager_compact": (C.c_int, [_P, _I32P, _I32P, C.c_int64, _I64P]),
    "qkv_pager_check": (C.c_int, [_P]),
}


def load_library(path: Path = LIB_PATH) -> C.CDLL:
    if not path.exists():
        raise RuntimeError(f"native library not built: {path} (run __graft_entry__.build())")
    lib = C.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = load_library()


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


def _ptr(a: np.ndarray, t):
    return a.ctypes.data_as(C.POINTER(t))


def model_config(d: dict) -> ModelConfig:
    return ModelConfig(d["n_layers"], d["hidden"], d["n_heads"], d["n_kv_heads"], d["head_dim"],
                       d["intermediate"], d["vocab"], d["rope_theta"], d["rms_norm_eps"])


def runtime_config(device=0, weight_dtype=F32, kv_dtype=F32, max_streams=1, max_context=256, max_pages=0,
                   max_batch_tokens=0, page_order_seed=0) -> RuntimeConfig:
    return RuntimeConfig(device, weight_dtype, kv_dtype, 16, max_streams, max_context, max_pages,
                         max_batch_tokens, page_order_seed)


def read_gguf_config(path) -> dict:
    cfg = ModelConfig()
    err = C.create_string_buffer(512)
    rc = lib.qkv_read_gguf_config(str(path).encode(), C.byref(cfg), err, 512)
    if rc != QKV_OK:
        raise QkvError(rc, err.value.decode())
    return {f: getattr(cfg, f) for f, _ in ModelConfig._fields_}


class Tokenizer:
    """Detokeniser of a model file's byte-level BPE vocabulary (host only):
    Tokenizer(path).decode(ids, skip_special=True) -> bytes."""

    def __init__(self, path):
        h = C.c_void_p()
        err = C.create_string_buffer(512)
        rc = lib.qkv_tokenizer_open(str(path).encode(), C.byref(h), err, 512)
        if rc != QKV_OK:
            raise QkvError(rc, err.value.decode())
        self.h = h

    def decode(self, ids, skip_special: bool = True) -> bytes:
        ids = _i32(ids)
        n = C.c_size_t(0)
        buf = C.create_string_buffer(max(16 * len(ids), 64))
        rc = lib.qkv_tokenizer_decode(self.h, _ptr(ids, C.c_int32), len(ids), int(skip_special), buf, len(buf),
                                      C.byref(n))
        if rc == QKV_ERR_CAPACITY:
            buf = C.create_string_buffer(n.value)
            rc = lib.qkv_tokenizer_decode(self.h, _ptr(ids, C.c_int32), len(ids), int(skip_special), buf,
                                          len(buf), C.byref(n))
        if rc != QKV_OK:
            raise QkvError(rc, "tokenizer decode failed")
        return buf.raw[:n.value]

    def _ids(self, call):
        n = C.c_size_t(0)
        out = np.zeros(256, np.int32)
        rc = call(out, n)
        if rc == QKV_ERR_CAPACITY:
            out = np.zeros(n.value, np.int32)
            rc = call(out, n)
        if rc != QKV_OK:
            raise QkvError(rc, "tokenizer encode failed")
        return out[:n.value].copy()

    def encode(self, text, add_eos: bool = False) -> np.ndarray:
        """Ids of text (str or bytes), as qwenasr_tokenizer_encode."""
        b = text.encode() if isinstance(text, str) else bytes(text)
        return self._ids(lambda out, n: lib.qkv_tokenizer_encode(self.h, b, len(b), int(add_eos),
                                                                 _ptr(out, C.c_int32), len(out), C.byref(n)))

    def asr_prompt_ids(self, audio_tokens: int, system_text: str = "", language: str = "") -> np.ndarray:
        """Ids of the ASR prompt (qwenasr_build_asr_prompt, then encoded)."""
        return self._ids(lambda out, n: lib.qkv_asr_prompt_ids(self.h, int(audio_tokens), system_text.encode(),
                                                               language.encode(), _ptr(out, C.c_int32), len(out),
                                                               C.byref(n)))

    def close(self):
        if self.h:
            lib.qkv_tokenizer_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def gguf_tensor(path, name: str, want_data: bool = True):
    """(ne[:n_dims], ggml_type, raw bytes) of one tensor via the native GGUF reader."""
    ne = (C.c_int64 * 4)()
    nd, ty = C.c_int32(), C.c_int32()
    err = C.create_string_buffer(512)
    rc = lib.qkv_gguf_tensor(str(path).encode(), name.encode(), ne, C.byref(nd), C.byref(ty), None, 0, err, 512)
    if rc != QKV_OK:
        raise QkvError(rc, err.value.decode())
    dims = [ne[i] for i in range(nd.value)]
    data = None
    if want_data:
        es = {0: 4, 1: 2, 24: 1, 30: 2}.get(ty.value, 0)
        nbytes = int(np.prod(dims)) * es
        buf = np.zeros(nbytes, np.uint8)
        rc = lib.qkv_gguf_tensor(str(path).encode(), name.encode(), ne, C.byref(nd), C.byref(ty),
                                 buf.ctypes.data, nbytes, err, 512)
        if rc != QKV_OK:
            raise QkvError(rc, err.value.decode())
        data = buf
    return dims, ty.value, data


class Decoder:
    """One handle = one GPU: weights (or QK-norm weights only), paged KV pool, streams."""

    def __init__(self, handle: int):
        self.h = C.c_void_p(handle)
        self.cfg = None

    @classmethod
    def from_gguf(cls, path, rt: RuntimeConfig, cfg: dict | None = None) -> "Decoder":
        out = C.c_void_p()
        err = C.create_string_buffer(1024)
        mc = C.byref(model_config(cfg)) if cfg else None
        rc = lib.qkv_create(str(path).encode(), mc, C.byref(rt), C.byref(out), err, 1024)
        if rc != QKV_OK:
            raise QkvError(rc, err.value.decode())
        d = cls(out.value)
        d.cfg = cfg or read_gguf_config(path)
        return d

    @classmethod
    def kv_only(cls, cfg: dict, rt: RuntimeConfig, q_norm_w: np.ndarray, k_norm_w: np.ndarray) -> "Decoder":
        out = C.c_void_p()
        err = C.create_string_buffer(1024)
        qn = np.ascontiguousarray(q_norm_w, np.float32)
        kn = np.ascontiguousarray(k_norm_w, np.float32)
        rc = lib.qkv_create_kv_only(C.byref(model_config(cfg)), C.byref(rt), _ptr(qn, C.c_float),
                                    _ptr(kn, C.c_float), C.byref(out), err, 1024)
        if rc != QKV_OK:
            raise QkvError(rc, err.value.decode())
        d = cls(out.value)
        d.cfg = cfg
        return d

    def close(self):
        if getattr(self, "h", None):
            lib.qkv_destroy(self.h)
            self.h = None

    def __del__(self):
        # A handle dropped without close() still returns its pool and weights.
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def _check(self, rc: int):
        if rc != QKV_OK:
            raise QkvError(rc, lib.qkv_last_error(self.h).decode())

    # ---- streams ----
    def open(self) -> int:
        s = C.c_int32()
        self._check(lib.qkv_stream_open(self.h, C.byref(s)))
        return s.value

    def close_stream(self, s: int):
        self._check(lib.qkv_stream_close(self.h, s))

    def length(self, s: int) -> int:
        t = C.c_int32()
        self._check(lib.qkv_stream_length(self.h, s, C.byref(t)))
        return t.value

    def pool_stats(self) -> tuple[int, int]:
        f, t = C.c_int64(), C.c_int64()
        self._check(lib.qkv_pool_stats(self.h, C.byref(f), C.byref(t)))
        return f.value, t.value

    def compact(self) -> int:
        m = C.c_int64()
        self._check(lib.qkv_compact(self.h, C.byref(m)))
        return m.value

    def pages(self, s: int) -> np.ndarray:
        n = C.c_int32()
        buf = np.zeros(4096, np.int32)
        self._check(lib.qkv_stream_pages(self.h, s, _ptr(buf, C.c_int32), len(buf), C.byref(n)))
        return buf[:n.value].copy()

    # ---- model level ----
    def prefill(self, streams, prompts: list[np.ndarray], want_logits=False):
        streams = _i32(streams)
        lens = _i32([p.shape[0] for p in prompts])
        # one block per stream (no concatenation); each must be C-contiguous f32
        blocks = [np.ascontiguousarray(p, np.float32) for p in prompts]
        ptrs = (C.c_void_p * max(len(blocks), 1))(*[b.ctypes.data for b in blocks])
        ids = np.zeros(len(streams), np.int32)
        logits = np.zeros((len(streams), self.cfg["vocab"]), np.float32) if want_logits else None
        self._check(lib.qkv_prefill_rows(self.h, len(streams), _ptr(streams, C.c_int32), _ptr(lens, C.c_int32),
                                         ptrs, _ptr(ids, C.c_int32),
                                         _ptr(logits, C.c_float) if want_logits else None))
        return (ids, logits) if want_logits else ids

    @staticmethod
    def _audio_table(audio, n):
        """(pointer table, per-prompt row counts, on_device, keep-alive) for a
        list of per-prompt audio blocks: numpy arrays (host) or torch CUDA
        tensors (device), None for a prompt without audio rows."""
        on_dev = any(a is not None and not isinstance(a, np.ndarray) for a in audio)
        keep, ptrs, counts = [], [], []
        for a in audio:
            if a is None:
                ptrs.append(None)
                counts.append(0)
            elif isinstance(a, np.ndarray):
                if on_dev:
                    raise ValueError("audio blocks must all be host arrays or all device tensors")
                b = np.ascontiguousarray(a, np.float32)
                keep.append(b)
                ptrs.append(b.ctypes.data)
                counts.append(b.shape[0])
            else:
                if not (a.is_cuda and a.is_contiguous() and str(a.dtype) == "torch.float32"):
                    raise ValueError("device audio blocks must be contiguous float32 CUDA tensors")
                ptrs.append(a.data_ptr())
                counts.append(a.shape[0])
        table = (C.c_void_p * max(n, 1))(*ptrs)
        return table, _i32(counts), on_dev, keep

    def audio_projector_width(self) -> int:
        """Width of the audio encoder rows the projector takes (0: the file has no projector)."""
        w = np.zeros(1, np.int32)
        self._check(lib.qkv_audio_projector_width(self.h, _ptr(w, C.c_int32)))
        return int(w[0])

    def audio_project(self, n: int, audio_ptr: int, out_ptr: int, stream=None):
        """Audio projector on the device (qkv_audio_project): n rows of width
        audio_projector_width() -> n decoder rows (device pointers, f32)."""
        self._check(lib.qkv_audio_project(self.h, n, audio_ptr, out_ptr, stream))

    def decoder_input(self, lens, ids, audio, audio_token_id: int, x_ptr: int, stream=None):
        """Prompt rows on the device from ids + audio rows (qkv_decoder_input): x_ptr receives sum(lens) x hidden f32."""
        lens = _i32(lens)
        ids = _i32(np.concatenate([np.asarray(i, np.int32) for i in ids]) if isinstance(ids, (list, tuple)) else ids)
        table, counts, on_dev, keep = self._audio_table(audio, len(lens))
        self._check(lib.qkv_decoder_input(self.h, len(lens), _ptr(lens, C.c_int32), _ptr(ids, C.c_int32), table,
                                          _ptr(counts, C.c_int32), int(on_dev), int(audio_token_id), x_ptr, stream))

    def prefill_ids(self, streams, ids, audio, audio_token_id: int, want_logits=False):
        """prefill with the prompt rows built on the device (qkv_prefill_ids):
        ids = one int array per prompt, audio = one block per prompt (host
        arrays or CUDA tensors, None for none)."""
        streams = _i32(streams)
        lens = _i32([len(i) for i in ids])
        flat = _i32(np.concatenate([np.asarray(i, np.int32) for i in ids]))
        table, counts, on_dev, keep = self._audio_table(audio, len(streams))
        out = np.zeros(len(streams), np.int32)
        logits = np.zeros((len(streams), self.cfg["vocab"]), np.float32) if want_logits else None
        self._check(lib.qkv_prefill_ids(self.h, len(streams), _ptr(streams, C.c_int32), _ptr(lens, C.c_int32),
                                        _ptr(flat, C.c_int32), table, _ptr(counts, C.c_int32), int(on_dev),
                                        int(audio_token_id), _ptr(out, C.c_int32),
                                        _ptr(logits, C.c_float) if want_logits else None))
        return (out, logits) if want_logits else out

    def decode_step(self, streams, in_ids=None, want_logits=False):
        streams = _i32(streams)
        ids = np.zeros(len(streams), np.int32)
        inp = _i32(in_ids) if in_ids is not None else None
        logits = np.zeros((len(streams), self.cfg["vocab"]), np.float32) if want_logits else None
        self._check(lib.qkv_decode_step(self.h, len(streams), _ptr(streams, C.c_int32),
                                        _ptr(inp, C.c_int32) if inp is not None else None, _ptr(ids, C.c_int32),
                                        _ptr(logits, C.c_float) if want_logits else None))
        return (ids, logits) if want_logits else ids

    def generate(self, prompt: np.ndarray, max_new_tokens: int, stop_ids=()):
        emb = np.ascontiguousarray(prompt, np.float32)
        stop = _i32(list(stop_ids) or [0])
        out = np.zeros(max(max_new_tokens, 1), np.int32)
        n, stopped = C.c_int32(), C.c_int32()
        self._check(lib.qkv_generate(self.h, _ptr(emb, C.c_float), emb.shape[0], max_new_tokens,
                                     _ptr(stop, C.c_int32), len(stop_ids), _ptr(out, C.c_int32), C.byref(n),
                                     C.byref(stopped)))
        return out[:n.value].copy(), bool(stopped.value)

    def layer_forward(self, layer: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros_like(x)
        self._check(lib.qkv_layer_forward(self.h, layer, x.shape[0], _ptr(x, C.c_float), _ptr(out, C.c_float)))
        return out

    # ---- operator level (device pointers, ints) ----
    def kv_append(self, layer, n, slots_ptr, pos_ptr, qkv_ptr, q_out_ptr, stream=None):
        self._check(lib.qkv_kv_append(self.h, layer, n, slots_ptr, pos_ptr, qkv_ptr, q_out_ptr, stream))

    def kv_attend(self, layer, n, slots_ptr, lens_ptr, q_ptr, out_ptr, stream=None):
        self._check(lib.qkv_kv_attend(self.h, layer, n, slots_ptr, lens_ptr, q_ptr, out_ptr, stream))

    def prefill_attend(self, layer, streams, lens, q_ptr: int, out_ptr: int, stream=None):
        """Causal attention of each stream's last lens[i] positions (device q/out pointers)."""
        streams, lens = _i32(streams), _i32(lens)
        self._check(lib.qkv_prefill_attend(self.h, layer, len(streams), _ptr(streams, C.c_int32),
                                           _ptr(lens, C.c_int32), q_ptr, out_ptr, stream))

    def prefill_attend_q16(self, layer, streams, lens, q16_ptr: int, out_ptr: int, stream=None):
        """prefill_attend with q16 = bf16 (f16 for an e4m3 cache) of q * log2(e) / sqrt(128)."""
        streams, lens = _i32(streams), _i32(lens)
        self._check(lib.qkv_prefill_attend_q16(self.h, layer, len(streams), _ptr(streams, C.c_int32),
                                               _ptr(lens, C.c_int32), q16_ptr, out_ptr, stream))

    def kv_step(self, streams, qkv_ptr: int, out_ptr: int, stream=None):
        streams = _i32(streams)
        self._check(lib.qkv_kv_step(self.h, len(streams), _ptr(streams, C.c_int32), qkv_ptr, out_ptr, stream))

    def kv_step_host(self, streams, qkv_host_ptr: int, out_host_ptr: int):
        streams = _i32(streams)
        self._check(lib.qkv_kv_step_host(self.h, len(streams), _ptr(streams, C.c_int32), qkv_host_ptr, out_host_ptr))

    def extend(self, s: int, tokens: int):
        self._check(lib.qkv_stream_extend(self.h, s, tokens))

    def fill_random(self, seed: int):
        self._check(lib.qkv_fill_random(self.h, seed))

    def gather(self, layer: int, s: int, kv_dtype: int):
        n = self.length(s)
        dt = {F32: np.float32, BF16: np.uint16, FP8: np.uint8, E4I8: np.uint8}[kv_dtype]
        k = np.zeros((n, 1024), dt)
        v = np.zeros((n, 1024), dt)
        npg = (n + 15) // 16
        scales = np.zeros((npg, 2, 8, 16), np.float32)   # 8-bit caches: one scale per (page, K|V, head, token)
        self._check(lib.qkv_gather(self.h, layer, s, k.ctypes.data, v.ctypes.data,
                                   _ptr(scales, C.c_float) if kv_dtype in (FP8, E4I8) else None))
        return (k, v, scales) if kv_dtype in (FP8, E4I8) else (k, v)

    def sync(self):
        self._check(lib.qkv_sync(self.h))

    def launches(self) -> int:
        n = C.c_int64()
        self._check(lib.qkv_last_launches(self.h, C.byref(n)))
        return n.value


class Pager:
    """Host-only page allocator (the one every handle uses)."""

    def __init__(self, n_pages, page_tokens=16, max_streams=8, max_pages_per_stream=64, seed=0):
        self.p = C.c_void_p(lib.qkv_pager_create(n_pages, page_tokens, max_streams, max_pages_per_stream, seed))
        if not self.p:
            raise QkvError(1, "bad pager configuration")

    def __del__(self):
        if getattr(self, "p", None):
            lib.qkv_pager_destroy(self.p)
            self.p = None

    def open(self) -> int:
        s = C.c_int32()
        rc = lib.qkv_pager_open(self.p, C.byref(s))
        if rc:
            raise QkvError(rc, "open")
        return s.value

    def close(self, s):
        rc = lib.qkv_pager_close(self.p, s)
        if rc:
            raise QkvError(rc, "close")

    def append(self, s, tokens) -> int:
        n = C.c_int32()
        rc = lib.qkv_pager_append(self.p, s, tokens, C.byref(n))
        if rc:
            raise QkvError(rc, "append")
        return n.value

    def length(self, s) -> int:
        t = C.c_int32()
        rc = lib.qkv_pager_length(self.p, s, C.byref(t))
        if rc:
            raise QkvError(rc, "length")
        return t.value

    def pages(self, s) -> list[int]:
        buf = np.zeros(1 << 16, np.int32)
        n = C.c_int32()
        rc = lib.qkv_pager_pages(self.p, s, _ptr(buf, C.c_int32), len(buf), C.byref(n))
        if rc:
            raise QkvError(rc, "pages")
        return buf[:n.value].tolist()

    def free_pages(self) -> int:
        return lib.qkv_pager_free_pages(self.p)

    def compact(self) -> list[tuple[int, int]]:
        cap = 1 << 16
        src, dst = np.zeros(cap, np.int32), np.zeros(cap, np.int32)
        n = C.c_int64()
        lib.qkv_pager_compact(self.p, _ptr(src, C.c_int32), _ptr(dst, C.c_int32), cap, C.byref(n))
        return list(zip(src[:n.value].tolist(), dst[:n.value].tolist()))

    def check(self) -> int:
        return lib.qkv_pager_check(self.p)
