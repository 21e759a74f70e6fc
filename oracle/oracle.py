"""ctypes access to the oracles -- TEST INFRASTRUCTURE ONLY.

`Oracle` wraps liboracle.so, this repo's C restatement of the reference
forward pass (oracle/w2v_oracle.c).  `RefOracle` wraps _ref/libw2v_ref.so, the
reference's own unmodified sources built against the oracle's ggml-API shim
(oracle/Makefile `ref`), when that build exists.  Only tests, the smoke check
and the benchmark's CPU-baseline leg use this module; the engine never does.
"""
from __future__ import annotations

import contextlib
import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIB = ORACLE_DIR / "liboracle.so"
REF_LIB = ORACLE_DIR / "_ref" / "libw2v_ref.so"
REF_CLI = ORACLE_DIR / "_ref" / "wav2vec2-cli"
REF_SRC = Path(os.environ.get("W2V_REFERENCE", "/root/reference"))

EXACT, GGML = 0, 1
_vp = ctypes.c_void_p


def _p(a: np.ndarray):
    return a.ctypes.data_as(_vp)


def build(with_ref: bool = True) -> None:
    """Build liboracle.so and, when the reference checkout is present, _ref/."""
    subprocess.run(["make", "-s", "-C", str(ORACLE_DIR), "all"], check=True)
    if with_ref and REF_SRC.is_dir():
        subprocess.run(["make", "-s", "-C", str(ORACLE_DIR), "ref", f"REF={REF_SRC}"], check=True)


def ref_available() -> bool:
    return REF_LIB.exists()


@contextlib.contextmanager
def linear_mode(mode: int):
    """Select the ggml shim's matmul mode for RefOracle calls in this block."""
    old = os.environ.get("W2V_ORACLE_LINEAR")
    os.environ["W2V_ORACLE_LINEAR"] = "exact" if mode == EXACT else "ggml"
    try:
        yield
    finally:
        if old is None:
            os.environ.pop("W2V_ORACLE_LINEAR", None)
        else:
            os.environ["W2V_ORACLE_LINEAR"] = old


class _Base:
    def info(self) -> dict:
        out = (ctypes.c_int * 10)()
        self._info(self.h, out)
        keys = ["conv_dim", "hidden", "n_layers", "n_heads", "ffn", "vocab", "pad_id",
                "stable", "n_conv", "group_norm"]
        return dict(zip(keys, list(out)))


class Oracle(_Base):
    """This repo's C restatement of the reference forward pass."""
    _lib = None

    @classmethod
    def lib(cls):
        if cls._lib is None:
            if not LIB.exists():
                build(with_ref=False)
            L = ctypes.CDLL(str(LIB))
            L.wvo_load.restype = _vp
            L.wvo_load.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int]
            L.wvo_free.argtypes = [_vp]
            L.wvo_info.argtypes = [_vp, _vp]
            L.wvo_features.argtypes = [_vp, _vp, ctypes.c_int, _vp, ctypes.c_long]
            L.wvo_encode_stages.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp]
            L.wvo_logits.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_long]
            L.wvo_lm_head.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp]
            L.wvo_linear.argtypes = [_vp, ctypes.c_char_p, _vp, ctypes.c_int, ctypes.c_int, _vp]
            L.wvo_weight.restype = ctypes.c_long
            L.wvo_weight.argtypes = [_vp, ctypes.c_char_p, _vp, ctypes.c_long]
            L.wvo_gelu.restype = ctypes.c_float
            L.wvo_gelu.argtypes = [ctypes.c_float]
            L.wvo_layer_norm.argtypes = [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int]
            L.wvo_group_norm.argtypes = [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int]
            L.wvo_softmax.argtypes = [_vp, ctypes.c_int]
            L.wvo_conv1d.argtypes = [_vp, _vp, _vp] + [ctypes.c_int] * 7 + [_vp]
            L.wvo_ctc_greedy_spans.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int]
            L.wvo_quantize_q8_0_row.argtypes = [_vp, ctypes.c_int, _vp]
            cls._lib = L
        return cls._lib

    def __init__(self, path):
        L = self.lib()
        err = ctypes.create_string_buffer(256)
        self.h = L.wvo_load(str(path).encode(), err, 256)
        if not self.h:
            raise RuntimeError(err.value.decode())
        self._info = L.wvo_info
        self.cfg = self.info()

    def __del__(self):
        if getattr(self, "h", None):
            self.lib().wvo_free(self.h)
            self.h = None

    def features(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        cap = (len(x) // 320 + 8) * self.cfg["conv_dim"]
        out = np.zeros(cap, np.float32)
        T = self.lib().wvo_features(self.h, _p(x), len(x), _p(out), cap)
        if T < 0:
            raise RuntimeError("wvo_features failed")
        return out[: T * self.cfg["conv_dim"]].reshape(T, -1)

    def encode_stages(self, feat: np.ndarray, mode: int = EXACT) -> np.ndarray:
        feat = np.ascontiguousarray(feat, np.float32)
        T, H, L = feat.shape[0], self.cfg["hidden"], self.cfg["n_layers"]
        out = np.zeros((L + 2, T, H), np.float32)
        self.lib().wvo_encode_stages(self.h, _p(feat), T, mode, _p(out))
        return out

    def logits(self, x: np.ndarray, mode: int = EXACT) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        V = self.cfg["vocab"]
        cap = (len(x) // 320 + 8) * V
        out = np.zeros(cap, np.float32)
        T = self.lib().wvo_logits(self.h, _p(x), len(x), mode, _p(out), cap)
        if T < 0:
            raise RuntimeError("wvo_logits failed")
        return out[: T * V].reshape(T, V)

    def lm_head(self, enc: np.ndarray, mode: int = EXACT) -> np.ndarray:
        enc = np.ascontiguousarray(enc, np.float32)
        out = np.zeros((enc.shape[0], self.cfg["vocab"]), np.float32)
        self.lib().wvo_lm_head(self.h, _p(enc), enc.shape[0], mode, _p(out))
        return out

    def linear(self, name: str, x: np.ndarray, mode: int = EXACT) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        w = self.weight(name)
        y = np.zeros((x.shape[0], w.shape[0]), np.float32)
        if self.lib().wvo_linear(self.h, name.encode(), _p(x), x.shape[0], mode, _p(y)) != 0:
            raise KeyError(name)
        return y

    def weight(self, name: str) -> np.ndarray:
        """Dequantized fp32 weight [N, K] of a named linear."""
        c = self.cfg
        K = c["conv_dim"] if name == "feature_projection.projection" else (
            c["ffn"] if name.endswith("output_dense") else c["hidden"])
        cap = 64 << 20
        out = np.zeros(cap, np.float32)
        n = self.lib().wvo_weight(self.h, name.encode(), _p(out), cap)
        if n < 0:
            raise KeyError(name)
        return out[:n].reshape(-1, K).copy()


def gelu(x: float) -> float:
    return Oracle.lib().wvo_gelu(float(x))


def layer_norm(x, w, b):
    x = np.array(x, np.float32, copy=True, order="C")
    T, D = x.shape
    Oracle.lib().wvo_layer_norm(_p(x), _p(np.ascontiguousarray(w, np.float32)),
                                _p(np.ascontiguousarray(b, np.float32)), T, D)
    return x


def group_norm(x, w, b):
    x = np.array(x, np.float32, copy=True, order="C")
    T, C = x.shape
    Oracle.lib().wvo_group_norm(_p(x), _p(np.ascontiguousarray(w, np.float32)),
                                _p(np.ascontiguousarray(b, np.float32)), T, C)
    return x


def softmax(x):
    x = np.array(x, np.float32, copy=True)
    Oracle.lib().wvo_softmax(_p(x), x.size)
    return x


def conv1d(x, w, b, stride=1, pad=0, groups=1):
    """x [L, Cin], w [Cout, Cin/groups, K] -> [Lout, Cout]."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    L, Cin = x.shape
    Cout, _, K = w.shape
    Lout = (L + 2 * pad - K) // stride + 1
    out = np.zeros((max(Lout, 0), Cout), np.float32)
    bb = None if b is None else np.ascontiguousarray(b, np.float32)
    Oracle.lib().wvo_conv1d(_p(x), _p(w), None if bb is None else _p(bb), L, Cin, Cout, K,
                            stride, pad, groups, _p(out))
    return out


def greedy_spans(logits) -> list[tuple[int, int, int]]:
    lg = np.ascontiguousarray(logits, np.float32)
    T, V = lg.shape
    out = np.zeros(3 * max(T, 1), np.int32)
    n = Oracle.lib().wvo_ctc_greedy_spans(_p(lg), T, V, _p(out), max(T, 1))
    return [tuple(int(v) for v in out[3 * i: 3 * i + 3]) for i in range(n)]


def collapse(spans, blank: int = 0) -> list[int]:
    """Token ids of greedy spans with the blank removed (wav2vec2.cpp:500-502)."""
    return [s[0] for s in spans if s[0] != blank]


def quantize_q8_0_rows(x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    for i in range(x.shape[0]):
        Oracle.lib().wvo_quantize_q8_0_row(_p(x[i]), x.shape[1], _p(out[i]))
    return out


def ref_load_wav(path, target_sr: int = 16000, cap: int | None = None):
    """The reference CLI's WAV reader (examples/main/main.cpp:20-82), compiled
    from its source.  Returns float32 samples, or raises RuntimeError with the
    reference's message.  The reader loops forever on a file with no "data"
    chunk (its chunk loop seeks, which clears end-of-file), so callers must
    not pass one."""
    if cap is None:
        cap = max(1 << 16, 8 * os.path.getsize(path) * max(1, target_sr // 8000))
    out = np.empty(cap, np.float32)
    err = ctypes.create_string_buffer(512)
    n = RefOracle.lib().w2vref_load_wav(str(path).encode(), target_sr, out.ctypes.data, cap, err, 512)
    if n == -1:
        raise RuntimeError(err.value.decode())
    if n < 0:
        raise RuntimeError("capacity")
    return out[:n].copy()


class RefOracle(_Base):
    """The reference's own sources (oracle/_ref/libw2v_ref.so)."""
    _lib = None

    @classmethod
    def lib(cls):
        if cls._lib is None:
            L = ctypes.CDLL(str(REF_LIB))
            L.w2vref_init.restype = _vp
            L.w2vref_init.argtypes = [ctypes.c_char_p]
            L.w2vref_free.argtypes = [_vp]
            L.w2vref_info.argtypes = [_vp, _vp]
            L.w2vref_features.argtypes = [_vp, _vp, ctypes.c_int, _vp, ctypes.c_long]
            L.w2vref_encode.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp]
            L.w2vref_encode_stages.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp]
            L.w2vref_logits.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_long]
            L.w2vref_logits_from_features.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp]
            L.w2vref_transcribe.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_char_p, ctypes.c_int]
            L.w2vref_greedy_spans.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int]
            L.w2vref_beam_search.argtypes = [_vp] + [ctypes.c_int] * 4 + [_vp, ctypes.c_int]
            L.w2vref_gelu.restype = ctypes.c_float
            L.w2vref_gelu.argtypes = [ctypes.c_float]
            L.w2vref_conv1d.argtypes = [_vp, _vp, _vp] + [ctypes.c_int] * 7 + [_vp]
            L.w2vref_layer_norm.argtypes = [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int]
            L.w2vref_group_norm.argtypes = [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int]
            L.w2vref_softmax.argtypes = [_vp, ctypes.c_int]
            L.w2vref_load_wav.restype = ctypes.c_long
            L.w2vref_load_wav.argtypes = [ctypes.c_char_p, ctypes.c_int, _vp, ctypes.c_long, ctypes.c_char_p,
                                          ctypes.c_int]
            cls._lib = L
        return cls._lib

    def __init__(self, path, n_threads: int | None = None):
        self.h = self.lib().w2vref_init(str(path).encode())
        if not self.h:
            raise RuntimeError(f"reference failed to load {path}")
        self._info = self.lib().w2vref_info
        self.cfg = self.info()
        self.nt = n_threads or os.cpu_count() or 1

    def __del__(self):
        if getattr(self, "h", None):
            self.lib().w2vref_free(self.h)
            self.h = None

    def features(self, x):
        x = np.ascontiguousarray(x, np.float32)
        cap = (len(x) // 320 + 8) * self.cfg["conv_dim"]
        out = np.zeros(cap, np.float32)
        T = self.lib().w2vref_features(self.h, _p(x), len(x), _p(out), cap)
        return out[: T * self.cfg["conv_dim"]].reshape(T, -1)

    def encode_stages(self, feat, mode: int = GGML):
        feat = np.ascontiguousarray(feat, np.float32)
        T, H, L = feat.shape[0], self.cfg["hidden"], self.cfg["n_layers"]
        out = np.zeros((L + 2, T, H), np.float32)
        with linear_mode(mode):
            self.lib().w2vref_encode_stages(self.h, _p(feat), T, self.nt, _p(out))
        return out

    def logits(self, x, mode: int = GGML):
        x = np.ascontiguousarray(x, np.float32)
        V = self.cfg["vocab"]
        cap = (len(x) // 320 + 8) * V
        out = np.zeros(cap, np.float32)
        with linear_mode(mode):
            T = self.lib().w2vref_logits(self.h, _p(x), len(x), self.nt, _p(out), cap)
        if T < 0:
            raise RuntimeError("reference logits failed")
        return out[: T * V].reshape(T, V)

    def transcribe(self, x, beam: int = 1, mode: int = GGML) -> str:
        x = np.ascontiguousarray(x, np.float32)
        buf = ctypes.create_string_buffer(1 << 16)
        with linear_mode(mode):
            n = self.lib().w2vref_transcribe(self.h, _p(x), len(x), self.nt, beam, buf, 1 << 16)
        if n < 0:
            raise RuntimeError("reference transcribe failed")
        return buf.value.decode()


def ref_words_from_logits(ref: "RefOracle", logits):
    """The reference's own greedy post-processing of given logits
    (src/wav2vec2.cpp:497-503, 515-530): (transcript, [(word, t_start,
    t_end)]) with times in seconds."""
    lg = np.ascontiguousarray(logits, np.float32)
    T = lg.shape[0]
    text = ctypes.create_string_buffer(1 << 16)
    words = ctypes.create_string_buffer(1 << 16)
    times = np.zeros(2 * (T + 1), np.float32)
    L = RefOracle.lib()
    L.w2vref_words_from_logits.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_char_p, ctypes.c_int,
                                           ctypes.c_char_p, ctypes.c_int, _vp, ctypes.c_int]
    n = L.w2vref_words_from_logits(ref.h, _p(lg), T, text, 1 << 16, words, 1 << 16, _p(times), T + 1)
    if n < 0:
        raise RuntimeError("reference word spans failed")
    names = words.value.decode().split("\n") if n else []
    return text.value.decode(), [(w, float(times[2 * i]), float(times[2 * i + 1])) for i, w in enumerate(names)]


def ref_beam_search(logits, blank: int, beam: int) -> list[int]:
    lg = np.ascontiguousarray(logits, np.float32)
    T, V = lg.shape
    out = np.zeros(max(T, 1) + 1, np.int32)
    n = RefOracle.lib().w2vref_beam_search(_p(lg), T, V, blank, beam, _p(out), out.size)
    return [int(v) for v in out[:n]]
