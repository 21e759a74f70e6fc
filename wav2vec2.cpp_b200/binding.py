"""ctypes binding of libwav2vec2_b200.so (public C API + kernel C-ABI).

`Model` mirrors the reference API (wav2vec2_init / transcribe / free) plus the
batched and device entry points of include/wav2vec2_b200.h.  `kernels`
exposes the raw launchers of include/w2v_kernels.h for the per-kernel parity
tests; they take device pointers (ints), e.g. torch tensors' data_ptr().
There is no fallback: if the library is missing, loading raises.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libwav2vec2_b200.so"

_vp, _i, _ll, _f = C.c_void_p, C.c_int, C.c_longlong, C.c_float


class Word(C.Structure):
    _fields_ = [("text", C.c_char_p), ("t_start", C.c_float), ("t_end", C.c_float)]


class Result(C.Structure):
    _fields_ = [("transcript", C.c_char_p), ("n_frames", C.c_int), ("words", C.POINTER(Word)),
                ("n_words", C.c_int)]


class Params(C.Structure):
    _fields_ = [("n_threads", C.c_int), ("beam_size", C.c_int), ("verbose", C.c_bool),
                ("word_timestamps", C.c_bool)]


# exported symbols and their ctypes signatures (restype, argtypes)
SIGNATURES = {
    "wav2vec2_default_params": (Params, []),
    "wav2vec2_init": (_vp, [C.c_char_p]),
    "wav2vec2_free": (None, [_vp]),
    "wav2vec2_transcribe": (C.POINTER(Result), [_vp, Params, _vp, _i]),
    "wav2vec2_result_free": (None, [C.POINTER(Result)]),
    "wav2vec2_b200_last_error": (C.c_char_p, []),
    "wav2vec2_b200_init": (_vp, [C.c_char_p, _vp, _i, _i]),
    "wav2vec2_b200_n_devices": (_i, [_vp]),
    "wav2vec2_b200_model_info": (_i, [_vp, _vp]),
    "wav2vec2_transcribe_batch": (_i, [_vp, Params, _vp, _vp, _i, _vp]),
    "wav2vec2_b200_n_frames": (_i, [_vp, _i]),
    "wav2vec2_b200_logits": (_i, [_vp, _vp, _vp, _i, _vp, _vp]),
    "wav2vec2_b200_forward_device": (_i, [_vp, _vp, _vp, _i, _vp]),
    "wav2vec2_b200_device_outputs": (_i, [_vp, _vp, _vp, _vp, _vp]),
    "wav2vec2_b200_debug_stages": (_i, [_vp, _vp, _i, _vp, _vp, _vp]),
    "wav2vec2_b200_profile": (_i, [_vp, _i]),
    "wav2vec2_b200_profile_read": (_i, [_vp, _vp, _vp, _vp, _vp, _i]),
    "wav2vec2_b200_launches_per_forward": (_ll, [_vp]),
    "wav2vec2_b200_device_stats": (_i, [_vp, _i, _vp, _vp, _vp, _i]),
    "wav2vec2_b200_ctc_beam_search": (_i, [_vp, _i, _i, _i, _i, _vp, _i]),
    "wav2vec2_b200_linear_weight_bytes": (_ll, [_vp]),
    "wav2vec2_b200_load_wav": (_i, [C.c_char_p, _i, _vp, _vp]),
    "wav2vec2_b200_free_samples": (None, [_vp]),
    # kernel layer (include/w2v_kernels.h)
    "w2v_gemm_f16": (_i, [_vp, _ll, _i, _i, _ll, _ll, _ll, _ll, _vp, _i, _vp, _ll, _ll, _i, _vp, _vp, _ll, _i,
                          _i, _vp, _vp]),
    "w2v_gemm_f16_ln_resid": (_i, [_vp, _ll, _i, _i, _ll, _ll, _ll, _ll, _vp, _i, _vp, _ll, _ll, _i, _vp, _vp,
                                   _ll, _vp, _vp, _vp, _i, _vp, _vp]),
    "w2v_gemm_q": (_i, [_vp, _ll, _ll, _vp, _vp, _ll, _i, _i, _vp, _ll, _vp, _vp, _ll, _i, _i, _vp, _vp]),
    "w2v_gemm_q_ln_resid": (_i, [_vp, _ll, _ll, _vp, _vp, _ll, _i, _i, _vp, _ll, _vp, _vp, _ll, _vp, _vp, _vp, _i,
                                 _vp, _vp]),
    "w2v_repack_q": (_i, [_vp, _i, _ll, _ll, _vp, _vp, _ll, _vp]),
    "w2v_layer_norm_stats": (_i, [_vp, _ll, _i, _vp, _vp, _vp, _vp, _vp]),
    "w2v_selftest_wait_timeout": (_i, [_vp, _i, _vp]),
    "w2v_dequant_f16": (_i, [_vp, _i, _ll, _ll, _vp, _vp]),
    "w2v_wave_stats": (_i, [_vp, _vp, _vp, _i, _vp, _vp]),
    "w2v_conv0": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _ll, _i,
                       _vp, _vp]),
    "w2v_conv0_noalloc": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp, _ll, _i,
                               _vp, _vp]),
    "w2v_layer_norm": (_i, [_vp, _i, _ll, _ll, _vp, _vp, _i, _i, _i, _vp, _vp, _i, _vp, _vp, _ll, _vp]),
    "w2v_pos_conv": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp, _i, _vp, _vp]),
    "w2v_attention": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _ll, _vp, _vp]),
    "w2v_ctc_greedy": (_i, [_vp, _vp, _vp, _i, _i, _vp, _vp, _vp, _i, _vp]),
}

_lib = None


def build(jobs: int = 8) -> None:
    subprocess.run(["make", "-s", "-C", str(PKG), f"-j{jobs}"], check=True)


def lib(path: str | Path | None = None):
    """Load the engine library (raises if it is missing: no fallback path)."""
    global _lib
    if _lib is None:
        p = Path(path) if path else LIB_PATH
        if not p.exists():
            raise FileNotFoundError(f"{p} not built (make -C {PKG})")
        L = C.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return (lib().wav2vec2_b200_last_error() or b"").decode()


def _ptr_array(arrs):
    return (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])


class EngineError(RuntimeError):
    pass


def ctc_beam_search(logits: np.ndarray, blank: int = 0, beam_width: int = 5) -> list[int]:
    """Prefix beam search on host logits [T, V] (wav2vec2_b200_ctc_beam_search)."""
    lg = np.ascontiguousarray(logits, np.float32)
    T, V = lg.shape
    out = np.zeros(max(T, 1), np.int32)
    n = lib().wav2vec2_b200_ctc_beam_search(lg.ctypes.data, T, V, blank, beam_width, out.ctypes.data, out.size)
    if n < 0:
        raise EngineError(last_error())
    return out[:n].tolist()


def load_wav(path: str | Path, target_sr: int = 16000) -> np.ndarray:
    """Mono float32 samples at target_sr from a WAV file
    (wav2vec2_b200_load_wav; the reference CLI's decoding)."""
    p = C.c_void_p()
    n = C.c_int()
    rc = lib().wav2vec2_b200_load_wav(str(path).encode(), target_sr, C.byref(p), C.byref(n))
    if rc != 0:
        raise EngineError(last_error())
    try:
        if n.value == 0:
            return np.zeros(0, np.float32)
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_float)), shape=(n.value,)).copy()
    finally:
        lib().wav2vec2_b200_free_samples(p)


class Model:
    """A loaded model (one replica per device)."""

    def __init__(self, path, devices=None, max_batch: int = 0):
        L = lib()
        if devices is None:
            self.h = L.wav2vec2_b200_init(str(path).encode(), None, 1, max_batch)
        else:
            devs = (C.c_int * len(devices))(*devices)
            self.h = L.wav2vec2_b200_init(str(path).encode(), C.cast(devs, _vp), len(devices), max_batch)
        if not self.h:
            raise EngineError(last_error())
        info = (C.c_int * 8)()
        L.wav2vec2_b200_model_info(self.h, C.cast(info, _vp))
        self.cfg = dict(zip(["conv_dim", "hidden", "n_layers", "n_heads", "ffn", "vocab", "pad_id", "stable"],
                            list(info)))

    def close(self):
        if getattr(self, "h", None):
            lib().wav2vec2_free(self.h)
            self.h = None

    __del__ = close

    def n_frames(self, n_samples: int) -> int:
        return lib().wav2vec2_b200_n_frames(self.h, int(n_samples))

    def logits(self, audios) -> list[np.ndarray]:
        audios = [np.ascontiguousarray(a, np.float32) for a in audios]
        n = (C.c_int * len(audios))(*[len(a) for a in audios])
        T = [self.n_frames(len(a)) for a in audios]
        V = self.cfg["vocab"]
        out = np.zeros((max(sum(T), 1), V), np.float32)
        nf = (C.c_int * len(audios))()
        rc = lib().wav2vec2_b200_logits(self.h, C.cast(_ptr_array(audios), _vp), C.cast(n, _vp), len(audios),
                                        out.ctypes.data, C.cast(nf, _vp))
        if rc:
            raise EngineError(last_error())
        res, o = [], 0
        for t in T:
            res.append(out[o:o + t].copy())
            o += t
        return res

    def transcribe_batch(self, audios, beam_size: int = 1, word_timestamps: bool = False, n_threads: int = 4):
        audios = [np.ascontiguousarray(a, np.float32) for a in audios]
        p = lib().wav2vec2_default_params()
        p.beam_size, p.word_timestamps, p.n_threads = beam_size, word_timestamps, n_threads
        n = (C.c_int * len(audios))(*[len(a) for a in audios])
        res = (C.POINTER(Result) * len(audios))()
        rc = lib().wav2vec2_transcribe_batch(self.h, p, C.cast(_ptr_array(audios), _vp), C.cast(n, _vp),
                                             len(audios), C.cast(res, _vp))
        if rc:
            raise EngineError(last_error())
        free = lib().wav2vec2_result_free
        out = []
        for r in res:
            c = r.contents
            nw = c.n_words
            words = [(w.text.decode(), w.t_start, w.t_end) for w in c.words[:nw]] if nw else []
            out.append({"text": c.transcript.decode(), "n_frames": c.n_frames, "words": words})
            free(r)
        return out

    def transcribe(self, audio, beam_size: int = 1, word_timestamps: bool = False) -> dict:
        a = np.ascontiguousarray(audio, np.float32)
        p = lib().wav2vec2_default_params()
        p.beam_size, p.word_timestamps = beam_size, word_timestamps
        r = lib().wav2vec2_transcribe(self.h, p, a.ctypes.data, len(a))
        if not r:
            raise EngineError(last_error())
        c = r.contents
        words = [(c.words[i].text.decode(), c.words[i].t_start, c.words[i].t_end) for i in range(c.n_words)]
        out = {"text": c.transcript.decode(), "n_frames": c.n_frames, "words": words}
        lib().wav2vec2_result_free(r)
        return out

    def debug_stages(self, audio):
        a = np.ascontiguousarray(audio, np.float32)
        T = self.n_frames(len(a))
        c = self.cfg
        feat = np.zeros((T, c["conv_dim"]), np.float32)
        stages = np.zeros((c["n_layers"] + 2, T, c["hidden"]), np.float32)
        logits = np.zeros((T, c["vocab"]), np.float32)
        rc = lib().wav2vec2_b200_debug_stages(self.h, a.ctypes.data, len(a), feat.ctypes.data, stages.ctypes.data,
                                              logits.ctypes.data)
        if rc:
            raise EngineError(last_error())
        return feat, stages, logits

    def forward_device(self, d_audio: int, n_samples, stream: int = 0) -> None:
        n = (C.c_int * len(n_samples))(*[int(x) for x in n_samples])
        rc = lib().wav2vec2_b200_forward_device(self.h, d_audio, C.cast(n, _vp), len(n_samples), stream or None)
        if rc:
            raise EngineError(last_error())

    def profile(self, enable: bool) -> None:
        lib().wav2vec2_b200_profile(self.h, 1 if enable else 0)

    def profile_read(self) -> dict:
        n = 16
        names = (C.c_char_p * n)()
        ms = (C.c_double * n)()
        nl = (C.c_longlong * n)()
        fl = (C.c_double * n)()
        k = lib().wav2vec2_b200_profile_read(self.h, C.cast(names, _vp), C.cast(ms, _vp), C.cast(nl, _vp),
                                             C.cast(fl, _vp), n)
        return {names[i].decode(): {"ms": ms[i], "launches": nl[i], "flops": fl[i]} for i in range(k)}

    def device_stats(self, reset: bool = False) -> list[dict]:
        """Per device: busy_ms (device time of its host batches), batches, samples."""
        n = 64
        ms = (C.c_double * n)()
        nb = (C.c_longlong * n)()
        ns = (C.c_longlong * n)()
        k = lib().wav2vec2_b200_device_stats(self.h, 1 if reset else 0, C.cast(ms, _vp), C.cast(nb, _vp),
                                             C.cast(ns, _vp), n)
        return [{"busy_ms": ms[i], "batches": nb[i], "samples": ns[i]} for i in range(max(k, 0))]

    def linear_weight_bytes(self) -> int:
        return int(lib().wav2vec2_b200_linear_weight_bytes(self.h))

    def launches_per_forward(self) -> int:
        return int(lib().wav2vec2_b200_launches_per_forward(self.h))

    def device_outputs(self):
        lg, sp, ns, M = _vp(), _vp(), _vp(), C.c_longlong()
        lib().wav2vec2_b200_device_outputs(self.h, C.byref(lg), C.byref(sp), C.byref(ns), C.byref(M))
        return lg.value, sp.value, ns.value, M.value


class kernels:
    """Thin wrappers over the C-ABI launchers (device pointers as ints)."""

    @staticmethod
    def check(rc, name):
        if rc != 0:
            raise EngineError(f"{name} returned status {rc}")

    @staticmethod
    def gemm(A, a_cin, a_taps, a_stride, a_row_stride, a_rows_in, a_batches, a_batch_stride, B, N, Cp, ldc,
             c_batch_rows, m_valid, bias=0, resid=0, ldr=0, epilogue=0, block_n=0, err=0, stream=0):
        kernels.check(lib().w2v_gemm_f16(A, a_cin, a_taps, a_stride, a_row_stride, a_rows_in, a_batches,
                                         a_batch_stride, B, N, Cp, ldc, c_batch_rows, m_valid, bias or None,
                                         resid or None, ldr, epilogue, block_n, err or None, stream or None),
                      "w2v_gemm_f16")

    @staticmethod
    def gemm_ln_resid(A, a_cin, a_taps, a_stride, a_row_stride, a_rows_in, a_batches, a_batch_stride, B, N, Cp,
                      ldc, c_batch_rows, m_valid, bias, resid, ldr, ln_stats, ln_w, ln_b, block_n=0, err=0,
                      stream=0):
        kernels.check(lib().w2v_gemm_f16_ln_resid(A, a_cin, a_taps, a_stride, a_row_stride, a_rows_in, a_batches,
                                                  a_batch_stride, B, N, Cp, ldc, c_batch_rows, m_valid,
                                                  bias or None, resid, ldr, ln_stats, ln_w, ln_b, block_n,
                                                  err or None, stream or None), "w2v_gemm_f16_ln_resid")

    @staticmethod
    def gemm_q(A, K, M, Bq, Bs, ld_s, gguf_type, N, Cp, ldc, bias=0, resid=0, ldr=0, epilogue=0, block_n=0, err=0,
               stream=0):
        kernels.check(lib().w2v_gemm_q(A, K, M, Bq, Bs, ld_s, gguf_type, N, Cp, ldc, bias or None, resid or None,
                                       ldr, epilogue, block_n, err or None, stream or None), "w2v_gemm_q")

    @staticmethod
    def gemm_q_ln_resid(A, K, M, Bq, Bs, ld_s, gguf_type, N, Cp, ldc, bias, resid, ldr, ln_stats, ln_w, ln_b,
                        block_n=0, err=0, stream=0):
        kernels.check(lib().w2v_gemm_q_ln_resid(A, K, M, Bq, Bs, ld_s, gguf_type, N, Cp, ldc, bias or None, resid,
                                                ldr, ln_stats, ln_w, ln_b, block_n, err or None, stream or None),
                      "w2v_gemm_q_ln_resid")

    @staticmethod
    def repack_q(raw, gguf_type, n_rows, K, codes, scales, ld_s, stream=0):
        kernels.check(lib().w2v_repack_q(raw, gguf_type, n_rows, K, codes, scales, ld_s, stream or None),
                      "w2v_repack_q")

    @staticmethod
    def layer_norm_stats(inp, M, D, w, b, out16, stats, stream=0):
        kernels.check(lib().w2v_layer_norm_stats(inp, M, D, w, b, out16, stats, stream or None),
                      "w2v_layer_norm_stats")

    @staticmethod
    def dequant(raw, gtype, n_rows, K, out, stream=0):
        kernels.check(lib().w2v_dequant_f16(raw, gtype, n_rows, K, out, stream or None), "w2v_dequant_f16")

    @staticmethod
    def wave_stats(audio, off, length, n_utt, stats, stream=0):
        kernels.check(lib().w2v_wave_stats(audio, off, length, n_utt, stats, stream or None), "w2v_wave_stats")

    @staticmethod
    def conv0(audio, off, length, frames, n_utt, stats, w0, b0, Cc, k0, s0, norm, gw, gb, gn, out, rows_max,
              max_frames, err=0, stream=0):
        kernels.check(lib().w2v_conv0(audio, off, length, frames, n_utt, stats, w0, b0 or None, Cc, k0, s0, norm,
                                      gw or None, gb or None, gn or None, out, rows_max, max_frames, err or None,
                                      stream or None), "w2v_conv0")

    @staticmethod
    def layer_norm(inp, in_f16, ld_in, in_batch_rows, rows, out_off, n_batch, n_rows, D, w, b, gelu, out32, out16,
                   ld_out, stream=0):
        kernels.check(lib().w2v_layer_norm(inp, in_f16, ld_in, in_batch_rows, rows or None, out_off or None,
                                           n_batch, n_rows, D, w, b, gelu, out32 or None, out16 or None, ld_out,
                                           stream or None), "w2v_layer_norm")

    @staticmethod
    def pos_conv(x, xin, off, T, n_utt, H, Kp, G, wt, bias, max_T, err=0, stream=0):
        kernels.check(lib().w2v_pos_conv(x, xin, off, T, n_utt, H, Kp, G, wt, bias, max_T, err or None,
                                         stream or None), "w2v_pos_conv")

    @staticmethod
    def attention(qkv, out, off, T, n_utt, H, n_heads, max_T, M, err=0, stream=0):
        kernels.check(lib().w2v_attention(qkv, out, off, T, n_utt, H, n_heads, max_T, M, err or None,
                                          stream or None), "w2v_attention")

    @staticmethod
    def ctc_greedy(logits, off, T, n_utt, V, ids, spans, n_spans, max_T, stream=0):
        kernels.check(lib().w2v_ctc_greedy(logits, off, T, n_utt, V, ids, spans, n_spans, max_T, stream or None),
                      "w2v_ctc_greedy")
