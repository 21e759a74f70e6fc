"""Seeded synthetic wav2vec2 models (GGUF) and audio.

The model files follow the reference's GGUF layout exactly -- KV keys, tensor
names, shapes (innermost first), 32-byte alignment and the Q8_0 / Q4_0 block
encodings written by the reference converter (scripts/convert_to_gguf.py:42-97
for the wire helpers and quantisers, :104-129 for tensor routing, :160-226 for
tensor order, :241-309 for the file layout).  The code here is an independent
vectorised implementation of that format; byte equality with the reference
quantisers is checked by tests/test_synth.py.

Weights are random: N(0, 0.02) with a fixed seed, norm gains 1 and biases 0
(optionally jittered for tests so that bias / gain paths are exercised).
Audio is a seeded sum of five sinusoids (80-4000 Hz, random phases, amplitudes
U(0.1, 1)) plus N(0, 0.05^2) noise, peak-normalised to 0.9.
"""
from __future__ import annotations

import hashlib
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

GGUF_F32, GGUF_F16, GGUF_Q4_0, GGUF_Q8_0 = 0, 1, 2, 8
GGUF_MAGIC = 0x46554747
ALIGN = 32


@dataclass(frozen=True)
class Arch:
    name: str
    conv_dim: int = 512
    conv_kernel: tuple = (10, 3, 3, 3, 3, 2, 2)
    conv_stride: tuple = (5, 2, 2, 2, 2, 2, 2)
    feat_norm: str = "group"          # "group" (norm on conv 0 only) or "layer" (every conv)
    conv_bias: bool = False
    hidden: int = 768
    n_layers: int = 12
    n_heads: int = 12
    ffn: int = 3072
    pos_kernel: int = 128
    pos_groups: int = 16
    vocab: int = 32
    stable_layer_norm: bool = False   # pre-LN encoder when True


ARCHS = {
    # wav2vec2-base: GroupNorm extractor, post-LN encoder
    "base": Arch("base"),
    # wav2vec2-large / XLS-R-300M: LayerNorm extractor, stable (pre-LN) encoder
    "large": Arch("large", feat_norm="layer", conv_bias=True, hidden=1024, n_layers=24,
                  n_heads=16, ffn=4096, vocab=64, stable_layer_norm=True),
    # XLS-R-1B
    "xlsr1b": Arch("xlsr1b", feat_norm="layer", conv_bias=True, hidden=1280, n_layers=48,
                   n_heads=16, ffn=5120, vocab=64, stable_layer_norm=True),
    # Small architectures for fast parity tests (same operator set).
    "tiny": Arch("tiny", conv_dim=128, hidden=128, n_layers=2, n_heads=2, ffn=256,
                 pos_kernel=16, pos_groups=4, vocab=32),
    "tiny_pre": Arch("tiny_pre", conv_dim=128, feat_norm="layer", conv_bias=True, hidden=128,
                     n_layers=2, n_heads=2, ffn=256, pos_kernel=16, pos_groups=4, vocab=64,
                     stable_layer_norm=True),
    # XLS-R-1B's head dim 80 and positional-conv group width 80 at small size
    "tiny80": Arch("tiny80", conv_dim=128, feat_norm="layer", conv_bias=True, hidden=320,
                   n_layers=2, n_heads=4, ffn=640, pos_kernel=16, pos_groups=4, vocab=64,
                   stable_layer_norm=True),
}


def vocab_tokens(n: int) -> list[str]:
    """Synthetic CTC vocabulary: id 0 is the blank '<pad>', '|' is the word delimiter."""
    base = ["<pad>", "<s>", "</s>", "<unk>", "|"] + [chr(ord("A") + i) for i in range(26)] + ["'"]
    extra = [chr(ord("a") + i) for i in range(26)] + [str(i) for i in range(10)]
    toks = (base + extra)[:n]
    while len(toks) < n:
        toks.append(f"<x{len(toks)}>")
    return toks


# ── model tensors ────────────────────────────────────────────────────────────

def model_tensors(arch: Arch, seed: int = 0, std: float = 0.02,
                  bias_std: float = 0.0, gain_jitter: float = 0.0) -> dict[str, np.ndarray]:
    """Random-init weights in the reference converter's tensor order (name -> float32)."""
    rng = np.random.default_rng(seed)
    t: dict[str, np.ndarray] = {}

    def w(*shape):
        return (rng.standard_normal(shape, dtype=np.float64) * std).astype(np.float32)

    def bias(n):
        if bias_std > 0:
            return (rng.standard_normal(n) * bias_std).astype(np.float32)
        return np.zeros(n, np.float32)

    def gain(n):
        if gain_jitter > 0:
            return (1.0 + rng.standard_normal(n) * gain_jitter).astype(np.float32)
        return np.ones(n, np.float32)

    C, H, F = arch.conv_dim, arch.hidden, arch.ffn
    cin = 1
    for i, k in enumerate(arch.conv_kernel):
        p = f"feature_extractor.conv_layers.{i}"
        t[f"{p}.conv.weight"] = w(C, cin, k)
        if arch.conv_bias:
            t[f"{p}.conv.bias"] = bias(C)
        if arch.feat_norm == "layer" or i == 0:
            t[f"{p}.layer_norm.weight"] = gain(C)
            t[f"{p}.layer_norm.bias"] = bias(C)
        cin = C
    t["feature_projection.layer_norm.weight"] = gain(C)
    t["feature_projection.layer_norm.bias"] = bias(C)
    t["feature_projection.projection.weight"] = w(H, C)
    t["feature_projection.projection.bias"] = bias(H)
    t["encoder.pos_conv_embed.conv.weight"] = w(H, H // arch.pos_groups, arch.pos_kernel)
    t["encoder.pos_conv_embed.conv.bias"] = bias(H)
    t["encoder.layer_norm.weight"] = gain(H)
    t["encoder.layer_norm.bias"] = bias(H)
    for i in range(arch.n_layers):
        p = f"encoder.layers.{i}"
        for proj in ("q_proj", "k_proj", "v_proj", "out_proj"):
            t[f"{p}.attention.{proj}.weight"] = w(H, H)
            t[f"{p}.attention.{proj}.bias"] = bias(H)
        t[f"{p}.feed_forward.intermediate_dense.weight"] = w(F, H)
        t[f"{p}.feed_forward.intermediate_dense.bias"] = bias(F)
        t[f"{p}.feed_forward.output_dense.weight"] = w(H, F)
        t[f"{p}.feed_forward.output_dense.bias"] = bias(H)
        t[f"{p}.layer_norm.weight"] = gain(H)
        t[f"{p}.layer_norm.bias"] = bias(H)
        t[f"{p}.final_layer_norm.weight"] = gain(H)
        t[f"{p}.final_layer_norm.bias"] = bias(H)
    t["lm_head.weight"] = w(arch.vocab, H)
    t["lm_head.bias"] = bias(arch.vocab)
    return t


# ── quantisers (GGUF Q8_0 / Q4_0 block formats) ──────────────────────────────

def quantize_q8_0(arr: np.ndarray) -> bytes:
    """Q8_0 blocks of 32: fp16 scale d = amax/127, int8 q = round_half_even(x/d)."""
    flat = np.ascontiguousarray(arr, dtype=np.float32).reshape(-1)
    assert flat.size % 32 == 0
    blk = flat.reshape(-1, 32)
    amax = np.abs(blk).max(axis=1)
    scale = np.where(amax > 0, amax / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    iscale = (np.float32(1.0) / scale).astype(np.float32)
    q = np.clip(np.round(blk * iscale[:, None]), -128, 127).astype(np.int8)
    out = np.empty((blk.shape[0], 34), np.uint8)
    out[:, 0:2] = scale.astype("<f2").view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.tobytes()


def quantize_q4_0(arr: np.ndarray) -> bytes:
    """Q4_0 blocks of 32: fp16 scale d = amax/7, nibble q = round_half_even(x/d)+8 in [0,15];
    byte j holds element j (low nibble) and element j+16 (high nibble)."""
    flat = np.ascontiguousarray(arr, dtype=np.float32).reshape(-1)
    assert flat.size % 32 == 0
    blk = flat.reshape(-1, 32)
    amax = np.abs(blk).max(axis=1)
    scale = np.where(amax > 0, amax / np.float32(7.0), np.float32(1.0)).astype(np.float32)
    iscale = (np.float32(1.0) / scale).astype(np.float32)
    q = np.clip(np.round(blk * iscale[:, None]) + np.float32(8), 0, 15).astype(np.uint8)
    packed = q[:, :16] | (q[:, 16:] << 4)
    out = np.empty((blk.shape[0], 18), np.uint8)
    out[:, 0:2] = scale.astype("<f2").view(np.uint8).reshape(-1, 2)
    out[:, 2:] = packed
    return out.tobytes()


def dequantize(raw: bytes, gtype: int, shape: tuple) -> np.ndarray:
    """Inverse of the encoders above (fp32 result, reference-format semantics)."""
    n = int(np.prod(shape))
    b = np.frombuffer(raw, np.uint8)
    if gtype == GGUF_F32:
        return b.view("<f4")[:n].reshape(shape).copy()
    if gtype == GGUF_F16:
        return b.view("<f2")[:n].astype(np.float32).reshape(shape)
    if gtype == GGUF_Q8_0:
        blk = b[: n // 32 * 34].reshape(-1, 34)
        d = blk[:, :2].copy().view("<f2").astype(np.float32)
        q = blk[:, 2:].view(np.int8).astype(np.float32)
        return (d * q).reshape(shape)
    if gtype == GGUF_Q4_0:
        blk = b[: n // 32 * 18].reshape(-1, 18)
        d = blk[:, :2].copy().view("<f2").astype(np.float32)
        lo = (blk[:, 2:] & 0xF).astype(np.float32) - 8
        hi = (blk[:, 2:] >> 4).astype(np.float32) - 8
        return (d * np.concatenate([lo, hi], axis=1)).reshape(shape)
    raise ValueError(f"unsupported gguf type {gtype}")


LINEAR_KEYS = ("projection.weight", "q_proj.weight", "k_proj.weight", "v_proj.weight",
               "out_proj.weight", "intermediate_dense.weight", "output_dense.weight",
               "lm_head.weight")


def is_linear_weight(name: str) -> bool:
    return name.endswith(".weight") and any(k in name for k in LINEAR_KEYS)


def encode_tensor(name: str, arr: np.ndarray, dtype: str) -> tuple[int, bytes]:
    """(gguf type, bytes) following the reference converter's routing."""
    if dtype in ("q8_0", "q4_0") and is_linear_weight(name):
        if arr.size % 32 != 0:
            return GGUF_F16, arr.astype(np.float16).tobytes()
        return (GGUF_Q8_0, quantize_q8_0(arr)) if dtype == "q8_0" else (GGUF_Q4_0, quantize_q4_0(arr))
    if dtype == "f16":
        return GGUF_F16, arr.astype(np.float16).tobytes()
    return GGUF_F32, arr.astype(np.float32).tobytes()


# ── GGUF writer ──────────────────────────────────────────────────────────────

def _str(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def gguf_bytes(arch: Arch, tensors: dict[str, np.ndarray], dtype: str) -> bytes:
    kv = []
    def u32(k, v): kv.append(_str(k) + struct.pack("<II", 4, v))
    def s(k, v): kv.append(_str(k) + struct.pack("<I", 8) + _str(v))
    u32("wav2vec2.n_conv_layers", len(arch.conv_kernel))
    u32("wav2vec2.conv_dim", arch.conv_dim)
    u32("wav2vec2.n_encoder_layers", arch.n_layers)
    u32("wav2vec2.n_heads", arch.n_heads)
    u32("wav2vec2.hidden_size", arch.hidden)
    u32("wav2vec2.intermediate_size", arch.ffn)
    u32("wav2vec2.vocab_size", arch.vocab)
    u32("wav2vec2.pad_token_id", 0)
    u32("wav2vec2.pos_conv_kernel", arch.pos_kernel)
    u32("wav2vec2.pos_conv_groups", arch.pos_groups)
    s("wav2vec2.feat_extract_norm", arch.feat_norm)
    s("wav2vec2.word_delimiter_token", "|")
    kv.append(_str("wav2vec2.stable_layer_norm") + struct.pack("<I?", 7, arch.stable_layer_norm))
    for key, arr in (("wav2vec2.conv_kernel", arch.conv_kernel), ("wav2vec2.conv_stride", arch.conv_stride)):
        kv.append(_str(key) + struct.pack("<IIQ", 9, 4, len(arr)) + b"".join(struct.pack("<I", v) for v in arr))
    toks = vocab_tokens(arch.vocab)
    kv.append(_str("tokenizer.ggml.tokens") + struct.pack("<IIQ", 9, 8, len(toks)) + b"".join(_str(t) for t in toks))

    enc = {n: encode_tensor(n, a, dtype) for n, a in tensors.items()}
    head = bytearray(struct.pack("<IIQQ", GGUF_MAGIC, 3, len(tensors), len(kv)))
    for k in kv:
        head += k
    off = 0
    for n, a in tensors.items():
        gtype, data = enc[n]
        shape = list(reversed(a.shape))
        head += _str(n) + struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", d) for d in shape)
        head += struct.pack("<IQ", gtype, off)
        off += len(data) + (-len(data)) % ALIGN
    head += b"\0" * ((-len(head)) % ALIGN)
    parts = [bytes(head)]
    for n in tensors:
        data = enc[n][1]
        parts.append(data)
        parts.append(b"\0" * ((-len(data)) % ALIGN))
    return b"".join(parts)


def write_model(path: str | Path, arch: Arch | str, dtype: str = "q8_0", seed: int = 0, **kw) -> str:
    """Write a seeded random-init GGUF; returns its sha256."""
    if isinstance(arch, str):
        arch = ARCHS[arch]
    data = gguf_bytes(arch, model_tensors(arch, seed, **kw), dtype)
    Path(path).write_bytes(data)
    return hashlib.sha256(data).hexdigest()


def cached_model(dirpath: str | Path, arch: str, dtype: str, seed: int = 0, **kw) -> Path:
    """Generate (once) and return a model path under dirpath."""
    tag = "".join(f"_{k}{v}" for k, v in sorted(kw.items()))
    p = Path(dirpath) / f"{arch}_{dtype}_s{seed}{tag}.gguf"
    if not p.exists():
        Path(dirpath).mkdir(parents=True, exist_ok=True)
        tmp = p.with_suffix(".tmp")
        write_model(tmp, arch, dtype, seed, **kw)
        tmp.rename(p)
    return p


# ── audio ────────────────────────────────────────────────────────────────────

def make_audio(n_samples: int, seed: int, sr: int = 16000) -> np.ndarray:
    """Seeded synthetic utterance: 5 sinusoids + N(0, 0.05^2) noise, peak 0.9, float32."""
    rng = np.random.default_rng(seed)
    if n_samples <= 0:
        return np.zeros(0, np.float32)
    f = rng.uniform(80.0, 4000.0, 5)
    ph = rng.uniform(0.0, 2 * np.pi, 5)
    amp = rng.uniform(0.1, 1.0, 5)
    t = np.arange(n_samples, dtype=np.float64) / sr
    x = (amp[:, None] * np.sin(2 * np.pi * f[:, None] * t[None, :] + ph[:, None])).sum(0)
    x = x + rng.normal(0.0, 0.05, n_samples)
    peak = np.abs(x).max()
    if peak > 0:
        x = x * (0.9 / peak)
    return x.astype(np.float32)


def batch_audio(n_utt: int, n_samples: int | list[int], seed: int = 0) -> list[np.ndarray]:
    """Utterance i is seeded with seed + i."""
    lens = n_samples if isinstance(n_samples, (list, tuple)) else [n_samples] * n_utt
    return [make_audio(int(lens[i]), seed + i) for i in range(n_utt)]


def write_wav_f32(path: str | Path, x: np.ndarray, sr: int = 16000) -> None:
    """IEEE-float mono WAV; the reference CLI reads it bit-exactly (main.cpp:62)."""
    data = np.ascontiguousarray(x, np.float32).tobytes()
    hdr = b"RIFF" + struct.pack("<I", 36 + len(data)) + b"WAVE"
    hdr += b"fmt " + struct.pack("<IHHIIHH", 16, 3, 1, sr, sr * 4, 4, 32)
    hdr += b"data" + struct.pack("<I", len(data))
    Path(path).write_bytes(hdr + data)


def wav_bytes(x: np.ndarray, sr: int = 16000, fmt: str = "pcm16", chunks_before: tuple = (),
              fmt_size: int = 16, data_size: int | None = None, truncate: int = 0) -> bytes:
    """RIFF/WAVE image of x ([n] or [n, channels], float in [-1, 1]).
    fmt: "pcm16", "pcm32" (integer PCM, rounded and clipped) or "f32" (IEEE
    float).  chunks_before: (4-byte id, payload) chunks placed between "fmt "
    and "data"; fmt_size > 16 pads the fmt chunk (WAVE_FORMAT_EX style);
    data_size overrides the declared data length; truncate drops bytes from
    the end of the image."""
    x = np.asarray(x, np.float64)
    if x.ndim == 1:
        x = x[:, None]
    n, ch = x.shape
    if fmt == "pcm16":
        data = np.clip(np.round(x * 32768.0), -32768, 32767).astype("<i2").tobytes()
        code, bits = 1, 16
    elif fmt == "pcm32":
        data = np.clip(np.round(x * 2147483648.0), -2147483648, 2147483647).astype("<i4").tobytes()
        code, bits = 1, 32
    elif fmt == "f32":
        data = x.astype("<f4").tobytes()
        code, bits = 3, 32
    else:
        raise ValueError(fmt)
    blk = ch * bits // 8
    fmt_body = struct.pack("<HHIIHH", code, ch, sr, sr * blk, blk, bits) + b"\0" * (fmt_size - 16)
    body = b"WAVE" + b"fmt " + struct.pack("<I", fmt_size) + fmt_body
    for cid, payload in chunks_before:
        body += cid + struct.pack("<I", len(payload)) + payload
    body += b"data" + struct.pack("<I", len(data) if data_size is None else data_size) + data
    img = b"RIFF" + struct.pack("<I", len(body)) + body
    return img[:len(img) - truncate] if truncate else img


def n_frames(n_samples: int, arch: Arch | str = "base") -> int:
    """Conv extractor output length (reference wav2vec2.cpp:278)."""
    if isinstance(arch, str):
        arch = ARCHS[arch]
    L = n_samples
    for k, s in zip(arch.conv_kernel, arch.conv_stride):
        L = (L - k) // s + 1
    return L
