"""Per-kernel parity on the GPU, through the C-ABI launchers.

Floating-point kernels are compared with an fp32/fp64 torch or oracle
computation on the same (fp16-rounded) inputs; integer/index kernels
(weight expansion, greedy CTC) must be bit-exact."""
import math

import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

EPI_F16, EPI_F16_GELU, EPI_F32, EPI_F32_RESID = 0, 1, 2, 3


@pytest.fixture(scope="module")
def K(pkg):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.backends.cuda.matmul.allow_tf32 = False
    import w2v_b200.binding as b
    b.lib()
    return b.kernels


def stream():
    return torch.cuda.current_stream().cuda_stream


def gelu_t(x):
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))


def dev(a):
    """Device copy of a numpy array.  Callers keep the returned tensor alive
    until the kernel that uses its pointer has completed."""
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def err_word():
    return torch.zeros(1, dtype=torch.int32, device="cuda")


@pytest.mark.parametrize("M,N,Kd,epi,bn", [
    (1, 64, 64, EPI_F32, 0), (200, 768, 768, EPI_F16, 0), (1000, 2304, 768, EPI_F16, 0),
    (777, 3072, 768, EPI_F16_GELU, 0), (333, 768, 3072, EPI_F32_RESID, 0), (499, 32, 768, EPI_F32, 64),
    (130, 128, 512, EPI_F32, 128), (257, 256, 1024, EPI_F32_RESID, 256), (4100, 1024, 1024, EPI_F32, 0),
    (99, 64, 768, EPI_F32, 64), (640, 5120, 1280, EPI_F16_GELU, 0)])
def test_gemm_plain(K, M, N, Kd, epi, bn):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    A = torch.randn(M, Kd, device="cuda", generator=g).half()
    W = (torch.randn(N, Kd, device="cuda", generator=g) * 0.05).half()
    bias = torch.randn(N, device="cuda", generator=g)
    resid = torch.randn(M, N, device="cuda", generator=g)
    f16 = epi in (EPI_F16, EPI_F16_GELU)
    out = torch.full((M, N), float("nan"), device="cuda", dtype=torch.float16 if f16 else torch.float32)
    err = err_word()
    K.gemm(A.data_ptr(), Kd, 1, 1, Kd, M, 1, M * Kd, W.data_ptr(), N, out.data_ptr(), N, M, M, bias.data_ptr(),
           resid.data_ptr() if epi == EPI_F32_RESID else 0, N, epi, bn, err.data_ptr(), stream())
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = A.double() @ W.double().T + bias.double()
    if epi == EPI_F16_GELU:
        ref = gelu_t(ref)
    if epi == EPI_F32_RESID:
        ref = ref + resid.double()
    d = (out.double() - ref).abs()
    # fp32 accumulation inside the tensor core over K products
    tol = (2e-3 if f16 else 1e-4) * (1 + ref.abs())
    assert torch.isfinite(out).all()
    assert (d <= tol).all(), f"max err {d.max().item()}"


@pytest.mark.parametrize("bn", [0, -256])
def test_gemm_gelu_epilogue_sweep(K, bn):
    """The GELU epilogue over a dense sweep of inputs: row i of A holds x_i in
    column 0 (exact in fp16), every weight row picks column 0, so each output
    is gelu(x_i); compared with the tanh form in fp64."""
    x = torch.linspace(-12, 12, 24001, device="cuda").half()
    M, N, Kd = x.numel(), 64, 64
    A = torch.zeros(M, Kd, device="cuda", dtype=torch.float16)
    A[:, 0] = x
    W = torch.zeros(N, Kd, device="cuda", dtype=torch.float16)
    W[:, 0] = 1
    out = torch.full((M, N), float("nan"), device="cuda", dtype=torch.float16)
    err = err_word()
    K.gemm(A.data_ptr(), Kd, 1, 1, Kd, M, 1, M * Kd, W.data_ptr(), N, out.data_ptr(), N, M, M, 0, 0, N,
           EPI_F16_GELU, bn, err.data_ptr(), stream())
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = gelu_t(x.double())[:, None]
    d = (out.double() - ref).abs()
    assert (d <= 2e-3 * (1 + ref.abs())).all(), (d / (1 + ref.abs())).max().item()
    assert (out[:, :1] == out).all(), "columns of one row differ"


@pytest.mark.parametrize("M,N,Kd,epi,bn", [
    (1, 256, 64, EPI_F32, -256), (255, 256, 768, EPI_F16, -256), (257, 512, 768, EPI_F32_RESID, -256),
    (20000, 2304, 768, EPI_F16, -256), (9000, 768, 3072, EPI_F32_RESID, -256), (7777, 3072, 768, EPI_F16_GELU, -256),
    (9000, 768, 768, EPI_F32_RESID, -128), (300, 200, 512, EPI_F32, -256), (513, 96, 256, EPI_F16, -128),
    (4000, 1280, 1280, EPI_F16_GELU, -128), (9000, 768, 3072, EPI_F32_RESID, -192),
    (5000, 768, 768, EPI_F32_RESID, 192), (777, 200, 512, EPI_F16_GELU, 192), (300, 500, 256, EPI_F16, -192)])
def test_gemm_cta_pair(K, M, N, Kd, epi, bn):
    """CTA-pair (cta_group::2) tiles of 256 x |bn|: ragged M and N, several
    tiles per pair (both TMEM accumulators in turn), every epilogue."""
    g = torch.Generator(device="cuda").manual_seed(M * 11 + N)
    A = torch.randn(M + 5, Kd, device="cuda", generator=g).half()
    W = (torch.randn(N, Kd, device="cuda", generator=g) * 0.05).half()
    bias = torch.randn(N, device="cuda", generator=g)
    resid = torch.randn(M, N, device="cuda", generator=g)
    f16 = epi in (EPI_F16, EPI_F16_GELU)
    out = torch.full((M + 5, N), float("nan"), device="cuda", dtype=torch.float16 if f16 else torch.float32)
    err = err_word()
    K.gemm(A.data_ptr(), Kd, 1, 1, Kd, M + 5, 1, (M + 5) * Kd, W.data_ptr(), N, out.data_ptr(), N, M + 5, M,
           bias.data_ptr(), resid.data_ptr() if epi == EPI_F32_RESID else 0, N, epi, bn, err.data_ptr(), stream())
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = A[:M].double() @ W.double().T + bias.double()
    if epi == EPI_F16_GELU:
        ref = gelu_t(ref)
    if epi == EPI_F32_RESID:
        ref = ref + resid.double()
    d = (out[:M].double() - ref).abs()
    tol = (2e-3 if f16 else 1e-4) * (1 + ref.abs())
    assert torch.isfinite(out[:M]).all()
    assert (d <= tol).all(), f"max err {d.max().item()}"
    assert torch.isnan(out[M:]).all(), "rows past m_valid were written"


@pytest.mark.parametrize("N,ldc", [(94, 104), (200, 216)])
@pytest.mark.parametrize("epi", [EPI_F16_GELU, EPI_F32_RESID])
@pytest.mark.parametrize("bn", [0, 128, 192, -256, -192])
def test_gemm_ragged_columns(K, epi, bn, N, ldc):
    """N not a multiple of the tile width inside a wider row pitch, columns
    N..ldc-1 untouched: N = 94 (not a multiple of 4: the last column group
    of each row is stored element by element) and N = 200 (fp16 C through
    TMA tile stores clipped at column N)."""
    M, Kd = 700, 256
    g = torch.Generator(device="cuda").manual_seed(5)
    A = torch.randn(M, Kd, device="cuda", generator=g).half()
    W = (torch.randn(N, Kd, device="cuda", generator=g) * 0.05).half()
    bias = torch.randn(N + 2, device="cuda", generator=g)
    f16 = epi == EPI_F16_GELU
    resid = torch.randn(M, ldc, device="cuda", generator=g)
    out = torch.full((M, ldc), float("nan"), device="cuda", dtype=torch.float16 if f16 else torch.float32)
    err = err_word()
    K.gemm(A.data_ptr(), Kd, 1, 1, Kd, M, 1, M * Kd, W.data_ptr(), N, out.data_ptr(), ldc, M, M, bias.data_ptr(),
           resid.data_ptr() if not f16 else 0, ldc, epi, bn, err.data_ptr(), stream())
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = A.double() @ W.double().T + bias[:N].double()
    ref = gelu_t(ref) if f16 else ref + resid[:, :N].double()
    d = (out[:, :N].double() - ref).abs()
    assert (d <= (2e-3 if f16 else 1e-4) * (1 + ref.abs())).all(), d.max().item()
    assert torch.isnan(out[:, N:]).all()


@pytest.mark.parametrize("M,N,Kd,bn", [(700, 768, 768, 0), (4100, 768, 3072, 0), (300, 1024, 1024, -256),
                                        (257, 1280, 5120, 192)])
def test_layer_norm_stats_and_ln_resid_gemm(K, M, N, Kd, bn):
    """Deferred LayerNorm of the post-LN encoder: w2v_layer_norm_stats writes
    LN(y) in fp16 plus per-row (mean, rstd); w2v_gemm_f16_ln_resid adds the
    fp32 LN(y) re-derived from y and those statistics to A.W^T + bias, in
    place over y (src/wav2vec2.cpp:360-373)."""
    g = torch.Generator(device="cuda").manual_seed(M + N)
    y = torch.randn(M, N, device="cuda", generator=g) * 3 + 0.7
    lw = 1 + torch.randn(N, device="cuda", generator=g) * 0.1
    lb = torch.randn(N, device="cuda", generator=g) * 0.1
    A = torch.randn(M, Kd, device="cuda", generator=g).half()
    W = (torch.randn(N, Kd, device="cuda", generator=g) * 0.05).half()
    bias = torch.randn(N, device="cuda", generator=g)
    xh = torch.empty(M, N, device="cuda", dtype=torch.float16)
    stats = torch.empty(M, 2, device="cuda")
    K.layer_norm_stats(y.data_ptr(), M, N, lw.data_ptr(), lb.data_ptr(), xh.data_ptr(), stats.data_ptr(), stream())
    torch.cuda.synchronize()
    yd = y.double()
    ln = (yd - yd.mean(1, keepdim=True)) / torch.sqrt(yd.var(1, unbiased=False, keepdim=True) + 1e-5) * lw.double() \
        + lb.double()
    assert (xh.double() - ln).abs().max().item() < 2e-3 * (1 + ln.abs().max().item())
    assert (stats[:, 0].double() - yd.mean(1)).abs().max().item() < 1e-5 * (1 + yd.abs().max().item())
    err = err_word()
    c = y.clone()
    K.gemm_ln_resid(A.data_ptr(), Kd, 1, 1, Kd, M, 1, M * Kd, W.data_ptr(), N, c.data_ptr(), N, M, M,
                    bias.data_ptr(), c.data_ptr(), N, stats.data_ptr(), lw.data_ptr(), lb.data_ptr(), bn,
                    err.data_ptr(), stream())
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = A.double() @ W.double().T + bias.double() + ln
    d = (c.double() - ref).abs()
    assert (d <= 1e-4 * (1 + ref.abs())).all(), d.max().item()


@pytest.mark.parametrize("B,C,Lin,k,s,bn", [(3, 512, 1001, 3, 2, -256), (2, 512, 8000, 2, 2, -256),
                                            (4, 128, 600, 3, 2, -128)])
def test_gemm_cta_pair_conv_view(K, B, C, Lin, k, s, bn):
    g = torch.Generator(device="cuda").manual_seed(Lin + 1)
    Lout = (Lin - k) // s + 1
    R = Lin + (-Lin) % s
    x = torch.randn(B, R, C, device="cuda", generator=g).half()
    w = (torch.randn(C, C, k, device="cuda", generator=g) * 0.05).half()
    wg = w.permute(0, 2, 1).reshape(C, k * C).contiguous()
    Rout = Lout + 3
    out = torch.full((B, Rout, C), float("nan"), device="cuda")
    err = err_word()
    K.gemm(x.data_ptr(), C, k, s, C, R, B, R * C, wg.data_ptr(), C, out.data_ptr(), C, Rout, Lout, 0, 0, 0,
           EPI_F32, bn, err.data_ptr(), stream())
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = torch.nn.functional.conv1d(x[:, :Lin].double().transpose(1, 2), w.double(), stride=s).transpose(1, 2)
    d = (out[:, :Lout].double() - ref).abs()
    assert (d <= 2e-5 * (1 + ref.abs())).all(), d.max().item()
    assert torch.isnan(out[:, Lout:]).all()


@pytest.mark.parametrize("B,C,Lin,k,s", [(3, 128, 257, 3, 2), (2, 512, 1000, 3, 2), (4, 128, 130, 2, 2),
                                         (1, 64, 77, 3, 2)])
def test_gemm_conv_view(K, B, C, Lin, k, s):
    """Strided conv as implicit GEMM over the 4-D TMA view (src/ops.h:76-99)."""
    g = torch.Generator(device="cuda").manual_seed(Lin)
    Lout = (Lin - k) // s + 1
    R = Lin + (-Lin) % s
    x = torch.randn(B, R, C, device="cuda", generator=g).half()
    w = (torch.randn(C, C, k, device="cuda", generator=g) * 0.05).half()          # [co][ci][k]
    wg = w.permute(0, 2, 1).reshape(C, k * C).contiguous()                         # [co][k*C + ci]
    Rout = Lout + 3
    out = torch.full((B, Rout, C), float("nan"), device="cuda")
    err = err_word()
    K.gemm(x.data_ptr(), C, k, s, C, R, B, R * C, wg.data_ptr(), C, out.data_ptr(), C, Rout, Lout, 0, 0, 0,
           EPI_F32, 0, err.data_ptr(), stream())
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = torch.nn.functional.conv1d(x[:, :Lin].double().transpose(1, 2), w.double(), stride=s).transpose(1, 2)
    d = (out[:, :Lout].double() - ref).abs()
    assert (d <= 2e-5 * (1 + ref.abs())).all(), d.max().item()


def test_gemm_rejects_bad_args(K):
    a = torch.zeros(64, 96, device="cuda", dtype=torch.float16)   # K not a multiple of 64
    w = torch.zeros(64, 96, device="cuda", dtype=torch.float16)
    o = torch.zeros(64, 64, device="cuda")
    import w2v_b200.binding as b
    with pytest.raises(b.EngineError):
        K.gemm(a.data_ptr(), 96, 1, 1, 96, 64, 1, 64 * 96, w.data_ptr(), 64, o.data_ptr(), 64, 64, 64,
               epilogue=EPI_F32, stream=stream())


@pytest.mark.parametrize("dtype", ["q8_0", "q4_0", "f16", "f32"])
def test_dequant_bit_exact(K, synth, dtype):
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((96, 256)) * 0.02).astype(np.float32)
    gt, raw = synth.encode_tensor("x.q_proj.weight", w, dtype)
    if dtype == "f32":
        gt, raw = synth.GGUF_F32, w.tobytes()
    ref = synth.dequantize(raw, gt, w.shape).astype(np.float16)
    d_raw = torch.from_numpy(np.frombuffer(raw, np.uint8).copy()).cuda()
    out = torch.empty(w.shape, dtype=torch.float16, device="cuda")
    K.dequant(d_raw.data_ptr(), gt, w.shape[0], w.shape[1], out.data_ptr(), stream())
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint16), ref.view(np.uint16))


def _meta(lens, k0=10, s0=5):
    off = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
    frames = np.array([(n - k0) // s0 + 1 if n >= k0 else 0 for n in lens], np.int32)
    return off, np.array(lens, np.int32), frames


@pytest.mark.parametrize("norm,C", [(0, 512), (1, 512), (2, 512), (2, 256)])
def test_conv0_norm_gelu(K, synth, norm, C):
    """Waveform normalisation + conv layer 0 + GroupNorm/LayerNorm + GELU
    (src/wav2vec2.cpp:262-287) against the oracle.  LayerNorm at 512 channels
    runs the warp-per-frame kernel, other widths the block kernel."""
    k0, s0 = 10, 5
    lens = [16000, 9000, 3210]
    audio = [synth.make_audio(n, 40 + i) for i, n in enumerate(lens)]
    off, ln, frames = _meta(lens)
    rng = np.random.default_rng(norm)
    w0 = (rng.standard_normal((C, 1, k0)) * 0.02).astype(np.float32)
    b0 = (rng.standard_normal(C) * 0.01).astype(np.float32)
    gw = (1 + rng.standard_normal(C) * 0.1).astype(np.float32)
    gb = (rng.standard_normal(C) * 0.02).astype(np.float32)
    d_audio, d_off, d_len, d_fr = dev(np.concatenate(audio)), dev(off), dev(ln), dev(frames)
    d_w0, d_b0, d_gw, d_gb = dev(w0.reshape(C, k0)), dev(b0), dev(gw), dev(gb)
    stats = torch.empty(2 * len(lens), device="cuda")
    gn = torch.empty(len(lens) * C * 2, device="cuda", dtype=torch.float64)
    rows = int(frames.max()) + 5
    out = torch.zeros(len(lens), rows, C, device="cuda", dtype=torch.float16)
    err = err_word()
    K.wave_stats(d_audio.data_ptr(), d_off.data_ptr(), d_len.data_ptr(), len(lens), stats.data_ptr(), stream())
    K.conv0(d_audio.data_ptr(), d_off.data_ptr(), d_len.data_ptr(), d_fr.data_ptr(), len(lens), stats.data_ptr(),
            d_w0.data_ptr(), d_b0.data_ptr(), C, k0, s0, norm,
            d_gw.data_ptr() if norm else 0, d_gb.data_ptr() if norm else 0,
            gn.data_ptr() if norm == 1 else 0, out.data_ptr(), rows, int(frames.max()), err.data_ptr(), stream())
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    got = out.float().cpu().numpy()
    for u in range(len(lens)):
        assert (got[u, frames[u]:] == 0).all(), f"rows past utterance {u}'s frames were written"
    for u, x in enumerate(audio):
        xd = x.astype(np.float64)
        xn = ((x - np.float32(xd.mean())) * np.float32(1 / np.sqrt(np.float32(xd.var()) + 1e-7))).astype(np.float32)
        y = O.conv1d(xn[:, None], w0, b0, stride=s0)
        if norm == 1:
            y = O.group_norm(y, gw, gb)
        elif norm == 2:
            y = O.layer_norm(y, gw, gb)
        ref = np.vectorize(O.gelu)(y) if y.size < 2000 else 0.5 * y * (1 + np.tanh(0.7978845608028654 * (y + 0.044715 * y ** 3)))
        g_u = got[u, :frames[u]]
        assert np.abs(g_u - ref).max() <= 2e-3 * (1 + np.abs(ref).max()), np.abs(g_u - ref).max()


@pytest.mark.parametrize("C", [512, 256])
def test_conv0_many_short_utterances(K, synth, C):
    """Tensor-core conv layer 0 (GroupNorm) over 300 short utterances, some
    empty: every CTA walks several (utterance, channel-half) groups, so the
    folded-weight buffers and the output boxes are each reused many times.
    Rows past each utterance's frames stay untouched."""
    k0, s0 = 10, 5
    rng = np.random.default_rng(C)
    lens = [int(n) for n in rng.integers(0, 1400, 300)]
    lens[3] = 4      # shorter than the kernel: no frames
    lens[7] = 650    # 129 frames: one full block and one frame
    audio = [synth.make_audio(n, 7 + i) if n else np.zeros(0, np.float32) for i, n in enumerate(lens)]
    off, ln, frames = _meta(lens)
    w0 = (rng.standard_normal((C, 1, k0)) * 0.02).astype(np.float32)
    b0 = (rng.standard_normal(C) * 0.01).astype(np.float32)
    gw = (1 + rng.standard_normal(C) * 0.1).astype(np.float32)
    gb = (rng.standard_normal(C) * 0.02).astype(np.float32)
    d_audio, d_off, d_len, d_fr = dev(np.concatenate(audio)), dev(off), dev(ln), dev(frames)
    d_w0, d_b0, d_gw, d_gb = dev(w0.reshape(C, k0)), dev(b0), dev(gw), dev(gb)
    n = len(lens)
    stats = torch.empty(2 * n, device="cuda")
    gn = torch.empty(n * C * 2, device="cuda", dtype=torch.float64)
    rows = int(frames.max()) + 3
    out = torch.zeros(n, rows, C, device="cuda", dtype=torch.float16)
    err = err_word()
    K.wave_stats(d_audio.data_ptr(), d_off.data_ptr(), d_len.data_ptr(), n, stats.data_ptr(), stream())
    K.conv0(d_audio.data_ptr(), d_off.data_ptr(), d_len.data_ptr(), d_fr.data_ptr(), n, stats.data_ptr(),
            d_w0.data_ptr(), d_b0.data_ptr(), C, k0, s0, 1, d_gw.data_ptr(), d_gb.data_ptr(), gn.data_ptr(),
            out.data_ptr(), rows, int(frames.max()), err.data_ptr(), stream())
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    got = out.float().cpu().numpy()
    for u, x in enumerate(audio):
        assert (got[u, frames[u]:] == 0).all(), f"rows past utterance {u}'s frames were written"
        if frames[u] == 0:
            continue
        xd = x.astype(np.float64)
        xn = ((x - np.float32(xd.mean())) * np.float32(1 / np.sqrt(np.float32(xd.var()) + 1e-7))).astype(np.float32)
        y = O.group_norm(O.conv1d(xn[:, None], w0, b0, stride=s0), gw, gb)
        ref = 0.5 * y * (1 + np.tanh(0.7978845608028654 * (y + 0.044715 * y ** 3)))
        d = np.abs(got[u, :frames[u]] - ref).max()
        assert d <= 2e-3 * (1 + np.abs(ref).max()), (u, d)


@pytest.mark.parametrize("D,f16in,gelu", [(768, 0, 0), (512, 1, 1), (1280, 0, 0), (128, 1, 0)])
def test_layer_norm(K, D, f16in, gelu):
    rng = np.random.default_rng(D)
    rows = [37, 0, 100]
    R = 110
    x = (rng.standard_normal((3, R, D)) * 2 + 0.5).astype(np.float32)
    if f16in:
        x = x.astype(np.float16).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    b = (0.1 * rng.standard_normal(D)).astype(np.float32)
    d_in = torch.from_numpy(x.astype(np.float16) if f16in else x).cuda()
    off = np.array([0, 37, 37], np.int64)
    M = sum(rows)
    out32 = torch.zeros(M, D, device="cuda")
    out16 = torch.zeros(M, D, device="cuda", dtype=torch.float16)
    d_rows, d_off = dev(np.array(rows, np.int32)), dev(off)
    d_w, d_b = dev(w), dev(b)
    K.layer_norm(d_in.data_ptr(), f16in, D, R, d_rows.data_ptr(), d_off.data_ptr(), 3, 0, D, d_w.data_ptr(),
                 d_b.data_ptr(), gelu, out32.data_ptr(), out16.data_ptr(), D, stream())
    torch.cuda.synchronize()
    ref = np.concatenate([O.layer_norm(x[u, :rows[u]], w, b) for u in range(3) if rows[u]])
    if gelu:
        ref = 0.5 * ref * (1 + np.tanh(0.7978845608028654 * (ref + 0.044715 * ref ** 3)))
    assert np.abs(out32.cpu().numpy() - ref).max() < 1e-4
    assert np.abs(out16.float().cpu().numpy() - ref).max() < 2e-3 * (1 + np.abs(ref).max())


@pytest.mark.parametrize("H,G,Kp", [(768, 16, 128), (128, 4, 16), (1024, 16, 128), (1280, 16, 128)])
def test_pos_conv(K, H, G, Kp):
    """Grouped positional conv + GELU + residual (src/wav2vec2.cpp:349-356).
    Two taps share each MMA and the odd taps' sums land one row early, so a
    CTA covers 511 frames (383 for 80-channel groups): lengths on both sides
    of those boundaries and of the 128-frame tiles inside a CTA."""
    rng = np.random.default_rng(H)
    T = [130, 7, 700, 512, 511, 383, 384, 385, 128, 1, 1023]
    off = np.concatenate([[0], np.cumsum(T)[:-1]]).astype(np.int64)
    M = sum(T)
    xin = rng.standard_normal((M, H)).astype(np.float16).astype(np.float32)
    Cg = H // G
    w = (rng.standard_normal((H, Cg, Kp)) * 0.02).astype(np.float16).astype(np.float32)
    b = (rng.standard_normal(H) * 0.1).astype(np.float32)
    # [G][Kp/2][Cg/8 (ci chunk)][2 Cg (tap parity, co)][8 (ci)]
    wt = (w.reshape(G, Cg, Cg // 8, 8, Kp // 2, 2).transpose(0, 4, 2, 5, 1, 3).astype(np.float16).copy())
    d_x = torch.full((M, H), float("nan"), device="cuda")
    d_xin, d_off, d_T, d_wt, d_b = dev(xin), dev(off), dev(np.array(T, np.int32)), dev(wt), dev(b)
    err = err_word()
    K.pos_conv(d_x.data_ptr(), d_xin.data_ptr(), d_off.data_ptr(), d_T.data_ptr(), len(T), H, Kp, G,
               d_wt.data_ptr(), d_b.data_ptr(), max(T), err.data_ptr(), stream())
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    got = d_x.cpu().numpy()
    assert np.isfinite(got).all()
    for u, t in enumerate(T):
        xs = torch.from_numpy(xin[off[u]:off[u] + t]).double()
        conv = torch.nn.functional.conv1d(xs.T[None], torch.from_numpy(w).double(), torch.from_numpy(b).double(),
                                          padding=Kp // 2, groups=G)[0].T[:t]
        ref = (xs + gelu_t(conv)).numpy()
        assert np.abs(got[off[u]:off[u] + t] - ref).max() < 2e-4 * (1 + np.abs(ref).max())


@pytest.mark.parametrize("H,nh,T", [(768, 12, [499, 1, 64, 65, 200]), (1280, 16, [499, 1, 64, 65, 200]),
                                    (128, 2, [499, 1, 64, 65, 200]), (1024, 8, [499, 1, 64, 65, 200]),
                                    (64, 1, [499, 1, 64, 65, 200]), (768, 12, [1499, 700]),
                                    (1280, 16, [1499, 33]), (1024, 8, [1499, 257]),
                                    (768, 12, [128, 129, 256, 257, 383, 384, 385, 2, 63])])
def test_attention(K, H, nh, T):
    """Flash attention vs fp64 softmax(QK^T/sqrt(d))V per utterance
    (src/wav2vec2.cpp:304-334), up to 30 s utterances (T = 1499: 24 key tiles,
    so the running max is raised mid-sequence); lengths on either side of
    the 128-query tile and the 32-key tile boundaries."""
    rng = np.random.default_rng(H + len(T))
    off = np.concatenate([[0], np.cumsum(T)[:-1]]).astype(np.int64)
    M = sum(T)
    qkv = (rng.standard_normal((M, 3 * H)) * 1.5).astype(np.float16)
    out = torch.zeros(M, H, device="cuda", dtype=torch.float16)
    d_qkv, d_off, d_T = dev(qkv), dev(off), dev(np.array(T, np.int32))
    err = err_word()
    K.attention(d_qkv.data_ptr(), out.data_ptr(), d_off.data_ptr(), d_T.data_ptr(), len(T), H, nh, max(T), M,
                err.data_ptr(), stream())
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    got = out.float().cpu().numpy()
    d = H // nh
    q = torch.from_numpy(qkv[:, :H].astype(np.float64))
    k = torch.from_numpy(qkv[:, H:2 * H].astype(np.float64))
    v = torch.from_numpy(qkv[:, 2 * H:].astype(np.float64))
    for u, t in enumerate(T):
        sl = slice(off[u], off[u] + t)
        qh = q[sl].view(t, nh, d).transpose(0, 1)
        kh = k[sl].view(t, nh, d).transpose(0, 1)
        vh = v[sl].view(t, nh, d).transpose(0, 1)
        p = torch.softmax(qh @ kh.transpose(1, 2) / math.sqrt(d), -1)
        ref = (p @ vh).transpose(0, 1).reshape(t, H).numpy()
        assert np.abs(got[sl] - ref).max() < 4e-3, np.abs(got[sl] - ref).max()


@pytest.mark.parametrize("N,Kd,epi", [(2304, 768, EPI_F16), (768, 3072, EPI_F32)])
def test_gemm_repeated_launches_identical(K, N, Kd, epi):
    """The CTA-pair GEMM hands stages and accumulators between its TMA,
    MMA and epilogue warps (and across the pair) through mbarriers; a
    handshake that loses a phase shows up only under timing skew.  30
    launches at an encoder shape (31936 rows, automatic tile) must give
    bitwise the same output and no expired wait."""
    M = 31936
    g = torch.Generator(device="cuda").manual_seed(N + Kd)
    A = torch.randn(M, Kd, device="cuda", generator=g).half()
    W = (torch.randn(N, Kd, device="cuda", generator=g) * 0.05).half()
    bias = torch.randn(N, device="cuda", generator=g)
    dt = torch.float16 if epi == EPI_F16 else torch.float32
    outs = [torch.zeros(M, N, device="cuda", dtype=dt) for _ in range(2)]
    err = err_word()
    for r in range(30):
        K.gemm(A.data_ptr(), Kd, 1, 1, Kd, M, 1, M * Kd, W.data_ptr(), N, outs[r % 2].data_ptr(), N, M, M,
               bias.data_ptr(), 0, N, epi, 0, err.data_ptr(), stream())
        if r % 2:
            torch.cuda.synchronize()
            assert int(err.item()) == 0, f"launch {r}: expired wait"
            assert torch.equal(outs[0], outs[1]), f"launch {r} differs from launch {r - 1}"


def test_conv0_repeated_launches_identical(K, synth):
    """Tensor-core conv layer 0 at the benchmark's batch (64 x 10 s): each
    CTA folds per-utterance weights into two shared buffers that it reuses
    once the MMAs reading them are done, and stores through TMA boxes it
    reuses once their stores have read them.  10 launches must give bitwise
    the same output and no expired wait."""
    C, k0, s0, n = 512, 10, 5, 64
    lens = [160000] * n
    audio = np.concatenate([synth.make_audio(L, 500 + i) for i, L in enumerate(lens)])
    off, ln, frames = _meta(lens)
    rng = np.random.default_rng(3)
    w0 = (rng.standard_normal((C, k0)) * 0.02).astype(np.float32)
    b0 = (rng.standard_normal(C) * 0.01).astype(np.float32)
    gw = (1 + rng.standard_normal(C) * 0.1).astype(np.float32)
    gb = (rng.standard_normal(C) * 0.02).astype(np.float32)
    d_audio, d_off, d_len, d_fr = dev(audio), dev(off), dev(ln), dev(frames)
    d_w0, d_b0, d_gw, d_gb = dev(w0), dev(b0), dev(gw), dev(gb)
    stats = torch.empty(2 * n, device="cuda")
    gn = torch.empty(n * C * 2, device="cuda", dtype=torch.float64)
    rows = int(frames.max())
    outs = [torch.zeros(n, rows, C, device="cuda", dtype=torch.float16) for _ in range(2)]
    err = err_word()
    K.wave_stats(d_audio.data_ptr(), d_off.data_ptr(), d_len.data_ptr(), n, stats.data_ptr(), stream())
    for r in range(10):
        K.conv0(d_audio.data_ptr(), d_off.data_ptr(), d_len.data_ptr(), d_fr.data_ptr(), n, stats.data_ptr(),
                d_w0.data_ptr(), d_b0.data_ptr(), C, k0, s0, 1, d_gw.data_ptr(), d_gb.data_ptr(), gn.data_ptr(),
                outs[r % 2].data_ptr(), rows, rows, err.data_ptr(), stream())
        if r % 2:
            torch.cuda.synchronize()
            assert int(err.item()) == 0, f"launch {r}: expired wait"
            assert torch.equal(outs[0], outs[1]), f"launch {r} differs from launch {r - 1}"


@pytest.mark.parametrize("H,nh", [(768, 12), (1024, 16)])
def test_attention_repeated_launches_identical(K, H, nh):
    """The softmax warps and the MMA thread hand S and P tiles back and forth
    through two TMEM buffers; a handshake that lets a fast warp's arrival
    count for a slow warp's tile shows up only under timing skew.  60
    launches at the benchmark's shape (64 utterances x 499 frames) on a loaded
    GPU must give bitwise the same output and no expired wait."""
    T = [499] * 64
    rng = np.random.default_rng(H)
    off = np.concatenate([[0], np.cumsum(T)[:-1]]).astype(np.int64)
    M = sum(T)
    d_qkv = torch.from_numpy((rng.standard_normal((M, 3 * H)) * 1.5).astype(np.float16)).cuda()
    d_off, d_T = dev(off), dev(np.array(T, np.int32))
    err = err_word()
    outs = [torch.zeros(M, H, device="cuda", dtype=torch.float16) for _ in range(2)]
    for r in range(60):
        K.attention(d_qkv.data_ptr(), outs[r % 2].data_ptr(), d_off.data_ptr(), d_T.data_ptr(), len(T), H, nh, 499, M,
                    err.data_ptr(), stream())
        if r % 2:
            torch.cuda.synchronize()
            assert int(err.item()) == 0, f"launch {r}: expired wait"
            assert torch.equal(outs[0], outs[1]), f"launch {r} differs from launch {r - 1}"



def test_ctc_greedy_bit_exact(K):
    """Per-frame argmax (first max wins) + run collapse (src/ops.h:132-149)."""
    rng = np.random.default_rng(9)
    T, V = [500, 1, 0, 37, 1024], 32
    off = np.concatenate([[0], np.cumsum(T)[:-1]]).astype(np.int64)
    M = sum(T)
    lg = rng.integers(-3, 3, (M, V)).astype(np.float32)      # many ties and long runs
    lg[10:40, 5] = 9
    d_lg = torch.from_numpy(lg).cuda()
    ids = torch.zeros(M, dtype=torch.int32, device="cuda")
    spans = torch.zeros(3 * M, dtype=torch.int32, device="cuda")
    ns = torch.zeros(len(T), dtype=torch.int32, device="cuda")
    d_off, d_T = dev(off), dev(np.array(T, np.int32))
    K.ctc_greedy(d_lg.data_ptr(), d_off.data_ptr(), d_T.data_ptr(), len(T), V, ids.data_ptr(), spans.data_ptr(),
                 ns.data_ptr(), max(T), stream())
    torch.cuda.synchronize()
    sp, n = spans.cpu().numpy(), ns.cpu().numpy()
    for u, t in enumerate(T):
        ref = O.greedy_spans(lg[off[u]:off[u] + t])
        got = [tuple(int(v) for v in sp[3 * (off[u] + i): 3 * (off[u] + i) + 3]) for i in range(n[u])]
        assert got == ref


def test_bounded_wait_expires_and_context_survives(K):
    """A wait that can never be satisfied ends with an error status (no hang,
    no trap), and the context keeps working afterwards."""
    import w2v_b200.binding as b
    err = err_word()
    assert b.lib().w2v_selftest_wait_timeout(err.data_ptr(), 50, stream()) == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 1                    # kErrBarrierTimeout
    A = torch.randn(128, 64, device="cuda").half()
    W = torch.randn(64, 64, device="cuda").half()
    out = torch.empty(128, 64, device="cuda")
    err2 = err_word()
    K.gemm(A.data_ptr(), 64, 1, 1, 64, 128, 1, 128 * 64, W.data_ptr(), 64, out.data_ptr(), 64, 128, 128,
           epilogue=EPI_F32, err=err2.data_ptr(), stream=stream())
    torch.cuda.synchronize()
    assert int(err2.item()) == 0
    assert torch.allclose(out, A.float() @ W.float().T, atol=1e-3, rtol=1e-3)
