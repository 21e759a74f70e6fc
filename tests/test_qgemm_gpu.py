"""Dequant-fused tcgen05 GEMM (w2v_gemm_q / w2v_gemm_q_ln_resid) on GGUF
Q8_0 and Q4_0 weights (blocks as written by the reference converter,
scripts/convert_to_gguf.py:63-97), through the C-ABI launchers.

The converter warps expand each block to fp16 in tensor memory with one
rounding of d*q, exactly the values of the load-time expansion
(w2v_dequant_f16).  The fused GEMM is compared with the fp16 GEMM on those
expanded weights (same products, fp32 accumulation: they may differ only in
the order the tensor core sums within one instruction) and with an fp64
product of the dequantised weights."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

EPI_F16, EPI_F16_GELU, EPI_F32, EPI_F32_RESID = 0, 1, 2, 3
Q8_0, Q4_0 = 8, 2


@pytest.fixture(scope="module")
def K(pkg):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import w2v_b200.binding as b
    b.lib()
    return b.kernels


def st():
    return torch.cuda.current_stream().cuda_stream


def gelu_t(x):
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))


class QLinear:
    """A quantised [N, K] weight on the device in both forms: the fused GEMM's
    planes (w2v_repack_q) and fp16 rows (w2v_dequant_f16)."""

    def __init__(self, K, synth, N, Kd, gtype, seed):
        rng = np.random.default_rng(seed)
        w = (rng.standard_normal((N, Kd)) * 0.02).astype(np.float32)
        w[0, :32] = 0.0                                    # an all-zero block
        raw = synth.quantize_q8_0(w) if gtype == Q8_0 else synth.quantize_q4_0(w)
        self.raw = torch.from_numpy(np.frombuffer(raw, np.uint8).copy()).cuda()
        self.N, self.K, self.gtype = N, Kd, gtype
        self.ld = (N + 7) // 8 * 8
        self.codes = torch.empty(N * Kd // (1 if gtype == Q8_0 else 2), dtype=torch.uint8, device="cuda")
        self.scales = torch.zeros(Kd // 32, self.ld, dtype=torch.int16, device="cuda")
        self.w16 = torch.empty(N, Kd, dtype=torch.float16, device="cuda")
        K.repack_q(self.raw.data_ptr(), gtype, N, Kd, self.codes.data_ptr(), self.scales.data_ptr(), self.ld, st())
        K.dequant(self.raw.data_ptr(), gtype, N, Kd, self.w16.data_ptr(), st())
        torch.cuda.synchronize()


def test_repack_planes_decode_to_the_expanded_weights(K, synth):
    """The planes hold exactly the blocks' codes and scales: decoding them on
    the host (layout of w2v_repack_q) gives the fp16 weights of the load-time
    expansion, bit for bit."""
    for gtype in (Q8_0, Q4_0):
        q = QLinear(K, synth, 96, 256, gtype, 5)
        codes = q.codes.cpu().numpy()
        d = q.scales.cpu().numpy()[:, :q.N].view(np.float16).astype(np.float32)     # [K/32, N]
        if gtype == Q8_0:
            c = codes.view(np.int8).reshape(q.N, q.K).astype(np.float32)
        else:
            words = codes.view(np.uint32).reshape(q.N, q.K // 8)
            c = np.zeros((q.N, q.K), np.float32)
            for j in range(4):
                c[:, 2 * j::8] = ((words >> (4 * j)) & 0xF).astype(np.float32) - 8
                c[:, 2 * j + 1::8] = ((words >> (16 + 4 * j)) & 0xF).astype(np.float32) - 8
        w = (c * np.repeat(d.T, 32, axis=1)).astype(np.float16)
        assert np.array_equal(w.view(np.uint16), q.w16.cpu().numpy().view(np.uint16)), gtype


def run_pair(K, q, M, epi, bn, seed):
    """The fused GEMM and the fp16 GEMM on the expanded weights, same inputs."""
    N, Kd = q.N, q.K
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randn(M, Kd, device="cuda", generator=g).half()
    bias = torch.randn(N, device="cuda", generator=g)
    resid = torch.randn(M, N, device="cuda", generator=g)
    f16 = epi in (EPI_F16, EPI_F16_GELU)
    dt = torch.float16 if f16 else torch.float32
    out_q = torch.full((M, N), float("nan"), device="cuda", dtype=dt)
    out_f = torch.full((M, N), float("nan"), device="cuda", dtype=dt)
    err = torch.zeros(2, dtype=torch.int32, device="cuda")
    rq, rf = resid.clone(), resid.clone()
    K.gemm_q(A.data_ptr(), Kd, M, q.codes.data_ptr(), q.scales.data_ptr(), q.ld, q.gtype, N, out_q.data_ptr(), N,
             bias.data_ptr(), rq.data_ptr() if epi == EPI_F32_RESID else 0, N, epi, bn, err.data_ptr(), st())
    K.gemm(A.data_ptr(), Kd, 1, 1, Kd, M, 1, M * Kd, q.w16.data_ptr(), N, out_f.data_ptr(), N, M, M, bias.data_ptr(),
           rf.data_ptr() if epi == EPI_F32_RESID else 0, N, epi, 0, err[1:].data_ptr(), st())
    torch.cuda.synchronize()
    assert err.tolist() == [0, 0]
    ref = A.double() @ q.w16.double().T + bias.double()
    if epi == EPI_F16_GELU:
        ref = gelu_t(ref)
    if epi == EPI_F32_RESID:
        ref = ref + resid.double()
    return out_q, out_f, ref, f16


@pytest.mark.parametrize("gtype", [Q8_0, Q4_0])
@pytest.mark.parametrize("M,N,Kd,epi,bn", [
    (499, 3072, 768, EPI_F16_GELU, 0), (499, 32, 768, EPI_F32, 0), (1, 128, 64, EPI_F32, 128),
    (31936, 2304, 768, EPI_F16, -192), (5000, 768, 3072, EPI_F32_RESID, -192), (777, 1024, 1024, EPI_F32, 128),
    (300, 768, 768, EPI_F32_RESID, -128), (2049, 200, 512, EPI_F16, 192), (130, 96, 256, EPI_F16_GELU, -128),
    (4000, 3072, 768, EPI_F16_GELU, 0), (3001, 768, 768, EPI_F32_RESID, -224), (700, 320, 512, EPI_F16, 224),
    (499, 2304, 768, EPI_F16, 64), (499, 768, 3072, EPI_F32_RESID, 64), (77, 200, 256, EPI_F32, 64)])
def test_gemm_q_matches_fp16_gemm(K, synth, gtype, M, N, Kd, epi, bn):
    """Every tile family (CTA pairs and single CTAs, 224, 192, 128 and 64
    activation rows), ragged rows and features, every epilogue."""
    q = QLinear(K, synth, N, Kd, gtype, M + N)
    out_q, out_f, ref, f16 = run_pair(K, q, M, epi, bn, M * 3 + N)
    assert torch.isfinite(out_q).all()
    tol = (2e-3 if f16 else 1e-4) * (1 + ref.abs())
    assert ((out_q.double() - ref).abs() <= tol).all(), (out_q.double() - ref).abs().max().item()
    # against the fp16 GEMM on the same fp16 weights: fp32 summation order only
    d = (out_q.double() - out_f.double()).abs()
    if f16:
        assert (d <= 1e-3 * (1 + out_f.double().abs())).all(), d.max().item()
    else:
        assert (d <= 2e-5 * (1 + out_f.double().abs())).all(), d.max().item()


@pytest.mark.parametrize("gtype,bn,Kd", [(Q8_0, -192, 3072), (Q4_0, -128, 3072), (Q8_0, 128, 3072), (Q8_0, 64, 3072),
                                         (Q4_0, -224, 3072), (Q8_0, -224, 768), (Q4_0, 128, 768), (Q8_0, 64, 768)])
def test_gemm_q_ln_resid(K, synth, gtype, bn, Kd):
    """Post-LN residual epilogue (the residual normalised on the fly from
    per-row statistics), in place over C, with two epilogue warps per lane
    quarter on alternate chunks (and one where the output cannot take TMA
    stores)."""
    M, N = 3000, 768
    q = QLinear(K, synth, N, Kd, gtype, 77)
    g = torch.Generator(device="cuda").manual_seed(9)
    A = torch.randn(M, Kd, device="cuda", generator=g).half()
    bias = torch.randn(N, device="cuda", generator=g)
    x0 = torch.randn(M, N, device="cuda", generator=g)
    stats = torch.stack([torch.randn(M, device="cuda", generator=g),
                         torch.rand(M, device="cuda", generator=g) + 0.5], 1).contiguous()
    lw = torch.randn(N, device="cuda", generator=g)
    lb = torch.randn(N, device="cuda", generator=g)
    xq, xf = x0.clone(), x0.clone()
    err = torch.zeros(2, dtype=torch.int32, device="cuda")
    K.gemm_q_ln_resid(A.data_ptr(), Kd, M, q.codes.data_ptr(), q.scales.data_ptr(), q.ld, gtype, N, xq.data_ptr(),
                      N, bias.data_ptr(), xq.data_ptr(), N, stats.data_ptr(), lw.data_ptr(), lb.data_ptr(), bn,
                      err.data_ptr(), st())
    K.gemm_ln_resid(A.data_ptr(), Kd, 1, 1, Kd, M, 1, M * Kd, q.w16.data_ptr(), N, xf.data_ptr(), N, M, M,
                    bias.data_ptr(), xf.data_ptr(), N, stats.data_ptr(), lw.data_ptr(), lb.data_ptr(),
                    err=err[1:].data_ptr(), stream=st())
    torch.cuda.synchronize()
    assert err.tolist() == [0, 0]
    ref = (A.double() @ q.w16.double().T + bias.double()
           + (x0.double() - stats[:, :1].double()) * stats[:, 1:].double() * lw.double() + lb.double())
    assert ((xq.double() - ref).abs() <= 1e-4 * (1 + ref.abs())).all()
    assert ((xq.double() - xf.double()).abs() <= 2e-5 * (1 + ref.abs())).all()


def test_gemm_q_repeated_launches_identical(K, synth):
    """The same launch 20 times at the benchmark's QKV shape: bitwise equal
    results (no race between the converters, the MMA and the epilogue)."""
    q = QLinear(K, synth, 2304, 768, Q8_0, 3)
    M = 31936
    A = torch.randn(M, 768, device="cuda").half()
    outs = []
    for _ in range(20):
        o = torch.full((M, 2304), float("nan"), device="cuda", dtype=torch.float16)
        K.gemm_q(A.data_ptr(), 768, M, q.codes.data_ptr(), q.scales.data_ptr(), q.ld, Q8_0, 2304, o.data_ptr(), 2304,
                 0, 0, 0, EPI_F16, 0, 0, st())
        outs.append(o)
    torch.cuda.synchronize()
    assert all(torch.equal(outs[0], o) for o in outs[1:])


def test_gemm_q_rejects_bad_arguments(K, synth):
    q = QLinear(K, synth, 64, 64, Q8_0, 1)
    A = torch.zeros(4, 64, device="cuda", dtype=torch.float16)
    out = torch.zeros(4, 64, device="cuda")
    import w2v_b200.binding as b
    L = b.lib()
    # unknown weight type, ld_s < N, ld_s not a multiple of 8, a tile not built
    for gtype, ld, bn in ((1, 64, 0), (8, 32, 0), (8, 68, 0), (8, 64, 256)):
        rc = L.w2v_gemm_q(A.data_ptr(), 64, 4, q.codes.data_ptr(), q.scales.data_ptr(), ld, gtype, 64, out.data_ptr(),
                          64, None, None, 64, EPI_F32, bn, None, None)
        assert rc == 1, (gtype, ld, bn)
