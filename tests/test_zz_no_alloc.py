"""w2v_conv0_noalloc: conv layer 0 for callers that cannot allocate device
memory (for example a host whose device memory belongs to another allocator,
or a real-time thread that must not make a call that can block on the
device).  It keeps its GroupNorm statistics in a buffer built into the library
instead of asking the caller for scratch, so it must give the same result as
the allocating entry point, call after call (each call re-zeroes the shared
buffer).  Kept in its own file, collected last."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

W2V_ERR_CAPACITY = 6


def test_conv0_noalloc_matches_allocating_entry_point(pkg, synth):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import w2v_b200.binding as b
    L = b.lib()
    C, k0, s0, norm = 512, 10, 5, 1                       # GroupNorm: the path that needs scratch
    lens = [16000, 9000, 3210, 40000]
    audio = [synth.make_audio(n, 300 + i) for i, n in enumerate(lens)]
    off = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
    frames = np.array([(n - k0) // s0 + 1 for n in lens], np.int32)
    rng = np.random.default_rng(11)
    w0 = (rng.standard_normal((C, k0)) * 0.02).astype(np.float32)
    gw = (1 + rng.standard_normal(C) * 0.1).astype(np.float32)
    gb = (rng.standard_normal(C) * 0.02).astype(np.float32)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    d_audio, d_off, d_len, d_fr = dev(np.concatenate(audio)), dev(off), dev(np.array(lens, np.int32)), dev(frames)
    d_w0, d_gw, d_gb = dev(w0), dev(gw), dev(gb)
    stats = torch.empty(2 * len(lens), device="cuda")
    rows = int(frames.max())
    st = torch.cuda.current_stream().cuda_stream
    assert L.w2v_wave_stats(d_audio.data_ptr(), d_off.data_ptr(), d_len.data_ptr(), len(lens), stats.data_ptr(),
                            st) == 0
    # allocating entry point: caller-provided statistics buffer
    gn = torch.empty(len(lens) * C * 2, device="cuda", dtype=torch.float64)
    ref = torch.zeros(len(lens), rows, C, device="cuda", dtype=torch.float16)
    assert L.w2v_conv0(d_audio.data_ptr(), d_off.data_ptr(), d_len.data_ptr(), d_fr.data_ptr(), len(lens),
                       stats.data_ptr(), d_w0.data_ptr(), None, C, k0, s0, norm, d_gw.data_ptr(), d_gb.data_ptr(),
                       gn.data_ptr(), ref.data_ptr(), rows, rows, None, st) == 0
    torch.cuda.synchronize()
    ref = ref.float()
    for call in range(2):
        out = torch.full((len(lens), rows, C), float("nan"), device="cuda", dtype=torch.float16)
        rc = L.w2v_conv0_noalloc(d_audio.data_ptr(), d_off.data_ptr(), d_len.data_ptr(), d_fr.data_ptr(),
                                 len(lens), stats.data_ptr(), d_w0.data_ptr(), None, C, k0, s0, norm,
                                 d_gw.data_ptr(), d_gb.data_ptr(), out.data_ptr(), rows, rows, None, st)
        assert rc == 0, f"call {call}: status {rc}"
        torch.cuda.synchronize()
        for u, f in enumerate(frames):
            got, want = out[u, :f].float(), ref[u, :f]
            assert torch.isfinite(got).all()
            # same tolerance as the conv0 parity test (fp16 output rounding)
            assert (got - want).abs().max().item() <= 2e-3 * (1 + want.abs().max().item()), (call, u)


def test_conv0_noalloc_rejects_oversized_requests(pkg):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import w2v_b200.binding as b
    L = b.lib()
    # 65 utterances exceed the built-in buffer: rejected before anything is launched
    rc = L.w2v_conv0_noalloc(None, None, None, None, 65, None, None, None, 512, 10, 5, 1, None, None, None, 1, 1,
                             None, None)
    assert rc == W2V_ERR_CAPACITY
    rc = L.w2v_conv0_noalloc(None, None, None, None, 4, None, None, None, 1024, 10, 5, 1, None, None, None, 1, 1,
                             None, None)
    assert rc == W2V_ERR_CAPACITY
