"""Host-side logic on the CPU: the C-ABI library loads and exports every
declared symbol, the model loader rejects bad files before touching a GPU,
the public header matches the reference's, and the batch planner /
fault-tolerant scheduler behave (simulated device failures re-queue work)."""
import json
import os
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
INC = ROOT / "include"
REF_HDR = Path(os.environ.get("W2V_REFERENCE", "/root/reference")) / "include" / "wav2vec2.h"


def declared_functions(header: Path) -> set[str]:
    txt = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
    txt = re.sub(r"//[^\n]*", "", txt)
    names = set()
    for m in re.finditer(r"^[ \t]*(?:struct\s+)?[A-Za-z_][\w \t\*]*?\b([a-z][\w]*)\s*\(", txt, flags=re.M):
        if m.group(1) not in ("if", "for", "while", "sizeof", "return"):
            names.add(m.group(1))
    return names


@pytest.fixture(scope="module")
def B(pkg):
    import w2v_b200.binding as b
    b.lib()
    return b


def test_library_exports_every_declared_symbol(B):
    L = B.lib()
    for h in ("wav2vec2.h", "wav2vec2_b200.h", "w2v_kernels.h"):
        names = declared_functions(INC / h)
        assert names, h
        for n in names:
            assert hasattr(L, n), f"{n} declared in {h} is not exported"
        for n in names:
            assert n in B.SIGNATURES, f"{n} has no ctypes signature in binding.py"


@pytest.mark.parametrize("C", [0, -4])
def test_conv0_rejects_non_positive_channels(B, C):
    """Channel counts <= 0 are rejected by the argument check, before any CUDA
    call (so this runs without a GPU), by both conv layer 0 entry points."""
    L = B.lib()
    W2V_ERR_ARGS = 1
    assert L.w2v_conv0(None, None, None, None, 4, None, None, None, C, 10, 5, 1, None, None, None, None, 1, 1,
                       None, None) == W2V_ERR_ARGS
    assert L.w2v_conv0_noalloc(None, None, None, None, 4, None, None, None, C, 10, 5, 1, None, None, None, 1, 1,
                               None, None) == W2V_ERR_ARGS


def test_public_header_matches_reference_api():
    ours = declared_functions(INC / "wav2vec2.h")
    assert ours == {"wav2vec2_default_params", "wav2vec2_init", "wav2vec2_free", "wav2vec2_transcribe",
                    "wav2vec2_result_free"}
    if REF_HDR.exists():
        assert declared_functions(REF_HDR) == ours
        norm = lambda t: re.sub(r"\s+", " ", re.sub(r"//[^\n]*|/\*.*?\*/", "", t, flags=re.S))
        for struct in ("wav2vec2_word", "wav2vec2_result", "wav2vec2_params"):
            pat = r"struct %s \{(.*?)\};" % struct
            assert re.search(pat, norm(REF_HDR.read_text())).group(1).strip() == \
                re.search(pat, norm((INC / "wav2vec2.h").read_text())).group(1).strip()


def _init_error(B, path):
    h = B.lib().wav2vec2_init(str(path).encode())
    if h:
        B.lib().wav2vec2_free(h)
        return None
    return B.last_error()


def test_init_missing_file(B, tmp_path):
    assert "Cannot open" in _init_error(B, tmp_path / "nope.gguf")


@pytest.mark.parametrize("corrupt,msg", [("magic", "Not GGUF"), ("truncated", "out of file bounds"),
                                         ("missing_key", "Missing key: wav2vec2.hidden_size"),
                                         ("bad_shape", "unsupported model")])
def test_init_rejects_bad_models_before_any_gpu_call(B, synth, tmp_path, corrupt, msg):
    import dataclasses
    arch = synth.ARCHS["tiny"]
    if corrupt == "bad_shape":
        arch = dataclasses.replace(arch, hidden=192, n_heads=2)     # head dim 96: unsupported
    data = bytearray(synth.gguf_bytes(arch, synth.model_tensors(arch, 0), "q8_0"))
    if corrupt == "magic":
        data[0] ^= 0xFF
    elif corrupt == "truncated":
        data = data[: len(data) // 3]
    elif corrupt == "missing_key":
        i = data.find(b"wav2vec2.hidden_size")
        data[i:i + 20] = b"wav2vec2.hidden_sizX"
    p = tmp_path / "bad.gguf"
    p.write_bytes(bytes(data))
    err = _init_error(B, p)
    assert err is not None and msg.lower() in err.lower(), err


def test_init_without_gpu_fails_cleanly(B, model_path):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    err = _init_error(B, model_path("tiny", "q8_0"))
    assert err is not None and "cuda" in err.lower()


def test_result_free_accepts_null(B):
    B.lib().wav2vec2_result_free(None)
    p = B.lib().wav2vec2_default_params()
    assert (p.n_threads, p.beam_size, p.verbose, p.word_timestamps) == (4, 1, False, False)


@pytest.fixture(scope="module")
def shard_runs(tmp_path_factory):
    exe = tmp_path_factory.mktemp("shard") / "shard_test"
    gxx = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else "g++"
    subprocess.run([gxx, "-std=c++17", "-O2", "-pthread", "-I", str(ROOT / "wav2vec2.cpp_b200" / "csrc"),
                    str(ROOT / "tests" / "cpp" / "shard_test.cpp"), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    return [json.loads(l) for l in out.splitlines()]


def test_batch_plan_is_a_length_bucketed_partition(shard_runs):
    plans = [r for r in shard_runs if r["scenario"] == "plan"]
    for r, max_batch in zip(plans, (64, 4, 64)):
        n = r["n"]
        flat = [i for b in r["batches"] for i in b]
        assert sorted(flat) == list(range(len(n)))                 # every utterance exactly once
        assert all(0 < len(b) <= max_batch for b in r["batches"])
        lens = [n[i] for b in r["batches"] for i in b]
        assert lens == sorted(lens, reverse=True)                  # longest first (bucketing)
        for b in r["batches"]:
            assert max(n[i] for i in b) * len(b) <= max_batch * 16000 * 32 or len(b) == 1


def test_scheduler_requeues_work_of_a_failed_device(shard_runs):
    s = [r for r in shard_runs if r["scenario"] == "sched"]
    ok, one_fails, all_fail, single = s
    assert not ok["threw"] and all(o >= 0 for o in ok["owner"]) and all(c == 1 for c in ok["runs"])
    assert not one_fails["threw"] and all(o >= 0 for o in one_fails["owner"])
    assert sum(c > 1 for c in one_fails["runs"]) == 1               # exactly the failed batch ran twice
    assert all_fail["threw"] and "injected failure" in all_fail["msg"]
    assert not single["threw"] and set(single["owner"]) == {0}
