"""The drop-in from C++: tests/cpp/engine_harness.cpp is compiled with g++
(-std=c++23) against include/kernels/kernels.hpp and linked to libb200attn.so,
then runs the reference engine's per-layer call sequence
(include/model_inference.hpp:272-292 prefill, :96-123 / :358-388 graph-captured
decode with node patching) and the reference's own kernel tests
(tests/test_causal_attention.cpp:15-228) restated in C++. Its outputs are
checked here against the CPU oracle."""
import os
import subprocess

import numpy as np
import pytest

import oracle
from _util import assert_attention_close, seeded_f16

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "cpp", "engine_harness.cpp")
OUT_DIR = os.path.join(ROOT, "tests", "cpp", "_build")
EXE = os.path.join(OUT_DIR, "engine_harness")
LIBDIR = os.path.join(ROOT, "llm-inference_b200", "b200attn")
MAGIC = 0x62323030656e67


def build_harness() -> str:
    """g++ -std=c++23 against the drop-in headers, linked to libb200attn.so
    (rpath to this checkout) and the CUDA runtime."""
    os.makedirs(OUT_DIR, exist_ok=True)
    tmp = EXE + f".tmp{os.getpid()}"
    cmd = ["g++", "-std=c++23", "-O2", "-Wall", "-Wextra", "-Werror", f"-I{ROOT}/include",
           "-I/usr/local/cuda/include", SRC, "-o", tmp, f"-L{LIBDIR}", "-lb200attn", "-L/usr/local/cuda/lib64",
           "-lcudart", f"-Wl,-rpath,{LIBDIR}", "-Wl,-rpath,/usr/local/cuda/lib64"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr[-4000:]
    os.replace(tmp, EXE)
    return EXE


def test_harness_compiles_and_links():
    """CPU: the harness builds against the shim and the library and starts
    (usage exit, no CUDA call)."""
    exe = build_harness()
    res = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert res.returncode == 2 and "usage" in res.stderr


@pytest.mark.gpu
def test_harness_known_answer_sweep(cuda):
    exe = build_harness()
    res = subprocess.run([exe, "known-answer"], capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "60 cases, 0 failures" in res.stdout


@pytest.mark.gpu
def test_harness_golden_fixture_tests(cuda):
    exe = build_harness()
    for sub in ("", "sharp"):
        res = subprocess.run([exe, "golden", os.path.join(ROOT, "tests", "golden", sub)], capture_output=True,
                             text=True, timeout=600)
        assert res.returncode == 0, res.stdout + res.stderr
        assert "0 failures" in res.stdout


@pytest.mark.gpu
def test_harness_engine_sequence_vs_oracle(cuda, tmp_path):
    """4 layers (layer 3 NoPE), a 300-token prompt, then 5 decode tokens through
    one captured graph whose RoPE / attention / merge nodes are patched per
    token. Prefill rows, decode outputs and the caches against the oracle."""
    L, S, T, H, KVH, d, max_seq = 4, 300, 5, 16, 4, 128, 512
    qd, kd = H * d, KVH * d
    total = qd + 2 * kd
    prompt = seeded_f16((L, S, total), 901)
    news = seeded_f16((T, L, total), 902)
    hdr = np.array([MAGIC, L, S, T, H, KVH, d, max_seq], np.uint64)
    inp, outp = tmp_path / "in.bin", tmp_path / "out.bin"
    with open(inp, "wb") as f:
        f.write(hdr.tobytes())
        f.write(prompt.tobytes())
        f.write(news.tobytes())
    exe = build_harness()
    res = subprocess.run([exe, "engine", str(inp), str(outp)], capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout + res.stderr
    raw = np.fromfile(outp, np.float16)
    n_pre, n_dec = L * S * qd, T * L * qd
    assert raw.size == n_pre + n_dec + L * 2 * (S + T) * kd
    pre = raw[:n_pre].reshape(L, S, qd)
    dec = raw[n_pre:n_pre + n_dec].reshape(T, L, qd)
    caches = raw[n_pre + n_dec:].reshape(L, 2, S + T, kd)
    cos, sin = oracle.rope_tables(max_seq, d, 5.0e6)
    for l in range(L):
        rot = (l + 1) % 4 != 0
        q = np.ascontiguousarray(prompt[l, :, :qd])
        k = np.ascontiguousarray(prompt[l, :, qd:qd + kd])
        v = np.ascontiguousarray(prompt[l, :, qd + kd:])
        kc = np.zeros((max_seq, kd), np.float16)
        vc = np.zeros((max_seq, kd), np.float16)
        oracle.rope_and_store_kv(q, k, v, kc, vc, cos, sin, S, H, KVH, d, qd, kd, 0, rot)
        _, o32 = oracle.causal_attention(q, kc, vc, S, H, KVH, d)
        assert_attention_close(pre[l], o32)
        for t in range(T):
            p = S + t
            qn = np.ascontiguousarray(news[t, l, :qd])
            kn = np.ascontiguousarray(news[t, l, qd:qd + kd])
            vn = np.ascontiguousarray(news[t, l, qd + kd:])
            oracle.rope_and_store_kv(qn, kn, vn, kc, vc, cos, sin, 1, H, KVH, d, qd, kd, p, rot)
            _, d32 = oracle.decode_attention(qn, kc, vc, p + 1, H, KVH, d)
            assert_attention_close(dec[t, l], d32.reshape(-1))
        # RoPE slot writes and the NoPE copy are exact
        np.testing.assert_array_equal(caches[l, 0].view(np.uint16), kc[:S + T].view(np.uint16))
        np.testing.assert_array_equal(caches[l, 1].view(np.uint16), vc[:S + T].view(np.uint16))


@pytest.mark.gpu
@pytest.mark.parametrize("S,start,rotate", [(300, 0, True), (254, 37, False)])
def test_harness_qkv_step_fused_vs_two_calls(cuda, tmp_path, S, start, rotate):
    """From C++: the engine's QKV step as launch_qkv_gemm + launch_rope_and_store_kv
    and as launch_qkv_gemm_rope_store_kv agree bit for bit (checked in the
    harness), and the fused rows and cache rows match the oracle on the host
    product."""
    hidden, H, KVH, d = 2048, 16, 4, 128
    qd, kd = H * d, KVH * d
    total = qd + 2 * kd
    max_seq = start + S + 16
    x = seeded_f16((S, hidden), 961 + S)
    w = (seeded_f16((total, hidden), 962) * np.float16(0.03)).astype(np.float16)
    hdr = np.array([0x62323030716b76, S, hidden, H, KVH, d, start, int(rotate), max_seq, 0], np.uint64)
    inp, outp = tmp_path / "qkv_in.bin", tmp_path / "qkv_out.bin"
    with open(inp, "wb") as f:
        f.write(hdr.tobytes())
        f.write(x.tobytes())
        f.write(w.tobytes())
    exe = build_harness()
    res = subprocess.run([exe, "qkv", str(inp), str(outp)], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "0 failures" in res.stdout
    raw = np.fromfile(outp, np.float16)
    assert raw.size == S * total + 2 * S * kd
    rows = raw[:S * total].reshape(S, total)
    kc = raw[S * total:S * total + S * kd].reshape(S, kd)
    vc = raw[S * total + S * kd:].reshape(S, kd)
    prod = (x.astype(np.float64) @ w.astype(np.float64).T).astype(np.float16)
    q = np.ascontiguousarray(prod[:, :qd])
    k = np.ascontiguousarray(prod[:, qd:qd + kd])
    v = np.ascontiguousarray(prod[:, qd + kd:])
    cos, sin = oracle.rope_tables(max_seq, d, 5.0e6)
    ek = np.zeros((max_seq, kd), np.float16)
    ev = np.zeros((max_seq, kd), np.float16)
    oracle.rope_and_store_kv(q, k, v, ek, ev, cos, sin, S, H, KVH, d, qd, kd, start, rotate)
    assert_attention_close(rows[:, :qd], q.astype(np.float32))
    assert_attention_close(rows[:, qd:], prod[:, qd:].astype(np.float32))
    assert_attention_close(kc, ek[start:start + S].astype(np.float32))
    assert_attention_close(vc, ev[start:start + S].astype(np.float32))
