"""weights.bin loader (include/b200attn/weights.hpp, b200attn/weights.py) on a
file written by the reference's own exporter (python/export_weights.py, see
tests/golden/make_weights_fixture.py): header, tokenizer JSON, the payload
offset and every tensor the loader carves, against the exporting model's
state dict (tests/golden/tiny_weights.json); and the layer-0 activations the
reference's fixture generator dumped for that model (tests/golden/tiny/) run
through RoPE, prefill and the o_proj carved from the loaded weights."""
import json
import os
import subprocess

import numpy as np
import pytest

from b200attn import weights as W

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FIX = os.path.join(ROOT, "tests", "golden", "tiny_weights.bin")
META = json.load(open(os.path.join(ROOT, "tests", "golden", "tiny_weights.json")))


def _expected():
    """(loader name, shape, sum, sumsq, first) in file order."""
    names = [n for n, _ in W.layout(W.read_weights(FIX).config)]
    return [(n, tuple(t["shape"]), t["sum"], t["sumsq"], t["first"]) for n, t in zip(names, META["tensors"])]


def _check(name, n_elems, s, sq, first, exp):
    en, shape, es, esq, efirst = exp
    assert name == en
    assert n_elems == int(np.prod(shape))
    assert s == pytest.approx(es, rel=1e-9, abs=1e-6)
    assert sq == pytest.approx(esq, rel=1e-9)
    assert list(first) == pytest.approx(efirst, abs=0)


def test_header_tokenizer_and_every_tensor():
    w = W.read_weights(FIX)
    h = META["header"]
    assert (w.config.vocab_size, w.config.hidden_size, w.config.num_layers, w.config.num_heads,
            w.config.num_kv_heads, w.config.head_dim, w.config.intermediate_size, w.config.max_seq_len) == \
        (h["vocab_size"], h["hidden_size"], h["num_layers"], h["num_heads"], h["num_kv_heads"], h["head_dim"],
         h["intermediate_size"], h["max_seq_len"])
    assert w.config.rope_theta == pytest.approx(h["rope_theta"])
    assert w.tokenizer_json.decode() == META["tokenizer_json"]
    assert W.weights_offset(len(w.tokenizer_json)) % 64 == 0
    exp = _expected()
    assert len(exp) == len(w.tensors) == len(META["tensors"])
    for e, (name, arr) in zip(exp, w.tensors.items()):
        a = arr.astype(np.float64)
        _check(name, a.size, float(a.sum()), float((a * a).sum()), a.reshape(-1)[:4], e)
    # the tied LM head is the embedding, written twice
    np.testing.assert_array_equal(w.tensors["lm_head"], w.tensors["embedding_tokens"])


def test_bad_files_are_rejected(tmp_path):
    raw = open(FIX, "rb").read()
    bad = tmp_path / "bad_magic.bin"
    bad.write_bytes(b"XXXX" + raw[4:])
    with pytest.raises(ValueError, match="magic"):
        W.read_weights(str(bad))
    short = tmp_path / "short.bin"
    short.write_bytes(raw[:-2])
    with pytest.raises(ValueError, match="payload"):
        W.read_weights(str(short))
    longer = tmp_path / "long.bin"          # e.g. extra q_norm / k_norm tensors
    longer.write_bytes(raw + b"\0" * 64)
    with pytest.raises(ValueError, match="q_norm"):
        W.read_weights(str(longer))


def _harness():
    from test_cpp_harness_gpu import build_harness
    return build_harness()


@pytest.mark.gpu
@pytest.mark.parametrize("chunk", [4096, 64 << 20])
def test_cpp_loader_uploads_every_tensor(cuda, chunk):
    """The C++ loader (two pinned staging buffers, chunk bytes each) puts every
    tensor on the GPU intact: each carved pointer copied back matches."""
    exe = _harness()
    res = subprocess.run([exe, "weights", FIX, str(chunk)], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    lines = res.stdout.splitlines()
    head = json.loads(lines[0])
    assert head["header"][:8] == [META["header"][k] for k in ("vocab_size", "hidden_size", "num_layers",
                                                               "num_heads", "num_kv_heads", "head_dim",
                                                               "intermediate_size", "max_seq_len")]
    assert lines[1] == "tokenizer " + META["tokenizer_json"]
    rows = [json.loads(x) for x in lines[2:]]
    exp = _expected()
    assert len(rows) == len(exp)
    for r, e in zip(rows, exp):
        _check(r["name"], r["n"], r["sum"], r["sumsq"], r["first"], e)


@pytest.mark.gpu
def test_cpp_loader_rejects_a_file_with_extra_tensors(cuda, tmp_path):
    exe = _harness()
    longer = tmp_path / "long.bin"
    longer.write_bytes(open(FIX, "rb").read() + b"\0" * 64)
    res = subprocess.run([exe, "weights", str(longer), "4096"], capture_output=True, text=True, timeout=120)
    assert res.returncode == 3 and "q_norm" in res.stderr


@pytest.mark.gpu
def test_python_upload_views(cuda):
    w = W.read_weights(FIX)
    buf, views = W.upload(w, cuda)
    assert buf.numel() == w.payload.size
    for name, arr in w.tensors.items():
        np.testing.assert_array_equal(views[name].cpu().numpy(), arr)


def _tiny_acts():
    base = os.path.join(ROOT, "tests", "golden", "tiny")
    h = META["header"]
    H, KVH, d, hid = h["num_heads"], h["num_kv_heads"], h["head_dim"], h["hidden_size"]
    S = 40

    def ld(name, cols):
        return np.fromfile(os.path.join(base, name + ".bin"), np.float16).reshape(S, cols)
    return (S, H, KVH, d, hid, h["rope_theta"]), {
        "q": ld("layer0_q_proj_out", H * d), "k": ld("layer0_k_proj_out", KVH * d),
        "v": ld("layer0_v_proj_out", KVH * d), "q_rope": ld("layer0_q_rope", H * d),
        "k_rope": ld("layer0_k_rope", KVH * d), "attn": ld("layer0_attn_out", H * d),
        "o_proj": ld("layer0_o_proj_out", hid)}


def test_oracle_on_the_exported_models_layer0():
    """The CPU oracle reproduces the reference generator's layer-0 dumps of the
    exported tiny model (head_dim 32), and the o_proj carved by the loader maps
    its attention output to the generator's o_proj output."""
    import oracle
    from _util import tensor_close_mismatches
    (S, H, KVH, d, hid, theta), g = _tiny_acts()
    cos, sin = oracle.rope_tables(512, d, theta)
    q, k = g["q"].copy(), g["k"].copy()
    oracle.rope_and_store_kv(q, k, None, None, None, cos, sin, S, H, KVH, d, H * d, KVH * d, 0, True)
    assert tensor_close_mismatches(q, g["q_rope"], 2e-2, 2e-2) == 0
    assert tensor_close_mismatches(k, g["k_rope"], 2e-2, 2e-2) == 0
    o16, _ = oracle.causal_attention(g["q_rope"], g["k_rope"], g["v"], S, H, KVH, d)
    assert tensor_close_mismatches(o16, g["attn"], 2e-2, 2e-2) == 0
    w = W.read_weights(FIX).tensors["layers.0.o_proj"].astype(np.float64)
    proj = g["attn"].astype(np.float64) @ w.T
    assert tensor_close_mismatches(proj, g["o_proj"], 2e-2, 2e-2) == 0


@pytest.mark.gpu
def test_exported_model_layer0_through_the_kernels(cuda):
    """weights.bin loaded and uploaded by the loader; the layer-0 projections the
    reference's generator dumped go through RoPE/append, causal prefill and the
    o_proj GEMM whose weight is the loader's carved layers.0.o_proj view; every
    stage against the generator's dump at the reference's tolerance."""
    import torch
    import b200attn
    from _gpu import dev, host
    from _util import tensor_close_mismatches
    (S, H, KVH, d, hid, theta), g = _tiny_acts()
    w = W.read_weights(FIX)
    _, views = W.upload(w, cuda)
    cos, sin = b200attn.rope_tables_host(512, d, theta)
    q, k, v = dev(g["q"]), dev(g["k"]), dev(g["v"])
    cache = b200attn.KVCache(1, 64, KVH, d, device=cuda)
    b200attn.launch_rope_and_store_kv(q, k, v, cache.get_k_cache(0), cache.get_v_cache(0), dev(cos), dev(sin), S, H,
                                      KVH, d, H * d, KVH * d, 0, True)
    attn = torch.empty((S, H * d), dtype=torch.float16, device=cuda)
    b200attn.launch_causal_attention_prefill(q, cache.get_k_cache(0), cache.get_v_cache(0), attn, S, H, KVH, d,
                                             H * d, KVH * d)
    out = torch.full((S, hid), float("nan"), dtype=torch.float16, device=cuda)
    b200attn.launch_attention_out_projection(attn, out, views["layers.0.o_proj"], S, hid, H, d, 0.0)
    torch.cuda.synchronize()
    assert tensor_close_mismatches(host(q), g["q_rope"], 2e-2, 2e-2) == 0
    assert tensor_close_mismatches(host(cache.get_k_cache(0))[:S], g["k_rope"], 2e-2, 2e-2) == 0
    assert tensor_close_mismatches(host(attn), g["attn"], 2e-2, 2e-2) == 0
    assert tensor_close_mismatches(host(out), g["o_proj"], 2e-2, 2e-2) == 0
