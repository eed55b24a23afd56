"""The C-ABI library: loads, exports every declared symbol, validates arguments
before touching CUDA (CPU only, no GPU calls)."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

import b200attn
import oracle
from b200attn import _lib
from _util import ROOT

HEADER = os.path.join(ROOT, "include", "b200attn.h")


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    src = re.sub(r"//[^\n]*", "", src)
    return sorted(set(re.findall(r"\b(b2_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    syms = declared_symbols()
    assert len(syms) >= 15
    L = b200attn.lib()
    for s in syms:
        assert hasattr(L, s), f"{s} declared in include/b200attn.h but not exported"
    # and the Python binding knows every one of them
    assert set(syms) <= set(_lib.SIGNATURES), set(syms) - set(_lib.SIGNATURES)
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\b(b2_[a-z0-9_]+)\b", out))
    assert set(syms) <= exported


def test_constants_and_workspace_sizing():
    assert b200attn.KV_CHUNK == 256
    # include/model_inference.hpp:192-198: H * ceil(max_seq / KV_CHUNK) * (d + 2)
    assert b200attn.decode_workspace_floats(16, 128, 65536) == 16 * 256 * 130
    assert b200attn.decode_workspace_floats(16, 128, 4097) == 16 * 17 * 130
    assert b200attn.decode_workspace_floats(16, 128, 1) == 16 * 130
    for st in (0, 1, -1, -2, -3, -4, -5, -6, 99):
        assert isinstance(b200attn.lib().b2_status_string(st), bytes)


def test_rope_tables_match_oracle():
    for (n, d, theta) in [(4096, 128, 5.0e6), (300, 32, 1.0e4), (17, 64, 2.0e6)]:
        c, s = b200attn.rope_tables_host(n, d, theta)
        oc, os_ = oracle.rope_tables(n, d, theta)
        np.testing.assert_array_equal(c.view(np.uint16), oc.view(np.uint16))
        np.testing.assert_array_equal(s.view(np.uint16), os_.view(np.uint16))
    L = b200attn.lib()
    assert L.b2_fill_rope_tables(4, 7, 1.0, None, None) == -1


NULL = None


def test_silent_skips_match_reference_without_cuda():
    """The reference launchers return early on these; so does the C ABI, before any CUDA call."""
    L = b200attn.lib()
    fake = 0x1000
    # rope.hip.cpp:156 seq_len == 0
    assert L.b2_launch_rope_and_store_kv(fake, fake, fake, fake, fake, fake, fake, 0, 16, 4, 128, 0, 0, 0, True, NULL) == 1
    # causal_attention.hip.cpp:392-399 prefill: seq 0, kv heads 0, H % KVH != 0
    assert L.b2_launch_causal_attention_prefill(fake, fake, fake, fake, 0, 16, 4, 128, 0, 0, NULL) == 1
    assert L.b2_launch_causal_attention_prefill(fake, fake, fake, fake, 8, 16, 0, 128, 0, 0, NULL) == 1
    assert L.b2_launch_causal_attention_prefill(fake, fake, fake, fake, 8, 16, 5, 128, 0, 0, NULL) == 1
    # :860-866 decode: query_len 0, kv_len 0, kv heads 0, H % KVH != 0; :945 head_dim 0
    args = (fake,) * 7
    for ql, kl, h, kvh, d in [(0, 5, 16, 4, 128), (1, 0, 16, 4, 128), (1, 5, 16, 0, 128), (1, 5, 16, 3, 128),
                              (1, 5, 16, 4, 0)]:
        for fn in (L.b2_launch_causal_attention_decode, L.b2_launch_causal_attention_decode_vectorized):
            assert fn(*args, ql, kl, 0, h, kvh, d, 0, 0, NULL, None, None) == 1


def test_invalid_arguments_are_errors_not_launches():
    L = b200attn.lib()
    fake = 0x1000
    # NoPE append needs a cache (the reference would write through a null pointer)
    assert L.b2_launch_rope_and_store_kv(fake, fake, fake, None, None, fake, fake, 4, 16, 4, 128, 0, 0, 0, False, NULL) == -1
    # odd head_dim cannot be rotated in halves
    assert L.b2_launch_rope_and_store_kv(fake, fake, fake, fake, fake, fake, fake, 4, 16, 4, 127, 0, 0, 0, True, NULL) == -1
    # null buffers
    assert L.b2_launch_causal_attention_prefill(None, fake, fake, fake, 8, 16, 4, 128, 0, 0, NULL) == -1
    assert L.b2_launch_causal_attention_decode(fake, fake, fake, fake, None, fake, fake, 1, 5, 4, 16, 4, 128, 0, 0,
                                               NULL, None, None) == -1
    assert L.b2_launch_merge_attention_decode_tiled(None, fake, fake, fake, 16, 3, 128, NULL) == -1
    # graph patchers reject a null exec
    assert L.b2_update_rope_and_store_kv_node(None, fake, 3, True) == -1
    assert L.b2_update_causal_attention_decode_node(None, fake, 3) == -1
    assert L.b2_update_merge_attention_decode_node(None, fake, 3) == -1
    # over-long decode (more chunks than a grid dimension)
    assert L.b2_launch_causal_attention_decode(fake, fake, fake, fake, fake, fake, fake, 1, 65536 * 256 + 1, 0, 16, 4,
                                               128, 0, 0, NULL, None, None) == -2
    with pytest.raises(b200attn.B2Error):
        b200attn.launch_causal_attention_prefill(None, fake, fake, fake, 8, 16, 4, 128)


def test_python_api_mirrors_reference_signatures():
    """Same parameter names and order as include/kernels/kernels.hpp (reference)."""
    import inspect
    expect = {
        "launch_rope": "d_q d_k d_cos d_sin seq_len num_heads num_kv_heads head_dim q_stride k_stride start_pos",
        "launch_rope_and_store_kv": "d_q d_k d_v d_k_cache d_v_cache d_cos d_sin seq_len num_heads num_kv_heads "
                                    "head_dim q_stride k_stride start_pos apply_rotation stream",
        "update_rope_and_store_kv_node": "graph_exec node start_pos apply_rotation",
        "launch_causal_attention_prefill": "d_q d_k d_v d_out seq_len num_heads num_kv_heads head_dim q_stride "
                                           "kv_stride",
        "launch_causal_attention_decode": "d_q d_k_cache d_v_cache d_out d_partial_out d_partial_max "
                                          "d_partial_weight_sum query_len kv_cache_len start_pos num_heads "
                                          "num_kv_heads head_dim q_stride kv_stride stream",
        "launch_causal_attention_decode_vectorized": "d_q d_k_cache d_v_cache d_out d_partial_out d_partial_max "
                                                     "d_partial_weight_sum query_len kv_cache_len start_pos "
                                                     "num_heads num_kv_heads head_dim q_stride kv_stride stream",
        "update_merge_attention_decode_node": "graph_exec node kv_cache_len",
        "update_causal_attention_decode_node": "graph_exec node kv_cache_len",
        "launch_merge_attention_decode_tiled": "d_partial_output d_partial_max d_partial_weight_sum d_out "
                                               "num_heads num_kv_chunks head_dim stream",
    }
    for name, params in expect.items():
        got = list(inspect.signature(getattr(b200attn, name)).parameters)
        want = params.split()
        assert got[:len(want)] == want, (name, got)


def test_kv_cache_layout_and_bookkeeping():
    torch = pytest.importorskip("torch")
    cache = b200attn.KVCache(3, 10, 4, 8, device="cpu")
    base = cache.buffer.data_ptr()
    kv_dim = 32
    for l in range(3):
        assert cache.get_k_cache(l).data_ptr() == base + 2 * (l * 2 * 10 * kv_dim)
        assert cache.get_v_cache(l).data_ptr() == base + 2 * (l * 2 * 10 * kv_dim + 10 * kv_dim)
    cache.set_cached_len(10)
    with pytest.raises(IndexError):
        cache.set_cached_len(11)
    cache.reset_cache()
    assert cache.get_cached_len() == 0
    with pytest.raises(ValueError):
        b200attn.launch_rope(torch.zeros(4), 0x10, 0x10, 0x10, 1, 1, 1, 2, 0, 0)


def test_cpp_shim_header_compiles():
    shim = os.path.join(ROOT, "include", "kernels", "kernels.hpp")
    if not os.path.exists(shim):
        pytest.fail("include/kernels/kernels.hpp missing")
    src = ('#include "kernels/kernels.hpp"\n#include "b200attn/kv_cache.hpp"\n#include "b200attn/rope_cache.hpp"\n'
           'int main() { static_assert(KV_CHUNK == 256, ""); return 0; }\n')
    res = subprocess.run(["g++", "-std=c++20", "-fsyntax-only", "-x", "c++", "-", f"-I{ROOT}/include",
                          "-I/usr/local/cuda/include"], input=src, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr


def test_fused_decode_step_validation_without_cuda():
    """b2_launch_decode_step_fused checks everything before its first CUDA call."""
    L = b200attn.lib()
    f = 0x1000
    ws = L.b2_decode_step_workspace_bytes(16, 4)
    assert ws % 256 == 0 and ws >= 16 * (256 * 130) * 4   # one partial per split and head
    assert L.b2_decode_step_workspace_bytes(32, 8) > 0 and L.b2_decode_step_workspace_bytes(16, 0) == 0

    def call(q=f, kn=f, vn=f, kc=f, vc=f, cos=f, sin=f, rows=100, rot=True, pos=f, ln=f, bias=1, cap=99, out=f,
             w=f, wb=ws, h=16, kvh=4, d=128):
        return L.b2_launch_decode_step_fused(q, kn, vn, kc, vc, cos, sin, rows, rot, pos, ln, bias, cap, out, w, wb,
                                             h, kvh, d, NULL)
    assert call(cap=0) == 1 and call(kvh=0) == 1 and call(kvh=3) == 1          # silent skips
    assert call(q=None) == -1 and call(ln=None) == -1 and call(w=None) == -1   # null buffers
    assert call(out=None) == -1
    assert call(vn=None) == -1                                                 # K without V
    assert call(cos=None) == -1 and call(pos=None) == -1 and call(rows=0) == -1  # RoPE inputs
    # NoPE needs none of them: this call gets as far as the workspace check
    assert call(rot=False, cos=None, sin=None, pos=None, rows=0, wb=ws - 1) == -5
    assert call(d=64) == -2 and call(h=48, kvh=4) == -2 and call(kvh=16, h=16) == -2
    assert call(cap=1 << 31) == -2
    assert call(kc=f + 2) == -3 and call(w=f + 8) == -3
    assert call(wb=ws - 1) == -5
    r = L.b2_launch_decode_step_fused_rank_partial(f, None, None, f, f, f, f, 100, True, f, f, 0, 99, None, f, f, f,
                                                   ws, 16, 4, 128, NULL)
    assert r == -1


def test_ragged_decode_validation_without_cuda():
    """b2_launch_causal_attention_decode_ragged / _rope_..._ragged check before any CUDA call."""
    L = b200attn.lib()
    f = 0x1000
    ws = L.b2_decode_ragged_workspace_bytes(64, 16, 4, 16384)
    assert ws % 256 == 0 and ws > 64 * 16 * 130 * 4
    assert L.b2_decode_ragged_workspace_bytes(64, 16, 3, 16384) == 0

    def call(q=f, qs=0, k=f, v=f, cs=0, ln=f, bias=0, mx=4096, out=f, os_=0, B=8, H=16, KVH=4, d=128, w=f, wb=ws):
        return L.b2_launch_causal_attention_decode_ragged(q, qs, k, v, cs, ln, bias, mx, out, os_, B, H, KVH, d, w,
                                                          wb, NULL)
    assert call(B=0) == 1 and call(mx=0) == 1 and call(KVH=3) == 1
    assert call(q=None) == -1 and call(ln=None) == -1 and call(w=None) == -1
    assert call(d=64) == -2 and call(B=2000) == -2 and call(H=48) == -2
    assert call(cs=100) == -1 and call(qs=8) == -1            # overlapping caches / rows
    assert call(k=f + 2) == -3 and call(qs=2052) == -3
    assert call(wb=16) == -5
    assert L.b2_launch_rope_and_store_kv_ragged(f, f, f, f, f, 0, f, f, 4, 16, 4, 128, 0, 0, None, 64, True,
                                                NULL) == -1
    assert L.b2_launch_rope_and_store_kv_ragged(f, f, f, f, f, 100, f, f, 4, 16, 4, 128, 0, 0, f, 64, True,
                                                NULL) == -1


def test_fused_ragged_step_validation_without_cuda():
    """b2_launch_decode_step_ragged_fused checks everything before its first CUDA call."""
    L = b200attn.lib()
    f = 0x1000
    ws = L.b2_decode_ragged_workspace_bytes(8, 16, 4, 4096)

    def call(q=f, qs=0, kn=f, vn=f, kns=0, k=f, v=f, cs=0, cos=f, sin=f, rows=4096, rot=True, pos=f, mx=4096,
             out=f, os_=0, B=8, H=16, KVH=4, d=128, w=f, wb=ws):
        return L.b2_launch_decode_step_ragged_fused(q, qs, kn, vn, kns, k, v, cs, cos, sin, rows, rot, pos, mx, out,
                                                    os_, B, H, KVH, d, w, wb, NULL)
    assert call(B=0) == 1 and call(mx=0) == 1 and call(KVH=3) == 1            # silent skips
    assert call(q=None) == -1 and call(pos=None) == -1 and call(w=None) == -1
    assert call(vn=None) == -1                                                 # K without V
    assert call(cos=None) == -1 and call(rows=0) == -1                         # RoPE inputs
    assert call(kns=100) == -1                                                 # K/V rows overlap
    assert call(d=64) == -2 and call(B=2000) == -2
    assert call(kn=f + 4) == -3 and call(kns=516) == -3 and call(cos=f + 2) == -3
    # NoPE needs no tables: this call gets as far as the workspace check
    assert call(rot=False, cos=None, sin=None, rows=0, wb=16) == -5
    assert L.b2_launch_rope_and_store_kv_ragged(f, f, f, f, f, 0, f, f, 0, 16, 4, 128, 0, 0, f, 64, True,
                                                NULL) == 1


def test_python_bindings_match_header():
    """Every function include/b200attn.h declares is bound in the ctypes table
    with the same number of parameters (guards the Python mirror against ABI
    drift)."""
    import re
    from b200attn._lib import SIGNATURES
    src = open(os.path.join(ROOT, "include", "b200attn.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    src = re.sub(r"//.*", "", src)
    decls = re.findall(r"\b(?:int|size_t|unsigned int|uint64_t|const char\s*\*|void)\s+\*?\s*(b2_\w+)\s*\(([^)]*)\)\s*;",
                       src)
    assert len(decls) >= 30
    for name, args in decls:
        args = args.strip()
        n = 0 if args in ("", "void") else len(args.split(","))
        assert name in SIGNATURES, name
        assert len(SIGNATURES[name][1]) == n, (name, n, len(SIGNATURES[name][1]))
