"""Decode through b2_launch_causal_attention_decode_noalloc, the entry point for
callers that cannot hand the library scratch memory (a plugin host that passes
only inputs and outputs, a memory pool that owns all of HBM, a thread that must
not call cudaMalloc). Its split partials live in a fixed device array inside
the library; the output must match the workspace entry point's.

Named to be collected last, so a run that stops at the first failure has run
every other test first; it also passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest

import b200attn
from _util import assert_attention_close, seeded_f16

pytestmark = pytest.mark.gpu


def _noalloc(q, k, v, out, kv_len, H, KVH, d, kv_stride=0):
    L = b200attn.lib()
    return L.b2_launch_causal_attention_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                                       1, kv_len, H, KVH, d, kv_stride, None)


def _with_workspace(q, k, v, out, kv_len, H, KVH, d, kv_stride=0):
    import torch
    n = b200attn.decode_workspace_floats(H, d, kv_len)
    ws = torch.empty(n, dtype=torch.float32, device=q.device)
    c = H * ((kv_len + 255) // 256)
    L = b200attn.lib()
    return L.b2_launch_causal_attention_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                               ws.data_ptr(), ws[c * d:].data_ptr(), ws[c * (d + 1):].data_ptr(),
                                               1, kv_len, kv_len - 1, H, KVH, d, 0, kv_stride, None, None, None)


def test_noalloc_decode_matches_workspace_decode_twice(cuda):
    import torch
    H, KVH, d = 16, 4, 128
    # two calls in a row with different lengths and data: the second must not
    # see anything the first left in the shared array
    for kv_len, seed in ((65537, 1), (3000, 2)):
        k = torch.from_numpy(seeded_f16((kv_len, KVH * d), seed, std=0.5)).to(cuda)
        v = torch.from_numpy(seeded_f16((kv_len, KVH * d), seed + 10, std=0.5)).to(cuda)
        q = torch.from_numpy(seeded_f16(H * d, seed + 20)).to(cuda)
        got = torch.full((H * d,), float("nan"), dtype=torch.float16, device=cuda)
        ref = torch.full((H * d,), float("nan"), dtype=torch.float16, device=cuda)
        assert _noalloc(q, k, v, got, kv_len, H, KVH, d) == 0
        torch.cuda.synchronize()
        assert _with_workspace(q, k, v, ref, kv_len, H, KVH, d) == 0
        torch.cuda.synchronize()
        g = got.cpu().numpy()
        r = ref.cpu().numpy()
        assert np.all(np.isfinite(g.astype(np.float32)))
        assert_attention_close(g, r.astype(np.float32))
    assert b200attn.lib().b2_device_error_word() == 0


def test_noalloc_decode_strided_cache_path(cuda):
    """Rows read from interleaved [Q|K|V] rows (stride 3072) take the register
    kernel; the no-workspace entry point follows it too."""
    import torch
    H, KVH, d, L_, stride = 16, 4, 128, 2049, 3072
    k = torch.from_numpy(seeded_f16(L_ * stride, 31)).to(cuda)
    v = torch.from_numpy(seeded_f16(L_ * stride, 32)).to(cuda)
    q = torch.from_numpy(seeded_f16(H * d, 33)).to(cuda)
    got = torch.empty(H * d, dtype=torch.float16, device=cuda)
    ref = torch.empty(H * d, dtype=torch.float16, device=cuda)
    for _ in range(2):
        assert _noalloc(q, k, v, got, L_, H, KVH, d, stride) == 0
        assert _with_workspace(q, k, v, ref, L_, H, KVH, d, stride) == 0
        torch.cuda.synchronize()
        assert_attention_close(got.cpu().numpy(), ref.cpu().numpy().astype(np.float32))


def test_noalloc_rejects_sizes_beyond_the_array(cuda):
    import torch
    L = b200attn.lib()
    limit = 4 * 1024 * 1024 // 4
    H, KVH, d = 16, 4, 128
    max_len = (limit // (H * (d + 2))) * 256          # largest accepted kv_len
    assert b200attn.decode_workspace_floats(H, d, max_len) <= limit
    assert b200attn.decode_workspace_floats(H, d, max_len + 1) > limit
    dummy = torch.zeros(8, dtype=torch.float16, device=cuda)
    p = dummy.data_ptr()
    assert L.b2_launch_causal_attention_decode_noalloc(p, p, p, p, 1, max_len + 1, H, KVH, d, 0, None) == -5
    assert b"workspace" in L.b2_status_string(-5)
    # the reference's silent cases stay silent
    assert L.b2_launch_causal_attention_decode_noalloc(p, p, p, p, 1, 0, H, KVH, d, 0, None) == 1
    assert L.b2_launch_causal_attention_decode_noalloc(p, p, p, p, 1, 5, H, 3, d, 0, None) == 1
