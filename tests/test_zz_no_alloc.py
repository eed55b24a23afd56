"""Decode through b2_launch_causal_attention_decode_noalloc, the entry point for
callers that cannot hand the library scratch memory (a plugin host that passes
only inputs and outputs, a memory pool that owns all of HBM, a thread that must
not call cudaMalloc). Its split partials live in a fixed device array inside
the library; the output must match the workspace entry point's.

Named to be collected last, so a run that stops at the first failure has run
every other test first; it also passes alone in a fresh process. Outputs are
checked against the FP32 CPU oracle as well as the workspace entry point."""
import ctypes

import numpy as np
import pytest

import b200attn
from _util import assert_attention_close, seeded_f16

pytestmark = pytest.mark.gpu

B2_NOALLOC_FLOATS = 4 * 1024 * 1024 // 4   # B2_NOALLOC_SCRATCH_BYTES / sizeof(float)


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


def _check_pair(cuda, kv_len, seed, H=16, KVH=4, d=128):
    """One no-workspace call and one workspace call on the same seeded inputs:
    both within the acceptance bar of the FP32 oracle, and of each other."""
    import torch
    import oracle
    kh = seeded_f16((kv_len, KVH * d), seed, std=0.5)
    vh = seeded_f16((kv_len, KVH * d), seed + 10, std=0.5)
    qh = seeded_f16(H * d, seed + 20)
    k, v, q = (torch.from_numpy(x).to(cuda) for x in (kh, vh, qh))
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
    _, o32 = oracle.decode_attention(qh, kh, vh, kv_len, H, KVH, d)
    assert_attention_close(g, o32.reshape(-1))


def test_noalloc_decode_matches_workspace_decode_twice(cuda):
    # calls in a row with different lengths and data: a call must not see
    # anything an earlier one left in the shared array, whether the earlier
    # call was longer (more partial rows) or shorter
    for kv_len, seed in ((65537, 1), (3000, 2), (65537, 3)):
        _check_pair(cuda, kv_len, seed)
    assert b200attn.lib().b2_device_error_word() == 0


def test_noalloc_decode_at_the_largest_accepted_length(cuda):
    """129,024 cached tokens at 16 heads x 128: the partials fill 1,048,320 of
    the array's 1,048,576 floats (TMA path, 4 KV heads)."""
    H, KVH, d = 16, 4, 128
    max_len = (B2_NOALLOC_FLOATS // (H * (d + 2))) * 256
    assert max_len == 129024
    assert b200attn.decode_workspace_floats(H, d, max_len) == 1048320
    _check_pair(cuda, max_len, 5)
    _check_pair(cuda, 4097, 6)
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
    limit = B2_NOALLOC_FLOATS
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
