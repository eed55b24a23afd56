"""Shared test helpers (golden fixtures, the reference's tolerance check)."""
from __future__ import annotations

import importlib.util
import json
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")

# Acceptance bar for attention outputs against the FP32 CPU oracle.
MAX_ABS = 1e-2
REL_L2 = 2e-3


def load_build_module():
    path = os.path.join(ROOT, "llm-inference_b200", "build.py")
    spec = importlib.util.spec_from_file_location("b200attn_build", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def golden(subset: str = ""):
    """The committed fixtures: the 40-token set, or subset "sharp" (160 tokens,
    peaked softmax)."""
    base = os.path.join(GOLDEN, subset) if subset else GOLDEN
    meta = json.load(open(os.path.join(base, "meta.json")))
    S, H, KVH, d = meta["seq_len"], meta["num_heads"], meta["num_kv_heads"], meta["head_dim"]

    def ld(name, cols):
        return np.fromfile(os.path.join(base, name + ".bin"), dtype=np.float16).reshape(S, cols)

    return meta, {
        "q": ld("layer0_q_proj_out", H * d), "k": ld("layer0_k_proj_out", KVH * d),
        "v": ld("layer0_v_proj_out", KVH * d), "q_rope": ld("layer0_q_rope", H * d),
        "k_rope": ld("layer0_k_rope", KVH * d), "attn": ld("layer0_attn_out", H * d),
    }


def tensor_close_mismatches(actual, expected, atol, rtol) -> int:
    """tests/test_utils.hpp:30-62: |a - e| <= atol + rtol * |e| elementwise."""
    a = np.asarray(actual, dtype=np.float32)
    e = np.asarray(expected, dtype=np.float32)
    assert a.shape == e.shape, (a.shape, e.shape)
    return int(np.count_nonzero(~(np.abs(a - e) <= atol + rtol * np.abs(e))))


def max_abs(a, b) -> float:
    return float(np.max(np.abs(np.asarray(a, np.float32) - np.asarray(b, np.float32))))


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def assert_attention_close(actual, expected32):
    """max-abs <= 1e-2 and relative L2 <= 2e-3 against the FP32 oracle."""
    ma, rl = max_abs(actual, expected32), rel_l2(actual, expected32)
    assert np.all(np.isfinite(np.asarray(actual, np.float32)))
    assert ma <= MAX_ABS and rl <= REL_L2, f"max_abs={ma:.3g} rel_l2={rl:.3g}"
    return ma, rl


def seeded_f16(shape, seed, std=1.0):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(shape, dtype=np.float32) * std).astype(np.float16)
