"""Build freshness (llm-inference_b200/build.py): the library is reused only
when the hash of its sources, headers, flags and nvcc version matches the one
recorded at link time. CPU only (nothing is compiled here unless the library
is missing or stale)."""
import os

from _util import load_build_module


def test_hash_recorded_and_reused():
    b = load_build_module()
    b.build(quiet=True)
    assert os.path.exists(b.LIB) and os.path.exists(b.STAMP)
    assert b.built_hash() == b.source_hash()
    assert not b.needs_build()


def test_hash_covers_flags_and_is_path_independent(monkeypatch):
    b = load_build_module()
    h0 = b.source_hash()
    assert h0 == b.source_hash()                 # deterministic
    monkeypatch.setattr(b, "NVCC_FLAGS", b.NVCC_FLAGS + ["-DB2_SOMETHING_ELSE"])
    assert b.source_hash() != h0                 # a flag change forces a rebuild
    monkeypatch.undo()
    # checkout paths are hashed relative to the repository root
    assert all(b.REPO_ROOT not in f.replace(b.REPO_ROOT, ".") for f in b.NVCC_FLAGS)


def test_stale_stamp_means_rebuild(monkeypatch):
    b = load_build_module()
    monkeypatch.setattr(b, "built_hash", lambda: "0" * 64)
    assert b.needs_build()
