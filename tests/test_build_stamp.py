"""The in-tree extension carries a digest of the sources it was compiled from: a stale build (sources
edited, extension not rebuilt) is detected instead of silently testing old kernels."""
import shutil

import pytest

from qwen38_b200.ops import build


def test_digest_tracks_source_content(tmp_path, monkeypatch):
    for name in ("misc.cu", "common.cuh"):
        shutil.copy(f"{build.CSRC}/{name}", tmp_path / name)
    monkeypatch.setattr(build, "CSRC", str(tmp_path))
    d0 = build.sources_digest()
    assert d0 == build.sources_digest()
    (tmp_path / "common.cuh").write_text((tmp_path / "common.cuh").read_text() + "\n// edit\n")
    d1 = build.sources_digest()
    assert d1 != d0
    (tmp_path / "extra.cu").write_text("// new file\n")
    assert build.sources_digest() != d1


def test_built_extension_matches_sources():
    st = build.stale()
    if st is None:
        pytest.skip("no built extension with a source stamp")
    assert st is False, "the extension is older than its sources: rebuild with __graft_entry__.build()"
