"""`NativeEngine` boundary checks that need no GPU (`seedplane/native.py:18-23,49,58`)."""
import pytest

from seedplane_b200.native import NativeEngine, find_engine


def test_missing_engine_raises_file_not_found(tmp_path, monkeypatch):
    monkeypatch.setenv("SEEDPLANE_NATIVE_ENGINE", str(tmp_path / "nope.so"))
    import seedplane_b200._native as N
    monkeypatch.setattr(N, "LIB_PATH", tmp_path / "missing.so")
    with pytest.raises(FileNotFoundError):
        find_engine(None)
    with pytest.raises(FileNotFoundError):
        NativeEngine(tmp_path, engine=str(tmp_path / "also-missing.so"))


def test_explicit_and_env_engine_resolution(tmp_path, monkeypatch):
    lib = tmp_path / "libseedplane_cuda.so"
    lib.write_bytes(b"")
    assert find_engine(str(lib)) == str(lib)
    monkeypatch.setenv("SEEDPLANE_NATIVE_ENGINE", str(lib))
    assert find_engine(None) == str(lib)
