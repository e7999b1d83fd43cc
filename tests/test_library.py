"""The C ABI library: it loads, exports every symbol include/iris_b200.h
declares, and rejects bad arguments before touching the device (no GPU needed:
every call here fails validation, which runs before any CUDA call)."""

import ctypes
import re
from pathlib import Path

import pytest

from conftest import REPO

HEADER = REPO / "include" / "iris_b200.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(iris_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from iris_b200 import _lib
    from iris_b200.build import build

    build()  # no-op when up to date; nvcc cross-compiles without a GPU
    return _lib.load()


def test_library_exports_every_declared_symbol(lib):
    symbols = declared_symbols()
    assert len(symbols) >= 20
    for name in symbols:
        assert hasattr(lib, name), name
    from iris_b200 import _lib

    assert sorted(_lib.exported_symbols()) == symbols
    assert lib.iris_abi_version() == 1


def test_binding_signatures_match_header(lib):
    """Each ctypes signature has as many arguments as the C declaration."""
    from iris_b200 import _lib

    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    for name, argtypes in _lib.SIGNATURES.items():
        decl = re.search(rf"\b{name}\s*\((.*?)\);", text, flags=re.S).group(1)
        assert len([a for a in decl.split(",") if a.strip()]) == len(argtypes), name


def _einval(lib, name, *args):
    fn = getattr(lib, name)
    assert fn(*args) == 1, name
    return lib.iris_last_error().decode()


def test_invalid_calls_are_rejected_before_launch(lib):
    msg = _einval(lib, "iris_qk_norm_rope", None, 1, 1, 1, 128, -1, 1, None, None, None, 1e-6, None, 1, 1, 0, None)
    assert re.search("positive.*nonnegative", msg)
    msg = _einval(lib, "iris_gemm_bf16", 16, 12, 16, 12, 16, 1, 32, 32, 32, 12, 0, None, None, 0, 32, 0, 0, 32, 0, 0, None)
    assert "multiples of 8" in msg
    msg = _einval(lib, "iris_rms_norm_modulate", 16, 0, 1, 0, 0, 16, 1, 16, 16, 16, 0, 1, 1, 100, 1e-6, None)
    assert "width % 128" in msg
    msg = _einval(lib, "iris_flash_attn_fwd", 16, 16, 16, 16, 1, 3, 2, 10, 128, 0.1, 384, None)
    assert "multiple of heads_kv" in msg
    msg = _einval(lib, "iris_patchify", 16, 16, 1, 3, 30, 32, 16, 0, 1, None)
    assert "divisible by patch_size" in msg
    msg = _einval(lib, "iris_patchify", 16, 16, 1, 3, 32, 32, 16, 3, 2, None)
    assert "token range" in msg
    msg = _einval(lib, "iris_block_copy", 16, 16, 16, 16, 16, 16, 16, 16, 1, 1, 1, 24, None)
    assert "multiples of 16" in msg
    msg = _einval(lib, "iris_timestep_embedding", 16, 16, 1, 255, 10.0, None)
    assert "even" in msg


def test_python_wrappers_reject_cpu_tensors_and_bad_offsets():
    import torch

    from iris_b200 import kernels

    x = torch.ones(1, 2, 128)
    weight = torch.ones(128)
    cos, sin = torch.ones(2, 64), torch.zeros(2, 64)
    for options in ({"col_offset": -1}, {"offset": -1}, {"heads": 0}):
        with pytest.raises(ValueError, match="positive.*nonnegative"):
            kernels.qk_norm_rope(x, weight, cos, sin, 1e-6, **{"heads": 1, **options})
    with pytest.raises(ValueError, match="CUDA"):
        kernels.qk_norm_rope(x, weight, cos, sin, 1e-6, 1)
    with pytest.raises(ValueError, match="FP32"):
        kernels.rms_norm_modulate(torch.ones(1, 2, 128), weight.bfloat16(), torch.zeros(1, 1, 128),
                                  torch.zeros(1, 1, 128), 1e-6, torch.bfloat16)  # fmt: skip


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    from iris_b200 import _lib

    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIBRARY", tmp_path / "libiris_b200.so")
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.load()


def test_sources_name_no_cluster_multicast_loads():
    """Multi-GPU runs must not reach a TMA load with cluster multicast."""
    csrc = REPO / "iris-3b-metal_b200" / "csrc"
    for path in list(csrc.glob("*.cu")) + list(csrc.glob("*.cuh")) + list(csrc.glob("*.h")):
        assert "multicast" not in path.read_text(), path
