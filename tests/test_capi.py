"""CPU checks of the native boundary: libokc_b200.so loads without a GPU, exports every
symbol that include/okc_b200.h declares, and its argument validation rejects bad calls
before touching the device."""

import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_functions():
    src = (ROOT / "include" / "okc_b200.h").read_text()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(okc_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from okc_b200 import _lib
    return _lib.load()


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), n


def test_ctypes_signatures_cover_header():
    from okc_b200 import _lib
    assert sorted(_lib.SIGNATURES) == declared_functions()


def test_version(lib):
    assert lib.okc_version().decode().startswith("okc_b200")


def test_validation_without_device(lib):
    from okc_b200 import _lib
    # null pointers / bad shapes are rejected before any CUDA call
    assert lib.okc_gemm_bf16(None, 0, None, 0, None, 0, None, 1, 1, 1, 0, None, 0, None) == _lib.OKC_ERR_INVALID
    assert lib.okc_gemm_bf16(8, 8, 16, 8, 32, 8, None, 1, 8, 12, 0, None, 0, None) == _lib.OKC_ERR_INVALID  # K % 8
    assert lib.okc_gemm_bf16(8, 8, 16, 8, 32, 8, None, 1, 8, 8, 0, None, 0, None) == _lib.OKC_ERR_ALIGNMENT
    assert lib.okc_gemm_bf16(16, 8, 16, 8, 33, 8, None, 1, 8, 8, 0, None, 0, None) == _lib.OKC_ERR_ALIGNMENT
    assert lib.okc_attn_decode_fp8(16, 64, 16, 16, 16, 4, 16, 16, 16, 16, 64, 1, 9, 8, 64, 16, 4, 0.1, 1,
                                   None, 0, None) == _lib.OKC_ERR_INVALID  # Hq % Hkv
    assert lib.okc_attn_decode_fp8(16, 64, 16, 16, 16, 4, 16, 16, 16, 16, 64, 1, 8, 8, 96, 16, 4, 0.1, 1,
                                   None, 0, None) == _lib.OKC_ERR_INVALID  # D = 96
    assert lib.okc_moe_route(16, 16, 16, 16, None, 1, 100, 64, 8, 1, None) == _lib.OKC_ERR_INVALID  # H % 256
    assert lib.okc_moe_permute(16, 20000, 8, 0, 64, 8, 16, 16, 16, 16, 100, None) == _lib.OKC_ERR_INVALID


def test_workspace_queries(lib):
    from okc_b200 import _lib
    n = lib.okc_attn_decode_workspace_bytes(64, 64, 8, 128, 148)
    rows = (148 + 64) * 1 * 64
    assert n == (256 + ((rows * 8 + 255) // 256) * 256 + ((rows * 128 * 4 + 255) // 256) * 256
                 + ((64 + 1) * 4 + 255) // 256 * 256)  # + the unit prefix for the merge
    assert lib.okc_attn_decode_workspace_bytes(8, 8, 1, 128, 10) > lib.okc_attn_decode_workspace_bytes(8, 8, 8, 128, 10)
    assert lib.okc_moe_experts_workspace_bytes(256, 8, 4096, 1536) > 256
