"""The C-ABI library: builds, loads, exports every declared symbol, matches the
ctypes struct layouts and rejects bad arguments on the host (no GPU needed)."""
import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="session")
def lib():
    from estudiocanciones_b200 import _lib, build
    build.build()
    return _lib.lib()


def declared_functions():
    text = (ROOT / "include" / "heartmula_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\**\s+\**(hm_[a-z0-9_]+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "hm_gemv_i8" in names and "hm_decode_attn" in names and "hm_cfg_topk_sample" in names
    assert len(names) >= 15


def test_every_declared_symbol_is_exported(lib):
    from estudiocanciones_b200 import _lib
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} missing from the ctypes signature table"


def test_ctypes_layout_matches_library(lib):
    from estudiocanciones_b200 import _lib
    assert _lib.abi_mismatches() == []


def test_version(lib):
    assert b"sm_100a" in lib.hm_version()


def test_host_argument_validation_without_gpu(lib):
    from estudiocanciones_b200._lib import GemvDesc
    # every call below is rejected before any CUDA call is made
    assert lib.hm_gemv_i8(None, 0, None, None, None, 0, None, 0, 0, 64, 128, None, 0, None, 0, None, 0, 0, None) == -1
    d = GemvDesc()
    d.M, d.N, d.K = 8, 64, 100          # K not a multiple of 128
    assert lib.hm_gemv_i8_fused(C.byref(d), None) == -1
    assert lib.hm_decode_attn(None, None, None, None, None, 1, 1, 8, 3, 128, 16, 0.1, 1, None, 0, None, 0, None,
                              0, None) == -1
    assert lib.hm_cfg_topk_sample(None, 0, 2, 1, 8197, None, 0, 1.5, 50, 1.0, None, 0, 0, None, 0, None) == -1
    assert lib.hm_rmsnorm(None, None, None, 1, 16, 1e-5, None) == -1
    # frame commit: n_keep beyond the rows; checkpoint quantisation: null / short rows / bad type
    assert lib.hm_frame_commit(1, 1, 2, 8, 1, 3, None, 1, 0, None, 8193, 0, None) == -1
    assert lib.hm_q8_rows(None, 0, 4, 16, 16, 1, 16, 1, None) == -1
    assert lib.hm_q8_rows(1, 0, 4, 16, 8, 1, 16, 1, None) == -1      # ldx < K
    assert lib.hm_q8_rows(1, 0, 4, 16, 16, 1, 8, 1, None) == -1      # ldq < K
    assert lib.hm_q8_rows(1, 9, 4, 16, 16, 1, 16, 1, None) == -1     # no such element type
    assert lib.hm_q8_rows(1, 0, 0, 16, 16, 1, 16, 1, None) == -1     # no rows
    # TMA request-form queries: argument checks come before any tensor-map encoding
    assert lib.hm_gemv_box_form(None, 64, 128, 0) == -1
    assert lib.hm_gemv_box_form(16, 64, 100, 0) == -1                 # K not a multiple of 16
    assert lib.hm_gemv_box_form(16, 48, 128, 2) == -1                 # SiLU: N not a multiple of 32
    assert lib.hm_decode_attn_box_form(None, 64) == -1
    assert lib.hm_decode_attn_box_form(24, 64) == -1                  # cache not 16-byte aligned
    assert lib.hm_decode_attn_box_form(16, 0) == -1


def test_workspace_sizing_is_consistent(lib):
    # decode shapes at <= 8 rows stage their whole K: no split, no scratch
    for (M, N, K) in [(8, 5120, 3072), (1, 3072, 8192), (8, 8197, 3072), (8, 3072, 8192)]:
        assert lib.hm_gemv_pick_kspan(M, N, K, 0, 0) == K
        assert lib.hm_gemv_workspace_bytes(M, N, K, 0, 0) == 0
    # many rows x long K: split, scratch = splits * tiles * 16 rows * M * 4 bytes
    ks = lib.hm_gemv_pick_kspan(32, 1024, 8192, 0, 0)
    assert 8192 % ks == 0 and ks < 8192
    assert lib.hm_gemv_workspace_bytes(32, 1024, 8192, 0, 0) == (8192 // ks) * 64 * 16 * 32 * 4
    assert lib.hm_gemv_counters(5120, 0) == 320
    assert lib.hm_gemv_counters(16384, 2) == 8192 // 16
    assert lib.hm_decode_attn_workspace_bytes(8, 24, 128, 1) == 0
    assert lib.hm_decode_attn_workspace_bytes(8, 24, 128, 5) == 8 * 24 * 5 * 130 * 4
