"""The C-ABI library loads, exports every entry point include/sdtw_b200.h
declares, and rejects bad arguments before touching a device."""
import ctypes
import os
import re

import pytest

from conftest import ROOT
from softdtw_cuda import _native

HEADER = os.path.join(ROOT, "include", "sdtw_b200.h")


def _declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(sdtw_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = _declared()
    assert "sdtw_forward_f32" in names and "sdtw_backward_xy_f32" in names


def test_library_exports_every_declared_symbol():
    L = ctypes.CDLL(_native.LIB_PATH)
    missing = [n for n in _declared() if not hasattr(L, n)]
    assert not missing, f"not exported: {missing}"
    assert set(_declared()) <= set(_native.EXPORTED), "binding lacks a signature for a declared symbol"


def test_sizes_without_gpu():
    L = _native.lib()
    n_diag = (64 + 31 + 15) // 16 * 16 + 16  # anti-diagonal rows per stripe, padded
    assert L.sdtw_score_elems(4, 64, 64) == 2 * 4 * 2 * n_diag * 32   # (hi, lo) per cell
    assert L.sdtw_score_elems(0, 4, 4) == 0
    cells = 4 * 2 * n_diag * 32
    assert L.sdtw_cost_elems(4, 64, 64) == cells
    # More than one stripe: the band-wrap ring (B x M slots of 16 bytes, sized
    # for any plan a pass may pick), then the wavefront-layout table of the
    # cost / E.
    assert L.sdtw_workspace_bytes(4, 64, 64) == -(-4 * 64 * 16 // 256) * 256 + -(-cells * 4 // 256) * 256
    # One stripe: no ring.
    assert L.sdtw_workspace_bytes(4, 32, 64) == -(-(4 * 1 * n_diag * 32) * 4 // 256) * 256
    # x/y backward adds the gradient operands.
    up = lambda v: -(-v // 256) * 256
    # Up to 16 features: column sums per split of 8 stripes (B x splits x M x
    # (4 + 1) floats for dim <= 4).
    assert L.sdtw_workspace_bytes_xy(4, 64, 64, 3) == L.sdtw_workspace_bytes(4, 64, 64) + up(4 * 1 * 64 * 5 * 4)
    assert L.sdtw_workspace_bytes_xy(2, 300, 40, 9) == L.sdtw_workspace_bytes(2, 300, 40) + up(2 * 2 * 40 * 17 * 4)
    # More features, one 128-row tile each way: G, G^T, x^T, y^T row-major with rows padded to 32.
    assert L.sdtw_workspace_bytes_xy(4, 64, 64, 20) == L.sdtw_workspace_bytes(4, 64, 64) + 2 * up(4 * 64 * 64 * 4) + 2 * up(4 * 20 * 64 * 4)
    # Longer: x, y chunked and transposed, rows of 36 floats per 32 positions.
    assert L.sdtw_workspace_bytes_xy(4, 200, 64, 20) == L.sdtw_workspace_bytes(4, 200, 64) + up(4 * 7 * 20 * 36 * 4) + up(4 * 2 * 20 * 36 * 4)
    # normalize: the x/y workspace of the 3B problems, then four (B,N,dim)
    # gradient blocks of the self pairs.
    for B, N, dim in ((4, 64, 3), (2, 200, 20)):
        assert L.sdtw_workspace_bytes_norm(B, N, dim) == up(L.sdtw_workspace_bytes_xy(3 * B, N, N, dim)) + 4 * up(B * N * dim * 4)
    assert L.sdtw_workspace_bytes_norm(0, 64, 3) == 0


def test_invalid_arguments_rejected():
    L = _native.lib()
    rc = L.sdtw_forward_f32(None, None, None, 0, 4, 4, 1.0, -1.0, None, 0, None)
    assert rc == 1
    assert b"must be > 0" in L.sdtw_last_error_message()
    rc = L.sdtw_forward_f32(None, None, None, 1, 4, 4, -1.0, -1.0, None, 0, None)
    assert rc == 1 and b"gamma" in L.sdtw_last_error_message()
    rc = L.sdtw_cost_sqeuclid_f32(None, None, None, 1, 4, 4, 0, 0, None)
    assert rc == 1
    assert L.sdtw_error_string(3) == b"device-side wait timed out"
    rc = L.sdtw_forward_xy_norm_f32(None, None, None, None, 0, 4, 3, 1.0, -1.0, None, 0, None)
    assert rc == 1 and b"must be > 0" in L.sdtw_last_error_message()
    rc = L.sdtw_backward_sqeuclid_norm_f32(None, None, None, None, None, None, None, 1, 4, 3, 0.0, -1.0, None, 0, None)
    assert rc == 1 and b"gamma" in L.sdtw_last_error_message()
    rc = L.sdtw_grad_sqeuclid_f64(None, None, None, None, None, 2, 4, 4, 3, None)
    assert rc == 1 and b"null pointer" in L.sdtw_last_error_message()
    rc = L.sdtw_grad_sqeuclid_f64(None, None, None, None, None, 0, 4, 4, 3, None)
    assert rc == 1 and b"must be > 0" in L.sdtw_last_error_message()


def test_timing_registry_without_gpu():
    _native.timing_enable(True)
    assert _native.timing_read() == {}
    _native.timing_enable(False)


def test_version():
    assert "sm_100a" in _native.version()


def test_native_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_native, "_lib", None)
    monkeypatch.setattr(_native, "LIB_PATH", str(tmp_path / "nope.so"))
    with pytest.raises(RuntimeError, match="native library"):
        _native.lib()
