"""The C-ABI library (no GPU needed): it loads, exports every function that
include/*.h declares with the binding's signature, and its host-only
functions agree with the oracle and the reference's ring order."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from aws_training_study_b200 import _capi
from oracle import pcp_oracle as orc

HEADERS = sorted((Path(__file__).resolve().parents[1] / "include").glob("*.h"))


def declared_functions() -> list[str]:
    names = []
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(pcp_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_library_exports_every_declared_function():
    lib = _capi.lib()
    names = declared_functions()
    assert len(names) >= 15, names
    for name in names:
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
        assert name in _capi.SIGNATURES, f"{name} has no ctypes signature"
    assert set(_capi.SIGNATURES) == set(names)


def test_abi_version_and_error_channel():
    lib = _capi.lib()
    assert lib.pcp_abi_version() == 2
    status = lib.pcp_ring_schedule(0, 4, 4, None, None, None, None)
    assert status == 1  # PCP_ERR_INVALID_ARGUMENT
    assert b"hop" in lib.pcp_last_error()
    with pytest.raises(_capi.PcpError, match="INVALID_ARGUMENT"):
        _capi.check(status)


def test_source_valid_len_matches_oracle():
    lib = _capi.lib()
    for total, P, I in ((2048, 4, 64), (30001, 8, 64), (500000, 8, 64), (1001, 4, 16), (131072, 64, 64), (5, 4, 2)):
        for r in range(P):
            assert lib.pcp_source_valid_len(total, P, I, r) == orc.source_valid_len(total, P, I, r)
    assert lib.pcp_source_valid_len(10, 4, 2, 4) == -1


@pytest.mark.parametrize("P", [2, 3, 4, 8, 64])
def test_ring_schedule_follows_reference_order(P):
    """reference.py:68-71: at step s rank r consumes the shard of (r - s) % P,
    received from its predecessor; the shard it forwards at hop s is the one
    it consumed at step s-1 (its own at s=1); no hop returns a shard to its owner."""
    lib = _capi.lib()
    sched = {}
    for r in range(P):
        for hop in range(1, P):
            ss, rs, to, frm = (ctypes.c_int32() for _ in range(4))
            _capi.check(lib.pcp_ring_schedule(r, P, hop, ctypes.byref(ss), ctypes.byref(rs), ctypes.byref(to),
                                              ctypes.byref(frm)))
            sched[r, hop] = (ss.value, rs.value, to.value, frm.value)
            assert rs.value == (r - hop) % P
            assert ss.value == (r - hop + 1) % P
            assert to.value == (r + 1) % P and frm.value == (r - 1) % P
            assert to.value != ss.value  # never back to the owner
    for r in range(P):
        for hop in range(1, P):
            # what r sends at this hop is what r+1 receives at this hop
            assert sched[r, hop][0] == sched[(r + 1) % P, hop][1]
        # after P-1 hops every rank has seen every source exactly once
        seen = {r} | {sched[r, hop][1] for hop in range(1, P)}
        assert seen == set(range(P))


def test_workspace_size_is_host_only():
    lib = _capi.lib()
    n = ctypes.c_size_t()
    # bf16 cache: dense bf16 K and V for 131072 keys x 2 heads x 256 dims
    dims = _capi.PcpDims(1, 4096, 256, 512, 32, 2, 256, 1)
    _capi.check(lib.pcp_history_attention_workspace_size(ctypes.byref(dims), 131072, ctypes.byref(n)))
    assert n.value >= 2 * 2 * 131072 * 256 * 2
    # e4m3 cache: by default a KV head with 65536 query rows reads a dense
    # copy; read in place there is no dense copy (and one split at P=1: no
    # partials either)
    dims = _capi.PcpDims(1, 4096, 256, 512, 32, 2, 256, 0)
    _capi.check(lib.pcp_history_attention_workspace_size(ctypes.byref(dims), 131072, ctypes.byref(n)))
    assert n.value >= 2 * 2 * 131072 * 256 * 2
    try:
        _capi.set_default_kv_path("in_place")
        _capi.check(lib.pcp_history_attention_workspace_size(ctypes.byref(dims), 131072, ctypes.byref(n)))
        assert n.value < 1 << 20
    finally:
        _capi.set_default_kv_path("auto")
    # a short query shard (16 x 64 rows per KV head) reads in place by default
    small = _capi.PcpDims(1, 64, 256, 512, 32, 2, 256, 0)
    _capi.check(lib.pcp_history_attention_workspace_size(ctypes.byref(small), 131072, ctypes.byref(n)))
    assert n.value < 2 * 2 * 131072 * 256 * 2
    with pytest.raises(_capi.PcpError, match="kv path"):
        _capi.check(lib.pcp_set_kv_path(None, 7))
    bad = _capi.PcpDims(1, 4096, 256, 512, 32, 2, 96, 0)
    assert lib.pcp_history_attention_workspace_size(ctypes.byref(bad), 10, ctypes.byref(n)) == 2  # UNSUPPORTED
    assert b"head_dim" in lib.pcp_last_error()


def test_missing_library_fails_loudly(tmp_path):
    """No silent fallback: with the extension absent, loading it raises."""
    import subprocess
    import sys

    code = (
        "import pathlib, aws_training_study_b200._capi as c\n"
        f"c.LIB_PATH = pathlib.Path({str(tmp_path / 'absent.so')!r})\n"
        "try:\n    c.lib()\nexcept ImportError as e:\n    print('raised:', e)\n"
    )
    r = subprocess.run([sys.executable, "-c", code], cwd=Path(__file__).resolve().parents[1], capture_output=True,
                       text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert "raised:" in r.stdout and "no fallback" in r.stdout
