"""The C ABI's newer entries reject invalid arguments with a status and a
message instead of touching memory (CPU only: every call below fails its
checks before any device work)."""

from __future__ import annotations

import ctypes

import pytest

from aws_training_study_b200 import _capi


def _dims(**kw):
    d = dict(pcp_size=2, local_q_len=128, max_local_blocks=4, block_size=512, num_q_heads=4, num_kv_heads=2,
             head_dim=128, kv_dtype=_capi.PCP_KV_E4M3)
    d.update(kw)
    return _capi.PcpDims(d["pcp_size"], d["local_q_len"], d["max_local_blocks"], d["block_size"],
                         d["num_q_heads"], d["num_kv_heads"], d["head_dim"], d["kv_dtype"])


def _status(rc):
    assert rc != 0
    msg = _capi.lib().pcp_last_error().decode()
    assert msg
    return msg


P = ctypes.c_void_p
FAKE = P(0x1000)  # never dereferenced: each call fails an argument check first


def test_cache_write_argument_checks():
    lib = _capi.lib()
    d = _dims()
    st = P(0x2000)
    assert "NULL" in _status(lib.pcp_cache_write(ctypes.byref(d), 64, 0, 0, 10, None, FAKE, FAKE, 4, FAKE, 8, st,
                                                 None))
    assert "interleave" in _status(lib.pcp_cache_write(ctypes.byref(d), 0, 0, 0, 10, FAKE, FAKE, FAKE, 4, FAKE, 8,
                                                       st, None))
    assert "rank" in _status(lib.pcp_cache_write(ctypes.byref(d), 64, 5, 0, 10, FAKE, FAKE, FAKE, 4, FAKE, 8, st,
                                                 None))
    assert "negative" in _status(lib.pcp_cache_write(ctypes.byref(d), 64, 0, -1, 10, FAKE, FAKE, FAKE, 4, FAKE, 8,
                                                     st, None))
    assert "aligned" in _status(lib.pcp_cache_write(ctypes.byref(d), 64, 0, 0, 10, P(0x1001), FAKE, FAKE, 4, FAKE,
                                                    8, st, None))


def test_paged_and_prefill_argument_checks():
    lib = _capi.lib()
    d = _dims()
    vl = _capi.int32_array([10, 10])
    assert "NULL" in _status(lib.pcp_history_attention_paged(ctypes.byref(d), FAKE, None, 8, FAKE, 2, vl, FAKE,
                                                             FAKE, 1 << 20, None))
    assert "pool" in _status(lib.pcp_history_attention_paged(ctypes.byref(d), FAKE, FAKE, 0, FAKE, 2, vl, FAKE,
                                                             FAKE, 1 << 20, None))
    assert "interleave" in _status(lib.pcp_prefill_attention(ctypes.byref(d), 0, 0, FAKE, FAKE, 2, vl, FAKE, FAKE,
                                                             FAKE, FAKE, 1 << 20, None))
    assert "rank" in _status(lib.pcp_prefill_attention(ctypes.byref(d), 64, 2, FAKE, FAKE, 2, vl, FAKE, FAKE, FAKE,
                                                       FAKE, 1 << 20, None))


def test_handle_entries_reject_null_handle():
    lib = _capi.lib()
    vl = _capi.int32_array([10, 10])
    for rc in (lib.pcp_forward_paged(None, FAKE, FAKE, 8, FAKE, vl, FAKE, None),
               lib.pcp_forward_bucketed(None, FAKE, FAKE, FAKE, vl, FAKE, None),
               lib.pcp_forward_prefill(None, 64, FAKE, FAKE, vl, FAKE, FAKE, FAKE, None),
               lib.pcp_set_comm_sms(None, 16),
               lib.pcp_set_exchange(None, 0)):
        assert "handle" in _status(rc)


@pytest.mark.parametrize("head_dim,kv", [(64, _capi.PCP_KV_E4M3), (128, 7)])
def test_unsupported_dims(head_dim, kv):
    size = ctypes.c_size_t()
    d = _dims(head_dim=head_dim, kv_dtype=kv)
    _status(_capi.lib().pcp_prefill_attention_workspace_size(ctypes.byref(d), 100, ctypes.byref(size)))
