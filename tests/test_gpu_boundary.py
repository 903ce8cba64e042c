"""The drop-in boundary, called the way the reference calls its kernel (needs a B200).

* ``wrap_for_native_torch(cfg)(q, packed_kv, block_valid_mask)`` -- the
  signature of the reference's ``pcp_attention/kernel.py:559-564`` -- with the
  reference's own input construction (``make_inputs``, ``shard_query``,
  ``shard_history``, ``pack_local_kv``, ``make_block_valid_mask``:
  ``run_poc.py:81-153,231-237``), checked against the CPU oracle.
* ``run_poc.main([... "--check", "full"])`` -- the ``--backend cuda`` runner,
  whose check is the reference's ``run_poc.py:257-264`` against dense fp32
  attention.
"""

from __future__ import annotations

import pytest
import torch

import run_poc
from aws_training_study_b200.pcp_attention import get_preset, pack_local_kv, shard_history, shard_query, wrap_for_native_torch
from aws_training_study_b200.pcp_attention.inputs import make_block_valid_mask, make_inputs

from parity import assert_parity, expected_rank_output

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("actual", [2048, 1500])
def test_wrap_for_native_torch_reference_signature(actual):
    cfg = get_preset("tiny").with_overrides(pcp_size=1, actual_history_len=actual)
    q, k, v = make_inputs(cfg, seed=1234)
    q_local = shard_query(q, cfg)[0]
    ks, vs = shard_history(k, v, cfg)
    packed = pack_local_kv(ks[0], vs[0])
    if packed.shape[0] < cfg.max_local_blocks:
        padded = torch.zeros((cfg.max_local_blocks, packed.shape[1]), dtype=packed.dtype)
        padded[: packed.shape[0]] = packed
        packed = padded
    mask = make_block_valid_mask(cfg)
    kernel = wrap_for_native_torch(cfg)
    try:
        out = kernel(q_local.cuda(), packed.cuda(), mask)
        kernel.history_attention.status()
        assert out.dtype == torch.bfloat16 and tuple(out.shape) == tuple(q_local.shape)
        assert_parity(out, expected_rank_output(cfg, q, k, v, 0), f"wrap_for_native_torch actual={actual}")
    finally:
        kernel.history_attention.close()


@pytest.mark.parametrize("extra", [[], ["--kv-dtype", "bf16"], ["--actual-history-len", "1777",
                                                                  "--benchmark-iterations", "3"]])
def test_run_poc_cuda_backend_full_check(extra, capsys):
    assert run_poc.main(["--backend", "cuda", "--preset", "tiny", "--pcp-size", "1", "--check", "full", *extra]) == 0
    text = capsys.readouterr().out
    assert "CUDA output OK" in text
