"""The oracle's paged-cache producer against the reference's own cache
construction (``shard_history`` + ``pack_local_kv`` + e4m3 encode, all pinned
to reference goldens by test_oracle_golden.py), on the CPU."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import pcp_oracle as orc


def _bf16_values(rng, shape, scale=0.5):
    x = (rng.standard_normal(shape) * scale).astype(np.float32)
    return orc.bf16_round(x)


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("P,I,bs,A", [(4, 16, 64, 1024), (3, 8, 32, 1000), (1, 16, 64, 200)])
def test_whole_history_matches_shard_and_pack(bf16, P, I, bs, A):
    hkv, d = 2, 16
    rng = np.random.default_rng(1)
    k, v = _bf16_values(rng, (hkv, A, d)), _bf16_values(rng, (hkv, A, d))
    cfg = orc.OracleConfig(P, P * I, A + bs, A, bs, I, 2, hkv, d)
    if bf16:
        enc = lambda x: (x.view(np.uint32) >> 16).astype(np.uint16)  # noqa: E731
    else:
        enc = orc.e4m3fn_encode
    ks, vs = orc.shard_history(enc(k), enc(v), cfg)
    elt = 2 if bf16 else 1
    for rank in range(P):
        expected = orc.pack_local_kv(ks[rank], vs[rank]).view(np.uint8)
        nb = expected.shape[0]
        pool = np.zeros((nb, 2 * hkv * bs * d * elt), dtype=np.uint8)
        orc.cache_write(pool, np.arange(nb), k, v, 0, cfg, rank, bf16)
        np.testing.assert_array_equal(pool, expected)


def test_appends_compose_and_tables_permute():
    """Several appends at unaligned positions through a permuted table read
    back (through the table) as one whole-history write."""
    P, I, bs, A, hkv, d = 4, 16, 64, 1500, 2, 8
    rng = np.random.default_rng(2)
    k, v = _bf16_values(rng, (hkv, A, d)), _bf16_values(rng, (hkv, A, d))
    cfg = orc.OracleConfig(P, P * I, A, A, bs, I, 2, hkv, d)
    for rank in range(P):
        nb = -(-orc.source_valid_len(A, P, I, rank) // bs)
        whole = np.zeros((nb, 2 * hkv * bs * d), dtype=np.uint8)
        orc.cache_write(whole, np.arange(nb), k, v, 0, cfg, rank, False)
        table = rng.permutation(nb + 5)[:nb]
        pool = np.zeros((nb + 5, whole.shape[1]), dtype=np.uint8)
        cuts = [0, 1, 63, 700, 701, 1499, A]
        for a, b in zip(cuts[:-1], cuts[1:]):
            orc.cache_write(pool, table, k[:, a:b], v[:, a:b], a, cfg, rank, False)
        np.testing.assert_array_equal(pool[table], whole)
