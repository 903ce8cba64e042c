"""CPU oracle for prefill context-parallel (PCP) history-only attention.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
module, and only as the checker or as the timed CPU baseline.  The product
path (``aws_training_study_b200``) never imports it and has no CPU fallback.

This is a numpy restatement of the reference's executable specification
(HandsomeHow/aws_training_study, ``pcp_attention/``):

* config arithmetic            -- ``pcp_attention/config.py:29-59``
* striped ownership / layout   -- ``pcp_attention/layout.py:10-132``
* KV ring payload packer       -- ``pcp_attention/kernel.py:17-29``
* additive block-valid mask    -- ``run_poc.py:137-153``
* dense GQA attention (fp32)   -- ``pcp_attention/reference.py:16-32``
* serial ring online softmax   -- ``pcp_attention/reference.py:35-95``

Parity pin: every function here is checked against golden vectors produced by
importing the reference itself (``tests/golden/make_golden.py`` writes
``tests/golden/*.npz``; ``tests/test_oracle_golden.py`` compares).

One deliberate generalisation, used only where the reference cannot express
the case: ``ring_history_attention`` accepts per-source-rank valid lengths.
The reference uses ``actual_history_len // pcp_size`` for every source rank
(``reference.py:64-67``), which is exact only when ``actual_history_len`` is a
multiple of ``pcp_size * interleave_size``; ``source_valid_len`` gives the
exact per-rank count for any length (it equals the reference's number in the
aligned case).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

# ----------------------------------------------------------------------------
# Number formats: FP8 E4M3FN and BF16, restated from their definitions.
# ----------------------------------------------------------------------------


def _e4m3fn_table() -> np.ndarray:
    """Exact fp32 value of every E4M3FN byte (1 sign, 4 exponent bits with
    bias 7, 3 mantissa bits; no infinities; S.1111.111 is NaN)."""
    codes = np.arange(256, dtype=np.int64)
    sign = np.where(codes & 0x80, -1.0, 1.0)
    exp = (codes >> 3) & 0xF
    man = codes & 0x7
    normal = (1.0 + man / 8.0) * np.exp2(exp - 7.0)
    subnormal = (man / 8.0) * np.exp2(-6.0)
    mag = np.where(exp == 0, subnormal, normal)
    vals = (sign * mag).astype(np.float32)
    vals[(exp == 0xF) & (man == 0x7)] = np.nan
    return vals


E4M3FN_VALUES = _e4m3fn_table()


def e4m3fn_decode(codes: np.ndarray) -> np.ndarray:
    """Dequantise E4M3FN bytes at unit scale, as ``tensor.float()`` does in
    ``reference.py:29-31,70-71``."""
    return E4M3FN_VALUES[np.asarray(codes, dtype=np.uint8)]


def e4m3fn_encode(x: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest E4M3FN value (ties to even).  Magnitudes that
    round above 448 and NaN/Inf inputs become the NaN code (0x7F/0xFF), the
    behaviour of ``tensor.to(torch.float8_e4m3fn)`` used by ``run_poc.py:96``."""
    x = np.asarray(x, dtype=np.float32)
    finite_vals = E4M3FN_VALUES[:0x7F]  # 0x00..0x7E, ascending, non-negative
    with np.errstate(invalid="ignore"):  # NaN inputs: their code is set below
        mag = np.abs(x).astype(np.float64)
    idx = np.searchsorted(finite_vals.astype(np.float64), mag, side="left")
    idx = np.clip(idx, 1, len(finite_vals) - 1)
    lo = finite_vals[idx - 1].astype(np.float64)
    hi = finite_vals[idx].astype(np.float64)
    pick_hi = (mag - lo > hi - mag) | ((mag - lo == hi - mag) & (idx % 2 == 0))
    code = np.where(pick_hi, idx, idx - 1).astype(np.int64)
    code = np.where(mag <= 0.0, 0, code)
    # Beyond the largest finite value: 448 < |x| <= 464 rounds down to 448
    # (tie at 464 goes to the even code 0x7E); anything larger is NaN.
    code = np.where(mag > 448.0, np.where(mag <= 464.0, 0x7E, 0x7F), code)
    code = np.where(np.isfinite(x), code, 0x7F)
    sign = np.where(np.signbit(x), 0x80, 0)
    return (code | sign).astype(np.uint8)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bfloat16 (round to nearest even), returned as fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000
    out = rounded.astype(np.uint32).view(np.float32).copy()
    nan = np.isnan(x)
    out[nan] = np.nan
    return out


def bf16_bits_to_float32(bits: np.ndarray) -> np.ndarray:
    b = np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16
    return b.view(np.float32)


# ----------------------------------------------------------------------------
# Configuration arithmetic (config.py:29-59)
# ----------------------------------------------------------------------------


@dataclass(frozen=True)
class OracleConfig:
    """Static fields and derived shapes of ``PCPAttentionConfig``
    (``config.py:9-59``).  No validation: the oracle accepts any positive
    shape, including the ones the reference's Trainium checks reject."""

    pcp_size: int
    current_len: int
    max_history_len: int
    actual_history_len: int
    block_size: int = 512
    interleave_size: int = 64
    num_q_heads: int = 32
    num_kv_heads: int = 2
    head_dim: int = 256

    @property
    def softmax_scale(self) -> float:  # config.py:29-31
        return 1.0 / math.sqrt(self.head_dim)

    @property
    def q_heads_per_kv_head(self) -> int:  # config.py:33-35
        return self.num_q_heads // self.num_kv_heads

    @property
    def local_q_len(self) -> int:  # config.py:37-39
        return self.current_len // self.pcp_size

    @property
    def max_local_history_len(self) -> int:  # config.py:41-43
        return self.max_history_len // self.pcp_size

    @property
    def actual_local_history_len(self) -> int:  # config.py:45-47
        return self.actual_history_len // self.pcp_size

    @property
    def max_local_blocks(self) -> int:  # config.py:49-51
        return math.ceil(self.max_local_history_len / self.block_size)

    @property
    def actual_local_blocks(self) -> int:  # config.py:53-55
        return math.ceil(self.actual_local_history_len / self.block_size)

    @property
    def rank_stride(self) -> int:  # config.py:57-59
        return self.pcp_size * self.interleave_size

    def source_valid_len(self, source_rank: int) -> int:
        return source_valid_len(
            self.actual_history_len, self.pcp_size, self.interleave_size, source_rank
        )

    def storage_blocks(self) -> int:
        """Cache blocks needed to hold the longest per-rank shard (rank 0)."""
        return math.ceil(self.source_valid_len(0) / self.block_size)


def source_valid_len(total_len: int, pcp_size: int, interleave_size: int, rank: int) -> int:
    """Number of positions ``p < total_len`` owned by ``rank`` under the striped
    map of ``layout.py:10-16``: every full rank-stride gives each rank
    ``interleave_size`` positions, and the ragged tail is dealt out in
    interleave-sized chunks starting from rank 0."""
    stride = pcp_size * interleave_size
    full, tail = divmod(total_len, stride)
    return full * interleave_size + min(max(tail - rank * interleave_size, 0), interleave_size)


# ----------------------------------------------------------------------------
# Striped layout (layout.py:10-132)
# ----------------------------------------------------------------------------


def owner_and_local_position(global_position: int, pcp_size: int, interleave_size: int):
    """``layout.py:10-16``."""
    chunk, within = divmod(global_position, interleave_size)
    owner = chunk % pcp_size
    local_chunk = chunk // pcp_size
    return owner, local_chunk * interleave_size + within


def global_positions_for_rank(total_len: int, rank: int, pcp_size: int, interleave_size: int) -> np.ndarray:
    """``layout.py:19-31`` for aligned ``total_len``; for any other length the
    positions of the aligned superset that are ``< total_len`` (the reference
    raises there)."""
    if not 0 <= rank < pcp_size:
        raise ValueError(f"rank {rank} is outside [0, {pcp_size})")
    stride = pcp_size * interleave_size
    chunks = -(-total_len // stride)
    base = (np.arange(chunks, dtype=np.int64) * pcp_size + rank) * interleave_size
    pos = (base[:, None] + np.arange(interleave_size, dtype=np.int64)[None, :]).reshape(-1)
    return pos[pos < total_len]


def shard_query(q: np.ndarray, cfg: OracleConfig) -> list[np.ndarray]:
    """``layout.py:34-51``: ``[Hq, current_len, D]`` -> P x ``[Hq, Qloc, D]``."""
    return [
        np.ascontiguousarray(
            q[:, global_positions_for_rank(cfg.current_len, r, cfg.pcp_size, cfg.interleave_size), :]
        )
        for r in range(cfg.pcp_size)
    ]


def shard_history(k: np.ndarray, v: np.ndarray, cfg: OracleConfig, num_blocks: int | None = None):
    """``layout.py:54-98``: striped K/V ``[Hkv, A, D]`` -> per-rank paged cache
    ``[blocks, Hkv, block_size, D]`` with the tail of the last block zeroed.
    ``num_blocks`` defaults to the reference's ``actual_local_blocks`` when the
    history is aligned, else to the block count of the longest shard."""
    if num_blocks is None:
        aligned = cfg.actual_history_len % cfg.rank_stride == 0
        num_blocks = cfg.actual_local_blocks if aligned else cfg.storage_blocks()
    out_k, out_v = [], []
    for r in range(cfg.pcp_size):
        pos = global_positions_for_rank(cfg.actual_history_len, r, cfg.pcp_size, cfg.interleave_size)

        def to_cache(t: np.ndarray) -> np.ndarray:
            padded = np.zeros((cfg.num_kv_heads, num_blocks * cfg.block_size, cfg.head_dim), dtype=t.dtype)
            padded[:, : len(pos), :] = t[:, pos, :]
            return np.ascontiguousarray(
                padded.reshape(cfg.num_kv_heads, num_blocks, cfg.block_size, cfg.head_dim).transpose(1, 0, 2, 3)
            )

        out_k.append(to_cache(k))
        out_v.append(to_cache(v))
    return out_k, out_v


def gather_history(shards: list[np.ndarray], cfg: OracleConfig) -> np.ndarray:
    """``layout.py:101-132``: inverse of ``shard_history`` for K or V."""
    sample = shards[0]
    result = np.empty((cfg.num_kv_heads, cfg.actual_history_len, cfg.head_dim), dtype=sample.dtype)
    for r, shard in enumerate(shards):
        pos = global_positions_for_rank(cfg.actual_history_len, r, cfg.pcp_size, cfg.interleave_size)
        local = shard.transpose(1, 0, 2, 3).reshape(cfg.num_kv_heads, -1, cfg.head_dim)
        result[:, pos, :] = local[:, : len(pos), :]
    return result


def pack_local_kv(k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """``kernel.py:17-29``: ``[blocks, Hkv, bs, D]`` x2 -> ``[blocks, 2*Hkv*bs*D]``
    with all K followed by all V inside every block."""
    if k.shape != v.shape or k.ndim != 4:
        raise ValueError("K and V must have equal [blocks, Hkv, block, D] shapes")
    return np.ascontiguousarray(np.stack((k, v), axis=1).reshape(k.shape[0], -1))


def make_block_valid_mask(cfg: OracleConfig) -> np.ndarray:
    """``run_poc.py:137-153``: additive bias ``[max_local_blocks, bs/128, 1, 128]``
    (bf16 values 0 / -9984, returned as fp32)."""
    kv_tiles = cfg.block_size // 128
    mask = np.full((cfg.max_local_blocks, kv_tiles, 1, 128), -9984.0, dtype=np.float32)
    remaining = cfg.actual_local_history_len
    for block in range(cfg.actual_local_blocks):
        valid_in_block = min(cfg.block_size, remaining)
        for tile in range(kv_tiles):
            valid_in_tile = min(128, max(0, valid_in_block - tile * 128))
            mask[block, tile, 0, :valid_in_tile] = 0.0
        remaining -= valid_in_block
    return mask


def block_valid_tokens(valid_len: int, block: int, block_size: int) -> int:
    return min(block_size, max(0, valid_len - block * block_size))


# ----------------------------------------------------------------------------
# Attention (reference.py:16-95)
# ----------------------------------------------------------------------------


def dense_history_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float, row_chunk: int = 1024) -> np.ndarray:
    """``reference.py:16-32``: exact fp32 GQA attention, ``softmax(Q K^T scale) V``.

    Q ``[Hq, Q, D]``, K/V ``[Hkv, K, D]`` -> fp32 ``[Hq, Q, D]``.  Computed per
    head and per ``row_chunk`` query rows so the score matrix stays small."""
    hq, nq, dim = q.shape
    hkv, nk, kdim = k.shape
    if k.shape != v.shape or dim != kdim or hq % hkv:
        raise ValueError("incompatible Q/K/V shapes for grouped-query attention")
    group = hq // hkv
    kf = k.astype(np.float32, copy=False)
    vf = v.astype(np.float32, copy=False)
    out = np.empty((hq, nq, dim), dtype=np.float32)
    for h in range(hq):
        g = h // group
        for r0 in range(0, nq, row_chunk):
            qs = q[h, r0 : r0 + row_chunk].astype(np.float32)
            s = (qs @ kf[g].T) * np.float32(scale)
            s -= s.max(axis=-1, keepdims=True)
            np.exp(s, out=s)
            s /= s.sum(axis=-1, keepdims=True)
            out[h, r0 : r0 + row_chunk] = s @ vf[g]
    return out


def ring_history_attention(q_shards, k_shards, v_shards, cfg: OracleConfig, valid_lens=None, ranks=None):
    """``reference.py:35-95``: the serial two-loop ring with online softmax.

    At outer iteration ``block`` every rank starts from its local cache block;
    ring step ``s`` processes the block of source rank ``(rank - s) % P``.  The
    per-head update is ``new_max = max(running, block_max)``,
    ``out = out*exp(running-new_max) + exp(S-new_max) V``, sum likewise, and the
    result is ``out / sum``.

    ``valid_lens[src]`` (default: the reference's ``actual_local_history_len``
    for every source) sets the number of valid tokens in each source's shard.
    Blocks with no valid token are skipped (the reference never reaches them
    in the aligned case).  ``ranks`` restricts the ranks computed (the ranks are
    independent), for bounded CPU timing samples."""
    P = cfg.pcp_size
    if valid_lens is None:
        valid_lens = [cfg.actual_local_history_len] * P
    n_blocks = max(k.shape[0] for k in k_shards)
    scale = np.float32(cfg.softmax_scale)
    group = cfg.q_heads_per_kv_head
    outputs = []
    for rank in (range(P) if ranks is None else ranks):
        qf = q_shards[rank].astype(np.float32)
        hq, nq, dim = qf.shape
        run_max = np.full((hq, nq, 1), -np.inf, dtype=np.float32)
        run_sum = np.zeros((hq, nq, 1), dtype=np.float32)
        run_out = np.zeros_like(qf)
        for block in range(n_blocks):
            for step in range(P):
                src = (rank - step) % P
                valid = block_valid_tokens(valid_lens[src], block, cfg.block_size)
                if valid <= 0:
                    continue
                kb = k_shards[src][block, :, :valid, :].astype(np.float32)
                vb = v_shards[src][block, :, :valid, :].astype(np.float32)
                for h in range(hq):
                    g = h // group
                    s = (qf[h] @ kb[g].T) * scale
                    bmax = s.max(axis=-1, keepdims=True)
                    new_max = np.maximum(run_max[h], bmax)
                    old_scale = np.exp(run_max[h] - new_max)
                    p = np.exp(s - new_max)
                    run_out[h] = run_out[h] * old_scale + p @ vb[g]
                    run_sum[h] = run_sum[h] * old_scale + p.sum(axis=-1, keepdims=True)
                    run_max[h] = new_max
        outputs.append(run_out / run_sum)
    return outputs


def history_flops(num_q_heads: int, q_len: int, hist_len: int, head_dim: int) -> float:
    """QK^T plus PV model FLOPs, ``4 * Hq * Q * Hist * D`` (reference README
    MFU formula, ``README.md:167-171``)."""
    return 4.0 * num_q_heads * q_len * hist_len * head_dim


# ----------------------------------------------------------------------------
# Prefill: history plus causal current-token attention.
#
# The reference stops at history-only attention and lists current-token
# attention as future work (``README.md:17-18``), so nothing upstream pins
# this part directly.  It is restated from the definition of causal prefill
# attention over a cached prefix: a current token at global position g (in
# the ``shard_query`` stripe layout, ``layout.py:19-51``) attends to every
# history key and to the current tokens at positions <= g, in one softmax.
# The history half is exactly ``dense_history_attention`` (pinned above).
# ----------------------------------------------------------------------------

def prefill_attention(q_shard: np.ndarray, k_hist: np.ndarray, v_hist: np.ndarray, k_cur: np.ndarray,
                      v_cur: np.ndarray, cfg: OracleConfig, rank: int, row_chunk: int = 1024) -> np.ndarray:
    """Rank ``rank``'s striped Q shard ``[Hq, Qloc, D]`` against the dense
    history K/V ``[Hkv, A, D]`` (A may be 0) and the current tokens' K/V in
    sequence order ``[Hkv, current_len, D]``, causally -> fp32 ``[Hq, Qloc, D]``."""
    hq, nq, dim = q_shard.shape
    hkv = k_cur.shape[0]
    if hq % hkv or k_cur.shape != v_cur.shape or k_hist.shape[0] != hkv or k_cur.shape[1] != cfg.current_len:
        raise ValueError("incompatible shapes for prefill attention")
    group = hq // hkv
    qpos = global_positions_for_rank(cfg.current_len, rank, cfg.pcp_size, cfg.interleave_size)
    if qpos.shape[0] != nq:
        raise ValueError("Q shard length does not match the stripe layout")
    kpos = np.arange(cfg.current_len, dtype=np.int64)
    kh, vh = k_hist.astype(np.float32, copy=False), v_hist.astype(np.float32, copy=False)
    kc, vc = k_cur.astype(np.float32, copy=False), v_cur.astype(np.float32, copy=False)
    scale = np.float32(1.0 / math.sqrt(dim))
    out = np.empty((hq, nq, dim), dtype=np.float32)
    for h in range(hq):
        g = h // group
        keys = np.concatenate([kh[g], kc[g]], axis=0)
        vals = np.concatenate([vh[g], vc[g]], axis=0)
        for r0 in range(0, nq, row_chunk):
            qs = q_shard[h, r0 : r0 + row_chunk].astype(np.float32)
            s = (qs @ keys.T) * scale
            future = kpos[None, :] > qpos[r0 : r0 + row_chunk, None]
            s[:, kh.shape[1]:][future] = -np.inf
            s -= s.max(axis=-1, keepdims=True)
            np.exp(s, out=s)
            s /= s.sum(axis=-1, keepdims=True)
            out[h, r0 : r0 + row_chunk] = s @ vals
    return out


def prefill_flops(cfg: OracleConfig, rank: int) -> float:
    """Useful FLOPs of one rank's prefill: the history part plus the causal
    pairs (query, visible current key) only."""
    qpos = global_positions_for_rank(cfg.current_len, rank, cfg.pcp_size, cfg.interleave_size)
    causal_pairs = float((qpos + 1).sum())
    return 4.0 * cfg.num_q_heads * (qpos.shape[0] * cfg.actual_history_len + causal_pairs) * cfg.head_dim


# ----------------------------------------------------------------------------
# Paged-cache producer.
#
# The reference builds caches on the host (``shard_history``, ``layout.py:
# 54-98``; ``pack_local_kv``, ``kernel.py:17-29``; e4m3 from ``tensor.to(
# torch.float8_e4m3fn)``, ``run_poc.py:81-134``).  This restates the same
# placement token by token into a block pool addressed through a block table,
# using ``owner_and_local_position`` (``layout.py:10-16``) for each token.
# ----------------------------------------------------------------------------

def cache_write(pool: np.ndarray, table: np.ndarray, k_seq: np.ndarray, v_seq: np.ndarray, first: int,
                cfg: OracleConfig, rank: int, kv_is_bf16: bool) -> None:
    """Write the tokens of ``k_seq``/``v_seq`` (``[Hkv, T, D]`` fp32 holding
    bf16 values, token t at absolute position ``first + t``) that ``rank``
    owns into ``pool`` (uint8 ``[pool_blocks, payload_bytes]``, packed payload
    layout ``[2][Hkv][bs][D]`` per block), in place.  FP8 codes come from
    ``e4m3fn_encode``; bf16 is stored as its bit pattern (little endian)."""
    hkv, T, dim = k_seq.shape
    bs = cfg.block_size
    elt = 2 if kv_is_bf16 else 1
    view = pool.reshape(pool.shape[0], 2, hkv, bs, dim * elt)
    pos = first + np.arange(T, dtype=np.int64)
    stride = cfg.pcp_size * cfg.interleave_size
    owner = (pos // cfg.interleave_size) % cfg.pcp_size
    local = (pos // stride) * cfg.interleave_size + pos % cfg.interleave_size
    mine = np.nonzero(owner == rank)[0]
    for t in mine:  # per token: the same (owner, local) as owner_and_local_position
        assert owner_and_local_position(int(pos[t]), cfg.pcp_size, cfg.interleave_size) == (rank, int(local[t]))
    blk, row = local[mine] // bs, local[mine] % bs
    phys = np.asarray(table)[blk]
    for kv, src in ((0, k_seq), (1, v_seq)):
        vals = np.ascontiguousarray(src[:, mine, :].transpose(1, 0, 2), dtype=np.float32)  # [n, Hkv, D]
        if kv_is_bf16:
            enc = (vals.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8).reshape(len(mine), hkv, dim * 2)
        else:
            enc = e4m3fn_encode(vals)
        view[phys, kv, :, row, :] = enc
