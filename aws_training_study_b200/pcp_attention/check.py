"""Output checks of the CUDA path against dense fp32 attention.

``dense_reference`` restates the reference's ``dense_history_attention``
(``pcp_attention/reference.py:16-32``: softmax(Q K^T * scale) V in fp32 with
the GQA heads of one KV head sharing it, K/V dequantised by ``.float()``) in
torch, with TF32 off, chunked over query rows so that every row of a
BASELINE-size shard can be checked on the GPU in seconds (the scores of a
whole shard would not fit: 8.6 GB per rank at configs[3]).  It is the
checker behind ``run_poc.py --check`` (the reference's ``run_poc.py:257-264``
check), ``bench.py``'s ``parity`` record and the full-size GPU tests; the
product path never calls it.
"""

from __future__ import annotations

import torch

from .config import PCPAttentionConfig

# Bounds on the bf16 output (the BASELINE tolerance, plus a relative bound:
# at long history |O| shrinks like 1/sqrt(hist), so an all-zero output would
# pass the absolute ones).
MAX_ABS = 2e-2
MEAN_ABS = 2e-3
REL_L2 = 1e-2
MIN_NORM_RATIO = 0.25


def dense_reference(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                    score_bytes: int = 512 << 20) -> torch.Tensor:
    """fp32 ``softmax(q k^T scale) v`` for ``q [Hq, R, D]`` and ``k``/``v``
    ``[Hkv, N, D]`` (any float dtype); query rows are processed in chunks
    whose scores take at most ``score_bytes``."""
    hq, rows, d = q.shape
    hkv, n, _ = k.shape
    group = hq // hkv
    out = torch.empty((hq, rows, d), dtype=torch.float32, device=q.device)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for g in range(hkv):
            kf, vf = k[g].float(), v[g].float()
            qg = q[g * group:(g + 1) * group].reshape(group * rows, d)
            chunk = max(1, min(group * rows, score_bytes // max(1, 4 * n)))
            og = out[g * group:(g + 1) * group].view(group * rows, d)
            for r0 in range(0, group * rows, chunk):
                s = torch.matmul(qg[r0:r0 + chunk].float(), kf.T)
                s.mul_(scale)
                s = torch.softmax(s, dim=-1)
                og[r0:r0 + chunk] = torch.matmul(s, vf)
                del s
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return out


def history_from_packed(cfg: PCPAttentionConfig, shards, valid_lens) -> tuple[torch.Tensor, torch.Tensor]:
    """K and V ``[Hkv, sum(valid), D]`` of packed shards (``pack_local_kv``
    payload ``[max_local_blocks, 2*Hkv*bs*D]``), the first ``valid_lens[i]``
    tokens of shard i, in shard order."""
    ks, vs = [], []
    for packed, valid in zip(shards, valid_lens):
        raw = packed.view(torch.uint8) if packed.dtype == torch.float8_e4m3fn else packed
        blk = raw.reshape(cfg.max_local_blocks, 2, cfg.num_kv_heads, cfg.block_size, cfg.head_dim)
        for kv, dst in ((0, ks), (1, vs)):
            t = blk[:, kv].permute(1, 0, 2, 3).reshape(cfg.num_kv_heads, -1, cfg.head_dim)[:, :valid]
            dst.append(t)
    k = torch.cat(ks, dim=1)
    v = torch.cat(vs, dim=1)
    if shards[0].dtype == torch.float8_e4m3fn:
        k, v = k.view(torch.float8_e4m3fn), v.view(torch.float8_e4m3fn)
    return k, v


def compare(actual: torch.Tensor, expected: torch.Tensor) -> dict:
    """Error metrics of ``actual`` against ``expected`` (both any shape)."""
    a = actual.float()
    e = expected.float()
    diff = (a - e).abs()
    en = torch.linalg.vector_norm(e).item()
    return {
        "max_abs": diff.max().item(),
        "mean_abs": diff.mean().item(),
        "rel_l2": torch.linalg.vector_norm(a - e).item() / max(en, 1e-30),
        "norm_ratio": torch.linalg.vector_norm(a).item() / max(en, 1e-30),
        "finite": bool(torch.isfinite(a).all().item()),
    }


def within_bounds(m: dict) -> bool:
    return (m["finite"] and m["max_abs"] <= MAX_ABS and m["mean_abs"] <= MEAN_ABS and m["rel_l2"] <= REL_L2
            and m["norm_ratio"] >= MIN_NORM_RATIO)
