"""Static and runtime configuration of PCP history attention.

Same dataclass, field names, defaults and derived shapes as the reference's
``PCPAttentionConfig`` (``pcp_attention/config.py:9-59``), so code written
against the reference constructs and reads it unchanged.

Differences, all in ``validate`` and in added methods:

* The Trainium-only checks are dropped: LNC core split (``config.py:84-85``),
  ``head_dim % 128`` (``:86-87``), ``block_size % 128`` (``:88-89``) and the
  128-token NKI Q tile (``:102-106``).  The CUDA kernel states its own limits
  (``cuda_backend.kernel_limits``) and raises where they are not met.
* ``actual_history_len`` need not be a multiple of ``pcp_size *
  interleave_size`` (``:92-101``).  Per-source-rank valid lengths
  (``source_valid_len``) describe the ragged tail exactly; the reference's
  single ``actual_local_history_len`` is kept bit-exact for the aligned case.
"""

from __future__ import annotations

from dataclasses import dataclass, replace
from math import ceil, sqrt


@dataclass(frozen=True)
class PCPAttentionConfig:
    """Configuration shared by layout, runner and the CUDA backend.

    ``actual_history_len`` is a runtime value no greater than
    ``max_history_len``; every other field fixes buffer shapes.
    """

    pcp_size: int
    current_len: int
    max_history_len: int
    actual_history_len: int
    block_size: int = 512
    interleave_size: int = 64
    num_q_heads: int = 32
    num_kv_heads: int = 2
    head_dim: int = 256
    lnc: int = 2
    alignment: int = 4096

    # -- derived shapes (reference config.py:29-59, bit-exact) ---------------
    @property
    def softmax_scale(self) -> float:
        return 1.0 / sqrt(self.head_dim)

    @property
    def q_heads_per_kv_head(self) -> int:
        return self.num_q_heads // self.num_kv_heads

    @property
    def local_q_len(self) -> int:
        return self.current_len // self.pcp_size

    @property
    def max_local_history_len(self) -> int:
        return self.max_history_len // self.pcp_size

    @property
    def actual_local_history_len(self) -> int:
        return self.actual_history_len // self.pcp_size

    @property
    def max_local_blocks(self) -> int:
        return ceil(self.max_local_history_len / self.block_size)

    @property
    def actual_local_blocks(self) -> int:
        return ceil(self.actual_local_history_len / self.block_size)

    @property
    def rank_stride(self) -> int:
        return self.pcp_size * self.interleave_size

    # -- additions -----------------------------------------------------------
    @property
    def history_aligned(self) -> bool:
        return self.actual_history_len % self.rank_stride == 0

    def source_valid_len(self, source_rank: int) -> int:
        """Valid history tokens held by ``source_rank``.

        Under the striped map (``layout.py:10-16``) every full rank-stride gives
        each rank ``interleave_size`` tokens and the ragged tail is dealt out
        in interleave chunks from rank 0.  Equals ``actual_local_history_len``
        for every rank when the history is aligned.
        """
        if not 0 <= source_rank < self.pcp_size:
            raise ValueError(f"rank {source_rank} is outside [0, {self.pcp_size})")
        full, tail = divmod(self.actual_history_len, self.rank_stride)
        extra = min(max(tail - source_rank * self.interleave_size, 0), self.interleave_size)
        return full * self.interleave_size + extra

    def source_valid_lens(self) -> list[int]:
        return [self.source_valid_len(r) for r in range(self.pcp_size)]

    @property
    def local_cache_blocks(self) -> int:
        """Cache blocks in every rank's shard as built by ``shard_history``:
        the reference's ``actual_local_blocks`` when aligned, otherwise enough
        blocks for the longest shard (rank 0)."""
        if self.history_aligned:
            return self.actual_local_blocks
        return ceil(self.source_valid_len(0) / self.block_size)

    def with_overrides(self, **kwargs: int) -> "PCPAttentionConfig":
        return replace(self, **kwargs).validate()

    def validate(self) -> "PCPAttentionConfig":
        positive = {
            "pcp_size": self.pcp_size,
            "current_len": self.current_len,
            "max_history_len": self.max_history_len,
            "actual_history_len": self.actual_history_len,
            "block_size": self.block_size,
            "interleave_size": self.interleave_size,
            "num_q_heads": self.num_q_heads,
            "num_kv_heads": self.num_kv_heads,
            "head_dim": self.head_dim,
            "lnc": self.lnc,
        }
        for name, value in positive.items():
            if value <= 0:
                raise ValueError(f"{name} must be positive, got {value}")
        if self.actual_history_len > self.max_history_len:
            raise ValueError("actual_history_len must not exceed max_history_len")
        if self.num_q_heads % self.num_kv_heads:
            raise ValueError("num_q_heads must be divisible by num_kv_heads")
        if self.block_size % self.interleave_size:
            raise ValueError("block_size must be divisible by interleave_size")
        for name, value in (
            ("current_len", self.current_len),
            ("max_history_len", self.max_history_len),
        ):
            if value % self.rank_stride:
                raise ValueError(
                    f"{name} must be divisible by pcp_size * interleave_size "
                    f"({self.rank_stride}), got {value}"
                )
        if self.local_cache_blocks > self.max_local_blocks:
            raise ValueError("actual history needs more local blocks than max_history_len provides")
        return self


_PRESETS = {
    # Same presets as config.py:110-131.
    "tiny": PCPAttentionConfig(
        pcp_size=4,
        current_len=256,
        max_history_len=2048,
        actual_history_len=2048,
        block_size=512,
        interleave_size=64,
        alignment=256,
    ),
    "full": PCPAttentionConfig(
        pcp_size=64,
        current_len=4096,
        max_history_len=131072,
        actual_history_len=131072,
        block_size=512,
        interleave_size=64,
        alignment=4096,
    ),
    # The Qwen3.5-397B target shape on 8 ranks (one per B200).
    "b200x8": PCPAttentionConfig(
        pcp_size=8,
        current_len=4096,
        max_history_len=131072,
        actual_history_len=131072,
        block_size=512,
        interleave_size=64,
        alignment=4096,
    ),
}


def get_preset(name: str) -> PCPAttentionConfig:
    try:
        return _PRESETS[name].validate()
    except KeyError as exc:
        choices = ", ".join(sorted(_PRESETS))
        raise ValueError(f"unknown preset {name!r}; choose one of: {choices}") from exc
