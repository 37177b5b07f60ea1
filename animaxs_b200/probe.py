"""Score-health probe of the attention calls: the host mirror of the
reference's NumericalMonitor score probes (.selfScores / .crossScores,
AnimaXS/Runtime/Diagnostics/NumericalMonitor.swift:17-161, bound by
AttentionExecutor.encode(probe:) to attention_softmax_rows_probe,
AnimaKernels.metal:1738-1830).

A probe slot is four device uint32 words (``animaxs_attn_set_score_probe`` in
``include/animaxs_attn.h``): OR-ed flags, the float bits of the largest
|score|, the smallest flagged key index, one unused word.
"""

from __future__ import annotations

import struct
from dataclasses import dataclass

FLAG_NAN = 1
FLAG_POS_INF = 2
FLAG_NEG_INF = 4
FLAG_HALF_OVERFLOW = 8
NO_INDEX = 0xFFFFFFFF


@dataclass(frozen=True)
class ProbeStats:
    """NumericalMonitor.Stats (NumericalMonitor.swift:136-161)."""
    flags: int = 0
    max_abs: float = 0.0
    first_index: int = NO_INDEX

    @property
    def has_issue(self) -> bool:
        return self.flags != 0

    @property
    def has_nan(self) -> bool:
        return bool(self.flags & FLAG_NAN)

    @property
    def has_pos_inf(self) -> bool:
        return bool(self.flags & FLAG_POS_INF)

    @property
    def has_neg_inf(self) -> bool:
        return bool(self.flags & FLAG_NEG_INF)

    @property
    def has_half_overflow(self) -> bool:
        return bool(self.flags & FLAG_HALF_OVERFLOW)

    @property
    def condition(self) -> str:
        """The reference's wording, in its order of precedence."""
        if self.has_nan:
            return "NaN detected"
        if self.has_pos_inf:
            return "positive Inf detected"
        if self.has_neg_inf:
            return "negative Inf detected"
        if self.has_half_overflow:
            return "value exceeded FP16 finite range"
        return "non-finite value detected"

    @classmethod
    def from_words(cls, words) -> "ProbeStats":
        w = [int(x) & 0xFFFFFFFF for x in words]
        return cls(flags=w[0], max_abs=struct.unpack("<f", struct.pack("<I", w[1]))[0], first_index=w[2])


class ScoreProbe:
    """One probe slot on ``device``: ``reset()`` (NumericalMonitor.beginRun:
    zeros, first index = UINT32_MAX), pass it to ``AttentionExecutor.encode(...,
    probe=...)`` or ``set_score_probe``, then ``read()`` after the work has
    completed."""

    def __init__(self, device):
        import torch
        self.words = torch.zeros(4, dtype=torch.int32, device=device)
        self.reset()

    def reset(self):
        self.words.zero_()
        self.words[2] = -1  # 0xFFFFFFFF

    def data_ptr(self) -> int:
        return self.words.data_ptr()

    def read(self) -> ProbeStats:
        return ProbeStats.from_words(self.words.cpu().tolist())
