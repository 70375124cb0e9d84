"""Greedy speculative-verification decision (chomikgrad/generation.py:1-28).

Backend-neutral host logic used with ``LlamaDecoderBlock`` verify programs:
accept the longest draft prefix the target agrees with, then the target's
token at the first mismatch.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence, Tuple


@dataclass(frozen=True)
class GreedyVerification:
    emitted_tokens: Tuple[int, ...]
    accepted_draft_tokens: int


def verify_greedy_candidates(draft_tokens: Sequence[int],
                             target_tokens: Sequence[int]) -> GreedyVerification:
    draft = tuple(int(t) for t in draft_tokens)
    target = tuple(int(t) for t in target_tokens)
    if not draft:
        raise ValueError("speculative verification requires at least one token")
    if len(draft) != len(target):
        raise ValueError("draft and target blocks must have equal lengths")
    for index, (proposed, verified) in enumerate(zip(draft, target)):
        if proposed != verified:
            return GreedyVerification(draft[:index] + (verified,), index)
    return GreedyVerification(draft, len(draft))
