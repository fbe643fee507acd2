"""Host-side sharding of utterance batches across GPUs (one process per GPU).

Utterances are independent, so there is no collective on the decode path: each
rank decodes a disjoint shard on its own device and the host gathers the token
lists afterwards. The partition is computed identically on every rank: by default
pk_shard_balanced (each shard's modelled decode time bounded: the longest
utterances, whose sequential decodes set a shard's call time, share shards, and
the short ones fill the rest), or pk_shard_lpt (longest-processing-time by frame
count).
"""
from __future__ import annotations

from typing import Dict, List, Sequence

import numpy as np


def shard_indices(n_frames: Sequence[int], world: int, policy: str = "balanced") -> List[np.ndarray]:
    """Utterance indices of each rank (ascending within a rank); policy "balanced"
    (pk_shard_balanced) or "lpt" (pk_shard_lpt)."""
    from . import shard_balanced, shard_lpt
    if policy not in ("balanced", "lpt"):
        raise ValueError(f"unknown sharding policy {policy!r}")
    owner = (shard_balanced if policy == "balanced" else shard_lpt)(n_frames, world)
    return [np.nonzero(owner == r)[0].astype(np.int64) for r in range(world)]


def sub_batch(enc: np.ndarray, offs: np.ndarray, n_frames: np.ndarray, idx: np.ndarray):
    """Contiguous copy of the utterances `idx` of a ragged batch: (enc, offs, n_frames)."""
    n = np.asarray(n_frames, np.int32)[idx]
    new_offs = np.zeros(len(idx), np.int64)
    if len(idx) > 1:
        new_offs[1:] = np.cumsum(n.astype(np.int64))[:-1]
    parts = [enc[int(offs[i]):int(offs[i]) + int(n_frames[i])] for i in idx]
    sub = np.concatenate(parts, axis=0) if parts else np.zeros((0, enc.shape[1]), enc.dtype)
    return np.ascontiguousarray(sub), new_offs, n


def gather_in_order(B: int, parts: List[Dict]) -> List[np.ndarray]:
    """Reassemble per-rank results {"idx": indices, "tokens": [...]} in batch order."""
    out: List[np.ndarray] = [None] * B  # type: ignore[list-item]
    for p in parts:
        for i, t in zip(p["idx"], p["tokens"]):
            out[int(i)] = np.asarray(t, np.int32)
    missing = [i for i, t in enumerate(out) if t is None]
    if missing:
        raise RuntimeError(f"utterances {missing[:8]} were not decoded by any rank")
    return out
