"""Per-rollout seed derivation (behaviour of the reference's ``verl_omni/agent_loop/utils.py:18-45``).

Every post-repeat rollout row gets ``(base * 1_000_003 + index) mod (2^63 - 1)`` where ``base`` is the
step's ``meta_info["rollout_seed"]`` and ``index`` the row's trainer-assigned global index (falls back
to the local position).  Keeping the formula lets a run seeded the same way draw the same noise per
row regardless of how rows are split over workers or packed into device batches.
"""

from __future__ import annotations

from typing import Optional

_MAX_SEED = (1 << 63) - 1


def derive_rollout_seed(base_seed: int, rollout_index: int) -> int:
    return (int(base_seed) * 1_000_003 + int(rollout_index)) % _MAX_SEED


def maybe_per_rollout_seeds(meta_info: dict, batch_size: int, global_indices=None) -> Optional[list[int]]:
    base = meta_info.get("rollout_seed")
    if base is None:
        return None
    if global_indices is None:
        return [derive_rollout_seed(base, i) for i in range(batch_size)]
    idx = [int(i) for i in list(global_indices)]
    if len(idx) != batch_size:
        raise ValueError(f"Expected {batch_size} global rollout indices, got {len(idx)}")
    return [derive_rollout_seed(base, i) for i in idx]
