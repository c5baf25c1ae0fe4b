"""Continuous-depth-batching exit routing, restated on the CPU.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Restates the per-token depth bookkeeping of ``CDBScheduler._run_core`` /
``_consume_gate`` (``python/loopsgl/managers/cdb_scheduler.py:189-267``) and the
state-pool phase of ``CDBModelRunner._execute_phase``
(``model_executor/cdb_model_runner.py:81-109``) for tokens that take part in
every core step from the one after their prelude until they exit (the cohort
schedule). Exit depths are integers and must match bit-exactly.
"""

from __future__ import annotations

from typing import Sequence

import torch


def exit_depth(signals: Sequence[bool], max_depth: int, lookahead: bool) -> int:
    """Depth at which a token leaves the core, given the gate signal of each core step.

    ``signals[k]`` is the signal computed after executing loop step ``k`` (the token
    then has depth ``k+1``). Direct timing (``disable_lookahead_exit``) exits at
    ``k+1`` for the first raised ``signals[k]``; lookahead consumes step ``k``'s
    gate only after step ``k+1`` launched, so the token exits at ``k+2``
    (cdb_scheduler.py:216-222, 250-260). Full depth always exits (:262-265).
    """
    delay = 1 if lookahead else 0
    for k, raised in enumerate(signals):
        if raised:
            return min(k + 1 + delay, max_depth)
        if k + 1 >= max_depth:
            break
    return max_depth


def replay_decision(token_depth: int, replay_depth: int, lookahead: bool) -> bool:
    """``decisions[i] = token.depth >= depths[out] - delay`` (cdb_scheduler.py:207-213)."""
    return token_depth >= replay_depth - (1 if lookahead else 0)


def replay_exit_depth(replay_depth: int, max_depth: int, lookahead: bool) -> int:
    """Exit depth when the gate is replaced by a prescribed depth: exactly that depth."""
    signals = [replay_decision(k + 1, replay_depth, lookahead) for k in range(max_depth)]
    return exit_depth(signals, max_depth, lookahead)


def core_phase(
    model,
    state_pool: dict[str, torch.Tensor],
    slots: torch.Tensor,
    depths: torch.Tensor,
    batch,
    kv_pool,
) -> torch.Tensor | None:
    """``CDBModelRunner._execute_phase("core")`` (cdb_model_runner.py:94-109).

    Gathers each row's hidden (and injection, exit) state by slot, runs one loop
    step at the rows' own depths, computes the exit gate and scatters the new
    states back. Returns the gate signals (or None without an exit threshold).
    """
    hidden = state_pool["hidden"].index_select(0, slots)
    inj_pool = state_pool.get("injection")
    injection = None if inj_pool is None else inj_pool.index_select(0, slots)
    exit_pool = state_pool.get("exit")
    exit_state = None if exit_pool is None else exit_pool.index_select(0, slots)
    if getattr(kv_pool, "versions", None) is not None:
        model.resolve_core(batch, kv_pool, depths.numpy())
    hidden = model.core_step(hidden, depths, injection, batch, kv_pool)
    gates = None
    if model.cfg.exit_threshold is not None:
        gates, exit_state = model.exit_signal(hidden, exit_state, depths)
        state_pool["exit"].index_copy_(0, slots, exit_state)
    state_pool["hidden"].index_copy_(0, slots, hidden)
    return gates
