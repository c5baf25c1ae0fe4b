"""Known answers from the reference's own unit tests, checked against the oracle.

Each test restates the inputs and expected values of one reference test:
``tests/core/test_exit_gates.py:16-60``, ``tests/core/test_loop_cache.py:35-67``,
``tests/kernel/test_store_correctness.py:67-96`` and the replay-depth routing of
``tests/core/test_cdb_integration.py:206-243``.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import cdb, kvmeta, ops


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_ouro_cumulative_exit_state(dtype: torch.dtype) -> None:
    """test_exit_gates.py:16-36: hazards 0.3 / 0.1 accumulate per token after reordering."""
    hidden = torch.logit(torch.tensor([[0.3], [0.1]])).to(dtype)
    w = torch.ones(1, 1, dtype=dtype)
    b = torch.zeros(1, dtype=dtype)
    initial = torch.zeros(2, dtype=torch.float32)
    s1, p1 = ops.ouro_exit_signal(hidden, initial, 0, w, b, 0.5)
    assert s1.dtype == torch.bool and not s1.any() and p1.dtype == torch.float32
    order = torch.tensor([1, 0])
    s2, p2 = ops.ouro_exit_signal(hidden[order], p1[order], 1, w, b, 0.5)
    assert s2.tolist() == [False, True]
    torch.testing.assert_close(p2, torch.tensor([0.19, 0.51]), atol=1e-3, rtol=1e-3)
    torch.testing.assert_close(p1, torch.tensor([0.3, 0.1]), atol=1e-3, rtol=1e-3)


def test_ouro_min_loop_steps_and_lookahead() -> None:
    """ouro.py:151-155: the signal also needs step+1(+1 for a lookahead gate) >= min steps."""
    h = torch.full((1, 1), 5.0)
    w, b = torch.ones(1, 1), torch.zeros(1)
    s, _ = ops.ouro_exit_signal(h, torch.zeros(1), 0, w, b, 0.5, min_loop_steps=2)
    assert not s.any()
    s, _ = ops.ouro_exit_signal(h, torch.zeros(1), 0, w, b, 0.5, min_loop_steps=2,
                                lookahead_gate=True)
    assert s.all()
    s, _ = ops.ouro_exit_signal(h.repeat(2, 1), torch.zeros(2), torch.tensor([0, 1]), w, b, 0.5,
                                min_loop_steps=2)
    assert s.tolist() == [False, True]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_huginn_previous_state_and_threshold(dtype: torch.dtype) -> None:
    """test_exit_gates.py:39-60: zero states stay finite, equality does not exit."""
    previous = torch.tensor([[0, 0], [1, 0], [-1, -1], [1, 1]], dtype=dtype)
    current = torch.tensor([[0, 0], [2, 0], [1, 1], [1, 1]], dtype=dtype)
    signal, state = ops.huginn_exit_signal(current, previous, 0.5)
    assert signal.dtype == torch.bool and signal.tolist() == [True, False, False, True]
    assert state is current
    nxt, _ = ops.huginn_exit_signal(current.clone(), state, 0.5)
    assert nxt.all()


@pytest.mark.parametrize(
    ("policy", "num_kv", "core_first", "coda", "ouro_kv"),
    [
        ("depth_indexed", 36, [2, 6, 10, 14, 18, 22, 26, 30], [34, 35], 96),
        ("shared", 8, [2] * 8, [6, 7], 24),
    ],
)
def test_loop_cache_layout(policy, num_kv, core_first, coda, ouro_kv) -> None:
    """test_loop_cache.py:35-67: 2 + 4x8 + 2 layout and Ouro 24x4."""
    assert kvmeta.num_kv_layers(policy, 8, 2, 4, 2) == num_kv
    prelude = [kvmeta.prelude_cache_layer_index(i) for i in range(2)]
    core = [[kvmeta.core_cache_layer_index(policy, 2, 4, i, s) for i in range(4)] for s in range(8)]
    codas = [kvmeta.coda_cache_layer_index(policy, 8, 2, 4, 2, i) for i in range(2)]
    assert prelude == [0, 1]
    assert [c[0] for c in core] == core_first
    assert codas == coda
    slots = {i for c in core for i in c}
    assert len(slots) == num_kv - 4
    assert set(prelude) | slots | set(codas) == set(range(num_kv))
    assert kvmeta.num_kv_layers(policy, 4, 0, 24, 0) == ouro_kv
    assert kvmeta.core_cache_layer_index(policy, 0, 24, 0, 0) == 0
    assert kvmeta.core_cache_layer_index(policy, 0, 24, 23, 3) == ouro_kv - 1


def test_depth_indexed_needs_scalar_step() -> None:
    """base.py:84-85."""
    with pytest.raises(ValueError):
        kvmeta.core_cache_layer_index("depth_indexed", 0, 4, 0, torch.tensor([1]))


def test_store_fallback_known_answer() -> None:
    """test_store_correctness.py:67-96: padding slot 0 untouched, empty batch accepted."""
    k_storage = torch.full((9, 6), -7.0, dtype=torch.bfloat16)
    k_cache = k_storage[:, ::2]
    v_cache = torch.full((9, 5), -7.0, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(0)
    k = torch.randn(3, 3, generator=g).to(torch.bfloat16)
    v = torch.randn(3, 5, generator=g).to(torch.bfloat16)
    idx = torch.tensor([0, 8, 4])
    ek, ev = k_storage.clone(), v_cache.clone()
    ek[idx[1:], ::2] = k[1:]
    ev[idx[1:]] = v[1:]
    ops.store_kv(k_cache, v_cache, idx, k, v)
    ops.store_kv(k_cache, v_cache, idx[:0], k[:0], v[:0])
    torch.testing.assert_close(k_storage, ek, rtol=0, atol=0)
    torch.testing.assert_close(v_cache, ev, rtol=0, atol=0)
    with pytest.raises(ValueError):
        ops.store_kv(k_cache, v_cache, torch.tensor([9, 0, 0]), k, v)


@pytest.mark.parametrize("lookahead", [True, False])
def test_replay_exit_depths(lookahead: bool) -> None:
    """test_cdb_integration.py:206-243: prescribed depths (2, 4, 3) are the exit depths."""
    for depth in (2, 4, 3):
        assert cdb.replay_exit_depth(depth, 4, lookahead) == depth


def test_exit_timing() -> None:
    """cdb_scheduler.py:216-265: lookahead exits one step after the raised gate."""
    assert cdb.exit_depth([True, False, False, False], 4, lookahead=False) == 1
    assert cdb.exit_depth([True, False, False, False], 4, lookahead=True) == 2
    assert cdb.exit_depth([False, False, True, False], 4, lookahead=True) == 4
    assert cdb.exit_depth([False] * 4, 4, lookahead=True) == 4
    assert cdb.exit_depth([False, False, False, True], 4, lookahead=False) == 4


def test_last_exited_layouts() -> None:
    """last_exited.py:124-129: Ouro-1.4B has one 24-layer group and 4 slots per token;
    Huginn 2+4+2 has 4-layer slots, one core and one fixed group."""
    ouro = kvmeta.LastExitedLayout(24, 0, 24, 4)
    assert (ouro.layers_per_slot, ouro.core_groups, ouro.fixed_groups, ouro.slots_per_token) == (
        24, 1, 0, 4)
    hug = kvmeta.LastExitedLayout(8, 2, 6, 32)
    assert (hug.layers_per_slot, hug.core_groups, hug.fixed_groups) == (4, 1, 1)
    assert [hug.group_and_lane(i) for i in range(8)] == [
        (0, 0), (0, 1), (0, 0), (0, 1), (0, 2), (0, 3), (0, 2), (0, 3)]
    assert ouro.num_kv_slots(11) == 11
    v = kvmeta.LastExitedVersions(ouro, 11)
    v.reserve(np.array([1, 2]))
    assert v.free_count == 10 - 8
    v.release(np.array([1]), np.array([2]))
    assert v.free_count == 10 - 8 + 2
    assert v.slot_map[2, 1] == v.slot_map[1, 1] == v.slot_map[3, 1]
