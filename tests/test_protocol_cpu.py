"""CPU: the fused collectives' flag / slot protocol explored under random interleavings at 2, 4 and 8
ranks (no race, no deadlock), and the checker catches the race when the partial slots do not alternate."""
import random

import pytest

from packmla.parallel.protocol import ProtocolError, ProtocolModel, explore


@pytest.mark.parametrize("rotate", [False, True])
@pytest.mark.parametrize("world,schedules", [(2, 1000), (4, 250), (8, 75)])
def test_protocol_has_no_race_or_deadlock(world, schedules, rotate):
    rng = random.Random(world)
    modes = [rng.random() < 0.5 for _ in range(6)]
    modes[:2] = [True, False]  # both modes, and a switch between them
    out = explore(world, tiles=3, modes=modes, schedules=schedules, seed=world, rotate_owners=rotate)
    assert out["checked_reads"] == schedules * sum(
        3 * (world * world if one else world + world) for one in modes)


def test_single_partial_slot_races_in_one_shot():
    with pytest.raises(ProtocolError, match="read recv"):
        explore(2, tiles=1, modes=[True] * 6, schedules=2000, seed=1, parity_slots=False)


def test_model_detects_a_missing_flag_wait():
    with pytest.raises(ProtocolError):
        for seed in range(200):
            m = ProtocolModel(2, 1, [True])
            for cta in m.active[0]:  # rank 0 reads before acquiring the peer's flag
                cta.steps = [s for s in cta.steps if s[0] != "acquire_rs"]
            m.run(random.Random(seed))


def test_fused_ep_exchange_protocol_has_no_race_and_the_early_dispatch_bug_is_caught():
    import pytest

    from packmla.parallel.ep_protocol import explore
    from packmla.parallel.protocol import ProtocolError

    for world in (2, 4, 8):
        assert explore(world, tokens=3, topk=2, experts=2 * world, calls=3, schedules=60, seed=world) == 60
        assert explore(world, tokens=3, topk=2, experts=2 * world, calls=3, schedules=60, seed=world,
                       arrival_order=True) == 60  # owners serve sources as their flags arrive
    for arrival in (False, True):
        with pytest.raises(ProtocolError):
            explore(4, tokens=3, topk=2, experts=8, calls=3, schedules=200, seed=1, wait_all_back=False,
                    arrival_order=arrival)


def test_fused_ep_exchange_data_path_matches_dense_moe():
    import torch

    from packmla.parallel.ep_protocol import emulate_exchange

    g = torch.Generator().manual_seed(3)
    world, T, k, H, E = 4, 5, 3, 16, 8
    W = torch.randn(E, H, H, generator=g)

    def expert_fn(rows, e):
        return torch.einsum("nh,nhg->ng", rows.float(), W[e])

    h = [torch.randn(T, H, generator=g) for _ in range(world)]
    ids = [torch.randint(0, E, (T, k), generator=g) for _ in range(world)]
    w = [torch.rand(T, k, generator=g) for _ in range(world)]
    out = emulate_exchange(h, ids, w, E, expert_fn)
    for r in range(world):
        dense = sum(w[r][:, j, None] * expert_fn(h[r], ids[r][:, j]) for j in range(k))
        torch.testing.assert_close(out[r], dense, atol=1e-4, rtol=1e-4)
