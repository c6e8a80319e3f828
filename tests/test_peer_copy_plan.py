"""Host logic of the peer-memory exchange of the owner-sharded groupby (sharded.peer_copy_plan):
executing every rank's planned copies in a model of the address space must leave each owner's
receive buffer laid out exactly as the all-to-all leaves it -- senders in rank order, each
sender's rows in digit order, hashes at the buffer's start and values cap * 8 bytes in."""
import numpy as np
import pytest

from winrapids_b200.sharded import RADIX_DIGITS, owned_digits, owner_totals, peer_copy_plan


@pytest.mark.parametrize("world", [2, 3, 4, 8])
@pytest.mark.parametrize("value_bytes", [4, 8])
def test_plan_reproduces_the_all_to_all_layout(world, value_bytes):
    lo = owned_digits(world)
    rng = np.random.default_rng(world * 10 + value_bytes)
    counts = rng.integers(0, 40, (world, RADIX_DIGITS))
    counts[rng.random((world, RADIX_DIGITS)) < 0.2] = 0  # empty digits, and some empty (sender, owner) blocks
    counts = counts.tolist()
    sends = [[(s, d, i) for d in range(RADIX_DIGITS) for i in range(counts[s][d])] for s in range(world)]
    want = [[r for s in range(world) for r in sends[s] if lo[q] <= r[1] < lo[q + 1]] for q in range(world)]
    cap = max(len(w) for w in want) + 5
    vgap = 1 << 30  # values of a sender's rows start this far after its hashes
    send_base = [(s + 1) << 40 for s in range(world)]
    recv_base = [(q + 1) << 50 for q in range(world)]
    mem = {}
    for s in range(world):
        for i, r in enumerate(sends[s]):
            mem[send_base[s] + 8 * i] = r
            mem[send_base[s] + vgap + value_bytes * i] = r
    n_recv = None
    for s in range(world):
        copies, n_recv = peer_copy_plan(counts, s, lo, cap, value_bytes, send_base[s], send_base[s] + vgap, recv_base)
        assert len(copies) <= 32
        for src, dst, nb in copies:
            assert nb > 0
            width = 8 if src - send_base[s] < vgap else value_bytes
            for k in range(0, nb, width):
                mem[dst + k] = mem[src + k]
    rows = owner_totals(counts, lo)
    for q in range(world):
        assert n_recv[q] == len(want[q]) == sum(rows[s][q] for s in range(world))
        got_h = [mem[recv_base[q] + 8 * i] for i in range(n_recv[q])]
        got_v = [mem[recv_base[q] + 8 * cap + value_bytes * i] for i in range(n_recv[q])]
        assert got_h == want[q] and got_v == want[q]


def test_owned_digits_cover_every_digit_once():
    for world in range(1, 9):
        lo = owned_digits(world)
        assert lo[0] == 0 and lo[-1] == RADIX_DIGITS and all(a <= b for a, b in zip(lo, lo[1:]))
