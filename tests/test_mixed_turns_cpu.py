"""Model check of the turn protocol of the mixed-attention kernel's two tiles.

In `mixed_attention_kernel` (csrc/mixed_attention.cu) the softmax warps of
tile x wait, before block j's maximum and exponentials, on mbarrier turn(x)
with parity (j & 1) for x = 1 and ((j - 1) & 1) for x = 0, j > 0; after
their exponentials they arrive on turn(1 - x). An mbarrier parity wait
returns as soon as the barrier's current phase has the other parity, so a
waiter that falls two phases behind (or runs one ahead) would pass on a stale
phase. This test explores every interleaving of the two tiles for a few
blocks, with the barrier modelled as a phase counter, and checks that each
wait is released exactly by the arrival it is meant for and that no
interleaving deadlocks.
"""
import functools


def _explore(n_blocks):
    # state: (pc_a, pc_b, phase_a, phase_b, done_a, done_b)
    # pc: next step index of the tile; each block has two steps: "wait" and "arrive"
    # phase_x: completed phases of turn(x); done_x: exponentials of tile x finished
    # (the number of blocks whose arrive step ran)
    def steps(x, pc):
        j, k = divmod(pc, 2)
        if j >= n_blocks:
            return None
        return (j, "wait" if k == 0 else "arrive")

    @functools.lru_cache(maxsize=None)
    def reach(state):
        pc = [state[0], state[1]]
        phase = [state[2], state[3]]
        done = [state[4], state[5]]
        progressed = False
        for x in (0, 1):
            st = steps(x, pc[x])
            if st is None:
                continue
            j, kind = st
            if kind == "wait":
                if x == 0 and j == 0:  # tile A's first block needs no turn
                    ok = True
                else:
                    parity = (j if x == 1 else j - 1) & 1
                    current = phase[x]  # index of the phase in progress
                    ok = (current & 1) != parity  # try_wait.parity semantics
                    if ok:
                        # the arrival this wait is meant for: the other tile's block
                        # j (x = 1) or j - 1 (x = 0) exponentials
                        want = j if x == 1 else j - 1
                        assert done[1 - x] == want + 1, (x, j, done, phase)
                if not ok:
                    continue
                npc = list(pc)
                npc[x] += 1
                reach((npc[0], npc[1], phase[0], phase[1], done[0], done[1]))
                progressed = True
            else:
                nphase = list(phase)
                nphase[1 - x] += 1  # all working threads of tile x arrive at once
                ndone = list(done)
                ndone[x] += 1
                npc = list(pc)
                npc[x] += 1
                reach((npc[0], npc[1], nphase[0], nphase[1], ndone[0], ndone[1]))
                progressed = True
        finished = steps(0, pc[0]) is None and steps(1, pc[1]) is None
        assert progressed or finished, ("deadlock", state)
        return True

    return reach((0, 0, 0, 0, 0, 0))


def test_turns_release_only_on_the_intended_arrival():
    for n in range(1, 7):
        assert _explore(n)


def test_turns_strictly_alternate():
    # A's exponentials of block j always precede B's of block j, which precede
    # A's of block j + 1: follow the only schedule the waits allow
    n = 5
    order = []
    pc = [0, 0]
    phase = [0, 0]
    while len(order) < 2 * n:
        moved = False
        for x in (0, 1):
            j, k = divmod(pc[x], 2)
            if j >= n:
                continue
            if k == 0:
                if not (x == 0 and j == 0):
                    parity = (j if x == 1 else j - 1) & 1
                    if (phase[x] & 1) == parity:
                        continue
                pc[x] += 1
            else:
                order.append((x, j))
                phase[1 - x] += 1
                pc[x] += 1
            moved = True
        assert moved
    assert order == [(x, j) for j in range(n) for x in (0, 1)]
