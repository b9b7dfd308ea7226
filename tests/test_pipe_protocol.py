"""Host-side model of the pipelined fused scan's hand-off protocol
(ssm_scan_pipe_kernel): four warps -- two staging + decay warps, the
recurrence warp, the gate warp -- pass chunks through PIPE_NR ring slots with
three named barriers per slot (decay done: both staging warps arrive, the
recurrence warp waits; recurrence done: recurrence -> gate; gate done: the
gate warp arrives, both staging warps wait before restaging the slot).  Each
warp is modelled by the kernel's own sequence of steps; a named barrier
completes a phase when the counted threads have arrived (32 per warp) and
then starts the next phase.  Random interleavings must always finish, and no
slot may be restaged before its gate step, or read before its producer's
barrier -- the properties the kernel's comments claim.  (The gate-done
barrier alone keeps restaging safe, whatever the staging distance; the
kernel's ring depth is sized for throughput.)  The same model without the
gate-done barrier must fail, which shows the checks can fail."""
import random

import pytest

PIPE_NR, PIPE_LA, SC = 4, 1, 8


class Barriers:
    def __init__(self):
        self.arrived = {}   # id -> threads arrived in the current phase
        self.phase = {}     # id -> completed phases

    def arrive(self, bid, count, threads=32):
        a = self.arrived.get(bid, 0) + threads
        if a > count:
            raise AssertionError(f"barrier {bid}: {a} arrivals for a count of {count}")
        if a == count:
            self.arrived[bid] = 0
            self.phase[bid] = self.phase.get(bid, 0) + 1
        else:
            self.arrived[bid] = a


def warp_programs(nchunks, la=PIPE_LA, nr=PIPE_NR, guard=True):
    BA, BB, BG = 0, nr, 2 * nr

    def staging(hf):
        for c in range(min(la, nchunks)):
            yield ("stage", c, hf)
        for c in range(nchunks):
            cn = c + la
            if cn < nchunks:
                if guard and cn >= nr:
                    yield ("sync", BG + cn % nr, 96)
                yield ("stage", cn, hf)
            yield ("decay", c, hf)  # reads and writes slot c % nr
            yield ("arrive", BA + c % nr, 96)

    def recurrence():
        for c in range(nchunks):
            yield ("sync", BA + c % nr, 96)
            yield ("recur", c)
            yield ("arrive", BB + c % nr, 64)

    def gate():
        for c in range(nchunks):
            yield ("sync", BB + c % nr, 64)
            yield ("gate", c)
            if guard and c < nchunks - nr:
                yield ("arrive", BG + c % nr, 96)

    return [staging(0), staging(1), recurrence(), gate()]


def run(nchunks, seed, la=PIPE_LA, nr=PIPE_NR, guard=True):
    rng = random.Random(seed)
    bars = Barriers()
    slot = {}   # slot -> (chunk, stage reached: 'staged'x2, 'decayed'x2, 'recurred', 'gated')
    progs = warp_programs(nchunks, la, nr, guard)
    pending = [next(p, None) for p in progs]
    waiting = [None] * 4  # (barrier id, phase to pass) for warps blocked in a sync
    done_decay = {}

    def execute(w, op):
        kind = op[0]
        if kind == "stage":
            c, hf = op[1], op[2]
            s = c % nr
            held = slot.get(s)
            if held is not None and held[0] != c:
                assert held[1] == "gated", f"slot {s} restaged with chunk {c} while chunk {held[0]} is {held[1]}"
            if held is None or held[0] != c:
                slot[s] = (c, "staged")
        elif kind == "decay":
            c, hf = op[1], op[2]
            assert slot[c % nr][0] == c, f"decay of chunk {c} reads another chunk's slot"
            done_decay[(c, hf)] = True
        elif kind == "recur":
            c = op[1]
            assert slot[c % nr][0] == c and done_decay.get((c, 0)) and done_decay.get((c, 1)), \
                f"recurrence of chunk {c} before its decay"
            slot[c % nr] = (c, "recurred")
        elif kind == "gate":
            c = op[1]
            assert slot[c % nr] == (c, "recurred"), f"gate of chunk {c} before its recurrence"
            slot[c % nr] = (c, "gated")

    steps = 0
    while any(p is not None for p in pending):
        runnable = []
        for w in range(4):
            if pending[w] is None:
                continue
            if waiting[w] is not None:
                bid, target = waiting[w]
                if bars.phase.get(bid, 0) >= target:
                    runnable.append(w)
            else:
                runnable.append(w)
        if not runnable:
            raise AssertionError(f"deadlock after {steps} steps (nchunks {nchunks}, seed {seed})")
        w = rng.choice(runnable)
        op = pending[w]
        if op[0] == "sync":
            if waiting[w] is None:  # arrive, then wait for the phase to complete
                target = bars.phase.get(op[1], 0) + 1
                bars.arrive(op[1], op[2])
                if bars.phase.get(op[1], 0) < target:
                    waiting[w] = (op[1], target)
                    continue
            waiting[w] = None
        elif op[0] == "arrive":
            bars.arrive(op[1], op[2])
        else:
            execute(w, op)
        pending[w] = next(progs[w], None)
        steps += 1
    # every chunk gated, no barrier left half-arrived
    assert all(v == 0 for v in bars.arrived.values()), bars.arrived


@pytest.mark.parametrize("nchunks", [1, 2, 3, 4, 5, 6, 9, 17, 33])
def test_protocol_finishes_and_keeps_slot_order(nchunks):
    for seed in range(200):
        run(nchunks, seed)


@pytest.mark.parametrize("la", [1, 2, 3])
def test_protocol_safe_for_any_staging_distance(la):
    for seed in range(100):
        run(13, seed, la=la)


def test_checker_catches_a_missing_gate_barrier():
    """Without the gate-done barrier the staging warps can restage a slot
    whose chunk is still in flight: the model must notice."""
    failures = 0
    for seed in range(200):
        try:
            run(12, seed, guard=False)
        except AssertionError:
            failures += 1
    assert failures > 0
