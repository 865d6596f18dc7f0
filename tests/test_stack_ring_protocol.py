"""A model of one CTA of the persistent stack kernel (moe_stack.cuh) run
under random schedules, to check its tile ring with per-layer tile counts
(mixed-type stacks) on the CPU.

The model keeps what the protocol's safety rests on: S stages with a `full`
and an `empty` mbarrier each, waited on by PARITY (a wait for parity p
returns once the barrier's completed-phase count is odd when p = 0 and even
when p = 1, so it cannot tell phase p from phase p + 2); the producer warp
issuing ring index g into stage g % S after waiting `empty` for parity
(g / S - 1) & 1, in rounds of min(32, S) tiles of one phase (gate/up or down
of one layer) issued in any order; tile g of the ring read by consumer warp
g % nw after waiting `full` for parity (g / S) & 1; a barrier of all 16
consumer warps after each layer's input staging, after gate/up, after the h
quantization and after down; the three routing buffers (the producer routes
layer j + 1 after layer j's gate/up tiles, and buffer j % 3 is free again
once the consumers have started layer j + 1). Copies land at random later
times. A consumer that finds another tile in its stage, or a schedule in
which no actor can move, fails the check.

The launcher's rule (moe_stack.cu fit_ring): S = the stages that fit when
no phase of any layer has more than that many tiles for one CTA, else that
count rounded down to a multiple of nw.
"""
import random

import pytest

W_CONSUMERS = 16


def plan_stages(fit, nw, layers):
    most = max(max(a, b) for a, b in layers)
    return fit if most <= fit else fit // nw * nw


def simulate(layers, S, nw, seed):
    """layers: [(tiles of gate/up, tiles of down)] for one CTA. Returns None
    or a description of the first violation."""
    rnd = random.Random(seed)
    full_done = [0] * S
    empty_done = [0] * S
    content = [-1] * S
    landing = []                                   # (stage, ring index) issued, not landed
    L = len(layers)
    starts, g = [], 0
    for a, b in layers:
        starts.append(g)
        g += a + b

    # producer program: ("route", j) | ("phase", first, n)
    prog = [("route", 0)]
    for l, (a, b) in enumerate(layers):
        prog.append(["phase", starts[l], a, 0])      # first ring index, tiles, tiles issued
        if l + 1 < L:
            prog.append(("route", l + 1))
        prog.append(["phase", starts[l] + a, b, 0])
    pc, rnd_left = 0, None
    routed = -1                                    # layers routed so far (last index)
    released = -1                                  # routing buffers of layers <= released are free

    # consumer programs: lists of steps per warp
    def warp_prog(w):
        out = []
        for l, (a, b) in enumerate(layers):
            out.append(("route_wait", l) if w == 0 else ("nop", l))
            out.append(("bar", 4 * l + 0))
            if w == 0:
                out.append(("release", l - 1))
            g0 = starts[l]
            out += [("tile", x) for x in range(g0, g0 + a) if x % nw == w and w < nw]
            out.append(("bar", 4 * l + 1))
            out.append(("bar", 4 * l + 2))
            out += [("tile", x) for x in range(g0 + a, g0 + a + b) if x % nw == w and w < nw]
            out.append(("bar", 4 * l + 3))
        return out

    progs = [warp_prog(w) for w in range(W_CONSUMERS)]
    pos = [0] * W_CONSUMERS
    bar_arrived = {}

    def parity_ok(done, p):
        return (done & 1) != p

    while True:
        moves = []
        # producer
        if pc < len(prog):
            kind = prog[pc][0]
            if kind == "route":
                j = prog[pc][1]
                if j < 3 or released >= j - 3:
                    moves.append(("p_route",))
            else:
                if rnd_left is None:
                    moves.append(("p_round",))
                else:
                    for x in rnd_left:
                        s = x % S
                        if x < S or parity_ok(empty_done[s], (x // S - 1) & 1):
                            moves.append(("p_issue", x))
        for i, (s, x) in enumerate(landing):
            moves.append(("land", i))
        for w in range(W_CONSUMERS):
            if pos[w] >= len(progs[w]):
                continue
            step = progs[w][pos[w]]
            if step[0] == "route_wait":
                if routed >= step[1]:
                    moves.append(("c", w))
            elif step[0] == "tile":
                x = step[1]
                if parity_ok(full_done[x % S], (x // S) & 1):
                    moves.append(("c", w))
            elif step[0] == "bar":
                if bar_arrived.get(step[1], set()) != set(range(W_CONSUMERS)) and w not in bar_arrived.get(step[1], set()):
                    moves.append(("c", w))
                elif bar_arrived.get(step[1], set()) == set(range(W_CONSUMERS)):
                    moves.append(("c", w))
            else:
                moves.append(("c", w))
        if not moves:
            if pc >= len(prog) and all(pos[w] >= len(progs[w]) for w in range(W_CONSUMERS)) and not landing:
                return None
            return "deadlock"
        m = rnd.choice(moves)
        if m[0] == "p_route":
            routed = prog[pc][1]
            pc += 1
        elif m[0] == "p_round":
            _, first, n, done = prog[pc]
            if done >= n:
                pc += 1
                continue
            cnt = min(min(32, S), n - done)
            rnd_left = list(range(first + done, first + done + cnt))
            prog[pc][3] = done + cnt
        elif m[0] == "p_issue":
            x = m[1]
            rnd_left.remove(x)
            landing.append((x % S, x))
            if not rnd_left:
                rnd_left = None
                if prog[pc][3] >= prog[pc][2]:
                    pc += 1
        elif m[0] == "land":
            s, x = landing.pop(m[1])
            content[s] = x
            full_done[s] += 1
        else:
            w = m[1]
            step = progs[w][pos[w]]
            if step[0] == "tile":
                x = step[1]
                if content[x % S] != x:
                    return f"warp {w} read stage {x % S} for ring index {x} but it holds {content[x % S]}"
                empty_done[x % S] += 1
                pos[w] += 1
            elif step[0] == "bar":
                arr = bar_arrived.setdefault(step[1], set())
                if w not in arr:
                    arr.add(w)
                    if arr != set(range(W_CONSUMERS)):
                        continue               # arrived; passes once all have arrived
                pos[w] += 1
            elif step[0] == "release":
                released = max(released, step[1])
                pos[w] += 1
            else:
                pos[w] += 1


def random_layers(rnd, n, a_choices, b_choices):
    return [(rnd.choice(a_choices), rnd.choice(b_choices)) for _ in range(n)]


@pytest.mark.parametrize("fit,nw,a_choices,b_choices", [
    (25, 16, [12], [12]),            # config 2 (Q2_K): 25 stages, any warp may take a stage
    (21, 16, [12, 24], [12, 16]),    # mixed with Q6_K gate/up (2-row tiles): S rounded to 16
    (21, 16, [12], [12, 16]),        # mixed without it: 21 stages
    (11, 11, [12], [16]),            # 20 KB stages: 11 stages, 11 tile warps
    (9, 9, [3, 5, 12], [2, 16]),     # small CTA shares next to large ones
])
def test_ring_never_aliases_under_the_launch_rule(fit, nw, a_choices, b_choices):
    rnd = random.Random(fit * 100 + nw)
    for run in range(60):
        layers = random_layers(rnd, 6, a_choices, b_choices)
        S = plan_stages(fit, nw, layers)
        err = simulate(layers, S, nw, seed=run)
        assert err is None, (layers, S, nw, err)


def test_the_model_catches_parity_aliasing():
    """Planted mistake, in the model only: 21 stages (not a multiple of 16
    tile warps) while a phase has 24 tiles. Some schedule then lets a warp
    pass a wait on a stage two phases ahead."""
    rnd = random.Random(7)
    found = None
    for run in range(400):
        layers = random_layers(rnd, 4, [24], [16])
        err = simulate(layers, 21, 16, seed=run)
        if err is not None:
            found = err
            break
    assert found is not None
