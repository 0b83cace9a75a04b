"""Discrete-event model of the fused relay's release / acquire protocol (reduce-scatter +
all-gather form), run on CPU with random timings.

It mirrors kernrelay_b200/csrc/relay.cu: the GEMM epilogues add to the local rs_done[t];
one signal job per (tile, counter) forwards a completed rs_done[t] / ag_done[t] to
rs_cnt[t][rank] / ag_cnt[t][rank] on every rank; the consumer's phase loop takes
reduce-scatter(next_rs) or all-gather(next_ag) by the kernel's rule -- the fixed pipeline
(rs(t+1) before ag(t), one tile per phase) or the readiness order (whichever of the two is
ready, reduce-scatter first, each merged with the following tiles that are ready too) --
and an all-gather never precedes its own reduce-scatter.  Each reduce-scatter completion
adds to ag_done[t] of every tile it covered.  Checked for k in
{2, 4, 8}, T in {1, 2, 4, 8}, both orders and several layers (monotone counters with
per-layer targets): every rank finishes every layer (no deadlock), and a rank's all-gather
of tile t starts only after every owner finished its reduce-scatter of tile t.
"""
import heapq
import random

import pytest


def simulate(k, T, layers, ready_order, seed):
    rng = random.Random(seed)
    gemm_per_tile = 3                      # GEMM tiles (epilogue releases) per row tile
    t_now = 0.0
    events = []                            # (time, seq, kind, payload)
    seq = [0]

    def push(dt, kind, payload):
        seq[0] += 1
        heapq.heappush(events, (t_now + dt, seq[0], kind, payload))

    rs_done = [[0] * T for _ in range(k)]          # local, per rank
    ag_done = [[0] * T for _ in range(k)]
    rs_cnt = [[[0] * k for _ in range(T)] for _ in range(k)]   # [rank][t][src]
    ag_cnt = [[[0] * k for _ in range(T)] for _ in range(k)]
    rs_finished = [[set() for _ in range(T)] for _ in range(layers)]  # owners done, per layer
    state = []
    for r in range(k):
        state.append({"layer": 0, "next_rs": 0, "next_ag": 0, "busy": False, "done": False})
    forwarded_rs = [[0] * T for _ in range(k)]     # layers forwarded by the signal jobs
    forwarded_ag = [[0] * T for _ in range(k)]

    def start_layer(r, l):
        # the GEMM of layer l on rank r: tiles of row tile t complete in band order
        base = 0.0
        for t in range(T):
            for _ in range(gemm_per_tile):
                base += rng.uniform(0.5, 1.5)
                push(base, "epi", (r, t))

    def ready(r, cnt, t, target):
        return all(cnt[r][t][s] >= target for s in range(k))

    def try_consume(r):
        st = state[r]
        if st["busy"] or st["done"]:
            return
        l = st["layer"]
        target = l + 1                        # per-layer target of the monotone counters
        if st["next_ag"] >= T:
            # layer finished: the next layer's GEMM starts (it needs the all-gathers done)
            st["layer"] += 1
            st["next_rs"] = st["next_ag"] = 0
            if st["layer"] == layers:
                st["done"] = True
                return
            start_layer(r, st["layer"])
            return
        nr, na = st["next_rs"], st["next_ag"]
        if not ready_order:
            # fixed pipeline: rs(t+1) before ag(t), one tile per phase, blocking waits
            do_rs = nr < T and nr <= na + 1
            t0 = nr if do_rs else na
            if not ready(r, rs_cnt if do_rs else ag_cnt, t0, target):
                return                         # blocking wait: resumed on a counter change
            t1 = t0 + 1
        else:
            # readiness order: the reduce-scatter when ready, else the all-gather (only
            # behind its own reduce-scatter), each extended over the following tiles that
            # are ready too (one merged phase)
            if nr < T and ready(r, rs_cnt, nr, target):
                do_rs, t0, t1 = True, nr, nr + 1
                while t1 < T and ready(r, rs_cnt, t1, target):
                    t1 += 1
            elif na < nr and ready(r, ag_cnt, na, target):
                do_rs, t0, t1 = False, na, na + 1
                while t1 < nr and ready(r, ag_cnt, t1, target):
                    t1 += 1
            else:
                return                         # poll again when a counter changes
        st["busy"] = True
        if do_rs:
            push(rng.uniform(0.2, 1.0) * (t1 - t0), "rs_end", (r, t0, t1, l))
        else:
            for t in range(t0, t1):
                # invariant: every owner finished its reduce-scatter of tile t in layer l
                assert rs_finished[l][t] == set(range(k)), (l, t, rs_finished[l][t])
            push(rng.uniform(0.2, 1.0) * (t1 - t0), "ag_end", (r, t0, t1, l))

    for r in range(k):
        start_layer(r, 0)
    steps = 0
    while events:
        t_now, _, kind, p = heapq.heappop(events)
        steps += 1
        assert steps < 10_000_000
        if kind == "epi":
            r, t = p
            rs_done[r][t] += 1
            # signal job: forwards once the local count for the next layer is complete
            while rs_done[r][t] >= (forwarded_rs[r][t] + 1) * gemm_per_tile:
                forwarded_rs[r][t] += 1
                push(rng.uniform(0.1, 0.5), "fwd_rs", (r, t))
        elif kind == "fwd_rs":
            r, t = p
            for dst in range(k):
                rs_cnt[dst][t][r] += 1
        elif kind == "rs_end":
            r, t0, t1, l = p
            state[r]["busy"] = False
            state[r]["next_rs"] = t1
            for t in range(t0, t1):
                rs_finished[l][t].add(r)
                ag_done[r][t] += 1
                while ag_done[r][t] >= forwarded_ag[r][t] + 1:
                    forwarded_ag[r][t] += 1
                    push(rng.uniform(0.1, 0.5), "fwd_ag", (r, t))
        elif kind == "fwd_ag":
            r, t = p
            for dst in range(k):
                ag_cnt[dst][t][r] += 1
        elif kind == "ag_end":
            r, t0, t1, l = p
            state[r]["busy"] = False
            state[r]["next_ag"] = t1
        for r in range(k):
            for _ in range(3):
                before = (state[r]["busy"], state[r]["layer"], state[r]["next_ag"])
                try_consume(r)
                if (state[r]["busy"], state[r]["layer"], state[r]["next_ag"]) == before:
                    break
    return [s["done"] for s in state], state


@pytest.mark.parametrize("ready_order", [False, True], ids=["pipeline", "ready"])
@pytest.mark.parametrize("k", [2, 4, 8])
@pytest.mark.parametrize("T", [1, 2, 4, 8])
def test_relay_protocol_terminates_and_orders_phases(k, T, ready_order):
    for seed in range(20):
        done, state = simulate(k, T, layers=3, ready_order=ready_order, seed=seed * 101 + k * 7 + T)
        assert all(done), (k, T, ready_order, seed, state)
