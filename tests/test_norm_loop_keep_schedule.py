"""The register-resident persistent RMSNorm loop (norm.cuh, norm_loop_keep_kernel), restated on the CPU.

Per CTA: rows g0, g0 + gstep, ...; iteration k uses stage k % S. Thread 0 fills stages 0 .. S-1 up
front; in iteration k every thread waits on stage k % S with parity (k / S) & 1, reads the stage
(first pass), writes its warp's partial sum into reduction slot k & 1, and joins the CTA barrier;
after the barrier thread 0 refills stage k % S with the row S iterations ahead, and every thread
reads the slot and runs the second pass from registers. No barrier closes the iteration.

The model below runs the threads of one CTA in random interleavings (bulk copies landing at random
later times) and checks what the kernel relies on: a wait never passes on a stale phase and never
sees a stage two phases ahead, a stage is refilled only after every thread has read it, each thread
reads the reduction slot written in its own iteration, every row is processed once, and the fills in
flight when an iteration's wait gives up are exactly the ones the kernel drains. A second group of
tests restates the host's launch shape (threads per row, shared memory, copy alignment) for every H
the kernel takes. The GPU tests check the results on the shapes they run.
"""
from __future__ import annotations

import math
import random

import pytest

KMAX_SMEM = 227 * 1024


def simulate(rows: int, g0: int, gstep: int, stages: int, threads: int, seed: int) -> list[int]:
    rng = random.Random(seed)
    my_rows = list(range(g0, rows, gstep))
    n = len(my_rows)
    fills = [[] for _ in range(stages)]        # per stage: rows filled, in order (phase i = fills[s][i])
    landed = [0] * stages                      # completed phases per stage
    in_flight = []                             # (stage, row) copies not yet landed
    slot = [None, None]                        # reduction slots: iteration that last wrote them
    writes_left = {}                           # iteration -> threads still to write its slot
    readers_left = [set(range(threads)) for _ in range(n)]  # threads still to read iteration k's stage
    pc = [(0, "wait")] * threads               # per thread: (iteration, next step)
    at_barrier = {}
    processed = []

    def issue(k):
        s = k % stages
        assert all(st != s for st, _ in in_flight)  # the stage's previous copy has landed
        fills[s].append(my_rows[k])
        in_flight.append((s, my_rows[k]))

    for k in range(min(stages, n)):
        issue(k)
    while True:
        runnable = []
        for t in range(threads):
            k, step = pc[t]
            if k >= n:
                continue
            s = k % stages
            if step == "wait" and landed[s] < k // stages + 1:
                continue
            if step == "barrier" and at_barrier.get(k, 0) < threads:
                continue
            runnable.append(t)
        if in_flight and (not runnable or rng.random() < 0.3):
            s, row = in_flight.pop(rng.randrange(len(in_flight)))  # copies land in any order
            assert fills[s][landed[s]] == row
            landed[s] += 1
            continue
        if not runnable:
            break
        t = rng.choice(runnable)
        k, step = pc[t]
        s = k % stages
        if step == "wait":
            # the parity wait passes on phase k // S, and the stage is never two phases ahead
            assert landed[s] in (k // stages + 1,), (k, landed[s])
            pc[t] = (k, "pass1")
        elif step == "pass1":
            assert fills[s][k // stages] == my_rows[k]  # the stage holds this iteration's row
            readers_left[k].discard(t)
            slot[k & 1] = k
            writes_left[k] = writes_left.get(k, threads) - 1
            at_barrier[k] = at_barrier.get(k, 0) + 1
            pc[t] = (k, "barrier")
        elif step == "barrier":
            if t == 0 and k + stages < n:
                assert not readers_left[k]  # every thread has read stage s before its refill
                issue(k + stages)
            pc[t] = (k, "pass2")
        elif step == "pass2":
            assert writes_left[k] == 0 and slot[k & 1] == k  # the slot still holds this iteration's sums
            if t == 0:
                processed.append(my_rows[k])
            pc[t] = (k + 1, "wait")
    assert all(pc[t][0] == n for t in range(threads))
    return processed


@pytest.mark.parametrize("stages", [2, 3, 4, 8])
@pytest.mark.parametrize("threads", [1, 2, 5])
def test_ring_schedule_in_random_interleavings(stages, threads):
    for seed in range(40):
        rows, gstep = 97, 13
        for g0 in (0, 5, 12):
            assert simulate(rows, g0, gstep, stages, threads, seed) == list(range(g0, rows, gstep))


@pytest.mark.parametrize("stages", [2, 3, 5])
def test_fills_outstanding_at_a_give_up_are_the_drained_ones(stages):
    # Fills are issued for iterations 0 .. S-1 up front and for k + S after iteration k's barrier. A
    # wait that gives up in iteration k is reached after barriers 0 .. k-1, so the fills issued are
    # those of iterations 0 .. min(n, k + S) - 1, and the ones not yet consumed are k .. k + S - 1
    # (clipped to the CTA's rows): exactly what the kernel waits for before it exits.
    for n in (1, 2, 7, 20):
        for k in range(n):
            issued = set(range(min(n, stages))) | {j + stages for j in range(k) if j + stages < n}
            unconsumed = issued - set(range(k))
            drained = {k + m for m in range(stages) if k + m < n}
            assert unconsumed == drained


def launch_shape(H: int, elem: int = 2, stages: int = 2):
    """The host's choice for norm_loop_keep_kernel (mas_b200.cu, run_norm), or None if it does not apply."""
    nv = H // 8
    if H % 8 or not (nv > 3 * 128 and nv <= 4 * 192):
        return None
    nt = math.ceil(math.ceil(nv / 4) / 32) * 32
    smem = stages * 2 * H * elem + stages * 8 + 2 * (nt // 32) * 4
    return nt, smem


def test_kernel_covers_3072_lt_h_le_6144():
    taken = [H for H in range(8, 16384, 8) if launch_shape(H)]
    assert taken[0] == 3080 and taken[-1] == 6144


@pytest.mark.parametrize("elem", [2])
def test_launch_shape_for_every_h(elem):
    for H in range(3080, 6145, 8):
        nt, smem = launch_shape(H, elem)
        nv = H // 8
        assert nt in (128, 160, 192)  # the three instantiated widths
        assert 4 * nt >= nv           # MAXV = 4 vectors per thread cover the row
        assert smem <= KMAX_SMEM
        row = H * elem
        stage = 2 * row
        assert row % 16 == 0          # bulk-copy sizes
        for s in range(8):
            assert (s * stage) % 16 == 0 and (s * stage + row) % 16 == 0  # bulk-copy destinations
            assert (s * stage) % 8 == 0                                    # mbarriers after s stages


def test_every_stage_count_the_host_allows_fits():
    # the host clamps MAS_NORM_STAGES to 2 .. 8; at the widest row (H = 6144, bf16: 24 KB of x and r
    # per stage) 8 stages still fit one CTA's shared memory, so the clamp never sends the kernel a
    # ring larger than the opt-in limit (the host also checks, and takes the older loop if not)
    for H in range(3080, 6145, 8):
        for stages in range(2, 9):
            assert launch_shape(H, stages=stages)[1] <= KMAX_SMEM
