"""Work split of the rope ring's consumer threads (rope.cuh, rope_ring_kernel), restated on the CPU.

Per token the consumers must rotate every (head, 8-pair group) exactly once and copy every v / k-tail
vector exactly once. With `ncons` consumer threads and `tpu` = rotary_dim / 16 groups per head:

* fixed pair groups (ncons % tpu == 0): thread ct keeps group ct % tpu and takes heads
  ct / tpu, ct / tpu + ncons / tpu, ...;
* otherwise thread ct walks the flat (head, group) list from ct in steps of ncons;
* the append copies go from the highest-numbered thread down: thread ct takes copy indices
  ncons - 1 - ct, 2 * ncons - 1 - ct, ...

The GPU tests check the results; this checks the index arithmetic over launch shapes they do not
reach (other consumer-warp counts, rotary_dims and head counts), and that every stage phase expects
exactly the bytes its copies deliver, with one arrival, in each way a token can be staged.
"""
from __future__ import annotations

import collections

import pytest


def rotations(ncons: int, tpu: int, nh: int) -> collections.Counter:
    done = collections.Counter()
    for ct in range(ncons):
        if ncons % tpu == 0:
            j, h = ct % tpu, ct // tpu
            while h < nh:
                done[(h, j)] += 1
                h += ncons // tpu
        else:
            gi = ct
            while gi < nh * tpu:
                done[(gi // tpu, gi % tpu)] += 1
                gi += ncons
    return done


def copies(ncons: int, n_copy: int) -> collections.Counter:
    done = collections.Counter()
    for ct in range(ncons):
        u = ncons - 1 - ct
        while u < n_copy:
            done[u] += 1
            u += ncons
    return done


@pytest.mark.parametrize("warps", [1, 4, 8, 12, 16])
@pytest.mark.parametrize("tpu", [1, 2, 3, 4, 5, 6, 7, 8, 16, 32])
def test_every_rotation_group_once(warps, tpu):
    ncons = 32 * warps
    for nh in (1, 2, 9, 40, 104, 130):
        done = rotations(ncons, tpu, nh)
        assert set(done) == {(h, j) for h in range(nh) for j in range(tpu)}
        assert set(done.values()) == {1}


@pytest.mark.parametrize("warps", [1, 8, 16])
def test_every_copy_once(warps):
    ncons = 32 * warps
    for n_copy in (0, 1, 64, 128, ncons, ncons + 1, 3 * ncons + 5):
        done = copies(ncons, n_copy)
        assert sorted(done) == list(range(n_copy)) and set(done.values()) <= {1}


def test_copies_go_to_the_threads_with_fewest_heads():
    # configuration 3 with the default 8 consumer warps: 40 heads of 8 groups over 256 threads, so
    # threads 0-63 rotate two groups and the rest one; the 128 v vectors go to threads 128-255
    ncons, tpu, nh = 256, 8, 40
    per_thread = collections.Counter()
    for ct in range(ncons):
        h = ct // tpu
        while h < nh:
            per_thread[ct] += 1
            h += ncons // tpu
    copy_threads = {ncons - 1 - u for u in range(128)}
    assert max(per_thread[ct] for ct in copy_threads) == 1
    assert max(per_thread.values()) == 2


def stage_accounting(pos_valid: bool, with_v: bool, prefetched: bool, q: int, k: int, v: int, c: int):
    """One stage phase of the rope ring (rope.cuh, rope_ring_kernel), following the kernel's statements:
    returns (bytes the barrier expects, bytes of the copies issued into the stage, arrivals). A
    prefetched token's q/k copies start with expect_tx before the positions are staged; the
    producer's loop then adds the cos|sin row (and v) with its one arrive.expect_tx, or arrives alone
    for a token whose position is out of range."""
    expect = []   # arguments of expect_tx / arrive.expect_tx
    copies = []   # sizes of the bulk copies issued
    arrivals = 0
    if prefetched:                       # prologue: mbar_expect_tx(q + k); q, k copies
        expect.append(q + k)
        copies += [b for b in (q, k) if b]
    if not pos_valid:                    # loop: pos < 0 -> mbar_arrive
        arrivals += 1
        return sum(expect), sum(copies), arrivals
    qk_in_flight = prefetched            # loop: arrive.expect_tx(c + v? + (q + k unless in flight))
    expect.append(c + (v if with_v else 0) + (0 if qk_in_flight else q + k))
    arrivals += 1
    if not qk_in_flight:
        copies += [b for b in (q, k) if b]
    if with_v:
        copies.append(v)
    copies.append(c)
    return sum(expect), sum(copies), arrivals


@pytest.mark.parametrize("shape", [(32 * 256, 8 * 256, 0, 512), (96 * 256, 8 * 256, 0, 512),
                                   (32 * 256, 8 * 256, 8 * 256, 512), (0, 8 * 256, 8 * 256, 256)])
def test_rope_stage_transaction_bytes_balance(shape):
    q, k, v, c = shape
    for pos_valid in (True, False):
        for with_v in ((True, False) if v else (False,)):
            for prefetched in (True, False):
                expected, copied, arrivals = stage_accounting(pos_valid, with_v, prefetched, q, k, v, c)
                assert expected == copied and arrivals == 1
                assert expected < (1 << 20)  # an mbarrier's transaction count holds under 2^20 bytes


def test_drain_waits_on_the_last_copy_into_each_stage():
    # common.cuh drain_ring: after `issued` loads into stages i % S, stage s (s < issued) is waited on
    # for the phase of load k = s + ((issued - 1 - s) // S) * S with parity (k // S) & 1. That must be
    # the last load into stage s (phases complete in order, so it covers the earlier ones).
    for stages in range(1, 9):
        for issued in range(0, 40):
            for s in range(min(stages, issued)):
                k = s + ((issued - 1 - s) // stages) * stages
                last = max(i for i in range(issued) if i % stages == s)
                assert k == last and k // stages == sum(1 for i in range(issued) if i % stages == s) - 1
