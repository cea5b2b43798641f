"""CPU: the plan of the tensor-core MLP forward's balanced two-launch schedule
(ttt_mlp_fwd_schedule_plan, the same host and segment code the launches use) covers every
stream's mini-batches exactly once, in order, and never keeps a stream on a shared SM for
its whole sequence."""

import pytest

import _lib


def _check_plan(S, NC, M, ratio_milli):
    launches, rows = _lib.forward_schedule_plan(S, NC, M, ratio_milli)
    assert launches == 2
    D = S - M
    seen = {}
    engines = {1: set(), 2: set()}
    paired = {1: set(), 2: set()}
    for launch, cta, eng, s, n0, n1 in rows:
        assert launch in (1, 2) and 0 <= cta < M and eng in (0, 1) and 0 <= s < S
        assert 0 <= n0 < n1 <= NC
        assert (cta, eng) not in engines[launch]  # one stream per engine per launch
        engines[launch].add((cta, eng))
        if eng == 1:
            assert cta < D  # only the first D CTAs run two streams
        if cta < D:
            paired[launch].add(s)
        seen.setdefault(s, []).append((launch, n0, n1))
    assert sorted(seen) == list(range(S))
    for s, segs in seen.items():
        segs.sort()
        assert [l for l, _, _ in segs] == [1, 2], s  # one segment per launch
        (_, a0, a1), (_, b0, b1) = segs
        assert a0 == 0 and a1 == b0 and b1 == NC, s  # [0, x) then [x, NC)
    for launch in (1, 2):  # D CTAs with two engines, the rest with one
        assert sum(1 for c, e in engines[launch] if c < D) == 2 * D
        assert len(paired[launch]) == 2 * D
    assert not (paired[1] & paired[2])  # no stream shares an SM in both launches
    # both launches last about kp * r alone-mini-batch times (rounding of kp aside)
    r = (ratio_milli or 1550) / 1000
    kp = next(n1 for l, c, e, s, n0, n1 in rows if l == 1 and c < D)
    ka = NC - kp
    assert abs(kp * r - ka) <= r + 1


@pytest.mark.parametrize("M", [148, 132, 160])
@pytest.mark.parametrize("extra", [1, 2, 17, "third"])
@pytest.mark.parametrize("NC", [4, 5, 13, 128, 512])
def test_plan_covers_every_mini_batch_once(M, extra, NC):
    S = M + (M // 3 if extra == "third" else extra)
    _check_plan(S, NC, M, 0)


@pytest.mark.parametrize("ratio", [1000, 1448, 2000, 4000])
def test_plan_follows_the_ratio(ratio):
    _check_plan(192, 128, 148, ratio)


@pytest.mark.parametrize("S,NC", [(148, 128), (100, 128), (198, 128), (296, 128), (192, 3), (1024, 512)])
def test_plan_not_applicable(S, NC):
    assert _lib.forward_schedule_plan(S, NC, 148)[0] == 0


def test_plan_respects_the_switch():
    try:
        _lib.set_forward_schedule(False)
        assert _lib.forward_schedule_plan(192, 128, 148)[0] == 0
    finally:
        _lib.set_forward_schedule(True)
    assert _lib.forward_schedule_plan(192, 128, 148)[0] == 2


def test_plan_rejects_bad_arguments():
    with pytest.raises(RuntimeError, match="ratio"):
        _lib.forward_schedule_plan(192, 128, 148, 999)
    with pytest.raises(RuntimeError, match="positive"):
        _lib.forward_schedule_plan(0, 128, 148)
