"""Host-side logic of bench.py that runs without a GPU: the step pipeline of the
end-to-end leg (launch / finish order with one or two steps in flight)."""
import pytest

import bench


def _trace(n, depth):
    ev = []
    bench.pipelined(n, lambda i: ev.append(("launch", i)), lambda i: ev.append(("finish", i)),
                    depth)
    return ev


def test_one_step_in_flight_is_serial():
    assert _trace(3, 1) == [("launch", 0), ("finish", 0), ("launch", 1), ("finish", 1),
                            ("launch", 2), ("finish", 2)]


def test_two_steps_in_flight():
    assert _trace(3, 2) == [("launch", 0), ("launch", 1), ("finish", 0), ("launch", 2),
                            ("finish", 1), ("finish", 2)]


@pytest.mark.parametrize("n", [0, 1, 2, 7])
@pytest.mark.parametrize("depth", [1, 2, 3])
def test_every_step_launched_and_finished_once_in_order(n, depth):
    ev = _trace(n, depth)
    assert [i for k, i in ev if k == "launch"] == list(range(n))
    assert [i for k, i in ev if k == "finish"] == list(range(n))
    live = set()
    for k, i in ev:
        if k == "launch":
            live.add(i)
            assert len(live) <= depth          # never more than depth steps in flight
        else:
            assert i in live                   # finished only after its launch
            live.remove(i)
    assert not live
