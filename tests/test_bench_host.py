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


@pytest.mark.parametrize("depth", [1, 2])
def test_e2e_leg_runs_on_a_cpu_pool(monkeypatch, depth):
    """bench.run_e2e's loop end to end on a small CPU pool: the CUDA stream / event calls
    are stubbed and attend returns zeros (no kernel runs), so this covers the leg's host
    flow -- copies, begin_forward / end_forward order, one output per step, byte counts
    -- with one and two steps in flight."""
    import time
    import torch
    from nanoslg_b200 import kv_cache

    class _Event:
        def __init__(self, enable_timing=False):
            self.t = None

        def record(self, stream=None):
            self.t = time.perf_counter()

        def synchronize(self):
            pass

        def elapsed_time(self, other):
            return (other.t - self.t) * 1e3

    seen = []

    def attend(self, layer, q, k, v, hq, hkv):
        seen.append(list(self.start_positions))
        return torch.zeros(q.shape[0], 1, hq * q.shape[-1], dtype=q.dtype)

    monkeypatch.setattr(torch.cuda, "Event", _Event)
    monkeypatch.setattr(torch.cuda, "current_stream", lambda device=None: None)
    monkeypatch.setattr(torch.cuda, "synchronize", lambda device=None: None)
    monkeypatch.setattr(torch.Tensor, "pin_memory", lambda self: self)
    monkeypatch.setattr(kv_cache.B200CacheContext, "attend", attend)
    monkeypatch.setattr(bench, "D", 16)
    monkeypatch.setattr(bench, "POOL_PAGES", 40000)
    r = bench.run_e2e(torch.device("cpu"), steps=4, warmup=3, seed=0, depth=depth)
    assert len(seen) == 7
    lens = bench.c2_lens(0)
    assert seen[0] == lens and seen[-1] == [n + 6 for n in lens]   # one token per step
    assert r["total_ms"] > 0
    assert r["d2h"] == bench.B * bench.HQ * 16 * 2
    assert r["h2d"] >= bench.B * (bench.HQ + 2 * bench.HKV) * 16 * 2
