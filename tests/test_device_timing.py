"""Device-time histogram of the device communicator, with stand-in events (no GPU)."""
from nexar_b200.device.comm import DeviceTimeHistogram


class FakeEvent:
    def __init__(self, t_ms, done=True):
        self.t, self.done = t_ms, done

    def query(self):
        return self.done

    def elapsed_time(self, end):
        return end.t - self.t


def test_histogram_buckets_and_pending():
    h = DeviceTimeHistogram()
    h.record("all_reduce", FakeEvent(0.0), FakeEvent(0.005))      # 5 us
    h.record("all_reduce", FakeEvent(1.0), FakeEvent(1.2))        # 200 us
    h.record("all_reduce", FakeEvent(2.0), FakeEvent(22.0))       # 20 ms
    h.record("broadcast", FakeEvent(0.0), FakeEvent(0.05, done=False))
    s = h.summary()
    ar = s["all_reduce"]
    assert ar["count"] == 3 and abs(ar["min_us"] - 5) < 1e-6 and abs(ar["max_us"] - 20000) < 1e-3
    assert ar["buckets"] == [1, 0, 0, 1, 0, 0, 0, 1]
    assert abs(ar["mean_us"] - (5 + 200 + 20000) / 3) < 1e-3
    assert "broadcast" not in s and len(h.pending) == 1  # not finished yet: kept for later
    h.pending[0][2].done = True
    assert h.summary()["broadcast"]["count"] == 1 and not h.pending
