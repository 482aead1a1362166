"""Host-side logic of spanqr_b200.core that runs without a GPU."""
import threading

import torch

from spanqr_b200 import core


def test_graph_cache_takes_its_lock_without_deadlock(monkeypatch):
    """building a graph entry (which needs the dust, whose cache shares the lock) must not wait on itself"""
    made = []

    def fake_zdust(K, r, dev):
        with core._lock:
            return torch.zeros(1)

    class FakeGraph:
        def __init__(self, dev, stream, K, r, Z):
            with core._lock:
                made.append((K, r))

    class FakeStream:
        cuda_stream = 7

    monkeypatch.setattr(core, "zdust", fake_zdust)
    monkeypatch.setattr(core, "_Graph", FakeGraph)
    monkeypatch.setattr(core, "_GRAPHS", {})
    done = []
    t = threading.Thread(target=lambda: done.append(core._graph("cpu", FakeStream(), 64, 32)), daemon=True)
    t.start()
    t.join(timeout=10)
    assert done and made == [(64, 32)]
    assert core._graph("cpu", FakeStream(), 64, 32) is done[0]   # cached: built once


def test_dispatch_rejects_cpu_tensors_loudly():
    """the padded (r % 32 != 0) and block (r > 512) branches of orth, like the main path, refuse CPU tensors: there is
    no CPU path"""
    import pytest
    from spanqr_b200 import orth
    for shape in [(100, 48), (2048, 768), (100, 64)]:
        with pytest.raises(TypeError):
            orth(torch.zeros(shape))
