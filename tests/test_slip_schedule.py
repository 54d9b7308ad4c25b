"""Layer-streaming slot schedule on CPU with fake CUDA streams / events: a slot is never
refilled while the layer in it is still in use (odd streamed-layer counts, resident layers)."""
import contextlib
import types

import pytest
import torch

from air_rs.stream import slip


class _Ev:
    def __init__(self, *a, **k):
        pass

    def record(self, *a):
        pass

    def synchronize(self):
        pass

    def elapsed_time(self, other):
        return 0.0


class _Stream:
    def __init__(self, *a, **k):
        pass

    def wait_event(self, ev):
        pass


@pytest.fixture
def fake_cuda(monkeypatch):
    fake = types.SimpleNamespace(Stream=_Stream, Event=_Ev, stream=lambda s: contextlib.nullcontext(),
                                 current_stream=lambda d=None: _Stream())
    monkeypatch.setattr(slip.torch, "cuda", fake)
    yield


def _layers(n):
    # a layer is one tensor holding its index; copies are synchronous on CPU
    L = []
    for i in range(n):
        lw = types.SimpleNamespace(w=torch.full((4,), float(i)))
        L.append(lw)
    return L


@pytest.mark.parametrize("n_layers,resident,slots", [(6, (), 2), (5, (), 2), (6, (0, 1, 2), 2), (7, (2,), 3),
                                                     (4, (0,), 2)])
def test_slots_never_overwritten_in_use(fake_cuda, monkeypatch, n_layers, resident, slots):
    monkeypatch.setattr(slip, "layer_tensors", lambda lw: [lw.w])
    monkeypatch.setattr(slip, "_device_clone", lambda lw, dev: types.SimpleNamespace(w=lw.w.clone()))
    st = slip.LayerStreamer(_layers(n_layers), "cpu", n_slots=slots, timing=False, resident=resident)
    for step in range(3):
        for li in range(n_layers):
            lw = st.get(li)
            # whatever prefetches happened inside get, the weights handed out are layer li's
            assert float(lw.w[0]) == li, (step, li)
            st.release(li)
    assert sorted(st.resident) == sorted(resident)
