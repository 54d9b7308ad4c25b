"""Host-side logic of the NVLS all-reduce (no GPU): the multicast / flag addresses handed to
the consumer kernel, parity alternation per collective, and the producer slots."""
import torch

from air_rs.parallel import nvls
from air_rs.parallel.nvls import NvlsComm


class _Handle:
    def __init__(self, mc, peers):
        self.multicast_ptr = mc
        self.buffer_ptrs = peers


class _Ext:
    def __init__(self):
        self.calls = []

    def tp_reduce_norm_nvls(self, meta, *args):
        self.calls.append(meta.clone())


def _comm(world=4, rank=1, rows=8, hidden=64):
    buf = torch.zeros(NvlsComm.buffer_bytes(rows, hidden, world), dtype=torch.uint8)
    peers = [0x10000000 * (r + 1) for r in range(world)]
    peers[rank] = buf.data_ptr()
    h = _Handle(0x70000000, peers)
    return NvlsComm(buf, h, rank, world, "cpu", rows, hidden, timeout_s=1.5), buf, h


def test_buffer_layout_and_metas():
    world, rank, rows, hidden = 4, 1, 8, 64
    c, buf, h = _comm(world, rank, rows, hidden)
    slot = rows * hidden * 4
    assert NvlsComm.buffer_bytes(rows, hidden, world) == 2 * slot + 2 * rows * world * 4
    # producer slots: the two parities' partial regions of this rank's copy, [rows, hidden] f32
    assert c.slots[0].data_ptr() == buf.data_ptr() and c.slots[1].data_ptr() == buf.data_ptr() + slot
    assert c.slots[0].shape == (rows, hidden) and c.slots[0].dtype == torch.float32
    for p in range(2):
        m = c.metas[p].tolist()
        assert m[0] == 0x70000000 + p * slot                       # multicast partial region
        foff = 2 * slot + p * rows * world * 4
        assert m[1] == buf.data_ptr() + foff                         # local flags
        assert m[2:2 + world] == [b + foff for b in h.buffer_ptrs]   # every rank's flags
        assert m[2 + world:10] == [0] * (8 - world)
        assert m[13:17] == [world, rank, int(1.5e9), rows * hidden]


def test_parity_alternates_per_collective(monkeypatch):
    c, _, _ = _comm()
    ext = _Ext()
    monkeypatch.setattr(nvls.ops, "require_ext", lambda: ext)
    monkeypatch.setattr(nvls.ops, "count_launch", lambda n=1: None)
    x = torch.zeros(2, 64)
    c.pending = True
    assert c._slot(2).data_ptr() == c.slots[0].data_ptr()
    for i in range(4):
        c.reduce_norm(x, None, 1e-5, B=2)
        assert not c.pending
        assert c._slot(2).data_ptr() == c.slots[(i + 1) % 2].data_ptr()
    assert [int(m[0]) for m in ext.calls] == [int(c.metas[i % 2][0]) for i in range(4)]


def test_fits_and_two_shot():
    c, _, _ = _comm(rows=8, hidden=64)
    assert c.fits(8, 64) and not c.fits(9, 64) and not c.fits(4, 128)
    assert not c.two_shot(64)
