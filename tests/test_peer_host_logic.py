"""PeerGroup's host arithmetic on the CPU: which ranks' buffers each call
names, the receive-slot addresses of the GEMM scatter, and when the scatter
applies. A fake kernel module records the calls; nothing reaches a device.
(No reference counterpart: the reference has no tensor parallelism.)"""

import pytest
import torch

from optimized.peer import PeerGroup

ROWS, D = 1024, 256


class _FakeKernels:
    def __init__(self):
        self.calls = []

    def allreduce_ln(self, *args, **kwargs):
        self.calls.append(("allreduce_ln", args, kwargs))

    def linear_peer(self, *args):
        self.calls.append(("linear_peer", args, {}))


def _group(world, rank, push=True):
    g = object.__new__(PeerGroup)
    g.k = _FakeKernels()
    g.world, g.rank, g.rows, g.d = world, rank, ROWS, D
    g.push, g.timeout_ms, g.blocks = push, 2000, 296
    g.signal_bytes = 296 * 17 * 4
    g.poisoned = False
    g.status = torch.zeros(1, dtype=torch.int32)
    g.device = torch.device("cpu")
    # distinct fake addresses per (buffer, rank), as rank `rank` maps them
    names = ("part", "recv", "xa", "xb", "n16", "out", "signal")
    g.ptrs = {n: [(i + 1) << 40 | (r + 1) << 32 for r in range(world)] for i, n in enumerate(names)}
    g._own = {n: g.ptrs[n][rank] for n in names}
    g._opened = []
    return g


def _ln_args():
    x = torch.zeros(ROWS, D)
    w, b = torch.ones(D), torch.zeros(D)
    return x, w, b


@pytest.mark.parametrize("world,rank", [(2, 0), (2, 1), (4, 3), (8, 5)])
def test_scatter_slots_are_this_ranks_slot_in_every_owner(world, rank):
    g = _group(world, rank)
    rows = ROWS
    a16 = torch.zeros(rows, 64, dtype=torch.float16)
    w16 = torch.zeros(D, 64, dtype=torch.float16)
    g.gemm_to_owners(a16, w16, rows)
    (_, args, _), = g.k.calls
    outs, per, ldo = args[3], args[4], args[5]
    assert per == rows // world and ldo == D
    slot = rank * per * D * 4
    assert outs == [g.ptrs["recv"][r] + slot for r in range(world)]


@pytest.mark.parametrize("world,rank", [(2, 1), (4, 2), (8, 7)])
def test_reduction_from_owners_reads_every_slot_of_its_own_recv(world, rank):
    g = _group(world, rank)
    x, w, b = _ln_args()
    g.allreduce_ln(x, None, w, b, 1e-5, "xa", "n16", ROWS, from_owners=True)
    (_, args, kw), = g.k.calls
    parts = args[2]
    per = ROWS // world
    base = g.ptrs["recv"][rank]
    assert parts == [base + s * per * D * 4 for s in range(world)]
    assert kw["parts_local"] is True
    # push: every rank's outputs are named
    assert args[4] == g.ptrs["xa"] and args[5] == g.ptrs["n16"] and args[6] is True


def test_one_shot_names_only_its_own_outputs():
    g = _group(4, 2, push=False)
    x, w, b = _ln_args()
    g.allreduce_ln(x, None, w, b, 1e-5, None, "out", ROWS)
    (_, args, kw), = g.k.calls
    assert args[2] == g.ptrs["part"]
    assert args[4] is None
    assert args[5] == [None, None, g.ptrs["out"][2], None]
    assert args[6] is False and args[7] is False
    assert kw["parts_local"] is False


def test_reduction_refuses_in_place_and_oversize():
    g = _group(2, 0)
    x, w, b = _ln_args()
    with pytest.raises(ValueError, match="exceed"):
        g.allreduce_ln(x, None, w, b, 1e-5, "xa", "n16", ROWS + 1)
    fake_x = type("T", (), {"data_ptr": lambda self: g._own["xa"]})()
    with pytest.raises(ValueError, match="must not be the buffer"):
        g.allreduce_ln(fake_x, None, w, b, 1e-5, "xa", "n16", ROWS)
    assert not g.k.calls


@pytest.mark.parametrize("world,rows,push,ok", [
    (2, 1024, True, True), (2, 256, True, True), (2, 128, True, False),   # 64-row shares straddle
    (4, 512, True, True), (4, 768, True, False), (8, 1024, True, True),
    (2, 1024, False, False),                                               # one-shot never scatters
    (2, 2048, True, False),                                                # more rows than the buffers
])
def test_scatter_ok(world, rows, push, ok):
    assert _group(world, 0, push).scatter_ok(rows) is ok


def test_timed_out_call_poisons_the_group():
    """A call whose wait ran out (the kernel stored the timeout bit into the
    status word) makes check() raise, and the group refuses further calls."""
    from optimized.peer import PeerTimeoutError

    g = _group(2, 0)
    x, w, b = _ln_args()
    g.allreduce_ln(x, None, w, b, 1e-5, "xa", "n16", ROWS)
    (_, args, kwargs), = g.k.calls
    assert kwargs["status"] == g.status.data_ptr() and kwargs["signal_bytes"] == g.signal_bytes
    g.check()                                   # nothing timed out yet
    g.status[0] = 4                             # what the kernel stores on a timeout
    assert g.failed()
    with pytest.raises(PeerTimeoutError):
        g.check()
    assert g.poisoned
    with pytest.raises(PeerTimeoutError):
        g.allreduce_ln(x, None, w, b, 1e-5, "xa", "n16", ROWS)
    assert len(g.k.calls) == 1                  # nothing more was launched
