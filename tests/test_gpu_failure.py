"""The failure path of the kernels that wait on another rank, exercised on one GPU without faulting or hanging it.

Each peer-memory step waits on a flag another rank raises (the expert-parallel dispatch and combine, the width
split's reduce and pull), and gives up after a bounded time with a status word and the device error word set. Here
the flag is one that nothing raises: its epoch word is ahead of every flag in a zeroed window, so the wait can only
run out. With the limit set to 10 ms (exl3b200_set_peer_wait_ns) each kernel must return promptly, report -1 in its
status, set bit 8 of the error word, and leave the context usable -- a decode right after is still bit-exact.

A positive control runs the same waits with the epoch at 0 (every flag already there): status 0, no error."""
import ctypes as C
import time

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle_bind import Oracle  # noqa: E402
from exl3b200 import library_path  # noqa: E402
from exl3b200.native import Native  # noqa: E402

_I64, _VP = C.c_int64, C.c_void_p
LIMIT_NS = 10_000_000          # 10 ms
WAIT_ERR = 8                   # the error word's bit for a peer wait that gave up


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    L = C.CDLL(str(library_path()))
    L.exl3b200_set_peer_wait_ns.argtypes = [_I64]
    L.exl3b200_p2p_wait_dispatch.argtypes = [_VP, _VP, _I64, _VP, _VP, _VP]
    L.exl3b200_p2p_wait_combine.argtypes = [_VP, _VP, _I64, _VP, _VP, _VP]
    L.exl3b200_tp_reduce.argtypes = [_VP, _VP, _I64, _I64, _I64, _I64, _I64, _VP, _VP]
    L.exl3b200_tp_pull.argtypes = [_VP, _VP, _I64, _I64, _I64, _I64, _I64, _VP, _I64, _VP, _VP, _VP]
    L.exl3b200_read_error.argtypes = [C.c_int, C.POINTER(C.c_int32)]
    yield L
    L.exl3b200_set_peer_wait_ns(0)      # back to the default for whatever runs next in this process


def _error_word(L):
    v = C.c_int32(0)
    assert L.exl3b200_read_error(1, C.byref(v)) == 0
    return v.value


class _Window:
    """A zeroed one-rank window: the p2p layout offs[6] = {rows, meta, yback, ctl, done, sink} and the width split's
    offs[4] = {part, red, ctl, done}, every flag at 0."""

    def __init__(self, hidden=64, t_cap=4):
        self.hidden, self.t_cap = hidden, t_cap
        part = t_cap * hidden * 4
        self.buf = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
        base = 0
        self.p2p_offs = torch.tensor([base, base + 4096, base + 8192, base + 12288, base + 12544, base + 12800],
                                     dtype=torch.int64)
        self.tp_offs = torch.tensor([16384, 16384 + part, 16384 + 2 * part, 16384 + 2 * part + 256],
                                    dtype=torch.int64)
        self.peers = torch.tensor([self.buf.data_ptr()], dtype=torch.int64, device="cuda")


def _epoch(v):
    return torch.tensor([v], dtype=torch.int32, device="cuda")


def test_a_flag_nothing_raises_times_out_and_reports(lib):
    w = _Window()
    assert lib.exl3b200_set_peer_wait_ns(LIMIT_NS) == 0
    _error_word(lib)                                   # start from a clear error word
    epoch = _epoch(1)                                  # every flag in the window is 0: behind this epoch
    hdr = torch.full((4,), 77, dtype=torch.int32, device="cuda")
    status = torch.full((1,), 77, dtype=torch.int32, device="cuda")
    out = torch.zeros((w.t_cap, w.hidden), dtype=torch.float32, device="cuda")
    pull_status = torch.full((1,), 77, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    assert lib.exl3b200_p2p_wait_dispatch(w.buf.data_ptr(), w.p2p_offs.data_ptr(), 1, epoch.data_ptr(),
                                          hdr.data_ptr(), None) == 0
    assert lib.exl3b200_p2p_wait_combine(w.buf.data_ptr(), w.p2p_offs.data_ptr(), 1, epoch.data_ptr(),
                                         status.data_ptr(), None) == 0
    assert lib.exl3b200_tp_reduce(w.peers.data_ptr(), w.tp_offs.data_ptr(), 0, 1, w.t_cap, w.hidden, w.t_cap,
                                  epoch.data_ptr(), None) == 0
    assert lib.exl3b200_tp_pull(w.peers.data_ptr(), w.tp_offs.data_ptr(), 0, 1, w.t_cap, w.hidden, w.t_cap,
                                out.data_ptr(), w.hidden, epoch.data_ptr(), pull_status.data_ptr(), None) == 0
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    # four waits of 10 ms each (the pull's waits run in every block at once): well under a second, nowhere near
    # the 5 s default -- the limit reached the kernels
    assert elapsed < 1.0, f"the waits took {elapsed:.3f} s"
    h = hdr.cpu().numpy()
    assert h[3] == -1 and (h[:3] == 0).all(), h          # dispatch: gave up, no counts handed on
    assert status.item() == -1                            # combine
    assert pull_status.item() == -1                       # pull
    assert (out.cpu().numpy() == 0).all()                 # the pull wrote nothing after giving up
    assert _error_word(lib) & WAIT_ERR


def test_the_same_waits_pass_when_the_flags_are_there(lib):
    w = _Window()
    assert lib.exl3b200_set_peer_wait_ns(LIMIT_NS) == 0
    _error_word(lib)
    epoch = _epoch(0)                                  # flags at 0 are at this epoch: nothing to wait for
    hdr = torch.full((4,), 77, dtype=torch.int32, device="cuda")
    status = torch.full((1,), 77, dtype=torch.int32, device="cuda")
    assert lib.exl3b200_p2p_wait_dispatch(w.buf.data_ptr(), w.p2p_offs.data_ptr(), 1, epoch.data_ptr(),
                                          hdr.data_ptr(), None) == 0
    assert lib.exl3b200_p2p_wait_combine(w.buf.data_ptr(), w.p2p_offs.data_ptr(), 1, epoch.data_ptr(),
                                         status.data_ptr(), None) == 0
    torch.cuda.synchronize()
    assert hdr[3].item() == 0 and status.item() == 0
    assert _error_word(lib) == 0


def test_the_context_is_usable_after_a_wait_gave_up(lib):
    w = _Window()
    assert lib.exl3b200_set_peer_wait_ns(LIMIT_NS) == 0
    status = torch.full((1,), 77, dtype=torch.int32, device="cuda")
    assert lib.exl3b200_p2p_wait_combine(w.buf.data_ptr(), w.p2p_offs.data_ptr(), 1, _epoch(5).data_ptr(),
                                         status.data_ptr(), None) == 0
    torch.cuda.synchronize()
    assert status.item() == -1
    _error_word(lib)
    assert lib.exl3b200_set_peer_wait_ns(0) == 0
    # a decode on the same context, bit-exact against the oracle
    rng = np.random.default_rng(3)
    rows, cols, bits = 64, 128, 4
    rec = rng.integers(0, 1 << 16, size=rows * cols * bits // 16, dtype=np.uint64).astype(np.uint16)
    out = torch.zeros(rows * cols, dtype=torch.int16, device="cuda")
    Native().decode_what(torch.from_numpy(rec.view(np.int16)).cuda().data_ptr(), rows, cols, bits, 2, out.data_ptr())
    torch.cuda.synchronize()
    want = Oracle().record_decode(rec, rows, cols, bits, "mul1")
    assert np.array_equal(out.cpu().numpy().view(np.uint16).reshape(rows, cols), want)


def test_the_limit_setter_refuses_an_absurd_value(lib):
    assert lib.exl3b200_set_peer_wait_ns(601 * 1_000_000_000) != 0
    assert lib.exl3b200_set_peer_wait_ns(-1) == 0          # <= 0: the default again
