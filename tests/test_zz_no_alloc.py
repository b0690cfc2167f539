"""exl3b200_moe_gather_noalloc: the gather for callers that cannot allocate device memory (an engine with a fixed
memory pool, a process under a strict device-memory budget). Its scratch is a fixed device array inside the
library instead of caller-provided memory.

Called through the C ABI, twice in a row, against the ordinary exl3b200_moe_gather on the same inputs: the
results must agree within the routed-expert tolerance the other GPU tests use (they run the same arithmetic, so
they agree to the bit), and the second call must not see the first call's leftovers. A request past the array's
limit is refused before anything is written. This file is named to be collected last."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from exl3b200 import cases as X  # noqa: E402
from exl3b200 import library_path  # noqa: E402

REL_TOL, COS_TOL = 1e-2, 0.9999
MAX_PAIRS = 1 << 18
RAD_E_SHAPE = -1          # the shape refusal status of include/rad_types.h
_I64, _VP = C.c_int64, C.c_void_p


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    L = C.CDLL(str(library_path()))
    L.exl3b200_moe_gather_noalloc.argtypes = [_VP, _I64, _VP, _I64, _VP, _I64, _I64, _I64, _VP, _VP]
    L.exl3b200_moe_gather.argtypes = [_VP, _I64, _VP, _I64, _VP, _I64, _I64, _I64, _VP, _VP, _VP]
    L.exl3b200_moe_gather_work_bytes.restype = _I64
    L.exl3b200_moe_gather_work_bytes.argtypes = [_I64, _I64]
    return L


def _inputs(seed, T, k, E, width):
    rng = np.random.default_rng(seed)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    ids[rng.random(ids.shape) < 0.1] = -1
    st, _ = X.stable_scatter(ids, E)
    rows = X.bf16_bits(rng.standard_normal((T * k, width)).astype(np.float32))
    w = rng.random((T, k)).astype(np.float32)
    dev = torch.device("cuda:0")
    return (torch.from_numpy(rows.view(np.int16)).to(dev), torch.from_numpy(st).to(dev),
            torch.from_numpy(w).to(dev))


def _close(a, b):
    a64, b64 = a.astype(np.float64), b.astype(np.float64)
    scale = np.abs(b64).max()
    rel = np.abs(a64 - b64).max() / scale
    cos = (a64 * b64).sum() / (np.linalg.norm(a64) * np.linalg.norm(b64))
    return rel <= REL_TOL and cos >= COS_TOL


@pytest.mark.parametrize("T,k,E,width", [(37, 4, 16, 256), (2048, 10, 512, 2048)])
def test_noalloc_gather_matches_the_gather_twice(lib, T, k, E, width):
    rows, st, w = _inputs(T + width, T, k, E, width)
    y_ref = torch.empty((T, width), dtype=torch.float32, device="cuda")
    work = torch.empty(lib.exl3b200_moe_gather_work_bytes(T, k), dtype=torch.uint8, device="cuda")
    assert lib.exl3b200_moe_gather(rows.data_ptr(), width, st.data_ptr(), T * k, w.data_ptr(), T, k, width,
                                   y_ref.data_ptr(), work.data_ptr(), None) == 0
    outs = []
    for _ in range(2):
        y = torch.full((T, width), float("nan"), dtype=torch.float32, device="cuda")
        assert lib.exl3b200_moe_gather_noalloc(rows.data_ptr(), width, st.data_ptr(), T * k, w.data_ptr(), T, k,
                                               width, y.data_ptr(), None) == 0
        torch.cuda.synchronize()
        outs.append(y.cpu().numpy())
    want = y_ref.cpu().numpy()
    for got in outs:
        assert not np.isnan(got).any()
        assert _close(got, want)
        assert np.array_equal(got, want)


def test_noalloc_gather_after_a_larger_call_sees_no_leftovers(lib):
    # a large call fills more of the fixed array than the small one that follows reads
    rows, st, w = _inputs(3, 1024, 8, 64, 128)
    y = torch.empty((1024, 128), dtype=torch.float32, device="cuda")
    assert lib.exl3b200_moe_gather_noalloc(rows.data_ptr(), 128, st.data_ptr(), 1024 * 8, w.data_ptr(), 1024, 8,
                                           128, y.data_ptr(), None) == 0
    rows2, st2, w2 = _inputs(4, 17, 8, 64, 128)
    y2 = torch.empty((17, 128), dtype=torch.float32, device="cuda")
    ref = torch.empty((17, 128), dtype=torch.float32, device="cuda")
    work = torch.empty(lib.exl3b200_moe_gather_work_bytes(17, 8), dtype=torch.uint8, device="cuda")
    assert lib.exl3b200_moe_gather(rows2.data_ptr(), 128, st2.data_ptr(), 17 * 8, w2.data_ptr(), 17, 8, 128,
                                   ref.data_ptr(), work.data_ptr(), None) == 0
    assert lib.exl3b200_moe_gather_noalloc(rows2.data_ptr(), 128, st2.data_ptr(), 17 * 8, w2.data_ptr(), 17, 8,
                                           128, y2.data_ptr(), None) == 0
    torch.cuda.synchronize()
    assert np.array_equal(y2.cpu().numpy(), ref.cpu().numpy())


def test_noalloc_gather_refuses_past_its_limit(lib):
    T, k = MAX_PAIRS // 4 + 1, 4
    y = torch.full((4, 8), 7.0, dtype=torch.float32, device="cuda")
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    rc = lib.exl3b200_moe_gather_noalloc(dummy.data_ptr(), 8, dummy.data_ptr(), 0, dummy.data_ptr(), T, k, 8,
                                         y.data_ptr(), None)
    torch.cuda.synchronize()
    assert rc == RAD_E_SHAPE
    assert (y.cpu().numpy() == 7.0).all()


@pytest.mark.parametrize("n_tok,top_k", [(1 << 40, 1 << 30), (1 << 62, 4), (3, (1 << 18) + 1), (1 << 33, 1 << 31)])
def test_noalloc_gather_refuses_sizes_whose_product_wraps(lib, n_tok, top_k):
    # n_tok * top_k of these would wrap around int64 (or pass the limit by one factor alone): the entry point must
    # refuse them with the shape status before it forms the product, and write nothing
    y = torch.full((4, 8), 7.0, dtype=torch.float32, device="cuda")
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    rc = lib.exl3b200_moe_gather_noalloc(dummy.data_ptr(), 8, dummy.data_ptr(), 0, dummy.data_ptr(), n_tok, top_k,
                                         8, y.data_ptr(), None)
    torch.cuda.synchronize()
    assert rc == RAD_E_SHAPE
    assert (y.cpu().numpy() == 7.0).all()
