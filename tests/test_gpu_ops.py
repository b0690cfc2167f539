"""The B200 library on a GPU, through its C ABI, against the oracle.

- the decode: bit-exact with the restatement (itself pinned to the reference and the vllm-exl3 golden) for every K
  1..8 and every codebook, on enough tiles to meet nearly every 16-bit state;
- every op through the plugin rows (layout hooks, redzones, NaN-prefilled outputs) against the reference library
  built from the reference sources, within the stated tolerance: max |got - want| / max |want| <= 1e-2 and cosine
  >= 0.9999, rows the reference leaves zero exactly zero;
- the chain identities inside this library, to the bit: gate_up(h_rot 1) -> down(h_rot 1) equals the h_rot 0
  pair; prep_gu -> gate_up(a_rot 1) equals gate_up(a_rot 0); gate_up_down equals its pair;
- the routing kernels: router top-k against numpy, the scatter to the bit against the stable contract, the gather
  against the restatement."""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle_bind import REF_SO, Oracle, compare  # noqa: E402
from exl3b200 import cases as X  # noqa: E402
from exl3b200 import load_plugin  # noqa: E402
from exl3b200.native import Native  # noqa: E402
from exl3b200.rad import Plugin  # noqa: E402

REL_TOL, COS_TOL = 1e-2, 0.9999


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(scope="module")
def plugin(dev):
    return load_plugin()


@pytest.fixture(scope="module")
def native(dev):
    return Native()


@pytest.fixture(scope="module")
def orc():
    return Oracle()


@pytest.fixture(scope="module")
def ref_plugin():
    if not REF_SO.exists():
        pytest.skip("oracle/_ref/libexl3ref.so not present")
    return Plugin(REF_SO)


@pytest.mark.parametrize("bits", range(1, 9))
@pytest.mark.parametrize("cb", ["3inst", "mcg", "mul1"])
def test_decode_is_bit_exact(dev, native, orc, bits, cb):
    rng = np.random.default_rng(1000 + 10 * bits + len(cb))
    rows, cols = (1024, 2048) if bits == 8 else (256, 512)
    rec = rng.integers(0, 1 << 16, size=rows * cols * bits // 16, dtype=np.uint64).astype(np.uint16)
    want = orc.record_decode(rec, rows, cols, bits, cb)
    rec_d = torch.from_numpy(rec.view(np.int16)).to(dev)
    out = torch.zeros(rows * cols, dtype=torch.int16, device=dev)
    native.decode_what(rec_d.data_ptr(), rows, cols, bits, {"3inst": 0, "mcg": 1, "mul1": 2}[cb], out.data_ptr())
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint16).reshape(rows, cols)
    assert np.array_equal(got, want), f"{(got != want).sum()} of {got.size} values differ"


def test_device_relayout_equals_oracle(orc, native):
    rng = np.random.default_rng(5)
    for bits in range(1, 9):
        sym = rng.integers(0, 1 << bits, size=(48, 256), dtype=np.uint32)
        codes = X.pack_codes(sym, bits)
        rec = np.zeros(48 * 256 * bits // 16, np.uint16)
        native.codes_to_record(codes.ctypes.data, codes.shape[1], 48, 256, bits, rec.ctypes.data)
        assert np.array_equal(rec, orc.codes_to_record(codes, 48, 256, bits))
        back = np.zeros_like(codes)
        native.record_to_codes(rec.ctypes.data, 48, 256, bits, back.ctypes.data, codes.shape[1])
        assert np.array_equal(back, codes)


# ---------------------------------------------------------------------------------------------- ops
OPS = [
    dict(op="moe_exl3_down", M=4, top_k=2, n_expert=5, geom=[(256, 128)], bits=4, codebook="mul1", drop=0.2),
    dict(op="moe_exl3_down", M=3, top_k=2, n_expert=4, geom=[(256, 256), (128, 128)], bits=3, codebook="mcg",
         n_protect=1, pitch_extra=8),
    dict(op="moe_exl3_down", M=16, top_k=1, n_expert=1, geom=[(512, 2048)], bits=4, codebook="mul1"),   # config 1
    dict(op="moe_exl3_gate_up", M=4, top_k=2, n_expert=5, geom=[(256, 256)], bits=4, codebook="mul1", drop=0.2),
    dict(op="moe_exl3_gate_up", M=3, top_k=2, n_expert=4, geom=[(512, 128), (256, 256)], bits=2, codebook="3inst",
         h_rot=1, x_dtype="bf16"),
    dict(op="moe_exl3_gate_up", M=4, top_k=2, n_expert=4, geom=[(256, 128)], bits=5, codebook="mcg", a_rot=1),
    dict(op="moe_exl3_gate_up", M=40, top_k=2, n_expert=3, geom=[(256, 256)], bits=3, codebook="mul1"),  # > 64 rows
    dict(op="moe_exl3_gate_up", M=8, top_k=1, n_expert=1, geom=[(1024, 2048)], bits=4, codebook="mul1"),  # config 2
    dict(op="moe_exl3_prep_gu", M=4, top_k=2, n_expert=3, geom=[(256, 256), (256, 128)], bits=4, drop=0.25),
    dict(op="moe_exl3_gate_up_down", M=3, top_k=2, n_expert=4, geom=[(256, 128)], bits=4, codebook="mul1"),
    dict(op="moe_exl3_gate_up_down", M=32, top_k=1, n_expert=1, geom=[(1024, 2048)], bits=4, codebook="mul1"),
    dict(op="moe_exl3_down_mod4", M=4, top_k=2, n_expert=6, geom=[(128, 128), (256, 128), (128, 256), (128, 128)],
         bits=6, codebook="mul1"),
    dict(op="moe_exl3_gate_up_mod4", M=4, top_k=2, n_expert=6,
         geom=[(256, 128), (512, 128), (256, 256), (256, 128)], bits=7, codebook="mcg", h_rot=1),
    dict(op="moe_exl3_down", M=2, top_k=2, n_expert=3, geom=[(256, 128)], bits=8, codebook="3inst"),
    # the decode band at the config's shapes (fewer than 64 units: live experts x 256-row output pairs)
    dict(op="moe_exl3_gate_up", M=1, top_k=10, n_expert=64, geom=[(1024, 2048)], bits=3, codebook="mul1"),
    dict(op="moe_exl3_down", M=1, top_k=4, n_expert=64, geom=[(2048, 512)], bits=4, codebook="mul1", h_rot=1),
    # the tensor-core band (at least 64 units: 64-row groups x 256-row output pairs; or 8 of them while the live experts
    # average >= 16 rows)
    dict(op="moe_exl3_down", M=8, top_k=10, n_expert=64, geom=[(2048, 512)], bits=4, codebook="mul1",
         table_form="stacked"),
    dict(op="moe_exl3_gate_up", M=8, top_k=10, n_expert=64, geom=[(1024, 2048)], bits=3, codebook="mul1"),
    dict(op="moe_exl3_down", M=100, top_k=2, n_expert=4, geom=[(512, 256)], bits=4, codebook="mul1", h_rot=1),
    dict(op="moe_exl3_gate_up", M=64, top_k=2, n_expert=4, geom=[(512, 256), (256, 128)], bits=2, codebook="3inst",
         drop=0.1),
    dict(op="moe_exl3_gate_up", M=48, top_k=1, n_expert=2, geom=[(1024, 512)], bits=5, codebook="mcg", a_rot=1),
    dict(op="moe_exl3_down", M=70, top_k=1, n_expert=1, geom=[(1024, 128)], bits=8, codebook="mul1"),
    dict(op="moe_exl3_gate_up", M=33, top_k=2, n_expert=2, geom=[(1024, 256)], bits=6, codebook="mul1", h_rot=1,
         x_dtype="bf16"),
    dict(op="moe_exl3_gate_up", M=200, top_k=10, n_expert=64, geom=[(1024, 2048)], bits=3, codebook="mul1",
         h_rot=1),
    dict(op="moe_exl3_down", M=200, top_k=10, n_expert=64, geom=[(2048, 512)], bits=4, codebook="mul1", h_rot=1),
    dict(op="moe_exl3_down_mod4", M=64, top_k=2, n_expert=8, geom=[(256, 128), (512, 128), (256, 256), (256, 128)],
         bits=7, codebook="mcg"),
    # the four-class forms of the rotation op (to the bit) and of the whole chain (tests/ref/test_exl3ref.py:1168-1205
    # runs the same four rank-width classes): classes of different widths over one hidden size
    dict(op="moe_exl3_prep_gu_mod4", M=4, top_k=2, n_expert=6, geom=[(256, 256), (512, 256), (256, 128), (256, 256)],
         bits=4, drop=0.2),
    dict(op="moe_exl3_prep_gu_mod4", M=9, top_k=3, n_expert=8, geom=[(512, 256)], bits=3, x_dtype="bf16"),
    dict(op="moe_exl3_gate_up_down_mod4", M=4, top_k=2, n_expert=8, geom=[(256, 256), (512, 256), (256, 256),
                                                                         (512, 256)], bits=4, codebook="mul1"),
    dict(op="moe_exl3_gate_up_down_mod4", M=6, top_k=2, n_expert=6, geom=[(512, 256), (256, 256)], bits=3,
         codebook="mcg", drop=0.15),
    # config 2, the expert MLP at M = 1 and 4 through the fused op (M = 8 and 32 are above)
    dict(op="moe_exl3_gate_up_down", M=1, top_k=1, n_expert=1, geom=[(1024, 2048)], bits=4, codebook="mul1"),
    dict(op="moe_exl3_gate_up_down", M=4, top_k=1, n_expert=1, geom=[(1024, 2048)], bits=4, codebook="mul1"),
    dict(op="moe_exl3_gate_up_down", M=8, top_k=1, n_expert=1, geom=[(1024, 2048)], bits=4, codebook="mul1"),
    # the other two codebooks at the config geometry, both bands
    dict(op="moe_exl3_gate_up", M=8, top_k=10, n_expert=64, geom=[(1024, 2048)], bits=3, codebook="mcg", h_rot=1),
    dict(op="moe_exl3_down", M=8, top_k=10, n_expert=64, geom=[(2048, 512)], bits=4, codebook="3inst", h_rot=1),
    dict(op="moe_exl3_gate_up", M=1, top_k=10, n_expert=64, geom=[(1024, 2048)], bits=3, codebook="3inst"),
    dict(op="moe_exl3_down", M=1, top_k=10, n_expert=64, geom=[(2048, 512)], bits=4, codebook="mcg", h_rot=1),
] + [
    # config 4, the bitrate sweep's linear: out 4096 x in 1536 (and the transpose), K = 2..8, one expert, every row
    # routed to it (the decode band at batch 1, the tensor-core band at batch 32 / 256)
    dict(op="moe_exl3_down", M=M, top_k=1, n_expert=1, geom=[geom], bits=K, codebook="mul1")
    for K in range(2, 9) for M, geom in ((1, (4096, 1536)), (32, (4096, 1536)))
] + [
    dict(op="moe_exl3_down", M=1, top_k=1, n_expert=1, geom=[(1536, 4096)], bits=4, codebook="mul1"),
    dict(op="moe_exl3_down", M=256, top_k=1, n_expert=1, geom=[(1536, 4096)], bits=4, codebook="mul1"),
    dict(op="moe_exl3_down", M=256, top_k=1, n_expert=1, geom=[(4096, 1536)], bits=2, codebook="mul1"),
    dict(op="moe_exl3_down", M=256, top_k=1, n_expert=1, geom=[(4096, 1536)], bits=8, codebook="mul1"),
]


def _case(spec, seed=4321):
    spec = dict(spec)
    return X.Case(spec.pop("op"), seed, **spec)


def _want(case, orc, ref_plugin):
    """The reference library itself for small cases; the restatement (pinned to it bit for bit on the CPU, see
    tests/test_oracle.py) with threads for the large ones."""
    if case.n_expert <= 8 and case.x_cols * max(r for r, _ in case.geom) <= 1 << 20:
        r = case.run(ref_plugin, device=False)
        assert r["rc"] == 0
        return r["y"]
    prefill = np.full((case.T, case.y_cols), 0xFFFF, np.uint16)
    return orc.run_case(case, n_threads=os.cpu_count() or 4, prefill=prefill)


@pytest.mark.parametrize("spec", OPS, ids=lambda s: f"{s['op']}-M{s['M']}-K{s['bits']}-{s.get('codebook', '')}")
def test_op_matches_the_reference(dev, plugin, orc, ref_plugin, spec):
    case = _case(spec)
    got = case.run(plugin, device=True)
    assert got["rc"] == 0, got["rc"]
    assert got["redzone_ok"], "a write outside an operand"
    assert got["inputs_ok"], "an input changed"
    assert got["unrelayout_ok"], "the layout hooks do not round-trip"
    want = _want(case, orc, ref_plugin)
    if case.base == "moe_exl3_prep_gu":
        # prep_gu is the rotation alone: to the bit, including the rows it must not write
        assert np.array_equal(got["y"], want)
        return
    ok, detail = compare(got["y"], want, case.out_dtype(), REL_TOL, COS_TOL)
    assert ok, detail
    assert np.array_equal(got["y_pitch_tail"], np.full_like(got["y_pitch_tail"], 0xFFFF)), "wrote past the width"
    assert Native().read_error() == 0


def test_h_rot_pair_is_bit_identical(dev, plugin):
    base = dict(M=6, top_k=2, n_expert=5, geom=[(512, 256)], bits=4, codebook="mul1", drop=0.1)
    gu1 = X.Case("moe_exl3_gate_up", 77, h_rot=1, **base)
    gu0 = X.Case("moe_exl3_gate_up", 0, h_rot=0, planes=gu1.planes, x=gu1.x, sorted_tok=gu1.sorted_tok,
                 expert_offset=gu1.expert_offset, **{k: v for k, v in base.items() if k != "drop"})
    h0 = gu0.run(plugin, device=True)["y"]
    h1 = gu1.run(plugin, device=True)["y"]
    dgeom = [(256, 256)]
    dplanes = []
    for p in gu1.planes:
        rng = np.random.default_rng(len(dplanes))
        d = X.random_planes(rng, 256, 256, 4, False)
        d["suh"] = p["dn_suh"]
        dplanes.append(d)
    common = dict(M=6, top_k=2, n_expert=5, geom=dgeom, bits=4, codebook="mul1", planes=dplanes,
                  sorted_tok=gu1.sorted_tok, expert_offset=gu1.expert_offset)
    y0 = X.Case("moe_exl3_down", 0, h_rot=0, x=h0, **common).run(plugin, device=True)["y"]
    y1 = X.Case("moe_exl3_down", 0, h_rot=1, x=h1, **common).run(plugin, device=True)["y"]
    assert np.array_equal(y0, y1)
    assert not np.array_equal(h0, h1)     # control: the flag moves gate_up's output


def test_prep_then_a_rot_is_bit_identical(dev, plugin):
    base = dict(M=5, top_k=2, n_expert=4, geom=[(256, 256), (512, 128)], bits=3, codebook="mcg", drop=0.1)
    gu0 = X.Case("moe_exl3_gate_up", 91, **base)
    pg = X.Case("moe_exl3_prep_gu", 0, planes=gu0.planes, x=gu0.x, sorted_tok=gu0.sorted_tok,
                expert_offset=gu0.expert_offset, **{k: v for k, v in base.items() if k != "drop"})
    xr = pg.run(plugin, device=True)["y"]
    xr = np.where(xr == 0xFFFF, 0, xr).astype(np.uint16)     # rows prep_gu does not write: gate_up ignores them
    gu1 = X.Case("moe_exl3_gate_up", 0, a_rot=1, planes=gu0.planes, x=xr, sorted_tok=gu0.sorted_tok,
                 expert_offset=gu0.expert_offset, **{k: v for k, v in base.items() if k != "drop"})
    assert np.array_equal(gu0.run(plugin, device=True)["y"], gu1.run(plugin, device=True)["y"])


def test_gate_up_down_equals_its_pair(dev, plugin):
    gd = X.Case("moe_exl3_gate_up_down", 5, M=5, top_k=2, n_expert=4, geom=[(512, 256)], bits=4, codebook="mul1",
                drop=0.1)
    y = gd.run(plugin, device=True)["y"]
    gu = X.Case("moe_exl3_gate_up", 0, M=5, top_k=2, n_expert=4, geom=[(512, 256)], bits=4, codebook="mul1",
                h_rot=1, planes=gd.planes, x=gd.x, sorted_tok=gd.sorted_tok, expert_offset=gd.expert_offset)
    h = gu.run(plugin, device=True)["y"]
    dplanes = [{"codes": p["dn_codes"], "suh": p["dn_suh"], "svh": p["dn_svh"]} for p in gd.planes]
    dn = X.Case("moe_exl3_down", 0, M=5, top_k=2, n_expert=4, geom=[(256, 256)], bits=4, codebook="mul1", h_rot=1,
                planes=dplanes, x=h, sorted_tok=gd.sorted_tok, expert_offset=gd.expert_offset)
    assert np.array_equal(y, dn.run(plugin, device=True)["y"])


@pytest.mark.parametrize("op", ["moe_exl3_down", "moe_exl3_gate_up"])
def test_wide_units_equal_the_64_row_units(dev, plugin, op):
    """Passes of many rows an expert over a wide input run the tensor-core kernel's wide form (a unit of up to 128
    rows decodes its weights once for both 64-row halves). Its output equals, bit for bit, the same rows run as
    passes small enough for the 64-row units (each output row depends only on its input row and its expert; the
    64-row units are the ones the oracle tests pin): two experts, one slot a token, the sorted rows cut in two
    halves. The down case (a 1024-column input: down of a 1024-wide expert) takes the same path."""
    gate_up = op == "moe_exl3_gate_up"
    # the wide form needs >= 128 rows an expert, 4 units an SM of the pass and an input of >= 1024 columns
    M = 19200 if gate_up else 9600
    geom = [(1024, 2048)] if gate_up else [(2048, 1024)]
    full = X.Case(op, 123, M=M, top_k=1, n_expert=2, geom=geom, bits=3 if gate_up else 4, codebook="mul1", h_rot=1)
    y = full.run(plugin, device=True)["y"]
    off = full.expert_offset.astype(np.int64)
    half = M // 2
    for a, b in ((0, half), (half, M)):
        n = b - a
        x = full.x[full.sorted_tok[a:b]] if gate_up else full.x[a:b]
        part = X.Case(op, 0, M=n, top_k=1, n_expert=2, geom=geom, bits=full.bits, codebook="mul1", h_rot=1,
                      planes=full.planes, x=x, sorted_tok=np.arange(n, dtype=np.int32),
                      expert_offset=np.clip(off - a, 0, n).astype(np.int32))
        assert np.array_equal(y[a:b], part.run(plugin, device=True)["y"]), (op, a, b)
    assert Native().read_error() == 0


def test_refusals_write_nothing(dev, plugin):
    case = _case(OPS[0])
    case.bits = 9          # a dtype no row serves
    with pytest.raises(Exception):
        case.run(plugin, device=True)


# ---------------------------------------------------------------------------------------------- routing
@pytest.mark.parametrize("T,E,k", [(1, 512, 10), (64, 512, 10), (2048, 512, 10), (33, 100, 3)])
def test_router_and_scatter(dev, native, T, E, k):
    rng = np.random.default_rng(T + E)
    logits = rng.standard_normal((T, E)).astype(np.float32)
    lg = torch.from_numpy(logits).to(dev)
    ids = torch.empty((T, k), dtype=torch.int32, device=dev)
    w = torch.empty((T, k), dtype=torch.float32, device=dev)
    native.router_topk(lg.data_ptr(), T, E, k, ids.data_ptr(), w.data_ptr())
    torch.cuda.synchronize()
    want_ids = np.argsort(-logits, axis=1, kind="stable")[:, :k]
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    p = np.exp(logits.astype(np.float64) - logits.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    assert np.allclose(w.cpu().numpy(), np.take_along_axis(p, want_ids, 1), rtol=1e-5, atol=1e-7)
    # the stable counting sort, to the bit (with some slots dropped)
    idn = want_ids.astype(np.int32).copy()
    idn[rng.random(idn.shape) < 0.05] = -1
    st_want, off_want = X.stable_scatter(idn, E)
    ids_d = torch.from_numpy(idn).to(dev)
    st = torch.empty(T * k, dtype=torch.int32, device=dev)
    off = torch.empty(E + 1, dtype=torch.int32, device=dev)
    work = torch.empty(max(1, native.scatter_work_bytes(T * k, E)), dtype=torch.uint8, device=dev)
    native.moe_scatter(ids_d.data_ptr(), T * k, E, 0, st.data_ptr(), off.data_ptr(), work.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(off.cpu().numpy(), off_want)
    assert np.array_equal(st.cpu().numpy(), st_want)


@pytest.mark.parametrize("T,E,k", [(7, 512, 10), (300, 1024, 32), (5, 256, 8), (9, 2000, 4), (64, 40, 32)])
def test_router_ties_zeros_and_infinities(dev, native, T, E, k):
    """The top-k choice on ties (logits on a coarse grid), +0 and -0 (equal: the lower id first), -inf logits, and
    every register width (256 / 512 / 1024 experts) plus the generic kernel (2000): ids exactly numpy's stable
    argsort of -logits, weights the softmax."""
    rng = np.random.default_rng(T * E + k)
    logits = (np.round(rng.standard_normal((T, E)) * 2) / 2).astype(np.float32)
    logits[rng.random((T, E)) < 0.05] = 0.0
    logits[rng.random((T, E)) < 0.05] = -0.0
    logits[rng.random((T, E)) < 0.02] = -np.inf
    lg = torch.from_numpy(logits).to(dev)
    ids = torch.empty((T, k), dtype=torch.int32, device=dev)
    w = torch.empty((T, k), dtype=torch.float32, device=dev)
    native.router_topk(lg.data_ptr(), T, E, k, ids.data_ptr(), w.data_ptr())
    torch.cuda.synchronize()
    want_ids = np.argsort(-logits, axis=1, kind="stable")[:, :k]
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    p = np.exp(logits.astype(np.float64) - logits.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    assert np.allclose(w.cpu().numpy(), np.take_along_axis(p, want_ids, 1), rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("n_pairs,E,base,skew",[(8192, 512, 0, 0.0), (8193, 512, 0, 0.0), (5000, 64, 32, 0.5),
                                                 (163840, 64, 0, 0.0), (20000, 512, 0, 0.6), (50000, 2048, 100, 0.0),
                                                 (3000, 1024, 0, 0.9), (1, 512, 0, 0.0)])
def test_scatter_is_the_stable_sort(dev, native, n_pairs, E, base, skew):
    """The counting sort to the bit on both paths (one block up to 8192 pairs, chunked beyond), the table-based
    placement (up to 1024 experts) and the warp-by-warp one (more), skewed routing (most pairs on one expert),
    ids outside [base, base + E) and -1 dropped."""
    rng = np.random.default_rng(n_pairs + E)
    ids = rng.integers(base - 4, base + E + 4, size=n_pairs).astype(np.int32)
    hot = rng.random(n_pairs) < skew
    ids[hot] = base + 3
    ids[rng.random(n_pairs) < 0.03] = -1
    st_want, off_want = X.stable_scatter(ids, E, expert_base=base)
    ids_d = torch.from_numpy(ids).to(dev)
    st = torch.empty(n_pairs, dtype=torch.int32, device=dev)
    off = torch.empty(E + 1, dtype=torch.int32, device=dev)
    work = torch.empty(max(1, native.scatter_work_bytes(n_pairs, E)), dtype=torch.uint8, device=dev)
    for _ in range(2):     # twice: the same bits again
        native.moe_scatter(ids_d.data_ptr(), n_pairs, E, base, st.data_ptr(), off.data_ptr(), work.data_ptr())
        torch.cuda.synchronize()
        assert np.array_equal(off.cpu().numpy(), off_want)
        assert np.array_equal(st.cpu().numpy(), st_want)


@pytest.mark.parametrize("T,k,E,width", [(37, 4, 16, 256), (1, 10, 512, 2048), (500, 10, 64, 512),
                                         (1100, 4, 16, 256), (3, 33, 64, 256)])
def test_gather(dev, native, orc, T, k, E, width):
    """The gather against the restatement, to the bit: one launch (each token finds its rows) up to 4096 rows and 32
    slots, the inverse map and the gather beyond."""
    rng = np.random.default_rng(9 + T)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    ids[rng.random(ids.shape) < 0.1] = -1
    st, off = X.stable_scatter(ids, E)
    rows = X.bf16_bits(rng.standard_normal((T * k, width)).astype(np.float32))
    w = rng.random((T, k)).astype(np.float32)
    want = orc.gather(rows, st, w, T, k, width)
    r_d = torch.from_numpy(rows.view(np.int16)).to(dev)
    st_d = torch.from_numpy(st).to(dev)
    w_d = torch.from_numpy(w).to(dev)
    y = torch.empty((T, width), dtype=torch.float32, device=dev)
    work = torch.empty(native.gather_work_bytes(T, k), dtype=torch.uint8, device=dev)
    native.moe_gather(r_d.data_ptr(), width, st_d.data_ptr(), T * k, w_d.data_ptr(), T, k, width, y.data_ptr(),
                      work.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(y.cpu().numpy(), want)


@pytest.mark.parametrize("T,E,k,n_local,base", [(1, 512, 10, 512, 0), (8, 512, 10, 512, 0), (32, 256, 8, 64, 64),
                                                 (33, 512, 10, 512, 0), (5, 1024, 32, 1024, 0), (4, 2048, 6, 512, 0)])
def test_router_scatter_is_the_two_calls(dev, native, T, E, k, n_local, base):
    """The fused router + sort (one launch for up to 32 tokens) equals router_topk then moe_scatter, to the bit."""
    rng = np.random.default_rng(T * 7 + E)
    lg = torch.from_numpy(rng.standard_normal((T, E)).astype(np.float32)).to(dev)
    out = []
    for fused in (True, False):
        ids = torch.full((T, k), -7, dtype=torch.int32, device=dev)
        w = torch.zeros((T, k), dtype=torch.float32, device=dev)
        st = torch.full((T * k,), -7, dtype=torch.int32, device=dev)
        off = torch.full((n_local + 1,), -7, dtype=torch.int32, device=dev)
        work = torch.empty(max(16, native.scatter_work_bytes(T * k, n_local)), dtype=torch.uint8, device=dev)
        if fused:
            native.router_scatter(lg.data_ptr(), T, E, k, ids.data_ptr(), w.data_ptr(), n_local, base, st.data_ptr(),
                                  off.data_ptr(), work.data_ptr())
        else:
            native.router_topk(lg.data_ptr(), T, E, k, ids.data_ptr(), w.data_ptr())
            native.moe_scatter(ids.data_ptr(), T * k, n_local, base, st.data_ptr(), off.data_ptr(), work.data_ptr())
        torch.cuda.synchronize()
        out.append([t.cpu() for t in (ids, w, st, off)])
    for a, b in zip(*out):
        assert torch.equal(a, b)


# ---------------------------------------------------------------------------------------------- the EP forms of the ops
def _small_layer(plugin, T, seed=3, max_rows=None):
    from exl3b200.layer import MoeLayer
    lay = MoeLayer(plugin, n_expert=16, hidden=2048, width=512, top_k=4, bits_gu=3, bits_dn=4, max_tokens=T,
                   seed=seed, max_rows=max_rows)
    g = torch.Generator(device="cuda")
    g.manual_seed(seed + 1)
    lay.x.copy_(torch.randn(lay.x.shape, generator=g, device="cuda").to(torch.float16))
    lay.logits.copy_(torch.randn(lay.logits.shape, generator=g, device="cuda"))
    return lay


@pytest.mark.parametrize("T", [2, 64])
def test_down_rows_writes_through_the_row_table(dev, plugin, T):
    """exl3b200_moe_down_rows: row i of down's output lands at row_dst[i] -- here a permutation of a second buffer --
    bit for bit the row the plugin's down row writes at y + i * pitch."""
    import ctypes as C
    lay = _small_layer(plugin, T)
    s = torch.cuda.current_stream().cuda_stream
    lay.forward(T, s)
    R = T * lay.k
    _, a_dn, _ = lay._build(T, R)
    perm = torch.randperm(R, generator=torch.Generator().manual_seed(T)).to(dev)
    alt = torch.full((R, lay.H), 7, dtype=torch.int16, device=dev)
    row_dst = (alt.data_ptr() + perm.to(torch.int64) * lay.H * 2).contiguous()
    lay.native.moe_down_rows(C.addressof(a_dn), row_dst.data_ptr(), s)
    torch.cuda.synchronize()
    assert torch.equal(alt[perm], lay.y_rows[:R].view(torch.int16))


@pytest.mark.parametrize("T,pad", [(3, 3), (128, 96)])   # the padding keeps each op in the same band
def test_live_only_pass_leaves_padding_untouched(dev, plugin, T, pad):
    """exl3b200_moe_op_live over a capacity-sized pass (sorted_tok padded with -1, the live count in expert_offset):
    the live rows equal the plugin rows' result bit for bit, the padding rows keep what was there."""
    lay = _small_layer(plugin, T, max_rows=T * 4 + pad)
    s = torch.cuda.current_stream().cuda_stream
    R = T * lay.k
    lay.forward(T, s)
    torch.cuda.synchronize()
    h_ref, y_ref = lay.h[:R].clone(), lay.y_rows[:R].clone()
    lay.sorted_tok[R:R + pad] = -1
    lay.h[R:R + pad].view(torch.int16).fill_(0x1234)
    lay.y_rows[R:R + pad].view(torch.int16).fill_(0x2345)
    lay.h[:R].zero_()
    lay.y_rows[:R].zero_()
    lay.experts(T, R + pad, s, live=True)
    torch.cuda.synchronize()
    assert torch.equal(lay.h[:R].view(torch.int16), h_ref.view(torch.int16))
    assert torch.equal(lay.y_rows[:R].view(torch.int16), y_ref.view(torch.int16))
    assert bool((lay.h[R:R + pad].view(torch.int16) == 0x1234).all())
    assert bool((lay.y_rows[R:R + pad].view(torch.int16) == 0x2345).all())


# ---------------------------------------------------------------------------------------------- the f16-output linear
# config 1: a single EXL3 linear, 16 rows of 2048 -> 512, f16 out (the decode band: two units; the tensor-core band for
# the 64-row 1536 -> 4096 case); the oracle's down with its output rounded to f16 instead of bf16
F16_OUT = [
    dict(op="moe_exl3_down", M=16, top_k=1, n_expert=1, geom=[(512, 2048)], bits=4, codebook="mul1"),     # config 1
    dict(op="moe_exl3_down", M=3, top_k=1, n_expert=1, geom=[(512, 2048)], bits=4, codebook="mul1"),
    dict(op="moe_exl3_down", M=64, top_k=1, n_expert=1, geom=[(4096, 1536)], bits=3, codebook="mcg"),
    dict(op="moe_exl3_down", M=5, top_k=2, n_expert=4, geom=[(256, 256)], bits=5, codebook="3inst", h_rot=1,
         drop=0.2),
]


@pytest.mark.parametrize("spec", F16_OUT, ids=lambda s: f"M{s['M']}-{s['geom'][0][0]}x{s['geom'][0][1]}-K{s['bits']}")
def test_down_with_f16_output_matches_the_oracle(dev, plugin, orc, native, spec):
    case = _case(spec, seed=99)
    got = case.run(plugin, device=True, out_dtype="f16", launch=lambda a, s: native.moe_down_f16(a, s),
                   scratch_fn=lambda a: native.moe_down_f16_scratch(a))
    assert got["rc"] == 0, got["rc"]
    assert got["redzone_ok"] and got["inputs_ok"]
    want = orc._run(case, 0, case.h_rot, 0, case.x, case.geom, "own", os.cpu_count() or 4, out_f16=True)
    ok, detail = compare(got["y"], want, "f16", REL_TOL, COS_TOL)
    assert ok, detail
    # the op's own bf16 rows from the same kernels (the f16 entry's scratch sized by its own hook, so both launches
    # take the same band): two roundings of one f32 value v (|bf16 - v| <= 2^-8 |v|, |f16 - v| <= 2^-11 |v| in the
    # normal range), so they agree within one bf16 ulp of the value
    bf = case.run(plugin, device=True)["y"]
    a, b = X.bits_to_f32(got["y"], "f16").astype(np.float64), X.bits_to_f32(bf, "bf16").astype(np.float64)
    bad = np.abs(a - b) > np.maximum(np.abs(a), np.abs(b)) * 2.0 ** -7 + 2.0 ** -24
    if bad.any():
        i = np.argwhere(bad)[0]
        raise AssertionError(f"{int(bad.sum())} of {bad.size} elements: at {tuple(i)} f16 {a[tuple(i)]!r} "
                             f"bf16 {b[tuple(i)]!r} (f16 bits {got['y'][tuple(i)]:#06x}, bf16 bits {bf[tuple(i)]:#06x})")


def test_down_f16_refuses_a_bf16_output(dev, plugin, native):
    case = _case(F16_OUT[0])
    got = case.run(plugin, device=True, launch=lambda a, s: native.moe_down_f16(a, s))   # y declared bf16
    assert got["rc"] == -2                                                             # RAD_E_DTYPE
    assert (got["y"] == 0xFFFF).all()                                                  # nothing written


# ---------------------------------------------------------------------------------------------- the layer driven from C
@pytest.mark.parametrize("T", [1, 8, 64, 300])
def test_c_layer_equals_the_per_op_path(dev, plugin, T):
    """exl3b200_moe_layer_forward (the layer sequence in C, one call) writes the same bits as the same kernels driven
    op by op through the plugin rows; its bf16 output is the f32 output rounded to nearest even."""
    import torch.nn.functional  # noqa: F401
    lay = _small_layer(plugin, T)
    assert lay.c_layer
    s = torch.cuda.current_stream().cuda_stream
    lay.forward(T, s)                                              # C layer, f32
    torch.cuda.synchronize()
    c_out = lay.out[:T].clone()
    ev = [torch.cuda.Event() for _ in range(3)]
    lay.forward(T, s, events=ev)                                   # the per-op path
    torch.cuda.synchronize()
    assert torch.equal(c_out, lay.out[:T])
    lay.forward(T, s, out=lay.out_bf16)                            # C layer, bf16
    torch.cuda.synchronize()
    assert torch.equal(lay.out_bf16[:T], c_out.to(torch.bfloat16))
    assert lay.native.read_error() == 0


def test_bf16_gather_is_the_f32_gather_rounded(dev, native):
    rng = np.random.default_rng(21)
    for T, k, E, width in ((3, 4, 16, 256), (700, 10, 64, 2048)):
        ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
        st, _ = X.stable_scatter(ids, E)
        rows = torch.from_numpy(X.bf16_bits(rng.standard_normal((T * k, width)).astype(np.float32)).view(np.int16))
        rows = rows.to(dev)
        w = torch.from_numpy(rng.random((T, k)).astype(np.float32)).to(dev)
        st_d = torch.from_numpy(st).to(dev)
        work = torch.empty(native.gather_work_bytes(T, k), dtype=torch.uint8, device=dev)
        y32 = torch.empty((T, width), dtype=torch.float32, device=dev)
        y16 = torch.empty((T, width), dtype=torch.bfloat16, device=dev)
        native.moe_gather(rows.data_ptr(), width, st_d.data_ptr(), T * k, w.data_ptr(), T, k, width, y32.data_ptr(),
                          work.data_ptr())
        native.moe_gather_bf16(rows.data_ptr(), width, st_d.data_ptr(), T * k, w.data_ptr(), T, k, width,
                               y16.data_ptr(), work.data_ptr())
        torch.cuda.synchronize()
        assert torch.equal(y16, y32.to(torch.bfloat16))
