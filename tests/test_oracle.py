"""The oracle pinned before it is trusted (CPU): the restatement in oracle/ against the vllm-exl3 golden decode, the
reference's hand-computed codebook values and tile map, and the reference library itself (oracle/_ref, built from
the reference sources) op by op. Fixtures: tests/golden/ (made by tests/golden/make_golden.py)."""
from pathlib import Path

import numpy as np
import pytest

from oracle_bind import REF_SO, Oracle, RefLib
from exl3b200 import cases as X
from exl3b200.rad import Plugin

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def orc():
    return Oracle()


@pytest.fixture(scope="module")
def ref():
    if not REF_SO.exists():
        pytest.skip("oracle/_ref/libexl3ref.so not built")
    return RefLib()


@pytest.fixture(scope="module")
def ref_plugin():
    if not REF_SO.exists():
        pytest.skip("oracle/_ref/libexl3ref.so not built")
    return Plugin(REF_SO)


def test_decode_matches_the_vllm_exl3_golden(orc):
    """common/tests/data/exl3_golden.npz (vllm-exl3 host decode; K = 3, 4 x mcg, mul1), every fp16 bit."""
    z = np.load(GOLDEN / "exl3_golden_decode.npz")
    for bits in (3, 4):
        for cb in ("mcg", "mul1"):
            want = z[f"w_hat_k{bits}_{cb}"].view(np.uint16)
            got = orc.trellis_decode(z[f"trellis_k{bits}_{cb}"], bits, cb)
            assert np.array_equal(got, want), (bits, cb)
            # negative controls: another codebook, one flipped stream bit
            other = "mcg" if cb == "mul1" else "mul1"
            assert not np.array_equal(orc.trellis_decode(z[f"trellis_k{bits}_{cb}"], bits, other), want)
            t = z[f"trellis_k{bits}_{cb}"].copy()
            t.reshape(-1)[5] ^= 0x0100
            assert not np.array_equal(orc.trellis_decode(t, bits, cb), want)


def test_codebooks_give_the_hand_computed_values(orc):
    """The reference's hand-computed values (common/tests/exl3_decode_test.c:47-66)."""
    v = [(0x0000, 0x3A25, 0x3F60, 0xC2E8), (0x0001, 0xBB5B, 0x304E, 0x3921),
         (0x1234, 0xC066, 0x3E0F, 0xB89E), (0xFFFF, 0xB110, 0x3ACD, 0xB936)]
    for s, i3, mcg, mul1 in v:
        assert orc.lib.orc_codebook_value(s, 0) == i3
        assert orc.lib.orc_codebook_value(s, 1) == mcg
        assert orc.lib.orc_codebook_value(s, 2) == mul1
    assert orc.lib.orc_codebook_value(0x10000, 2) == 0xC2E8
    assert orc.lib.orc_codebook_value(0, 7) == 0x7E00


def test_codebook_tables_equal_the_reference_for_every_state(orc, ref):
    for cb in ("3inst", "mcg", "mul1"):
        mine = orc.codebook_table(cb)
        theirs = np.array([ref.codebook_value(s, cb) for s in range(65536)], np.uint16)
        assert np.array_equal(mine, theirs), cb


def test_a_hand_built_3inst_tile(orc):
    """At K = 8 the state of p is (sym[p-1] << 8) | sym[p] circularly (common/tests/exl3_decode_test.c:69-90)."""
    sym = np.arange(256, dtype=np.uint32)
    plane = np.zeros((16, 16), np.uint32)
    # tile position p holds W_hat[k = r][n = c]; the canonical plane keeps it at (n = c, k = r)
    p = np.arange(256)
    L, j = p // 8, p % 8
    r = 2 * (L % 4) + np.array([0, 1, 8, 9])[j % 4]
    c = L // 4 + 8 * (j // 4)
    plane[c, r] = sym
    rec = orc.codes_to_record(X.pack_codes(plane, 8), 16, 16, 8)
    w = orc.record_decode(rec, 16, 16, 8, "3inst")
    # position 1 = tile (r=1, c=0) has state 0x0001 -> 0xBB5B; position 0 has state 0xFF00
    assert w[0, 1] == 0xBB5B
    assert w[0, 0] == orc.lib.orc_codebook_value(0xFF00, 0)


@pytest.mark.parametrize("bits", range(1, 9))
def test_relayout_matches_the_reference_and_round_trips(orc, ref, bits):
    rng = np.random.default_rng(100 + bits)
    rows, cols = 64, 128
    sym = rng.integers(0, 1 << bits, size=(rows, cols), dtype=np.uint32)
    codes = X.pack_codes(sym, bits)
    rec = orc.codes_to_record(codes, rows, cols, bits)
    assert np.array_equal(rec, ref.codes_to_record(codes, rows, cols, bits))
    assert np.array_equal(orc.record_to_codes(rec, rows, cols, bits), codes)


@pytest.mark.parametrize("bits", range(1, 9))
@pytest.mark.parametrize("cb", ["3inst", "mcg", "mul1"])
def test_record_decode_equals_the_reference_trellis_decode(orc, ref, bits, cb):
    rng = np.random.default_rng(7 * bits + len(cb))
    rows, cols = 32, 48
    trellis = rng.integers(-32768, 32768, size=(cols // 16, rows // 16, 16 * bits)).astype(np.int16)
    want = ref.trellis_decode(trellis, bits, cb)               # [k][n]
    got = orc.record_decode(trellis.view(np.uint16), rows, cols, bits, cb)   # [n][k]
    assert np.array_equal(got.T, want)


def test_had128_equals_the_reference(orc, ref):
    rng = np.random.default_rng(3)
    v = rng.standard_normal(1024).astype(np.float32)
    assert np.array_equal(orc.had128(v).view(np.uint32), ref.had128(v).view(np.uint32))


# ---------------------------------------------------------------------------------------------- the ops
OP_CASES = [
    dict(op="moe_exl3_down", M=4, top_k=2, n_expert=5, geom=[(256, 128)], bits=4, codebook="mul1", drop=0.2),
    dict(op="moe_exl3_down", M=3, top_k=2, n_expert=4, geom=[(256, 256), (128, 128)], bits=3, codebook="mcg",
         n_protect=1),
    dict(op="moe_exl3_gate_up", M=4, top_k=2, n_expert=5, geom=[(256, 256)], bits=4, codebook="mul1", drop=0.2),
    dict(op="moe_exl3_gate_up", M=3, top_k=2, n_expert=4, geom=[(512, 128), (256, 256)], bits=2, codebook="3inst",
         h_rot=1, x_dtype="bf16"),
    dict(op="moe_exl3_gate_up", M=4, top_k=2, n_expert=4, geom=[(256, 128)], bits=5, codebook="mcg", a_rot=1),
    dict(op="moe_exl3_prep_gu", M=4, top_k=2, n_expert=3, geom=[(256, 256), (256, 128)], bits=4, drop=0.25),
    dict(op="moe_exl3_gate_up_down", M=3, top_k=2, n_expert=4, geom=[(256, 128)], bits=4, codebook="mul1"),
    dict(op="moe_exl3_down_mod4", M=4, top_k=2, n_expert=6, geom=[(128, 128), (256, 128), (128, 256), (128, 128)],
         bits=6, codebook="mul1"),
    dict(op="moe_exl3_gate_up_mod4", M=4, top_k=2, n_expert=6,
         geom=[(256, 128), (512, 128), (256, 256), (256, 128)], bits=7, codebook="mcg", h_rot=1),
]


@pytest.mark.parametrize("spec", OP_CASES, ids=lambda s: f"{s['op']}-K{s['bits']}")
def test_restated_ops_equal_the_reference_library(orc, ref_plugin, spec):
    """The restatement and the reference library (both host, both -ffp-contract=off, the same libm) agree to the
    bit on every op, including the rows they must leave zero or unwritten."""
    spec = dict(spec)
    case = X.Case(spec.pop("op"), 1234, **spec)
    r = case.run(ref_plugin, device=False)
    assert r["rc"] == 0, r["rc"]
    assert r["redzone_ok"] and r["inputs_ok"]
    prefill = np.full((case.T, case.y_cols), 0xFFFF, np.uint16)
    want = orc.run_case(case, prefill=prefill)
    assert np.array_equal(r["y"], want)
