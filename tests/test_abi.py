"""The drop-in boundary on the CPU (no GPU needed): libexl3b200.so loads, exports every symbol include/exl3b200.h
declares, reports ABI 17, exports schemas identical field for field to the reference library's (the engine refuses
a second library whose schemas differ, include/exl3_abi.h:5-9), describes operands as the reference does, lays
codes out and back losslessly, and refuses what the reference refuses -- before touching the device."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

from oracle_bind import REF_SO
from exl3b200 import cases as X
from exl3b200 import load_plugin, library_path
from exl3b200 import rad
from exl3b200.rad import Plugin

REPO = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def plugin():
    return load_plugin()


@pytest.fixture(scope="module")
def ref_plugin():
    if not REF_SO.exists():
        pytest.skip("oracle/_ref/libexl3ref.so not built")
    return Plugin(REF_SO)


def declared_functions():
    text = (REPO / "include" / "exl3b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b((?:rad|exl3b200)_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported():
    lib = C.CDLL(str(library_path()))
    names = declared_functions()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), n


def test_identity(plugin):
    assert plugin.lib.rad_plugin_abi_version() == 17
    info = plugin.info
    assert info["name"] == "exl3b200" and info["target"] == "sm_100a" and info["kind"] == 1


def test_schemas_equal_the_reference_library(plugin, ref_plugin):
    assert plugin.schemas() == ref_plugin.schemas()


def test_rows_cover_every_op_on_the_device(plugin):
    ops = {r.op.decode() for r in plugin.rows()}
    assert ops == {s["op"] for s in plugin.schemas()}
    assert all(r.domain == rad.DOMAIN_DEVICE for r in plugin.rows())
    assert all(plugin.lib.rad_kernel_concurrent(i) == 1 for i in range(len(plugin.rows())))


SHAPE_PARAMS = [
    ("moe_exl3_gate_up", {"M": (1, 16), "N": 1024, "K": 2048, "n_expert": 512, "top_k": 10, "dtype": "exl3k3",
                          "codebook": "mul1", "h_rot": 1, "a_rot": 0}),
    ("moe_exl3_down", {"M": (1, 2048), "N": 2048, "K": 512, "n_expert": 512, "top_k": 10, "dtype": "exl3k4",
                       "codebook": "mul1", "h_rot": 0, "N_odd": 2048, "K_odd": 384}),
    ("moe_exl3_prep_gu", {"M": 4, "K": 256, "n_expert": 3, "top_k": 2, "dtype": "exl3k4", "K_odd": 128}),
    ("moe_exl3_gate_up_down", {"M": 3, "N": 512, "K": 256, "n_expert": 4, "top_k": 2, "dtype": "exl3k5",
                               "codebook": "mcg"}),
    ("moe_exl3_gate_up_mod4", {"M": 4, "N": 512, "K": 256, "n_expert": 7, "top_k": 2, "dtype": "exl3k2",
                               "codebook": "3inst", "N_2": 256, "K_3": 128, "h_rot": 1, "a_rot": 1}),
    ("moe_exl3_down_mod4", {"M": 4, "N": 256, "K": 256, "n_expert": 7, "top_k": 2, "dtype": "exl3k8",
                            "codebook": "mul1", "N_1": 128, "h_rot": 0}),
    ("moe_exl3_prep_gu_mod4", {"M": 4, "K": 256, "n_expert": 6, "top_k": 2, "dtype": "exl3k4", "K_2": 128}),
    ("moe_exl3_gate_up_down_mod4", {"M": 2, "N": 512, "K": 256, "n_expert": 8, "top_k": 2, "dtype": "exl3k4",
                                    "codebook": "mul1", "N_3": 256}),
]


@pytest.mark.parametrize("op,params", SHAPE_PARAMS, ids=[o for o, _ in SHAPE_PARAMS])
def test_shape_hook_equals_the_reference(plugin, ref_plugin, op, params):
    mine, theirs = plugin.row(op), ref_plugin.row(op)
    P, nP, keep = rad.make_params(params)
    n_opd = next(s for s in plugin.schemas() if s["op"] == op)["operands"]
    for i in range(len(n_opd)):
        a, b = rad.RadOpdDesc(), rad.RadOpdDesc()
        ra = mine.opd_shape(P, nP, i, C.byref(a))
        rb = theirs.opd_shape(P, nP, i, C.byref(b))
        assert ra == rb, (op, i)
        assert bytes(a) == bytes(b), (op, i)


def test_constraints_select_every_bitrate_and_codebook(plugin):
    row = plugin.row("moe_exl3_gate_up")
    cons = [row.constraints[k] for k in range(row.n_constraints)]
    for bits in range(2, 9):
        for cb in ("mul1", "mcg", "3inst"):
            p = {"M": 8, "N": 1024, "K": 2048, "n_expert": 512, "top_k": 10, "dtype": f"exl3k{bits}",
                 "codebook": cb, "h_rot": 1, "a_rot": 0}
            assert all(rad.constraint_holds(c, p) for c in cons)
    bad = {"M": 8, "N": 1024, "K": 2000, "n_expert": 512, "top_k": 10, "dtype": "exl3k4", "codebook": "mul1",
           "h_rot": 1, "a_rot": 0}
    assert not all(rad.constraint_holds(c, bad) for c in cons)


@pytest.mark.parametrize("op", ["moe_exl3_gate_up", "moe_exl3_down", "moe_exl3_gate_up_down"])
def test_layout_hook_round_trips(plugin, op):
    case = X.Case(op, 3, M=2, top_k=1, n_expert=2, geom=[(512, 256)], bits=3, codebook="mcg", h_rot=1)
    row = plugin.row(op)
    P, nP, keep = rad.make_params(case.params())
    enc = X.encoding(3, "mcg", stacked=op != "moe_exl3_down")
    sel = C.c_int(0)
    R, Cc = case.geom[0]
    codes = np.ascontiguousarray(case.planes[0]["codes"])
    pt = rad.tensor(codes.ctypes.data, rad.DT_UK[3], [R, Cc])
    L = rad.RadLayout()
    assert row.layout(P, nP, 1, C.byref(enc), C.byref(sel), C.byref(pt), 1, C.byref(L)) == 0
    assert L.bytes == R * Cc * 3 // 8 and L.align >= 16
    rec = np.zeros(L.bytes, np.uint8)
    assert row.relayout(P, nP, 1, C.byref(enc), C.byref(sel), C.byref(pt), 1, rec.ctypes.data, L.bytes) == 0
    back = np.zeros_like(codes)
    bt = rad.tensor(back.ctypes.data, rad.DT_UK[3], [R, Cc])
    assert row.unrelayout(P, nP, 1, C.byref(enc), C.byref(sel), rec.ctypes.data, L.bytes, C.byref(bt), 1) == 0
    assert np.array_equal(back, codes)
    # a scale plane is stored as it is
    sel.value = 1
    st = rad.tensor(0, rad.DT["f16"], [1, Cc])
    assert row.layout(P, nP, 2, C.byref(enc), C.byref(sel), C.byref(st), 1, C.byref(L)) == rad.RAD["UNSUPPORTED"]
    # a codebook the encoding does not name is refused by the hook
    enc2 = X.encoding(3, "mul1", stacked=op != "moe_exl3_down")
    sel.value = 0
    assert row.layout(P, nP, 1, C.byref(enc2), C.byref(sel), C.byref(pt), 1, C.byref(L)) == rad.RAD["DTYPE"]


def _launch(plugin, op, params, tensors):
    row = plugin.row(op)
    P, nP, keep = rad.make_params(params)
    arr = (rad.RadTensor * len(tensors))(*tensors)
    a = rad.RadArgs()
    a.t, a.n_t, a.p, a.n_p, a.world_size = arr, len(tensors), P, nP, 1
    return row.launch(C.byref(a), None)


def test_refusals_come_before_any_device_work(plugin):
    """The reference's refusal codes (docs/OPS-exl3.md:292-301), returned by the host side with no GPU present."""
    p = {"M": 2, "N": 256, "K": 128, "n_expert": 2, "top_k": 1, "dtype": "exl3k4", "codebook": "mul1", "h_rot": 0}
    x = np.zeros((2, 128), np.uint16)
    y = np.zeros((2, 256), np.uint16)
    st = np.zeros(2, np.int32)
    off = np.array([0, 1, 2], np.int32)
    codes = np.zeros(8, np.uint64)
    sc = np.zeros((2, 1, 256), np.uint16)

    def tens(xdt=rad.DT["f16"], ydt=rad.DT["bf16"], ycols=256, codes_dt=1970):
        return [rad.tensor(x.ctypes.data, xdt, [2, 128]),
                rad.tensor(codes.ctypes.data, codes_dt, [2, 256, 128], [0, 128, 1]),
                rad.tensor(sc.ctypes.data, rad.DT["f16"], [2, 1, 128]),
                rad.tensor(sc.ctypes.data, rad.DT["f16"], [2, 256, 1]),
                rad.tensor(st.ctypes.data, rad.DT["i32"], [2]),
                rad.tensor(off.ctypes.data, rad.DT["i32"], [3]),
                rad.RadTensor(), rad.RadTensor(), rad.RadTensor(),
                rad.tensor(y.ctypes.data, ydt, [2, ycols])]

    op = "moe_exl3_down"
    assert _launch(plugin, op, dict(p, dtype="exl3k9"), tens()) == rad.RAD["DTYPE"]
    assert _launch(plugin, op, dict(p, codebook="nope"), tens()) == rad.RAD["DTYPE"]
    assert _launch(plugin, op, dict(p, h_rot=2), tens()) == rad.RAD["INVAL"]
    assert _launch(plugin, op, {k: v for k, v in p.items() if k != "h_rot"}, tens()) == rad.RAD["SCHEMA"]
    assert _launch(plugin, op, dict(p, K=100), tens()) == rad.RAD["SHAPE"]
    assert _launch(plugin, op, p, tens(ydt=rad.DT["f16"])) == rad.RAD["DTYPE"]
    assert _launch(plugin, op, p, tens(ycols=128)) == rad.RAD["SHAPE"]
    assert _launch(plugin, op, p, tens(codes_dt=rad.DT_UK[4])) == rad.RAD["DTYPE"]   # not laid out
    t = tens()
    t[6] = rad.tensor(codes.ctypes.data, 1970, [1, 256, 128], [0, 128, 1])     # odd tables partly present
    assert _launch(plugin, op, p, t) == rad.RAD["INVAL"]
    assert (y == 0).all()


@pytest.mark.parametrize("op,E,H,W,k", [("moe_exl3_gate_up", 512, 2048, 512, 10), ("moe_exl3_down", 512, 2048, 512, 10),
                                        ("moe_exl3_gate_up", 64, 2048, 512, 8), ("moe_exl3_down", 32, 2048, 128, 8),
                                        ("moe_exl3_gate_up", 1, 1536, 2048, 1), ("moe_exl3_down", 1, 1536, 4096, 1)])
def test_layer_band_rule_mirrors_the_library(plugin, op, E, H, W, k):
    """exl3b200/layer.py names the band each op runs on (bench lines, tests) by restating the library's rule; the
    library's own scratch hook says the same thing (it asks for rotated-input scratch exactly on the tensor-core
    band when the op rotates its own input), for every pass size from one token to prefill."""
    from types import SimpleNamespace

    from exl3b200.layer import MoeLayer
    gate_up = op == "moe_exl3_gate_up"
    row = plugin.row(op)
    mirror = SimpleNamespace(n_local=E, W=W, H=H)
    fake = 1 << 20                       # the hook reads shapes only; no pointer is dereferenced
    for T in (1, 2, 3, 4, 6, 8, 16, 33, 64, 512, 2048):
        rows = T * k
        p = {"M": T, "N": 2 * W if gate_up else H, "K": H if gate_up else W, "n_expert": E, "top_k": k,
             "dtype": "exl3k3" if gate_up else "exl3k4", "codebook": "mul1", "h_rot": 0}
        if gate_up:
            p["a_rot"] = 0
        P, nP, keep = rad.make_params(p)
        if gate_up:
            ts = [rad.tensor(fake, rad.DT["f16"], [T, H]),
                  rad.tensor(fake, 1970, [E, 2 * W, H], [0, H, 1]),
                  rad.tensor(fake, rad.DT["f16"], [E, 1, H]), rad.tensor(fake, rad.DT["f16"], [E, 1, H]),
                  rad.tensor(fake, rad.DT["f16"], [E, 2 * W, 1]), rad.RadTensor(),
                  rad.tensor(fake, rad.DT["i32"], [rows]), rad.tensor(fake, rad.DT["i32"], [E + 1]),
                  rad.RadTensor(), rad.RadTensor(), rad.RadTensor(), rad.RadTensor(), rad.RadTensor(),
                  rad.tensor(fake, rad.DT["f16"], [rows, W])]
        else:
            ts = [rad.tensor(fake, rad.DT["f16"], [rows, W]),
                  rad.tensor(fake, 1970, [E, H, W], [0, W, 1]),
                  rad.tensor(fake, rad.DT["f16"], [E, 1, W]), rad.tensor(fake, rad.DT["f16"], [E, H, 1]),
                  rad.tensor(fake, rad.DT["i32"], [rows]), rad.tensor(fake, rad.DT["i32"], [E + 1]),
                  rad.RadTensor(), rad.RadTensor(), rad.RadTensor(),
                  rad.tensor(fake, rad.DT["bf16"], [rows, H])]
        arr = (rad.RadTensor * len(ts))(*ts)
        a = rad.RadArgs()
        a.t, a.n_t, a.p, a.n_p, a.world_size = arr, len(ts), P, nP, 1
        need = int(row.scratch(C.byref(a)))
        want = (rows * (2 * H if gate_up else W) * 2 + 255) // 256 * 256
        tc = MoeLayer._tc(mirror, "gate_up" if gate_up else "down", rows)
        assert need == (want if tc else 0), (T, need, tc)


def _layer_desc(E, n_local, base, H=2048, W=512, k=10):
    from exl3b200.native import LayerDesc
    d = LayerDesc()
    d.n_expert, d.n_local, d.expert_base, d.hidden, d.width, d.top_k = E, n_local, base, H, W, k
    d.bits_gu, d.bits_dn, d.codebook = 3, 4, 2
    d.gu_codes = d.dn_codes = d.suh = d.suh1 = d.svh_gu = d.dn_suh = d.svh_dn = 1 << 20
    return d


def _regions(bufs, sizes):
    """(start, end) of every carved buffer named in `sizes` (bytes), checked 256-byte aligned."""
    out = []
    for name, n in sizes.items():
        p = getattr(bufs, name)
        assert p is not None and p % 256 == 0, name
        out.append((p, p + n, name))
    return sorted(out)


@pytest.mark.parametrize("world,rank,T,fuse", [(1, 0, 192, True), (2, 1, 2048, True), (8, 5, 2048, True),
                                               (4, 3, 8, False)])
def test_ep_step_carve_is_disjoint_and_in_bounds(world, rank, T, fuse):
    """The expert-parallel step's C driver carves one caller block (pure host arithmetic: no device address is
    touched): every buffer 256-byte aligned, inside the block, none overlapping another; the window layout puts its
    six regions in order with room for the sizes the exchange kernels write."""
    from exl3b200.native import EpDesc, Native
    nat = Native()
    E, H, W, k = 512, 2048, 512, 10
    nl = E // world
    offs, wbytes = nat.ep_window_layout(world, T, k, H)
    P = T * k
    need = [world * T * H * 2, world * P * 4, P * H * 2, world * 32, 8, H * 2]
    for i in range(6):
        end = offs[i + 1] if i < 5 else wbytes
        assert offs[i] % 256 == 0 and end - offs[i] >= need[i], (i, offs)
    d = EpDesc()
    d.layer = _layer_desc(E, nl, rank * nl, H, W, k)
    d.rank, d.world, d.max_tokens, d.fuse_combine = rank, world, T, int(fuse)
    d.window, d.peers, d.epoch, d.status = 1 << 30, 1 << 30, 1 << 30, 1 << 30
    for i, o in enumerate(offs):
        d.offs[i] = o
    nbytes = nat.ep_step_work_bytes(d)
    base = 1 << 40
    b = nat.ep_step_carve(d, base, nbytes)
    Q = world * P
    assert b.cap == Q and b.max_tokens == T
    sizes = {"ids": P * 4, "w": P * 4, "dest": P * 4, "sorted_pairs": P * 4, "row_tok": P * 4, "send_meta": P * 4,
             "dest_off": (world + 1) * 4, "counts": 2 * world * 4, "hdr": (3 * world + 1) * 4, "pair_e": Q * 4,
             "pair_row": Q * 4, "dst_rank": Q * 4, "dst_pos": Q * 4, "sorted_pair": Q * 4, "sorted_row": Q * 4,
             "expert_offset": (nl + 1) * 4, "row_dst": Q * 8, "h": Q * W * 2,
             "scatter_rank": max(1, nat.scatter_work_bytes(P, world)),
             "scatter_local": max(1, nat.scatter_work_bytes(Q, nl)),
             "gather_work": max(1, nat.gather_work_bytes(T, k))}
    if not fuse:
        sizes["y_rows"] = Q * H * 2
    else:
        assert not b.y_rows
    if b.gu_scratch:
        sizes["gu_scratch"] = b.gu_scratch_bytes
    if b.dn_scratch:
        sizes["dn_scratch"] = b.dn_scratch_bytes
    # gate_up at capacity runs the tensor-core band: its rotated input rows are carved
    assert b.gu_scratch_bytes >= Q * 2 * H * 2
    regs = _regions(b, sizes)
    assert regs[0][0] >= base and regs[-1][1] <= base + nbytes
    for (s0, e0, n0), (s1, e1, n1) in zip(regs, regs[1:]):
        assert e0 <= s1, (n0, n1)


def test_step_descriptions_are_refused_before_any_device_work():
    """The drivers check their descriptions on the host: a rank outside the world, an expert base that is not the
    rank's block, an expert count the world does not divide, a missing window or epoch -- refused (-1 bytes; a
    carve or forward returns an error) with nothing enqueued."""
    from exl3b200.native import EpDesc, Native, TpDesc
    nat = Native()

    def ep(world=2, rank=1, nl=256, base=256, window=1 << 30, epoch=1 << 30):
        d = EpDesc()
        d.layer = _layer_desc(world * nl if nl else 512, nl or 1, base)
        d.rank, d.world, d.max_tokens, d.fuse_combine = rank, world, 64, 1
        d.window, d.peers, d.epoch, d.status = window, 1 << 30, epoch, 1 << 30
        return d

    assert nat.lib.exl3b200_ep_step_work_bytes(C.byref(ep())) > 0
    for bad in (ep(rank=2), ep(base=0), ep(world=33, rank=0, base=0), ep(window=None), ep(epoch=None)):
        assert nat.lib.exl3b200_ep_step_work_bytes(C.byref(bad)) == -1
    d = ep()
    d.layer.n_expert = 511                      # the world does not divide the experts
    assert nat.lib.exl3b200_ep_step_work_bytes(C.byref(d)) == -1
    assert nat.lib.exl3b200_ep_window_layout(0, 64, 10, 2048, (C.c_int64 * 6)()) == -1
    assert nat.lib.exl3b200_tp_window_layout(2, 0, 2048, (C.c_int64 * 4)()) == -1
    # the width-split driver refuses a slice layer that does not hold every expert, before any launch
    from exl3b200.native import LayerBufs
    t = TpDesc()
    t.layer = _layer_desc(512, 256, 0)
    t.rank, t.world, t.max_tokens = 0, 2, 64
    t.window, t.peers, t.epoch, t.status = 1 << 30, 1 << 30, 1 << 30, 1 << 30
    rc = nat.lib.exl3b200_tp_step_forward(C.byref(t), C.byref(LayerBufs()), 1 << 30, 1 << 30, 8, 1 << 30, 2048,
                                          None, None)
    assert rc == -1


def test_block_carve_and_refusals():
    """The MoE block's C driver carves one caller block into the routed layer's and the shared expert's buffers
    (host arithmetic only: fake addresses), each buffer inside the block and no two overlapping; a shared expert that
    is not one expert of top-1 over the routed hidden size, or a misaligned gate column, is refused."""
    from exl3b200.native import BlockDesc, Native
    nat = Native()

    def desc(sh_experts=1, sh_k=1, sh_hidden=2048, gate=1 << 20):
        d = BlockDesc()
        d.routed = _layer_desc(512, 512, 0)
        d.shared = _layer_desc(sh_experts, sh_experts, 0, H=sh_hidden, W=1024, k=sh_k)
        d.sgate_w = gate
        return d

    d = desc()
    n = nat.block_work_bytes(d, 2048)
    base = 1 << 40
    b = nat.block_carve(d, 2048, base, n)
    P, H = 2048 * 10, 2048
    sizes = {}
    for part, rows, W in (("routed", P, 512), ("shared", 2048, 1024)):
        lb = getattr(b, part)
        for name, nb in (("ids", rows * 4), ("w", rows * 4), ("sorted_tok", rows * 4), ("h", rows * W * 2),
                         ("y_rows", rows * H * 2)):
            sizes[(part, name)] = (getattr(lb, name), nb)
        for name in ("gu_scratch", "dn_scratch"):
            if getattr(lb, name):
                sizes[(part, name)] = (getattr(lb, name), getattr(lb, name + "_bytes"))
    regs = sorted((p, p + nb, k) for k, (p, nb) in sizes.items())
    assert regs[0][0] >= base and regs[-1][1] <= base + n
    for (s0, e0, n0), (s1, e1, n1) in zip(regs, regs[1:]):
        assert e0 <= s1, (n0, n1)
    for bad in (desc(sh_experts=2), desc(sh_k=2), desc(sh_hidden=1024), desc(gate=(1 << 20) + 8), desc(gate=None)):
        assert nat.lib.exl3b200_moe_block_work_bytes(C.byref(bad), 2048) == -1
