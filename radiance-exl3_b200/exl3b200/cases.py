"""cases.py -- seeded EXL3 routed-expert cases, built once as canonical planes and run through any plugin.

A case is one launch of one op: its parameters, its experts' planes (canonical form: uK codes plane, f16 scales),
its routing (a stable counting sort of seeded top-k ids) and its input rows. `run(plugin, device=...)` drives a
plugin's row the way the engine does -- every weight table through the row's own layout hooks (relayout, and an
unrelayout round trip checked byte for byte), operands between poisoned margins, outputs prefilled with 0xFF --
and returns the output and what the harness saw (redzones, inputs unchanged, the round trip).

Distributions follow BASELINE.json's configs: codes uniform random symbols (every sequence is a valid trellis),
suh random +-1, svh +-|N(0,1)| * 0.02 (the per-channel scale lives in svh), activations N(0,1).
"""
import ctypes as C

import numpy as np

from . import rad

RED = 256          # poisoned margin bytes on each side of every buffer
RED_FILL = 0xA5

PLANE_OF = {"codes": 0, "suh": 1, "suh1": 2, "svh": 3, "dn_suh": 4, "dn_codes": 5, "dn_svh": 6}
ENC_PLANE = {0: 0, 1: 1, 2: 3, 3: 2, 4: 1, 5: 0, 6: 2}   # EXL3B_P_* -> the encoding's plane index
BASE_OPS = {"moe_exl3_gate_up": "gu", "moe_exl3_down": "dn", "moe_exl3_prep_gu": "pg", "moe_exl3_gate_up_down": "gd"}


def base_op(op):
    return op[:-5] if op.endswith("_mod4") else op


def split_name(name):
    """operand name -> (plane name, class): 'codes_odd' -> ('codes', 1), 'suh1_2' -> ('suh1', 2)."""
    if name.endswith("_odd"):
        return name[:-4], 1
    for q in (1, 2, 3):
        if name.endswith(f"_{q}") and name[:-2] in PLANE_OF:
            return name[:-2], q
    return name, 0


# ------------------------------------------------------------------------------------------ planes
def pack_codes(sym, bits):
    """[rows, cols] K-bit symbols -> the canonical uK plane: rows of ceil(cols*K/8) bytes, LSB first."""
    rows, cols = sym.shape
    b = ((sym.astype(np.uint32)[..., None] >> np.arange(bits, dtype=np.uint32)) & 1).astype(np.uint8)
    flat = b.reshape(rows, cols * bits)
    pad = (-(cols * bits)) % 8
    if pad:
        flat = np.concatenate([flat, np.zeros((rows, pad), np.uint8)], 1)
    return np.packbits(flat, axis=1, bitorder="little")


def f16(x):
    return np.asarray(x, np.float32).astype(np.float16)


def bits_f16(a):
    return np.ascontiguousarray(a).view(np.uint16)


def random_planes(rng, rows, cols, bits, stacked):
    """One weight's canonical planes: codes uK [rows, cols], suh f16 [cols] (+-1), svh f16 [rows] (+-|N|*0.02),
    suh1 f16 [cols] for a stacked gate_up."""
    sym = rng.integers(0, 1 << bits, size=(rows, cols), dtype=np.uint32)
    sign = lambda m: (rng.integers(0, 2, size=m) * 2 - 1).astype(np.float32)  # noqa: E731
    p = {"codes": pack_codes(sym, bits), "sym": sym,
         "suh": f16(sign(cols)),
         "svh": f16(sign(rows) * np.abs(rng.standard_normal(rows)).astype(np.float32) * 0.02)}
    if stacked:
        p["suh1"] = f16(sign(cols))
    return p


def stable_scatter(ids, n_expert, expert_base=0):
    """The routing contract (include/exl3_abi.h:96-158): a stable counting sort of the flattened pairs by
    expert - expert_base; pairs outside [0, n_expert) dropped; -1 past the live count."""
    flat = np.asarray(ids, np.int64).reshape(-1)
    local = flat - expert_base
    valid = (local >= 0) & (local < n_expert)
    key = np.where(valid, local, n_expert)
    order = np.argsort(key, kind="stable")
    counts = np.bincount(local[valid], minlength=n_expert)[:n_expert]
    off = np.zeros(n_expert + 1, np.int32)
    off[1:] = np.cumsum(counts)
    sorted_tok = np.full(flat.size, -1, np.int32)
    live = int(off[-1])
    sorted_tok[:live] = order[:live].astype(np.int32)
    return sorted_tok, off


def route(rng, M, top_k, n_total, drop=0.0):
    """top_k distinct experts a token, uniformly; with `drop`, some slots -1 or past the range (dropped)."""
    ids = np.stack([rng.permutation(n_total)[:top_k] for _ in range(M)]).astype(np.int32) if M else \
        np.zeros((0, top_k), np.int32)
    if drop:
        hit = rng.random(ids.shape) < drop
        ids[hit] = np.where(rng.random(int(hit.sum())) < 0.5, -1, n_total + 3)
    return ids


# ------------------------------------------------------------------------------------------ a case
class Case:
    """One launch of one op over seeded planes and routing.

    geom: per class (rows, cols) of the op's OWN weight (gate_up / gate_up_down: the stacked [2W, H]; down: [H, W];
    prep_gu: (2W, H) too -- it reads only cols). n_class: 1 (odd tables absent), 2, or 4 (a _mod4 op)."""

    def __init__(self, op, seed, *, M, top_k, n_expert, geom, bits=4, codebook="mul1", h_rot=0, a_rot=0,
                 n_class=None, drop=0.0, n_protect=0, x_dtype="f16", pitch_extra=0, table_form="table",
                 x=None, planes=None, sorted_tok=None, expert_offset=None):
        rng = np.random.default_rng(seed)
        self.op, self.base = op, base_op(op)
        self.mod4 = op.endswith("_mod4")
        self.n_class = n_class or (4 if self.mod4 else len(geom))
        self.geom = [tuple(geom[c % len(geom)]) for c in range(self.n_class)]
        self.M, self.top_k, self.n_expert, self.bits, self.codebook = M, top_k, n_expert, bits, codebook
        self.h_rot = 1 if self.base == "moe_exl3_gate_up_down" else h_rot
        self.a_rot = a_rot
        self.T = M * top_k
        self.table_form = table_form
        gate_up = self.base in ("moe_exl3_gate_up", "moe_exl3_prep_gu", "moe_exl3_gate_up_down")
        self.x_cols = max(c for _, c in self.geom)
        if self.base == "moe_exl3_prep_gu":
            self.y_cols = 2 * self.x_cols
        elif self.base == "moe_exl3_gate_up_down":
            self.y_cols = self.x_cols
        else:
            self.y_cols = max(r for r, _ in self.geom) // (2 if gate_up else 1)
        # planes, expert by expert (expert e: class e % n_class)
        if planes is None:
            planes = []
            for e in range(n_expert):
                R, Cc = self.geom[e % self.n_class]
                p = random_planes(rng, R, Cc, bits, gate_up)
                if gate_up and (self.h_rot or self.base == "moe_exl3_gate_up_down"):
                    sign = (rng.integers(0, 2, size=R // 2) * 2 - 1).astype(np.float32)
                    p["dn_suh"] = f16(sign)
                if self.base == "moe_exl3_gate_up_down":
                    dn = random_planes(rng, Cc, R // 2, bits, False)
                    p["dn_codes"], p["dn_sym"], p["dn_svh"] = dn["codes"], dn["sym"], dn["svh"]
                planes.append(p)
        self.planes = planes
        # routing
        if sorted_tok is None:
            ids = route(rng, M, top_k, n_expert + n_protect, drop)
            self.ids = ids
            sorted_tok, expert_offset = stable_scatter(ids, n_expert)
            # protected experts sort last and are not this op's: their rows hold valid flat indices past the live
            # count (include/exl3_abi.h:125-134)
            live = int(expert_offset[-1])
            flat = ids.reshape(-1)
            prot = np.nonzero(flat >= n_expert)[0]
            prot = prot[flat[prot] < n_expert + n_protect]
            sorted_tok[live:live + prot.size] = prot.astype(np.int32)
        self.sorted_tok = np.asarray(sorted_tok, np.int32)
        self.expert_offset = np.asarray(expert_offset, np.int32)
        # input rows
        self.x_dtype = x_dtype
        if x is None:
            if self.base == "moe_exl3_down" or (self.base == "moe_exl3_gate_up" and a_rot):
                rows, width = self.T, (2 * self.x_cols if a_rot else self.x_cols)
            else:
                rows, width = M, self.x_cols
            xv = rng.standard_normal((rows, width)).astype(np.float32)
            x = bits_f16(f16(xv)) if x_dtype == "f16" else bf16_bits(xv)
        self.x = np.ascontiguousarray(x, np.uint16)
        self.pitch_extra = pitch_extra

    # -------------------------------------------------------------- parameters
    def params(self, M_range=None):
        p = {"M": M_range or self.M}
        if self.base != "moe_exl3_prep_gu":
            p["N"] = self.geom[0][0]
        p["K"] = self.geom[0][1]
        p["n_expert"] = self.n_expert
        p["top_k"] = self.top_k
        p["dtype"] = f"exl3k{self.bits}"
        if self.base != "moe_exl3_prep_gu":
            p["codebook"] = self.codebook
        if self.mod4:
            for q in (1, 2, 3):
                if self.base != "moe_exl3_prep_gu":
                    p[f"N_{q}"] = self.geom[q][0]
                p[f"K_{q}"] = self.geom[q][1]
        elif self.n_class == 2:
            if self.base != "moe_exl3_prep_gu":
                p["N_odd"] = self.geom[1][0]
            p["K_odd"] = self.geom[1][1]
        if self.base in ("moe_exl3_gate_up", "moe_exl3_down"):
            p["h_rot"] = self.h_rot
        if self.base == "moe_exl3_gate_up":
            p["a_rot"] = self.a_rot
        return p

    def class_entries(self, c):
        return (self.n_expert - c + self.n_class - 1) // self.n_class

    def table(self, plane, c):
        """[entries, r, cols] array of class c's plane (codes as uK bytes [entries, rows, row_bytes])."""
        ents = [self.planes[e] for e in range(c, self.n_expert, self.n_class)]
        return ents

    def out_dtype(self):
        return "bf16" if self.base in ("moe_exl3_down", "moe_exl3_gate_up_down") else "f16"

    # -------------------------------------------------------------- running
    def run(self, plugin, device=False, domain=None, stream=0, scratch=True, out_dtype=None, launch=None,
            scratch_fn=None):
        """Launch this case on `plugin`'s row for the op. Returns dict(rc, y (uint16 bits [T, y_cols]) or None,
        redzone_ok, inputs_ok, unrelayout_ok, layouts). `out_dtype` ("f16" / "bf16") overrides the output operand's
        type and `launch(args_ptr, stream)` the row's launch: an entry point that takes the row's RadArgs with
        another output type (exl3b200_moe_down_f16) runs through the same harness; `scratch_fn(args_ptr)` then sizes
        its scratch in place of the row's hook."""
        schema = {s["op"]: s for s in plugin.schemas()}[self.op]
        row = plugin.row(self.op, domain)
        if row is None:
            raise LookupError(f"{plugin.path}: no row for {self.op}")
        params = self.params()
        P, nP, keep = rad.make_params(params)
        mem = DeviceMem() if device else HostMem()
        tensors = (rad.RadTensor * len(schema["operands"]))()
        enc_own = encoding(self.bits, self.codebook, stacked=self.base != "moe_exl3_down")
        enc_dn = encoding(self.bits, self.codebook, stacked=False)
        report = {"layouts": [], "unrelayout_ok": True}
        outputs = {}
        inputs = []
        for i, (name, role, optional) in enumerate(schema["operands"]):
            pname, c = split_name(name)
            if role == rad.OPD_WTAB:
                if c >= self.n_class or (pname == "dn_suh" and not self.h_rot):
                    if optional or c >= self.n_class:
                        tensors[i] = rad.RadTensor()
                        continue
                tensors[i] = self._table(plugin, row, mem, i, pname, c, P, nP, enc_own, enc_dn, report)
                continue
            if name in ("sorted_tok", "expert_offset"):
                arr = self.sorted_tok if name == "sorted_tok" else self.expert_offset
                ptr = mem.put(arr.view(np.uint8))
                inputs.append((ptr, arr.view(np.uint8)))
                tensors[i] = rad.tensor(ptr, rad.DT["i32"], [arr.size])
                continue
            if name == "topk_ids":
                tensors[i] = rad.RadTensor()
                continue
            if role == rad.OPD_IN:
                rows, width = self.x.shape
                pitch = width + self.pitch_extra
                buf = np.full((rows, pitch), 0x5A5A, np.uint16)
                buf[:, :width] = self.x
                ptr = mem.put(buf.view(np.uint8))
                inputs.append((ptr, buf.view(np.uint8)))
                tensors[i] = rad.tensor(ptr, rad.DT[self.x_dtype if self._token_rows() else "f16"], [rows, width],
                                        [pitch, 1])
                continue
            # the output: prefilled with 0xFF (NaN in f16 and bf16), row pitch with garbage past the width
            pitch = self.y_cols + self.pitch_extra
            ptr = mem.alloc(self.T * pitch * 2, 0xFF)
            outputs[i] = (ptr, pitch)
            tensors[i] = rad.tensor(ptr, rad.DT[out_dtype or self.out_dtype()], [self.T, self.y_cols], [pitch, 1])
        a = rad.RadArgs()
        a.t = tensors
        a.n_t = len(schema["operands"])
        a.p = P
        a.n_p = nP
        a.world_size = 1
        if scratch and (scratch_fn or row.scratch):
            need = (scratch_fn or row.scratch)(C.byref(a))
            if need > 0:
                a.scratch = mem.alloc(need, 0)
                a.scratch_bytes = need
        rc = (launch or row.launch)(C.byref(a), stream)
        mem.sync()
        report["rc"] = rc
        ptr, pitch = next(iter(outputs.values()))
        raw = mem.get(ptr, self.T * pitch * 2).view(np.uint16).reshape(self.T, pitch) if self.T else \
            np.zeros((0, pitch), np.uint16)
        report["y"] = raw[:, :self.y_cols].copy()
        report["y_pitch_tail"] = raw[:, self.y_cols:].copy()
        report["redzone_ok"] = mem.redzones_ok()
        report["inputs_ok"] = all(np.array_equal(mem.get(p, a_.nbytes), a_.reshape(-1)) for p, a_ in inputs)
        mem.free()
        return report

    def _token_rows(self):
        return self.base in ("moe_exl3_prep_gu", "moe_exl3_gate_up_down") or \
            (self.base == "moe_exl3_gate_up" and not self.a_rot)

    def _table(self, plugin, row, mem, operand, pname, c, P, nP, enc_own, enc_dn, report):
        ents = [self.planes[e] for e in range(c, self.n_expert, self.n_class)]
        n_ent = len(ents)
        R, Cc = self.geom[c]
        plane = PLANE_OF[pname]
        key = {"dn_codes": "dn_codes", "dn_svh": "dn_svh"}.get(pname, pname)
        if plane in (0, 5):
            rows_p, cols_p = (R, Cc) if plane == 0 else (Cc, R // 2)
            dt = rad.DT_UK[self.bits]
            blobs = [np.ascontiguousarray(p[key]).view(np.uint8).reshape(-1) for p in ents]
            shape = [n_ent, rows_p, cols_p]
        else:
            blobs = [np.ascontiguousarray(p[key]).view(np.uint8).reshape(-1) for p in ents]
            n_el = blobs[0].size // 2
            rows_p, cols_p = ((1, n_el) if plane in (1, 2, 4) else (n_el, 1))
            dt = rad.DT["f16"]
            shape = [n_ent, rows_p, cols_p]
        ent_b = blobs[0].size
        # the row's layout hook, with the canonical plane of one entry
        lrc, L, sel = rad.RAD["UNSUPPORTED"], rad.RadLayout(), C.c_int(-1)
        enc = enc_dn if plane >= 4 else enc_own
        if row.layout:
            sel.value = ENC_PLANE[plane]
            pt = rad.tensor(0, dt, [rows_p, cols_p])
            lrc = row.layout(P, nP, operand, C.byref(enc), C.byref(sel), C.byref(pt), 1, C.byref(L))
        if lrc not in (rad.RAD["OK"], rad.RAD["UNSUPPORTED"]):
            raise RuntimeError(f"layout refused operand {operand} ({pname}): {lrc}")
        if lrc == rad.RAD["OK"]:
            al = max(256, int(L.align))
            stored_b = (int(L.bytes) + al - 1) // al * al
            stored = np.zeros(n_ent * stored_b, np.uint8)
            ok = True
            for j, b in enumerate(blobs):
                src = np.ascontiguousarray(b)
                pt = rad.tensor(src.ctypes.data, dt, [rows_p, cols_p])
                dst = stored[j * stored_b:(j + 1) * stored_b]
                if row.relayout(P, nP, operand, C.byref(enc), C.byref(sel), C.byref(pt), 1,
                                dst.ctypes.data, int(L.bytes)) != 0:
                    raise RuntimeError(f"relayout failed for operand {operand}")
                if row.unrelayout:
                    back = np.zeros_like(src)
                    bt = rad.tensor(back.ctypes.data, dt, [rows_p, cols_p])
                    ok &= row.unrelayout(P, nP, operand, C.byref(enc), C.byref(sel), dst.ctypes.data, int(L.bytes),
                                         C.byref(bt), 1) == 0 and np.array_equal(back, src)
            report["unrelayout_ok"] &= ok
            report["layouts"].append((operand, L.tag.decode() if L.tag else "?"))
            base = mem.put(stored)
            ptrs = np.array([base + j * stored_b for j in range(n_ent)], np.uint64)
            tab = mem.put(ptrs.view(np.uint8))
            return rad.tensor(tab, int(L.dtype), shape, [0] + rad_dense(shape)[1:])
        data = np.concatenate(blobs) if blobs else np.zeros(0, np.uint8)
        base = mem.put(data)
        if self.table_form == "stacked":
            st = rad_dense(shape)
            return rad.tensor(base, dt, shape, st)
        ptrs = np.array([base + j * ent_b for j in range(n_ent)], np.uint64)
        tab = mem.put(ptrs.view(np.uint8))
        return rad.tensor(tab, dt, shape, [0] + rad_dense(shape)[1:])


def rad_dense(shape):
    st, s = [0] * len(shape), 1
    for r in range(len(shape) - 1, -1, -1):
        st[r] = s
        s *= shape[r]
    return st


def bf16_bits(x):
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)


def bits_to_f32(bits, dtype):
    b = np.asarray(bits, np.uint16)
    if dtype == "bf16":
        return (b.astype(np.uint32) << 16).view(np.float32)
    return b.view(np.float16).astype(np.float32)


def encoding(bits, codebook, stacked):
    """The canonical exl3 encoding of a K-bit weight (include/exl3_encoding.h:84-98)."""
    e = rad.RadEncoding()
    e.scheme = b"exl3"
    e.transform = f"{codebook}/h128".encode()
    planes = [("codes", rad.DT_UK[bits], 1, 1), ("suh", 2, 0, 1), ("svh", 2, 1, 0)]
    if stacked:
        planes.append(("suh.1", 2, 0, 1))
    e.n_planes = len(planes)
    for i, (n, dt, r, c) in enumerate(planes):
        e.plane[i].name = n.encode()
        e.plane[i].dtype = dt
        e.plane[i].tile_r = r
        e.plane[i].tile_c = c
    return e


# ------------------------------------------------------------------------------------------ memory
class HostMem:
    """Host buffers between poisoned margins (the reference library is a host row)."""

    def __init__(self):
        self.bufs = {}

    def alloc(self, nbytes, fill):
        b = np.full(nbytes + 2 * RED, RED_FILL, np.uint8)
        b[RED:RED + nbytes] = fill
        ptr = b.ctypes.data + RED
        self.bufs[ptr] = (b, nbytes)
        return ptr

    def put(self, arr):
        a = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
        ptr = self.alloc(a.size, 0)
        self.bufs[ptr][0][RED:RED + a.size] = a
        return ptr

    def get(self, ptr, nbytes):
        b, n = self.bufs[ptr]
        return b[RED:RED + nbytes].copy()

    def sync(self):
        pass

    def redzones_ok(self):
        return all((b[:RED] == RED_FILL).all() and (b[RED + n:] == RED_FILL).all() for b, n in self.bufs.values())

    def free(self):
        self.bufs.clear()


class DeviceMem:
    """Device buffers (torch, as plumbing) between poisoned margins."""

    def __init__(self):
        import torch
        self.torch = torch
        self.bufs = {}

    def alloc(self, nbytes, fill):
        t = self.torch
        b = t.full((nbytes + 2 * RED,), RED_FILL, dtype=t.uint8, device="cuda")
        if nbytes:
            b[RED:RED + nbytes] = fill
        ptr = b.data_ptr() + RED
        self.bufs[ptr] = (b, nbytes)
        return ptr

    def put(self, arr):
        a = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
        ptr = self.alloc(a.size, 0)
        if a.size:
            self.bufs[ptr][0][RED:RED + a.size].copy_(self.torch.from_numpy(a.copy()))
        return ptr

    def get(self, ptr, nbytes):
        b, n = self.bufs[ptr]
        return b[RED:RED + nbytes].cpu().numpy()

    def sync(self):
        self.torch.cuda.synchronize()

    def redzones_ok(self):
        ok = True
        for b, n in self.bufs.values():
            h = b.cpu().numpy()
            ok &= bool((h[:RED] == RED_FILL).all() and (h[RED + n:] == RED_FILL).all())
        return ok

    def free(self):
        self.bufs.clear()
