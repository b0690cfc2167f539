"""oracle_bind.py -- TEST INFRASTRUCTURE: ctypes bindings of the two CPU checkers under oracle/.

  Oracle   oracle/liboracle.so        this repository's C restatement of the reference algorithm
  REF_LIB  oracle/_ref/libexl3ref.so  the reference's kernels/exl3ref + common/ built unmodified (a host plugin)

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use these; the product never does."""
import ctypes as C
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent.parent
ORACLE_SO = REPO / "oracle" / "liboracle.so"
REF_SO = REPO / "oracle" / "_ref" / "libexl3ref.so"
CB = {"3inst": 0, "mcg": 1, "mul1": 2}


class OrcOp(C.Structure):
    _fields_ = [("op", C.c_int), ("bits", C.c_int), ("codebook", C.c_int), ("h_rot", C.c_int), ("a_rot", C.c_int),
                ("T", C.c_int64), ("n_expert", C.c_int64), ("top_k", C.c_int64), ("n_class", C.c_int64),
                ("rows", C.c_int64 * 4), ("cols", C.c_int64 * 4), ("x_cols", C.c_int64), ("y_cols", C.c_int64),
                ("x", C.c_void_p), ("x_dtype", C.c_int), ("x_rows", C.c_int64), ("x_pitch", C.c_int64),
                ("y", C.c_void_p), ("y_pitch", C.c_int64), ("sorted_tok", C.c_void_p), ("expert_offset", C.c_void_p),
                ("codes", C.POINTER(C.c_void_p)), ("suh", C.POINTER(C.c_void_p)), ("suh1", C.POINTER(C.c_void_p)),
                ("svh", C.POINTER(C.c_void_p)), ("dn_suh", C.POINTER(C.c_void_p)), ("n_threads", C.c_int),
                ("out_f16", C.c_int)]


class Oracle:
    def __init__(self, path=ORACLE_SO):
        if not Path(path).exists():
            raise FileNotFoundError(f"{path} not built: make -C oracle")
        L = self.lib = C.CDLL(str(path))
        L.orc_codebook_value.restype = C.c_uint16
        L.orc_codebook_value.argtypes = [C.c_uint32, C.c_int]
        for f in ("orc_trellis_decode", "orc_record_decode"):
            getattr(L, f).argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int, C.c_int, C.c_void_p]
        L.orc_codes_to_record.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_int, C.c_void_p]
        L.orc_record_to_codes.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int, C.c_void_p, C.c_int64]
        L.orc_had128.argtypes = [C.c_void_p, C.c_int64]
        L.orc_moe_op.argtypes = [C.POINTER(OrcOp)]
        L.orc_moe_scatter.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p]
        L.orc_moe_gather.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_int64,
                                     C.c_int64, C.c_void_p]

    def codebook_table(self, cb):
        return np.array([self.lib.orc_codebook_value(s, CB[cb]) for s in range(65536)], np.uint16)

    def trellis_decode(self, trellis, bits, cb):
        kt, nt = trellis.shape[:2]
        out = np.zeros((kt * 16, nt * 16), np.uint16)
        t = np.ascontiguousarray(trellis, np.int16)
        assert self.lib.orc_trellis_decode(t.ctypes.data, kt, nt, bits, CB[cb], out.ctypes.data) == 0
        return out

    def record_decode(self, record, rows, cols, bits, cb):
        out = np.zeros((rows, cols), np.uint16)
        r = np.ascontiguousarray(record).view(np.uint16)
        assert self.lib.orc_record_decode(r.ctypes.data, rows, cols, bits, CB[cb], out.ctypes.data) == 0
        return out

    def codes_to_record(self, codes, rows, cols, bits):
        rec = np.zeros(rows * cols * bits // 16, np.uint16)
        c = np.ascontiguousarray(codes, np.uint8)
        rb = (cols * bits + 7) // 8
        assert self.lib.orc_codes_to_record(c.ctypes.data, rb, rows, cols, bits, rec.ctypes.data) == 0
        return rec

    def record_to_codes(self, record, rows, cols, bits):
        rb = (cols * bits + 7) // 8
        codes = np.zeros((rows, rb), np.uint8)
        r = np.ascontiguousarray(record, np.uint16)
        assert self.lib.orc_record_to_codes(r.ctypes.data, rows, cols, bits, codes.ctypes.data, rb) == 0
        return codes

    def had128(self, v):
        x = np.array(v, np.float32, copy=True)
        assert self.lib.orc_had128(x.ctypes.data, x.size) == 0
        return x

    def scatter(self, ids, n_expert, base=0):
        flat = np.ascontiguousarray(np.asarray(ids, np.int32).reshape(-1))
        st = np.zeros(flat.size, np.int32)
        off = np.zeros(n_expert + 1, np.int32)
        assert self.lib.orc_moe_scatter(flat.ctypes.data, flat.size, n_expert, base, st.ctypes.data,
                                        off.ctypes.data) == 0
        return st, off

    def gather(self, rows_bf16, sorted_tok, w, n_tok, top_k, width):
        r = np.ascontiguousarray(rows_bf16, np.uint16)
        st = np.ascontiguousarray(sorted_tok, np.int32)
        ww = np.ascontiguousarray(w, np.float32)
        y = np.zeros((n_tok, width), np.float32)
        assert self.lib.orc_moe_gather(r.ctypes.data, r.shape[1], st.ctypes.data, st.size, ww.ctypes.data, n_tok,
                                       top_k, width, y.ctypes.data) == 0
        return y

    def run_case(self, case, n_threads=1, prefill=None):
        """The restatement of case.op on case's planes: returns the output bits [T, y_cols] (uint16). For
        gate_up_down, the pair gate_up(a_rot 0, h_rot 1) -> down(h_rot 1) it is defined as."""
        base = case.base
        if base == "moe_exl3_gate_up_down":
            h = self._run(case, 1, 1, 0, case.x, case.geom, "gu", n_threads)
            dgeom = [(c, r // 2) for r, c in case.geom]
            return self._run(case, 0, 1, 0, h, dgeom, "dn_of_gd", n_threads)
        op = {"moe_exl3_down": 0, "moe_exl3_gate_up": 1, "moe_exl3_prep_gu": 2}[base]
        return self._run(case, op, case.h_rot, case.a_rot, case.x, case.geom, "own", n_threads, prefill)

    def _run(self, case, op, h_rot, a_rot, x, geom, which, n_threads, prefill=None, out_f16=False):
        o = OrcOp()
        o.out_f16 = 1 if out_f16 else 0
        o.op, o.bits, o.codebook, o.h_rot, o.a_rot = op, case.bits, CB.get(case.codebook, 0), h_rot, a_rot
        o.T, o.n_expert, o.top_k, o.n_class = case.T, case.n_expert, case.top_k, case.n_class
        for c in range(4):
            r, cc = geom[c % len(geom)]
            o.rows[c], o.cols[c] = r, cc
        o.x_cols = max(c for _, c in geom)
        if op == 2:
            o.y_cols = 2 * o.x_cols
        else:
            o.y_cols = max(r for r, _ in geom) // (2 if op == 1 else 1)
        xx = np.ascontiguousarray(x, np.uint16)
        o.x, o.x_rows, o.x_pitch = xx.ctypes.data, xx.shape[0], xx.shape[1]
        token_rows = op == 2 or (op == 1 and not a_rot)
        o.x_dtype = 1 if (token_rows and case.x_dtype == "bf16" and which != "dn_of_gd") else 0
        y = np.full((case.T, o.y_cols), 0xFFFF if op == 2 else 0, np.uint16) if prefill is None else prefill.copy()
        o.y, o.y_pitch = y.ctypes.data, o.y_cols
        st = np.ascontiguousarray(case.sorted_tok)
        off = np.ascontiguousarray(case.expert_offset)
        o.sorted_tok, o.expert_offset = st.ctypes.data, off.ctypes.data
        keep = []

        def arr(key):
            ptrs = (C.c_void_p * max(1, case.n_expert))()
            for e, p in enumerate(case.planes):
                if key in p:
                    a = np.ascontiguousarray(p[key])
                    keep.append(a)
                    ptrs[e] = a.ctypes.data
            keep.append(ptrs)
            return ptrs

        if which == "dn_of_gd":
            o.codes, o.suh, o.svh = arr("dn_codes"), arr("dn_suh"), arr("dn_svh")
            o.suh1, o.dn_suh = arr("suh1"), arr("dn_suh")
        else:
            o.codes, o.suh, o.suh1, o.svh, o.dn_suh = arr("codes"), arr("suh"), arr("suh1"), arr("svh"), arr("dn_suh")
        o.n_threads = n_threads
        rc = self.lib.orc_moe_op(C.byref(o))
        if rc != 0:
            raise RuntimeError(f"orc_moe_op: {rc}")
        return y


class RefLib:
    """The reference's common/ functions out of oracle/_ref/libexl3ref.so (built from the reference sources)."""

    def __init__(self, path=REF_SO):
        if not Path(path).exists():
            raise FileNotFoundError(f"{path} not built (make -C oracle ref, needs the reference tree)")
        L = self.lib = C.CDLL(str(path))
        L.exl3_codebook_value.restype = C.c_uint16
        L.exl3_codebook_value.argtypes = [C.c_uint32, C.c_int]
        L.exl3_trellis_decode.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int, C.c_int, C.c_void_p]
        L.exl3_codes_to_record.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_int, C.c_void_p]
        L.exl3_had128.argtypes = [C.c_void_p, C.c_int64]

    def codebook_value(self, s, cb):
        return self.lib.exl3_codebook_value(s, CB[cb])

    def trellis_decode(self, trellis, bits, cb):
        kt, nt = trellis.shape[:2]
        out = np.zeros((kt * 16, nt * 16), np.uint16)
        t = np.ascontiguousarray(trellis, np.int16)
        assert self.lib.exl3_trellis_decode(t.ctypes.data, kt, nt, bits, CB[cb], out.ctypes.data) == 0
        return out

    def codes_to_record(self, codes, rows, cols, bits):
        rec = np.zeros(rows * cols * bits // 16, np.uint16)
        c = np.ascontiguousarray(codes, np.uint8)
        assert self.lib.exl3_codes_to_record(c.ctypes.data, (cols * bits + 7) // 8, rows, cols, bits,
                                             rec.ctypes.data) == 0
        return rec

    def had128(self, v):
        x = np.array(v, np.float32, copy=True)
        assert self.lib.exl3_had128(x.ctypes.data, x.size) == 0
        return x


def compare(got_bits, want_bits, dtype, rel_tol=1e-2, cos_tol=0.9999):
    """The expert-output tolerance (fp32 accumulation in another order): max |got - want| / max |want| <= rel_tol
    and cosine >= cos_tol over all elements; zeros where the reference has zeros, exactly; no NaN."""
    from exl3b200.cases import bits_to_f32
    g = bits_to_f32(got_bits, dtype).astype(np.float64)
    w = bits_to_f32(want_bits, dtype).astype(np.float64)
    if np.isnan(g).any():
        return False, "NaN in output (a row left unwritten)"
    zero_w = (w == 0).all(axis=-1)
    if not (g[zero_w] == 0).all():
        return False, "a zero row of the reference is not zero"
    scale = np.abs(w).max() if w.size else 0.0
    if scale == 0:
        return bool((g == 0).all()), "all zero"
    rel = np.abs(g - w).max() / scale
    cos = float((g * w).sum() / (np.linalg.norm(g) * np.linalg.norm(w) + 1e-300))
    return bool(rel <= rel_tol and cos >= cos_tol), f"max rel err {rel:.3e}, cosine {cos:.7f}"
