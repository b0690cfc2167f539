"""rad.py -- the radiance kernel-plugin ABI (ABI 17) as ctypes records, and a loader that drives a plugin the way
the engine does: dlopen, the schema and row tables, the shape, scratch and layout hooks, and a row's launch.

The records mirror include/rad_abi.h, include/rad_types.h, include/rad_encoding.h and include/rad_plugin.h field
for field. Any plugin built against those headers can be driven: this repository's libexl3b200.so (device rows)
and the reference's kernels/exl3ref library (host rows). This is the harness role tests/ref/exl3ref_run.cpp plays
in the reference (dlopen, rad_kernel_at, opd_shape, layout/relayout/unrelayout, scratch, launch).
"""
import ctypes as C

MAX_RANK = 6
ENC_STR = 32
ENC_MAX_PLANES = 8

# element types (include/rad_types.h)
DT = {"f32": 1, "f16": 2, "bf16": 3, "u8": 9, "i32": 11, "u4": 19, "u2": 20, "u1": 22, "u3": 24, "u5": 26,
      "u6": 28, "u7": 30}
DT_UK = {1: 22, 2: 20, 3: 24, 4: 19, 5: 26, 6: 28, 7: 30, 8: 9}
DT_BITS = {1: 32, 2: 16, 3: 16, 9: 8, 11: 32, 19: 4, 20: 2, 22: 1, 24: 3, 26: 5, 28: 6, 30: 7}

# status codes
RAD = {"OK": 0, "SHAPE": -1, "DTYPE": -2, "ALIGN": -3, "STRIDE": -4, "SCRATCH": -5, "DEVICE": -6, "NOMEM": -7,
       "FORMAT": -8, "SCHEMA": -9, "UNSUPPORTED": -10, "INVAL": -12}

P_INT, P_STR = 1, 2
OPD_IN, OPD_OUT, OPD_WTAB = 1, 2, 3
OPD_F_ABSENT, OPD_F_IDX_CU = 1, 4
DOMAIN_HOST, DOMAIN_DEVICE = 1, 2
C_IN, C_EQ, C_LE, C_GE, C_DIV = 1, 2, 3, 4, 5


class RadTensor(C.Structure):
    _fields_ = [("data", C.c_void_p), ("dtype", C.c_uint32), ("rank", C.c_uint32),
                ("shape", C.c_int64 * MAX_RANK), ("stride", C.c_int64 * MAX_RANK)]


class RadParam(C.Structure):
    _fields_ = [("key", C.c_char_p), ("kind", C.c_int32), ("ival", C.c_int64), ("ihi", C.c_int64),
                ("sval", C.c_char_p), ("dval", C.c_double)]


class RadArgs(C.Structure):
    _fields_ = [("t", C.POINTER(RadTensor)), ("n_t", C.c_int), ("p", C.POINTER(RadParam)), ("n_p", C.c_int),
                ("scratch", C.c_void_p), ("scratch_bytes", C.c_int64), ("instance", C.c_void_p),
                ("rank", C.c_int), ("world_size", C.c_int)]


class RadParamSpec(C.Structure):
    _fields_ = [("key", C.c_char_p), ("type", C.c_int32), ("required", C.c_int32), ("role", C.c_int32)]


class RadOperandSpec(C.Structure):
    _fields_ = [("name", C.c_char_p), ("role", C.c_int32), ("optional", C.c_int32)]


class RadOpSchema(C.Structure):
    _fields_ = [("op", C.c_char_p), ("params", C.POINTER(RadParamSpec)), ("n_params", C.c_int),
                ("operands", C.POINTER(RadOperandSpec)), ("n_operands", C.c_int), ("doc", C.c_char_p)]


class RadOpdDesc(C.Structure):
    _fields_ = [("dtype", C.c_uint32), ("rank", C.c_uint32), ("shape", C.c_int64 * MAX_RANK),
                ("flags", C.c_uint32), ("fill", C.c_uint32), ("idx_max", C.c_int64), ("idx_const", C.c_int64)]


class RadConstraint(C.Structure):
    _fields_ = [("key", C.c_char_p), ("op", C.c_int32), ("ival", C.c_int64), ("sval", C.c_char_p)]


class RadEncPlane(C.Structure):
    _fields_ = [("name", C.c_char * ENC_STR), ("dtype", C.c_uint32), ("tile_r", C.c_int32), ("tile_c", C.c_int32)]


class RadEncoding(C.Structure):
    _fields_ = [("scheme", C.c_char * ENC_STR), ("transform", C.c_char * ENC_STR), ("n_planes", C.c_int32),
                ("plane", RadEncPlane * ENC_MAX_PLANES)]


class RadLayout(C.Structure):
    _fields_ = [("dtype", C.c_uint32), ("bytes", C.c_int64), ("align", C.c_int64), ("tag", C.c_char_p)]


LAUNCH = C.CFUNCTYPE(C.c_int, C.POINTER(RadArgs), C.c_void_p)
OPD_SHAPE = C.CFUNCTYPE(C.c_int, C.POINTER(RadParam), C.c_int, C.c_int, C.POINTER(RadOpdDesc))
SCRATCH = C.CFUNCTYPE(C.c_int64, C.POINTER(RadArgs))
INIT = C.CFUNCTYPE(C.c_int, C.POINTER(RadParam), C.c_int, C.c_int, C.c_int, C.POINTER(C.c_void_p))
FINI = C.CFUNCTYPE(None, C.c_void_p)
LAYOUT = C.CFUNCTYPE(C.c_int, C.POINTER(RadParam), C.c_int, C.c_int, C.POINTER(RadEncoding), C.POINTER(C.c_int),
                     C.POINTER(RadTensor), C.c_int, C.POINTER(RadLayout))
RELAYOUT = C.CFUNCTYPE(C.c_int, C.POINTER(RadParam), C.c_int, C.c_int, C.POINTER(RadEncoding), C.POINTER(C.c_int),
                       C.POINTER(RadTensor), C.c_int, C.c_void_p, C.c_int64)
UNRELAYOUT = C.CFUNCTYPE(C.c_int, C.POINTER(RadParam), C.c_int, C.c_int, C.POINTER(RadEncoding), C.POINTER(C.c_int),
                         C.c_void_p, C.c_int64, C.POINTER(RadTensor), C.c_int)


class RadKernelInfo(C.Structure):
    _fields_ = [("name", C.c_char_p), ("op", C.c_char_p), ("family", C.c_char_p), ("computes", C.c_char_p),
                ("shape", C.c_char_p), ("dtypes", C.c_char_p), ("domain", C.c_int32), ("priority", C.c_int32),
                ("constraints", C.POINTER(RadConstraint)), ("n_constraints", C.c_int),
                ("launch", LAUNCH), ("opd_shape", OPD_SHAPE), ("scratch", SCRATCH), ("init", INIT), ("fini", FINI),
                ("layout", LAYOUT), ("relayout", RELAYOUT), ("unrelayout", UNRELAYOUT)]


class RadPluginInfo(C.Structure):
    _fields_ = [("kind", C.c_int32), ("name", C.c_char_p), ("version", C.c_char_p), ("description", C.c_char_p),
                ("target", C.c_char_p)]


ABI_VERSION = 17


def make_params(params):
    """{key: int | str | (lo, hi)} -> (RadParam array, keepalive). A (lo, hi) tuple is a ranged integer (the op's M)."""
    arr = (RadParam * max(1, len(params)))()
    keep = []
    for i, (k, v) in enumerate(params.items()):
        kb = k.encode()
        keep.append(kb)
        arr[i].key = kb
        if isinstance(v, str):
            sb = v.encode()
            keep.append(sb)
            arr[i].kind, arr[i].sval = P_STR, sb
        elif isinstance(v, tuple):
            arr[i].kind, arr[i].ival, arr[i].ihi = P_INT, int(v[0]), int(v[1])
        else:
            arr[i].kind, arr[i].ival = P_INT, int(v)
    return arr, len(params), keep


def tensor(ptr, dtype, shape, stride=None):
    """A RadTensor over `ptr` (an int address, 0 = absent) with `shape`; dense strides unless given."""
    t = RadTensor()
    t.data = ptr or None
    t.dtype = dtype
    t.rank = len(shape)
    s = 1
    dense = [0] * len(shape)
    for r in range(len(shape) - 1, -1, -1):
        dense[r] = s
        s *= shape[r]
    for r, n in enumerate(shape):
        t.shape[r] = int(n)
        t.stride[r] = int(stride[r]) if stride is not None else dense[r]
    return t


class Plugin:
    """A kernel plugin loaded as the engine loads it."""

    def __init__(self, path):
        self.path = str(path)
        self.lib = C.CDLL(self.path, mode=C.RTLD_LOCAL)
        L = self.lib
        L.rad_plugin_abi_version.restype = C.c_uint32
        L.rad_plugin_info.restype = C.POINTER(RadPluginInfo)
        L.rad_kernel_schema_count.restype = C.c_int
        L.rad_kernel_schema_at.restype = C.POINTER(RadOpSchema)
        L.rad_kernel_schema_at.argtypes = [C.c_int]
        L.rad_kernel_count.restype = C.c_int
        L.rad_kernel_at.restype = C.POINTER(RadKernelInfo)
        L.rad_kernel_at.argtypes = [C.c_int]
        if L.rad_plugin_abi_version() != ABI_VERSION:
            raise RuntimeError(f"{self.path}: plugin ABI {L.rad_plugin_abi_version()}, expected {ABI_VERSION}")

    @property
    def info(self):
        i = self.lib.rad_plugin_info().contents
        return {"kind": i.kind, "name": i.name.decode(), "version": i.version.decode(),
                "description": i.description.decode(), "target": i.target.decode()}

    def schemas(self):
        out = []
        for i in range(self.lib.rad_kernel_schema_count()):
            s = self.lib.rad_kernel_schema_at(i).contents
            out.append({
                "op": s.op.decode(), "doc": s.doc.decode(),
                "params": [(s.params[k].key.decode(), s.params[k].type, s.params[k].required, s.params[k].role)
                           for k in range(s.n_params)],
                "operands": [(s.operands[k].name.decode(), s.operands[k].role, s.operands[k].optional)
                             for k in range(s.n_operands)],
            })
        return out

    def rows(self):
        return [self.lib.rad_kernel_at(i).contents for i in range(self.lib.rad_kernel_count())]

    def row(self, op, domain=None):
        for r in self.rows():
            if r.op.decode() == op and (domain is None or r.domain == domain):
                return r
        return None


def constraint_holds(c, params):
    """Selection's reading of one constraint (tests/ref/exl3ref_run.cpp:150-172): an absent key never holds."""
    key = c.key.decode()
    if key.startswith("device."):
        return True
    if key not in params:
        return False
    v = params[key]
    if c.op == C_IN:
        want = v if isinstance(v, str) else str(v[1] if isinstance(v, tuple) else v)
        return want in c.sval.decode().split()
    if isinstance(v, str):
        return False
    iv = v[1] if isinstance(v, tuple) else v
    return {C_EQ: iv == c.ival, C_LE: iv <= c.ival, C_GE: iv >= c.ival,
            C_DIV: c.ival != 0 and iv % c.ival == 0}.get(c.op, False)
