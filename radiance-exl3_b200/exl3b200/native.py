"""native.py -- ctypes bindings of libexl3b200.so's direct entry points (include/exl3b200.h, part 2).

Device buffers are passed as integer addresses (a torch tensor's data_ptr(), torch being plumbing here);
`stream` is a cudaStream_t as an integer (0 = the legacy default stream)."""
import ctypes as C

from . import library_path

_I64, _VP, _I = C.c_int64, C.c_void_p, C.c_int


class Native:
    def __init__(self, path=None):
        L = self.lib = C.CDLL(str(path or library_path()))
        L.exl3b200_decode_what.argtypes = [_VP, _I64, _I64, _I, _I, _VP, _VP]
        L.exl3b200_codes_to_record.argtypes = [_VP, _I64, _I64, _I64, _I, _VP]
        L.exl3b200_record_to_codes.argtypes = [_VP, _I64, _I64, _I, _VP, _I64]
        L.exl3b200_router_topk.argtypes = [_VP, _I64, _I64, _I64, _VP, _VP, _VP]
        L.exl3b200_moe_scatter_work_bytes.restype = _I64
        L.exl3b200_moe_scatter_work_bytes.argtypes = [_I64, _I64]
        L.exl3b200_moe_scatter.argtypes = [_VP, _I64, _I64, _I64, _VP, _VP, _VP, _VP]
        L.exl3b200_moe_gather_work_bytes.restype = _I64
        L.exl3b200_moe_gather_work_bytes.argtypes = [_I64, _I64]
        L.exl3b200_moe_gather.argtypes = [_VP, _I64, _VP, _I64, _VP, _I64, _I64, _I64, _VP, _VP, _VP]
        L.exl3b200_read_error.argtypes = [_I, C.POINTER(C.c_int32)]
        L.exl3b200_ep_pack.argtypes = [_VP, _I64, _VP, _I64, _VP, _I64, _VP, _I64, _I64, _I64, _VP, _VP, _VP, _VP]
        L.exl3b200_rows_scatter.argtypes = [_VP, _I64, _VP, _I64, _I64, _VP, _I64, _I64, _VP]
        L.exl3b200_ep_dest.argtypes = [_VP, _I64, _I64, _I64, _VP, _VP]
        L.exl3b200_ep_pack_dedup.argtypes = [_VP, _I64, _VP, _I64, _VP, _VP, _I64, _I64, _I64, _I64, _VP, _VP, _VP, _VP, _VP]
        L.exl3b200_ep_unpack.argtypes = [_VP, _I64, _VP, _I64, _VP, _VP, _VP]
        L.exl3b200_ep_map.argtypes = [_VP, _I64, _VP, _I64, _VP, _VP]

    @staticmethod
    def _check(rc, what):
        if rc != 0:
            raise RuntimeError(f"{what}: status {rc}")

    def decode_what(self, record_ptr, rows, cols, bits, codebook, out_ptr, stream=0):
        self._check(self.lib.exl3b200_decode_what(record_ptr, rows, cols, bits, codebook, out_ptr, stream),
                    "exl3b200_decode_what")

    def codes_to_record(self, codes_ptr, row_bytes, rows, cols, bits, record_ptr):
        self._check(self.lib.exl3b200_codes_to_record(codes_ptr, row_bytes, rows, cols, bits, record_ptr),
                    "exl3b200_codes_to_record")

    def record_to_codes(self, record_ptr, rows, cols, bits, codes_ptr, row_bytes):
        self._check(self.lib.exl3b200_record_to_codes(record_ptr, rows, cols, bits, codes_ptr, row_bytes),
                    "exl3b200_record_to_codes")

    def router_topk(self, logits, n_tok, n_expert, top_k, ids, w, stream=0):
        self._check(self.lib.exl3b200_router_topk(logits, n_tok, n_expert, top_k, ids, w, stream),
                    "exl3b200_router_topk")

    def scatter_work_bytes(self, n_pairs, n_expert):
        return int(self.lib.exl3b200_moe_scatter_work_bytes(n_pairs, n_expert))

    def moe_scatter(self, ids, n_pairs, n_expert, expert_base, sorted_tok, expert_offset, work, stream=0):
        self._check(self.lib.exl3b200_moe_scatter(ids, n_pairs, n_expert, expert_base, sorted_tok, expert_offset,
                                                  work, stream), "exl3b200_moe_scatter")

    def gather_work_bytes(self, n_tok, top_k):
        return int(self.lib.exl3b200_moe_gather_work_bytes(n_tok, top_k))

    def moe_gather(self, rows, row_pitch, sorted_tok, n_rows, w, n_tok, top_k, width, y, work, stream=0):
        self._check(self.lib.exl3b200_moe_gather(rows, row_pitch, sorted_tok, n_rows, w, n_tok, top_k, width, y,
                                                 work, stream), "exl3b200_moe_gather")

    def read_error(self, clear=True):
        v = C.c_int32(0)
        self._check(self.lib.exl3b200_read_error(1 if clear else 0, C.byref(v)), "exl3b200_read_error")
        return v.value

    # ------------------------------------------------------------------ expert parallelism
    def ep_pack(self, x, x_pitch, ids, top_k, sorted_pairs, n_pairs, expert_offset, n_local, world, hidden, send_x,
                send_e, send_counts, stream=0):
        self._check(self.lib.exl3b200_ep_pack(x, x_pitch, ids, top_k, sorted_pairs, n_pairs, expert_offset, n_local,
                                              world, hidden, send_x, send_e, send_counts, stream), "exl3b200_ep_pack")

    def rows_scatter(self, src, src_pitch, idx, n_rows, row_bytes, dst, dst_pitch, n_dst, stream=0):
        self._check(self.lib.exl3b200_rows_scatter(src, src_pitch, idx, n_rows, row_bytes, dst, dst_pitch, n_dst,
                                                   stream), "exl3b200_rows_scatter")

    def ep_dest(self, ids, n_pairs, n_local, world, dest, stream=0):
        self._check(self.lib.exl3b200_ep_dest(ids, n_pairs, n_local, world, dest, stream), "exl3b200_ep_dest")

    def ep_pack_dedup(self, x, x_pitch, ids, top_k, sorted_pairs, dest_off, n_pairs, n_local, world, hidden,
                      send_x, send_meta, row_tok, counts, stream=0):
        self._check(self.lib.exl3b200_ep_pack_dedup(x, x_pitch, ids, top_k, sorted_pairs, dest_off, n_pairs, n_local,
                                                    world, hidden, send_x, send_meta, row_tok, counts, stream),
                    "exl3b200_ep_pack_dedup")

    def ep_unpack(self, meta, n_pairs, recv_counts, world, expert, row, stream=0):
        self._check(self.lib.exl3b200_ep_unpack(meta, n_pairs, recv_counts, world, expert, row, stream),
                    "exl3b200_ep_unpack")

    def ep_map(self, idx, n, table, n_table, out, stream=0):
        self._check(self.lib.exl3b200_ep_map(idx, n, table, n_table, out, stream), "exl3b200_ep_map")
