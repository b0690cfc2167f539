"""native.py -- ctypes bindings of libexl3b200.so's direct entry points (include/exl3b200.h, part 2).

Device buffers are passed as integer addresses (a torch tensor's data_ptr(), torch being plumbing here);
`stream` is a cudaStream_t as an integer (0 = the legacy default stream)."""
import ctypes as C

from . import library_path

_I64, _VP, _I = C.c_int64, C.c_void_p, C.c_int


class LayerDesc(C.Structure):
    """Exl3bLayerDesc (include/exl3b200.h)."""
    _fields_ = [("n_expert", _I64), ("n_local", _I64), ("expert_base", _I64), ("hidden", _I64), ("width", _I64),
                ("top_k", _I64), ("bits_gu", C.c_int32), ("bits_dn", C.c_int32), ("codebook", C.c_int32),
                ("pad0", C.c_int32), ("gu_codes", _VP), ("dn_codes", _VP), ("suh", _VP), ("suh1", _VP),
                ("svh_gu", _VP), ("dn_suh", _VP), ("svh_dn", _VP)]


class LayerBufs(C.Structure):
    """Exl3bLayerBufs (include/exl3b200.h): device addresses inside the caller's work block."""
    _fields_ = [("max_tokens", _I64), ("ids", _VP), ("w", _VP), ("sorted_tok", _VP), ("expert_offset", _VP),
                ("scatter_work", _VP), ("h", _VP), ("y_rows", _VP), ("gu_scratch", _VP), ("gu_scratch_bytes", _I64),
                ("dn_scratch", _VP), ("dn_scratch_bytes", _I64), ("gather_work", _VP)]


class BlockDesc(C.Structure):
    """Exl3bBlockDesc (include/exl3b200.h)."""
    _fields_ = [("routed", LayerDesc), ("shared", LayerDesc), ("sgate_w", _VP)]


class BlockBufs(C.Structure):
    """Exl3bBlockBufs (include/exl3b200.h)."""
    _fields_ = [("routed", LayerBufs), ("shared", LayerBufs)]


class EpDesc(C.Structure):
    """Exl3bEpDesc (include/exl3b200.h)."""
    _fields_ = [("layer", LayerDesc), ("rank", _I64), ("world", _I64), ("max_tokens", _I64),
                ("fuse_combine", C.c_int32), ("pad0", C.c_int32), ("window", _VP), ("peers", _VP),
                ("offs", _I64 * 6), ("epoch", _VP), ("status", _VP)]


class EpBufs(C.Structure):
    """Exl3bEpBufs (include/exl3b200.h): device addresses inside the caller's work block."""
    _fields_ = [("max_tokens", _I64), ("cap", _I64)] + [(n, _VP) for n in (
        "ids", "w", "dest", "sorted_pairs", "row_tok", "send_meta", "dest_off", "counts", "hdr", "pair_e", "pair_row",
        "dst_rank", "dst_pos", "sorted_pair", "sorted_row", "expert_offset", "row_dst", "h", "y_rows", "scatter_rank",
        "scatter_local", "gu_scratch")] + [("gu_scratch_bytes", _I64), ("dn_scratch", _VP),
                                           ("dn_scratch_bytes", _I64), ("gather_work", _VP)]


class TpDesc(C.Structure):
    """Exl3bTpDesc (include/exl3b200.h)."""
    _fields_ = [("layer", LayerDesc), ("rank", _I64), ("world", _I64), ("max_tokens", _I64), ("window", _VP),
                ("peers", _VP), ("offs", _I64 * 4), ("epoch", _VP), ("status", _VP)]


def marks_array(events):
    """A C array of cudaEvent_t from torch.cuda.Event objects (None entries stay NULL), or None. torch creates an
    event's handle at its first record, so each is recorded once here before its handle is taken."""
    if not events:
        return None
    arr = (_VP * len(events))()
    for i, e in enumerate(events):
        if e is not None:
            if not e.cuda_event:
                e.record()
            arr[i] = e.cuda_event
    return arr


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
        L.exl3b200_router_scatter.argtypes = [_VP, _I64, _I64, _I64, _VP, _VP, _I64, _I64, _VP, _VP, _VP, _VP]
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
        L.exl3b200_ep_dedup_scan.argtypes = [_VP, _I64, _VP, _VP, _I64, _I64, _I64, _VP, _VP, _VP, _VP]
        L.exl3b200_ep_window_alloc.argtypes = [_I64, C.POINTER(_VP)]
        L.exl3b200_ep_window_free.argtypes = [_VP]
        L.exl3b200_ep_window_handle.argtypes = [_VP, _VP]
        L.exl3b200_ep_window_open.argtypes = [_VP, C.POINTER(_VP)]
        L.exl3b200_ep_window_close.argtypes = [_VP]
        _U32 = C.c_uint32
        L.exl3b200_p2p_dispatch.argtypes = [_VP, _I64, _VP, _VP, _VP, _VP, _I64, _VP, _VP, _I64, _I64, _I64, _I64,
                                            _I64, _VP, _VP]
        L.exl3b200_p2p_wait_dispatch.argtypes = [_VP, _VP, _I64, _VP, _VP, _VP]
        L.exl3b200_p2p_unpack.argtypes = [_VP, _VP, _VP, _I64, _I64, _I64, _I64, _VP, _VP, _VP, _VP, _VP]
        L.exl3b200_p2p_combine.argtypes = [_VP, _I64, _VP, _I64, _VP, _VP, _VP, _VP, _I64, _I64, _I64, _I64, _VP, _VP]
        L.exl3b200_p2p_wait_combine.argtypes = [_VP, _VP, _I64, _VP, _VP, _VP]
        L.exl3b200_p2p_row_dst.argtypes = [_VP, _I64, _VP, _VP, _VP, _VP, _I64, _I64, _I64, _I64, _VP, _VP]
        L.exl3b200_p2p_signal_combine.argtypes = [_VP, _VP, _I64, _I64, _VP, _VP]
        L.exl3b200_moe_down_rows.argtypes = [_VP, _VP, _VP]
        L.exl3b200_moe_down_f16.argtypes = [_VP, _VP]
        L.exl3b200_moe_down_f16_scratch.restype = _I64
        L.exl3b200_moe_down_f16_scratch.argtypes = [_VP]
        L.exl3b200_moe_gather_bf16.argtypes = [_VP, _I64, _VP, _I64, _VP, _I64, _I64, _I64, _VP, _VP, _VP]
        L.exl3b200_moe_layer_work_bytes.restype = _I64
        L.exl3b200_moe_layer_work_bytes.argtypes = [C.POINTER(LayerDesc), _I64]
        L.exl3b200_moe_layer_carve.argtypes = [C.POINTER(LayerDesc), _I64, _VP, _I64, C.POINTER(LayerBufs)]
        L.exl3b200_moe_layer_forward.argtypes = [C.POINTER(LayerDesc), C.POINTER(LayerBufs), _VP, _VP, _I64, _VP,
                                                 C.c_int, _VP]
        L.exl3b200_set_peer_wait_ns.argtypes = [_I64]
        L.exl3b200_moe_block_work_bytes.restype = _I64
        L.exl3b200_moe_block_work_bytes.argtypes = [C.POINTER(BlockDesc), _I64]
        L.exl3b200_moe_block_carve.argtypes = [C.POINTER(BlockDesc), _I64, _VP, _I64, C.POINTER(BlockBufs)]
        L.exl3b200_moe_block_forward.argtypes = [C.POINTER(BlockDesc), C.POINTER(BlockBufs), _VP, _VP, _I64, _VP,
                                                 C.c_int, _VP]
        L.exl3b200_moe_gather_fold.argtypes = [_VP, _I64, _VP, _I64, _VP, _I64, _I64, _I64, _VP, _VP, _I64, _VP, _VP,
                                               C.c_int, _VP, _VP]
        L.exl3b200_identity_routing.argtypes = [_I64, _VP, _VP, _VP]
        L.exl3b200_ep_window_layout.restype = _I64
        L.exl3b200_ep_window_layout.argtypes = [_I64, _I64, _I64, _I64, C.POINTER(_I64)]
        L.exl3b200_tp_window_layout.restype = _I64
        L.exl3b200_tp_window_layout.argtypes = [_I64, _I64, _I64, C.POINTER(_I64)]
        L.exl3b200_ep_step_work_bytes.restype = _I64
        L.exl3b200_ep_step_work_bytes.argtypes = [C.POINTER(EpDesc)]
        L.exl3b200_ep_step_carve.argtypes = [C.POINTER(EpDesc), _VP, _I64, C.POINTER(EpBufs)]
        L.exl3b200_ep_step_forward.argtypes = [C.POINTER(EpDesc), C.POINTER(EpBufs), _VP, _VP, _I64, _VP, C.c_int,
                                               _VP, C.POINTER(_VP)]
        L.exl3b200_tp_step_forward.argtypes = [C.POINTER(TpDesc), C.POINTER(LayerBufs), _VP, _VP, _I64, _VP, _I64,
                                               _VP, C.POINTER(_VP)]
        L.exl3b200_p2p_begin.argtypes = [_VP, _VP]
        L.exl3b200_moe_op_live.argtypes = [_VP, _I, _VP, _VP]
        L.exl3b200_tp_gather_rs.argtypes = [_VP, _I64, _VP, _I64, _VP, _I64, _I64, _I64, _VP, _VP, _VP, _I64, _I64,
                                            _I64, _VP, _VP, _VP]
        L.exl3b200_tp_reduce.argtypes = [_VP, _VP, _I64, _I64, _I64, _I64, _I64, _VP, _VP]
        L.exl3b200_tp_pull.argtypes = [_VP, _VP, _I64, _I64, _I64, _I64, _I64, _VP, _I64, _VP, _VP, _VP]

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

    def router_scatter(self, logits, n_tok, n_route, top_k, ids, w, n_expert, expert_base, sorted_tok,
                       expert_offset, work, stream=0):
        self._check(self.lib.exl3b200_router_scatter(logits, n_tok, n_route, top_k, ids, w, n_expert, expert_base,
                                                     sorted_tok, expert_offset, work, stream),
                    "exl3b200_router_scatter")

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

    def ep_dedup_scan(self, ids, top_k, sorted_pairs, dest_off, n_pairs, n_local, world, send_meta, row_tok, counts,
                      stream=0):
        self._check(self.lib.exl3b200_ep_dedup_scan(ids, top_k, sorted_pairs, dest_off, n_pairs, n_local, world,
                                                    send_meta, row_tok, counts, stream), "exl3b200_ep_dedup_scan")

    # ------------------------------------------------------------------ peer-memory windows
    def window_alloc(self, nbytes):
        p = C.c_void_p()
        self._check(self.lib.exl3b200_ep_window_alloc(nbytes, C.byref(p)), "exl3b200_ep_window_alloc")
        return p.value

    def window_free(self, ptr):
        self._check(self.lib.exl3b200_ep_window_free(ptr), "exl3b200_ep_window_free")

    def window_handle(self, ptr):
        buf = C.create_string_buffer(64)
        self._check(self.lib.exl3b200_ep_window_handle(ptr, buf), "exl3b200_ep_window_handle")
        return bytes(buf.raw)

    def window_open(self, handle):
        p = C.c_void_p()
        buf = C.create_string_buffer(handle, 64)
        self._check(self.lib.exl3b200_ep_window_open(buf, C.byref(p)), "exl3b200_ep_window_open")
        return p.value

    def window_close(self, ptr):
        self._check(self.lib.exl3b200_ep_window_close(ptr), "exl3b200_ep_window_close")

    def p2p_dispatch(self, x, x_pitch, row_tok, meta, dest_off, counts, n_slots, peers, offs, rank, world, t_cap,
                     p_cap, hidden, epoch, stream=0):
        self._check(self.lib.exl3b200_p2p_dispatch(x, x_pitch, row_tok, meta, dest_off, counts, n_slots, peers, offs,
                                                   rank, world, t_cap, p_cap, hidden, epoch, stream),
                    "exl3b200_p2p_dispatch")

    def p2p_wait_dispatch(self, own, offs, world, epoch, hdr, stream=0):
        self._check(self.lib.exl3b200_p2p_wait_dispatch(own, offs, world, epoch, hdr, stream),
                    "exl3b200_p2p_wait_dispatch")

    def p2p_unpack(self, own, offs, hdr, world, t_cap, p_cap, n_pairs, expert, row, dst_rank, dst_pos, stream=0):
        self._check(self.lib.exl3b200_p2p_unpack(own, offs, hdr, world, t_cap, p_cap, n_pairs, expert, row, dst_rank,
                                                 dst_pos, stream), "exl3b200_p2p_unpack")

    def p2p_combine(self, y_rows, y_pitch, sorted_pair, n_rows, dst_rank, dst_pos, peers, offs, rank, world, p_cap,
                    hidden, epoch, stream=0):
        self._check(self.lib.exl3b200_p2p_combine(y_rows, y_pitch, sorted_pair, n_rows, dst_rank, dst_pos, peers, offs,
                                                  rank, world, p_cap, hidden, epoch, stream), "exl3b200_p2p_combine")

    def p2p_wait_combine(self, own, offs, world, epoch, status, stream=0):
        self._check(self.lib.exl3b200_p2p_wait_combine(own, offs, world, epoch, status, stream),
                    "exl3b200_p2p_wait_combine")

    def p2p_row_dst(self, sorted_pair, n_rows, dst_rank, dst_pos, peers, offs, rank, world, p_cap, hidden, row_dst,
                    stream=0):
        self._check(self.lib.exl3b200_p2p_row_dst(sorted_pair, n_rows, dst_rank, dst_pos, peers, offs, rank, world,
                                                  p_cap, hidden, row_dst, stream), "exl3b200_p2p_row_dst")

    def p2p_signal_combine(self, peers, offs, rank, world, epoch, stream=0):
        self._check(self.lib.exl3b200_p2p_signal_combine(peers, offs, rank, world, epoch, stream),
                    "exl3b200_p2p_signal_combine")

    def moe_down_rows(self, args_ref, row_dst, stream=0):
        self._check(self.lib.exl3b200_moe_down_rows(args_ref, row_dst, stream), "exl3b200_moe_down_rows")

    def moe_gather_bf16(self, rows, row_pitch, sorted_tok, n_rows, w, n_tok, top_k, width, y, work, stream=0):
        self._check(self.lib.exl3b200_moe_gather_bf16(rows, row_pitch, sorted_tok, n_rows, w, n_tok, top_k, width, y,
                                                      work, stream), "exl3b200_moe_gather_bf16")

    def layer_work_bytes(self, desc, max_tokens):
        n = int(self.lib.exl3b200_moe_layer_work_bytes(C.byref(desc), max_tokens))
        if n < 0:
            raise RuntimeError("exl3b200_moe_layer_work_bytes: the layer description was refused")
        return n

    def layer_carve(self, desc, max_tokens, work, work_bytes):
        b = LayerBufs()
        self._check(self.lib.exl3b200_moe_layer_carve(C.byref(desc), max_tokens, work, work_bytes, C.byref(b)),
                    "exl3b200_moe_layer_carve")
        return b

    def layer_forward(self, desc, bufs, x, logits, n_tok, out, out_dtype, stream=0):
        """out_dtype: 1 (RAD_F32) or 3 (RAD_BF16)."""
        self._check(self.lib.exl3b200_moe_layer_forward(C.byref(desc), C.byref(bufs), x, logits, n_tok, out, out_dtype,
                                                        stream), "exl3b200_moe_layer_forward")

    def moe_down_f16(self, args_ref, stream=0):
        """moe_exl3_down with f16 output rows (the row's RadArgs, y f16); returns the status."""
        return int(self.lib.exl3b200_moe_down_f16(args_ref, stream))

    def moe_down_f16_scratch(self, args_ref):
        """Scratch bytes moe_down_f16 uses for these RadArgs (0: none, or refused)."""
        return int(self.lib.exl3b200_moe_down_f16_scratch(args_ref))

    def set_peer_wait_ns(self, ns):
        self._check(self.lib.exl3b200_set_peer_wait_ns(ns), "exl3b200_set_peer_wait_ns")

    def p2p_begin(self, epoch, stream=0):
        self._check(self.lib.exl3b200_p2p_begin(epoch, stream), "exl3b200_p2p_begin")

    def moe_op_live(self, args_ref, down, row_dst, stream=0):
        self._check(self.lib.exl3b200_moe_op_live(args_ref, down, row_dst, stream), "exl3b200_moe_op_live")

    # ---- the width split over peer memory (exl3b200_tp.cu)
    def tp_gather_rs(self, rows, row_pitch, sorted_tok, n_rows, w, n_tok, top_k, width, work, peers, offs, rank,
                     world, s_cap, epoch, status, stream=0):
        self._check(self.lib.exl3b200_tp_gather_rs(rows, row_pitch, sorted_tok, n_rows, w, n_tok, top_k, width, work,
                                                   peers, offs, rank, world, s_cap, epoch, status, stream),
                    "exl3b200_tp_gather_rs")

    def tp_reduce(self, peers, offs, rank, world, n_tok, width, s_cap, epoch, stream=0):
        self._check(self.lib.exl3b200_tp_reduce(peers, offs, rank, world, n_tok, width, s_cap, epoch, stream),
                    "exl3b200_tp_reduce")

    def tp_pull(self, peers, offs, rank, world, n_tok, width, s_cap, out, out_pitch, epoch, status, stream=0):
        self._check(self.lib.exl3b200_tp_pull(peers, offs, rank, world, n_tok, width, s_cap, out, out_pitch, epoch,
                                              status, stream), "exl3b200_tp_pull")

    # ---- whole multi-GPU steps driven from C (exl3b200_layer.c)
    def ep_window_layout(self, world, t_cap, top_k, hidden):
        """(offs[6], bytes) of the expert-parallel window."""
        offs = (_I64 * 6)()
        n = int(self.lib.exl3b200_ep_window_layout(world, t_cap, top_k, hidden, offs))
        if n < 0:
            raise RuntimeError("exl3b200_ep_window_layout: refused")
        return tuple(offs), n

    def tp_window_layout(self, world, max_tokens, hidden):
        """(offs[4], bytes) of the width split's window."""
        offs = (_I64 * 4)()
        n = int(self.lib.exl3b200_tp_window_layout(world, max_tokens, hidden, offs))
        if n < 0:
            raise RuntimeError("exl3b200_tp_window_layout: refused")
        return tuple(offs), n

    def ep_step_work_bytes(self, desc):
        n = int(self.lib.exl3b200_ep_step_work_bytes(C.byref(desc)))
        if n < 0:
            raise RuntimeError("exl3b200_ep_step_work_bytes: the step description was refused")
        return n

    def ep_step_carve(self, desc, work, work_bytes):
        b = EpBufs()
        self._check(self.lib.exl3b200_ep_step_carve(C.byref(desc), work, work_bytes, C.byref(b)),
                    "exl3b200_ep_step_carve")
        return b

    def ep_step_forward(self, desc, bufs, x, logits, n_tok, out, out_dtype, stream=0, marks=None):
        """out_dtype: 1 (RAD_F32) or 3 (RAD_BF16); marks: None or marks_array() of 10 events."""
        self._check(self.lib.exl3b200_ep_step_forward(C.byref(desc), C.byref(bufs), x, logits, n_tok, out, out_dtype,
                                                      stream, marks), "exl3b200_ep_step_forward")

    def tp_step_forward(self, desc, bufs, x, logits, n_tok, out, out_pitch, stream=0, marks=None):
        """bufs: the slice layer's LayerBufs; out f32; marks: None or marks_array() of 7 events."""
        self._check(self.lib.exl3b200_tp_step_forward(C.byref(desc), C.byref(bufs), x, logits, n_tok, out, out_pitch,
                                                      stream, marks), "exl3b200_tp_step_forward")

    # ---- the MoE block (routed layer + shared expert, the fold; exl3b200_layer.c)
    def block_work_bytes(self, desc, max_tokens):
        n = int(self.lib.exl3b200_moe_block_work_bytes(C.byref(desc), max_tokens))
        if n < 0:
            raise RuntimeError("exl3b200_moe_block_work_bytes: the block description was refused")
        return n

    def block_carve(self, desc, max_tokens, work, work_bytes):
        b = BlockBufs()
        self._check(self.lib.exl3b200_moe_block_carve(C.byref(desc), max_tokens, work, work_bytes, C.byref(b)),
                    "exl3b200_moe_block_carve")
        return b

    def block_forward(self, desc, bufs, x, logits, n_tok, out, out_dtype, stream=0):
        """out_dtype: 1 (RAD_F32) or 3 (RAD_BF16)."""
        self._check(self.lib.exl3b200_moe_block_forward(C.byref(desc), C.byref(bufs), x, logits, n_tok, out, out_dtype,
                                                        stream), "exl3b200_moe_block_forward")
