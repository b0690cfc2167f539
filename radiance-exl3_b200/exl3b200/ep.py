"""ep.py -- expert parallelism for the routed-MoE layer: one process a GPU, torch.distributed (NCCL) for the
exchange, the library's kernels for every device step.

The reference runs the layer on one device; this is the multi-GPU form the path shards into. Experts are held in
contiguous blocks (expert e on rank e // n_local); every rank routes its own tokens. One step on each rank:

    router_topk                      ids, w                          [T, top_k]
    ep_dest + moe_scatter over ranks sorted_pairs, dest_off          pairs grouped by owning rank, token order inside
    ep_pack_dedup                    send_x: ONE row a distinct (token, rank); a meta word a pair (row, local expert)
    all-to-all of the counts         -> the one host read of a step: the split sizes
    all-to-all of rows and metas     -> recv_x (rows), recv_meta (pairs), in source-rank order
    ep_unpack, moe_scatter (local)   each received pair's local expert and row; pairs sorted by local expert
    ep_map                           sorted pair -> its token row (the sorted_tok the ops read, top_k 1)
    moe_exl3_gate_up, moe_exl3_down  y_rows (bf16, one a pair, sorted order), the plugin rows as on one GPU
    rows_scatter                     y_recv (arrival order of the pairs)
    all-to-all back                  y_back, in the order the pairs were sent
    moe_gather over sorted_pairs     out f32 [T, H]: slots summed in ascending order, as on one GPU

A token row crosses to a rank once however many of its slots that rank serves (dispatch bytes: distinct
(token, rank) pairs, not slots); every pair still returns its own down row, so each pair's down row is the one a
single GPU computes and the gather sums a token's slots in the same order -- the layer's output does not depend on
the number of ranks. The all-to-alls move bf16/fp16 rows bit for bit (as float16 views: a copy, no arithmetic).

`ops` supplies the device steps: `DeviceOps` (the library, CUDA tensors, NCCL) or a host stand-in with the same
methods for testing the exchange on CPU ranks over gloo."""
import ctypes as C

import numpy as np


class DeviceOps:
    """The device steps of an EP step on this rank's GPU: libexl3b200.so's kernels on torch's current stream and
    the local experts' resident weights (a MoeLayer over experts [rank * n_local, (rank + 1) * n_local))."""

    def __init__(self, plugin, *, n_local, hidden, width, bits_gu, bits_dn, codebook, max_rows, seed, device):
        from .layer import MoeLayer
        self.local = MoeLayer(plugin, n_expert=n_local, hidden=hidden, width=width, top_k=1, bits_gu=bits_gu,
                              bits_dn=bits_dn, codebook=codebook, max_tokens=1, max_rows=max_rows, seed=seed,
                              device=device)
        self.nat = self.local.native
        self.H = hidden
        self._works = {}

    # the buffers of the local pass live in the local layer (its RadArgs point at them)
    def local_buffers(self):
        return self.local.sorted_tok, self.local.offset, self.local.y_rows

    @staticmethod
    def _stream():
        import torch
        return torch.cuda.current_stream().cuda_stream

    def _work(self, key, nbytes, torch_dev):
        import torch
        buf = self._works.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = self._works[key] = torch.empty(max(16, nbytes), dtype=torch.uint8, device=torch_dev)
        return buf

    def router(self, logits, T, E, k, ids, w):
        self.nat.router_topk(logits.data_ptr(), T, E, k, ids.data_ptr(), w.data_ptr(), self._stream())

    def scatter(self, ids, n_pairs, n_expert, sorted_tok, offset):
        work = self._work(("scatter", n_expert), self.nat.scatter_work_bytes(sorted_tok.numel(), n_expert), ids.device)
        self.nat.moe_scatter(ids.data_ptr(), n_pairs, n_expert, 0, sorted_tok.data_ptr(), offset.data_ptr(),
                             work.data_ptr(), self._stream())

    def dest(self, ids, n_pairs, n_local, world, dest):
        self.nat.ep_dest(ids.data_ptr(), n_pairs, n_local, world, dest.data_ptr(), self._stream())

    def pack_dedup(self, x, ids, k, sorted_pairs, dest_off, n_pairs, n_local, world, send_x, send_meta, row_tok,
                   counts):
        self.nat.ep_pack_dedup(x.data_ptr(), x.shape[1], ids.data_ptr(), k, sorted_pairs.data_ptr(),
                               dest_off.data_ptr(), n_pairs, n_local, world, x.shape[1], send_x.data_ptr(),
                               send_meta.data_ptr(), row_tok.data_ptr(), counts.data_ptr(), self._stream())

    def unpack(self, meta, n_pairs, recv_counts, world, expert, row):
        self.nat.ep_unpack(meta.data_ptr(), n_pairs, recv_counts.data_ptr(), world, expert.data_ptr(),
                           row.data_ptr(), self._stream())

    def map(self, idx, n, table, n_table, out):
        self.nat.ep_map(idx.data_ptr(), n, table.data_ptr(), n_table, out.data_ptr(), self._stream())

    def experts(self, recv_x, n_rows, n_pairs, events=None, x_ptr=None, down_row_dst=None, live=False):
        self.local.experts(n_rows, n_pairs, self._stream(), x_ptr=x_ptr or recv_x.data_ptr(), top_k=1, M=n_rows,
                           events=events, down_row_dst=down_row_dst, live=live)

    def rows_scatter(self, src, idx, n_rows, dst, n_dst):
        rb = src.shape[1] * src.element_size()
        self.nat.rows_scatter(src.data_ptr(), rb, idx.data_ptr(), n_rows, rb, dst.data_ptr(),
                              dst.shape[1] * dst.element_size(), n_dst, self._stream())

    def gather(self, rows, sorted_pairs, n_rows, w, T, k, out, rows_ptr=None):
        work = self._work(("gather", k), self.nat.gather_work_bytes(w.numel() // k, k), out.device)
        import torch
        gather = self.nat.moe_gather_bf16 if out.dtype == torch.bfloat16 else self.nat.moe_gather
        gather(rows_ptr or rows.data_ptr(), out.shape[1], sorted_pairs.data_ptr(), n_rows, w.data_ptr(), T, k,
               out.shape[1], out.data_ptr(), work.data_ptr(), self._stream())

    def kernels(self, T, k, E, R):
        """How many of the library's kernels one step launches: router, ep_dest, rank scatter, the two pack
        kernels, ep_unpack, local scatter, ep_map, gate_up (+ prep), down, rows_scatter, the gather (one launch up to
        4096 rows, else two)."""
        P = T * k
        tc = R > 0 and self.local._tc("gate_up", R)
        n = 1 + 1 + (1 if P <= 2048 else 3) + 2
        if R > 0:
            n += 1 + (1 if R <= 2048 else 3) + 1 + 2 + (1 if tc else 0) + 1
        return n + (1 if P <= 4096 and k <= 32 else 2)


class IpcWindow:
    """This rank's peer-memory window (exl3b200_ep_window_*: device memory, zeroed, exported by CUDA IPC) and every
    peer's, mapped here: `ptrs[r]` rank r's base as this rank sees it (its own for itself), `peers` the same as a
    device int64 table. `offs` the layout's byte offsets (the same on every rank). Built and closed collectively."""

    def __init__(self, nat, dist, group, rank, world, offs, nbytes, device):
        import torch
        self.nat, self.dist, self.group, self.rank, self.world = nat, dist, group, rank, world
        self.offs = (C.c_int64 * len(offs))(*offs)
        self.base = nat.window_alloc(nbytes)
        handles = [None] * world
        dist.all_gather_object(handles, nat.window_handle(self.base), group=group)
        self.ptrs = [self.base if r == rank else nat.window_open(handles[r]) for r in range(world)]
        self.peers = torch.tensor(self.ptrs, dtype=torch.int64, device=device)
        dist.barrier(group=group)

    def close(self):
        """Collective: unmap the peers' windows, then (after every rank has) free this one."""
        if self.base is None:
            return
        for r, p in enumerate(self.ptrs):
            if r != self.rank:
                self.nat.window_close(p)
        self.dist.barrier(group=self.group)
        self.nat.window_free(self.base)
        self.base = None


class P2pWindow(IpcWindow):
    """The expert-parallel window, laid out by the library (exl3b200_ep_window_layout): rows [world][t_cap][H] f16 |
    meta [world][p_cap] u32 | yback [p_cap][H] bf16 | ctl [world][8] u32 | done [2] u32 | sink [H] bf16."""

    def __init__(self, nat, dist, group, rank, world, t_cap, top_k, hidden, device):
        offs, nbytes = nat.ep_window_layout(world, t_cap, top_k, hidden)
        super().__init__(nat, dist, group, rank, world, offs, nbytes, device)

    def rows_ptr(self):
        return self.base + self.offs[0]

    def yback_ptr(self):
        return self.base + self.offs[2]


class EpLayer:
    """The routed-MoE layer over `world` ranks. Buffers are sized for the largest step: this rank sends at most
    max_tokens * top_k rows and receives at most world times that (every rank routing everything here)."""

    def __init__(self, plugin=None, *, rank, world, n_expert, hidden, width, top_k, bits_gu=3, bits_dn=4,
                 codebook="mul1", max_tokens=2048, seed=0, group=None, device="cuda", ops=None, full=None,
                 transport="nccl", fuse_combine=True):
        import torch
        import torch.distributed as dist
        if n_expert % world:
            raise ValueError(f"n_expert {n_expert} is not a multiple of the world size {world}")
        self.torch, self.dist, self.group = torch, dist, group
        self.rank, self.G = rank, world
        self.E, self.H, self.W, self.k = n_expert, hidden, width, top_k
        self.nl = n_expert // world
        self.max_tokens = max_tokens
        dev = self.dev = torch.device(device) if not isinstance(device, torch.device) else device
        P, H = max_tokens * top_k, hidden
        self.Rcap = world * P
        if ops is None:
            # the weights of this rank's experts; over NCCL also the buffers of the local pass (over peer memory the
            # C driver carves its own)
            ops = DeviceOps(plugin, n_local=self.nl, hidden=hidden, width=width, bits_gu=bits_gu, bits_dn=bits_dn,
                            codebook=codebook, max_rows=self.Rcap if transport == "nccl" else 1, seed=seed,
                            device=dev)
            if full is not None:
                ops.local.load_experts(full, rank * self.nl)
        self.ops = ops
        e = lambda *shape, dt: torch.empty(shape, dtype=dt, device=dev)  # noqa: E731
        f16, bf16, i32, f32 = torch.float16, torch.bfloat16, torch.int32, torch.float32
        self.x, self.logits = e(max_tokens, H, dt=f16), e(max_tokens, n_expert, dt=f32)
        self.out = e(max_tokens, H, dt=f32)
        self.last = {"R": 0, "sent": 0}
        if transport not in ("nccl", "p2p"):
            raise ValueError(f"transport {transport!r}")
        self.transport, self.win = transport, None
        if transport == "p2p":
            self._init_p2p(fuse_combine, bits_gu, bits_dn, codebook, width)
            return
        self.ids, self.w, self.dest = e(P, dt=i32), e(P, dt=f32), e(P, dt=i32)
        self.sorted_pairs, self.row_tok = e(P, dt=i32), e(P, dt=i32)
        # one host read a step: [send counts 2G | receive counts 2G | rank offsets of the sorted pairs G + 1]
        self.hdr = torch.zeros(5 * world + 1, dtype=i32, device=dev)
        self.counts_send, self.counts_recv = self.hdr[:2 * world], self.hdr[2 * world:4 * world]
        self.dest_off = self.hdr[4 * world:]
        self.send_x, self.send_meta = e(P, H, dt=f16), e(P, dt=i32)
        self.recv_x = e(world * max_tokens, H, dt=f16)                # rows: at most T from each source
        self.recv_meta, self.pair_e, self.pair_row = e(self.Rcap, dt=i32), e(self.Rcap, dt=i32), e(self.Rcap, dt=i32)
        self.sorted_pair = e(self.Rcap, dt=i32)
        self.y_recv, self.y_back = e(self.Rcap, H, dt=bf16), e(P, H, dt=bf16)
        self.sorted_row, self.off_loc, self.y_rows = ops.local_buffers()

    def _init_p2p(self, fuse_combine, bits_gu, bits_dn, codebook, width):
        """The peer-memory step: one call of the library's C driver (exl3b200_ep_step_forward) over one device block
        it carves; the local experts' weights stay in ops.local. The views below are what the accounting reads."""
        import torch
        from .native import EpDesc
        nat = self.nat = self.ops.nat
        G, k, H, dev = self.G, self.k, self.H, self.dev
        self.win = P2pWindow(nat, self.dist, self.group, self.rank, G, self.max_tokens, k, H, dev)
        self.epoch_dev = torch.zeros(1, dtype=torch.int32, device=dev)     # the step's epoch, advanced on the device
        self.status_p = torch.zeros(1, dtype=torch.int32, device=dev)
        self.fuse_combine = fuse_combine
        d = self.desc = EpDesc()
        ld = d.layer
        ld.n_expert, ld.n_local, ld.expert_base = self.E, self.nl, self.rank * self.nl
        ld.hidden, ld.width, ld.top_k = H, width, k
        ld.bits_gu, ld.bits_dn, ld.codebook = bits_gu, bits_dn, {"3inst": 0, "mcg": 1, "mul1": 2}[codebook]
        d.rank, d.world, d.max_tokens, d.fuse_combine = self.rank, G, self.max_tokens, int(fuse_combine)
        d.window, d.peers = self.win.base, self.win.peers.data_ptr()
        for i, o in enumerate(self.win.offs):
            d.offs[i] = o
        d.epoch, d.status = self.epoch_dev.data_ptr(), self.status_p.data_ptr()
        self._sync_weights()
        nbytes = nat.ep_step_work_bytes(d)
        self.work = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        b = self.bufs = nat.ep_step_carve(d, self.work.data_ptr(), nbytes)
        base = self.work.data_ptr()

        def view(ptr, n):
            return self.work[ptr - base:ptr - base + 4 * n].view(torch.int32)

        self.hdr_p, self.counts_p = view(b.hdr, 3 * G + 1), view(b.counts, 2 * G)
        self.off_loc, self.sorted_row = view(b.expert_offset, self.nl + 1), view(b.sorted_row, self.Rcap)

    def _sync_weights(self):
        """Point the step's layer description at ops.local's current weight set (a stack swaps sets)."""
        L, ld = self.ops.local, self.desc.layer
        ld.gu_codes, ld.dn_codes = L.gu_tab.data_ptr(), L.dn_tab.data_ptr()
        ld.suh, ld.suh1, ld.svh_gu = L.suh.data_ptr(), L.suh1.data_ptr(), L.svh_gu.data_ptr()
        ld.dn_suh, ld.svh_dn = L.dn_suh.data_ptr(), L.svh_dn.data_ptr()

    # ------------------------------------------------------------------ the exchange
    def _a2a(self, out, inp, out_splits, in_splits):
        """One all-to-all of rows (dim 0), bit for bit: 16-bit rows go as float16 views, the collective's type
        being only a width here."""
        t = self.torch
        if out.dtype == t.bfloat16:
            out, inp = out.view(t.float16), inp.view(t.float16)
        self.dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    PHASES = ("route+pack", "counts+dispatch", "local sort", "experts", "combine", "gather")

    def forward(self, T, stream=None, events=None, phases=None, x=None, logits=None, out=None):
        """The layer over the first T tokens of self.x / self.logits into self.out[:T] (`x`, `logits`, `out`
        replace them, e.g. for double-buffered inputs). `stream` must be torch's current stream (the collectives
        run there); `events` as MoeLayer.experts; `phases`: len(PHASES) + 1 CUDA events recorded between the steps
        (for a per-phase breakdown)."""
        if T > self.max_tokens:
            raise ValueError(f"T {T} > max_tokens {self.max_tokens}")
        x = self.x if x is None else x
        logits = self.logits if logits is None else logits
        out = self.out if out is None else out
        if self.transport == "p2p":
            return self._forward_p2p(T, events, phases, x, logits, out)
        o, G, k, P = self.ops, self.G, self.k, T * self.k
        mark = (lambda i: phases[i].record()) if phases else (lambda i: None)
        mark(0)
        o.router(logits, T, self.E, k, self.ids, self.w)
        o.dest(self.ids, P, self.nl, G, self.dest)
        o.scatter(self.dest, P, G, self.sorted_pairs[:P], self.dest_off)
        o.pack_dedup(x, self.ids, k, self.sorted_pairs, self.dest_off, P, self.nl, G, self.send_x,
                     self.send_meta, self.row_tok, self.counts_send)
        mark(1)
        self.dist.all_to_all_single(self.counts_recv, self.counts_send, group=self.group)
        h = self.hdr.cpu().tolist()             # the split sizes: the one host read of a step
        rows_s, pairs_s = h[0:2 * G:2], h[1:2 * G:2]
        rows_r, pairs_r = h[2 * G:4 * G:2], h[2 * G + 1:4 * G:2]
        S, Rr, R = sum(pairs_s), sum(rows_r), sum(pairs_r)
        self._a2a(self.recv_x[:Rr], self.send_x[:sum(rows_s)], rows_r, rows_s)
        self._a2a(self.recv_meta[:R], self.send_meta[:S], pairs_r, pairs_s)
        mark(2)
        o.unpack(self.recv_meta, R, self.counts_recv, G, self.pair_e, self.pair_row)
        o.scatter(self.pair_e[:R], R, self.nl, self.sorted_pair[:R], self.off_loc)
        o.map(self.sorted_pair, R, self.pair_row, R, self.sorted_row)
        mark(3)
        o.experts(self.recv_x, Rr, R, events)
        mark(4)
        o.rows_scatter(self.y_rows, self.sorted_pair, R, self.y_recv, R)
        self._a2a(self.y_back[:S], self.y_recv[:R], pairs_s, pairs_r)
        mark(5)
        o.gather(self.y_back, self.sorted_pairs, S, self.w, T, k, out)
        mark(6)
        self.last = {"R": R, "rows_recv": Rr, "sent": S, "rows_sent": sum(rows_s), "send_counts": pairs_s,
                     "recv_counts": pairs_r, "send_rows": rows_s, "recv_rows": rows_r}

    def _forward_p2p(self, T, events, phases, x, logits, out):
        """The same step with the exchange over peer memory, as ONE call of the library's C driver
        (exl3b200_ep_step_forward): no host synchronisation at all -- the local pass runs at capacity (world * T *
        top_k received pairs) with its live count on the device, and the epoch lives on the device -- so the step
        can be captured in a CUDA graph and replayed. `phases` and `events` become the driver's marks."""
        from .native import marks_array
        self._sync_weights()
        marks = None
        if phases or events:
            marks = marks_array(list(phases or [None] * 7) + list(events or [None] * 3))
        dt = 3 if out.dtype == self.torch.bfloat16 else 1
        self.nat.ep_step_forward(self.desc, self.bufs, x.data_ptr(), logits.data_ptr(), T, out.data_ptr(), dt,
                                 self.ops._stream(), marks)
        self.last = {"p2p": True, "sent": T * self.k}

    def _p2p_counts(self):
        """The last step's received counts, read from the device (synchronises): rows and pairs from each source."""
        h = self.hdr_p.cpu().tolist()
        G = self.G
        rows_r, pairs_r = h[0:3 * G:3], h[1:3 * G:3]
        self.last.update({"R": sum(pairs_r), "rows_recv": sum(rows_r), "recv_counts": pairs_r,
                          "recv_rows": rows_r, "dispatch_status": h[3 * G]})
        return self.last

    def check(self):
        """Raise if a peer's dispatch or combine did not arrive within the wait limit in the last step, or a row fell
        outside a window (reads the status words and the device error word: synchronises)."""
        if self.transport != "p2p":
            return
        if self._p2p_counts()["dispatch_status"] != 0 or int(self.status_p.item()) != 0:
            raise RuntimeError("expert parallelism: a peer's exchange did not arrive within the wait limit")
        err = self.nat.read_error(clear=False)
        if err & 12:
            raise RuntimeError(f"expert parallelism: device error word {err:#x}")

    def close(self):
        """Collective: release the peer-memory window (p2p transport)."""
        if self.win is not None:
            self.win.close()
            self.win = None

    # ------------------------------------------------------------------ accounting (this rank)
    def live_experts(self):
        off = self.off_loc.cpu().numpy()
        return int((np.diff(off) > 0).sum())

    def expert_bytes(self):
        return self.ops.local.expert_bytes()

    def time_prep_step(self, T, n=5):
        """The local pass's gate_up input rotation alone (ms), over the rows the last step received."""
        R = self._R()
        Rr = self.last.get("rows_recv", R)
        if self.transport == "p2p":
            return self.ops.local.time_prep(self.G * self.max_tokens, R, x_ptr=self.win.rows_ptr(), top_k=1, n=n,
                                            sorted_tok=self.sorted_row.data_ptr(), offset=self.off_loc.data_ptr())
        return self.ops.local.time_prep(Rr, R, x_ptr=self.recv_x.data_ptr(), top_k=1, n=n)

    def expert_flops(self, rows):
        return self.ops.local.expert_flops(rows)

    def _R(self):
        if self.last.get("p2p") and "R" not in self.last:
            self._p2p_counts()
        return self.last.get("R", 0)

    def band_name(self, op, T):
        return self.ops.local.band_name(op, self._R()) + " (rows received by this rank)"

    def launches_per_step(self, T):
        if self.transport == "p2p":
            # begin, router, ep_dest, rank scatter, dedup scan, dispatch, wait, unpack, local scatter (capacity),
            # map, row table, gate_up (+ prep), down, signal (or combine), wait, the gather's two
            Q = self.Rcap
            tc = self.ops.local._tc("gate_up", Q)
            P = T * self.k
            return 1 + 1 + 1 + (1 if P <= 2048 else 3) + 1 + 2 + 1 + (1 if Q <= 2048 else 3) + 1 + \
                (1 if self.fuse_combine else 0) + 2 + (1 if tc else 0) + 1 + 1 + (1 if P <= 4096 and self.k <= 32 else 2)
        return self.ops.kernels(T, self.k, self.E, self._R())

    def exchange_bytes(self):
        """Bytes this rank sent to other ranks in the last step: token rows and pair metas out, the down rows of the
        pairs it served back; what it keeps for itself excluded."""
        if self.last.get("p2p"):
            c = self.counts_p.cpu().tolist()     # rows, pairs sent to each rank
            r = self.rank
            rows_out = sum(c[0::2]) - c[2 * r]
            metas_out = sum(c[1::2]) - c[2 * r + 1]
            L = self._p2p_counts()
            rows_back = L["R"] - L["recv_counts"][r]
            return rows_out * 2 * self.H + metas_out * 4 + rows_back * 2 * self.H
        if "send_counts" not in self.last:
            return 0
        L, r = self.last, self.rank
        rows_out = L["rows_sent"] - L["send_rows"][r]
        metas_out = L["sent"] - L["send_counts"][r]
        rows_back = L["R"] - L["recv_counts"][r]
        return rows_out * 2 * self.H + metas_out * 4 + rows_back * 2 * self.H
