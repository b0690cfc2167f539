"""ep.py -- expert parallelism for the routed-MoE layer: one process a GPU, torch.distributed (NCCL) for the
exchange, the library's kernels for every device step.

The reference runs the layer on one device; this is the multi-GPU form the path shards into. Experts are held in
contiguous blocks (expert e on rank e // n_local); every rank routes its own tokens. One step on each rank:

    router_topk                      ids, w                          [T, top_k]
    moe_scatter over ALL experts     sorted_pairs, expert_offset     the pairs grouped by the rank of their expert
    ep_pack                          send_x (token rows), send_e (local expert ids), send counts per rank
    all-to-all of the counts         -> the one host read of a step: the split sizes
    all-to-all of send_x, send_e     -> recv_x, recv_e               rows in arrival order (source rank, then sorted)
    moe_scatter over local experts   sorted_loc, off_loc             (top_k 1: a received row is its own token)
    moe_exl3_gate_up, moe_exl3_down  y_rows (bf16, sorted order)     the plugin rows, exactly as on one GPU
    rows_scatter                     y_recv (arrival order)
    all-to-all back                  y_back                          in the order the pairs were sent
    moe_gather over sorted_pairs     out f32 [T, H]                  slots summed in ascending order, as on one GPU

Each pair's down row is the one a single GPU computes (same expert, same input row), and the gather sums a
token's slots in the same order, so the layer's output does not depend on the number of ranks. The all-to-alls
move bf16/fp16 rows bit for bit (as float16 views: a copy, no arithmetic).

`ops` supplies the device steps: `DeviceOps` (the library, CUDA tensors, NCCL) or a host stand-in with the same
methods for testing the exchange on CPU ranks over gloo."""
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

    def pack(self, x, ids, k, sorted_pairs, n_pairs, offset, n_local, world, send_x, send_e, counts):
        self.nat.ep_pack(x.data_ptr(), x.shape[1], ids.data_ptr(), k, sorted_pairs.data_ptr(), n_pairs,
                         offset.data_ptr(), n_local, world, x.shape[1], send_x.data_ptr(), send_e.data_ptr(),
                         counts.data_ptr(), self._stream())

    def experts(self, recv_x, R, events=None):
        self.local.experts(R, R, self._stream(), x_ptr=recv_x.data_ptr(), top_k=1, M=R, events=events)

    def rows_scatter(self, src, idx, n_rows, dst, n_dst):
        rb = src.shape[1] * src.element_size()
        self.nat.rows_scatter(src.data_ptr(), rb, idx.data_ptr(), n_rows, rb, dst.data_ptr(),
                              dst.shape[1] * dst.element_size(), n_dst, self._stream())

    def gather(self, rows, sorted_pairs, n_rows, w, T, k, out):
        work = self._work(("gather", k), self.nat.gather_work_bytes(w.numel() // k, k), rows.device)
        self.nat.moe_gather(rows.data_ptr(), rows.shape[1], sorted_pairs.data_ptr(), n_rows, w.data_ptr(), T, k,
                            out.shape[1], out.data_ptr(), work.data_ptr(), self._stream())

    def kernels(self, T, k, E, R):
        """How many of the library's kernels one step launches (ep_pack and rows_scatter counted)."""
        P = T * k
        tc = R > 0 and self.local._tc("gate_up", R)
        n = 1 + (1 if P <= 8192 else 3) + 1 + (1 if R <= 8192 else 3)
        n += (2 + (1 if tc else 0)) if R > 0 else 0
        n += 1 if R > 0 else 0
        return n + 2


class EpLayer:
    """The routed-MoE layer over `world` ranks. Buffers are sized for the largest step: this rank sends at most
    max_tokens * top_k rows and receives at most world times that (every rank routing everything here)."""

    def __init__(self, plugin=None, *, rank, world, n_expert, hidden, width, top_k, bits_gu=3, bits_dn=4,
                 codebook="mul1", max_tokens=2048, seed=0, group=None, device="cuda", ops=None, full=None):
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
            ops = DeviceOps(plugin, n_local=self.nl, hidden=hidden, width=width, bits_gu=bits_gu, bits_dn=bits_dn,
                            codebook=codebook, max_rows=self.Rcap, seed=seed, device=dev)
            if full is not None:
                ops.local.load_experts(full, rank * self.nl)
        self.ops = ops
        e = lambda *shape, dt: torch.empty(shape, dtype=dt, device=dev)  # noqa: E731
        f16, bf16, i32, f32 = torch.float16, torch.bfloat16, torch.int32, torch.float32
        self.x, self.logits = e(max_tokens, H, dt=f16), e(max_tokens, n_expert, dt=f32)
        self.ids, self.w = e(P, dt=i32), e(P, dt=f32)
        self.sorted_pairs, self.offset = e(P, dt=i32), e(n_expert + 1, dt=i32)
        self.send_x, self.send_e = e(P, H, dt=f16), e(P, dt=i32)
        self.counts = torch.zeros(2 * world, dtype=i32, device=dev)     # [send counts | receive counts]
        self.recv_x, self.recv_e = e(self.Rcap, H, dt=f16), e(self.Rcap, dt=i32)
        self.y_recv, self.y_back = e(self.Rcap, H, dt=bf16), e(P, H, dt=bf16)
        self.out = e(max_tokens, H, dt=f32)
        self.sorted_loc, self.off_loc, self.y_rows = ops.local_buffers()
        self.last = {"R": 0, "sent": 0}

    # ------------------------------------------------------------------ the exchange
    def _a2a(self, out, inp, out_splits, in_splits):
        """One all-to-all of rows (dim 0), bit for bit: 16-bit rows go as float16 views, the collective's type
        being only a width here."""
        t = self.torch
        if out.dtype == t.bfloat16:
            out, inp = out.view(t.float16), inp.view(t.float16)
        self.dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    PHASES = ("route+pack", "counts+dispatch", "local sort", "experts", "combine", "gather")

    def forward(self, T, stream=None, events=None, phases=None):
        """The layer over the first T tokens of self.x / self.logits into self.out[:T]. `stream` must be torch's
        current stream (the collectives run there); `events` as MoeLayer.experts; `phases`: len(PHASES) + 1 CUDA
        events recorded between the steps (for a per-phase breakdown)."""
        if T > self.max_tokens:
            raise ValueError(f"T {T} > max_tokens {self.max_tokens}")
        o, G, k, P = self.ops, self.G, self.k, T * self.k
        mark = (lambda i: phases[i].record()) if phases else (lambda i: None)
        mark(0)
        o.router(self.logits, T, self.E, k, self.ids, self.w)
        o.scatter(self.ids, P, self.E, self.sorted_pairs[:P], self.offset)
        o.pack(self.x, self.ids, k, self.sorted_pairs, P, self.offset, self.nl, G, self.send_x, self.send_e,
               self.counts[:G])
        mark(1)
        self.dist.all_to_all_single(self.counts[G:], self.counts[:G], group=self.group)
        c = self.counts.cpu().tolist()          # the split sizes: the one host read of a step
        send_c, recv_c = c[:G], c[G:]
        S, R = sum(send_c), sum(recv_c)
        self._a2a(self.recv_x[:R], self.send_x[:S], recv_c, send_c)
        self._a2a(self.recv_e[:R], self.send_e[:S], recv_c, send_c)
        mark(2)
        o.scatter(self.recv_e[:R], R, self.nl, self.sorted_loc[:R], self.off_loc)
        mark(3)
        o.experts(self.recv_x, R, events)
        mark(4)
        o.rows_scatter(self.y_rows, self.sorted_loc, R, self.y_recv, R)
        self._a2a(self.y_back[:S], self.y_recv[:R], send_c, recv_c)
        mark(5)
        o.gather(self.y_back, self.sorted_pairs, S, self.w, T, k, self.out)
        mark(6)
        self.last = {"R": R, "sent": S, "send_counts": send_c, "recv_counts": recv_c}

    # ------------------------------------------------------------------ accounting (this rank)
    def live_experts(self):
        off = self.off_loc.cpu().numpy()
        return int((np.diff(off) > 0).sum())

    def expert_bytes(self):
        return self.ops.local.expert_bytes()

    def time_prep_step(self, T, n=5):
        """The local pass's gate_up input rotation alone (ms), over the rows the last step received."""
        R = self.last["R"]
        return self.ops.local.time_prep(R, R, x_ptr=self.recv_x.data_ptr(), top_k=1, n=n)

    def expert_flops(self, rows):
        return self.ops.local.expert_flops(rows)

    def band_name(self, op, T):
        return self.ops.local.band_name(op, self.last["R"]) + " (rows received by this rank)"

    def launches_per_step(self, T):
        return self.ops.kernels(T, self.k, self.E, self.last["R"])

    def exchange_bytes(self):
        """Bytes this rank sent to other ranks in the last step (rows out and back, ids), its own rows excluded."""
        if "send_counts" not in self.last:
            return 0
        own_s, own_r = self.last["send_counts"][self.rank], self.last["recv_counts"][self.rank]
        rows_out = self.last["sent"] - own_s
        rows_back = self.last["R"] - own_r
        return rows_out * (2 * self.H + 4) + rows_back * 2 * self.H
