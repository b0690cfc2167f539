"""tp.py -- the width ("column-block") tensor split of the routed-MoE layer: the reference's alternate multi-GPU mode.

Every rank holds a slice of EVERY expert's intermediate width in whole 128-column blocks, routes every token (the
router and the routed tokens are replicated), runs gate_up and down over all routed rows on its slice and gathers a
PARTIAL of the layer's output; the partials summed over the ranks are the layer's output
(architectures/qwen4exp_exl3/rad_block_moe_exl3.h:438-470). The slice rule is the reference's
(architectures/qwen4exp_exl3/qwen4exp_exl3.cpp:296-301, 576-634): an even cut when the blocks divide over the ranks,
otherwise two classes by expert parity (four by number mod 4 at four ranks) whose cuts rotate the extra block, and
more ranks than blocks refused.

A slice of an expert is an EXL3 weight of its own: gate_up's output rows [lo, hi) of the gate and of the up half,
down's input columns [lo, hi). Both rotations stay local to a 128-column block (the output rotation of gate_up and
h_rot; down's input rotation), so the slice's planes are the full planes cut: the codes plane's rows (gate_up) or
columns (down), svh's gate_up rows and dn_suh's columns; suh, suh.1 and down's svh whole. In the stored tile-stream
record ([cols/16][rows/16][16K] per record, a stacked gate_up being the gate record then the up record) the same
cut is a slice of whole tiles.

The sum runs on the device: over NCCL (the engine's all_reduce) or fused into the gather over peer memory
(exl3b200_tp_gather_rs / tp_reduce / tp_pull: each token's partial stored into the rank that reduces it, the reduced
slices pulled by every rank), which needs no host synchronisation, so a step is capturable in a CUDA graph."""
import ctypes as C

import numpy as np

BLOCK = 128          # the reference's split granule: an expert's width is cut in whole 128-column blocks


def block_slice(nb, world, place):
    """Blocks [b0, b1) that place `place` takes when nb blocks are cut over `world` ranks, the first nb % world
    places one block wider (qwen4exp_exl3.cpp:296-301)."""
    base, extra = divmod(nb, world)
    b0 = place * base + min(place, extra)
    return b0, b0 + base + (1 if place < extra else 0)


def width_slices(width, world, rank, block=BLOCK):
    """This rank's columns of every expert's width, one (lo, hi) a class: expert e takes class e % len(result)
    (qwen4exp_exl3.cpp:576-634).

    - the blocks divide evenly over the ranks: one class, [rank * w, (rank + 1) * w);
    - otherwise two classes by expert parity, class q's cut placing this rank at (rank - q) mod world, so the rank
      taking the extra block alternates with the parity; at four ranks four classes by number mod 4, the same cut
      shifted by the class;
    - more ranks than blocks: refused (some rank would hold no slice of an expert)."""
    if width <= 0 or width % block:
        raise ValueError(f"width {width} is not a whole number of {block}-column blocks")
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    nb = width // block
    if nb % world == 0:
        w = width // world
        return [(rank * w, (rank + 1) * w)]
    if world > nb:
        raise ValueError(f"{world} ranks is more ranks than an expert has {block}-column blocks ({nb}): some rank "
                         f"would hold no slice of it; split over {nb} or fewer")
    n_class = 4 if world == 4 else 2
    return [tuple(b * block for b in block_slice(nb, world, (rank - q + world) % world)) for q in range(n_class)]


# ------------------------------------------------------------------------------------------ cutting the planes
def _cut_cols(codes, bits, lo, hi):
    """Columns [lo, hi) of a canonical uK codes plane (rows of ceil(cols*K/8) bytes, LSB first); lo, hi multiples
    of 8 so the cut falls on byte boundaries."""
    if lo % 8 or hi % 8:
        raise ValueError("a column cut off a byte boundary")
    return np.ascontiguousarray(codes[:, lo * bits // 8: hi * bits // 8])


def slice_planes(p, width, bits_gu, bits_dn, lo, hi):
    """One expert's canonical planes (a gate_up + down pair: codes [2W, H], suh, suh1 [H], svh [2W], dn_suh [W],
    dn_codes [H, W], dn_svh [H]) cut to width columns [lo, hi)."""
    W = width
    q = {"codes": np.ascontiguousarray(np.concatenate([p["codes"][lo:hi], p["codes"][W + lo:W + hi]])),
         "suh": p["suh"], "suh1": p["suh1"],
         "svh": np.ascontiguousarray(np.concatenate([p["svh"][lo:hi], p["svh"][W + lo:W + hi]])),
         "dn_suh": np.ascontiguousarray(p["dn_suh"][lo:hi]),
         "dn_codes": _cut_cols(p["dn_codes"], bits_dn, lo, hi), "dn_svh": p["dn_svh"]}
    return q


def slice_gu_record(rec, hidden, width, bits, lo, hi):
    """A stacked gate_up record (gate then up, each [H/16][W/16][16K] u16; leading dims kept) cut to output rows
    [lo, hi) of each half: whole tiles. Works on numpy arrays and torch tensors."""
    lead = tuple(rec.shape[:-1])
    r = rec.reshape(lead + (2, hidden // 16, width // 16, 16 * bits))[..., lo // 16:hi // 16, :]
    return r.reshape(lead + (-1,))


def slice_dn_record(rec, hidden, width, bits, lo, hi):
    """A down record ([W/16][H/16][16K] u16; leading dims kept) cut to input columns [lo, hi): whole tile rows."""
    lead = tuple(rec.shape[:-1])
    r = rec.reshape(lead + (width // 16, hidden // 16, 16 * bits))[..., lo // 16:hi // 16, :, :]
    return r.reshape(lead + (-1,))


def load_slice(dst, src, lo, hi):
    """Fill `dst` (a MoeLayer of width hi - lo over the same experts) with columns [lo, hi) of `src`'s experts."""
    W, H = src.W, src.H
    if dst.W != hi - lo or dst.H != H or dst.n_local != src.n_local:
        raise ValueError("the slice layer's shapes do not match the cut")
    dst.gu_rec.copy_(slice_gu_record(src.gu_rec, H, W, src.bits_gu, lo, hi))
    dst.dn_rec.copy_(slice_dn_record(src.dn_rec, H, W, src.bits_dn, lo, hi))
    dst.suh.copy_(src.suh)
    dst.suh1.copy_(src.suh1)
    dst.svh_gu.copy_(src.torch.cat([src.svh_gu[:, lo:hi], src.svh_gu[:, W + lo:W + hi]], 1))
    dst.dn_suh.copy_(src.dn_suh[:, :, lo:hi])
    dst.svh_dn.copy_(src.svh_dn)


def load_classes(dst, src, cuts):
    """Fill `dst` (a ClassMoeLayer over src's experts) with the uneven cut: class c (experts c, c + n, ... of src,
    n = len(cuts)) holds columns cuts[c] of those experts."""
    import torch
    n, W, H = len(cuts), src.W, src.H
    if dst.n_class != n or dst.widths != [hi - lo for lo, hi in cuts] or dst.n_local != src.n_local:
        raise ValueError("the class layer's shapes do not match the cut")
    for c, (lo, hi) in enumerate(cuts):
        t = dst.cls[c]
        idx = torch.arange(c, src.n_local, n, device=src.dev)
        t["gu_rec"].copy_(slice_gu_record(src.gu_rec[idx], H, W, src.bits_gu, lo, hi))
        t["dn_rec"].copy_(slice_dn_record(src.dn_rec[idx], H, W, src.bits_dn, lo, hi))
        t["suh"].copy_(src.suh[idx])
        t["suh1"].copy_(src.suh1[idx])
        t["svh_gu"].copy_(torch.cat([src.svh_gu[idx, lo:hi], src.svh_gu[idx, W + lo:W + hi]], 1))
        t["dn_suh"].copy_(src.dn_suh[idx][:, :, lo:hi])
        t["svh_dn"].copy_(src.svh_dn[idx])


# ------------------------------------------------------------------------------------------ the layer
class TpLayer:
    """The routed-MoE layer with every expert's width split over `world` ranks. Every rank builds the same seeded
    full-width experts (or takes `full`, a MoeLayer) and keeps its slice; x and logits are the same on every rank
    (replicated); forward leaves the whole layer's output in `out` on every rank."""

    PHASES = ("route", "experts", "all-reduce")

    def __init__(self, plugin=None, *, rank, world, n_expert, hidden, width, top_k, bits_gu=3, bits_dn=4,
                 codebook="mul1", max_tokens=2048, seed=0, group=None, device="cuda", full=None, transport="p2p"):
        import torch
        import torch.distributed as dist
        from . import load_plugin
        from .layer import MoeLayer
        slices = width_slices(width, world, rank)
        self.cuts = slices
        self.lo, self.hi = slices[0]
        if transport not in ("nccl", "p2p"):
            raise ValueError(f"transport {transport!r}")
        self.torch, self.dist, self.group = torch, dist, group
        self.rank, self.G, self.transport = rank, world, transport
        self.E, self.H, self.W, self.k = n_expert, hidden, width, top_k
        self.max_tokens = max_tokens
        dev = self.dev = torch.device(device) if not isinstance(device, torch.device) else device
        plugin = plugin or load_plugin()
        kw = dict(n_expert=n_expert, hidden=hidden, top_k=top_k, bits_gu=bits_gu, bits_dn=bits_dn,
                  codebook=codebook, device=dev)
        src = full if full is not None else MoeLayer(plugin, width=width, max_tokens=1, seed=seed, **kw)
        if len(slices) == 1:
            self.layer = MoeLayer(plugin, width=self.hi - self.lo, max_tokens=max_tokens, seed=seed + 7919, **kw)
            load_slice(self.layer, src, self.lo, self.hi)
        else:
            # the uneven cut: this rank's experts in classes (parity, or number mod 4) of different widths
            from .layer import ClassMoeLayer
            self.layer = ClassMoeLayer(plugin, widths=[hi - lo for lo, hi in slices], max_tokens=max_tokens,
                                       seed=seed + 7919, **kw)
            load_classes(self.layer, src, slices)
        del src
        L = self.layer
        self.nat = L.native
        self.x, self.logits, self.out = L.x, L.logits, L.out
        self.win = None
        if transport == "p2p":
            # the window laid out by the library (exl3b200_tp_window_layout): part [world][s_cap][H] f32 |
            # red [s_cap][H] f32 | ctl [world][8] u32 | done [4] u32, s_cap = ceil(max_tokens / world)
            self.s_cap = (max_tokens + world - 1) // world
            offs, nbytes = self.nat.tp_window_layout(world, max_tokens, hidden)
            from .ep import IpcWindow
            self.win = IpcWindow(self.nat, dist, group, rank, world, offs, nbytes, dev)
            self.epoch_dev = torch.zeros(1, dtype=torch.int32, device=dev)
            self.status = torch.zeros(1, dtype=torch.int32, device=dev)
            if getattr(L, "c_layer", False):
                # the even cut: the whole step is one call of the library's C driver (exl3b200_tp_step_forward)
                from .native import TpDesc
                d = self.desc = TpDesc()
                d.layer = L.desc
                d.rank, d.world, d.max_tokens = rank, world, max_tokens
                d.window, d.peers = self.win.base, self.win.peers.data_ptr()
                for i, o in enumerate(offs):
                    d.offs[i] = o
                d.epoch, d.status = self.epoch_dev.data_ptr(), self.status.data_ptr()

    def forward(self, T, stream=None, events=None, phases=None, x=None, logits=None, out=None):
        """The layer over the first T tokens of x / logits (self.x / self.logits by default; the same on every
        rank) into out[:T] (f32 [T, H], self.out by default), on torch's current stream. `events`, `phases` as
        EpLayer.forward."""
        if T > self.max_tokens:
            raise ValueError(f"T {T} > max_tokens {self.max_tokens}")
        L, nat, k = self.layer, self.nat, self.k
        st = self.torch.cuda.current_stream().cuda_stream
        x = self.x if x is None else x
        logits = self.logits if logits is None else logits
        out = self.out if out is None else out
        rows = T * k
        if self.win is not None and getattr(L, "c_layer", False):
            from .native import marks_array
            d = self.desc
            d.layer = L.desc                      # the slice layer's current weight set
            marks = marks_array(list(phases or [None] * 4) + list(events or [None] * 3)) \
                if (phases or events) else None
            nat.tp_step_forward(d, L.bufs, x.data_ptr(), logits.data_ptr(), T, out.data_ptr(), out.shape[1], st,
                                marks)
            return
        # the uneven cut (class rows) or NCCL: the same steps composed here
        mark = (lambda i: phases[i].record()) if phases else (lambda i: None)
        mark(0)
        if self.win is not None:
            nat.p2p_begin(self.epoch_dev.data_ptr(), st)
        nat.router_scatter(logits.data_ptr(), T, self.E, k, L.ids.data_ptr(), L.w.data_ptr(), self.E, 0,
                           L.sorted_tok.data_ptr(), L.offset.data_ptr(), L.scatter_work.data_ptr(), st)
        mark(1)
        L.experts(T, rows, st, x_ptr=x.data_ptr(), events=events)
        mark(2)
        if self.win is None:
            nat.moe_gather(L.y_rows.data_ptr(), self.H, L.sorted_tok.data_ptr(), rows, L.w.data_ptr(), T, k, self.H,
                           out.data_ptr(), L.gather_work.data_ptr(), st)
            if self.G > 1:
                self.dist.all_reduce(out[:T], group=self.group)
        else:
            w, ep = self.win, self.epoch_dev.data_ptr()
            nat.tp_gather_rs(L.y_rows.data_ptr(), self.H, L.sorted_tok.data_ptr(), rows, L.w.data_ptr(), T, k,
                             self.H, L.gather_work.data_ptr(), w.peers.data_ptr(), w.offs, self.rank, self.G,
                             self.s_cap, ep, self.status.data_ptr(), st)
            nat.tp_reduce(w.peers.data_ptr(), w.offs, self.rank, self.G, T, self.H, self.s_cap, ep, st)
            nat.tp_pull(w.peers.data_ptr(), w.offs, self.rank, self.G, T, self.H, self.s_cap, out.data_ptr(),
                        out.shape[1], ep, self.status.data_ptr(), st)
        mark(3)

    def check(self):
        """Raise if a peer's partials or reduced slice did not arrive within the wait limit in the last step
        (reads the status word and the device error word: synchronises)."""
        if self.win is None:
            return
        if int(self.status.item()) != 0:
            raise RuntimeError("width split: a peer's partials did not arrive within the wait limit")
        err = self.nat.read_error(clear=False)
        if err & 8:
            raise RuntimeError(f"width split: device error word {err:#x}")

    def close(self):
        """Collective: release the peer-memory window (p2p transport)."""
        if self.win is not None:
            self.win.close()
            self.win = None

    # ------------------------------------------------------------------ accounting (this rank)
    def tokens_per_step(self, T):
        return T                                   # the tokens are replicated: the group serves T a step

    def live_experts(self):
        return self.layer.live_experts()

    def expert_bytes(self):
        return self.layer.expert_bytes()           # this rank's slice of one expert

    def expert_flops(self, rows):
        return self.layer.expert_flops(rows)

    def time_prep_step(self, T, n=5):
        return self.layer.time_prep_step(T, n=n)

    def band_name(self, op, T):
        return self.layer.band_name(op, T) + f" (width slices {self.cuts})"

    def launches_per_step(self, T):
        L = self.layer
        n = L.route_launches(T) + L.expert_launches(T)
        # peer memory: begin, the inverse map, gather_rs, reduce, pull; NCCL: the gather (its all-reduce is NCCL's)
        return n + (5 if self.win is not None else L.gather_launches(T))

    def exchange_bytes(self, T):
        """Bytes this rank sends over NVLink a step (p2p): its partials of the other ranks' slices, then the other
        ranks' pulls of its reduced slice."""
        s = (T + self.G - 1) // self.G
        own = max(0, min(s, T - self.rank * s))
        return (T - own) * self.H * 4 + (self.G - 1) * own * self.H * 4
