"""layer.py -- one routed-MoE layer on the B200 library: router -> scatter -> moe_exl3_gate_up -> moe_exl3_down ->
gather, every step a kernel of libexl3b200.so, the two expert ops called through the plugin rows exactly as the
engine calls them (RadArgs, RadStream; rad_block_moe_exl3.h's pass issues the same sequence).

Weights are synthetic and resident in HBM: each expert's codes as its stored tile-stream record (uniform random
u16 words: every symbol sequence is a valid trellis, so a uniform record is a uniform canonical plane), suh / suh.1
random +-1 fp16, svh +-|N(0,1)| * 0.02 fp16 (the per-channel scale lives in svh). h crosses
between the two ops rotated (h_rot = 1, docs/OPS-exl3.md "EPI 1").

Expert parallelism: `expert_base` / `n_local` select the experts this rank holds ([base, base + n_local)); the
layer then serves rows whose expert is local (the dispatch in bench.py's multi-GPU path sends them here)."""
import ctypes as C

import numpy as np

from . import cases as X
from . import rad
from .native import Native


class MoeLayer:
    def __init__(self, plugin, *, n_expert=512, hidden=2048, width=512, top_k=10, bits_gu=3, bits_dn=4,
                 codebook="mul1", max_tokens=2048, seed=0, device="cuda", n_local=None, expert_base=0,
                 max_rows=None):
        import torch
        self.torch = torch
        self.plugin, self.native = plugin, Native(plugin.path)
        self.E, self.H, self.W, self.k = n_expert, hidden, width, top_k
        self.n_local = n_local or n_expert
        self.base = expert_base
        self.bits_gu, self.bits_dn, self.codebook = bits_gu, bits_dn, codebook
        self.max_tokens = max_tokens
        self.max_rows = max_rows or max_tokens * top_k
        dev = self.dev = torch.device(device)
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        E, H, W = self.n_local, hidden, width
        # ---- weights: records and scales, resident
        self.gu_bytes = 2 * W * H * bits_gu // 8          # stacked gate + up record
        self.dn_bytes = H * W * bits_dn // 8
        self.gu_rec = torch.randint(-32768, 32768, (E, self.gu_bytes // 2), generator=g, device=dev,
                                    dtype=torch.int32).to(torch.int16)
        self.dn_rec = torch.randint(-32768, 32768, (E, self.dn_bytes // 2), generator=g, device=dev,
                                    dtype=torch.int32).to(torch.int16)

        def sign(*shape):
            return (torch.randint(0, 2, shape, generator=g, device=dev) * 2 - 1).to(torch.float16)

        def svh(*shape):
            return (sign(*shape).float() * torch.randn(shape, generator=g, device=dev).abs() * 0.02).to(torch.float16)

        self.suh, self.suh1 = sign(E, 1, H), sign(E, 1, H)
        self.svh_gu = svh(E, 2 * W, 1)
        self.dn_suh = sign(E, 1, W)
        self.svh_dn = svh(E, H, 1)
        self.gu_tab = torch.tensor([self.gu_rec[e].data_ptr() for e in range(E)], dtype=torch.int64, device=dev)
        self.dn_tab = torch.tensor([self.dn_rec[e].data_ptr() for e in range(E)], dtype=torch.int64, device=dev)
        # ---- activations and routing buffers (the largest pass)
        T, R = max_tokens, self.max_rows
        self.x = torch.empty((T, H), dtype=torch.float16, device=dev)
        self.logits = torch.empty((T, n_expert), dtype=torch.float32, device=dev)
        self.out = torch.empty((T, H), dtype=torch.float32, device=dev)
        self.out_bf16 = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        self.rec_dtype = self._stored_dtype()
        self._args = {}
        # a plain layer (a pass is at most max_tokens * top_k sorted rows) runs as ONE call of the library's C layer
        # (exl3b200_moe_layer_forward) over one device block the library carves into every buffer; the routing and
        # row buffers below are views of that block. A layer whose passes are capacity-sized (expert parallelism's
        # local pass) keeps buffers of its own and drives the plugin rows itself.
        self.c_layer = R == T * top_k
        if self.c_layer:
            from .native import LayerDesc
            d = self.desc = LayerDesc()
            d.n_expert, d.n_local, d.expert_base = n_expert, self.n_local, expert_base
            d.hidden, d.width, d.top_k = H, W, top_k
            d.bits_gu, d.bits_dn, d.codebook = bits_gu, bits_dn, {"3inst": 0, "mcg": 1, "mul1": 2}[codebook]
            d.gu_codes, d.dn_codes = self.gu_tab.data_ptr(), self.dn_tab.data_ptr()
            d.suh, d.suh1, d.svh_gu = self.suh.data_ptr(), self.suh1.data_ptr(), self.svh_gu.data_ptr()
            d.dn_suh, d.svh_dn = self.dn_suh.data_ptr(), self.svh_dn.data_ptr()
            nbytes = self.native.layer_work_bytes(d, T)
            self.work = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            b = self.bufs = self.native.layer_carve(d, T, self.work.data_ptr(), nbytes)
            base = self.work.data_ptr()

            def view(ptr, n, dt, shape):
                off = ptr - base
                nb = n * torch.tensor([], dtype=dt).element_size()
                return self.work[off:off + nb].view(dt).view(shape)

            self.ids = view(b.ids, T * top_k, torch.int32, (T, top_k))
            self.w = view(b.w, T * top_k, torch.float32, (T, top_k))
            self.sorted_tok = view(b.sorted_tok, R, torch.int32, (R,))
            self.offset = view(b.expert_offset, self.n_local + 1, torch.int32, (self.n_local + 1,))
            self.h = view(b.h, R * W, torch.float16, (R, W))
            self.y_rows = view(b.y_rows, R * H, torch.bfloat16, (R, H))
            self.scatter_work = view(b.scatter_work, 16, torch.uint8, (16,))
            self.gather_work = view(b.gather_work, 16, torch.uint8, (16,))
        else:
            self.ids = torch.empty((T, top_k), dtype=torch.int32, device=dev)
            self.w = torch.empty((T, top_k), dtype=torch.float32, device=dev)
            self.sorted_tok = torch.empty(R, dtype=torch.int32, device=dev)
            self.offset = torch.empty(self.n_local + 1, dtype=torch.int32, device=dev)
            self.scatter_work = torch.empty(max(16, self.native.scatter_work_bytes(R, self.n_local)),
                                            dtype=torch.uint8, device=dev)
            self.h = torch.empty((R, W), dtype=torch.float16, device=dev)
            self.y_rows = torch.empty((R, H), dtype=torch.bfloat16, device=dev)
            self.gather_work = torch.empty(max(16, self.native.gather_work_bytes(T, top_k)), dtype=torch.uint8,
                                           device=dev)

    def load_experts(self, src, base):
        """Copy experts [base, base + n_local) of `src` (a layer of the same shapes holding more experts) into this
        layer's resident weights: the records, suh, suh.1, svh and the down scales."""
        sl = slice(base, base + self.n_local)
        for name in ("gu_rec", "dn_rec", "suh", "suh1", "svh_gu", "dn_suh", "svh_dn"):
            getattr(self, name).copy_(getattr(src, name)[sl])

    # ------------------------------------------------------------------ weight sets (a stack of layers)
    WEIGHTS = ("gu_rec", "dn_rec", "suh", "suh1", "svh_gu", "dn_suh", "svh_dn", "gu_tab", "dn_tab")

    def add_weight_set(self, seed):
        """Another layer's weights for this layer's experts (seeded as the constructor seeds them), kept resident
        beside the others; returns its index. A stack of layers shares one set of activation buffers and swaps
        weights with use_weight_set."""
        torch, dev, E, H, W = self.torch, self.dev, self.n_local, self.H, self.W
        if not hasattr(self, "_sets"):
            self._sets = [{n: getattr(self, n) for n in self.WEIGHTS}]
            self._retired = []
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        rnd = lambda nb: torch.randint(-32768, 32768, (E, nb // 2), generator=g, device=dev,  # noqa: E731
                                       dtype=torch.int32).to(torch.int16)
        sign = lambda *sh: (torch.randint(0, 2, sh, generator=g, device=dev) * 2 - 1).to(torch.float16)  # noqa: E731
        svh = lambda *sh: (sign(*sh).float() * torch.randn(sh, generator=g, device=dev).abs() * 0.02  # noqa: E731
                           ).to(torch.float16)
        st = {"gu_rec": rnd(self.gu_bytes), "dn_rec": rnd(self.dn_bytes), "suh": sign(E, 1, H), "suh1": sign(E, 1, H),
              "svh_gu": svh(E, 2 * W, 1), "dn_suh": sign(E, 1, W), "svh_dn": svh(E, H, 1)}
        st["gu_tab"] = torch.tensor([st["gu_rec"][e].data_ptr() for e in range(E)], dtype=torch.int64, device=dev)
        st["dn_tab"] = torch.tensor([st["dn_rec"][e].data_ptr() for e in range(E)], dtype=torch.int64, device=dev)
        self._sets.append(st)
        return len(self._sets) - 1

    def use_weight_set(self, i):
        """Point the layer (its C description and its per-op launch arguments) at weight set i. Launch arguments
        built for the previous set are kept alive with their scratch, so a CUDA graph captured over several sets
        still owns every buffer its kernels use."""
        for n, t in self._sets[i].items():
            setattr(self, n, t)
        if self.c_layer:
            d = self.desc
            d.gu_codes, d.dn_codes = self.gu_tab.data_ptr(), self.dn_tab.data_ptr()
            d.suh, d.suh1, d.svh_gu = self.suh.data_ptr(), self.suh1.data_ptr(), self.svh_gu.data_ptr()
            d.dn_suh, d.svh_dn = self.dn_suh.data_ptr(), self.svh_dn.data_ptr()
        self._retired.append(self._args)
        self._args = {}

    # ------------------------------------------------------------------ the stored codes dtype
    def _stored_dtype(self):
        """Ask the gate_up row's layout hook what it stores a codes plane as (its RadLayout dtype)."""
        row = self.plugin.row("moe_exl3_gate_up")
        params = self._params_gu(self.max_tokens)
        P, nP, keep = rad.make_params(params)
        enc = X.encoding(self.bits_gu, self.codebook, stacked=True)
        sel = C.c_int(0)
        pt = rad.tensor(0, rad.DT_UK[self.bits_gu], [2 * self.W, self.H])
        L = rad.RadLayout()
        rc = row.layout(P, nP, 1, C.byref(enc), C.byref(sel), C.byref(pt), 1, C.byref(L))
        if rc != 0 or L.bytes != self.gu_bytes:
            raise RuntimeError(f"layout hook: rc {rc}, bytes {L.bytes} (expected {self.gu_bytes})")
        return int(L.dtype)

    def _params_gu(self, M):
        return {"M": M, "N": 2 * self.W, "K": self.H, "n_expert": self.n_local, "top_k": self.k,
                "dtype": f"exl3k{self.bits_gu}", "codebook": self.codebook, "h_rot": 1, "a_rot": 0}

    def _params_dn(self, M):
        return {"M": M, "N": self.H, "K": self.W, "n_expert": self.n_local, "top_k": self.k,
                "dtype": f"exl3k{self.bits_dn}", "codebook": self.codebook, "h_rot": 1}

    # ------------------------------------------------------------------ the RadArgs of one pass size
    def _build(self, T, rows, x_ptr=None, top_k=None, M=None):
        """RadArgs of gate_up and down for a pass of `rows` sorted rows over `T` input rows."""
        key = (T, rows, x_ptr, top_k, M)
        if key in self._args:
            return self._args[key]
        if len(self._args) >= 32:     # pass sizes that vary step to step (expert parallelism): keep the cache bounded
            self._args.clear()
        k = top_k or self.k
        E, H, W = self.n_local, self.H, self.W
        keep = []
        M = M or T

        def args(params, tensors):
            P, nP, kp = rad.make_params(params)
            arr = (rad.RadTensor * len(tensors))(*tensors)
            a = rad.RadArgs()
            a.t, a.n_t, a.p, a.n_p, a.world_size = arr, len(tensors), P, nP, 1
            keep.extend([P, kp, arr])
            return a

        absent = rad.RadTensor()
        xp = x_ptr or self.x.data_ptr()
        pg = self._params_gu(M)
        pg["top_k"] = k
        gu_t = [rad.tensor(xp, rad.DT["f16"], [T, H]),
                rad.tensor(self.gu_tab.data_ptr(), self.rec_dtype, [E, 2 * W, H], [0, H, 1]),
                rad.tensor(self.suh.data_ptr(), rad.DT["f16"], [E, 1, H]),
                rad.tensor(self.suh1.data_ptr(), rad.DT["f16"], [E, 1, H]),
                rad.tensor(self.svh_gu.data_ptr(), rad.DT["f16"], [E, 2 * W, 1]),
                rad.tensor(self.dn_suh.data_ptr(), rad.DT["f16"], [E, 1, W]),
                rad.tensor(self.sorted_tok.data_ptr(), rad.DT["i32"], [rows]),
                rad.tensor(self.offset.data_ptr(), rad.DT["i32"], [E + 1]),
                absent, absent, absent, absent, absent,
                rad.tensor(self.h.data_ptr(), rad.DT["f16"], [rows, W])]
        pd = self._params_dn(M)
        pd["top_k"] = k
        dn_t = [rad.tensor(self.h.data_ptr(), rad.DT["f16"], [rows, W]),
                rad.tensor(self.dn_tab.data_ptr(), self.rec_dtype, [E, H, W], [0, W, 1]),
                rad.tensor(self.dn_suh.data_ptr(), rad.DT["f16"], [E, 1, W]),
                rad.tensor(self.svh_dn.data_ptr(), rad.DT["f16"], [E, H, 1]),
                rad.tensor(self.sorted_tok.data_ptr(), rad.DT["i32"], [rows]),
                rad.tensor(self.offset.data_ptr(), rad.DT["i32"], [E + 1]),
                absent, absent, absent,
                rad.tensor(self.y_rows.data_ptr(), rad.DT["bf16"], [rows, H])]
        a_gu, a_dn = args(pg, gu_t), args(pd, dn_t)
        # the scratch each row's hook asks for (the tensor-core band's rotated input rows): one buffer a row, grown to
        # the largest pass seen and shared by every pass size and weight set (the passes run one after another on
        # one stream); a buffer that is outgrown stays alive for the graphs that captured it
        if not hasattr(self, "_scratch"):
            self._scratch, self._old_scratch = {}, []
        for row_name, a in (("moe_exl3_gate_up", a_gu), ("moe_exl3_down", a_dn)):
            row = self.plugin.row(row_name)
            need = int(row.scratch(C.byref(a))) if row.scratch else 0
            if need > 0:
                buf = self._scratch.get(row_name)
                if buf is None or buf.numel() < need:
                    if buf is not None:
                        self._old_scratch.append(buf)
                    buf = self._scratch[row_name] = self.torch.empty(need, dtype=self.torch.uint8, device=self.dev)
                a.scratch, a.scratch_bytes = buf.data_ptr(), need
        res = (a_gu, a_dn, keep)
        self._args[key] = res
        return res

    # ------------------------------------------------------------------ one pass
    def experts(self, T, rows, stream, x_ptr=None, top_k=None, M=None, events=None, down_row_dst=None, live=False):
        """gate_up then down over the sorted rows already in sorted_tok / offset. `events`: three
        torch.cuda.Event recorded before gate_up, between the two and after down (on the current stream)."""
        if rows == 0:                 # nothing routed here: no launch, the events still mark the (empty) ops
            for e in events or ():
                e.record()
            return
        a_gu, a_dn, _ = self._build(T, rows, x_ptr, top_k, M)
        if events:
            events[0].record()
        if live:
            # the live rows only (a capacity-sized pass whose live count is on the device): nothing else is touched
            self.native.moe_op_live(C.addressof(a_gu), 0, None, stream)
            if events:
                events[1].record()
            self.native.moe_op_live(C.addressof(a_dn), 1, down_row_dst, stream)
            if events:
                events[2].record()
            return
        rc = self.plugin.row("moe_exl3_gate_up").launch(C.byref(a_gu), stream)
        if rc != 0:
            raise RuntimeError(f"moe_exl3_gate_up launch: {rc}")
        if events:
            events[1].record()
        if down_row_dst:
            # down writing each output row at its address in a device table (the expert-parallel combine)
            self.native.moe_down_rows(C.addressof(a_dn), down_row_dst, stream)
        else:
            rc = self.plugin.row("moe_exl3_down").launch(C.byref(a_dn), stream)
            if rc != 0:
                raise RuntimeError(f"moe_exl3_down launch: {rc}")
        if events:
            events[2].record()

    def time_prep(self, T, rows, x_ptr=None, top_k=None, n=5, sorted_tok=None, offset=None):
        """Mean device time (ms, CUDA events on the current stream) of the gate_up input rotation alone: the
        moe_exl3_prep_gu row over the same sorted rows, i.e. the k_prep launch the tensor-core gate_up runs first.
        The bench subtracts it from the gate_up op to time k_gemm_tc by itself. `sorted_tok`, `offset`: the routing
        of a pass whose buffers live elsewhere (device addresses; this layer's by default)."""
        torch = self.torch
        if rows == 0:
            return 0.0
        k = top_k or self.k
        if getattr(self, "_xr", None) is None or self._xr.shape[0] < rows:
            self._xr = torch.empty((rows, 2 * self.H), dtype=torch.float16, device=self.dev)
        absent = rad.RadTensor()
        E, H = self.n_local, self.H
        P, nP, kp = rad.make_params({"M": T, "K": H, "n_expert": E, "top_k": k, "dtype": f"exl3k{self.bits_gu}"})
        ts = [rad.tensor(x_ptr or self.x.data_ptr(), rad.DT["f16"], [T, H]),
              rad.tensor(self.suh.data_ptr(), rad.DT["f16"], [E, 1, H]),
              rad.tensor(self.suh1.data_ptr(), rad.DT["f16"], [E, 1, H]),
              rad.tensor(sorted_tok or self.sorted_tok.data_ptr(), rad.DT["i32"], [rows]),
              rad.tensor(offset or self.offset.data_ptr(), rad.DT["i32"], [E + 1]),
              absent, absent,
              rad.tensor(self._xr.data_ptr(), rad.DT["f16"], [rows, 2 * H])]
        arr = (rad.RadTensor * len(ts))(*ts)
        a = rad.RadArgs()
        a.t, a.n_t, a.p, a.n_p, a.world_size = arr, len(ts), P, nP, 1
        row = self.plugin.row("moe_exl3_prep_gu")
        stream = torch.cuda.current_stream().cuda_stream
        for _ in range(2):
            if row.launch(C.byref(a), stream) != 0:
                raise RuntimeError("moe_exl3_prep_gu launch failed")
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            row.launch(C.byref(a), stream)
        e1.record()
        torch.cuda.synchronize()
        del kp
        return e0.elapsed_time(e1) / n

    def _tc(self, op, rows):
        """The library's band rule (exl3b200_host.c tc_band): the tensor-core band once the pass makes 64 of its units
        ((live experts + rows / 64) x 256-row output pairs), or 8 of them while the live experts average 16 rows."""
        live = min(self.n_local, rows)
        if live <= 0:
            return False
        pairs = (2 * self.W if op == "gate_up" else self.H) // 256
        units = (live + rows // 64) * pairs
        return units >= 64 or (rows // live >= 16 and units >= 8)

    def band_name(self, op, T, rows=None):
        """Which kernels serve one op at T tokens, or over `rows` sorted rows (gate_up's input rotation runs once a
        row in k_prep on the tensor-core band)."""
        rows = T * self.k if rows is None else rows
        tc = self._tc(op, rows)
        if op == "gate_up":
            return "moe_exl3_gate_up row: k_prep + k_gemm_tc" if tc else "moe_exl3_gate_up row: k_gemm_skinny"
        return "moe_exl3_down row: k_gemm_tc" if tc else "moe_exl3_down row: k_gemm_skinny"

    def launches_per_step(self, T):
        """Kernels of this library one forward launches: router and scatter (one fused launch at up to 32 tokens; else
        the router and 1 small / 3 chunked sort launches), gate_up (+ prep on the tensor-core band), down, the gather
        (one launch up to 4096 rows; else the inverse map and the gather)."""
        return self.route_launches(T) + self.expert_launches(T) + self.gather_launches(T)

    def route_launches(self, T):
        rows = T * self.k
        if T <= 32 and rows <= 2048 and self.E <= 512 and self.n_local <= 1024:
            return 1
        return 1 + (1 if rows <= 2048 else 3)

    def expert_launches(self, T):
        return 2 + (1 if self._tc("gate_up", T * self.k) else 0)

    def gather_launches(self, T):
        return 1 if T * self.k <= 4096 and self.k <= 32 else 2

    def forward(self, T, stream, events=None, x=None, logits=None, out=None):
        """The whole layer over the first T tokens of self.x / self.logits into self.out (f32 [T, H]); `x`,
        `logits`, `out` (tensors of the same shapes) replace them, e.g. for double-buffered inputs. An `out` of
        dtype bfloat16 receives the layer's output in bf16 (the engine's hidden-state type). A plain layer is one
        call of the library's C layer; `events` (three CUDA events around gate_up and down) take the per-op path."""
        nat, rows = self.native, T * self.k
        o = out if out is not None else self.out
        if self.c_layer and not events:
            xx = x if x is not None else self.x
            lg = logits if logits is not None else self.logits
            nat.layer_forward(self.desc, self.bufs, xx.data_ptr(), lg.data_ptr(), T, o.data_ptr(),
                              3 if o.dtype == self.torch.bfloat16 else 1, stream)
            return
        xp = x.data_ptr() if x is not None else None
        lp = (logits if logits is not None else self.logits).data_ptr()
        op_ = o.data_ptr()
        nat.router_scatter(lp, T, self.E, self.k, self.ids.data_ptr(), self.w.data_ptr(), self.n_local, self.base,
                           self.sorted_tok.data_ptr(), self.offset.data_ptr(), self.scatter_work.data_ptr(), stream)
        self.experts(T, rows, stream, x_ptr=xp, events=events)
        gather = nat.moe_gather_bf16 if o.dtype == self.torch.bfloat16 else nat.moe_gather
        gather(self.y_rows.data_ptr(), self.H, self.sorted_tok.data_ptr(), rows, self.w.data_ptr(), T, self.k, self.H,
               op_, self.gather_work.data_ptr(), stream)

    # ------------------------------------------------------------------ accounting
    def time_prep_step(self, T, n=5):
        return self.time_prep(T, T * self.k, n=n)

    def expert_bytes(self):
        """Algorithmic bytes of one expert: both records plus every scale vector the pass reads."""
        H, W = self.H, self.W
        gu = self.gu_bytes + 2 * H * 2 + 2 * W * 2 + W * 2       # record, suh + suh.1, svh, dn_suh
        dn = self.dn_bytes + H * 2                                # record, svh (suh not read at h_rot 1)
        return gu, dn

    def expert_flops(self, rows):
        return 2 * rows * (2 * self.W * self.H + self.H * self.W)

    def live_experts(self):
        off = self.offset.cpu().numpy()
        return int((np.diff(off) > 0).sum())


class MoeBlock:
    """The MoE block pass (architectures/qwen4exp_exl3/rad_block_moe_exl3.h:1763-1967) through the library's C driver,
    exl3b200_moe_block_forward: the routed layer beside a shared EXL3 expert over every token, the gather folding the
    shared arm in through its one-column sigmoid gate, out[t] = routed[t] + sigmoid(x[t] . sgate_w) * shared(x[t]).
    `routed` is a MoeLayer (its weights and buffers), `shared` a one-expert MoeLayer (top_k 1) of width
    `shared_width`; sgate_w f16 [hidden], seeded N(0, 1/hidden). The protected experts and the norm / residual add
    around the block are not part of it."""

    def __init__(self, plugin, *, n_expert=512, hidden=2048, width=512, top_k=10, bits_gu=3, bits_dn=4,
                 shared_width=512, shared_bits=4, codebook="mul1", max_tokens=2048, seed=0, device="cuda"):
        import torch
        from .native import BlockBufs, BlockDesc
        self.torch = torch
        self.routed = MoeLayer(plugin, n_expert=n_expert, hidden=hidden, width=width, top_k=top_k, bits_gu=bits_gu,
                               bits_dn=bits_dn, codebook=codebook, max_tokens=max_tokens, seed=seed, device=device)
        self.shared = MoeLayer(plugin, n_expert=1, hidden=hidden, width=shared_width, top_k=1, bits_gu=shared_bits,
                               bits_dn=shared_bits, codebook=codebook, max_tokens=max_tokens, seed=seed + 104729,
                               device=device)
        self.native, self.H, self.max_tokens = self.routed.native, hidden, max_tokens
        dev = self.routed.dev
        g = torch.Generator(device=dev)
        g.manual_seed(seed + 7)
        self.sgate_w = (torch.randn(hidden, generator=g, device=dev) / hidden ** 0.5).to(torch.float16)
        self.x, self.logits = self.routed.x, self.routed.logits
        self.out = torch.empty((max_tokens, hidden), dtype=torch.float32, device=dev)
        d = self.desc = BlockDesc()
        d.routed, d.shared, d.sgate_w = self.routed.desc, self.shared.desc, self.sgate_w.data_ptr()
        b = self.bufs = BlockBufs()
        b.routed, b.shared = self.routed.bufs, self.shared.bufs

    def forward(self, T, stream, x=None, logits=None, out=None):
        """The block over the first T tokens of x / logits (self.x / self.logits by default) into out (f32 or bf16
        [T, hidden]; self.out by default)."""
        o = self.out if out is None else out
        xx = self.x if x is None else x
        lg = self.logits if logits is None else logits
        self.desc.routed, self.desc.shared = self.routed.desc, self.shared.desc     # the current weight sets
        self.native.block_forward(self.desc, self.bufs, xx.data_ptr(), lg.data_ptr(), T, o.data_ptr(),
                                  3 if o.dtype == self.torch.bfloat16 else 1, stream)

    def launches_per_step(self, T):
        """The routed layer's launches less its gather, the shared expert's identity routing, its gate_up (+ prep)
        and down, and the fold (one launch up to 4096 routed rows; else the map's memset aside, two)."""
        r, s = self.routed, self.shared
        fold = 1 if T * r.k <= 4096 and r.k <= 32 else 2
        return r.route_launches(T) + r.expert_launches(T) + 1 + s.expert_launches(T) + fold

    def expert_bytes(self):
        """Algorithmic bytes of a step: every live routed expert's (as MoeLayer) plus the shared expert's and the
        gate column."""
        gu, dn = self.shared.expert_bytes()
        return gu + dn + 2 * self.H


class Linears:
    """`n` independent EXL3 linears of one shape (config 4: out `rows`, in `cols`, K bits), each served by one call of
    the moe_exl3_down row as the engine issues a single linear (n_expert 1, top_k 1, every input row routed to it,
    h_rot 0: the input rotation inside the op), over `batch` input rows. The copies exist so a timed loop over them
    streams every call's weights from HBM rather than L2. Weights as the layer's: uniform random record words, suh
    +-1, svh +-|N(0,1)| * 0.02."""

    def __init__(self, plugin, rows, cols, bits, batch, n, codebook="mul1", seed=0, device="cuda", out_f16=False):
        import torch
        self.torch, self.plugin = torch, plugin
        self.out_f16 = out_f16
        self.rows, self.cols, self.bits, self.B, self.n, self.codebook = rows, cols, bits, batch, n, codebook
        dev = self.dev = torch.device(device)
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        self.rec_bytes = rows * cols * bits // 8
        self.rec = torch.randint(-32768, 32768, (n, self.rec_bytes // 2), generator=g, device=dev,
                                 dtype=torch.int32).to(torch.int16)
        sign = (torch.randint(0, 2, (n, 1, cols), generator=g, device=dev) * 2 - 1).to(torch.float16)
        self.suh = sign
        s2 = (torch.randint(0, 2, (n, rows, 1), generator=g, device=dev) * 2 - 1).float()
        self.svh = (s2 * torch.randn((n, rows, 1), generator=g, device=dev).abs() * 0.02).to(torch.float16)
        self.tab = torch.tensor([[self.rec[i].data_ptr()] for i in range(n)], dtype=torch.int64, device=dev)
        self.x = torch.randn((batch, cols), generator=g, device=dev).to(torch.float16)
        self.y = torch.empty((batch, rows), dtype=torch.float16 if out_f16 else torch.bfloat16, device=dev)
        self.sorted_tok = torch.arange(batch, dtype=torch.int32, device=dev)
        self.offset = torch.tensor([0, batch], dtype=torch.int32, device=dev)
        self.row = plugin.row("moe_exl3_down")
        self.native = Native(plugin.path) if out_f16 else None
        params = {"M": batch, "N": rows, "K": cols, "n_expert": 1, "top_k": 1, "dtype": f"exl3k{bits}",
                  "codebook": codebook, "h_rot": 0}
        P, nP, kp = rad.make_params(params)
        enc = X.encoding(bits, codebook, stacked=False)
        sel = C.c_int(0)
        pt = rad.tensor(0, rad.DT_UK[bits], [rows, cols])
        L = rad.RadLayout()
        rc = self.row.layout(P, nP, 1, C.byref(enc), C.byref(sel), C.byref(pt), 1, C.byref(L))
        if rc != 0 or L.bytes != self.rec_bytes:
            raise RuntimeError(f"layout hook: rc {rc}, bytes {L.bytes} (expected {self.rec_bytes})")
        rec_dtype = int(L.dtype)
        absent = rad.RadTensor()
        self._keep, self.args = [kp], []
        for i in range(n):
            P, nP, kp = rad.make_params(params)
            ts = [rad.tensor(self.x.data_ptr(), rad.DT["f16"], [batch, cols]),
                  rad.tensor(self.tab[i].data_ptr(), rec_dtype, [1, rows, cols], [0, cols, 1]),
                  rad.tensor(self.suh[i].data_ptr(), rad.DT["f16"], [1, 1, cols]),
                  rad.tensor(self.svh[i].data_ptr(), rad.DT["f16"], [1, rows, 1]),
                  rad.tensor(self.sorted_tok.data_ptr(), rad.DT["i32"], [batch]),
                  rad.tensor(self.offset.data_ptr(), rad.DT["i32"], [2]),
                  absent, absent, absent,
                  rad.tensor(self.y.data_ptr(), rad.DT["f16" if out_f16 else "bf16"], [batch, rows])]
            arr = (rad.RadTensor * len(ts))(*ts)
            a = rad.RadArgs()
            a.t, a.n_t, a.p, a.n_p, a.world_size = arr, len(ts), P, nP, 1
            if out_f16:
                need = self.native.moe_down_f16_scratch(C.addressof(a))
            else:
                need = int(self.row.scratch(C.byref(a))) if self.row.scratch else 0
            if need > 0:
                buf = torch.empty(need, dtype=torch.uint8, device=dev)
                self._keep.append(buf)
                a.scratch, a.scratch_bytes = buf.data_ptr(), need
            self._keep.extend([P, kp, arr])
            self.args.append(a)

    def run(self, i, stream):
        if self.out_f16:
            rc = self.native.moe_down_f16(C.addressof(self.args[i]), stream)
        else:
            rc = self.row.launch(C.byref(self.args[i]), stream)
        if rc != 0:
            raise RuntimeError(f"moe_exl3_down launch: {rc}")

    def bytes_per_call(self):
        """Algorithmic bytes of one call: the record plus suh and svh (read once)."""
        return self.rec_bytes + 2 * self.cols + 2 * self.rows

    def flops_per_call(self):
        return 2 * self.B * self.rows * self.cols


class ExpertMlps:
    """`n` independent copies of one expert MLP (config 2: gate [W, H] and up [W, H] at K bits, down [H, W]), each
    served by one call of the moe_exl3_gate_up_down row (n_expert 1, top_k 1, every input row routed to the expert;
    gate_up(h_rot 1) -> down(h_rot 1) inside the op, h in the row's scratch) over `batch` input rows. Weights as the
    layer's. The copies let a timed loop stream every call's weights from HBM rather than L2; one scratch serves all
    copies (the calls run one after another on one stream)."""

    def __init__(self, plugin, hidden, width, bits, batch, n, codebook="mul1", seed=0, device="cuda"):
        import torch
        self.torch, self.plugin = torch, plugin
        self.H, self.W, self.bits, self.B, self.n = hidden, width, bits, batch, n
        dev = self.dev = torch.device(device)
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        H, W = hidden, width
        self.gu_bytes, self.dn_bytes = 2 * W * H * bits // 8, H * W * bits // 8
        rnd = lambda nb: torch.randint(-32768, 32768, (n, nb // 2), generator=g, device=dev,  # noqa: E731
                                       dtype=torch.int32).to(torch.int16)
        self.gu_rec, self.dn_rec = rnd(self.gu_bytes), rnd(self.dn_bytes)

        def sign(*shape):
            return (torch.randint(0, 2, shape, generator=g, device=dev) * 2 - 1).to(torch.float16)

        def svh(*shape):
            return (sign(*shape).float() * torch.randn(shape, generator=g, device=dev).abs() * 0.02).to(torch.float16)

        self.suh, self.suh1, self.svh_gu = sign(n, 1, H), sign(n, 1, H), svh(n, 2 * W, 1)
        self.dn_suh, self.svh_dn = sign(n, 1, W), svh(n, H, 1)
        self.gu_tab = torch.tensor([[self.gu_rec[i].data_ptr()] for i in range(n)], dtype=torch.int64, device=dev)
        self.dn_tab = torch.tensor([[self.dn_rec[i].data_ptr()] for i in range(n)], dtype=torch.int64, device=dev)
        self.x = torch.randn((batch, H), generator=g, device=dev).to(torch.float16)
        self.y = torch.empty((batch, H), dtype=torch.bfloat16, device=dev)
        self.sorted_tok = torch.arange(batch, dtype=torch.int32, device=dev)
        self.offset = torch.tensor([0, batch], dtype=torch.int32, device=dev)
        self.row = plugin.row("moe_exl3_gate_up_down")
        params = {"M": batch, "N": 2 * W, "K": H, "n_expert": 1, "top_k": 1, "dtype": f"exl3k{bits}",
                  "codebook": codebook}
        P, nP, kp = rad.make_params(params)
        enc = X.encoding(bits, codebook, stacked=True)
        sel = C.c_int(0)
        L = rad.RadLayout()
        pt = rad.tensor(0, rad.DT_UK[bits], [2 * W, H])
        if self.row.layout(P, nP, 1, C.byref(enc), C.byref(sel), C.byref(pt), 1, C.byref(L)) != 0:
            raise RuntimeError("layout hook refused the gate_up codes")
        rec_dtype = int(L.dtype)
        schema = {s_["op"]: s_ for s_ in plugin.schemas()}["moe_exl3_gate_up_down"]
        self._keep, self.args, scratch = [kp], [], None
        for i in range(n):
            P, nP, kp = rad.make_params(params)
            ts = []
            for name, role, optional in schema["operands"]:
                if name == "a":
                    ts.append(rad.tensor(self.x.data_ptr(), rad.DT["f16"], [batch, H]))
                elif name == "codes":
                    ts.append(rad.tensor(self.gu_tab[i].data_ptr(), rec_dtype, [1, 2 * W, H], [0, H, 1]))
                elif name == "dn_codes":
                    ts.append(rad.tensor(self.dn_tab[i].data_ptr(), rec_dtype, [1, H, W], [0, W, 1]))
                elif name in ("suh", "suh1", "dn_suh"):
                    t = {"suh": self.suh, "suh1": self.suh1, "dn_suh": self.dn_suh}[name][i]
                    ts.append(rad.tensor(t.data_ptr(), rad.DT["f16"], [1] + list(t.shape)))
                elif name == "svh":
                    ts.append(rad.tensor(self.svh_gu[i].data_ptr(), rad.DT["f16"], [1, 2 * W, 1]))
                elif name == "dn_svh":
                    ts.append(rad.tensor(self.svh_dn[i].data_ptr(), rad.DT["f16"], [1, H, 1]))
                elif name == "sorted_tok":
                    ts.append(rad.tensor(self.sorted_tok.data_ptr(), rad.DT["i32"], [batch]))
                elif name == "expert_offset":
                    ts.append(rad.tensor(self.offset.data_ptr(), rad.DT["i32"], [2]))
                elif name == "y":
                    ts.append(rad.tensor(self.y.data_ptr(), rad.DT["bf16"], [batch, H]))
                else:
                    ts.append(rad.RadTensor())
            arr = (rad.RadTensor * len(ts))(*ts)
            a = rad.RadArgs()
            a.t, a.n_t, a.p, a.n_p, a.world_size = arr, len(ts), P, nP, 1
            need = int(self.row.scratch(C.byref(a)))
            if scratch is None or scratch.numel() < need:
                scratch = torch.empty(max(256, need), dtype=torch.uint8, device=dev)
                self._keep.append(scratch)
            a.scratch, a.scratch_bytes = scratch.data_ptr(), need
            self._keep.extend([P, kp, arr])
            self.args.append(a)

    def run(self, i, stream):
        rc = self.row.launch(C.byref(self.args[i]), stream)
        if rc != 0:
            raise RuntimeError(f"moe_exl3_gate_up_down launch: {rc}")

    def bytes_per_call(self):
        """Algorithmic bytes of one call: both records plus suh, suh.1, svh (gate_up), dn_suh and svh (down)."""
        H, W = self.H, self.W
        return self.gu_bytes + self.dn_bytes + 2 * H * 2 + 2 * W * 2 + W * 2 + H * 2

    def flops_per_call(self):
        return 2 * self.B * 3 * self.H * self.W


class ClassMoeLayer(MoeLayer):
    """The layer with its experts in classes by expert number mod n_class (2: the `_odd` tables, 4: the `_mod4`
    ops), class c of intermediate width widths[c] -- the width split's uneven cut, where a rank holds different
    slices of even and odd experts (architectures/qwen4exp_exl3/rad_block_moe_exl3.h:438-470). Expert e is entry
    e // n_class of class e % n_class. h is the widest class's width; a narrower class's rows are zero past its own
    (the ops' rule). Weights are filled by `tp.load_classes` (the width split's cut of a full-width layer)."""

    def __init__(self, plugin, *, widths, **kw):
        import torch
        if len(widths) not in (2, 4):
            raise ValueError("classes: 2 (by parity) or 4 (by number mod 4)")
        super().__init__(plugin, width=max(widths), **kw)
        self.c_layer = False          # its experts are the class tables below, served through the class rows
        self.widths = list(widths)
        self.n_class = len(widths)
        E, H, dev = self.n_local, self.H, self.dev
        self.cls = []
        for c, w in enumerate(self.widths):
            ec = len(range(c, E, self.n_class))
            t = {"n": ec, "w": w,
                 "gu_rec": torch.empty((ec, 2 * w * H * self.bits_gu // 16), dtype=torch.int16, device=dev),
                 "dn_rec": torch.empty((ec, H * w * self.bits_dn // 16), dtype=torch.int16, device=dev),
                 "suh": torch.empty((ec, 1, H), dtype=torch.float16, device=dev),
                 "suh1": torch.empty((ec, 1, H), dtype=torch.float16, device=dev),
                 "svh_gu": torch.empty((ec, 2 * w, 1), dtype=torch.float16, device=dev),
                 "dn_suh": torch.empty((ec, 1, w), dtype=torch.float16, device=dev),
                 "svh_dn": torch.empty((ec, H, 1), dtype=torch.float16, device=dev)}
            t["gu_tab"] = torch.tensor([t["gu_rec"][j].data_ptr() for j in range(ec)], dtype=torch.int64, device=dev)
            t["dn_tab"] = torch.tensor([t["dn_rec"][j].data_ptr() for j in range(ec)], dtype=torch.int64, device=dev)
            self.cls.append(t)
        self.op_gu = "moe_exl3_gate_up_mod4" if self.n_class == 4 else "moe_exl3_gate_up"
        self.op_dn = "moe_exl3_down_mod4" if self.n_class == 4 else "moe_exl3_down"
        self._args = {}

    def _class_params(self, p, down):
        keys = [("N_1", "K_1"), ("N_2", "K_2"), ("N_3", "K_3")] if self.n_class == 4 else [("N_odd", "K_odd")]
        w0 = self.widths[0]
        p["N"], p["K"] = (self.H, w0) if down else (2 * w0, self.H)
        for c, (kn, kk) in enumerate(keys, start=1):
            w = self.widths[c]
            p[kn], p[kk] = (self.H, w) if down else (2 * w, self.H)
        p["n_expert"] = self.n_local
        return p

    def _build(self, T, rows, x_ptr=None, top_k=None, M=None):
        key = (T, rows, x_ptr, top_k, M)
        if key in self._args:
            return self._args[key]
        if len(self._args) >= 32:
            self._args.clear()
        from .cases import split_name
        k = top_k or self.k
        H, W = self.H, self.W
        keep = []
        schemas = {s["op"]: s for s in self.plugin.schemas()}
        xp = x_ptr or self.x.data_ptr()

        def table(plane, c, down):
            t = self.cls[c]
            n, w = t["n"], t["w"]
            if plane == "codes":
                return (rad.tensor(t["dn_tab"].data_ptr(), self.rec_dtype, [n, H, w], [0, w, 1]) if down else
                        rad.tensor(t["gu_tab"].data_ptr(), self.rec_dtype, [n, 2 * w, H], [0, H, 1]))
            if down:
                ten = {"suh": t["dn_suh"], "svh": t["svh_dn"]}[plane]
            else:
                ten = {"suh": t["suh"], "suh1": t["suh1"], "svh": t["svh_gu"], "dn_suh": t["dn_suh"]}[plane]
            return rad.tensor(ten.data_ptr(), rad.DT["f16"], list(ten.shape))

        def args(op, down):
            p = self._params_dn(M or T) if down else self._params_gu(M or T)
            p["top_k"] = k
            p = self._class_params(p, down)
            P, nP, kp = rad.make_params(p)
            ts = []
            for name, role, optional in schemas[op]["operands"]:
                plane, c = split_name(name)
                if role == rad.OPD_WTAB:
                    ts.append(table(plane, c, down))
                elif name == "sorted_tok":
                    ts.append(rad.tensor(self.sorted_tok.data_ptr(), rad.DT["i32"], [rows]))
                elif name == "expert_offset":
                    ts.append(rad.tensor(self.offset.data_ptr(), rad.DT["i32"], [self.n_local + 1]))
                elif name == "a":
                    ts.append(rad.tensor(xp, rad.DT["f16"], [T, H]))
                elif name == "h":
                    ts.append(rad.tensor(self.h.data_ptr(), rad.DT["f16"], [rows, W]))
                elif name == "y":
                    ts.append(rad.tensor(self.y_rows.data_ptr(), rad.DT["bf16"], [rows, H]))
                else:
                    ts.append(rad.RadTensor())
            arr = (rad.RadTensor * len(ts))(*ts)
            a = rad.RadArgs()
            a.t, a.n_t, a.p, a.n_p, a.world_size = arr, len(ts), P, nP, 1
            keep.extend([P, kp, arr])
            row = self.plugin.row(op)
            need = int(row.scratch(C.byref(a))) if row.scratch else 0
            if need > 0:
                buf = self.torch.empty(need, dtype=self.torch.uint8, device=self.dev)
                keep.append(buf)
                a.scratch, a.scratch_bytes = buf.data_ptr(), need
            return a

        res = (args(self.op_gu, False), args(self.op_dn, True), keep)
        self._args[key] = res
        return res

    def experts(self, T, rows, stream, x_ptr=None, top_k=None, M=None, events=None, down_row_dst=None, live=False):
        if down_row_dst is not None or live:
            raise NotImplementedError("the class layer serves the plugin rows' plain launches")
        if rows == 0:
            for e in events or ():
                e.record()
            return
        a_gu, a_dn, _ = self._build(T, rows, x_ptr, top_k, M)
        if events:
            events[0].record()
        rc = self.plugin.row(self.op_gu).launch(C.byref(a_gu), stream)
        if rc != 0:
            raise RuntimeError(f"{self.op_gu} launch: {rc}")
        if events:
            events[1].record()
        rc = self.plugin.row(self.op_dn).launch(C.byref(a_dn), stream)
        if rc != 0:
            raise RuntimeError(f"{self.op_dn} launch: {rc}")
        if events:
            events[2].record()

    def expert_bytes(self):
        """Algorithmic bytes of one expert, averaged over the classes (this rank's slices)."""
        H, n = self.H, self.n_class
        gu = sum(2 * w * H * self.bits_gu // 8 + 2 * H * 2 + 2 * w * 2 + w * 2 for w in self.widths) / n
        dn = sum(H * w * self.bits_dn // 8 + H * 2 for w in self.widths) / n
        return gu, dn

    def expert_flops(self, rows):
        return 2 * rows * sum(3 * w * self.H for w in self.widths) / self.n_class
