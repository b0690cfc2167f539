"""bench.py -- the routed-MoE layer on B200: tokens/s and packed-weight HBM GB/s per chip.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--tokens T] [--impl ours|reference]

Workload ("config 3"): one routed-MoE layer -- 512 experts of hidden 2048 / width 512,
gate_up at K=3 and down at K=4 (mul1 codebook), top-10 softmax routing of seeded N(0,1) logits -- over T tokens
(default 2048) of N(0,1) fp16 activations. A step is the whole layer: router -> stable scatter -> moe_exl3_gate_up
(h_rot 1) -> moe_exl3_down (h_rot 1) -> weighted gather, each a kernel of libexl3b200.so, the expert ops called
through the plugin rows. Weights are synthetic and resident (679 MB > the 126 MB L2, so every step streams them
from HBM; no flush is needed). N > 1: expert parallelism -- each rank holds 512/N experts and its own T tokens
(weak scaling), a dispatch and a combine all-to-all over NCCL carry the token rows.

--impl reference: the reference's own CPU implementation of the path (kernels/exl3ref built from its sources,
oracle/_ref) timed on this box's host cores, every thread running a bounded sample of the same workload.
Prints ONE JSON line (rank 0)."""
import argparse
import ctypes as C
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "radiance-exl3_b200"))
sys.path.insert(0, str(REPO / "tests"))

METRIC = "routed-MoE layer tokens/s and packed-weight HBM GB/s/chip at batch 1-2048, 1/2/4/8 B200"
E, H, W, TOPK, KGU, KDN, CB = 512, 2048, 512, 10, 3, 4, "mul1"
WORKLOAD = (f"config 3: routed-MoE layer, {E} experts of [hidden {H}, width {W}], top-{TOPK} softmax routing, "
            f"gate_up K={KGU} / down K={KDN} {CB}, h_rot 1")


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


# ------------------------------------------------------------------------------------------ clocks
class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons while the GPU works."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------------------ the reference sample
def reference_sample_setup(T=2048, n_experts=4, seed=7):
    """A bounded sample of the workload for the reference's host library: the first `n_experts` experts of a
    T-token top-10 routing (all of their rows, so the per-row decode amortisation is the workload's), their
    canonical planes, and the token rows. Returns (launch callables, tokens the sample stands for)."""
    from exl3b200 import cases as X
    from exl3b200 import rad
    from oracle_bind import REF_SO
    rng = np.random.default_rng(seed)
    logits = rng.standard_normal((T, E)).astype(np.float32)
    ids = np.argsort(-logits, axis=1, kind="stable")[:, :TOPK].astype(np.int32)
    st, off = X.stable_scatter(ids, E)
    rows = int(off[n_experts])
    st_s = np.ascontiguousarray(st[:rows])
    off_s = np.ascontiguousarray(off[:n_experts + 1])
    x = X.bits_f16(X.f16(rng.standard_normal((T, H)).astype(np.float32)))
    gu = [X.random_planes(rng, 2 * W, H, KGU, True) for _ in range(n_experts)]
    dn = [X.random_planes(rng, H, W, KDN, False) for _ in range(n_experts)]
    dn_suh = [X.f16((rng.integers(0, 2, W) * 2 - 1).astype(np.float32)) for _ in range(n_experts)]
    plugin = rad.Plugin(REF_SO)
    row_gu, row_dn = plugin.row("moe_exl3_gate_up"), plugin.row("moe_exl3_down")

    def stack(arrs):
        return np.ascontiguousarray(np.stack([np.ascontiguousarray(a).view(np.uint8).reshape(-1) for a in arrs]))

    keep = []

    def T_(arr, dt, shape, stride=None):
        keep.append(arr)
        return rad.tensor(arr.ctypes.data, dt, shape, stride)

    n = n_experts
    gcodes, gsuh, gsuh1, gsvh = stack([p["codes"] for p in gu]), stack([p["suh"] for p in gu]), \
        stack([p["suh1"] for p in gu]), stack([p["svh"] for p in gu])
    dsuh, dcodes, dsvh = stack(dn_suh), stack([p["codes"] for p in dn]), stack([p["svh"] for p in dn])

    def make():
        h = np.zeros((rows, W), np.uint16)
        y = np.zeros((rows, H), np.uint16)
        absent = rad.RadTensor()
        gu_t = [T_(x, rad.DT["f16"], [T, H]), T_(gcodes, rad.DT_UK[KGU], [n, 2 * W, H]),
                T_(gsuh, rad.DT["f16"], [n, 1, H]), T_(gsuh1, rad.DT["f16"], [n, 1, H]),
                T_(gsvh, rad.DT["f16"], [n, 2 * W, 1]), T_(dsuh, rad.DT["f16"], [n, 1, W]),
                T_(st_s, rad.DT["i32"], [rows]), T_(off_s, rad.DT["i32"], [n + 1]),
                absent, absent, absent, absent, absent, T_(h, rad.DT["f16"], [rows, W])]
        dn_t = [T_(h, rad.DT["f16"], [rows, W]), T_(dcodes, rad.DT_UK[KDN], [n, H, W]),
                T_(dsuh, rad.DT["f16"], [n, 1, W]), T_(dsvh, rad.DT["f16"], [n, H, 1]),
                T_(st_s, rad.DT["i32"], [rows]), T_(off_s, rad.DT["i32"], [n + 1]),
                absent, absent, absent, T_(y, rad.DT["bf16"], [rows, H])]
        out = []
        for params, ts in (({"M": T, "N": 2 * W, "K": H, "n_expert": n, "top_k": TOPK, "dtype": f"exl3k{KGU}",
                             "codebook": CB, "h_rot": 1, "a_rot": 0}, gu_t),
                           ({"M": T, "N": H, "K": W, "n_expert": n, "top_k": TOPK, "dtype": f"exl3k{KDN}",
                             "codebook": CB, "h_rot": 1}, dn_t)):
            P, nP, kp = rad.make_params(params)
            arr = (rad.RadTensor * len(ts))(*ts)
            a = rad.RadArgs()
            a.t, a.n_t, a.p, a.n_p, a.world_size = arr, len(ts), P, nP, 1
            keep.extend([P, kp, arr, a])
            out.append(a)
        return out

    def run(args_pair):
        a_gu, a_dn = args_pair
        rc = row_gu.launch(C.byref(a_gu), None)
        rc = rc or row_dn.launch(C.byref(a_dn), None)
        if rc:
            raise RuntimeError(f"exl3ref launch: {rc}")

    return make, run, rows / TOPK, keep


def time_reference(threads, steps, warmup, n_experts=4, T=2048):
    """Every thread runs the same bounded sample concurrently (ctypes releases the GIL); a step is one sample on
    every thread. Returns (tokens/s aggregate, seconds a step, sample description)."""
    make, run, tokens, keep = reference_sample_setup(T, n_experts)
    arg_sets = [make() for _ in range(threads)]
    times = []
    for it in range(warmup + steps):
        ths = [threading.Thread(target=run, args=(arg_sets[i],)) for i in range(threads)]
        t0 = time.perf_counter()
        for t in ths:
            t.start()
        for t in ths:
            t.join()
        dt = time.perf_counter() - t0
        if it >= warmup:
            times.append(dt)
    step = float(np.mean(times))
    sample = (f"kernels/exl3ref (unmodified, -O2 -ffp-contract=off) gate_up(K={KGU}, h_rot 1) + down(K={KDN}, h_rot 1) "
              f"over the first {n_experts} experts of a T={T} top-{TOPK} routing ({int(tokens * TOPK)} sorted rows = "
              f"{tokens:.1f} tokens' worth), {threads} thread(s) each running it; router/scatter/gather not included")
    return threads * tokens / step, step, sample


# ------------------------------------------------------------------------------------------ our arm
def bitrate_sweep(plugin, hbm, tflops):
    """Config 4: one EXL3 linear of out 4096 x in 1536 (and its transpose), K = 2..8, batch 1 and 256, each call the
    moe_exl3_down row (n_expert 1, top_k 1, h_rot 0). Every timed call reads its own copy of the weights (copies
    totalling over 3x the 126 MB L2, replayed as one CUDA graph), so each streams its record from HBM. Reports
    microseconds a call, algorithmic GB/s (record + suh + svh) and TFLOP/s (2 * batch * out * in)."""
    import torch
    from exl3b200.layer import Linears
    res = {}
    st = torch.cuda.current_stream()
    for R, Cc in ((4096, 1536), (1536, 4096)):
        shape = {}
        for K in range(2, 9):
            for B in (1, 256):
                n = int(np.ceil(3 * 126e6 / (R * Cc * K / 8)))
                lin = Linears(plugin, R, Cc, K, B, n, seed=100 * K + B)
                for i in range(n):
                    lin.run(i, st.cuda_stream)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    cs = torch.cuda.current_stream().cuda_stream
                    for i in range(n):
                        lin.run(i, cs)
                for _ in range(3):
                    g.replay()
                reps = 5
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(reps):
                    g.replay()
                e1.record()
                torch.cuda.synchronize()
                us = e0.elapsed_time(e1) * 1e3 / (reps * n)
                gbs = lin.bytes_per_call() / (us / 1e6) / 1e9
                tf = lin.flops_per_call() / (us / 1e6) / 1e12
                shape[f"K{K}_B{B}"] = {"us": round(us, 2), "gbs": round(gbs, 1), "frac_hbm": round(gbs / hbm, 3),
                                       "tflops": round(tf, 2), "frac_tensor": round(tf / tflops, 4),
                                       "band": "k_gemm_tc" if B >= 16 else "k_gemm_skinny", "copies": n}
                del g, lin
                torch.cuda.synchronize()
        res[f"out{R}_in{Cc}"] = shape
    return res


def bitrate_cpu_reference():
    """The reference's exl3ref beside the config-4 sweep: one call of moe_exl3_down on the out 4096 x in 1536 linear
    at batch 1 for every K, and at batch 256 for K = 4 (one host core, the launch alone)."""
    out = {}
    for K in range(2, 9):
        t = reference_op_seconds("moe_exl3_down", reps=1, M=1, top_k=1, n_expert=1, geom=[(4096, 1536)], bits=K,
                                 codebook="mul1")
        out[f"K{K}_B1"] = {"us": round(t * 1e6, 1), "gbs": round((4096 * 1536 * K / 8 + 3072 + 8192) / t / 1e9, 4)}
    t = reference_op_seconds("moe_exl3_down", reps=1, M=256, top_k=1, n_expert=1, geom=[(4096, 1536)], bits=4,
                             codebook="mul1")
    out["K4_B256"] = {"us": round(t * 1e6, 1), "tflops": round(2 * 256 * 4096 * 1536 / t / 1e12, 5)}
    out["cores"], out["kind"], out["orientation"] = 1, "reference", "out 4096 x in 1536"
    return out


def _graph_time(run_all, reps=5):
    """Microseconds of one replay of a CUDA graph of `run_all(stream)` (a warm-up, then `reps` replays between CUDA
    events on the current stream)."""
    import torch
    run_all(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        run_all(torch.cuda.current_stream().cuda_stream)
    for _ in range(3):
        g.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) * 1e3 / reps


def reference_op_seconds(op, reps=3, **case_kw):
    """The reference's own CPU implementation (kernels/exl3ref built from its sources, oracle/_ref) of one op on a
    seeded case of the given shape: the median wall time of the row's launch alone (buffers and layout hooks set up
    outside the timed call), single-threaded as exl3ref is."""
    from exl3b200 import cases as X
    from exl3b200 import rad
    from oracle_bind import REF_SO
    plugin = rad.Plugin(REF_SO)
    row = plugin.row(op)
    case = X.Case(op, 77, **case_kw)
    times = []

    def timed(a, s):
        t0 = time.perf_counter()
        rc = row.launch(a, s)
        times.append(time.perf_counter() - t0)
        return rc

    for _ in range(reps):
        r = case.run(plugin, device=False, launch=timed)
        if r["rc"] != 0:
            raise RuntimeError(f"exl3ref {op}: {r['rc']}")
    return float(np.median(times))


def single_expert_configs(plugin, hbm, with_cpu):
    """Config 1 (one EXL3 linear, 16 rows of 2048 -> 512, K=4 mul1, f16 out: exl3b200_moe_down_f16) and config 2
    (one expert MLP, gate/up [512, 2048] and down [2048, 512] at K=4, M = 1, 4, 8, 32 rows: the moe_exl3_gate_up_down
    row), each timed as one call over its own copy of the weights (copies totalling over 3x the 126 MB L2, replayed
    as one CUDA graph, so every call streams its weights from HBM). Beside each: the reference's exl3ref on one host
    core (moe_exl3_down with bf16 rows for config 1 -- the reference has no f16-output form -- and
    moe_exl3_gate_up_down for config 2)."""
    from exl3b200.layer import ExpertMlps, Linears
    res = {}
    n1 = int(np.ceil(3 * 126e6 / 529408))
    lin = Linears(plugin, 512, 2048, 4, 16, n1, seed=11, out_f16=True)
    us = _graph_time(lambda s: [lin.run(i, s) for i in range(n1)]) / n1
    c1 = {"us": round(us, 2), "gbs": round(lin.bytes_per_call() / (us / 1e6) / 1e9, 1),
          "frac_hbm": round(lin.bytes_per_call() / (us / 1e6) / 1e9 / hbm, 3), "bytes_per_call": lin.bytes_per_call(),
          "tokens_per_s": round(16 / (us / 1e6), 1), "copies": n1, "out": "f16", "entry": "exl3b200_moe_down_f16"}
    if with_cpu:
        t = reference_op_seconds("moe_exl3_down", M=16, top_k=1, n_expert=1, geom=[(512, 2048)], bits=4,
                                 codebook="mul1")
        c1["cpu_reference"] = {"us": round(t * 1e6, 1), "tokens_per_s": round(16 / t, 1), "cores": 1,
                               "kind": "reference", "op": "moe_exl3_down (bf16 rows)"}
        c1["speedup_vs_cpu"] = round(t * 1e6 / us, 1)
    del lin
    res["config1_linear_16x2048_to_512"] = c1
    c2 = {}
    n2 = int(np.ceil(3 * 126e6 / 1588224))
    for M in (1, 4, 8, 32):
        mlp = ExpertMlps(plugin, 2048, 512, 4, M, n2, seed=20 + M)
        us = _graph_time(lambda s: [mlp.run(i, s) for i in range(n2)]) / n2
        e = {"us": round(us, 2), "gbs": round(mlp.bytes_per_call() / (us / 1e6) / 1e9, 1),
             "frac_hbm": round(mlp.bytes_per_call() / (us / 1e6) / 1e9 / hbm, 3),
             "tokens_per_s": round(M / (us / 1e6), 1), "copies": n2}
        if with_cpu:
            t = reference_op_seconds("moe_exl3_gate_up_down", M=M, top_k=1, n_expert=1, geom=[(1024, 2048)], bits=4,
                                     codebook="mul1")
            e["cpu_reference"] = {"us": round(t * 1e6, 1), "tokens_per_s": round(M / t, 1), "cores": 1,
                                  "kind": "reference"}
            e["speedup_vs_cpu"] = round(t * 1e6 / us, 1)
        c2[f"M{M}"] = e
        del mlp
    res["config2_expert_mlp_2048x512_K4"] = c2
    res["bytes_per_call"] = {"config1": 529408, "config2": 1588224}
    return res


def _time_steps(step, sh, reps, use_graph):
    """ms of one call of step(stream): captured once in a CUDA graph and replayed `reps` times between CUDA events
    (or run eagerly when capture is not possible), after a warm-up."""
    import torch
    step(sh)
    torch.cuda.synchronize()
    run = None
    if use_graph:
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                step(torch.cuda.current_stream().cuda_stream)
            run = g.replay
        except Exception:
            run = None
    if run is None:
        run = lambda: step(sh)  # noqa: E731
    for _ in range(2):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        run()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def moe_block(plugin, dev, sh, T=2048, shared_width=512):
    """The MoE block pass (one GPU): config 3's routed layer beside a shared EXL3 expert (width 512, K = 4) whose
    output the gather folds in through its sigmoid gate, one call of exl3b200_moe_block_forward, against the routed
    layer alone over the same tokens. Every step reads all 512 experts' weights (679 MB, over 5x the L2)."""
    import torch
    from exl3b200.layer import MoeBlock
    blk = MoeBlock(plugin, n_expert=E, hidden=H, width=W, top_k=TOPK, bits_gu=KGU, bits_dn=KDN,
                   shared_width=shared_width, shared_bits=4, codebook=CB, max_tokens=T, seed=23, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(4242)
    blk.x[:T] = torch.randn((T, H), generator=g, device=dev).to(torch.float16)
    blk.logits[:T] = torch.randn((T, E), generator=g, device=dev)
    ms = _time_steps(lambda s: blk.forward(T, s), sh, 10, True)
    ms_layer = _time_steps(lambda s: blk.routed.forward(T, s), sh, 10, True)
    gu, dn = blk.routed.expert_bytes()
    shared_bytes = blk.expert_bytes()
    res = {"tokens": T, "shared_width": shared_width, "ms": round(ms, 4), "tokens_per_s": round(T / (ms / 1e3), 1),
           "routed_layer_ms": round(ms_layer, 4), "shared_arm_ms": round(ms - ms_layer, 4),
           "launches": blk.launches_per_step(T),
           "packed_weight_gbs": round((E * (gu + dn) + shared_bytes) / (ms / 1e3) / 1e9, 1)}
    del blk
    torch.cuda.empty_cache()
    return res


def skewed_routing(layer, T, sh, world, rank, dev, use_graph):
    """Config 3 under the reference's skewed draw (tools/perfmoe.cpp:50-51): expert popularity lognormal with
    sigma 0.8 (the same draw on every rank), each token's top-10 a Gumbel-top-k sample of it -- logits = log
    popularity + Gumbel noise, which the router's softmax top-k then selects exactly. Returns ms a step, tokens/s
    and how uneven the experts' rows came out."""
    import torch
    gp = torch.Generator(device=dev)
    gp.manual_seed(4242)
    log_pop = torch.randn((E,), generator=gp, device=dev) * 0.8
    gn = torch.Generator(device=dev)
    gn.manual_seed(4343 + rank)
    u = torch.rand((T, E), generator=gn, device=dev).clamp_(1e-12, 1 - 1e-7)
    logits = (log_pop[None, :] - torch.log(-torch.log(u))).contiguous()
    ms = _time_steps(lambda s: layer.forward(T, s, logits=logits), sh, 10, use_graph)
    layer.forward(T, sh, logits=logits)
    torch.cuda.synchronize()
    ids = layer.ids.reshape(-1)[:T * TOPK].cpu().numpy()
    counts = np.bincount(ids[ids >= 0], minlength=E)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())
    return {"ms": round(ms, 4), "tokens_per_s": round(T * world / (ms / 1e3), 1),
            "rows_per_expert_max": int(counts.max()), "rows_per_expert_mean": round(float(counts.mean()), 2),
            "live_experts_rank0_routing": int((counts > 0).sum()),
            "draw": "log popularity ~ 0.8 N(0,1) per expert (shared), Gumbel(0,1) noise per (token, expert)"}


def stack48(layer, world, rank, dev, sh, use_graph, n_layers=48, tokens=(2048, 8)):
    """Config 5: a stack of 48 routed-MoE layers, each with its own weights (seeded, resident: 48 x 679 MB / N per
    GPU) and its own routing (seeded logits per layer), run back to back over the same token rows; the weights of
    every layer stream from HBM each step. tokens/s = tokens a GPU x N / the stack's time."""
    import torch
    base = layer.ops.local if world > 1 else layer
    for i in range(1, n_layers):
        base.add_weight_set(seed=9000 + 131 * i + 7 * rank)
    out = {}
    for T in tokens:
        if T > layer.max_tokens:
            continue
        lgs = []
        for i in range(n_layers):
            g = torch.Generator(device=dev)
            g.manual_seed(12000 + 17 * i + 1009 * rank + T)
            lgs.append(torch.randn((T, E), generator=g, device=dev))

        def step(s):
            for i in range(n_layers):
                base.use_weight_set(i)
                layer.forward(T, s, logits=lgs[i])

        ms = _time_steps(step, sh, 5, use_graph)
        t = torch.tensor([ms], device=dev)
        if world > 1:
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
        out[f"T{T}"] = {"ms_per_stack_step": round(ms, 3), "ms_per_layer": round(ms / n_layers, 4),
                        "tokens_per_s": round(T * world / (ms / 1e3), 1)}
    base.use_weight_set(0)
    out["layers"] = n_layers
    out["weights_resident_gb_per_gpu"] = round(n_layers * sum(base.expert_bytes()) * base.n_local / 1e9, 2)
    return out


def bench_ours(args, rank, world, local_rank):
    import torch
    torch.cuda.set_device(local_rank)
    from exl3b200 import load_plugin
    from exl3b200.layer import MoeLayer
    dev = torch.device("cuda", local_rank)
    plugin = load_plugin()
    T = args.tokens
    tp_mode = world > 1 and args.mode == "tp"
    # N > 1: every rank also builds the whole 512-expert layer from the same seed (its weights are the ones the ranks
    # hold in slices), used once after the timed region to check this rank's multi-GPU output against the one-GPU
    # layer on the same tokens
    full = None
    if world > 1:
        full = MoeLayer(plugin, n_expert=E, hidden=H, width=W, top_k=TOPK, bits_gu=KGU, bits_dn=KDN, codebook=CB,
                        max_tokens=T, seed=1)
    if tp_mode:
        # the width split: every rank holds half (a quarter, ...) of every expert's width and serves ALL T tokens
        # (replicated), so the group's throughput is T a step (strong scaling)
        from exl3b200.tp import TpLayer
        layer = TpLayer(plugin, rank=rank, world=world, n_expert=E, hidden=H, width=W, top_k=TOPK, bits_gu=KGU,
                        bits_dn=KDN, codebook=CB, max_tokens=T, seed=1, transport=args.transport, full=full)
    elif world > 1:
        from exl3b200.ep import EpLayer
        layer = EpLayer(plugin, rank=rank, world=world, n_expert=E, hidden=H, width=W, top_k=TOPK, bits_gu=KGU,
                        bits_dn=KDN, codebook=CB, max_tokens=T, seed=1, transport=args.transport, full=full)
    else:
        layer = MoeLayer(plugin, n_expert=E, hidden=H, width=W, top_k=TOPK, bits_gu=KGU, bits_dn=KDN, codebook=CB,
                         max_tokens=T, seed=1)
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + (0 if tp_mode else rank))      # width split: the same tokens on every rank
    layer.x.copy_(torch.randn(layer.x.shape, generator=g, device=dev).to(torch.float16))
    layer.logits.copy_(torch.randn(layer.logits.shape, generator=g, device=dev))
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    hbm, tflops, peak_kind = peaks()

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    # ---- warm-up, then a clock soak of about a second, then EXACTLY K timed steps
    clocks = Clocks(local_rank)
    for _ in range(args.warmup):
        layer.forward(T, sh)
    barrier()
    clocks.start()
    if world > 1:
        # every rank must run the same number of steps (each step exchanges with every peer): the soak length is
        # one rank-agreed count, about a second's worth, not each rank's own clock
        t0 = time.perf_counter()
        layer.forward(T, sh)
        torch.cuda.synchronize()
        n_soak = torch.tensor([0 if args.profile else max(1, int(1.0 / max(time.perf_counter() - t0, 1e-4)))],
                              device=dev)
        torch.distributed.all_reduce(n_soak, op=torch.distributed.ReduceOp.MAX)
        for _ in range(int(n_soak.item())):
            layer.forward(T, sh)
    else:
        soak_t0 = time.perf_counter()
        while not args.profile and time.perf_counter() - soak_t0 < 1.0:
            layer.forward(T, sh)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    kev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    pev = ([[torch.cuda.Event(enable_timing=True) for _ in range(len(layer.PHASES) + 1)] for _ in range(args.steps)]
           if world > 1 else None)
    # The step captured once in a CUDA graph and replayed (no per-launch host cost between steps) -- one GPU, and
    # N > 1 over peer memory (a step there never synchronises with the host); the per-op (and per-phase) times come
    # from an eager pass with events. N > 1 over NCCL: eager (a step reads the split sizes on the host).
    graph = None
    if (world == 1 or args.transport == "p2p") and not args.profile:
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                layer.forward(T, torch.cuda.current_stream().cuda_stream)
            for _ in range(3):
                g.replay()
            torch.cuda.synchronize()
            graph = g
        except Exception:   # capture refused: the timed loop runs eagerly
            graph = None
    barrier()
    wall0 = time.perf_counter()
    ev[0].record(stream)
    for s in range(args.steps):
        if graph is not None:
            graph.replay()
        elif world > 1:
            layer.forward(T, sh, events=kev[s], phases=pev[s])
        else:
            layer.forward(T, sh, events=kev[s])
    ev[1].record(stream)
    barrier()
    wall = time.perf_counter() - wall0
    clk = clocks.stop()
    ms = ev[0].elapsed_time(ev[1]) / args.steps
    if graph is not None:
        for s in range(args.steps):
            if world > 1:
                layer.forward(T, sh, events=kev[s], phases=pev[s])
            else:
                layer.forward(T, sh, events=kev[s])
        torch.cuda.synchronize()
    gu_ms = float(np.mean([k[0].elapsed_time(k[1]) for k in kev]))
    dn_ms = float(np.mean([k[1].elapsed_time(k[2]) for k in kev]))
    ep_phases = None
    if world > 1:
        t = torch.tensor([ms, gu_ms, dn_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, gu_ms, dn_ms = (float(v) for v in t.cpu())
        ph = torch.tensor([float(np.mean([p[i].elapsed_time(p[i + 1]) for p in pev]))
                           for i in range(len(layer.PHASES))], device=dev)
        torch.distributed.all_reduce(ph, op=torch.distributed.ReduceOp.MAX)
        ep_phases = {n: round(float(v), 4) for n, v in zip(layer.PHASES, ph.cpu())}
    live = layer.live_experts()
    gu_b, dn_b = layer.expert_bytes()
    tokens_total = T if tp_mode else T * world
    value = tokens_total / (ms / 1e3)
    step_bytes = live * (gu_b + dn_b)
    # the dominant kernel's roofline (the weight bytes it must read once / its measured duration). On the
    # tensor-core band the gate_up op is k_prep then k_gemm_tc: k_prep is timed alone (moe_exl3_prep_gu over the
    # same rows, CUDA events) and subtracted, so the figure is k_gemm_tc's own.
    gu_band = layer.band_name("gate_up", T)
    prep_ms = layer.time_prep_step(T, n=max(3, args.steps)) if "k_prep" in gu_band else 0.0
    if world > 1:
        t = torch.tensor([prep_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        prep_ms = float(t.item())
    gu_kernel_ms = max(gu_ms - prep_ms, 1e-6)
    dom = "gate_up" if gu_kernel_ms >= dn_ms else "down"
    dom_ms = gu_kernel_ms if dom == "gate_up" else dn_ms
    dom_bytes = live * (gu_b if dom == "gate_up" else dn_b)
    achieved = dom_bytes / (dom_ms / 1e3) / 1e9
    # DRAM traffic per launch of that kernel (dram__bytes_read.sum + dram__bytes_write.sum), as one ncu capture of this
    # workload recorded it in the repository's traffic table, where it applies
    traffic = None
    traffic_key = f"k_gemm_tc {dom} config3 T{T}"
    tpath = REPO / "profiles" / "traffic.json"
    if world == 1 and "k_gemm_tc" in layer.band_name(dom, T) and tpath.exists():
        ent = json.loads(tpath.read_text()).get(traffic_key)
        traffic = ent["dram_bytes_per_launch"] if ent else None
    launches_per_step = layer.launches_per_step(T)

    # ---- end to end: pinned host inputs in, the layer, the output back, every step. Double-buffered: step i's
    # copies (H2D on one stream, D2H on another) overlap the layer of steps i - 1 and i + 1; every step still moves
    # its own inputs and result across PCIe inside the timed region.
    e2e = None
    if not args.no_e2e:
        nb = 2
        hx = [torch.empty(layer.x[:T].shape, dtype=layer.x.dtype, pin_memory=True) for _ in range(nb)]
        hl = [torch.empty(layer.logits[:T].shape, dtype=layer.logits.dtype, pin_memory=True) for _ in range(nb)]
        # the layer's output in the engine's hidden-state type (bf16: the MoE block adds it to a bf16 stream); the
        # width split sums f32 partials across ranks and returns f32
        odt = torch.float32 if tp_mode else torch.bfloat16
        ho = [torch.empty(layer.out[:T].shape, dtype=odt, pin_memory=True) for _ in range(nb)]
        for b in range(nb):
            hx[b].copy_(layer.x[:T].cpu())
            hl[b].copy_(layer.logits[:T].cpu())
        dx = [torch.empty_like(layer.x[:T]) for _ in range(nb)]
        dl = [torch.empty_like(layer.logits[:T]) for _ in range(nb)]
        do = [torch.empty(layer.out[:T].shape, dtype=odt, device=dev) for _ in range(nb)]
        s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
        in_ready = [torch.cuda.Event() for _ in range(nb)]
        comp_done = [torch.cuda.Event() for _ in range(nb)]
        out_done = [torch.cuda.Event() for _ in range(nb)]
        for b in range(nb):
            comp_done[b].record(stream)
            out_done[b].record(stream)

        def e2e_step(i):
            b = i % nb
            s_in.wait_event(comp_done[b])            # step i - nb has finished reading this buffer
            with torch.cuda.stream(s_in):
                dx[b].copy_(hx[b], non_blocking=True)
                dl[b].copy_(hl[b], non_blocking=True)
                in_ready[b].record(s_in)
            stream.wait_event(in_ready[b])
            stream.wait_event(out_done[b])           # step i - nb's result has left this buffer
            layer.forward(T, sh, x=dx[b], logits=dl[b], out=do[b])
            comp_done[b].record(stream)
            s_out.wait_event(comp_done[b])
            with torch.cuda.stream(s_out):
                ho[b].copy_(do[b], non_blocking=True)
                out_done[b].record(s_out)

        for i in range(args.warmup):
            e2e_step(i)
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        s_in.wait_event(e0)
        for i in range(args.steps):
            e2e_step(i)
        stream.wait_event(out_done[(args.steps - 1) % nb])
        e1.record(stream)
        barrier()
        e_ms = e0.elapsed_time(e1) / args.steps
        if world > 1:
            t = torch.tensor([e_ms], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            e_ms = float(t.item())
        e2e = {"value": tokens_total / (e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e_ms,
               "h2d_bytes_per_step": int(hx[0].numel() * 2 + hl[0].numel() * 4),
               "d2h_bytes_per_step": int(ho[0].numel() * ho[0].element_size()),
               "path": "pinned host x + logits -> router/scatter kernels -> plugin rows moe_exl3_gate_up, "
                       f"moe_exl3_down (RadArgs launch) -> gather kernel ({'f32' if tp_mode else 'bf16'} y) -> "
                       "pinned host y; copies on two streams, double-buffered so each step's copies overlap the "
                       "neighbouring steps' layers"}

    # ---- the batch sweep (1 GPU): each T captured in a CUDA graph. Below T = 2048 a step reads only its live
    # experts' weights (13 MB at T = 1, 99 MB at T = 8), which a repeated step would find in the 126 MB L2; so the
    # timed graph runs `nrot` steps, each over its own seeded logits (its own experts), the weights they touch
    # together over three times the L2 -- every step streams its weights from HBM, as a layer of a deep model does.
    sweep = None
    if world == 1 and not args.no_sweep:
        sweep = {}
        per_expert = gu_b + dn_b
        for Ts in (1, 8, 64, 512, 2048):
            if Ts > T:
                continue
            live_est = E * (1 - (1 - TOPK / E) ** Ts)
            nrot = int(min(64, max(1, np.ceil(3 * 126e6 / (live_est * per_expert)))))
            gl = torch.Generator(device=dev)
            gl.manual_seed(5000 + Ts)
            lgs = [torch.randn((Ts, E), generator=gl, device=dev) for _ in range(nrot)]

            def steps(s_):
                for lg in lgs:
                    layer.forward(Ts, s_, logits=lg)

            steps(sh)
            torch.cuda.synchronize()
            graph_ok = True
            try:
                gph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gph):
                    steps(torch.cuda.current_stream().cuda_stream)
                run = gph.replay
            except Exception:
                graph_ok = False
                run = lambda: steps(sh)  # noqa: E731
            for _ in range(2):
                run()
            torch.cuda.synchronize()
            n = max(2, int(np.ceil(max(args.steps, 20) / nrot)))
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record()
            for _ in range(n):
                run()
            a1.record()
            torch.cuda.synchronize()
            sms = a0.elapsed_time(a1) / (n * nrot)
            lv_all = []
            for lg in lgs[:8]:
                layer.forward(Ts, sh, logits=lg)
                lv_all.append(layer.live_experts())
            lv = float(np.mean(lv_all))
            sweep[str(Ts)] = {"ms": round(sms, 4), "tokens_per_s": round(Ts / (sms / 1e3), 1),
                              "live_experts": round(lv, 1),
                              "weight_gbs": round(lv * per_expert / (sms / 1e3) / 1e9, 1),
                              "frac_hbm": round(lv * per_expert / (sms / 1e3) / 1e9 / hbm, 3),
                              "graph": graph_ok, "routings_rotated": nrot}
            del run
            if graph_ok:
                del gph

    # ---- config 4: the bitrate sweep of one linear (1 GPU), configs 1 and 2 (single expert), the reference beside
    bitrates = singles = None
    if world == 1 and not args.no_sweep:
        bitrates = bitrate_sweep(plugin, hbm, tflops)
        if rank == 0 and not args.no_cpu_baseline:
            try:
                bitrates["cpu_reference"] = bitrate_cpu_reference()
            except Exception as exc:
                bitrates["cpu_reference"] = {"unavailable": str(exc)}
        singles = single_expert_configs(plugin, hbm, with_cpu=rank == 0 and not args.no_cpu_baseline)

    # ---- skewed routing (config 3 under perfmoe's popularity draw) and config 5 (the 48-layer stack)
    use_graph = (world == 1 or args.transport == "p2p") and not args.profile
    skew = stack = block = None
    if not args.no_sweep and not tp_mode:
        skew = skewed_routing(layer, T, sh, world, rank, dev, use_graph)
    if not args.no_sweep and world == 1:
        block = moe_block(plugin, dev, sh, T=T)
    if not args.no_stack and not tp_mode and use_graph:
        stack = stack48(layer, world, rank, dev, sh, use_graph)

    # ---- the CPU baseline (rank 0, one GPU): the reference library on a bounded sample
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            v, step, sample = time_reference(threads=1, steps=1, warmup=0, n_experts=32)
            cpu = {"value": round(v, 3), "unit": "tokens/s", "cores": 1, "kind": "reference",
                   "sample": sample, "seconds": round(step, 2), "host_cores_available": os.cpu_count()}
        except Exception as exc:  # the reference library is absent on this box
            cpu = {"value": None, "unit": "tokens/s", "cores": 0, "kind": "reference", "sample": f"unavailable: {exc}"}

    multi_check = None
    if world > 1:
        layer.check()
        # this rank's output of the last step against the one-GPU layer on the same tokens and weights: expert
        # parallelism returns every pair's own down row and sums a token's slots in the same order, so the two must
        # be equal to the bit; the width split sums per-rank partials (each rounded to bf16 rows), so it is held to
        # the expert-output tolerance (max |diff| <= 1e-2 max |ref|, cosine >= 0.9999)
        layer.forward(T, sh)                 # this rank's tokens again (the sections above ran other routings)
        full.x[:T].copy_(layer.x[:T])
        full.logits[:T].copy_(layer.logits[:T])
        full.forward(T, sh)
        torch.cuda.synchronize()
        a, b = full.out[:T].double(), layer.out[:T].double()
        same = bool(torch.equal(full.out[:T], layer.out[:T]))
        rel = float((a - b).abs().max() / a.abs().max().clamp_min(1e-30))
        cos = float((a * b).sum() / (a.norm() * b.norm()).clamp_min(1e-30))
        ok = same if not tp_mode else (rel <= 1e-2 and cos >= 0.9999)
        v = torch.tensor([1.0 if ok else 0.0, 1.0 if same else 0.0, rel, -cos], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(v, op=torch.distributed.ReduceOp.MIN)
        v2 = torch.tensor([rel, -cos], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(v2, op=torch.distributed.ReduceOp.MAX)
        multi_check = {"ranks_ok": bool(v[0].item() == 1.0), "bit_identical_all_ranks": bool(v[1].item() == 1.0),
                       "max_rel_err": float(v2[0].item()), "min_cosine": float(-v2[1].item()),
                       "against": "the one-GPU layer (all 512 experts, same seed) on each rank's own tokens"}
        exch = layer.exchange_bytes(T) if tp_mode else layer.exchange_bytes()
        if ep_phases is not None:
            ep_phases["exchange_bytes_rank0"] = exch
            ep_phases["transport"] = args.transport
            ep_phases["mode"] = args.mode
        layer.close()          # collective: every rank releases its peer-memory window
    if rank != 0:
        return None
    flops = layer.expert_flops(T * TOPK) * world      # (width split: every rank's slice of all T * TOPK rows)
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "strong" if tp_mode else "weak", "vs_baseline": None,
        "dtype": "fp16 operands (decoded trellis), f32 accumulate", "data": "synthetic",
        "config": {"workload": WORKLOAD, ("tokens_per_step" if tp_mode else "tokens_per_gpu"): T, "n_expert": E,
                   "hidden": H, "width": W, "top_k": TOPK,
                   "bits": {"gate_up": KGU, "down": KDN}, "codebook": CB,
                   "parallelism": f"{args.mode}{world} ({args.transport})" if world > 1 else "single",
                   "launch": "cuda graph replay" if graph is not None else "eager",
                   "l2": ("no flush: each timed step reads all 512 experts' packed weights (679 MB, over 5x the 126 MB "
                          "L2); the batch sweep rotates seeded routings so its steps' weights exceed 3x the L2"),
                   "inputs": "codes uniform random record words, suh +-1, svh +-|N(0,1)|*0.02, x and logits N(0,1)"},
        "hbm_gbs_per_chip": round(step_bytes / (ms / 1e3) / 1e9, 1),
        "tflops": round(flops / (ms / 1e3) / 1e12, 2),
        "roofline": {"bound": "hbm", "kernel": ("k_gemm_tc (gate_up)" if dom == "gate_up" and prep_ms > 0
                                                else layer.band_name(dom, T)),
                     "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                     "peak_source": ("of measured: hbm_gbs in MEASURED_PEAKS.json" if peak_kind == "measured"
                                     else "of fallback: 6650 GB/s (MEASURED_PEAKS.json absent)"),
                     "bytes_per_launch": int(dom_bytes), "ms_per_launch": round(dom_ms, 4),
                     "traffic": int(traffic) if traffic else None,
                     "traffic_source": f"ncu capture: {traffic_key}" if traffic else None,
                     "other": {"gate_up_op_ms": round(gu_ms, 4), "k_prep_ms": round(prep_ms, 4),
                               "down_op_ms": round(dn_ms, 4)}},
        "clocks": clk, "gpu_launches": int(launches_per_step * args.steps),
        "e2e": e2e, "cpu_baseline": cpu, "sweep": sweep, "bitrate_sweep": bitrates, "single_expert": singles,
        "skewed_routing": skew, "moe_block": block, "stack48": stack, "wall_s": round(wall, 3),
        "ep_phases_ms": ep_phases,
    }
    if multi_check is not None:
        line["ep_bit_identical" if not tp_mode else "tp_within_tolerance"] = multi_check["ranks_ok"]
        line["multi_gpu_check"] = multi_check
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--tokens", type=int, default=2048)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--transport", default="p2p", choices=["p2p", "nccl"],
                    help="N > 1: the expert-parallel exchange over peer memory (default) or NCCL all-to-alls")
    ap.add_argument("--mode", default="ep", choices=["ep", "tp"],
                    help="N > 1: expert parallelism (default) or the width split of every expert (tp, N <= 4)")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-stack", action="store_true", help="skip config 5, the 48-layer stack")
    ap.add_argument("--profile", action="store_true",
                    help="for a profiler run: no clock soak, sweep, end-to-end leg or CPU baseline")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.profile:
        args.no_sweep = args.no_e2e = args.no_cpu_baseline = args.no_stack = True
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))

    if args.impl == "reference":
        if rank != 0:
            return 0
        threads = max(1, min(os.cpu_count() or 1, 64))
        v, step, sample = time_reference(threads, args.steps, args.warmup, n_experts=2)
        line = {"metric": METRIC, "impl": "reference", "value": round(v, 3), "unit": "tokens/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step * 1e3, 2),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 host",
                "data": "synthetic",
                "config": {"workload": WORKLOAD, "tokens_per_gpu": args.tokens, "n_expert": E, "top_k": TOPK},
                "cpu_baseline": {"value": round(v, 3), "unit": "tokens/s", "cores": threads, "kind": "reference",
                                 "sample": sample},
                "e2e": {"value": round(v, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    if world > 1:
        import datetime

        import torch
        torch.cuda.set_device(local_rank)
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                                             device_id=torch.device("cuda", local_rank))
    try:
        line = bench_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
    if rank == 0 and line is not None:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
