"""The width ("column-block") tensor split of exl3b200/tp.py.

On CPU: the slice rule against the reference's (architectures/qwen4exp_exl3/qwen4exp_exl3.cpp:296-301, 576-634),
the record cut against the cut of the canonical plane (through the oracle's relayout), and -- on gloo ranks -- the
whole split through the oracle: each rank's sliced experts, its partial gather, the all-reduce, against the
full-width layer within the expert-output tolerance, and the uneven cuts' classes (parity, mod 4) through the
oracle's class ops. On the GPU: the slices' layers on one GPU summed against the full layer (even cuts, and uneven
cuts through the class layer and the `_odd` / `_mod4` rows), the peer-memory sum at world size 1 (bit for bit the
one-GPU gather), and two ranks over NVLink and over NCCL against the one-GPU layer."""
import os
import socket

import numpy as np
import pytest
import torch

from oracle_bind import Oracle

from exl3b200 import cases as X
from exl3b200 import tp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# ------------------------------------------------------------------------------------------ the slice rule
def test_even_cuts():
    assert tp.width_slices(512, 1, 0) == [(0, 512)]
    assert [tp.width_slices(512, 2, r) for r in range(2)] == [[(0, 256)], [(256, 512)]]
    assert [tp.width_slices(512, 4, r) for r in range(4)] == [[(128 * r, 128 * (r + 1))] for r in range(4)]


def test_parity_classes_rotate_the_extra_block():
    # a 640-column expert (five blocks) over two ranks: 384/256 by the expert's parity
    assert tp.width_slices(640, 2, 0) == [(0, 384), (384, 640)]
    assert tp.width_slices(640, 2, 1) == [(384, 640), (0, 384)]
    # four blocks over three ranks
    assert tp.width_slices(512, 3, 0) == [(0, 256), (384, 512)]
    assert tp.width_slices(512, 3, 1) == [(256, 384), (0, 256)]
    assert tp.width_slices(512, 3, 2) == [(384, 512), (256, 384)]


def test_four_classes_at_four_ranks():
    # five blocks over four ranks: every rank two blocks of one class and one of each other (five of every four
    # experts)
    got = [tp.width_slices(640, 4, r) for r in range(4)]
    assert got[0] == [(0, 256), (512, 640), (384, 512), (256, 384)]
    for r in range(4):
        assert sum(hi - lo for lo, hi in got[r]) == 5 * 128


@pytest.mark.parametrize("width,world", [(512, 1), (512, 2), (512, 3), (512, 4), (640, 2), (640, 3), (640, 4),
                                         (640, 5), (1536, 4), (1536, 5), (1536, 7)])
def test_every_block_has_one_owner(width, world):
    cuts = [tp.width_slices(width, world, r) for r in range(world)]
    n_class = len(cuts[0])
    for q in range(n_class):
        owner = np.zeros(width // 128, np.int32)
        for r in range(world):
            lo, hi = cuts[r][q]
            assert lo < hi and lo % 128 == 0 and hi % 128 == 0
            owner[lo // 128:hi // 128] += 1
        assert (owner == 1).all(), (q, owner)


def test_more_ranks_than_blocks_is_refused():
    with pytest.raises(ValueError, match="more ranks than an expert has"):
        tp.width_slices(512, 8, 0)
    with pytest.raises(ValueError):
        tp.width_slices(500, 2, 0)


# ------------------------------------------------------------------------------------------ the record cut
@pytest.mark.parametrize("bits_gu,bits_dn,lo,hi", [(3, 4, 0, 256), (3, 4, 256, 512), (4, 2, 128, 384),
                                                   (5, 3, 384, 512)])
def test_record_cut_is_the_cut_plane(bits_gu, bits_dn, lo, hi):
    """Cutting the stored record by whole tiles equals relayouting the cut canonical plane (gate_up: the gate and
    up halves' rows; down: the input columns)."""
    orc = Oracle()
    rng = np.random.default_rng(lo + 7 * bits_gu)
    H, W = 256, 512
    gu = X.random_planes(rng, 2 * W, H, bits_gu, True)
    dn = X.random_planes(rng, H, W, bits_dn, False)
    rec_gu = np.concatenate([orc.codes_to_record(gu["codes"][:W], W, H, bits_gu),
                             orc.codes_to_record(gu["codes"][W:], W, H, bits_gu)])
    rec_dn = orc.codes_to_record(dn["codes"], H, W, bits_dn)
    p = {"codes": gu["codes"], "suh": gu["suh"], "suh1": gu["suh1"], "svh": gu["svh"],
         "dn_suh": np.zeros(W, np.float16), "dn_codes": dn["codes"], "dn_svh": dn["svh"]}
    q = tp.slice_planes(p, W, bits_gu, bits_dn, lo, hi)
    w = hi - lo
    want_gu = np.concatenate([orc.codes_to_record(q["codes"][:w], w, H, bits_gu),
                              orc.codes_to_record(q["codes"][w:], w, H, bits_gu)])
    want_dn = orc.codes_to_record(q["dn_codes"], H, w, bits_dn)
    assert np.array_equal(tp.slice_gu_record(rec_gu, H, W, bits_gu, lo, hi), want_gu)
    assert np.array_equal(tp.slice_dn_record(rec_dn, H, W, bits_dn, lo, hi), want_dn)
    # and the torch form (what load_slice runs on the device), with a leading expert dimension
    t = torch.from_numpy(np.stack([rec_gu, rec_gu]).view(np.int16))
    assert np.array_equal(tp.slice_gu_record(t, H, W, bits_gu, lo, hi)[1].numpy().view(np.uint16), want_gu)


# ------------------------------------------------------------------------------------------ the split on CPU ranks
def _case(seed, M, k, E, H, W, bits):
    return X.Case("moe_exl3_gate_up_down", seed, M=M, top_k=k, n_expert=E, geom=[(2 * W, H)], bits=bits)


def _layer_out(orc, case, w):
    y = orc.run_case(case)                          # the down rows (bf16 bits), sorted order
    return orc.gather(y, case.sorted_tok, w, case.M, case.top_k, case.x_cols)


def _tp_rank(rank, world, port, q, M, k, E, H, W, bits):
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        orc = Oracle()
        full = _case(11, M, k, E, H, W, bits)       # the same seeded experts, routing and tokens on every rank
        w = np.random.default_rng(5).random((M, k)).astype(np.float32)
        (lo, hi), = tp.width_slices(W, world, rank)
        planes = [tp.slice_planes(p, W, bits, bits, lo, hi) for p in full.planes]
        mine = X.Case("moe_exl3_gate_up_down", 11, M=M, top_k=k, n_expert=E, geom=[(2 * (hi - lo), H)], bits=bits,
                      planes=planes, sorted_tok=full.sorted_tok, expert_offset=full.expert_offset, x=full.x)
        part = torch.from_numpy(_layer_out(orc, mine, w))
        dist.all_reduce(part)
        q.put((rank, part.numpy(), _layer_out(orc, full, w) if rank == 0 else None))
    except Exception as exc:
        q.put((rank, repr(exc), None))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_partials_sum_to_the_layer_on_cpu_ranks(world):
    import torch.multiprocessing as mp
    M, k, E, H, W, bits = 6, 3, 4, 256, 512, 4
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_rank, args=(r, world, port, q, M, k, E, H, W, bits)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=300) for _ in range(world)), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    for rank, got, _ in res:
        assert not isinstance(got, str), f"rank {rank}: {got}"
    want = res[0][2]
    for rank, got, _ in res:
        assert np.array_equal(got, res[0][1])     # every rank holds the same sum
    err = float(np.abs(res[0][1] - want).max())
    scale = float(np.abs(want).max())
    cos = float((res[0][1] * want).sum() / np.sqrt((res[0][1] ** 2).sum() * (want ** 2).sum()))
    assert err <= 1e-2 * scale and cos >= 0.9999, (err, scale, cos)


@pytest.mark.parametrize("width,world", [(640, 2), (512, 3), (640, 3), (640, 4)])
def test_uneven_cut_classes_sum_to_the_layer(width, world):
    """A width the ranks do not divide: each rank's experts fall in classes (by parity, or by number mod 4 at four
    ranks) of different slice widths -- the class ops (`_odd` / `_mod4` tables) over the sliced planes, run by the
    oracle for every rank and summed, equal the full-width layer within the expert-output tolerance."""
    orc = Oracle()
    M, k, E, H, bits = 5, 3, 8, 256, 4
    full = _case(23, M, k, E, H, width, bits)
    w = np.random.default_rng(7).random((M, k)).astype(np.float32)
    want = _layer_out(orc, full, w)
    acc = np.zeros_like(want, dtype=np.float64)
    for r in range(world):
        cuts = tp.width_slices(width, world, r)
        n_class = len(cuts)
        assert n_class in (2, 4)
        planes = [tp.slice_planes(p, width, bits, bits, *cuts[e % n_class]) for e, p in enumerate(full.planes)]
        op = "moe_exl3_gate_up_down_mod4" if n_class == 4 else "moe_exl3_gate_up_down"
        mine = X.Case(op, 23, M=M, top_k=k, n_expert=E, geom=[(2 * (hi - lo), H) for lo, hi in cuts], n_class=n_class,
                      bits=bits, planes=planes, sorted_tok=full.sorted_tok, expert_offset=full.expert_offset, x=full.x)
        acc += _layer_out(orc, mine, w)
    err = float(np.abs(acc - want).max())
    scale = float(np.abs(want).max())
    cos = float((acc * want).sum() / np.sqrt((acc ** 2).sum() * (want.astype(np.float64) ** 2).sum()))
    assert err <= 1e-2 * scale and cos >= 0.9999, (err, scale, cos)


# ------------------------------------------------------------------------------------------ on the GPU
def _compare(a, b):
    a, b = a.double(), b.double()
    err = float((a - b).abs().max())
    scale = float(a.abs().max())
    cos = float(torch.nn.functional.cosine_similarity(a.reshape(1, -1), b.reshape(1, -1)))
    return err, scale, cos


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("T", [4, 96])
def test_width_slices_on_one_gpu_sum_to_the_layer(world, T):
    """Each rank's slice layer (load_slice on the device: records cut by whole tiles) run on one GPU; the partial
    outputs summed equal the full-width layer within the expert-output tolerance."""
    from exl3b200 import load_plugin
    from exl3b200.layer import MoeLayer
    plugin = load_plugin()
    dev = torch.device("cuda", 0)
    E, H, W, k = 32, 2048, 512, 8
    full = MoeLayer(plugin, n_expert=E, hidden=H, width=W, top_k=k, max_tokens=T, seed=3, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(T)
    full.x[:T] = torch.randn((T, H), generator=g, device=dev).to(torch.float16)
    full.logits[:T] = torch.randn((T, E), generator=g, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    full.forward(T, s)
    acc = torch.zeros((T, H), dtype=torch.float64, device=dev)
    for r in range(world):
        (lo, hi), = tp.width_slices(W, world, r)
        part = MoeLayer(plugin, n_expert=E, hidden=H, width=hi - lo, top_k=k, max_tokens=T, seed=99, device=dev)
        tp.load_slice(part, full, lo, hi)
        part.x[:T], part.logits[:T] = full.x[:T], full.logits[:T]
        part.forward(T, s)
        acc += part.out[:T].double()
    torch.cuda.synchronize()
    err, scale, cos = _compare(full.out[:T], acc)
    assert err <= 1e-2 * scale and cos >= 0.9999, (err, scale, cos)


@pytest.mark.gpu
@pytest.mark.parametrize("width,world", [(512, 3), (640, 2), (640, 4)])
@pytest.mark.parametrize("T", [4, 96])
def test_uneven_cut_class_layers_on_one_gpu_sum_to_the_layer(width, world, T):
    """The uneven cut on the device: each rank's experts in classes of different widths (ClassMoeLayer through the
    `_odd` / `_mod4` plugin rows, weights cut by load_classes), run on one GPU; the partials summed equal the
    full-width layer within the expert-output tolerance."""
    from exl3b200 import load_plugin
    from exl3b200.layer import ClassMoeLayer, MoeLayer
    plugin = load_plugin()
    dev = torch.device("cuda", 0)
    E, H, k = 32, 2048, 8
    full = MoeLayer(plugin, n_expert=E, hidden=H, width=width, top_k=k, max_tokens=T, seed=5, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(T + width)
    full.x[:T] = torch.randn((T, H), generator=g, device=dev).to(torch.float16)
    full.logits[:T] = torch.randn((T, E), generator=g, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    full.forward(T, s)
    acc = torch.zeros((T, H), dtype=torch.float64, device=dev)
    for r in range(world):
        cuts = tp.width_slices(width, world, r)
        assert len(cuts) in (2, 4)
        part = ClassMoeLayer(plugin, widths=[hi - lo for lo, hi in cuts], n_expert=E, hidden=H, top_k=k,
                             max_tokens=T, seed=99, device=dev)
        tp.load_classes(part, full, cuts)
        part.x[:T], part.logits[:T] = full.x[:T], full.logits[:T]
        part.forward(T, s)
        acc += part.out[:T].double()
    torch.cuda.synchronize()
    err, scale, cos = _compare(full.out[:T], acc)
    assert err <= 1e-2 * scale and cos >= 0.9999, (err, scale, cos)


def _tp_gpu(rank, world, port, q, cases):
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from exl3b200 import load_plugin
        from exl3b200.layer import MoeLayer
        plugin = load_plugin()
        E, H, W, k = 32, 2048, 512, 8
        res = []
        for T, transport in cases:
            full = MoeLayer(plugin, n_expert=E, hidden=H, width=W, top_k=k, max_tokens=T, seed=13, device=dev)
            lay = tp.TpLayer(plugin, rank=rank, world=world, n_expert=E, hidden=H, width=W, top_k=k, max_tokens=T,
                             seed=13, device=dev, full=full, transport=transport)
            g = torch.Generator(device=dev)
            g.manual_seed(400 + T)               # the same tokens on every rank (replicated)
            x = torch.randn((T, H), generator=g, device=dev).to(torch.float16)
            lg = torch.randn((T, E), generator=g, device=dev)
            full.x[:T], full.logits[:T], lay.x[:T], lay.logits[:T] = x, lg, x, lg
            s = torch.cuda.current_stream().cuda_stream
            full.forward(T, s)
            for _ in range(3):                   # the window and flags are reused step to step
                lay.forward(T, s)
            torch.cuda.synchronize()
            lay.check()
            same = bool(torch.equal(full.out[:T], lay.out[:T]))
            err, scale, cos = _compare(full.out[:T], lay.out[:T])
            mine = lay.out[:T].clone()
            ref = mine.clone()
            dist.broadcast(ref, 0)
            res.append((T, transport, same, err, scale, cos, bool(torch.equal(mine, ref))))
            lay.close()
        q.put((rank, res))
    except Exception as exc:
        import traceback
        q.put((rank, repr(exc) + traceback.format_exc()[-1500:]))
    finally:
        dist.barrier()
        dist.destroy_process_group()


def _spawn(world, cases):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_gpu, args=(r, world, port, q, cases)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    return res


@pytest.mark.gpu
def test_width_split_at_world_one_is_the_gather():
    """World size 1 over peer memory: gather_rs, reduce and pull over a window that maps only itself give the
    one-GPU layer's output bit for bit."""
    res = _spawn(1, [(5, "p2p"), (160, "p2p")])
    for rank, r in res:
        assert isinstance(r, list), f"rank {rank}: {r}"
        for T, transport, same, err, scale, cos, agree in r:
            assert same, (T, transport, err)


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_width_split_over_two_gpus_equals_one_gpu():
    """Two ranks, each holding half of every expert's width: over peer memory every rank holds the same bits, and
    both transports match the one-GPU layer within the expert-output tolerance."""
    res = _spawn(2, [(3, "p2p"), (256, "p2p"), (3, "nccl"), (256, "nccl")])
    for rank, r in res:
        assert isinstance(r, list), f"rank {rank}: {r}"
        for T, transport, same, err, scale, cos, agree in r:
            assert err <= 1e-2 * scale and cos >= 0.9999, (rank, T, transport, err, scale, cos)
            if transport == "p2p":
                assert agree, (rank, T)
