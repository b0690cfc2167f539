"""The headline configuration as a whole layer, on the GPU, against the oracle.

The bench's workload -- 512 experts of hidden 2048 / width 512, top-10 softmax routing, gate_up K=3 (h_rot 1) and
down K=4 (h_rot 1), mul1 -- run through MoeLayer (router -> stable scatter -> the moe_exl3_gate_up and moe_exl3_down
plugin rows -> weighted gather, every step a kernel of libexl3b200.so) at T = 1, 8, 64, 512 and 2048 tokens, and
compared with the oracle's chain on the same weights and the same routing:

- routing to the bit: the top-10 ids are numpy's stable argsort of -logits, sorted_tok / expert_offset the stable
  counting sort of the routing contract (include/exl3_abi.h:96-158), the weights the softmax (rel 1e-5);
- every token's output: the oracle's gate_up (kernels/exl3ref/ref.c:171-228 restated) into h, its down into the
  bf16 rows, its gather (ascending slots, f32) -- within the expert-output tolerance the op tests use:
  max |got - want| / max |want| <= 1e-2 and cosine >= 0.9999, no NaN.

The layer's weights live on the device as tile-stream records; the oracle reads canonical planes, recovered from the
records by the oracle's own relayout (pinned to the reference's common/exl3_layout.c on the CPU)."""
import os
import types
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle_bind import Oracle  # noqa: E402
from exl3b200 import cases as X  # noqa: E402
from exl3b200 import load_plugin  # noqa: E402

REL_TOL, COS_TOL = 1e-2, 0.9999
E, H, W, K_TOP, KGU, KDN = 512, 2048, 512, 10, 3, 4
T_MAX = 2048
THREADS = max(1, os.cpu_count() or 1)


@pytest.fixture(scope="module")
def layer():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from exl3b200.layer import MoeLayer
    lay = MoeLayer(load_plugin(), n_expert=E, hidden=H, width=W, top_k=K_TOP, bits_gu=KGU, bits_dn=KDN,
                   codebook="mul1", max_tokens=T_MAX, seed=11)
    g = torch.Generator(device="cuda")
    g.manual_seed(12)
    lay.x.copy_(torch.randn(lay.x.shape, generator=g, device="cuda").to(torch.float16))
    lay.logits.copy_(torch.randn(lay.logits.shape, generator=g, device="cuda"))
    torch.cuda.synchronize()
    return lay


@pytest.fixture(scope="module")
def planes(layer):
    """Every expert's canonical planes, recovered from the layer's device records by the oracle's relayout."""
    orc = Oracle()
    gu_rec = layer.gu_rec.cpu().numpy().view(np.uint16)
    dn_rec = layer.dn_rec.cpu().numpy().view(np.uint16)
    suh = layer.suh.cpu().numpy().view(np.uint16).reshape(E, H)
    suh1 = layer.suh1.cpu().numpy().view(np.uint16).reshape(E, H)
    svh_gu = layer.svh_gu.cpu().numpy().view(np.uint16).reshape(E, 2 * W)
    dn_suh = layer.dn_suh.cpu().numpy().view(np.uint16).reshape(E, W)
    svh_dn = layer.svh_dn.cpu().numpy().view(np.uint16).reshape(E, H)
    half = W * H * KGU // 16

    def one(e):
        gate = orc.record_to_codes(gu_rec[e, :half], W, H, KGU)
        up = orc.record_to_codes(gu_rec[e, half:], W, H, KGU)
        return {"codes": np.concatenate([gate, up], 0), "suh": suh[e].copy(), "suh1": suh1[e].copy(),
                "svh": svh_gu[e].copy(), "dn_suh": dn_suh[e].copy(),
                "dn_codes": orc.record_to_codes(dn_rec[e], H, W, KDN), "dn_svh": svh_dn[e].copy()}

    with ThreadPoolExecutor(THREADS) as ex:
        return list(ex.map(one, range(E)))


def _oracle_layer(orc, pl, x_bits, ids, w):
    """The oracle's layer over the given routing: gate_up (h_rot 1) -> down (h_rot 1) -> gather; f32 [T, H]."""
    T = x_bits.shape[0]
    st, off = X.stable_scatter(ids, E)
    gu = types.SimpleNamespace(base="moe_exl3_gate_up", bits=KGU, codebook="mul1", T=T * K_TOP, n_expert=E,
                               top_k=K_TOP, n_class=1, x_dtype="f16", planes=pl, sorted_tok=st, expert_offset=off)
    h = orc._run(gu, 1, 1, 0, x_bits, [(2 * W, H)], "own", THREADS)
    dpl = [{"codes": p["dn_codes"], "suh": p["dn_suh"], "svh": p["dn_svh"]} for p in pl]
    dn = types.SimpleNamespace(base="moe_exl3_down", bits=KDN, codebook="mul1", T=T * K_TOP, n_expert=E,
                               top_k=K_TOP, n_class=1, x_dtype="f16", planes=dpl, sorted_tok=st, expert_offset=off)
    y = orc._run(dn, 0, 1, 0, h, [(H, W)], "own", THREADS)
    return orc.gather(y, st, w, T, K_TOP, H)


@pytest.mark.parametrize("T", [1, 8, 64, 512, 2048])
def test_config3_layer_matches_the_oracle(layer, planes, T):
    orc = Oracle()
    s = torch.cuda.current_stream().cuda_stream
    layer.forward(T, s)
    torch.cuda.synchronize()
    assert layer.native.read_error() == 0
    logits = layer.logits[:T].cpu().numpy()
    ids = layer.ids[:T].cpu().numpy()
    w = layer.w[:T].cpu().numpy()
    # routing, to the bit
    want_ids = np.argsort(-logits, axis=1, kind="stable")[:, :K_TOP].astype(np.int32)
    assert np.array_equal(ids, want_ids)
    p = np.exp(logits.astype(np.float64) - logits.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    assert np.allclose(w, np.take_along_axis(p, want_ids, 1), rtol=1e-5, atol=1e-7)
    st_want, off_want = X.stable_scatter(ids, E)
    assert np.array_equal(layer.offset.cpu().numpy(), off_want)
    assert np.array_equal(layer.sorted_tok[:T * K_TOP].cpu().numpy(), st_want)
    # every token's output against the oracle's layer on the same weights and routing
    x_bits = layer.x[:T].cpu().numpy().view(np.uint16)
    want = _oracle_layer(orc, planes, x_bits, ids, w).astype(np.float64)
    got = layer.out[:T].cpu().numpy().astype(np.float64)
    assert not np.isnan(got).any()
    rel = np.abs(got - want).max() / np.abs(want).max()
    cos = float((got * want).sum() / (np.linalg.norm(got) * np.linalg.norm(want)))
    assert rel <= REL_TOL and cos >= COS_TOL, f"T {T}: max rel err {rel:.3e}, cosine {cos:.7f}"
