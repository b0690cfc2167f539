"""The MoE block pass on a GPU (exl3b200_moe_block_forward): the routed layer beside the shared expert, the gather
folding the shared arm in through its sigmoid gate (architectures/qwen4exp_exl3/rad_block_moe_exl3.h:1535-1548,
1961-1965: moe_gather with act "sigmoid" over the routed rows, the shared output and the shared gate).

The routed part and the shared expert are the library's own oracle-pinned ops, so the block is checked against
their composition: the routed layer's f32 output (the same kernels), the shared expert's rows (a one-expert layer of
top-1, whose gather multiplies each row by a weight of exactly 1), and the fold restated in numpy --
out = routed + sigmoid(x . gate_w) * shared. The gate's dot product is summed in a different order on the device,
so the comparison allows max |got - want| <= 1e-5 * max |want|; the bf16 output is the f32 output rounded, to the
bit."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from exl3b200 import load_plugin  # noqa: E402
from exl3b200.layer import MoeBlock  # noqa: E402
from exl3b200.native import Native  # noqa: E402


@pytest.fixture(scope="module")
def block():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda:0")
    return MoeBlock(load_plugin(), n_expert=64, hidden=2048, width=512, top_k=10, bits_gu=3, bits_dn=4,
                    shared_width=1024, shared_bits=4, max_tokens=512, seed=11, device=dev)


@pytest.mark.parametrize("T", [1, 8, 512])
def test_block_is_the_routed_layer_plus_the_gated_shared_expert(block, T):
    dev = block.routed.dev
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + T)
    x = torch.randn((T, 2048), generator=g, device=dev).to(torch.float16)
    lg = torch.randn((T, 64), generator=g, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    out = torch.full((T, 2048), float("nan"), device=dev)
    block.forward(T, s, x=x, logits=lg, out=out)
    out_bf = torch.zeros((T, 2048), dtype=torch.bfloat16, device=dev)
    block.forward(T, s, x=x, logits=lg, out=out_bf)
    # the composition: the routed layer, and the shared expert as a one-expert top-1 layer (its gather weight is 1)
    routed = torch.empty((T, 2048), device=dev)
    block.routed.forward(T, s, x=x, logits=lg, out=routed)
    shared = torch.empty((T, 2048), device=dev)
    block.shared.forward(T, s, x=x, logits=torch.zeros((T, 1), device=dev), out=shared)
    torch.cuda.synchronize()
    xf = x.float().cpu().numpy()
    gw = block.sgate_w.float().cpu().numpy()
    gate = (xf * gw).sum(1, dtype=np.float32)
    sig = (np.float32(1) / (np.float32(1) + np.exp(-gate))).astype(np.float32)
    want = routed.cpu().numpy() + sig[:, None] * shared.cpu().numpy()
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    err = float(np.abs(got - want).max())
    assert err <= 1e-5 * float(np.abs(want).max()), err
    # the shared arm moves the output (a control), and the bf16 output is the f32 one rounded
    assert float(np.abs(got - routed.cpu().numpy()).max()) > 1e-3
    assert torch.equal(out_bf, out.to(torch.bfloat16))
    assert Native().read_error() == 0


def test_block_replays_in_a_cuda_graph(block):
    dev = block.routed.dev
    T = 64
    g = torch.Generator(device=dev)
    g.manual_seed(77)
    block.x[:T] = torch.randn((T, 2048), generator=g, device=dev).to(torch.float16)
    block.logits[:T] = torch.randn((T, 64), generator=g, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    block.forward(T, s)
    torch.cuda.synchronize()
    ref = block.out[:T].clone()
    block.out.zero_()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        block.forward(T, torch.cuda.current_stream().cuda_stream)
    gr.replay()
    torch.cuda.synchronize()
    assert torch.equal(ref, block.out[:T])
