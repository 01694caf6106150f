"""GraphedForward: the forward captured as one CUDA graph replays the same
kernels on the same data, so its output equals the eager forward's bit for
bit (bf16 and fp32 modules, fixed and adaptive k)."""
import pytest
import torch

from gsa_gdn_benchmarkstudy_b200 import GatedSparseAttention, _lib
from gsa_gdn_benchmarkstudy_b200.build import build
from gsa_gdn_benchmarkstudy_b200.workloads import TEST_CONFIGS, init_weights_, make_input

pytestmark = pytest.mark.gpu
torch.set_grad_enabled(False)


@pytest.fixture(scope="module", autouse=True)
def _lib_built():
    build()
    _lib.load()
    yield
    assert _lib.device_error() == 0


def _model(cfg, adaptive=False):
    m = GatedSparseAttention(**cfg.module_kwargs(), adaptive_k=adaptive)
    init_weights_(m, seed=1)
    m = m.to(cfg.torch_dtype).cuda().eval()
    m.fuse_projections()
    return m


@pytest.mark.parametrize("name,adaptive", [("tiny_bf16", False), ("small_bf16", False),
                                           ("tiny_fp32", False), ("small_bf16", True)])
def test_replay_equals_eager(name, adaptive):
    cfg = TEST_CONFIGS[name]
    m = _model(cfg, adaptive)
    x0 = make_input(cfg).cuda()
    x1 = torch.randn(x0.shape, generator=torch.Generator().manual_seed(7)).to(x0)
    g = m.graphed(x0.shape)
    ref0, ref1 = m(x0).clone(), m(x1).clone()
    assert torch.equal(g(x0), ref0)
    assert torch.equal(g(x1), ref1)
    # an eager call between replays uses its own scratch and leaves the graph's alone
    eager = m(x0)
    g.x.copy_(x0)
    assert torch.equal(g(), ref0) and torch.equal(eager, ref0)
    torch.cuda.synchronize()


def test_replay_on_another_stream_and_shape_check():
    cfg = TEST_CONFIGS["tiny_bf16"]
    m = _model(cfg)
    x = make_input(cfg).cuda()
    g = m.graphed(x.shape)
    ref = m(x).clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        out = g(x).clone()
    torch.cuda.current_stream().wait_stream(s)
    assert torch.equal(out, ref)
    with pytest.raises(RuntimeError, match="captured for"):
        g(x[:, :-1])


@pytest.mark.parametrize("name,chunks,adaptive", [
    ("tiny_bf16", 2, False), ("tiny_fp32", 2, False), ("cfg2", 4, False), ("cfg2", None, False),
    ("small_bf16", None, True)])
def test_host_replay_equals_forward_host(name, chunks, adaptive):
    """The captured host-to-host pipeline (pinned copies in, row blocks or batch
    groups on two streams, pinned copies out) equals forward_host bit for bit."""
    from gsa_gdn_benchmarkstudy_b200.workloads import CONFIGS
    cfg = TEST_CONFIGS.get(name) or CONFIGS[name]
    m = _model(cfg, adaptive)
    x0 = make_input(cfg)
    x1 = torch.randn(x0.shape, generator=torch.Generator().manual_seed(3)).to(x0.dtype)
    ref0 = m.forward_host(x0, chunks=chunks).clone()
    ref1 = m.forward_host(x1, chunks=chunks).clone()
    g = m.graphed_host(x0.shape, chunks=chunks)
    out = g(x0)
    assert out is g.out and not out.is_cuda and torch.equal(out, ref0)
    assert torch.equal(g(x1), ref1)
    g.x.copy_(x0)
    assert torch.equal(g(), ref0)
    with pytest.raises(RuntimeError, match="captured for"):
        g(x0.cuda())
