"""PyTorch custom operators over the C ABI (bag_b200.torch_ops): registration,
shape inference without a GPU, and on the GPU results, autograd, the in-place
form and tracing by torch.compile (eager backend: dynamo only)."""

from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")
import bag_b200.torch_ops  # noqa: E402,F401  (registers torch.ops.bag_b200.*)


def test_ops_are_registered():
    assert hasattr(torch.ops.bag_b200, "matmul")
    assert hasattr(torch.ops.bag_b200, "sgemm_")


def test_shape_inference_on_meta_tensors():
    a = torch.empty(96, 40, device="meta")
    b = torch.empty(40, 72, device="meta")
    c = torch.ops.bag_b200.matmul(a, b, 1, "minimal", "ffma")
    assert c.shape == (96, 72) and c.device.type == "meta"
    with pytest.raises(Exception):
        torch.ops.bag_b200.matmul(a, torch.empty(41, 72, device="meta"))


def _rel(x, ref):
    return float((x.double() - ref).norm() / ref.norm())


@pytest.mark.gpu
@pytest.mark.parametrize("m,k,n,depth,math", [(512, 512, 512, 1, "ffma"), (1000, 768, 520, 2, "ffma"),
                                              (2048, 2048, 2048, 1, "3xtf32")])
def test_matmul_op(cuda, m, k, n, depth, math):
    g = torch.Generator(device="cuda").manual_seed(m + k + n)
    a = torch.randn(m, k, device="cuda", generator=g)
    b = torch.randn(k, n, device="cuda", generator=g)
    c = torch.ops.bag_b200.matmul(a, b, depth, "minimal", math)
    ref = a.double() @ b.double()
    assert c.shape == (m, n) and _rel(c, ref) <= 1e-5
    c2 = torch.randn(m, n, device="cuda", generator=g)
    c2_ref = c2.double() + ref
    torch.ops.bag_b200.sgemm_(c2, a, b, 1.0, depth, "minimal", math)
    assert _rel(c2, c2_ref) <= 1e-5


@pytest.mark.gpu
def test_autograd_through_the_op(cuda):
    g = torch.Generator(device="cuda").manual_seed(7)
    a = torch.randn(256, 384, device="cuda", generator=g, requires_grad=True)
    b = torch.randn(384, 320, device="cuda", generator=g, requires_grad=True)
    w = torch.randn(256, 320, device="cuda", generator=g)
    (torch.ops.bag_b200.matmul(a, b, 1, "minimal", "ffma") * w).sum().backward()
    wd = w.double()
    assert _rel(a.grad, wd @ b.detach().double().t()) <= 1e-5
    assert _rel(b.grad, a.detach().double().t() @ wd) <= 1e-5


@pytest.mark.gpu
def test_traced_by_torch_compile(cuda):
    def f(x, y):
        return torch.ops.bag_b200.matmul(x, y, 1, "minimal", "ffma") + 1.0

    compiled = torch.compile(f, backend="eager", fullgraph=True)
    g = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn(512, 256, device="cuda", generator=g)
    y = torch.randn(256, 384, device="cuda", generator=g)
    assert _rel(compiled(x, y), x.double() @ y.double() + 1.0) <= 1e-5


class _FakeWorkspace:
    def __init__(self, key):
        self.key, self.closed = key, False

    def close(self):
        self.closed = True


def test_workspace_cache_is_bounded_and_per_stream(monkeypatch):
    """Least recently used workspaces are freed beyond the limit, and two
    streams never share one (a workspace is scratch for one call at a time)."""
    from bag_b200 import torch_ops as T
    made = []

    def fake_create(device, m, n, k, depth, basis, math):
        made.append(_FakeWorkspace((device.index, m, n, k)))
        return made[-1]

    monkeypatch.setattr(T, "_create", fake_create)
    T.clear_workspaces()
    old = T.workspace_cache_limit()
    dev = torch.device("cuda", 0)
    try:
        T.set_workspace_cache_limit(2)
        with T._lock:
            w1 = T._workspace(dev, 11, 64, 64, 64, 1, "minimal", "ffma")
            assert T._workspace(dev, 11, 64, 64, 64, 1, "minimal", "ffma") is w1
            w2 = T._workspace(dev, 22, 64, 64, 64, 1, "minimal", "ffma")   # another stream
            assert w2 is not w1
            T._workspace(dev, 11, 64, 64, 64, 1, "minimal", "ffma")        # w1 most recent
            w3 = T._workspace(dev, 11, 128, 64, 64, 1, "minimal", "ffma")
        assert w2.closed and not w1.closed and not w3.closed
        T.set_workspace_cache_limit(1)
        assert w1.closed and not w3.closed
        with pytest.raises(ValueError):
            T.set_workspace_cache_limit(0)
    finally:
        T.clear_workspaces()
        T.set_workspace_cache_limit(old)
    assert all(w.closed for w in made)


def test_cache_miss_during_graph_capture_raises(monkeypatch):
    """A workspace miss (or a cache change) while a CUDA graph is being captured
    raises instead of calling cudaMalloc/cudaFree inside the capture."""
    from bag_b200 import torch_ops as T
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: True)
    monkeypatch.setattr(T, "_create", lambda *a: _FakeWorkspace(a))
    monkeypatch.setattr(T, "_workspaces", T.OrderedDict())
    dev = torch.device("cuda", 0)
    with pytest.raises(RuntimeError, match="warm-up"):
        T._workspace(dev, 1, 64, 64, 64, 1, "minimal", "ffma")
    with pytest.raises(RuntimeError, match="capture"):
        T.clear_workspaces()
    with pytest.raises(RuntimeError, match="capture"):
        T.set_workspace_cache_limit(2)
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: False)
    ws = T._workspace(dev, 1, 64, 64, 64, 1, "minimal", "ffma")   # warm-up: created
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: True)
    assert T._workspace(dev, 1, 64, 64, 64, 1, "minimal", "ffma") is ws   # hit: fine


@pytest.mark.gpu
def test_3xtf32_op_sizes_its_workspace_for_the_prepared_path(cuda):
    """torch.ops.bag_b200.matmul(math="3xtf32") creates its workspace in that
    mode, so the call runs the prepared-operand CTA-pair kernel."""
    import bag_b200 as bag
    from bag_b200 import torch_ops as T
    n, depth = 4096, 2
    g = torch.Generator(device="cuda").manual_seed(41)
    a = torch.randn(n, n, device="cuda", generator=g)
    b = torch.randn(n, n, device="cuda", generator=g)
    c = torch.ops.bag_b200.matmul(a, b, depth, "minimal", "3xtf32")
    torch.cuda.synchronize()
    assert bag.last_leaf_kernel() == "tf32_pair"
    key = (a.device.index, torch.cuda.current_stream().cuda_stream, n, n, n, depth, "minimal",
           "3xtf32")
    assert T._workspaces[key].bytes() == bag.workspace_bytes_for(n, n, n, depth, math="3xtf32")
    assert _rel(c, a.double() @ b.double()) <= 1e-5
    assert bag.device_error() == 0


@pytest.mark.gpu
def test_op_replays_in_a_cuda_graph_after_warm_up(cuda):
    g = torch.Generator(device="cuda").manual_seed(43)
    a = torch.randn(1024, 768, device="cuda", generator=g)
    b = torch.randn(768, 640, device="cuda", generator=g)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        torch.ops.bag_b200.matmul(a, b, 2, "minimal", "ffma")   # warm-up: workspace cached
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        out = torch.ops.bag_b200.matmul(a, b, 2, "minimal", "ffma")
    a.copy_(torch.randn(1024, 768, device="cuda", generator=g))
    graph.replay()
    torch.cuda.synchronize()
    assert _rel(out, a.double() @ b.double()) <= 1e-5
