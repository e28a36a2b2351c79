"""BAG matmul as PyTorch custom operators, backed by the C ABI.

Importing this module registers

* ``torch.ops.bag_b200.matmul(a, b, depth=1, basis="minimal", math="ffma") -> c``:
  ``c = a @ b`` for 2-D FP32 CUDA tensors of any shape (a functional op with a
  fake implementation for shape inference, so it traces into torch graphs,
  and an autograd formula: ``da = dc @ b^T``, ``db = a^T @ dc``, each through
  the same op);
* ``torch.ops.bag_b200.sgemm_(c, a, b, beta=1.0, depth=1, basis="minimal",
  math="ffma")``: ``c <- a @ b + beta * c`` in place (``beta`` 0 or 1).

``math`` selects the leaf arithmetic for the call ("ffma": the reference's
sequential-fmaf numerics; "3xtf32": tcgen05 tensor cores on TF32 hi/lo
splits, used where every leaf has K >= 1024).  Workspaces are created on
first use for each (device, stream, shape, depth, basis, math) and kept, so
they are never allocated inside a timed call after that; one per stream,
because a workspace is scratch for one call at a time.  At most
``workspace_cache_limit()`` of them are kept (4 by default): the least
recently used is freed first (``cudaFree`` waits for the work still using
it).  Creating or freeing a workspace is not allowed while a CUDA graph is
being captured (``torch.cuda.graph``, ``torch.compile(mode="reduce-overhead")``):
run each shape once on the capturing stream before capture (a warm-up), so
the captured calls find their workspace cached; a miss during capture raises
instead of allocating.  This is the counterpart of
the reference's Triton entry (``src/bag_triton/bag.py:955``) in PyTorch's
operator registry; ``bag_b200.bag_matmul`` keeps the reference's own
signature and errors.
"""

from __future__ import annotations

import threading
from collections import OrderedDict

import torch

import bag_b200 as _bag

# Guards the cache and spans lookup + launch, so a workspace is never freed
# while a thread is launching into it.
_lock = threading.RLock()
_workspaces: "OrderedDict[tuple, _bag.Workspace]" = OrderedDict()
_limit = 4
_MATH = ("ffma", "3xtf32")


def _create(device: torch.device, m: int, n: int, k: int, depth: int, basis: str, math: str):
    previous = _bag.get_math_mode()
    _bag.set_math_mode(math)
    try:
        with torch.cuda.device(device):
            # Column-major view of the row-major call: C^T (n x m) = B^T A^T.
            return _bag.Workspace.for_problem(n, m, k, depth, basis)
    finally:
        _bag.set_math_mode(previous)


def _no_capture(what: str) -> None:
    if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
        raise RuntimeError(
            f"bag_b200: {what} during CUDA graph capture would call cudaMalloc/cudaFree; run "
            "this shape once on the same stream before capturing (a warm-up) so its "
            "workspace is cached, and keep the cache limit above the shapes in use")


def _workspace(device: torch.device, stream: int, m: int, n: int, k: int, depth: int,
               basis: str, math: str):
    """The cached workspace for this call (caller holds ``_lock``)."""
    key = (device.index, stream, m, n, k, depth, basis, math)
    ws = _workspaces.get(key)
    if ws is not None:
        _workspaces.move_to_end(key)
        return ws
    _no_capture(f"creating a workspace for {m}x{n}x{k} depth {depth} ({basis}, {math})")
    ws = _create(device, m, n, k, depth, basis, math)
    _workspaces[key] = ws
    while len(_workspaces) > _limit:
        _workspaces.popitem(last=False)[1].close()
    return ws


def set_workspace_cache_limit(limit: int) -> None:
    """Keep at most ``limit`` (>= 1) workspaces; frees the oldest beyond it."""
    global _limit
    if int(limit) < 1:
        raise ValueError("the workspace cache keeps at least one workspace")
    _no_capture("changing the workspace cache")
    with _lock:
        _limit = int(limit)
        while len(_workspaces) > _limit:
            _workspaces.popitem(last=False)[1].close()


def workspace_cache_limit() -> int:
    return _limit


def clear_workspaces() -> None:
    """Free the cached workspaces."""
    _no_capture("freeing workspaces")
    with _lock:
        for ws in _workspaces.values():
            ws.close()
        _workspaces.clear()


def _check(a: torch.Tensor, b: torch.Tensor, math: str) -> None:
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[0]:
        raise ValueError(f"bag_b200.matmul: shapes {tuple(a.shape)} @ {tuple(b.shape)}")
    if a.dtype != torch.float32 or b.dtype != torch.float32:
        raise ValueError("bag_b200.matmul computes in FP32: pass float32 tensors")
    if not a.is_cuda or a.device != b.device:
        raise ValueError("bag_b200.matmul: a and b must be on the same CUDA device")
    if math not in _MATH:
        raise ValueError(f"math must be one of {_MATH}, got {math!r}")


def _run(c: torch.Tensor, a: torch.Tensor, b: torch.Tensor, beta: float, depth: int, basis: str,
         math: str) -> None:
    m, k = a.shape
    n = b.shape[1]
    stream = torch.cuda.current_stream(a.device)
    with _lock:
        ws = _workspace(a.device, stream.cuda_stream, m, n, k, depth, basis, math)
        previous = _bag.get_math_mode()
        _bag.set_math_mode(math)
        try:
            with torch.cuda.device(a.device):
                _bag.sgemm(a, b, c, beta=beta, depth=depth, basis=basis, workspace=ws,
                           stream=stream)
        finally:
            _bag.set_math_mode(previous)


@torch.library.custom_op("bag_b200::matmul", mutates_args=())
def matmul(a: torch.Tensor, b: torch.Tensor, depth: int = 1, basis: str = "minimal",
           math: str = "ffma") -> torch.Tensor:
    _check(a, b, math)
    a, b = a.contiguous(), b.contiguous()
    c = torch.empty((a.shape[0], b.shape[1]), device=a.device, dtype=torch.float32)
    _run(c, a, b, 0.0, depth, basis, math)
    return c


@matmul.register_fake
def _(a, b, depth=1, basis="minimal", math="ffma"):
    torch._check(a.dim() == 2 and b.dim() == 2, lambda: "bag_b200.matmul takes 2-D tensors")
    torch._check(a.shape[1] == b.shape[0], lambda: "bag_b200.matmul: inner extents differ")
    return a.new_empty((a.shape[0], b.shape[1]))


def _setup_context(ctx, inputs, output):
    a, b, depth, basis, math = inputs
    ctx.save_for_backward(a, b)
    ctx.cfg = (depth, basis, math)


def _backward(ctx, grad):
    a, b = ctx.saved_tensors
    depth, basis, math = ctx.cfg
    grad_a = grad_b = None
    if ctx.needs_input_grad[0]:
        grad_a = torch.ops.bag_b200.matmul(grad, b.t().contiguous(), depth, basis, math)
    if ctx.needs_input_grad[1]:
        grad_b = torch.ops.bag_b200.matmul(a.t().contiguous(), grad, depth, basis, math)
    return grad_a, grad_b, None, None, None


matmul.register_autograd(_backward, setup_context=_setup_context)


@torch.library.custom_op("bag_b200::sgemm_", mutates_args=("c",))
def sgemm_(c: torch.Tensor, a: torch.Tensor, b: torch.Tensor, beta: float = 1.0, depth: int = 1,
           basis: str = "minimal", math: str = "ffma") -> None:
    _check(a, b, math)
    if tuple(c.shape) != (a.shape[0], b.shape[1]) or c.dtype != torch.float32 or c.device != a.device:
        raise ValueError("bag_b200.sgemm_: c must be a float32 (M, N) tensor on a's device")
    if not c.is_contiguous():
        raise ValueError("bag_b200.sgemm_: c must be contiguous (row-major)")
    _run(c, a.contiguous(), b.contiguous(), float(beta), depth, basis, math)


@sgemm_.register_fake
def _(c, a, b, beta=1.0, depth=1, basis="minimal", math="ffma"):
    return None
