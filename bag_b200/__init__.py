"""B200-native BAG (alternative-basis Strassen-Winograd) FP32 matmul.

Python host mirror of the reference's operator interfaces, over the C ABI of
``libbag_b200.so`` (``include/bag_capi.h``):

* :func:`bag_matmul` / :func:`allocate_bag_workspace` / :func:`bag_primitive`
  mirror ``src/bag_triton/bag.py:865-994`` and ``src/bag_triton/primitive.py:256-300``
  (same names, argument meaning and exception types), computing on the CUDA
  kernels of this package at any recursion depth.
* :func:`sgemm` / :func:`sgemm_batched` expose the C ABI's rectangular,
  row/column-major and batched entry points.
* :class:`Workspace` and :func:`matmul` follow ``bag_cuda::Workspace`` /
  ``bag_cuda::matmul`` (``include/bag/cuda/bag.cuh:34-55,247-260``):
  column-major ``C <- A@B + C``.

There is no CPU fallback: every call runs the CUDA kernels and raises if the
shared library has not been built.
"""

from __future__ import annotations

import ctypes
import json
import os
import warnings
from typing import NamedTuple, Optional

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libbag_b200.so")

BASIS = {"minimal": 0, "full": 1, "classic": 2, "winograd": 3}
SCHEDULE = {"serial": 0, "seven": 1, "seven-stream": 1, "batched": 2}
LAYOUT = {"col": 0, "row": 1}

# strassen_cuda::Backend names in enum order (include/bag/cuda/strassen.cuh:11-55).
BACKENDS = (
    "legacy", "large", "medium", "huge", "sync64_k8_r8", "pipe64_k8_r8", "pipe64_k16_r8",
    "pipe64_k16_r4", "pipe64x32_k16_r4", "pipe128x64_k16_r8x4", "pipe128_k16_r8",
    "swizzle64_k16_r4", "swizzle64x32_k16_r4", "swizzle32x64_k16_r4", "coalesced64_k16_r4",
    "swizzle_coalesced64_k16_r4", "swizzle64_k8_r8x4", "swizzle64_k16_r8x4",
    "swizzle_coalesced64_k8_r4", "swizzle_coalesced64_k32_r4", "exact_coalesced64_k16_r4",
    "exact_swizzle_coalesced64_k16_r4", "deferred_exact_coalesced64_k16_r4",
    "deferred_exact_swizzle_coalesced64_k16_r4", "sliced1_64x32_k8_r8x4",
    "sliced2_64x32_k8_r8x4", "sliced4_64x32_k8_r8x4", "striped_sliced1_64x32_k8_r8x4",
    "striped_sliced2_64x32_k8_r8x4", "striped_sliced4_64x32_k8_r8x4",
    "cg_exact_swizzle_coalesced64_k16_r4", "cg_deferred_exact_swizzle_coalesced64_k16_r4",
    "ldg_deferred_exact_swizzle_coalesced64_k16_r4", "striped_tile64_k16_r8x4",
    "striped_tile128x64_k16_r8x4", "striped_tile64x128_k16_r8x4", "register_stage64_k16_r4x4",
    "column_tile64_k16_r4x8", "register_stage64_k16_r4x8", "column_tile64_k8_r4x8",
    "column_immediate64_k16_r4x8", "column_min5_64_k16_r4x8",
)
BACKEND_IDS = {name: i for i, name in enumerate(BACKENDS)}

STATUS = {0: "ok", 1: "invalid", 2: "shape", 3: "workspace", 4: "unsupported", 5: "cuda",
          6: "internal"}

# Every C entry point, with its ctypes signature (checked by the CPU tests).
_VP, _I, _LL, _F, _SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_float, ctypes.c_size_t
SIGNATURES = {
    "bag_last_error": (ctypes.c_char_p, []),
    "bag_version": (ctypes.c_char_p, []),
    "bag_local_elements": (_I, [_I, _I, _I, ctypes.POINTER(_SZ)]),
    "bag_workspace_create": (_I, [_I, _I, _I, ctypes.POINTER(_VP)]),
    "bag_workspace_create_ex": (_I, [_I, _I, _I, _I, _I, _I, ctypes.POINTER(_VP)]),
    "bag_workspace_destroy": (_I, [_VP]),
    "bag_workspace_bytes_for": (_I, [_I, _I, _I, _I, _I, _I, _I, ctypes.POINTER(_SZ)]),
    "bag_workspace_bytes": (_SZ, [_VP]),
    "bag_workspace_data": (_VP, [_VP]),
    "bag_matmul": (_I, [_VP, _VP, _VP, _I, _VP, _VP, _I, _I]),
    "bag_sgemm_ex": (_I, [_I, _I, _I, _I, _VP, _LL, _VP, _LL, _VP, _LL, _F, _I, _I, _VP, _VP]),
    "bag_sgemm_batched": (_I, [_I, _I, _I, _I, _VP, _LL, _LL, _VP, _LL, _LL, _VP, _LL, _LL, _I,
                               _F, _I, _I, _VP, _VP]),
    "bag_sgemm_noalloc": (_I, [_I, _I, _I, _I, _VP, _LL, _VP, _LL, _VP, _LL, _F, _I, _I, _VP]),
    "bag_primitive": (_I, [_I, _I, _I, _I, _I, _VP, _VP, _VP, _VP, _VP, _VP, _I, _I, _I, _LL, _LL,
                           _LL, _LL, _LL, _LL, _VP]),
    "bag_primitive_pair": (_I, [_I, _I, _I, _I, _I, ctypes.POINTER(_VP), ctypes.POINTER(_VP), _I,
                                _LL, _VP]),
    "bag_strassen_one_level": (_I, [_I, _I, _VP, _VP, _VP, _I, _VP]),
    "bag_valid_shape": (_I, [_I, _I, ctypes.POINTER(_I)]),
    "bag_plan_dump": (_I, [_I, _I, _I, _LL, _LL, _LL, _I, _I, ctypes.c_char_p, _SZ,
                           ctypes.POINTER(_SZ)]),
    "bag_profile_set_events": (_I, [_VP, _VP]),
    "bag_profile_set_phase_events": (_I, [_VP, _VP]),
    "bag_launch_count": (ctypes.c_ulonglong, []),
    "bag_device_allocations": (ctypes.c_ulonglong, []),
    "bag_ffma_probe": (_I, [_VP, _I, _VP, ctypes.POINTER(ctypes.c_double)]),
    "bag_device_error": (_I, [ctypes.POINTER(ctypes.c_uint)]),
    "bag_set_math_mode": (_I, [_I]),
    "bag_get_math_mode": (_I, []),
    "bag_last_leaf_path": (_I, []),
    "bag_last_leaf_kernel": (_I, []),
    "bag_last_prepare_table": (_I, []),
    "bag_selftest_bounded_wait": (_I, [ctypes.c_ulonglong, ctypes.POINTER(_I)]),
    "bag_multi_grid": (_I, [_I, ctypes.POINTER(_I), ctypes.POINTER(_I)]),
    "bag_multi_workspace_create": (_I, [_I, ctypes.POINTER(_I), _I, _I, _I, _I, _I, _I,
                                        ctypes.POINTER(_VP)]),
    "bag_multi_workspace_destroy": (_I, [_VP]),
    "bag_sgemm_multi": (_I, [_I, ctypes.POINTER(_I), _I, _I, _I, _I, _VP, _LL, _VP, _LL, _VP, _LL,
                             _F, _I, _I, _VP, _VP]),
}
MATH = {"ffma": 0, "3xtf32": 1}
LEAF_KERNELS = {0: "ffma", 1: "tf32_fused", 2: "tf32_single", 3: "tf32_pair"}

_lib = None


class BagError(RuntimeError):
    """A C-ABI call failed; ``status`` is the ``bag_status`` name."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = STATUS.get(status, str(status))


def lib() -> ctypes.CDLL:
    """Load ``libbag_b200.so``; raises when it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python bag_b200/build.py` "
                               "(there is no CPU fallback)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = handle
    return _lib


def _check(status: int) -> None:
    if status != 0:
        msg = lib().bag_last_error().decode()
        if status in (1, 2, 3):
            raise ValueError(f"{STATUS[status]}: {msg}")
        raise BagError(status, msg)


DEPTH_AUTO = -1   # BAG_DEPTH_AUTO


def _depth(depth) -> int:
    """An explicit depth, or "auto" / -1 for the library's choice (BAG_DEPTH_AUTO)."""
    if isinstance(depth, str):
        if depth != "auto":
            raise ValueError(f"unknown depth {depth!r}")
        return DEPTH_AUTO
    return int(depth)


def _basis(basis) -> int:
    if isinstance(basis, int):
        return basis
    if basis not in BASIS:
        raise ValueError(f"basis must be one of {sorted(BASIS)}, got {basis!r}")
    return BASIS[basis]


def plan_dump(m: int, n: int, k: int, lda: int, ldb: int, ldc: int, depth: int,
              basis="minimal") -> dict:
    """The host plan of a column-major problem as a dict (no GPU needed)."""
    need = ctypes.c_size_t(0)
    depth = _depth(depth)
    _check(lib().bag_plan_dump(m, n, k, lda, ldb, ldc, depth, _basis(basis), None, 0,
                               ctypes.byref(need)))
    buf = ctypes.create_string_buffer(need.value)
    _check(lib().bag_plan_dump(m, n, k, lda, ldb, ldc, depth, _basis(basis), buf, need.value,
                               ctypes.byref(need)))
    return json.loads(buf.value.decode())


def launch_count() -> int:
    """Kernels this process has launched through the library."""
    return int(lib().bag_launch_count())


def device_allocations() -> int:
    """Device allocations (cudaMalloc calls) the library has made in this process."""
    return int(lib().bag_device_allocations())


def workspace_bytes_for(m: int, n: int, k: int, depth=1, basis="minimal", batch: int = 1,
                        math: Optional[str] = None) -> int:
    """Bytes a workspace for column-major ``C(m x n) += A(m x k) B(k x n)``
    takes when created in math mode ``math`` (default: this thread's mode)."""
    mode = MATH[get_math_mode() if math is None else math]
    out = ctypes.c_size_t(0)
    _check(lib().bag_workspace_bytes_for(mode, m, n, k, _depth(depth), _basis(basis), batch,
                                         ctypes.byref(out)))
    return out.value


def profile_events(start=None, end=None) -> None:
    """Bracket later leaf launches of this thread with two ``torch.cuda.Event``s."""
    handle = lambda ev: None if ev is None else ev.cuda_event  # noqa: E731
    _check(lib().bag_profile_set_events(handle(start), handle(end)))


def profile_phase_events(after_stages=None, after_last=None) -> None:
    """Record ``after_stages`` once later calls' materialisation launches are
    queued and ``after_last`` after their last launch (``torch.cuda.Event``s)."""
    handle = lambda ev: None if ev is None else ev.cuda_event  # noqa: E731
    _check(lib().bag_profile_set_phase_events(handle(after_stages), handle(after_last)))


def set_math_mode(mode: str) -> None:
    """Leaf arithmetic of later calls on this thread: "ffma" (default) or "3xtf32"."""
    if mode not in MATH:
        raise ValueError(f"math mode must be one of {sorted(MATH)}, got {mode!r}")
    _check(lib().bag_set_math_mode(MATH[mode]))


def get_math_mode() -> str:
    return {v: k for k, v in MATH.items()}[int(lib().bag_get_math_mode())]


def last_leaf_path() -> str:
    """Leaf arithmetic ("ffma" or "3xtf32") the last call on this thread used."""
    return {v: k for k, v in MATH.items()}[int(lib().bag_last_leaf_path())]


def last_leaf_kernel() -> str:
    """Leaf kernel the last call on this thread ran: "ffma", "tf32_fused"
    (transforms in the tensor kernel's prologue), "tf32_single" (prepared
    operands, 128 x 256 tiles per SM) or "tf32_pair" (prepared operands,
    256 x 256 tiles per cluster of two SMs)."""
    return LEAF_KERNELS[int(lib().bag_last_leaf_kernel())]


def last_prepare_table() -> int:
    """Prepare kernel of the last call: 1 Minimal, 2 Full, 3 Classic, 4 Winograd
    for a basis whose operand expressions are compiled in, 0 for the
    plan-reading kernel, -1 when the last call prepared nothing."""
    return int(lib().bag_last_prepare_table())


def selftest_bounded_wait(limit_ns: int = 1_000_000) -> bool:
    """Run the bounded-wait self-test (a wait on an mbarrier nothing arrives on,
    giving up after ``limit_ns``); True when the wait gave up and the kernel
    returned.  Leaves the device error word at 1 (see ``device_error``)."""
    flag = _I(0)
    _check(lib().bag_selftest_bounded_wait(int(limit_ns), ctypes.byref(flag)))
    return bool(flag.value)


def device_error() -> int:
    """Read and clear the device error word (0 when no in-kernel wait timed out)."""
    out = ctypes.c_uint(0)
    _check(lib().bag_device_error(ctypes.byref(out)))
    return int(out.value)


def local_elements(n: int, depth: int, basis="minimal") -> int:
    """``bag_cuda::local_elements`` (``bag.cuh:23-30``)."""
    out = ctypes.c_size_t(0)
    _check(lib().bag_local_elements(n, depth, _basis(basis), ctypes.byref(out)))
    return out.value


def valid_shape(backend, s: int) -> bool:
    """``strassen_cuda::valid_shape`` (``strassen.cuh:57-66``)."""
    out = ctypes.c_int(0)
    _check(lib().bag_valid_shape(_backend(backend), s, ctypes.byref(out)))
    return bool(out.value)


def _backend(backend) -> int:
    if isinstance(backend, int):
        return backend
    if backend not in BACKEND_IDS:
        raise ValueError(f"unknown backend {backend!r}")
    return BACKEND_IDS[backend]


# ---------------------------------------------------------------------------
# CUDA-side helpers (torch is plumbing: device memory and streams).
# ---------------------------------------------------------------------------

def _torch():
    import torch
    return torch


def _stream_handle(stream=None, device: Optional[int] = None) -> Optional[int]:
    """The raw cudaStream_t of `stream`, else torch's current stream on `device`
    (the current device when None) -- read without building a Stream object,
    which costs more than the rest of a small call's Python work."""
    if stream is not None:
        return stream.cuda_stream
    torch = _torch()
    if device is None:
        device = torch.cuda.current_device()
    return torch._C._cuda_getCurrentRawStream(device)


def _layout_of(t) -> Optional[tuple[str, int]]:
    """('row', ld) / ('col', ld) for a 2-D tensor with one unit stride."""
    r, c = t.shape
    s0, s1 = t.stride()
    if (s1 == 1 or c <= 1) and s0 >= max(c, 1):
        return "row", max(s0, 1)
    if (s0 == 1 or r <= 1) and s1 >= max(r, 1):
        return "col", max(s1, 1)
    return None


class Workspace:
    """Device workspace for one problem shape (``bag_cuda::Workspace``, ``bag.cuh:34-55``).

    Allocation happens here, never inside a matmul call.  Not reentrant: one
    workspace per concurrently running call.
    """

    def __init__(self, n: int, depth: int = 1, basis="minimal", *, m: Optional[int] = None,
                 k: Optional[int] = None, batch: int = 1, square: bool = True):
        self.n, self.depth, self.basis = n, depth, basis
        self.m = n if m is None else m
        self.k = n if k is None else k
        self.batch = batch
        handle = ctypes.c_void_p()
        if square and m is None and k is None and batch == 1 and _depth(depth) >= 0:
            _check(lib().bag_workspace_create(n, depth, _basis(basis), ctypes.byref(handle)))
        else:
            _check(lib().bag_workspace_create_ex(self.m, n, self.k, _depth(depth), _basis(basis), batch,
                                                 ctypes.byref(handle)))
        self._handle = handle

    @classmethod
    def for_problem(cls, m: int, n: int, k: int, depth: int = 1, basis="minimal", batch: int = 1):
        """Workspace for column-major ``C(m x n) += A(m x k) B(k x n)``."""
        return cls(n, depth, basis, m=m, k=k, batch=batch, square=False)

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._handle

    def bytes(self) -> int:
        return int(lib().bag_workspace_bytes(self._handle))

    def close(self) -> None:
        if getattr(self, "_handle", None) and self._handle.value:
            lib().bag_workspace_destroy(self._handle)
            self._handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def matmul(a, b, c, n: int, workspace: Workspace, backend="column_tile64_k16_r4x8",
           schedule="batched", stream=None) -> None:
    """``bag_cuda::matmul``: column-major ``C <- A@B + C`` on device pointers or tensors."""
    ptr = lambda x: x if isinstance(x, int) else x.data_ptr()  # noqa: E731
    _check(lib().bag_matmul(ptr(a), ptr(b), ptr(c), n, _stream_handle(stream), workspace.handle,
                            _backend(backend), SCHEDULE[schedule]))


def sgemm(a, b, c, *, beta: float = 1.0, depth: int = 1, basis="minimal",
          workspace: Optional[Workspace] = None, stream=None):
    """``c <- a @ b + beta*c`` (beta 0 or 1) for FP32 CUDA tensors of any shape.

    All three tensors must be row-major or all column-major (one unit stride);
    ragged extents are peeled inside the library.  Returns ``c``.
    """
    m, k = a.shape
    k2, n = b.shape
    if k2 != k or tuple(c.shape) != (m, n):
        raise ValueError(f"shape mismatch: {tuple(a.shape)} @ {tuple(b.shape)} -> {tuple(c.shape)}")
    la, lb, lc = _layout_of(a), _layout_of(b), _layout_of(c)
    if la is None or lb is None or lc is None or not (la[0] == lb[0] == lc[0]):
        raise ValueError("sgemm needs a, b, c all row-major or all column-major")
    ws = workspace.handle if workspace is not None else None
    _check(lib().bag_sgemm_ex(LAYOUT[la[0]], m, n, k, a.data_ptr(), la[1], b.data_ptr(), lb[1],
                              c.data_ptr(), lc[1], float(beta), _depth(depth), _basis(basis),
                              _stream_handle(stream, c.get_device()), ws))
    _warn_if_fused(workspace)
    return c


def _warn_if_fused(workspace) -> None:
    """Warn (once per call site) when a 3xTF32 call ran the fused-transform
    tensor kernel although a workspace was given: that workspace was created
    in FFMA mode and lacks the prepared operands of the fast path."""
    # Kernel id 1 (the fused-transform tensor kernel) runs only in 3xTF32 mode.
    if workspace is not None and int(lib().bag_last_leaf_kernel()) == 1:
        warnings.warn("bag_b200: this 3xTF32 call ran the fused-transform tensor kernel because "
                      "its workspace was created in FFMA mode; create the workspace after "
                      "set_math_mode('3xtf32') (size: workspace_bytes_for(..., math='3xtf32')) "
                      "for the prepared-operand kernel", RuntimeWarning, stacklevel=3)


def multi_grid(ngpus: int) -> tuple[int, int]:
    """The R x S device grid ``sgemm_multi`` uses for ``ngpus`` devices."""
    r, c = _I(0), _I(0)
    _check(lib().bag_multi_grid(int(ngpus), ctypes.byref(r), ctypes.byref(c)))
    return r.value, c.value


class MultiWorkspace:
    """Shard buffers, per-device workspaces and streams for ``sgemm_multi`` of
    one row-major problem ``C(m x n) = A(m x k) B(k x n)`` over ``devices``
    (the first holds A, B and C).  Created in the calling thread's math mode."""

    def __init__(self, devices, m: int, n: int, k: int, depth: int = 1, basis="minimal"):
        self.devices = [int(d) for d in devices]
        self.shape, self.depth, self.basis = (m, n, k), depth, basis
        self._devs = (_I * len(self.devices))(*self.devices)
        handle = ctypes.c_void_p()
        _check(lib().bag_multi_workspace_create(len(self.devices), self._devs, LAYOUT["row"], m, n, k,
                                                _depth(depth), _basis(basis), ctypes.byref(handle)))
        self._handle = handle

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._handle

    def close(self) -> None:
        if getattr(self, "_handle", None) and self._handle.value:
            lib().bag_multi_workspace_destroy(self._handle)
            self._handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def sgemm_multi(a, b, c, workspace: MultiWorkspace, *, beta: float = 1.0, stream=None):
    """``c <- a @ b + beta*c`` over ``workspace.devices`` (row-major FP32 tensors
    on the first device): each device computes its row/column bands of C from
    peer-copied shards; ``stream`` (of the first device) waits for all of them."""
    m, k = a.shape
    k2, n = b.shape
    if k2 != k or tuple(c.shape) != (m, n) or (m, n, k) != workspace.shape:
        raise ValueError("shape differs from the multi-GPU workspace's")
    for t in (a, b, c):
        if not t.is_contiguous():
            raise ValueError("sgemm_multi needs contiguous row-major tensors")
    ws = workspace
    if stream is None:
        stream = _torch().cuda.current_stream(ws.devices[0])
    _check(lib().bag_sgemm_multi(len(ws.devices), ws._devs, LAYOUT["row"], m, n, k, a.data_ptr(), k,
                                 b.data_ptr(), n, c.data_ptr(), n, float(beta), _depth(ws.depth),
                                 _basis(ws.basis), _stream_handle(stream), ws.handle))
    return c


def sgemm_batched(a, b, c, *, beta: float = 1.0, depth: int = 1, basis="minimal",
                  workspace: Optional[Workspace] = None, stream=None):
    """Batched ``c[i] <- a[i] @ b[i] + beta*c[i]`` for contiguous 3-D row-major tensors."""
    batch, m, k = a.shape
    _, k2, n = b.shape
    if k2 != k or tuple(c.shape) != (batch, m, n) or b.shape[0] != batch:
        raise ValueError("batched shape mismatch")
    for t in (a, b, c):
        if not t.is_contiguous():
            raise ValueError("sgemm_batched needs contiguous row-major tensors")
    ws = workspace.handle if workspace is not None else None
    _check(lib().bag_sgemm_batched(LAYOUT["row"], m, n, k, a.data_ptr(), k, m * k, b.data_ptr(), n,
                                   k * n, c.data_ptr(), n, m * n, batch, float(beta), _depth(depth),
                                   _basis(basis), _stream_handle(stream, c.get_device()), ws))
    _warn_if_fused(workspace)
    return c


def strassen_one_level(a, b, c, n: int, backend="column_tile64_k16_r4x8",
                       schedule="four_batched_atomic", stream=None) -> None:
    """``strassen_cuda::one_level`` (``strassen.cuh:225-276``): column-major ``C <- A@B + C``."""
    names = ["serial_atomic", "serial_normal", "seven_atomic", "dependency_normal",
             "paired_atomic", "paired_normal", "four_batched_atomic"]
    ptr = lambda x: x if isinstance(x, int) else x.data_ptr()  # noqa: E731
    _check(lib().bag_strassen_one_level(_backend(backend), names.index(schedule), ptr(a), ptr(b),
                                        ptr(c), n, _stream_handle(stream)))


# ---------------------------------------------------------------------------
# The reference's Python operator interface (src/bag_triton), on these kernels.
# ---------------------------------------------------------------------------

class BagWorkspace(NamedTuple):
    """Workspace handle for :func:`bag_matmul` (``bag.py:28-46`` analogue)."""

    workspace: Optional[Workspace]
    depth: int
    basis: str


def _check_square_matrix(name, tensor, size, device, *, output=False):
    torch = _torch()
    if not isinstance(tensor, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if tensor.ndim != 2 or tuple(tensor.shape) != (size, size):
        raise ValueError(f"{name} must have shape ({size}, {size}), got {tuple(tensor.shape)}")
    if tensor.device != device:
        raise ValueError(f"{name} must be on {device}, got {tensor.device}")
    if tensor.dtype != torch.float32:
        raise TypeError(f"{name} must have dtype torch.float32, got {tensor.dtype}")
    if any(stride < 0 for stride in tensor.stride()):
        raise ValueError(f"{name} must have non-negative strides, got {tensor.stride()}")
    if output and any(e > 1 and s == 0 for e, s in zip(tensor.shape, tensor.stride())):
        raise ValueError(f"{name} must not have broadcasted output dimensions")
    if tensor.requires_grad:
        raise ValueError(f"{name} must not require gradients")


def allocate_bag_workspace(a, b=None, out=None, *, depth: int = 1, basis: str = "minimal",
                           **_ignored) -> BagWorkspace:
    """Allocate the workspace :func:`bag_matmul` needs (``bag.py:865-953``)."""
    torch = _torch()
    if not isinstance(a, torch.Tensor) or a.ndim != 2 or a.shape[0] != a.shape[1]:
        raise ValueError("a must be a square two-dimensional torch.Tensor")
    size = a.shape[0]
    if size <= 0 or size % 2:
        raise ValueError(f"BAG requires a positive even matrix size, got {size}")
    ws = Workspace.for_problem(size, size, size, depth, basis)
    return BagWorkspace(ws if ws.bytes() else None, depth, basis)


def _as_unit_stride(t):
    return t if _layout_of(t) is not None else t.contiguous()


def bag_matmul(a, b, *, out=None, workspace: Optional[BagWorkspace] = None,
               allow_tf32: bool = False, schedule: str = "auto", depth: int = 1,
               basis: str = "minimal"):
    """``out = a @ b`` by BAG (``src/bag_triton/bag.py:955-1050`` interface).

    Validation, exception types and the returned object match the reference;
    ``schedule`` is accepted for compatibility (every schedule is one grouped
    launch here) and ``allow_tf32`` must stay False (FP32 FFMA only).
    """
    torch = _torch()
    if not isinstance(a, torch.Tensor) or a.ndim != 2:
        raise ValueError("a must be a two-dimensional torch.Tensor")
    if not a.is_cuda:
        raise ValueError(f"a must be a CUDA tensor, got device {a.device}")
    if a.shape[0] != a.shape[1]:
        raise ValueError(f"a must be square, got shape {tuple(a.shape)}")
    size = a.shape[0]
    if size <= 0 or size % 2:
        raise ValueError(f"BAG requires a positive even matrix size, got {size}")
    if not isinstance(allow_tf32, bool):
        raise TypeError(f"allow_tf32 must be bool, got {type(allow_tf32).__name__}")
    if allow_tf32:
        raise ValueError("allow_tf32=True is not offered: this build computes in IEEE FP32")
    if schedule not in ("auto", "serial", "multistream", "seven-stream", "hybrid", "grouped"):
        raise ValueError(
            "schedule must be 'auto', 'serial', 'multistream', "
            f"'seven-stream', 'hybrid', or 'grouped', got {schedule!r}")
    device = a.device
    _check_square_matrix("a", a, size, device)
    _check_square_matrix("b", b, size, device)
    if out is None:
        out = torch.empty_like(a, memory_format=torch.preserve_format)
    else:
        _check_square_matrix("out", out, size, device, output=True)
    if workspace is None:
        workspace = allocate_bag_workspace(a, b, out, depth=depth, basis=basis)
    elif not isinstance(workspace, BagWorkspace):
        raise TypeError("workspace must be a BagWorkspace from allocate_bag_workspace")
    ws = workspace.workspace
    aa, bb = _as_unit_stride(a), _as_unit_stride(b)
    la, lb, lo = _layout_of(aa), _layout_of(bb), _layout_of(out)
    if lo is not None and la[0] == lb[0] == lo[0]:
        sgemm(aa, bb, out, beta=0.0, depth=workspace.depth, basis=workspace.basis, workspace=ws)
        return out
    # Mixed or strided layouts: compute row-major, then copy into `out`.
    tmp = torch.empty((size, size), device=device, dtype=torch.float32)
    sgemm(aa.contiguous(), bb.contiguous(), tmp, beta=0.0, depth=workspace.depth,
          basis=workspace.basis, workspace=ws)
    out.copy_(tmp)
    return out


def bag_primitive(x, y, v, w, d, e, *, delta: int, epsilon: int, gamma_d: int, gamma_e: int,
                  allow_tf32: bool = False, _atomic_accumulate: bool = True):
    """The fused BAG primitive (``src/bag_triton/primitive.py:256-461`` interface).

    ``product = (x + delta*y) @ (v + epsilon*w)``; ``d += gamma_d*product`` for
    gamma +-1 (atomically unless ``_atomic_accumulate=False``), ``d =
    +-product`` for gamma +-2, untouched for 0; the same for ``e``.
    Returns ``(d, e)``.
    """
    torch = _torch()
    for name, val, allowed in (("delta", delta, (-1, 0, 1)), ("epsilon", epsilon, (-1, 0, 1)),
                               ("gamma_d", gamma_d, (-2, -1, 0, 1, 2)),
                               ("gamma_e", gamma_e, (-2, -1, 0, 1, 2))):
        if isinstance(val, bool) or not isinstance(val, int):
            raise TypeError(f"{name} must be an int, got {type(val).__name__}")
        if val not in allowed:
            raise ValueError(f"{name} must be one of {allowed}, got {val}")
    if allow_tf32:
        raise ValueError("allow_tf32=True is not offered: this build computes in IEEE FP32")
    if not isinstance(x, torch.Tensor) or x.ndim != 2:
        raise ValueError("x must be a two-dimensional torch.Tensor")
    if not x.is_cuda:
        raise ValueError(f"x must be a CUDA tensor, got device {x.device}")
    m, k = x.shape
    if not isinstance(v, torch.Tensor) or v.ndim != 2 or v.shape[0] != k:
        raise ValueError(f"v must have shape ({k}, N)")
    n = v.shape[1]
    if y is None and delta != 0:
        raise ValueError("y may be None only when delta == 0")
    if w is None and epsilon != 0:
        raise ValueError("w may be None only when epsilon == 0")
    if d is None and gamma_d != 0:
        raise ValueError("d may be None only when gamma_d == 0")
    if e is None and gamma_e != 0:
        raise ValueError("e may be None only when gamma_e == 0")
    for name, t, shape in (("x", x, (m, k)), ("y", y, (m, k)), ("v", v, (k, n)), ("w", w, (k, n)),
                           ("d", d, (m, n)), ("e", e, (m, n))):
        if t is None:
            continue
        if tuple(t.shape) != shape:
            raise ValueError(f"{name} must have shape {shape}, got {tuple(t.shape)}")
        if t.dtype != torch.float32:
            raise TypeError(f"{name} must have dtype torch.float32, got {t.dtype}")
        if t.device != x.device:
            raise ValueError(f"{name} must be on {x.device}")
    if (gamma_d == 0 and gamma_e == 0) or m == 0 or n == 0:
        return d, e

    def colmajor(t):
        # Column-major copy (or the tensor itself) for the column-major C ABI.
        if t is None:
            return None
        lay = _layout_of(t)
        if lay is not None and lay[0] == "col":
            return t
        return t.t().contiguous().t()

    outs = []
    for t, g in ((d, gamma_d), (e, gamma_e)):
        if t is None or g == 0:
            outs.append((t, None))
        else:
            lay = _layout_of(t)
            outs.append((t, t if lay is not None and lay[0] == "col" else colmajor(t)))
    xx, yy, vv, ww = colmajor(x), colmajor(y), colmajor(v), colmajor(w)
    ld = lambda t: 1 if t is None else max(_layout_of(t)[1], 1)  # noqa: E731
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    dd, ee = outs[0][1], outs[1][1]
    _check(lib().bag_primitive(delta, epsilon, gamma_d, gamma_e, int(bool(_atomic_accumulate)),
                               ptr(xx), ptr(yy), ptr(vv), ptr(ww), ptr(dd), ptr(ee), m, n, k,
                               ld(xx), ld(yy), ld(vv), ld(ww), ld(dd), ld(ee),
                               _stream_handle(None)))
    for orig, work in outs:
        if work is not None and work is not orig:
            orig.copy_(work)
    return d, e


__all__ = [
    "BagError", "BagWorkspace", "Workspace", "allocate_bag_workspace", "bag_matmul",
    "bag_primitive", "lib", "local_elements", "matmul", "plan_dump", "sgemm", "sgemm_batched",
    "MultiWorkspace", "multi_grid", "sgemm_multi",
    "strassen_one_level", "valid_shape",
]
