"""Python mirror of the reference optimizer API (crates/mmn-optim/src/lib.rs)
over the sm_100a C-ABI library.

Names, argument meaning and state semantics follow the Rust types:
``AdamW.step_param(id, param, grad)``, ``Muon.step_matrix(id, param, grad)``,
``newton_schulz5(g, steps)``, ``HybridOptimizer.classify_param(shape)`` /
``.step(id, param, grad)`` and ``GradAccumulator``. ``param`` is updated in
place. Arrays may be float32 numpy arrays (host memory: copied in and out per
call) or float32 CUDA torch tensors (device memory: work is enqueued on the
handle's stream, which defaults to torch's current stream).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np

from . import _native as N


def _torch():
    try:
        import torch  # noqa: F401

        return torch
    except ImportError:  # pragma: no cover - torch is in the image
        return None


def _mem_ptr(x, writable: bool, device: int | None = None):
    """(pointer, mem kind, shape) of a float32 numpy array or torch tensor; a
    CUDA tensor must live on `device` (the handle's GPU) when one is given."""
    torch = _torch()
    if torch is not None and isinstance(x, torch.Tensor):
        if x.dtype != torch.float32:
            raise TypeError("expected a float32 tensor")
        if not x.is_contiguous():
            raise ValueError("tensor must be contiguous")
        if x.is_cuda:
            if device is not None and x.device.index != device:
                raise ValueError(f"tensor on {x.device}, optimizer on cuda:{device}")
            return ctypes.c_void_p(x.data_ptr()), N.MEM_DEVICE, tuple(x.shape)
        x = x.numpy()
    if not isinstance(x, np.ndarray) or x.dtype != np.float32:
        raise TypeError("expected a float32 numpy array or torch tensor")
    if not x.flags.c_contiguous:
        raise ValueError("array must be C-contiguous")
    if writable and not x.flags.writeable:
        raise ValueError("param array is read-only")
    return ctypes.c_void_p(x.ctypes.data), N.MEM_HOST, tuple(x.shape)


_CUDA_STREAM_LEGACY = 1  # cudaStreamLegacy: the legacy default stream


def _stream_of(device: int, stream):
    """The cudaStream_t to hand to the library. torch reports its default
    stream as 0, which the C ABI would read as "no stream given" (the library
    would then use a stream of its own, unordered with torch's work), so the
    default stream is passed explicitly as cudaStreamLegacy."""
    if stream is None:
        torch = _torch()
        if torch is None or not torch.cuda.is_available():
            return ctypes.c_void_p(0)
        stream = torch.cuda.current_stream(device).cuda_stream
    stream = int(stream)
    return ctypes.c_void_p(stream if stream != 0 else _CUDA_STREAM_LEGACY)


def is_available() -> bool:
    """crates/mmn-cuda/src/lib.rs:5-12 is_available()."""
    return bool(N.lib().mmn_cuda_is_available())


def require_cuda(cuda_requested: bool) -> None:
    """crates/mmn-core/src/device.rs:29-37: raises CUDAError when cuda is requested
    and no usable B200 is present."""
    N.check(N.lib().mmn_require_cuda(int(bool(cuda_requested))))


@dataclass
class AdamWConfig:
    """lib.rs:6-22."""

    lr: float = 3e-4
    betas: tuple = (0.9, 0.95)
    eps: float = 1e-8
    weight_decay: float = 0.01

    def c(self) -> N.AdamWConfigC:
        return N.AdamWConfigC(self.lr, self.betas[0], self.betas[1], self.eps, self.weight_decay)


@dataclass
class MuonConfig:
    """lib.rs:63-80."""

    lr: float = 0.02
    momentum: float = 0.95
    nesterov: bool = True
    ns_steps: int = 5

    def c(self) -> N.MuonConfigC:
        return N.MuonConfigC(self.lr, self.momentum, int(self.nesterov), int(self.ns_steps))


NS_MODES = {"reference": N.NS_REFERENCE, "bf16": N.NS_BF16, "tf32": N.NS_TF32,
            "fp32": N.NS_FP32}


class AdamW:
    """AdamW (lib.rs:24-61) with device-resident state keyed by id."""

    def __init__(self, config: AdamWConfig | None = None, device: int = 0, stream=None,
                 _handle=None):
        self.config = config or AdamWConfig()
        self.device = device
        self._owned = _handle is None
        if _handle is None:
            h = ctypes.c_void_p()
            cfg = self.config.c()
            N.check(N.lib().mmn_adamw_create(ctypes.byref(cfg), device,
                                             _stream_of(device, stream), ctypes.byref(h)))
            _handle = h
        self._h = _handle

    def step_param(self, id: int, param, grad, grad_divisor: float = 1.0) -> None:
        pp, mem, shape = _mem_ptr(param, True, self.device)
        gp, gmem, gshape = _mem_ptr(grad, False, self.device)
        if gmem != mem or gshape != shape:
            raise N.ShapeError(N.MMN_E_SHAPE, "param and grad must match in shape and memory")
        N.check(N.lib().mmn_adamw_step_param(self._h, id, pp, gp, N.shape_array(shape),
                                             len(shape), grad_divisor, mem))

    @property
    def step(self) -> int:
        v = ctypes.c_uint64()
        N.check(N.lib().mmn_adamw_get_step(self._h, ctypes.byref(v)))
        return v.value

    @step.setter
    def step(self, value: int) -> None:
        N.check(N.lib().mmn_adamw_set_step(self._h, int(value)))

    def export_state(self, id: int, which: str, numel: int) -> np.ndarray:
        out = np.empty(numel, np.float32)
        N.check(N.lib().mmn_adamw_export_state(self._h, id, {"m": 0, "v": 1}[which],
                                               out.ctypes.data, numel, N.MEM_HOST))
        return out

    def import_state(self, id: int, which: str, values: np.ndarray) -> None:
        v = np.ascontiguousarray(values, np.float32).reshape(-1)
        N.check(N.lib().mmn_adamw_import_state(self._h, id, {"m": 0, "v": 1}[which],
                                               v.ctypes.data, v.size, N.MEM_HOST))

    def close(self) -> None:
        if self._owned and self._h:
            N.lib().mmn_adamw_destroy(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Muon:
    """Muon (lib.rs:128-176) with device-resident velocity keyed by id."""

    def __init__(self, config: MuonConfig | None = None, ns_mode: str = "reference",
                 device: int = 0, stream=None, _handle=None):
        self.config = config or MuonConfig()
        self.ns_mode = ns_mode
        self.device = device
        self._owned = _handle is None
        if _handle is None:
            h = ctypes.c_void_p()
            cfg = self.config.c()
            N.check(N.lib().mmn_muon_create(ctypes.byref(cfg), NS_MODES[ns_mode], device,
                                            _stream_of(device, stream), ctypes.byref(h)))
            _handle = h
        self._h = _handle

    def step_matrix(self, id: int, param, grad, grad_divisor: float = 1.0) -> None:
        pp, mem, shape = _mem_ptr(param, True, self.device)
        gp, gmem, gshape = _mem_ptr(grad, False, self.device)
        if gmem != mem or gshape != shape:
            raise N.ShapeError(N.MMN_E_SHAPE, "param and grad must match in shape and memory")
        N.check(N.lib().mmn_muon_step_matrix(self._h, id, pp, gp, N.shape_array(shape),
                                             len(shape), grad_divisor, mem))

    def import_velocity(self, id: int, values: np.ndarray) -> None:
        v = np.ascontiguousarray(values, np.float32)
        N.check(N.lib().mmn_muon_register(self._h, id, N.shape_array(v.shape), v.ndim))
        N.check(N.lib().mmn_muon_import_velocity(self._h, id, v.ctypes.data, v.size, N.MEM_HOST))

    def export_velocity(self, id: int, shape) -> np.ndarray:
        out = np.empty(shape, np.float32)
        N.check(N.lib().mmn_muon_export_velocity(self._h, id, out.ctypes.data, out.size,
                                                 N.MEM_HOST))
        return out

    def close(self) -> None:
        if self._owned and self._h:
            N.lib().mmn_muon_destroy(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def newton_schulz5(g, steps: int = 5, ns_mode: str = "reference", device: int = 0, stream=None):
    """newton_schulz5 (lib.rs:83-126). Returns a new float32 array (numpy in,
    numpy out; CUDA tensor in, CUDA tensor out) of the 2-D (or zero-padded
    square) shape."""
    gp, mem, shape = _mem_ptr(g, False)
    if len(shape) == 2:
        oshape = shape
    else:
        n = int(np.prod(shape)) if shape else 1
        side = int(np.ceil(np.sqrt(np.float32(n), dtype=np.float32)))
        oshape = (side, side)
    if mem == N.MEM_DEVICE:
        torch = _torch()
        out = torch.empty(oshape, dtype=torch.float32, device=g.device)
        optr = ctypes.c_void_p(out.data_ptr())
        dev = g.device.index or 0
    else:
        out = np.empty(oshape, np.float32)
        optr = ctypes.c_void_p(out.ctypes.data)
        dev = device
    N.check(N.lib().mmn_newton_schulz5(gp, N.shape_array(shape), len(shape), steps,
                                       NS_MODES[ns_mode], optr, dev, _stream_of(dev, stream),
                                       mem))
    return out


class ParamKind:
    MATRIX = "Matrix"
    OTHER = "Other"


class HybridOptimizer:
    """HybridOptimizer (lib.rs:183-210): Muon for 2-D matrices, AdamW otherwise."""

    def __init__(self, muon: MuonConfig | None = None, adamw: AdamWConfig | None = None,
                 ns_mode: str = "reference", device: int = 0, stream=None):
        h = ctypes.c_void_p()
        mc = (muon or MuonConfig())
        ac = (adamw or AdamWConfig())
        mcc, acc = mc.c(), ac.c()
        N.check(N.lib().mmn_hybrid_create(ctypes.byref(mcc), ctypes.byref(acc), NS_MODES[ns_mode],
                                          device, _stream_of(device, stream), ctypes.byref(h)))
        self._h = h
        self.device = device
        self.muon = Muon(mc, ns_mode, device,
                         _handle=ctypes.c_void_p(N.lib().mmn_hybrid_muon(h)))
        self.adamw = AdamW(ac, device, _handle=ctypes.c_void_p(N.lib().mmn_hybrid_adamw(h)))

    @staticmethod
    def classify_param(shape) -> str:
        r = N.lib().mmn_hybrid_classify_param(N.shape_array(shape), len(shape))
        return ParamKind.MATRIX if r == N.ROUTE_MUON else ParamKind.OTHER

    def step(self, id: int, param, grad, route: str | None = None,
             grad_divisor: float = 1.0) -> None:
        pp, mem, shape = _mem_ptr(param, True, self.device)
        gp, gmem, gshape = _mem_ptr(grad, False, self.device)
        if gmem != mem or gshape != shape:
            raise N.ShapeError(N.MMN_E_SHAPE, "param and grad must match in shape and memory")
        r = {None: N.ROUTE_AUTO, ParamKind.MATRIX: N.ROUTE_MUON, ParamKind.OTHER: N.ROUTE_ADAMW}[route]
        N.check(N.lib().mmn_hybrid_step(self._h, id, pp, gp, N.shape_array(shape), len(shape), r,
                                        grad_divisor, mem))

    def close(self) -> None:
        if self._h:
            self.muon._h = None
            self.adamw._h = None
            N.lib().mmn_hybrid_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclass
class GradAccumulator:
    """GradAccumulator (lib.rs:212-262). Holds per-position grad sums; the
    average sum/n is folded into the fused step via ``divisor``."""

    grads: list = field(default_factory=list)
    micro_batches: int = 0
    param_index: int = 0

    def clear(self) -> None:
        self.grads.clear()
        self.micro_batches = 0
        self.param_index = 0

    def begin_micro_batch(self) -> None:
        self.param_index = 0

    def finish_micro_batch(self) -> None:
        self.micro_batches += 1
        self.param_index = 0

    def add_param_grad(self, grad) -> None:
        if self.param_index < len(self.grads):
            self.grads[self.param_index] += grad
        else:
            self.grads.append(grad.copy() if isinstance(grad, np.ndarray) else grad.clone())
        self.param_index += 1

    @property
    def divisor(self) -> float:
        """max(micro_batches, 1) as the step's grad_divisor (lib.rs:255)."""
        return float(max(self.micro_batches, 1))

    def averaged_grad(self, index: int):
        return self.grads[index] / np.float32(self.divisor)

    def __len__(self) -> int:
        return len(self.grads)
