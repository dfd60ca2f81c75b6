"""The batched, device-resident optimizer step (mmn_optim_* in include/mmn_optim.h)
and the trainer-facing configuration (crates/mmn-train/src/lib.rs:22-41,
crates/mmn-py/src/train_config.rs:4-56).

One ``OptimizerStep`` owns every parameter, grad and optimizer-state buffer of
a model on one GPU and steps them all with one call, replacing the per-tensor
``optim_step_weight`` calls of crates/mmn-models/src/chatbot.rs:208-227.
Parameters must be registered in the reference's call order
(``chatbot_param_order`` gives it for the Chatbot model).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _native as N
from .optim import AdamWConfig, MuonConfig, NS_MODES, _stream_of


@dataclass
class TrainConfig:
    """TrainConfig (crates/mmn-train/src/lib.rs:22-41); Python defaults of
    crates/mmn-py/src/train_config.rs:21."""

    epochs: int = 1
    batch_size: int = 8
    cuda: bool = False
    optimizer: str = "hybrid"
    learning_rate: float = 3e-4

    def __repr__(self) -> str:  # crates/mmn-py/src/train_config.rs:37-44
        return (f"TrainConfig(epochs={self.epochs}, batch_size={self.batch_size}, "
                f"cuda={'true' if self.cuda else 'false'}, optimizer={self.optimizer!r}, "
                f"learning_rate={self.learning_rate})").replace("'", '"')


class _CudaArray:
    """Minimal __cuda_array_interface__ wrapper so torch can view library memory."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3,
                                         "strides": None}


def _view(ptr: int, shape, dtype: str, device: int):
    import torch

    t = torch.as_tensor(_CudaArray(ptr, shape, {"f32": "<f4", "bf16": "<i2"}[dtype]),
                        device=f"cuda:{device}")
    return t.view(torch.bfloat16) if dtype == "bf16" else t


ROUTES = {"auto": N.ROUTE_AUTO, "muon": N.ROUTE_MUON, "adamw": N.ROUTE_ADAMW}


@dataclass
class StepConfig:
    adamw: AdamWConfig = None
    muon: MuonConfig = None
    use_hybrid: bool = True
    ns_mode: str = "reference"
    fresh_state: bool = False
    grad_dtype: str = "f32"
    bf16_param_shadow: bool = False
    loss_scaling: bool = False
    loss_scale_init: float = 65536.0
    growth_interval: int = 2000
    rank: int = 0
    world_size: int = 1
    use_graph: bool = True
    reduce_grads: bool = False
    scan_shard: bool = False

    def c(self) -> N.OptimConfigC:
        c = N.lib().mmn_optim_config_default()
        c.adamw = (self.adamw or AdamWConfig()).c()
        c.muon = (self.muon or MuonConfig()).c()
        c.use_hybrid = int(self.use_hybrid)
        c.ns_mode = NS_MODES[self.ns_mode]
        c.fresh_state = int(self.fresh_state)
        c.grad_dtype = {"f32": N.DTYPE_F32, "bf16": N.DTYPE_BF16}[self.grad_dtype]
        c.bf16_param_shadow = int(self.bf16_param_shadow)
        c.loss_scaling = int(self.loss_scaling)
        c.loss_scale_init = self.loss_scale_init
        c.growth_interval = self.growth_interval
        c.rank = self.rank
        c.world_size = self.world_size
        c.use_graph = int(self.use_graph)
        c.reduce_grads = int(self.reduce_grads)
        c.scan_shard = int(self.scan_shard)
        return c


def step_config_for(train: TrainConfig, **overrides) -> StepConfig:
    """The optimizer the trainer builds (crates/mmn-train/src/lib.rs:367-380):
    Muon with MuonConfig::default() (TrainConfig.learning_rate never reaches
    Muon), AdamW with lr = learning_rate and default betas/eps/decay, hybrid
    routing only for optimizer == "hybrid", and fresh state every step because
    the trainer's param ids are never reused."""
    if train.cuda:
        from .optim import require_cuda

        require_cuda(True)
    cfg = StepConfig(adamw=AdamWConfig(lr=train.learning_rate), muon=MuonConfig(),
                     use_hybrid=train.optimizer == "hybrid", fresh_state=True)
    for k, v in overrides.items():
        setattr(cfg, k, v)
    return cfg


def _host_ptr(buf, numel: int, itemsize: int, what: str, slot: int, writable: bool = False):
    """Address of a contiguous host buffer of numel items of itemsize bytes
    (numpy array or CPU torch tensor), or None for a None entry."""
    if buf is None:
        return None
    if isinstance(buf, np.ndarray):
        ok = buf.flags.c_contiguous and (buf.flags.writeable or not writable)
        size, isz, ptr = buf.size, buf.itemsize, buf.ctypes.data
    else:  # torch tensor
        ok = (not buf.is_cuda) and buf.is_contiguous()
        size, isz, ptr = buf.numel(), buf.element_size(), buf.data_ptr()
    if not ok or size != numel or isz != itemsize:
        raise ValueError(f"{what} {slot}: need a contiguous host buffer of {numel} items of "
                         f"{itemsize} bytes")
    return ptr


class OptimizerStep:
    """Whole-model optimizer step on one GPU (or one rank's shard of it)."""

    def __init__(self, params, config: StepConfig | None = None, device: int = 0, stream=None):
        """params: iterable of (id, shape) or (id, shape, route) in call order;
        route is "auto" (reference shape rule), "muon" or "adamw"."""
        self.config = config or StepConfig()
        self.device = device
        h = ctypes.c_void_p()
        cfg = self.config.c()
        N.check(N.lib().mmn_optim_create(ctypes.byref(cfg), device, _stream_of(device, stream),
                                         ctypes.byref(h)))
        self._h = h
        self.shapes = []
        self.routes = []
        self._spec = []
        self._plan = None
        for p in params:
            pid, shape = p[0], tuple(int(s) for s in p[1])
            route = p[2] if len(p) > 2 else "auto"
            self._spec.append((pid, shape, route))
            slot = ctypes.c_int()
            N.check(N.lib().mmn_optim_add_param(h, pid, N.shape_array(shape), len(shape),
                                                ROUTES[route], ctypes.byref(slot)))
            self.shapes.append(shape)
        N.check(N.lib().mmn_optim_finalize(h))
        for i in range(len(self.shapes)):
            owner = ctypes.c_int()
            N.check(N.lib().mmn_optim_slot_owner(h, i, ctypes.byref(owner)))
            self.routes.append("muon" if owner.value >= 0 else "adamw")
        self._views = {}

    # -- buffers -----------------------------------------------------------------
    def _ptrs(self, slot: int):
        p, g, b = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        N.check(N.lib().mmn_optim_slot_ptrs(self._h, slot, ctypes.byref(p), ctypes.byref(g),
                                            ctypes.byref(b)))
        return p.value, g.value, b.value

    def param(self, slot: int):
        """torch view (fp32, device) of a slot's parameter inside the library arena."""
        return _view(self._ptrs(slot)[0], self.shapes[slot], "f32", self.device)

    def grad(self, slot: int):
        """torch view of a slot's grad buffer (fp32 or bf16 per grad_dtype)."""
        return _view(self._ptrs(slot)[1], self.shapes[slot],
                     "bf16" if self.config.grad_dtype == "bf16" else "f32", self.device)

    def param_bf16(self, slot: int):
        ptr = self._ptrs(slot)[2]
        return None if not ptr else _view(ptr, self.shapes[slot], "bf16", self.device)

    def _numel(self, slot: int) -> int:
        return int(np.prod(self.shapes[slot], dtype=np.int64))

    def set_param(self, slot: int, values: np.ndarray) -> None:
        v = np.ascontiguousarray(values, np.float32)
        N.check(N.lib().mmn_optim_set_param(
            self._h, slot, _host_ptr(v, self._numel(slot), 4, "param", slot), N.MEM_HOST))

    def get_param(self, slot: int) -> np.ndarray:
        out = np.empty(self.shapes[slot], np.float32)
        N.check(N.lib().mmn_optim_get_param(self._h, slot, out.ctypes.data, N.MEM_HOST))
        return out

    def set_grad(self, slot: int, values: np.ndarray) -> None:
        """fp32 grads, or with grad_dtype "bf16" their 16-bit patterns (uint16)."""
        v = np.ascontiguousarray(values)
        gsz = 2 if self.config.grad_dtype == "bf16" else 4
        N.check(N.lib().mmn_optim_set_grad(
            self._h, slot, _host_ptr(v, self._numel(slot), gsz, "grad", slot), N.MEM_HOST))

    def set_state(self, slot: int, which: str, values) -> None:
        """Seed a slot's m, v or velocity from a host array, or from a contiguous
        fp32 CUDA tensor on the handle's GPU (copied device to device; the call
        returns once the copy is done)."""
        kind = {"m": 0, "v": 1, "velocity": 2}[which]
        if getattr(values, "is_cuda", False):
            import torch

            if (values.dtype != torch.float32 or not values.is_contiguous()
                    or values.numel() != self._numel(slot)
                    or values.device.index != self.device):
                raise ValueError(f"{which} {slot}: need a contiguous fp32 tensor of "
                                 f"{self._numel(slot)} elements on cuda:{self.device}")
            torch.cuda.current_stream(self.device).synchronize()  # values are written
            N.check(N.lib().mmn_optim_set_state(self._h, slot, kind, values.data_ptr(),
                                                N.MEM_DEVICE))
            self.sync()
            return
        v = np.ascontiguousarray(values, np.float32)
        N.check(N.lib().mmn_optim_set_state(self._h, slot, kind,
                                            _host_ptr(v, self._numel(slot), 4, which, slot),
                                            N.MEM_HOST))

    def get_state(self, slot: int, which: str) -> np.ndarray:
        out = np.empty(self.shapes[slot], np.float32)
        N.check(N.lib().mmn_optim_get_state(self._h, slot, {"m": 0, "v": 1, "velocity": 2}[which],
                                            out.ctypes.data, N.MEM_HOST))
        return out

    @property
    def adamw_step(self) -> int:
        v = ctypes.c_uint64()
        N.check(N.lib().mmn_optim_get_adamw_step(self._h, ctypes.byref(v)))
        return v.value

    @adamw_step.setter
    def adamw_step(self, value: int) -> None:
        N.check(N.lib().mmn_optim_set_adamw_step(self._h, int(value)))

    # -- stepping ------------------------------------------------------------------
    def step(self, grad_divisor: float = 1.0) -> None:
        N.check(N.lib().mmn_optim_step(self._h, grad_divisor))

    def step_host(self, grads, params, grad_divisor: float = 1.0) -> None:
        """One step from host memory (mmn_optim_step_host): grads[slot] are copied
        in, params[slot] receive the updated fp32 values. Entries are numpy arrays
        or CPU torch tensors (pinned ones let the copies overlap the compute), or
        None to skip that slot's copy. Returns when params hold the result."""
        n = len(self.shapes)
        if len(grads) != n or len(params) != n:
            raise ValueError(f"need {n} grads and {n} params (one per slot)")
        gsz = 2 if self.config.grad_dtype == "bf16" else 4
        gp = (ctypes.c_void_p * n)()
        pp = (ctypes.c_void_p * n)()
        for k in range(n):
            numel = int(np.prod(self.shapes[k], dtype=np.int64))
            gp[k] = _host_ptr(grads[k], numel, gsz, "grad", k)
            pp[k] = _host_ptr(params[k], numel, 4, "param", k, writable=True)
        N.check(N.lib().mmn_optim_step_host(self._h, gp, pp, grad_divisor))

    def sync(self) -> None:
        N.check(N.lib().mmn_optim_sync(self._h))

    def stepped_range(self, slot: int):
        """Element range [lo, hi) of a slot that this rank steps (and whose
        optimizer state it holds): a whole Muon matrix it owns, or the overlap
        of an AdamW tensor with its AdamW range; (0, 0) for none."""
        cfg = self.config
        if self._plan is None:
            steps = (cfg.muon or MuonConfig()).ns_steps
            self._plan = shard_plan(self._spec, cfg.world_size, cfg.use_hybrid, steps)
        n = int(np.prod(self.shapes[slot], dtype=np.int64))
        owner = self._plan["owner"][slot]
        if owner >= 0:
            return (0, n) if owner == cfg.rank else (0, 0)
        off, reg = self._plan["offset"][slot], self._plan["adamw_region"]
        lo = max(off, cfg.rank * reg) - off
        hi = min(off + n, (cfg.rank + 1) * reg) - off
        return (lo, hi) if hi > lo else (0, 0)

    def loss_state(self):
        """(scale, skipped steps, clean steps since the scale last changed)."""
        s, k, g = ctypes.c_float(), ctypes.c_int64(), ctypes.c_int32()
        N.check(N.lib().mmn_optim_get_loss_state(self._h, ctypes.byref(s), ctypes.byref(k),
                                                 ctypes.byref(g)))
        return s.value, k.value, g.value

    def set_loss_state(self, scale: float, skipped_steps: int, good_steps: int) -> None:
        N.check(N.lib().mmn_optim_set_loss_state(self._h, scale, skipped_steps, good_steps))

    def loss_scale(self):
        s, k = ctypes.c_float(), ctypes.c_int64()
        N.check(N.lib().mmn_optim_loss_scale(self._h, ctypes.byref(s), ctypes.byref(k)))
        return s.value, k.value

    def enable_timing(self, on: bool = True) -> None:
        N.check(N.lib().mmn_optim_enable_timing(self._h, int(on)))

    def last_timing(self) -> dict:
        """Mean per-step device time (ms) of each phase over the timed steps:
        AdamW kernel, Muon momentum pass, Newton-Schulz input norms, Newton-
        Schulz GEMMs, Muon update, whole step."""
        ms = (ctypes.c_float * 6)()
        N.check(N.lib().mmn_optim_last_timing_ex(self._h, ms))
        return dict(zip(("adamw", "muon_momentum", "muon_norm", "newton_schulz", "muon_update",
                         "step"), list(ms)))

    def gather_layout(self) -> dict:
        g = N.GatherLayoutC()
        N.check(N.lib().mmn_optim_get_gather_layout(self._h, ctypes.byref(g)))
        return {k: getattr(g, k) for k, _ in N.GatherLayoutC._fields_}

    IPC_BLOB_BYTES = 512

    def connect_peers(self, group=None) -> None:
        """Fused exchange (world_size > 1): every rank publishes IPC handles of
        its parameter arenas (one all-gather of 512-byte blobs over the given
        torch.distributed group) and maps its peers', after which each step
        also stores this rank's final values into every peer. Order the ranks
        after each step (e.g. ``exchange_fence``) before reading parameters."""
        import torch
        import torch.distributed as dist

        blob = (ctypes.c_uint8 * self.IPC_BLOB_BYTES)()
        N.check(N.lib().mmn_optim_export_ipc(self._h, blob))
        dev = torch.device(f"cuda:{self.device}")
        mine = torch.tensor(bytearray(blob), dtype=torch.uint8, device=dev)
        world = dist.get_world_size(group)
        everyone = torch.empty(world * self.IPC_BLOB_BYTES, dtype=torch.uint8, device=dev)
        dist.all_gather_into_tensor(everyone, mine, group=group)
        N.check(N.lib().mmn_optim_connect_peers(self._h, everyone.cpu().numpy().tobytes()))
        self._fence = torch.zeros(1, dtype=torch.int32, device=dev)

    def exchange_fence(self, group=None) -> None:
        """Orders the ranks after a fused-exchange step: a one-element
        all-reduce queued on the current stream after the step."""
        import torch.distributed as dist

        dist.all_reduce(self._fence, group=group)

    def reduce_grads(self, group=None) -> None:
        """Data-parallel grad reduction (mmn_optim_reduce_grads; needs
        StepConfig(reduce_grads=True) and connect_peers): this rank's regions
        become the rank-ordered sum of every rank's local grads, read over NVLink.
        Fenced on both sides with one-element all-reduces, as the call requires."""
        import torch.distributed as dist

        dist.all_reduce(self._fence, group=group)
        N.check(N.lib().mmn_optim_reduce_grads(self._h))
        dist.all_reduce(self._fence, group=group)

    def scan_grads(self, grads=None, group=None) -> None:
        """Sharded non-finite scan (mmn_optim_scan_grads; needs
        StepConfig(scan_shard=True, loss_scaling=True) and connect_peers): this
        rank scans only what it steps and sets every rank's skip flag. `grads`:
        None when the grads are on the device, else host buffers per slot (None
        entries skipped) whose parts this rank steps are copied in first; then
        call step_host with None grads. Fenced on both sides with one-element
        all-reduces, as the call requires."""
        import torch.distributed as dist

        gp = None
        if grads is not None:
            n = len(self.shapes)
            if len(grads) != n:
                raise ValueError(f"need {n} grads (one per slot)")
            gsz = 2 if self.config.grad_dtype == "bf16" else 4
            gp = (ctypes.c_void_p * n)()
            for k in range(n):
                gp[k] = _host_ptr(grads[k], int(np.prod(self.shapes[k], dtype=np.int64)), gsz,
                                  "grad", k)
        dist.all_reduce(self._fence, group=group)
        N.check(N.lib().mmn_optim_scan_grads(self._h, gp))
        dist.all_reduce(self._fence, group=group)

    def param_counts(self):
        t, a, m = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        N.check(N.lib().mmn_optim_param_counts(self._h, ctypes.byref(t), ctypes.byref(a),
                                               ctypes.byref(m)))
        return t.value, a.value, m.value

    def kernel_launches(self):
        """(launches per step, launches per reduce_grads) on this rank."""
        a, b = ctypes.c_int64(), ctypes.c_int64()
        N.check(N.lib().mmn_optim_kernel_launches(self._h, ctypes.byref(a), ctypes.byref(b)))
        return a.value, b.value

    def ns_flops(self) -> float:
        f = ctypes.c_double()
        N.check(N.lib().mmn_optim_ns_flops(self._h, ctypes.byref(f)))
        return f.value

    def close(self) -> None:
        if self._h:
            N.lib().mmn_optim_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def shard_plan(params, world_size: int, use_hybrid: bool = True, ns_steps: int = 5) -> dict:
    """The arena layout and rank ownership OptimizerStep uses (host only, no GPU).
    params: (id, shape[, route]) as for OptimizerStep. Returns per-tensor
    `owner` (Muon owner rank, -1 for AdamW) and `offset` (element offset in its
    arena), and the per-rank region sizes of the AdamW and Muon arenas."""
    shapes, ndims, routes = [], [], []
    for p in params:
        s = tuple(int(d) for d in p[1])
        shapes.extend(s)
        ndims.append(len(s))
        routes.append(ROUTES[p[2] if len(p) > 2 else "auto"])
    n = len(ndims)
    sh = (ctypes.c_int64 * max(len(shapes), 1))(*shapes)
    nd = (ctypes.c_int * max(n, 1))(*ndims)
    rt = (ctypes.c_int * max(n, 1))(*routes)
    owner = (ctypes.c_int * max(n, 1))()
    off = (ctypes.c_int64 * max(n, 1))()
    ar, mr = ctypes.c_int64(), ctypes.c_int64()
    N.check(N.lib().mmn_optim_plan(sh, nd, rt, n, int(use_hybrid), ns_steps, world_size, owner, off,
                                   ctypes.byref(ar), ctypes.byref(mr)))
    return {"owner": list(owner)[:n], "offset": list(off)[:n], "adamw_region": ar.value,
            "muon_region": mr.value}


def chatbot_param_order(vocab_size: int, n_layer: int, d_model: int, ffn_mult: int = 4,
                        pos_embed_len: int | None = None):
    """(name, shape) of every trained tensor of the reference Chatbot in the order
    its LM step calls the optimizer (crates/mmn-models/src/chatbot.rs:1104-1196,
    block order :118-206): lm_head; blocks L-1..0 as ffn2, ffn, out, q, k, v,
    ln2.gamma, ln2.beta, ln1.gamma, ln1.beta; embed; [pos_embed]. Linear weights
    are [out, in] (crates/mmn-nn/src/lib.rs:305-307)."""
    d, f = d_model, ffn_mult * d_model
    out = [("lm_head", (vocab_size, d))]
    for layer in reversed(range(n_layer)):
        b = f"blocks.{layer}."
        out += [(b + "ffn2", (d, f)), (b + "ffn", (f, d)), (b + "out", (d, d)), (b + "q", (d, d)),
                (b + "k", (d, d)), (b + "v", (d, d)), (b + "ln2.gamma", (d,)),
                (b + "ln2.beta", (d,)), (b + "ln1.gamma", (d,)), (b + "ln1.beta", (d,))]
    out.append(("embed", (vocab_size, d)))
    if pos_embed_len:
        out.append(("pos_embed", (pos_embed_len, d)))
    return out


def classifier_param_order(num_labels: int, input_dim: int):
    """(name, shape) of the Classifier's trained weights in the order its step
    calls AdamW (crates/mmn-models/src/chatbot.rs:1483-1548: head, then backbone;
    backbone input_dim -> 128, head 128 -> labels, :1399-1400). The classifier is
    stepped with AdamW only (use_hybrid = False)."""
    return [("head", (max(num_labels, 1), 128)), ("backbone", (128, input_dim))]


def diffusion_param_order():
    """(name, shape) of the diffusion UNet's conv weights in the order
    train_step_denoise calls AdamW (crates/mmn-models/src/chatbot.rs:2311-2320:
    down, mid, up; [out_ch, in_ch, k, k] as crates/mmn-nn/src/lib.rs:1989-1991
    builds them with UNet2D::new, :2167-2171). AdamW only."""
    return [("unet.down", (64, 4, 3, 3)), ("unet.mid", (64, 64, 3, 3)),
            ("unet.up", (4, 64, 3, 3))]
