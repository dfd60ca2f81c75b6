"""Optimizer-state checkpoints for ``OptimizerStep``.

The reference saves model weights only (``mmn-safetensors-v1``,
crates/mmn-io/src/chatbot_io.rs:25-110) and drops the optimizer state, so a
resumed run restarts AdamW's m, v and step count and Muon's velocity. This file
format sits beside the weights: a standard binary safetensors file (the layout
the reference's own HF import reads, crates/mmn-io/src/hf_safetensors.rs:128)
whose ``__metadata__`` says ``"format": "mmn-optim-state-v1"``.

Tensors, all F32, keyed by the model's tensor names:
  ``<name>.m``, ``<name>.v``   AdamW moments (absent with ``fresh_state``);
  ``<name>.velocity``          Muon velocity (absent with ``fresh_state``).
A sharded handle (``world_size > 1``) writes one file per rank with what that
rank steps: its whole Muon matrices and its slice of every AdamW tensor it
touches; ``ranges`` in the metadata gives each slice's element range.
Metadata also holds the AdamW call counter, the loss-scaling state, the
configuration and the tensor list, which loading checks against the handle.
"""
from __future__ import annotations

import json
import struct

import numpy as np

FORMAT = "mmn-optim-state-v1"
_DTYPES = {"F32": np.float32, "BF16": np.uint16, "I64": np.int64}
_NAMES = {np.dtype(np.float32): "F32", np.dtype(np.uint16): "BF16", np.dtype(np.int64): "I64"}


def write_safetensors(path: str, tensors: dict, metadata: dict | None = None) -> None:
    """Standard safetensors layout: u64 header length (little endian), a JSON
    header {name: {dtype, shape, data_offsets}, "__metadata__": {str: str}}
    padded with spaces to 8 bytes, then the raw little-endian data."""
    header = {}
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    off = 0
    arrays = []
    for name in sorted(tensors):
        a = np.ascontiguousarray(tensors[name])
        if a.dtype not in _NAMES:
            raise TypeError(f"{name}: unsupported dtype {a.dtype}")
        header[name] = {"dtype": _NAMES[a.dtype], "shape": list(a.shape),
                        "data_offsets": [off, off + a.nbytes]}
        off += a.nbytes
        arrays.append(a)
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for a in arrays:
            f.write(a.astype(a.dtype.newbyteorder("<"), copy=False).tobytes())


def read_safetensors(path: str):
    """Returns ({name: array}, metadata dict)."""
    with open(path, "rb") as f:
        data = f.read()
    if len(data) < 8:
        raise ValueError(f"{path}: not a safetensors file")
    (n,) = struct.unpack("<Q", data[:8])
    if n > len(data) - 8:
        raise ValueError(f"{path}: header length {n} exceeds the file")
    header = json.loads(data[8:8 + n])
    meta = header.pop("__metadata__", {})
    base = 8 + n
    out = {}
    for name, e in header.items():
        dt = _DTYPES.get(e["dtype"])
        if dt is None:
            raise ValueError(f"{name}: unsupported dtype {e['dtype']}")
        b, end = e["data_offsets"]
        isz = np.dtype(dt).itemsize
        numel = int(np.prod(e["shape"], dtype=np.int64))
        if not (0 <= b <= end <= len(data) - base) or end - b != numel * isz:
            raise ValueError(f"{path}: {name}: data_offsets {[b, end]} do not hold shape "
                             f"{e['shape']} of {e['dtype']} inside the file")
        a = np.frombuffer(data, dtype=np.dtype(dt).newbyteorder("<"), count=numel,
                          offset=base + b)
        out[name] = a.astype(dt).reshape(e["shape"])
    return out, meta


def _config_meta(cfg) -> dict:
    a, m = cfg.adamw, cfg.muon
    return {"use_hybrid": bool(cfg.use_hybrid), "ns_mode": cfg.ns_mode,
            "fresh_state": bool(cfg.fresh_state), "grad_dtype": cfg.grad_dtype,
            "loss_scaling": bool(cfg.loss_scaling),
            "adamw": None if a is None else {"lr": a.lr, "betas": list(a.betas), "eps": a.eps,
                                            "weight_decay": a.weight_decay},
            "muon": None if m is None else {"lr": m.lr, "momentum": m.momentum,
                                           "nesterov": bool(m.nesterov), "ns_steps": m.ns_steps}}


def save_state(step, path: str, names=None) -> None:
    """Writes the optimizer state of ``step`` (an OptimizerStep, after its last
    step completed) to ``path``. ``names`` are the tensor names in slot order
    (default ``slot<k>``)."""
    names = list(names) if names is not None else [f"slot{k}" for k in range(len(step.shapes))]
    if len(names) != len(step.shapes):
        raise ValueError("one name per slot")
    cfg = step.config
    step.sync()
    tensors, ranges = {}, {}
    if not cfg.fresh_state:
        for k, name in enumerate(names):
            lo, hi = step.stepped_range(k)
            if hi <= lo:
                continue
            n = int(np.prod(step.shapes[k], dtype=np.int64))
            whole = lo == 0 and hi == n
            if step.routes[k] == "adamw":
                for which in ("m", "v"):
                    full = step.get_state(k, which).reshape(-1)
                    tensors[f"{name}.{which}"] = full.reshape(step.shapes[k]) if whole else \
                        np.ascontiguousarray(full[lo:hi])
                    if not whole:
                        ranges[f"{name}.{which}"] = [lo, hi, n]
            else:
                tensors[f"{name}.velocity"] = step.get_state(k, "velocity")
    scale, skipped, good = step.loss_state()
    meta = {"format": FORMAT, "world_size": cfg.world_size, "rank": cfg.rank,
            "adamw_step": step.adamw_step, "loss_scale": repr(float(scale)),
            "skipped_steps": skipped, "good_steps": good,
            "ranges": json.dumps(ranges),
            "tensors": json.dumps([[nm, list(s)] for nm, s in zip(names, step.shapes)]),
            "config": json.dumps(_config_meta(cfg))}
    write_safetensors(path, tensors, meta)


def load_state(step, path: str, names=None) -> None:
    """Restores a state written by ``save_state`` into a handle with the same
    tensors, configuration, world size and rank."""
    names = list(names) if names is not None else [f"slot{k}" for k in range(len(step.shapes))]
    tensors, meta = read_safetensors(path)
    if meta.get("format") != FORMAT:
        raise ValueError(f"{path}: expected a {FORMAT} file, got {meta.get('format')!r}")
    cfg = step.config
    if int(meta["world_size"]) != cfg.world_size or int(meta["rank"]) != cfg.rank:
        raise ValueError(f"{path}: saved by rank {meta['rank']} of {meta['world_size']}, "
                         f"this handle is rank {cfg.rank} of {cfg.world_size}")
    want = [[nm, list(s)] for nm, s in zip(names, step.shapes)]
    if json.loads(meta["tensors"]) != want:
        raise ValueError(f"{path}: tensor names or shapes differ from this handle's")
    if json.loads(meta["config"]) != _config_meta(cfg):
        raise ValueError(f"{path}: optimizer configuration differs from this handle's")
    ranges = json.loads(meta["ranges"])
    for key, arr in tensors.items():
        name, which = key.rsplit(".", 1)
        k = names.index(name)
        if key in ranges:
            lo, hi, n = ranges[key]
            full = step.get_state(k, which).reshape(-1)
            full[lo:hi] = arr
            step.set_state(k, which, full.reshape(step.shapes[k]))
        else:
            step.set_state(k, which, arr.reshape(step.shapes[k]))
    step.adamw_step = int(meta["adamw_step"])
    step.set_loss_state(float(meta["loss_scale"]), int(meta["skipped_steps"]),
                        int(meta["good_steps"]))
