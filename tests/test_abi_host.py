"""CPU-only checks of the boundary and the host logic: the C-ABI library loads
and exports every function include/mmn_optim.h declares; configuration, call
order and CUDA gating behave like the reference's."""
import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    text = open(os.path.join(ROOT, "include", "mmn_optim.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mmn_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from magicmindnet_b200 import _native as N

    L = N.lib()
    names = declared_functions()
    assert len(names) >= 45
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    # the ctypes table covers exactly the declared functions, each with the
    # header's parameter count
    assert sorted(N.SIGNATURES) == names
    header = _header_functions()
    for name, (_, argtypes) in N.SIGNATURES.items():
        assert len(argtypes) == header[name], (name, len(argtypes), header[name])


def test_abi_version_and_defaults():
    from magicmindnet_b200 import _native as N

    L = N.lib()
    assert L.mmn_abi_version() == 3
    a = L.mmn_adamw_config_default()
    assert (round(a.lr, 7), round(a.beta1, 6), round(a.beta2, 6), a.eps, round(a.weight_decay, 6)) \
        == (3e-4, 0.9, 0.95, np.float32(1e-8), 0.01)
    m = L.mmn_muon_config_default()
    assert (round(m.lr, 6), round(m.momentum, 6), m.nesterov, m.ns_steps) == (0.02, 0.95, 1, 5)


def test_classify_param_matches_reference_table():
    import magicmindnet_b200 as mmn

    H = mmn.HybridOptimizer.classify_param
    assert H((64, 32)) == "Matrix"
    assert H((16,)) == "Other"
    assert H((16, 1)) == "Other"
    assert H((1, 3, 3, 3)) == "Other"
    assert H((2, 2)) == "Matrix"


def test_cuda_gate_without_gpu():
    """crates/mmn-core/src/device.rs:29-37 + tests/test_cuda_parity.py of the
    reference: cuda=True without a usable device raises CUDAError; cuda=False
    never does."""
    import magicmindnet_b200 as mmn

    mmn.require_cuda(False)
    if mmn.is_available():
        mmn.require_cuda(True)
        return
    with pytest.raises(mmn.CUDAError):
        mmn.require_cuda(True)
    with pytest.raises(mmn.CUDAError):
        mmn.step_config_for(mmn.TrainConfig(cuda=True))
    with pytest.raises(mmn.CUDAError):
        mmn.AdamW()


def test_train_config_defaults_and_repr():
    """crates/mmn-py/src/train_config.rs:21,37-44."""
    import magicmindnet_b200 as mmn

    c = mmn.TrainConfig()
    assert (c.epochs, c.batch_size, c.cuda, c.optimizer, c.learning_rate) == (1, 8, False, "hybrid",
                                                                            3e-4)
    assert repr(c) == ('TrainConfig(epochs=1, batch_size=8, cuda=false, optimizer="hybrid", '
                       'learning_rate=0.0003)')


def test_step_config_follows_trainer_construction():
    """crates/mmn-train/src/lib.rs:367-380: AdamW gets learning_rate, Muon keeps
    its defaults, only "hybrid" routes to Muon, ids never repeat."""
    import magicmindnet_b200 as mmn

    s = mmn.step_config_for(mmn.TrainConfig(learning_rate=1e-3, optimizer="hybrid"))
    assert s.use_hybrid and s.fresh_state and s.adamw.lr == 1e-3 and s.muon.lr == 0.02
    for opt in ("adamw", "muon"):
        assert not mmn.step_config_for(mmn.TrainConfig(optimizer=opt)).use_hybrid


def test_chatbot_param_order_vocab512_layers2_d64():
    """22 tensors / 164,352 params; 14 Muon matrices (163,840) under the
    reference rule, in the call order of crates/mmn-models/src/chatbot.rs."""
    import magicmindnet_b200 as mmn

    order = mmn.chatbot_param_order(512, 2, 64)
    assert len(order) == 22
    assert sum(int(np.prod(s)) for _, s in order) == 164352
    muon = [s for _, s in order if mmn.HybridOptimizer.classify_param(s) == "Matrix"]
    assert len(muon) == 14 and sum(int(np.prod(s)) for s in muon) == 163840
    names = [n for n, _ in order]
    assert names[0] == "lm_head" and names[-1] == "embed"
    assert names[1:11] == ["blocks.1." + x for x in ("ffn2", "ffn", "out", "q", "k", "v",
                                                      "ln2.gamma", "ln2.beta", "ln1.gamma",
                                                      "ln1.beta")]


def test_grad_accumulator_mirror():
    import magicmindnet_b200 as mmn

    acc = mmn.GradAccumulator()
    for val in (1.0, 3.0):
        acc.begin_micro_batch()
        acc.add_param_grad(np.array([[val]], np.float32))
        acc.finish_micro_batch()
    assert acc.divisor == 2.0
    assert abs(acc.averaged_grad(0)[0, 0] - 2.0) < 1e-6
    acc.clear()
    assert len(acc) == 0 and acc.divisor == 1.0


def test_bench_workload_sizes():
    import bench

    n1b = bench.count_params(bench.WORKLOADS["hybrid_1b"]["model"]())
    n8b = bench.count_params(bench.WORKLOADS["hybrid_8b"]["model"]())
    assert n1b == 1339228160 and n8b == 5362941952
    muon_1b = sum(s[0] * s[1] for _, s, r in bench.WORKLOADS["hybrid_1b"]["model"]() if r == "muon")
    assert muon_1b == 1207959552


def test_errors_report_through_last_error():
    from magicmindnet_b200 import _native as N

    h = ctypes.c_void_p()
    rc = N.lib().mmn_optim_create(None, -5, None, ctypes.byref(h))
    assert rc in (N.MMN_E_INVALID, N.MMN_E_NO_DEVICE)
    assert N.lib().mmn_last_error()


def test_ns_mode_constants_agree():
    """The Newton-Schulz modes have one numbering: the header's MMN_NS_*, the
    Python mode names and the oracle's REF_NS_* variants."""
    import magicmindnet_b200 as mmn  # noqa: F401
    from magicmindnet_b200.optim import NS_MODES
    from oracle import reference_optim as R

    text = open(os.path.join(ROOT, "include", "mmn_optim.h")).read()
    header = {k.lower(): int(v) for k, v in re.findall(r"#define MMN_NS_(\w+) (\d+)", text)}
    assert header == {"reference": 0, "bf16": 1, "tf32": 2, "fp32": 3}
    assert NS_MODES == header
    assert (R.NS_REFERENCE, R.NS_BF16, R.NS_TF32, R.NS_FP32) == (0, 1, 2, 3)
    ref_h = open(os.path.join(ROOT, "oracle", "mmn_optim_ref.h")).read()
    assert dict(re.findall(r"REF_NS_(\w+) = (\d)", ref_h)) == {
        "REFERENCE": "0", "BF16": "1", "TF32": "2", "FP32": "3"}


def test_optim_config_validation_before_device():
    """Configuration errors are reported before any device is touched: a
    sharded scan needs loss scaling, several ranks and no grad reduction, and
    an unknown Newton-Schulz mode is rejected."""
    from magicmindnet_b200 import _native as N

    L = N.lib()
    h = ctypes.c_void_p()
    c = L.mmn_optim_config_default()
    assert c.scan_shard == 0 and c.ns_mode == N.NS_REFERENCE
    c.scan_shard = 1  # without loss scaling and with one rank
    assert L.mmn_optim_create(ctypes.byref(c), 0, None, ctypes.byref(h)) == N.MMN_E_INVALID
    assert b"scan_shard" in L.mmn_last_error()
    c = L.mmn_optim_config_default()
    c.ns_mode = 4
    assert L.mmn_optim_create(ctypes.byref(c), 0, None, ctypes.byref(h)) == N.MMN_E_INVALID
    # the allocation-free entry point rejects the fp32-storage modes before any
    # pointer is used (the dummy buffers are never read)
    buf = np.zeros(4, np.float32)
    for mode in (N.NS_TF32, N.NS_FP32):
        rc = L.mmn_newton_schulz5_noalloc(buf.ctypes.data, 2, 2, 5, mode, buf.ctypes.data, 0, None)
        assert rc == N.MMN_E_UNSUPPORTED


def test_host_buffers_checked_before_the_library_reads_them():
    """Host setters hand the library a pointer only for a contiguous buffer of
    exactly the slot's element count and element size, so a short or wrongly
    typed array cannot be read past its end."""
    import torch

    from magicmindnet_b200.step import _host_ptr

    a = np.zeros(12, np.float32)
    assert _host_ptr(a, 12, 4, "param", 0) == a.ctypes.data
    assert _host_ptr(None, 12, 4, "grad", 0) is None
    for bad, n, isz in ((a[:11], 12, 4), (a, 12, 2), (a[::2], 6, 4),
                        (np.zeros(12, np.uint16), 12, 4)):
        with pytest.raises(ValueError):
            _host_ptr(bad, n, isz, "grad", 3)
    ro = np.zeros(12, np.float32)
    ro.flags.writeable = False
    assert _host_ptr(ro, 12, 4, "grad", 0) == ro.ctypes.data
    with pytest.raises(ValueError):
        _host_ptr(ro, 12, 4, "param", 0, writable=True)
    t = torch.zeros(12, dtype=torch.bfloat16)
    assert _host_ptr(t, 12, 2, "grad", 0) == t.data_ptr()
    with pytest.raises(ValueError):
        _host_ptr(torch.zeros(4, 3).t(), 12, 4, "grad", 0)


def test_plan_rejects_oversized_shapes_without_a_device():
    """The host-only plan refuses element counts of 2^62 or more (byte counts
    would overflow) and Muon dimensions above 2^30, with MMN_E_SHAPE."""
    from magicmindnet_b200 import _native as N

    L = N.lib()

    def plan(shape, route):
        shapes = (ctypes.c_int64 * len(shape))(*shape)
        ndims = (ctypes.c_int * 1)(len(shape))
        routes = (ctypes.c_int * 1)(route)
        return L.mmn_optim_plan(shapes, ndims, routes, 1, 1, 5, 1, None, None, None, None)

    assert plan((4, 8), N.ROUTE_MUON) == N.MMN_OK
    assert plan((1 << 40, 1 << 40), N.ROUTE_ADAMW) == N.MMN_E_SHAPE
    assert b"too large" in L.mmn_last_error()
    assert plan(((1 << 31), 2), N.ROUTE_MUON) == N.MMN_E_SHAPE
    assert plan((-1, 2), N.ROUTE_ADAMW) == N.MMN_E_INVALID


def _header_functions():
    """{name: parameter count} of every function the C header declares."""
    text = open(os.path.join(ROOT, "include", "mmn_optim.h")).read()
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    out = {}
    for m in re.finditer(r"\b(mmn_\w+)\s*\(([^()]*)\)\s*;", text):
        args = m.group(2).strip()
        out[m.group(1)] = 0 if args in ("", "void") else args.count(",") + 1
    return out


def test_caller_buffer_reduction_checks_arguments_before_the_device():
    """mmn_grad_reduce / mmn_grad_nonfinite_scan refuse bad arguments before
    touching a device, and without a GPU a well-formed call reports the CUDA
    gate's error (CUDAError), never a CPU result."""
    from magicmindnet_b200 import _native as N

    L = N.lib()
    vp = ctypes.c_void_p
    two = (vp * 2)(vp(0x10000), vp(0x20000))
    assert L.mmn_grad_reduce(two, 1, vp(0x30000), 64, N.DTYPE_F32, None, 0, None) == \
        N.MMN_E_INVALID  # one source
    assert L.mmn_grad_reduce(two, 2, vp(0x30004), 64, N.DTYPE_F32, None, 0, None) == \
        N.MMN_E_INVALID  # misaligned destination
    assert L.mmn_grad_reduce(two, 2, vp(0x10010), 64, N.DTYPE_F32, None, 0, None) == \
        N.MMN_E_INVALID  # overlaps the first source
    assert L.mmn_grad_reduce(two, 2, vp(0x30000), 64, 7, None, 0, None) == N.MMN_E_INVALID
    # well formed: the CUDA gate without a GPU; with one, the made-up addresses
    # are refused as not CUDA memory before any kernel is launched
    gate = N.MMN_E_INVALID if L.mmn_cuda_is_available() else N.MMN_E_NO_DEVICE
    rc = L.mmn_grad_reduce(two, 2, vp(0x30000), 64, N.DTYPE_BF16, None, 0, None)
    assert rc == gate and L.mmn_last_error()
    flags = (vp * 1)(vp(0x40000))
    assert L.mmn_grad_nonfinite_scan(vp(0x10008), 64, N.DTYPE_F32, flags, 1, 0, None) == \
        N.MMN_E_INVALID  # misaligned grads
    assert L.mmn_grad_nonfinite_scan(vp(0x10000), 64, N.DTYPE_F32, flags, 0, 0, None) == \
        N.MMN_E_INVALID  # no flags
    assert L.mmn_grad_nonfinite_scan(vp(0x10000), 64, N.DTYPE_F32, flags, 1, 0, None) == gate
